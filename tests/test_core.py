"""Core contracts on CPU: patchify round trips and mask/noise reductions, token
streams as pytrees, the model ABI's unconditional branch, dense batches,
purpose-separated RNG streams and on-device step metrics
(reference test strategy: tests/test_core_contracts.py)."""
from __future__ import annotations

import pytest
import torch
from torch.utils import _pytree

from avgen_b200.core import (ConditionMode, GridPatchifier, MediaBatch, ModelInput, PatchLayout, RNGStreams,
                             StepMetrics, TextContext, TokenStream, TrainState)
from avgen_b200.core.batch import stack_batches
from avgen_b200.core.patchify import patchify_grid, unpatchify_grid
from avgen_b200.data.synthetic_batch import random_batch


def _stream(b: int = 2, t: int = 3, h: int = 4, w: int = 6, c: int = 4, seed: int = 0):  # noqa: ANN202
    g = torch.Generator().manual_seed(seed)
    grid = torch.randn(b, c, t, h, w, generator=g)
    mask = torch.ones(b, t, h, w, dtype=torch.bool)
    pos = torch.arange(t, dtype=torch.float32)[None].expand(b, t) / 8.0
    return grid, mask, pos


def test_patchify_round_trip_and_layout() -> None:
    grid, mask, pos = _stream()
    p = GridPatchifier()
    s = p.to_tokens(grid, positions=pos, mask=mask, noise_level=torch.tensor([0.3, 0.7]))
    lay = s.layout
    assert isinstance(lay, PatchLayout)
    assert s.tokens.shape == (2, 3 * 2 * 3, 4 * 2 * 2) == (2, lay.num_tokens, lay.patch_dim)
    assert torch.equal(p.to_grid(s), grid)
    assert torch.equal(unpatchify_grid(patchify_grid(grid, lay), lay), grid)
    # token order is time-major, then row, then column: the first tokens share frame 0
    assert torch.all(s.coords[:, : lay.num_tokens // 3, 0] == 0)
    assert s.coords.dtype == torch.float32


def test_patchify_mask_any_conditioned_all_and_noise_mean() -> None:
    grid, mask, pos = _stream(b=1)
    mask[0, 0, 0, 0] = False  # one pixel of the first patch invalid: the token stays valid (any)
    mask[0, 1, :2, :2] = False  # a whole patch invalid: the token is masked
    cond = torch.zeros_like(mask)
    cond[0, 2, :2, :2] = True  # a full patch conditioned
    cond[0, 2, 2, 2] = True  # one pixel of another patch: not conditioned (all)
    noise = torch.rand(1, 3, 4, 6)
    s = GridPatchifier().to_tokens(grid, positions=pos, mask=mask, noise_level=noise, conditioned=cond)
    per_frame = 2 * 3
    assert bool(s.mask[0, 0])
    assert not bool(s.mask[0, per_frame])
    assert bool(s.conditioned[0, 2 * per_frame]) and int(s.conditioned.sum()) == 1
    torch.testing.assert_close(s.noise_level[0, 0], noise[0, 0, :2, :2].mean())
    assert s.per_token_noise
    assert not bool(s.loss_mask()[0, 2 * per_frame])  # conditioned tokens are excluded from the loss


def test_token_stream_is_a_pytree_and_empty_streams() -> None:
    grid, mask, pos = _stream()
    s = GridPatchifier().to_tokens(grid, positions=pos, mask=mask, noise_level=torch.tensor([0.1, 0.2]))
    leaves, spec = _pytree.tree_flatten(s)
    assert any(leaf is s.tokens for leaf in leaves)
    back = _pytree.tree_unflatten([leaf.clone() if isinstance(leaf, torch.Tensor) else leaf for leaf in leaves], spec)
    assert isinstance(back, TokenStream) and torch.equal(back.tokens, s.tokens)
    e = TokenStream.empty_like(2, 8)
    assert e.is_empty and e.length == 0 and e.batch_size == 2


def test_model_input_unconditional_nulls_only_text() -> None:
    grid, mask, pos = _stream()
    s = GridPatchifier().to_tokens(grid, positions=pos, mask=mask, noise_level=torch.tensor([0.1, 0.2]))
    text = TextContext(features=torch.randn(2, 5, 16), mask=torch.ones(2, 5, dtype=torch.bool))
    mi = ModelInput(video=s, audio=TokenStream.empty_like(2, s.width), text=text)
    assert int(mi.condition_mode[0]) == int(ConditionMode.JOINT)
    u = mi.unconditional()
    assert u.video is mi.video and u.audio is mi.audio
    assert not bool(u.text.mask.any()) or bool((u.text.features == 0).all())
    assert mi.total_tokens == s.length and mi.has_text


def test_media_batch_pin_to_stack_validate() -> None:
    a = random_batch(batch=1, channels=4, frames=2, height=8, width=8, text_tokens=3, text_width=16)
    b = random_batch(batch=1, channels=4, frames=2, height=8, width=8, text_tokens=3, text_width=16,
                     generator=torch.Generator().manual_seed(1))
    a.validate()
    s = stack_batches([a, b])
    assert isinstance(s, MediaBatch) and s.video.shape[0] == 2 and s.spec.batch_size == 2
    assert torch.equal(s.video[1], b.video[0])
    assert s.nbytes() == a.nbytes() + b.nbytes()
    moved = s.to("cpu")
    assert moved.device.type == "cpu"


def test_rng_streams_are_separated_and_rank_mixed() -> None:
    r = RNGStreams.from_seed(7)
    x = torch.randn(4, generator=r.noise)
    y = torch.randn(4, generator=r.timestep)
    assert not torch.equal(x, y)  # purposes draw from different streams
    a = RNGStreams.for_rank(7, data_rank=0)
    b = RNGStreams.for_rank(7, data_rank=0)
    c = RNGStreams.for_rank(7, data_rank=1)
    assert torch.equal(torch.randn(3, generator=a.noise), torch.randn(3, generator=b.noise))
    assert not torch.equal(torch.randn(3, generator=a.sampler), torch.randn(3, generator=c.sampler))
    state = a.state_dict()
    first = torch.randn(5, generator=a.noise)
    a.load_state_dict(state)
    assert torch.equal(torch.randn(5, generator=a.noise), first)
    forked = a.fork("eval")
    assert isinstance(forked, torch.Generator)


def test_step_metrics_single_sync_and_train_state_progress() -> None:
    m = StepMetrics.zeros()
    values = m.to_mapping()
    assert set(values) >= {"loss", "grad_norm", "nonfinite", "skipped"}
    assert all(isinstance(v, float) for v in values.values())
    model = torch.nn.Linear(2, 2)
    st = TrainState(model=model, optimizer=torch.optim.SGD(model.parameters(), lr=0.1), rng=RNGStreams.from_seed(0))
    st.step, st.samples_seen, st.tokens_seen = 3, 12, 480
    prog = st.progress()
    assert prog["step"] == 3 and prog["tokens_seen"] == 480
    other = TrainState(model=model, optimizer=st.optimizer, rng=RNGStreams.from_seed(0))
    other.load_progress(prog)
    assert other.step == 3 and other.samples_seen == 12


def test_invalid_shapes_fail_with_field_names() -> None:
    with pytest.raises((ValueError, TypeError)):
        GridPatchifier().layout_for((1, 4, 8, 8))
    grid, mask, pos = _stream()
    with pytest.raises((ValueError, RuntimeError)):
        GridPatchifier().to_tokens(grid[:, :, :, :3], positions=pos, mask=mask[:, :, :3], noise_level=torch.zeros(2))
