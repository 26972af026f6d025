"""Model building blocks on CPU against closed forms: the attention oracle
against PyTorch's SDPA (masks, grouped-query heads, fully masked queries),
3-D RoPE (axis split, rotation is norm-preserving and relative, scaling modes),
the model registry and config validation, and the DiT's output shapes and
masking at several geometries (reference test strategy: tests/test_models*.py)."""
from __future__ import annotations

import math
from dataclasses import asdict

import pytest
import torch
import torch.nn.functional as F

from avgen_b200.models import build_model, preset
from avgen_b200.models.attention import attention, key_padding_mask, reference_attention
from avgen_b200.models.rope import (RoPEScaling, RotaryEmbedding, apply_rotary, axis_frequencies, build_rotary_tables,
                                    rope_axis_pairs)

# ----------------------------------------------------------------------------- attention oracle


@pytest.mark.parametrize("h,hk", [(4, 4), (4, 2), (6, 1)])
@pytest.mark.parametrize("lq,lk", [(5, 7), (16, 16), (1, 9)])
def test_reference_attention_matches_sdpa(h: int, hk: int, lq: int, lk: int) -> None:
    g = torch.Generator().manual_seed(h * 100 + lq)
    q = torch.randn(2, h, lq, 16, generator=g, dtype=torch.float64)
    k = torch.randn(2, hk, lk, 16, generator=g, dtype=torch.float64)
    v = torch.randn(2, hk, lk, 16, generator=g, dtype=torch.float64)
    rep = h // hk
    want = F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1))
    got = attention(q, k, v)  # the oracle computes in fp32
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    assert attention(q, k, v, layout="blhd").shape == (2, lq, h, 16)


def test_reference_attention_masks_keys_and_empty_queries() -> None:
    g = torch.Generator().manual_seed(1)
    q = torch.randn(2, 2, 4, 8, generator=g, dtype=torch.float64)
    k = torch.randn(2, 2, 6, 8, generator=g, dtype=torch.float64)
    v = torch.randn(2, 2, 6, 8, generator=g, dtype=torch.float64)
    mask = torch.tensor([[True, True, False, True, False, False], [False] * 6])
    got = reference_attention(q, k, v, mask, 1 / math.sqrt(8))
    want0 = F.scaled_dot_product_attention(q[:1], k[:1, :, mask[0]], v[:1, :, mask[0]])
    torch.testing.assert_close(got[:1].transpose(1, 2), want0, rtol=1e-5, atol=1e-6)
    assert bool((got[1] == 0).all())  # a sample without a valid key attends to nothing


def test_attention_scale_and_empty_inputs() -> None:
    q = torch.randn(1, 1, 3, 8, dtype=torch.float64)
    k = torch.randn(1, 1, 3, 8, dtype=torch.float64)
    v = torch.randn(1, 1, 3, 8, dtype=torch.float64)
    want = F.scaled_dot_product_attention(q, k, v, scale=0.3)
    torch.testing.assert_close(attention(q, k, v, scale=0.3), want, rtol=1e-5, atol=1e-6)
    empty = attention(q[:, :, :0], k, v)
    assert empty.shape == (1, 1, 0, 8)


def test_key_padding_mask_on_cpu() -> None:
    assert key_padding_mask(None) is None
    full = torch.ones(2, 5, dtype=torch.bool)
    assert key_padding_mask(full) is None  # all valid: no mask on the CPU path
    part = full.clone()
    part[0, -1] = False
    assert torch.equal(key_padding_mask(part), part)
    assert key_padding_mask(part, assume_dense=True) is None


# ----------------------------------------------------------------------------- RoPE


@pytest.mark.parametrize("head_dim,expect", [(6, (1, 1, 1)), (64, (12, 10, 10)), (128, (22, 21, 21)),
                                             (96, (16, 16, 16))])
def test_rope_axis_pairs(head_dim: int, expect: tuple[int, int, int]) -> None:
    pairs = rope_axis_pairs(head_dim)
    assert pairs == expect and sum(pairs) == head_dim // 2


@pytest.mark.parametrize("head_dim", [4, 7, 0])
def test_rope_axis_pairs_rejects(head_dim: int) -> None:
    with pytest.raises(ValueError):
        rope_axis_pairs(head_dim)


def _coords(length: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(2, length, 3, generator=g) * 5


def test_rotation_preserves_norms_and_is_relative() -> None:
    d = 32
    tables = build_rotary_tables(_coords(7), head_dim=d)
    x = torch.randn(2, 3, 7, d, dtype=torch.float32)
    y = apply_rotary(x, tables)
    torch.testing.assert_close(y.norm(dim=-1), x.norm(dim=-1), rtol=1e-5, atol=1e-5)
    # q.k after rotation depends only on the coordinate difference
    q = torch.randn(d)
    k = torch.randn(d)
    c1 = torch.tensor([[[1.0, 2.0, 3.0], [4.0, 0.5, -1.0]]])
    shift = torch.tensor([2.5, -1.0, 7.0])
    c2 = c1 + shift
    def score(c: torch.Tensor) -> float:
        t = build_rotary_tables(c, head_dim=d)
        qq = apply_rotary(q.expand(1, 1, 2, d).contiguous(), t)
        kk = apply_rotary(k.expand(1, 1, 2, d).contiguous(), t)
        return float((qq[0, 0, 0] * kk[0, 0, 1]).sum())
    assert score(c1) == pytest.approx(score(c2), rel=1e-4, abs=1e-4)


def test_zero_coordinates_are_identity() -> None:
    tables = build_rotary_tables(torch.zeros(1, 4, 3), head_dim=16)
    x = torch.randn(1, 2, 4, 16)
    torch.testing.assert_close(apply_rotary(x, tables), x)


@pytest.mark.parametrize("mode,factor", [("linear", 2.0), ("ntk", 4.0)])
def test_rope_scaling_modes_lower_frequencies(mode: str, factor: float) -> None:
    base, _ = axis_frequencies(64)
    scaled, axes = axis_frequencies(64, scaling=RoPEScaling(mode=mode, time_factor=factor, spatial_factor=factor))
    assert bool((scaled <= base + 1e-12).all()) and bool((scaled < base).any())
    if mode == "linear":
        torch.testing.assert_close(scaled, base / factor)
    assert axes.tolist() == [0] * 12 + [1] * 10 + [2] * 10
    assert RoPEScaling().is_identity and RoPEScaling(mode="linear").is_identity
    with pytest.raises(ValueError):
        RoPEScaling(mode="yarn")
    with pytest.raises(ValueError):
        RoPEScaling(time_factor=0.0)


def test_time_scale_only_touches_the_time_axis() -> None:
    base, axes = axis_frequencies(64)
    fast, _ = axis_frequencies(64, time_scale=2.0)
    torch.testing.assert_close(fast[axes == 0], 2 * base[axes == 0])
    torch.testing.assert_close(fast[axes != 0], base[axes != 0])


def test_rotary_validation_and_module() -> None:
    with pytest.raises(ValueError):
        build_rotary_tables(torch.zeros(1, 4, 2), head_dim=16)
    with pytest.raises(TypeError):
        build_rotary_tables(torch.zeros(1, 4, 3, dtype=torch.float64), head_dim=16)
    tables = build_rotary_tables(torch.zeros(1, 4, 3), head_dim=16)
    tables.validate()
    with pytest.raises(ValueError):
        apply_rotary(torch.zeros(1, 2, 5, 16), tables)  # wrong length
    with pytest.raises(ValueError):
        apply_rotary(torch.zeros(1, 2, 4, 8), tables)  # wrong head_dim
    mod = RotaryEmbedding(16)
    assert mod(torch.zeros(1, 4, 3)).pairs == 8 and "pairs(t,h,w)" in mod.extra_repr()
    freq, axis = mod.kernel_frequencies(torch.device("cpu"))
    assert freq.shape == (8,) and axis.dtype == torch.int32


# ----------------------------------------------------------------------------- registry and DiT


def test_registry_and_config_errors() -> None:
    from avgen_b200.models.registry import list_models, model_config_class

    assert "video_dit" in list_models()
    assert model_config_class("video_dit").__name__.endswith("Config")
    with pytest.raises(KeyError):
        build_model("unet3d")
    with pytest.raises((TypeError, ValueError, KeyError)):
        build_model("video_dit", {"no_such_field": 1})
    for bad in ({"width": 100, "num_heads": 3}, {"num_kv_heads": 5}, {"depth": 0}):
        with pytest.raises(ValueError):
            build_model("video_dit", {**_tiny(), **bad})


def _tiny() -> dict:
    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    return cfg


@pytest.mark.parametrize("frames,height,width", [(1, 4, 4), (2, 8, 8), (3, 4, 12)])
def test_dit_output_shape_and_masking(frames: int, height: int, width: int) -> None:
    from avgen_b200.core.tokens import TextContext
    from avgen_b200.infer.conditioning import StreamState, build_model_input

    torch.manual_seed(0)
    model = build_model("video_dit", _tiny())
    model.init_weights()
    with torch.no_grad():  # the zero-initialised output projections would hide the text path
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    c = model.config
    lat = torch.randn(1, c.in_channels, frames, height, width)
    text = TextContext(features=torch.randn(1, 3, c.text_width), mask=torch.ones(1, 3, dtype=torch.bool))
    inp = build_model_input(video=StreamState(lat, fps=8.0), sigma=0.5, text=text, patchifier=model.patchifier)
    out = model(inp)
    tokens = frames * (height // c.patch_height) * (width // c.patch_width)
    assert out.video.shape == (1, tokens, c.in_channels * c.patch_frames * c.patch_height * c.patch_width)
    assert bool(torch.isfinite(out.video).all())
    # the unconditional branch (null text) changes the prediction
    out_u = model(inp.unconditional())
    assert not torch.allclose(out.video, out_u.video)


def test_dit_zero_init_head_predicts_zero() -> None:
    from avgen_b200.core.tokens import TextContext
    from avgen_b200.infer.conditioning import StreamState, build_model_input

    model = build_model("video_dit", _tiny())
    model.init_weights()  # the output projection starts at zero
    c = model.config
    lat = torch.randn(1, c.in_channels, 2, 4, 4)
    text = TextContext(features=torch.randn(1, 3, c.text_width), mask=torch.ones(1, 3, dtype=torch.bool))
    out = model(build_model_input(video=StreamState(lat, fps=8.0), sigma=0.5, text=text,
                                  patchifier=model.patchifier))
    assert bool((out.video == 0).all())
