"""The fused DiT block's orchestration on CPU, with its kernels replaced by the
PyTorch statements of their contracts (``kernel_emulator``): forward, input and
every parameter gradient against the fp32 eager block for each FFN, masks,
grouped and per-token modulation, recompute versus kept intermediates, frozen
weights, LoRA (low-rank gradients, with and without a trainable base) and DoRA
adapters, and head-parallel shards with sequence parallelism on a two-rank
``gloo`` group. The kernels' own numerics are the GPU tests' business."""
from __future__ import annotations

import copy
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from kernel_emulator import emulate_kernels

from avgen_b200.models import blocks as blocks_mod
from avgen_b200.models.blocks import DiTBlock, RopeInputs
from avgen_b200.models.rope import RotaryEmbedding

WIDTH, HEADS, HEAD_DIM, HIDDEN = 64, 2, 32, 128


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _block(ffn: str = "swiglu", seed: int = 0, heads: int = HEADS) -> DiTBlock:
    torch.manual_seed(seed)
    block = DiTBlock(heads * HEAD_DIM, heads, hidden=HIDDEN, ffn=ffn)
    block.init_weights(depth=2)
    with torch.no_grad():  # non-zero gates, tables and output projections so every path matters
        for p in block.parameters():
            p.add_(0.05 * torch.randn_like(p))
    return block


def _run(block: DiTBlock, fused: bool, x, mod, ctx, coords, kmask, cmask, mod_index, g):  # noqa: ANN001, ANN202
    """Forward + backward; returns (out, dx, dmod, dctx)."""
    xr, modr, ctxr = (v.clone().requires_grad_() for v in (x, mod, ctx))
    calls = {"n": 0}
    import avgen_b200.models.fused as fused_mod

    original = fused_mod.fused_block_forward

    def counting(*args, **kwargs):  # noqa: ANN002, ANN003, ANN202
        calls["n"] += 1
        return original(*args, **kwargs)

    eligible = blocks_mod._fused_eligible
    try:
        if fused:
            fused_mod.fused_block_forward = counting
            blocks_mod._fused_eligible = lambda b, h: True
        out = block(xr, modulation=modr, rope=RopeInputs(coords, RotaryEmbedding(HEAD_DIM)), key_mask=kmask,
                    context=ctxr, context_mask=cmask, modulation_index=mod_index)
        out.backward(g)
    finally:
        fused_mod.fused_block_forward = original
        blocks_mod._fused_eligible = eligible
    assert calls["n"] == (1 if fused else 0)
    return out, xr.grad, modr.grad, ctxr.grad


def _inputs(b: int, length: int, t: int, *, masked: bool, modulation: str, seed: int = 1):  # noqa: ANN202
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(b, length, WIDTH, generator=gen)
    mod_index = None
    if modulation == "grouped":  # two rows per sample: clean first tokens, noisy rest
        mod = 0.1 * torch.randn(2 * b, 6, WIDTH, generator=gen)
        mod_index = (torch.arange(b)[:, None] * 2 + (torch.arange(length) < length // 4).long()[None]).int()
    elif modulation == "token":
        mod = 0.1 * torch.randn(b, length, 6, WIDTH, generator=gen)
    else:
        mod = 0.1 * torch.randn(b, 6, WIDTH, generator=gen)
    ctx = torch.randn(b, t, WIDTH, generator=gen)
    coords = torch.rand(b, length, 3, generator=gen) * 8
    cmask = torch.ones(b, t, dtype=torch.bool)
    cmask[-1, t - 3:] = False
    kmask = None
    if masked:
        kmask = torch.ones(b, length, dtype=torch.bool)
        kmask[0, length - 5:] = False
    return x, mod, ctx, coords, kmask, cmask, mod_index


def _compare(block: DiTBlock, b: int = 2, length: int = 40, t: int = 7, *, masked: bool = False,
             modulation: str = "sample") -> None:
    x, mod, ctx, coords, kmask, cmask, mod_index = _inputs(b, length, t, masked=masked, modulation=modulation)
    ref = copy.deepcopy(block)
    out_r, dx_r, dmod_r, dctx_r = _run(ref, False, x, mod, ctx, coords, kmask, cmask, mod_index,
                                       g := torch.randn(b, length, WIDTH))
    with emulate_kernels():
        out, dx, dmod, dctx = _run(block, True, x, mod, ctx, coords, kmask, cmask, mod_index, g)
    assert _rel(out, out_r) < 2e-2
    assert _rel(dx, dx_r) < 3e-2
    assert _rel(dmod, dmod_r) < 3e-2
    assert _rel(dctx, dctx_r) < 3e-2
    ref_params = dict(ref.named_parameters())
    for name, p in block.named_parameters():
        q = ref_params[name]
        if not p.requires_grad:
            assert p.grad is None, name
            continue
        assert p.grad is not None, name
        assert p.grad.shape == p.shape and p.grad.dtype == p.dtype, name
        assert _rel(p.grad, q.grad) < 4e-2, name


@pytest.mark.parametrize("ffn,masked,modulation,keep", [
    ("swiglu", False, "sample", "none"), ("gelu", True, "sample", "none"), ("swiglu", True, "grouped", "none"),
    ("swiglu", False, "token", "none"), ("swiglu", False, "sample", "all"), ("swiglu", True, "grouped", "no_mlp"),
    ("gelu", True, "sample", "all"),
])
def test_fused_block_orchestration_matches_eager(ffn: str, masked: bool, modulation: str, keep: str,
                                                 monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("AVGEN_KEEP_ACTIVATIONS", keep)
    _compare(_block(ffn), masked=masked, modulation=modulation)


def test_frozen_weights_get_no_gradient(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("AVGEN_KEEP_ACTIVATIONS", "none")
    block = _block()
    for name, p in block.named_parameters():
        if name.startswith(("attention.k_proj", "feed_forward.up_proj", "cross_attention.v_proj")):
            p.requires_grad_(False)
    _compare(block)


@pytest.mark.parametrize("mode", ["lora", "lora+base", "dora"])
def test_adapted_block_gradients(mode: str, monkeypatch: pytest.MonkeyPatch) -> None:
    """Plain LoRA takes the rank-r gradient route (no dense weight gradient unless the
    base trains); DoRA the dense effective-weight route through autograd."""
    from avgen_b200.finetune.lora import LoRAConfig, apply_lora, lora_modules, mark_only_lora_trainable

    monkeypatch.setenv("AVGEN_KEEP_ACTIVATIONS", "none")
    block = _block()
    apply_lora(block, LoRAConfig(rank=8, alpha=16.0, use_dora=mode == "dora",
                                 target_modules=("q_proj", "k_proj", "v_proj", "out_proj", "gate_proj", "up_proj",
                                                 "down_proj")))
    with torch.no_grad():
        for _, m in lora_modules(block):
            m.lora_b.normal_(0.0, 0.05)
            if m.lora_magnitude is not None:
                m.lora_magnitude.mul_(1.0 + 0.1 * torch.randn_like(m.lora_magnitude))
    mark_only_lora_trainable(block)
    if mode == "lora+base":
        for name, p in block.named_parameters():
            if name.endswith("proj.weight"):
                p.requires_grad_(True)
    import avgen_b200.models.fused as fused_mod

    dense = {"n": 0}
    original = fused_mod._weight_grads

    def counting(blk, members, dy, x, weights, need, out):  # noqa: ANN001, ANN202
        dense["n"] += sum(need.get(f"{p}.weight", False) for p, _ in members)
        return original(blk, members, dy, x, weights, need, out)

    monkeypatch.setattr(fused_mod, "_weight_grads", counting)
    _compare(block)
    linears = 11  # q, k, v, out, gate, up, down, and the cross-attention q, k, v, out
    assert dense["n"] == {"lora": 0, "lora+base": linears, "dora": linears}[mode]


# ----------------------------------------------------------------------------- head-parallel shards


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank: int, world: int, port: int, heads: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AVGEN_KEEP_ACTIVATIONS="none")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from avgen_b200.parallel.heads import HeadParallel, _shard_attention, _shard_mlp

        full = _block(heads=heads)
        b, length, t = 1, 48, 7
        width = heads * HEAD_DIM
        gen = torch.Generator().manual_seed(5)
        x = torch.randn(b, length, width, generator=gen)
        mod = 0.1 * torch.randn(b, 6, width, generator=gen)
        ctx = torch.randn(b, t, width, generator=gen)
        coords = torch.rand(b, length, 3, generator=gen) * 8
        g = torch.randn(b, length, width, generator=gen)
        ref = copy.deepcopy(full)
        out_r, dx_r, dmod_r, dctx_r = _run(ref, False, x, mod, ctx, coords, None, None, None, g)
        tp = HeadParallel(dist.group.WORLD, rank, world, True)
        block = copy.deepcopy(full)
        _shard_attention(block.attention, tp)
        _shard_attention(block.cross_attention, tp)
        _shard_mlp(block.feed_forward, tp)
        block.tp = tp
        chunk = tp.token_slice(length)
        with emulate_kernels():
            out, dx, dmod, dctx = _run(block, True, x[:, chunk], mod, ctx, coords, None, None, None, g[:, chunk])
        assert _rel(out, out_r[:, chunk]) < 2e-2
        assert _rel(dx, dx_r[:, chunk]) < 3e-2
        dmod_all = dmod.clone()
        dist.all_reduce(dmod_all)  # each rank holds its tokens' share of the modulation gradient
        assert _rel(dmod_all, dmod_r) < 3e-2
        assert _rel(dctx, dctx_r) < 3e-2  # the text context's gradient is summed over the group already
        modules = dict(block.named_modules())
        ref_params = dict(ref.named_parameters())
        for name, p in block.named_parameters():
            want = ref_params[name].grad
            shard = getattr(modules.get(name.rsplit(".", 1)[0]), "_avgen_tp_shard", None)
            if shard is not None:
                dim, sizes, _ = shard
                want = want.narrow(dim, sum(sizes[:rank]), sizes[rank])
            elif "q_norm" in name or "k_norm" in name:  # head-space norms: summed over the heads' ranks already
                pass
            else:  # token-space parameters: each rank's gradient covers its own tokens
                got = p.grad.clone()
                dist.all_reduce(got)
                assert _rel(got, want) < 4e-2, name
                continue
            assert _rel(p.grad, want) < 4e-2, name
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,heads", [(2, 3)])
def test_head_parallel_fused_block_matches_unsharded(world: int, heads: int) -> None:
    mp.spawn(_tp_worker, args=(world, _free_port(), heads), nprocs=world, join=True)


def test_lora_packed_weights_are_cached_until_an_adapter_changes(monkeypatch: pytest.MonkeyPatch) -> None:
    """The packed bf16 weights of a LoRA-adapted block are built once per adapter state:
    the backward's recompute reuses the forward's, an in-place adapter update rebuilds
    them, and the effective weight is never kept beside its packed copy."""
    import avgen_b200.models.fused as fused_mod
    from avgen_b200.finetune.lora import LoRAConfig, apply_lora, lora_modules, mark_only_lora_trainable

    monkeypatch.setenv("AVGEN_KEEP_ACTIVATIONS", "none")
    block = _block()
    apply_lora(block, LoRAConfig(rank=8, alpha=16.0, target_modules=("q_proj", "out_proj", "down_proj")))
    mark_only_lora_trainable(block)
    built = {"n": 0}
    original = fused_mod._LoRAWeight.value

    def counting(self):  # noqa: ANN001, ANN202
        built["n"] += 1
        return original(self)

    monkeypatch.setattr(fused_mod._LoRAWeight, "value", counting)
    x, mod, ctx, coords, kmask, cmask, mod_index = _inputs(1, 16, 5, masked=False, modulation="sample")
    g = torch.randn(1, 16, WIDTH)
    with emulate_kernels():
        _run(block, True, x, mod, ctx, coords, kmask, cmask, mod_index, g)
        first = built["n"]
        assert first == 5  # self q, self out, cross q, cross out, MLP down: once each for forward and recompute
        _run(block, True, x, mod, ctx, coords, kmask, cmask, mod_index, g)
        assert built["n"] == first  # nothing changed: every packed weight served from the cache
        with torch.no_grad():
            next(m for _, m in lora_modules(block)).lora_b.add_(0.01)
        _run(block, True, x, mod, ctx, coords, kmask, cmask, mod_index, g)
        assert built["n"] == first + 1  # only the updated adapter's pack was rebuilt
    assert not any("_avgen_effective" in m.__dict__ for m in block.modules())
