"""The fused DiT block (sm_100a kernels) against the fp32 eager oracle on the CPU."""
from __future__ import annotations

import copy

import pytest
import torch

from avgen_b200.models.blocks import DiTBlock, RopeInputs
from avgen_b200.models.rope import RotaryEmbedding

pytestmark = pytest.mark.gpu


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("ffn,masked,grouped,keep", [("swiglu", False, False, "none"), ("gelu", True, False, "none"),
                                                      ("swiglu", True, True, "none"), ("swiglu", False, False, "all"),
                                                      ("swiglu", True, True, "no_mlp"), ("gelu", True, False, "all")])
def test_fused_block_matches_eager(ffn: str, masked: bool, grouped: bool, keep: str,
                                   monkeypatch: pytest.MonkeyPatch) -> None:
    """Forward and gradients against the CPU oracle, with the backward recomputing
    the block ("none") or using what the forward kept ("all", "no_mlp")."""
    monkeypatch.setenv("AVGEN_KEEP_ACTIVATIONS", keep)
    torch.manual_seed(0)
    width, heads, hidden, b, length, t = 256, 2, 512, 2, 384, 24
    block = DiTBlock(width, heads, hidden=hidden, ffn=ffn)
    block.init_weights(depth=2)
    with torch.no_grad():  # non-zero gates, tables and cross-attention output so every path matters
        for p in block.parameters():
            p.add_(0.02 * torch.randn_like(p))
    rope = RotaryEmbedding(128)
    x = torch.randn(b, length, width)
    mod_index = None
    if grouped:  # two modulation rows per sample: clean first frame (row 2b+1), noisy rest (row 2b)
        mod = 0.1 * torch.randn(2 * b, 6, width)
        mod_index = (torch.arange(b)[:, None] * 2 + (torch.arange(length) < 96).long()[None]).int()
    else:
        mod = 0.1 * torch.randn(b, 6, width)
    ctx = torch.randn(b, t, width)
    coords = torch.rand(b, length, 3) * 8
    kmask = None
    cmask = torch.ones(b, t, dtype=torch.bool)
    cmask[1, 20:] = False
    if masked:
        kmask = torch.ones(b, length, dtype=torch.bool)
        kmask[0, 300:] = False
    # oracle: CPU fp32 eager
    ref_block = copy.deepcopy(block)
    xr, modr, ctxr = (v.clone().requires_grad_() for v in (x, mod, ctx))
    out_ref = ref_block(xr, modulation=modr, rope=RopeInputs(coords, rope), key_mask=kmask, context=ctxr,
                        context_mask=cmask, modulation_index=mod_index)
    g = torch.randn_like(out_ref)
    out_ref.backward(g)
    # fused on the GPU
    gb = copy.deepcopy(block).cuda()
    xg = x.cuda().bfloat16().requires_grad_()
    modg = mod.cuda().requires_grad_()
    ctxg = ctx.cuda().bfloat16().requires_grad_()
    out = gb(xg, modulation=modg, rope=RopeInputs(coords.cuda(), rope), key_mask=None if kmask is None else kmask.cuda(),
             context=ctxg, context_mask=cmask.cuda(), modulation_index=None if mod_index is None else mod_index.cuda())
    out.backward(g.cuda().bfloat16())
    assert _rel(out, out_ref) < 3e-2
    assert _rel(xg.grad, xr.grad) < 5e-2
    assert _rel(modg.grad, modr.grad) < 5e-2
    assert _rel(ctxg.grad, ctxr.grad) < 5e-2
    for (name, p), (_, q) in zip(gb.named_parameters(), ref_block.named_parameters()):
        assert p.grad is not None, name
        assert _rel(p.grad, q.grad) < 6e-2, name
    from avgen_b200.ops._ext import check_errors

    assert check_errors() == 0


def test_tiny_gpu_model_trains() -> None:
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.models import build_model, preset
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)
    from dataclasses import asdict

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny_gpu")).items() if k != "rope_scaling"}
    model = build_model("video_dit", cfg).cuda()
    model.init_weights()
    torch.nn.init.normal_(model.final_proj.weight, std=0.02)
    opt = build_optimizer(model, lr=1e-3)
    state = TrainState(model=model, optimizer=opt, rng=RNGStreams.from_seed(0))
    obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("logit_normal"), MultiTaskConditioning())
    batch = random_batch(batch=2, channels=4, frames=4, height=16, width=32, text_tokens=16, text_width=128,
                         device="cuda")
    losses = []
    for _ in range(4):
        _, m = train_step(state, batch, obj, patchifier=model.patchifier, max_grad_norm=1.0)
        losses.append(m.to_mapping())
    assert all(torch.isfinite(torch.tensor([l["loss"] for l in losses])))
    assert losses[-1]["grad_norm"] > 0


def test_generation_fused_guided_euler_matches_unfused(monkeypatch: pytest.MonkeyPatch) -> None:
    """The fused CFG + Euler kernel step reproduces guidance followed by the Euler update."""
    from dataclasses import asdict

    from avgen_b200.codecs import ReferenceTextEncoder, ReferenceVideoCodec
    from avgen_b200.infer import GenerationPipeline, GuidanceConfig
    from avgen_b200.models import build_model, preset
    from avgen_b200.ops import kernels as K

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny_gpu")).items() if k != "rope_scaling"}
    codec = ReferenceVideoCodec(channels=1, spatial_compression=2)
    cfg["in_channels"] = codec.latent_channels
    model = build_model("video_dit", cfg).to("cuda")
    model.init_weights()
    with torch.no_grad():
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    model.eval()
    pipe = GenerationPipeline(model, video_codec=codec, text_encoder=ReferenceTextEncoder(width=cfg["text_width"]),
                              device="cuda")
    kw = dict(steps=3, guidance=GuidanceConfig(scale=4.0), height=32, width=64, num_frames=4, seed=3,
              return_latents=True)
    n0 = K.launch_count()
    fused = pipe(["a cat"], **kw)
    assert K.launch_count() > n0
    monkeypatch.setattr(GenerationPipeline, "_fusable_euler", lambda *a, **k: False)
    plain = pipe(["a cat"], **kw)
    assert _rel(fused.latents, plain.latents) < 1e-3


@pytest.mark.parametrize("mode", ["lora", "dora", "lora+base"])
def test_fused_block_with_adapters_matches_eager(mode: str) -> None:
    """LoRA / DoRA adapters on every attention and MLP linear: the block still runs
    through the fused node (effective weights in the kernels; LoRA gradients from
    rank-r products, DoRA's through the dense effective-weight gradient) and matches
    the CPU fp32 eager block with the same adapters, forward and every adapter
    gradient. Frozen base weights get no gradient; trainable ones ("lora+base") get
    their dense gradient beside the adapters'."""
    dora = mode == "dora"
    import avgen_b200.models.fused as fused_mod
    from avgen_b200.finetune.lora import LoRAConfig, apply_lora, lora_modules, mark_only_lora_trainable

    torch.manual_seed(1)
    width, heads, hidden, b, length, t = 256, 2, 512, 1, 256, 16
    block = DiTBlock(width, heads, hidden=hidden)
    block.init_weights(depth=2)
    with torch.no_grad():
        for p in block.parameters():
            p.add_(0.02 * torch.randn_like(p))
    cfg = LoRAConfig(rank=8, alpha=16.0, use_dora=dora,
                     target_modules=("q_proj", "k_proj", "v_proj", "out_proj", "gate_proj", "up_proj", "down_proj"))
    apply_lora(block, cfg)
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
    rope = RotaryEmbedding(128)
    x = torch.randn(b, length, width)
    mod = 0.1 * torch.randn(b, 6, width)
    ctx = torch.randn(b, t, width)
    coords = torch.rand(b, length, 3) * 8
    ref_block = copy.deepcopy(block)
    out_ref = ref_block(x, modulation=mod, rope=RopeInputs(coords, rope), context=ctx)
    g = torch.randn_like(out_ref)
    out_ref.backward(g)
    calls = {"n": 0}
    original = fused_mod.fused_block_forward

    def counting(*args, **kwargs):  # noqa: ANN002, ANN003, ANN202
        calls["n"] += 1
        return original(*args, **kwargs)

    fused_mod.fused_block_forward = counting
    try:
        gb = copy.deepcopy(block).cuda()
        out = gb(x.cuda().bfloat16(), modulation=mod.cuda(), rope=RopeInputs(coords.cuda(), rope),
                 context=ctx.cuda().bfloat16())
        out.backward(g.cuda().bfloat16())
    finally:
        fused_mod.fused_block_forward = original
    assert calls["n"] == 1, "the adapted block must run the fused node"
    assert _rel(out, out_ref) < 3e-2
    ref_params = dict(ref_block.named_parameters())
    checked = 0
    for name, p in gb.named_parameters():
        if p.requires_grad:
            assert p.grad is not None, name
            assert _rel(p.grad, ref_params[name].grad) < 6e-2, name
            checked += 1
        else:
            assert p.grad is None, name  # frozen
    assert checked >= (14 if mode != "lora+base" else 21)
    from avgen_b200.ops._ext import check_errors

    assert check_errors() == 0
