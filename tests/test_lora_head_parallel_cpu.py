"""LoRA adapters on head-parallel tensor-parallel shards (gloo, 3 heads over 2 ranks
as [2, 1], sequence parallelism): the adapter factor that is sharded with its base
weight (B of a column-parallel layer, A of a row-parallel one) gets this rank's
slice of the unsharded gradient, the replicated factor gets the full gradient
(its per-rank partial sums are added over the group), through the eager layers and
through the fused block with its kernels restated in PyTorch; and a checkpoint of
the sharded model holds full tensors for base weights and adapters alike."""
from __future__ import annotations

import os
import socket
from dataclasses import asdict
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HEADS = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():  # noqa: ANN202
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    cfg.update(num_heads=HEADS, width=16 * HEADS, depth=1)
    model = build_model("video_dit", cfg)
    model.init_weights()
    with torch.no_grad():
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    return model


def _lora(model):  # noqa: ANN001, ANN202
    from avgen_b200.finetune.lora import LoRAConfig, apply_lora, mark_only_lora_trainable

    apply_lora(model, LoRAConfig(rank=4, alpha=8.0))
    mark_only_lora_trainable(model)
    return model


def _inputs(model):  # noqa: ANN001, ANN202
    from avgen_b200.core.tokens import TextContext
    from avgen_b200.infer.conditioning import StreamState, condition_first_frame

    g = torch.Generator().manual_seed(71)
    c = model.config
    lat = torch.randn(1, c.in_channels, 2, 8, 8, generator=g)  # 2 x 4 x 4 = 32 tokens
    text = TextContext(features=torch.randn(1, 6, c.text_width, generator=g), mask=torch.ones(1, 6, dtype=torch.bool))
    return condition_first_frame(StreamState(lat, fps=8.0), lat[:, :, 0], sigma=0.6, text=text,
                                 patchifier=model.patchifier)


def _loss(out) -> torch.Tensor:  # noqa: ANN001
    return (out.video * torch.linspace(-1.0, 1.0, out.video.shape[-1])).sum()


def _slice(full: torch.Tensor, shard: tuple | None, factor: str, rank: int) -> torch.Tensor:
    """This rank's part of an unsharded adapter factor (whole for replicated layers)."""
    if shard is None:  # a layer outside the blocks (time embedding, text refiner): replicated
        return full
    dim, sizes, _ = shard
    start = sum(sizes[:rank])
    if dim == 0 and factor == "lora_b":
        return full.narrow(0, start, sizes[rank])
    if dim == 1 and factor == "lora_a":
        return full.narrow(1, start, sizes[rank])
    return full


def _worker(rank: int, world: int, port: int, fused: bool) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AVGEN_KEEP_ACTIVATIONS="none")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from avgen_b200.finetune.lora import lora_modules
        from avgen_b200.parallel import ParallelConfig, ParallelDims, parallelize

        ref = _lora(_model())
        with torch.no_grad():  # non-zero B so every factor gets a gradient
            for _, m in lora_modules(ref):
                m.lora_b.copy_(0.05 * torch.randn(m.lora_b.shape, generator=torch.Generator().manual_seed(3)))
        dims = ParallelDims(world_size=world, tensor=world)
        pm = parallelize(_model(), dims, mesh=dims.build_mesh("cpu"), adapt=_lora,
                         config=ParallelConfig(sequence_parallel=True))
        full = dict(lora_modules(ref))
        with torch.no_grad():  # the same adapter values, sliced like their base weights
            for name, m in lora_modules(pm.model):
                shard = getattr(m, "_avgen_tp_shard", None)
                for factor in ("lora_a", "lora_b"):
                    getattr(m, factor).copy_(_slice(getattr(full[name], factor), shard, factor, rank))
        _loss(ref(_inputs(ref))).backward()
        if fused:
            from test_fused_model_emulated_cpu import _ForcedFused

            with _ForcedFused() as forced:
                _loss(pm.model(_inputs(ref))).backward()
            assert forced.calls == len(pm.model.blocks)
        else:
            _loss(pm.model(_inputs(ref))).backward()
        tol = 4e-2 if fused else 1e-4
        for name, m in lora_modules(pm.model):
            for factor in ("lora_a", "lora_b"):
                got = getattr(m, factor).grad
                want = _slice(getattr(full[name], factor).grad, getattr(m, "_avgen_tp_shard", None), factor, rank)
                assert got is not None and got.shape == want.shape, (name, factor)
                err = float((got - want).norm() / (want.norm() + 1e-12))
                assert err < tol, (name, factor, err)
        if not fused:  # checkpoints hold full tensors (gathered on save) for bases and adapters
            state = pm.model.state_dict()
            for key, value in ref.state_dict().items():
                if ".lora_" in key or key.endswith("proj.weight"):
                    assert tuple(state[key].shape) == tuple(value.shape), key
                    torch.testing.assert_close(state[key], value, rtol=1e-6, atol=1e-6)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [False, True], ids=["eager", "fused"])
def test_lora_on_head_parallel_shards_matches_unsharded(fused: bool) -> None:
    mp.spawn(_worker, args=(2, _free_port(), fused), nprocs=2, join=True)
