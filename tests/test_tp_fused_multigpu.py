"""Head-parallel tensor parallelism with sequence parallelism on the fused
sm_100a block, on 2 and 4 GPUs: the sharded model (uneven head split: 3 heads
over 2 ranks is [2, 1]) runs every block through the fused path and its output
and every gradient (this rank's slice of the sharded weights, the full tensor
of the replicated ones) match the unsharded model's fused run on the same
weights and inputs, within bf16 rounding. Both collective paths run: the
all-gather and reduce-scatter fused with their GEMMs over NVLink peer memory
(default; canary guards around every peer buffer stay intact) and NCCL
collectives between the kernels (``AVGEN_TP_PEER=0``)."""
from __future__ import annotations

import os
import socket
from dataclasses import asdict

import pytest
import torch
from multigpu_util import leave_on_failure

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(dev: torch.device, heads: int):  # noqa: ANN202
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny_gpu")).items() if k != "rope_scaling"}
    cfg.update(num_heads=heads, width=128 * heads)
    model = build_model("video_dit", cfg)
    model.init_weights()
    with torch.no_grad():  # non-zero output projections: every parameter gets a gradient
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    return model.to(dev)


def _inputs(model, dev: torch.device):  # noqa: ANN001, ANN202
    from avgen_b200.core.tokens import TextContext
    from avgen_b200.infer.conditioning import StreamState, condition_first_frame

    g = torch.Generator().manual_seed(71)
    c = model.config
    lat = torch.randn(1, c.in_channels, 4, 16, 32, generator=g).to(dev)  # 4 x 8 x 16 = 512 tokens
    text = TextContext(features=torch.randn(1, 16, c.text_width, generator=g).to(dev),
                       mask=torch.ones(1, 16, dtype=torch.bool, device=dev))
    return condition_first_frame(StreamState(lat, fps=8.0), lat[:, :, 0], sigma=0.6, text=text,
                                 patchifier=model.patchifier)


def _loss(out) -> torch.Tensor:  # noqa: ANN001
    w = torch.linspace(-1.0, 1.0, out.video.shape[-1], device=out.video.device)
    return (out.video.float() * w).sum()


def _close(got: torch.Tensor, want: torch.Tensor, what: str, rel: float) -> None:
    err = (got.float() - want.float()).abs().max().item()
    scale = want.float().abs().max().item()
    assert err <= 1e-6 + rel * scale, f"{what}: max err {err} vs max {scale}"


def _worker(rank: int, world: int, port: int, heads: int, peer: bool) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AVGEN_TP_PEER="1" if peer else "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        import avgen_b200.models.fused as fused_mod
        from avgen_b200.ops._ext import check_errors
        from avgen_b200.parallel import ParallelConfig, ParallelDims, parallelize
        from avgen_b200.parallel.heads import head_partition

        calls = {"n": 0}
        original = fused_mod.fused_block_forward

        def counting(*args, **kwargs):  # noqa: ANN002, ANN003, ANN202
            calls["n"] += 1
            return original(*args, **kwargs)

        fused_mod.fused_block_forward = counting
        ref = _model(dev, heads)
        want = ref(_inputs(ref, dev))
        _loss(want).backward()
        ref_calls = calls["n"]
        assert ref_calls == len(ref.blocks), "the unsharded reference must run the fused block"
        ref_grads = {n: p.grad.detach().clone() for n, p in ref.named_parameters()}

        dims = ParallelDims(world_size=world, tensor=world)
        pm = parallelize(_model(dev, heads), dims, config=ParallelConfig(sequence_parallel=True))
        assert any("sequence_parallel=True" in a for a in pm.applied), pm.applied
        assert pm.model.blocks[0].attention.num_heads == head_partition(heads, world)[rank]
        out = pm.model(_inputs(ref, dev))
        _loss(out).backward()
        assert calls["n"] - ref_calls == len(pm.model.blocks), "every sharded block must run fused"
        torch.cuda.synchronize()
        _close(out.video.detach(), want.video.detach(), "output", 2e-2)
        modules = dict(pm.model.named_modules())
        for name, p in pm.model.named_parameters():
            g = ref_grads[name]
            owner = modules[name.rsplit(".", 1)[0]]
            shard = getattr(owner, "_avgen_tp_shard", None)
            if shard is not None and (name.endswith("weight") or shard[0] == 0):
                dim, sizes, _ = shard
                g = g.narrow(dim, sum(sizes[:rank]), sizes[rank])
            assert p.grad is not None, name
            _close(p.grad, g, f"grad {name}", 3e-2)
        assert check_errors(dev) == 0
        assert bool(fused_mod._TP_PEER) == peer, "the peer path must run exactly when it is on"
        assert fused_mod.tp_peer_guard_violations() == []
        fused_mod.close_tp_peer()
        fused_mod.fused_block_forward = original
    except BaseException:
        leave_on_failure()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.parametrize("peer", [True, False])
@pytest.mark.parametrize("world,heads", [(2, 3), (4, 4)])
def test_fused_head_parallel_matches_unsharded(world: int, heads: int, peer: bool) -> None:
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port(), heads, peer), nprocs=world, join=True)
