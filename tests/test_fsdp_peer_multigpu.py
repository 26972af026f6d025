"""FSDP2 with its collectives over NVLink peer memory (copy-engine all-gather,
pull-reduce reduce-scatter kernel) on 2 to 4 GPUs, against FSDP2 with NCCL on
the same model and inputs: two training steps of the fused-block VideoDiT with
the multi-tensor sharded AdamW must give the same parameters, gradient norm
and optimizer state; the symmetric buffers' canary guards must be intact and
no kernel may record an error."""
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


def _build(dev: torch.device, peer: bool, world: int):  # noqa: ANN202
    from avgen_b200.models import build_model, preset
    from avgen_b200.parallel import FSDPConfig, ParallelConfig, ParallelDims, parallelize
    from avgen_b200.train import build_optimizer

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny_gpu")).items() if k != "rope_scaling"}
    cfg["num_heads"] = 2
    cfg["width"] = 256
    model = build_model("video_dit", cfg).to(dev)
    model.init_weights()
    with torch.no_grad():  # non-zero output projection: every parameter gets a gradient
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    dims = ParallelDims(world_size=world, dp_shard=world)
    pm = parallelize(model, dims, config=ParallelConfig(fsdp=FSDPConfig(peer_collectives=peer)))
    tag = "collectives=peer" if peer else "collectives=nccl"
    assert any(tag in a for a in pm.applied), pm.applied
    return pm, build_optimizer(pm.model, lr=1e-3, weight_decay=0.1)


def _worker(rank: int, world: int, port: int) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), LOCAL_WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from torch.distributed.tensor import DTensor

        from avgen_b200.core import RNGStreams, TrainState
        from avgen_b200.data.synthetic_batch import random_batch
        from avgen_b200.ops._ext import check_errors
        from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning,
                                      build_timestep_sampler, train_step)
        from avgen_b200.train.optimizer import MultiTensorAdamW

        runs = {}
        for peer in (True, False):
            pm, opt = _build(dev, peer, world)
            assert isinstance(opt, MultiTensorAdamW)
            state = TrainState(model=pm.model, optimizer=opt, rng=RNGStreams.for_rank(0, data_rank=rank))
            obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"),
                                        MultiTaskConditioning())
            g = torch.Generator().manual_seed(50 + rank)
            norms = []
            grads = {}
            for step in range(2):
                batch = random_batch(batch=1, channels=4, frames=4, height=16, width=32, text_tokens=16,
                                     text_width=128, generator=g, device=dev)
                if step == 0:  # the reduced gradient shards themselves, before any optimizer step
                    opt.zero_grad()
                    loss = obj(pm.model, batch, RNGStreams.for_rank(9, data_rank=rank), patchifier=pm.model.patchifier)
                    loss.loss.backward()
                    grads = {n: p.grad.full_tensor().clone() for n, p in pm.model.named_parameters()}
                _, metrics = train_step(state, batch, obj, patchifier=pm.model.patchifier,
                                        max_grad_norm=0.5 if step else None)
                norms.append(metrics.grad_norm)
            torch.cuda.synchronize()
            params = {n: (p.full_tensor() if isinstance(p, DTensor) else p).detach().clone()
                      for n, p in pm.model.named_parameters()}
            moments = {n: opt.state[p]["exp_avg"].full_tensor().clone() for n, p in pm.model.named_parameters()}
            runs[peer] = (params, torch.stack([torch.as_tensor(x, device=dev).float() for x in norms]), moments,
                          grads)
            if peer:
                gather, reduce = pm.model._avgen_peer_collectives
                assert gather.calls > 0 and reduce.calls > 0
                assert not gather.slots.buf.check_guards() and not reduce.slots.buf.check_guards()
        assert check_errors(dev) == 0
        (p_peer, n_peer, m_peer, g_peer), (p_nccl, n_nccl, m_nccl, g_nccl) = runs[True], runs[False]
        for name in g_nccl:
            # the same fp32 sums of each rank's gradient; those gradients are bf16 (FSDP's parameter dtype)
            # and come from GEMMs with fp32 atomic split-K, so two runs may differ by one bf16 rounding
            # step (2^-8 relative); a misplaced shard or offset would differ by the gradient's own size
            err = (g_peer[name] - g_nccl[name]).abs().max().item()
            assert err <= 1e-6 + 8e-3 * g_nccl[name].abs().max().item(), f"grad {name}: {err}"
        torch.testing.assert_close(n_peer, n_nccl, rtol=1e-4, atol=1e-6)
        for name in p_nccl:
            # AdamW divides by sqrt(v): rounding-level gradient differences on near-zero entries
            # can move a parameter by up to ~lr per step, so compare at that scale
            err = (p_peer[name] - p_nccl[name]).abs().max().item()
            assert err <= 2.5e-3, f"param {name}: {err}"
            torch.testing.assert_close(m_peer[name], m_nccl[name], rtol=1e-3, atol=1e-6, msg=name)
    except BaseException:
        leave_on_failure()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_fsdp_peer_collectives_match_nccl(world: int) -> None:
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port()), nprocs=world, join=True)
