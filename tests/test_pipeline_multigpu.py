"""Pipeline parallelism over NCCL on 2 GPUs with the fused sm_100a blocks: 1F1B
and interleaved 1F1B (4 chunks over 2 ranks) take one clipped optimizer step over
4 micro-batches; the loss and the parameters after the step match the unsharded
model trained with gradient accumulation on the same GPU (within bf16 rounding)."""
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


def _model(dev: torch.device):  # noqa: ANN202
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny_gpu")).items() if k != "rope_scaling"}
    cfg["depth"] = 4
    m = build_model("video_dit", cfg)
    m.init_weights()
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.02 * torch.randn_like(p))
    return m.to(dev)


def _worker(rank: int, world: int, port: int, schedule: str, chunks: int) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from avgen_b200.core import RNGStreams, TrainState
        from avgen_b200.data.synthetic_batch import random_batch
        from avgen_b200.ops._ext import check_errors
        from avgen_b200.parallel import ParallelConfig, ParallelDims, PipelineConfig, PrecisionConfig, parallelize
        from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning,
                                      build_optimizer, build_timestep_sampler, train_step)
        from avgen_b200.train.trainer import pipeline_train_step

        ref = _model(dev)
        dims = ParallelDims(world_size=world, pipeline=world)
        pm = parallelize(_model(dev), dims, config=ParallelConfig(
            precision=PrecisionConfig(param_dtype="float32"),
            pipeline=PipelineConfig(schedule=schedule, stages_per_rank=chunks, microbatches=4)))
        objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"),
                                          MultiTaskConditioning())
        state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-3),
                           rng=RNGStreams.for_rank(0, data_rank=0))
        ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-3),
                               rng=RNGStreams.for_rank(0, data_rank=0))
        c = ref.config
        gen = torch.Generator().manual_seed(8)
        micro = [random_batch(batch=1, channels=c.in_channels, frames=4, height=16, width=32, text_tokens=16,
                              text_width=c.text_width, generator=gen, device=dev) for _ in range(4)]
        _, metrics = pipeline_train_step(state, micro, objective, pm.pipeline, patchifier=ref.patchifier,
                                         max_grad_norm=1.0, pp_mesh=pm.pp_mesh)
        losses = []
        for i, b in enumerate(micro):
            _, rm = train_step(ref_state, b, objective, patchifier=ref.patchifier, gradient_accumulation_steps=4,
                               microbatch_index=i, max_grad_norm=1.0)
            losses.append(float(rm.loss))
        torch.cuda.synchronize()
        want = sum(losses) / 4
        assert abs(float(metrics.loss) - want) <= 2e-2 * max(1.0, abs(want)), (float(metrics.loss), want)
        mine = dict(pm.model.named_parameters())
        for name, q in ref.named_parameters():
            if name in mine:
                err = (mine[name].detach() - q.detach()).abs().max().item()
                assert err <= 2.5e-3, f"{name}: {err}"  # AdamW moves each parameter by about lr
        assert check_errors(dev) == 0
    except BaseException:
        leave_on_failure()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.parametrize("schedule,chunks", [("1f1b", 1), ("interleaved_1f1b", 2)])
def test_pipeline_over_nccl_matches_unsharded(schedule: str, chunks: int) -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), schedule, chunks), nprocs=2, join=True)
