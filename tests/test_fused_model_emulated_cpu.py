"""Whole-model training steps through the fused DiT block on CPU, with the kernels
restated in PyTorch (``kernel_emulator``) and the fused path forced on: a
flow-matching step of the tiny model matches the eager model, and a two-stage
1F1B pipeline over ``gloo`` with fused blocks on both stages matches the
unsharded eager model with gradient accumulation (loss and gradient norm, bf16
tolerance), and so does a two-rank context-parallel step whose fused blocks
attend over the whole sequence (K/V gathered, dK/dV reduce-scattered) with their
parameters sharded over the cp ranks by FSDP2 (the flagship's layout at two GPUs),
an interleaved 1F1B pipeline (4 chunks over 2 ranks) and head-parallel tensor
parallelism with sequence parallelism (3 heads as [2, 1], two samples per batch). The
pipeline is the path where a wrong gradient list from the fused node leaves one
rank waiting on the other."""
from __future__ import annotations

import os
import socket
from dataclasses import asdict
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from kernel_emulator import emulate_kernels

from avgen_b200.models import blocks as blocks_mod


def _model():  # noqa: ANN202
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    cfg["depth"] = 2
    model = build_model("video_dit", cfg)
    model.init_weights()
    with torch.no_grad():  # non-zero gates and output projections: every parameter gets a gradient
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    return model


class _ForcedFused:
    """Run every block through the fused node (kernels emulated) and count the calls."""

    def __enter__(self) -> _ForcedFused:
        import avgen_b200.models.fused as fused_mod

        self.calls = 0
        self._eligible = blocks_mod._fused_eligible
        self._forward = fused_mod.fused_block_forward
        self._emulation = emulate_kernels()
        self._emulation.__enter__()
        blocks_mod._fused_eligible = lambda b, h: True
        original = self._forward

        def counting(*args, **kwargs):  # noqa: ANN002, ANN003, ANN202
            self.calls += 1
            return original(*args, **kwargs)

        fused_mod.fused_block_forward = counting
        return self

    def __exit__(self, *exc: object) -> None:
        import avgen_b200.models.fused as fused_mod

        fused_mod.fused_block_forward = self._forward
        blocks_mod._fused_eligible = self._eligible
        self._emulation.__exit__(*exc)


def _objective():  # noqa: ANN202
    from avgen_b200.train import FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, \
        build_timestep_sampler

    return FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())


def _batches(model, n: int, seed: int):  # noqa: ANN001, ANN202
    from avgen_b200.data.synthetic_batch import random_batch

    c = model.config
    gen = torch.Generator().manual_seed(seed)
    return [random_batch(batch=2, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                         text_width=c.text_width, generator=gen) for _ in range(n)]


def test_fused_training_step_matches_eager(monkeypatch: pytest.MonkeyPatch) -> None:
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.train import build_optimizer, train_step

    monkeypatch.setenv("AVGEN_KEEP_ACTIVATIONS", "none")
    results = []
    for fused in (False, True):
        model = _model()
        state = TrainState(model=model, optimizer=build_optimizer(model, lr=1e-3),
                           rng=RNGStreams.for_rank(0, data_rank=0))
        batch = _batches(model, 1, seed=3)[0]
        if fused:
            with _ForcedFused() as forced:
                _, metrics = train_step(state, batch, _objective(), patchifier=model.patchifier, max_grad_norm=None)
            assert forced.calls == len(model.blocks)
        else:
            _, metrics = train_step(state, batch, _objective(), patchifier=model.patchifier, max_grad_norm=None)
        results.append((float(metrics.loss), float(metrics.grad_norm)))
    (loss_e, norm_e), (loss_f, norm_f) = results
    assert abs(loss_f - loss_e) <= 2e-2 * abs(loss_e)
    assert abs(norm_f - norm_e) <= 5e-2 * norm_e


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pipeline_worker(rank: int, world: int, port: int) -> None:
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PipelineConfig, PrecisionConfig, parallelize
    from avgen_b200.train import build_optimizer, train_step
    from avgen_b200.train.trainer import pipeline_train_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AVGEN_KEEP_ACTIVATIONS="none")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        ref = _model()
        dims = ParallelDims(world_size=world, pipeline=world)
        pm = parallelize(_model(), dims, mesh=dims.build_mesh("cpu"),
                         config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32"),
                                               pipeline=PipelineConfig(schedule="1f1b")))
        state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-3),
                           rng=RNGStreams.for_rank(0, data_rank=0))
        ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-3),
                               rng=RNGStreams.for_rank(0, data_rank=0))
        micro = _batches(ref, 3, seed=5)
        with _ForcedFused() as forced:
            _, metrics = pipeline_train_step(state, micro, _objective(), pm.pipeline, patchifier=ref.patchifier,
                                             max_grad_norm=1.0, pp_mesh=pm.pp_mesh)
        assert forced.calls == len(pm.model.blocks) * len(micro)  # this stage's blocks, every micro-batch
        losses = []
        for i, b in enumerate(micro):
            _, rm = train_step(ref_state, b, _objective(), patchifier=ref.patchifier, gradient_accumulation_steps=3,
                               microbatch_index=i, max_grad_norm=1.0)
            losses.append(float(rm.loss))
        want = sum(losses) / 3
        assert abs(float(metrics.loss) - want) <= 2e-2 * abs(want), (float(metrics.loss), want)
        assert abs(float(metrics.grad_norm) - float(rm.grad_norm)) <= 5e-2 * float(rm.grad_norm)
    finally:
        dist.destroy_process_group()


def test_two_stage_pipeline_with_fused_blocks_matches_unsharded() -> None:
    mp.spawn(_pipeline_worker, args=(2, _free_port()), nprocs=2, join=True)


def _context_worker(rank: int, world: int, port: int) -> None:
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PrecisionConfig, parallelize
    from avgen_b200.parallel.context import ContextParallelAttention
    from avgen_b200.train import build_optimizer, train_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AVGEN_KEEP_ACTIVATIONS="none")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        ref = _model()
        dims = ParallelDims(world_size=world, context=world)
        pm = parallelize(_model(), dims, mesh=dims.build_mesh("cpu"),
                         config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32")))
        assert all(isinstance(b.attention_impl, ContextParallelAttention) for b in pm.model.blocks)
        assert any(a.startswith("fsdp(cp=") for a in pm.applied), pm.applied  # parameters sharded over cp
        state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-3),
                           rng=RNGStreams.for_rank(0, data_rank=0))
        ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-3),
                               rng=RNGStreams.for_rank(0, data_rank=0))
        batch = _batches(ref, 1, seed=9)[0]
        with _ForcedFused() as forced:
            _, metrics = train_step(state, batch, _objective(), patchifier=ref.patchifier, max_grad_norm=None,
                                    cp_mesh=pm.cp_mesh)
        assert forced.calls == len(pm.model.blocks)
        _, want = train_step(ref_state, batch, _objective(), patchifier=ref.patchifier, max_grad_norm=None)
        loss = metrics.loss.detach().reshape(1).clone()
        dist.all_reduce(loss)  # each rank reports its shard's share; the step's loss is their mean
        assert abs(float(loss) / world - float(want.loss)) <= 2e-2 * abs(float(want.loss))
        assert abs(float(metrics.grad_norm) - float(want.grad_norm)) <= 5e-2 * float(want.grad_norm)
    finally:
        dist.destroy_process_group()


def test_context_parallel_step_with_fused_blocks_matches_unsharded() -> None:
    mp.spawn(_context_worker, args=(2, _free_port()), nprocs=2, join=True)


def _deep_model(depth: int = 4, heads: int | None = None):  # noqa: ANN202
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    cfg["depth"] = depth
    if heads is not None:
        cfg.update(num_heads=heads, width=16 * heads)
    model = build_model("video_dit", cfg)
    model.init_weights()
    with torch.no_grad():
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    return model


def _layout_worker(rank: int, world: int, port: int, layout: str) -> None:
    """Interleaved 1F1B (4 chunks over 2 ranks) or head-parallel TP with sequence
    parallelism (3 heads as [2, 1]), fused blocks emulated, against the eager model."""
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PipelineConfig, PrecisionConfig, parallelize
    from avgen_b200.train import build_optimizer, train_step
    from avgen_b200.train.trainer import pipeline_train_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), AVGEN_KEEP_ACTIVATIONS="none")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        heads = 3 if layout == "tp" else None
        ref = _deep_model(heads=heads)
        fp32 = PrecisionConfig(param_dtype="float32")
        if layout == "tp":
            dims = ParallelDims(world_size=world, tensor=world)
            cfg = ParallelConfig(precision=fp32, sequence_parallel=True)
        else:
            dims = ParallelDims(world_size=world, pipeline=world)
            cfg = ParallelConfig(precision=fp32, pipeline=PipelineConfig(schedule="interleaved_1f1b",
                                                                         stages_per_rank=2, microbatches=4))
        pm = parallelize(_deep_model(heads=heads), dims, mesh=dims.build_mesh("cpu"), config=cfg)
        state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-3),
                           rng=RNGStreams.for_rank(0, data_rank=0))
        ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-3),
                               rng=RNGStreams.for_rank(0, data_rank=0))
        micro = _batches(ref, 4 if layout != "tp" else 1, seed=13)
        with _ForcedFused() as forced:
            if layout == "tp":
                _, metrics = train_step(state, micro[0], _objective(), patchifier=ref.patchifier, max_grad_norm=None)
            else:
                _, metrics = pipeline_train_step(state, micro, _objective(), pm.pipeline, patchifier=ref.patchifier,
                                                 max_grad_norm=1.0, pp_mesh=pm.pp_mesh)
        assert forced.calls > 0
        losses = []
        for i, b in enumerate(micro):
            _, rm = train_step(ref_state, b, _objective(), patchifier=ref.patchifier,
                               gradient_accumulation_steps=len(micro), microbatch_index=i,
                               max_grad_norm=None if layout == "tp" else 1.0)
            losses.append(float(rm.loss))
        want = sum(losses) / len(losses)
        assert abs(float(metrics.loss) - want) <= 2e-2 * abs(want), (layout, float(metrics.loss), want)
        assert abs(float(metrics.grad_norm) - float(rm.grad_norm)) <= 5e-2 * float(rm.grad_norm)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", ["interleaved", "tp"])
def test_other_layouts_with_fused_blocks_match_unsharded(layout: str) -> None:
    mp.spawn(_layout_worker, args=(2, _free_port(), layout), nprocs=2, join=True)
