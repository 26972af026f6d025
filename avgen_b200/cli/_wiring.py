"""Build a training run from a :class:`~avgen_b200.config.RunConfig` (the stack behind
``avgen-b200 train`` / ``finetune`` / ``rl``; avgen/cli/_wiring.py:381-485 role).

Order: process group -> parallel dims and mesh -> model (meta, then
materialised on the device) -> ``parallelize`` (with the ``adapt`` hook for
fine-tuning) -> optimizer (fused AdamW over native data parallelism) -> LR
schedule -> EMA -> objective -> data loader -> checkpoint manager (with resume)
-> logger -> :class:`~avgen_b200.train.Trainer` with checkpoint callbacks.
"""
from __future__ import annotations

import logging
from collections.abc import Callable
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from torch import nn

__all__ = ["RunStack", "build_run", "build_telemetry", "run_training"]

_LOG = logging.getLogger(__name__)


@dataclass(slots=True)
class RunStack:
    config: Any
    env: Any
    parallel: Any
    state: Any
    objective: Any
    loader: Any
    trainer: Any
    manager: Any
    logger: Any
    accumulation: int
    output_dir: Path


class _CheckpointCallback:
    def __init__(self, manager: Any, parallel: Any, async_save: bool) -> None:
        self.manager, self.parallel, self.async_save = manager, parallel, async_save

    def on_checkpoint(self, trainer: Any, state: Any) -> None:
        self.manager.save(state.step, state, parallel=self.parallel, async_save=self.async_save)


def build_run(config: Any, *, adapt: Callable[[nn.Module], nn.Module] | None = None,
              model_hook: Callable[[nn.Module], nn.Module] | None = None, objective: Any = None,
              output_dir: str | None = None) -> RunStack:
    from avgen_b200.checkpoint import CheckpointManager
    from avgen_b200.config.resolve import build_model, build_parallel_config, build_parallel_dims
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.loader import build_loader
    from avgen_b200.parallel import init_distributed, parallelize
    from avgen_b200.telemetry.logger import build_logger
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, ShardedEMA,
                                  Trainer, TrainerConfig, build_optimizer, build_schedule, build_timestep_sampler)

    env = init_distributed()
    dims = build_parallel_dims(config, world_size=env.world_size)
    mesh = dims.build_mesh(env.device.type) if env.world_size > 1 else None
    torch.manual_seed(config.seed)
    model = build_model(config, meta=True).to_empty(device=env.device)
    model.init_weights()
    if model_hook is not None:
        model = model_hook(model)
    pm = parallelize(model, dims, mesh=mesh, config=build_parallel_config(config), adapt=adapt)
    data_rank, data_world = dims.data_coordinates(mesh)
    t = config.train
    opt = build_optimizer(pm.model, name=t.optimizer, lr=t.lr, weight_decay=t.weight_decay, betas=tuple(t.betas),
                          eps=t.eps, dp_group=pm.data_group)
    sched = build_schedule(t.schedule, opt, total_steps=t.steps, warmup_steps=t.warmup_steps,
                           decay_fraction=t.decay_ratio, min_lr_ratio=t.min_lr_ratio)
    ema = ShardedEMA(pm.model, decay=t.ema_decay, warmup_steps=t.ema_warmup_steps,
                     optimizer=opt) if t.ema_decay > 0 else None
    state = TrainState(model=pm.model, optimizer=opt, schedule=sched, ema=ema,
                       rng=RNGStreams.for_rank(t.seed or config.seed, data_rank=data_rank, device=env.device))
    if objective is None:
        sampler = build_timestep_sampler(t.timestep_sampler, _sampler_options(t))
        objective = FlowMatchingObjective(FlowMatchingConfig(audio_weight=t.audio_loss_weight), sampler,
                                          MultiTaskConditioning(text_dropout=config.data.caption_dropout))
    from avgen_b200.config.resolve import gradient_accumulation

    accumulation = gradient_accumulation(config, world_size=env.world_size)
    loader = build_loader(config, data_rank=data_rank, data_world=data_world)
    out = Path(output_dir or config.output_dir)
    ck = config.checkpoint
    manager = CheckpointManager(ck.dir or out / "checkpoints", keep_last_n=ck.keep_last_n,
                                keep_every_n_steps=ck.keep_every_n_steps)
    tel = config.telemetry
    logger = build_logger(tel.loggers, output_dir=out, jsonl_path=tel.jsonl_path, tensorboard_dir=tel.tensorboard_dir,
                          project=tel.project, run_name=config.resolved_run_name())
    trainer = Trainer(state, objective, pm, TrainerConfig(gradient_accumulation_steps=accumulation,
                                                          max_grad_norm=t.max_grad_norm, log_every=tel.log_every,
                                                          eval_every=t.eval_every, checkpoint_every=ck.save_every,
                                                          data_world=data_world),
                      patchifier=getattr(model, "patchifier", None),
                      callbacks=[_CheckpointCallback(manager, pm, ck.async_save)], logger=logger,
                      telemetry=build_telemetry(config, env=env, mesh=mesh, output_dir=out))
    if ck.resume:
        step = None if ck.resume == "latest" else None
        path = manager.root if ck.resume == "latest" else Path(ck.resume)
        if ck.load_model_only:
            from avgen_b200.checkpoint import load_model

            load_model(path, pm.model, strict=False)
        else:
            found = manager.load(state, parallel=pm, step=step) if ck.resume == "latest" else \
                CheckpointManager(path.parent).load(state, parallel=pm, step=_step_of(path))
            _LOG.info("resumed at step %s", found)
    return RunStack(config, env, pm, state, objective, loader, trainer, manager, logger, accumulation, out)


def build_telemetry(config: Any, *, env: Any, mesh: Any, output_dir: Path) -> Any:
    """The fit loop's measurements from ``config.telemetry``: metric means over each
    log window (averaged over data ranks), device-timed throughput with MFU of the
    configured model (max over ranks), an optional profiler window and memory
    reports."""
    from avgen_b200.config.resolve import build_model_shape
    from avgen_b200.simulate.compute import transformer_flops
    from avgen_b200.telemetry.metrics import MemoryReporter, MetricAccumulator, ThroughputMeter
    from avgen_b200.telemetry.profiler import profile_steps
    from avgen_b200.train import TrainerTelemetry

    tel = config.telemetry
    data_mesh = None
    if mesh is not None:
        from avgen_b200.parallel.dims import submesh

        data_mesh = next((m for m in (submesh(mesh, n) for n in ("dp_cp", "dp_shard_cp", "dp_replicate", "dp_shard",
                                                                   "cp")) if m is not None), None)
    shape = build_model_shape(config)
    per_sample = transformer_flops(shape)["total"] / max(1, shape.micro_batch_size) if tel.report_mfu else 0.0
    import torch.distributed as dist

    world_group = dist.group.WORLD if env.world_size > 1 else None
    throughput = ThroughputMeter(flops_per_sample=per_sample, world_size=env.world_size, group=world_group)
    profiler = (profile_steps(output_dir / "profile", active=tel.profile_steps, warmup=tel.profile_warmup)
                if tel.profile_steps > 0 else None)
    memory = MemoryReporter(env.device) if tel.memory_report_every > 0 else None
    return TrainerTelemetry(accumulator=MetricAccumulator(mesh=data_mesh), throughput=throughput, profiler=profiler,
                            memory=memory, memory_every=tel.memory_report_every)


def _sampler_options(t: Any) -> dict[str, Any]:
    if t.timestep_sampler == "logit_normal":
        return {"mean": t.logit_normal_mean, "std": t.logit_normal_std}
    if t.timestep_sampler == "shifted_logit_normal":
        return {"mean": t.logit_normal_mean, "std": t.logit_normal_std, "base_shift": t.base_shift,
                "max_shift": t.max_shift, "base_seq_len": t.base_seq_len, "max_seq_len": t.max_seq_len}
    return {}


def _step_of(path: Path) -> int | None:
    from avgen_b200.checkpoint.manager import _parse_step

    return _parse_step(path.name)


def run_training(stack: RunStack) -> None:
    """Fit to ``train.steps``, then write a final checkpoint and flush the logger."""
    cfg = stack.config
    try:
        stack.trainer.fit(stack.loader, total_steps=cfg.train.steps)
        stack.manager.save(stack.state.step, stack.state, parallel=stack.parallel, async_save=False)
    finally:
        stack.manager.close()
        close = getattr(stack.logger, "close", None)
        if callable(close):
            close()
