"""Functional train step and the Trainer loop (avgen/train/trainer.py:169-683).

``train_step``: zero grads on the first micro-step, gradient sync only on the
last, loss / accumulation backward, then on the last micro-step clip by the
global norm, neutralise a non-finite step without any collective (its
gradients count as zero, so ranks never desync or deadlock), optimizer,
schedule and EMA steps, progress counters. With :class:`FusedAdamW` the norm,
clip coefficient and non-finite flag never leave the device.
"""
from __future__ import annotations

import bisect
import logging
from collections.abc import Iterable, Iterator, Sequence
from contextlib import nullcontext
from dataclasses import dataclass, field
from typing import Any, Protocol, runtime_checkable

import torch
from torch.distributed.device_mesh import DeviceMesh

from avgen_b200.core._validate import require_name
from avgen_b200.core.limits import Limit, enforce
from avgen_b200.core.batch import MediaBatch
from avgen_b200.core.metrics import StepMetrics
from avgen_b200.core.patchify import GridPatchifier, Patchifier
from avgen_b200.core.state import TrainState
from avgen_b200.train.objective import Objective, ObjectiveOutput
from avgen_b200.train.optimizer import FusedAdamW, MultiTensorAdamW

__all__ = ["Curriculum", "CurriculumStage", "MetricSink", "ResolutionBucket", "Trainer", "TrainerCallback",
           "TrainerConfig", "TrainerTelemetry", "optimizer_update", "pipeline_train_step", "train_step"]

_LOG = logging.getLogger("avgen_b200.train")


@runtime_checkable
class MetricSink(Protocol):
    def log_metrics(self, metrics: dict[str, float], step: int) -> None: ...


@runtime_checkable
class TrainerCallback(Protocol):
    def on_step_end(self, trainer: Trainer, state: TrainState, metrics: StepMetrics) -> None: ...

    def on_checkpoint(self, trainer: Trainer, state: TrainState) -> None: ...

    def on_eval(self, trainer: Trainer, state: TrainState) -> None: ...


@dataclass(frozen=True, slots=True)
class ResolutionBucket:
    name: str
    frames: int
    height: int
    width: int

    def __post_init__(self) -> None:
        require_name("name", self.name)
        enforce(self, _GRID_LIMITS)

    @property
    def latents(self) -> int:
        return self.frames * self.height * self.width


@dataclass(frozen=True, slots=True)
class CurriculumStage:
    name: str
    until_step: int
    buckets: tuple[tuple[ResolutionBucket, float], ...]

    def __post_init__(self) -> None:
        require_name("name", self.name)
        enforce(self, {"until_step": Limit(lo=1, integer=True)})
        weights = [w for _, w in self.buckets]
        if not weights or min(weights) < 0 or not sum(weights) > 0:
            raise ValueError(f"stage {self.name!r} needs at least one bucket, no negative weight and a positive "
                             f"total; got weights {weights}")


@dataclass(frozen=True, slots=True)
class Curriculum:
    stages: tuple[CurriculumStage, ...] = ()

    def __post_init__(self) -> None:
        bounds = [s.until_step for s in self.stages]
        if bounds != sorted(set(bounds)):
            raise ValueError(f"curriculum stages must have strictly increasing until_step; got {bounds}")

    @property
    def is_empty(self) -> bool:
        return not self.stages

    def stage_for(self, step: int) -> CurriculumStage | None:
        """The first stage whose ``until_step`` lies beyond ``step`` (the last stage
        stays active after the schedule ends)."""
        if not self.stages:
            return None
        at = bisect.bisect_right([s.until_step for s in self.stages], step)
        return self.stages[min(at, len(self.stages) - 1)]


@dataclass(frozen=True, slots=True)
class TrainerConfig:
    gradient_accumulation_steps: int = 1
    max_grad_norm: float | None = 1.0
    log_every: int = 10
    eval_every: int = 0
    checkpoint_every: int = 0
    autocast_dtype: str = "bfloat16"
    curriculum: Curriculum = field(default_factory=Curriculum)
    data_world: int = 1

    def __post_init__(self) -> None:
        enforce(self, _TRAINER_LIMITS)
        if not isinstance(getattr(torch, self.autocast_dtype, None), torch.dtype):
            raise ValueError(f"unknown autocast dtype {self.autocast_dtype!r}")

    @property
    def torch_autocast_dtype(self) -> torch.dtype:
        return getattr(torch, self.autocast_dtype)


_GRID_LIMITS = {axis: Limit(lo=1, integer=True) for axis in ("frames", "height", "width")}
# cadences of 0 switch eval / checkpoint callbacks off; logging always has one
_TRAINER_LIMITS = {"gradient_accumulation_steps": Limit(lo=1, integer=True), "log_every": Limit(lo=1, integer=True),
                   "data_world": Limit(lo=1, integer=True), "eval_every": Limit(lo=0, integer=True),
                   "checkpoint_every": Limit(lo=0, integer=True),
                   "max_grad_norm": Limit(lo=0.0, lo_open=True, optional=True)}


def _native(model: torch.nn.Module) -> bool:
    from avgen_b200.models.dit import VideoDiT

    inner = getattr(model, "module", model)
    return isinstance(inner, VideoDiT)


def _autocast(model: torch.nn.Module, device: torch.device, dtype: torch.dtype) -> Any:
    # Native models pick bf16 per op themselves (fp32 coords and statistics stay fp32).
    if device.type != "cuda" or _native(model):
        return nullcontext()
    return torch.autocast(device_type="cuda", dtype=dtype)


@dataclass(frozen=True, slots=True)
class _MicroStep:
    """Where a micro-batch sits in its optimizer step."""

    index: int
    count: int

    def __post_init__(self) -> None:
        if not 0 <= self.index < self.count:
            raise ValueError(f"microbatch_index={self.index} must lie in [0, {self.count})")

    @property
    def opens(self) -> bool:
        return self.index == 0

    @property
    def closes(self) -> bool:
        return self.index == self.count - 1

    @property
    def loss_scale(self) -> float:
        return 1.0 / self.count


def _device_clipping(opt: Any) -> bool:
    """Optimizers that clip, skip and report the norm on the device themselves."""
    return isinstance(opt, (FusedAdamW, MultiTensorAdamW))


def _clear_gradients(opt: Any) -> None:
    # the flat-buffer optimizer keeps its gradient views alive; the others drop them
    opt.zero_grad(set_to_none=not isinstance(opt, FusedAdamW))


def _set_gradient_sync(model: torch.nn.Module, enabled: bool) -> None:
    setter = getattr(model, "set_requires_gradient_sync", None)
    if callable(setter):
        setter(enabled)


def _host_clip_and_step(state: TrainState, max_grad_norm: float | None, pp_mesh: DeviceMesh | None,
                        data_group: Any, finite: torch.Tensor, dev: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """The path for optimizers without device-side clipping: average over the data
    group, global norm (clip when asked), zero a non-finite step's gradients on the
    device (no collective decides it), step."""
    import torch.distributed as dist

    from avgen_b200.parallel.comm import clip_grad_norm, global_grad_norm

    params = [p for p in state.model.parameters() if p.grad is not None]
    if not params:
        state.optimizer.step()
        return torch.zeros((), dtype=torch.float32, device=dev), finite
    if data_group is not None and dist.is_initialized() and dist.get_world_size(data_group) > 1:
        world = dist.get_world_size(data_group)
        for p in params:
            dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=data_group)
            p.grad.div_(world)
    if max_grad_norm is not None:
        norm = clip_grad_norm(params, max_grad_norm, pp_mesh=pp_mesh)
    else:  # still the whole model's norm (stages and head-parallel slices), only not clipped
        norm = global_grad_norm(params, pp_mesh=pp_mesh)
    norm = norm.to(torch.float32)
    finite = finite & torch.isfinite(norm)
    with torch.no_grad():
        for p in params:
            p.grad.mul_(finite.to(p.grad.dtype)).nan_to_num_(0.0, 0.0, 0.0)
    state.optimizer.step()
    return norm, finite


def optimizer_update(state: TrainState, *, max_grad_norm: float | None = None, pp_mesh: DeviceMesh | None = None,
                     data_group: Any = None, finite: torch.Tensor | None = None,
                     ) -> tuple[torch.Tensor, torch.Tensor]:
    """The end of an optimizer step after ``backward``: clip by the global norm,
    neutralise a non-finite step on device (no collective), optimizer, schedule
    and EMA steps, ``state.step += 1``. Returns ``(grad_norm, finite)``.
    Shared by :func:`train_step` and the RL trainers."""
    opt = state.optimizer
    dev = next((p.device for p in state.model.parameters()), torch.device("cpu"))
    finite = torch.ones((), dtype=torch.bool, device=dev) if finite is None else finite
    if _device_clipping(opt):
        opt.step(max_grad_norm=max_grad_norm)
        norm = opt.last_grad_norm.to(device=dev, dtype=torch.float32)
        finite = finite & ~opt.last_nonfinite.to(dev)
    else:
        norm, finite = _host_clip_and_step(state, max_grad_norm, pp_mesh, data_group, finite, dev)
    for follower in (state.schedule, state.ema):
        if follower is None:
            continue
        if follower is state.ema:
            follower.update(state.model)
        else:
            follower.step()
    state.step += 1
    return norm, finite


def train_step(state: TrainState, batch: MediaBatch, objective: Objective, *, patchifier: Patchifier,
               gradient_accumulation_steps: int = 1, microbatch_index: int = 0, max_grad_norm: float | None = None,
               cp_mesh: DeviceMesh | None = None, pp_mesh: DeviceMesh | None = None,
               autocast_dtype: torch.dtype = torch.bfloat16, data_world: int = 1,
               data_group: Any = None) -> tuple[TrainState, StepMetrics]:
    """One micro-step (and the optimizer step on the last micro-step).

    ``data_group`` (native data parallelism, see ``ParallelModel.data_group``):
    ranks whose gradients are averaged before the optimizer step. The fused
    AdamW averages its flat buffer over its own ``dp_group`` instead.
    """
    micro = _MicroStep(microbatch_index, gradient_accumulation_steps)
    dev = batch.device
    if micro.opens:
        _clear_gradients(state.optimizer)
    # sharded / replicated gradients are reduced once, after the step's last micro-batch
    _set_gradient_sync(state.model, micro.closes)
    with _autocast(state.model, dev, autocast_dtype):
        out: ObjectiveOutput = objective(state.model, batch, state.rng, patchifier=patchifier, cp_mesh=cp_mesh)
    (out.loss * micro.loss_scale).backward()
    finite = torch.isfinite(out.loss.detach())
    norm = torch.zeros((), dtype=torch.float32, device=dev)
    if micro.closes:
        norm, finite = optimizer_update(state, max_grad_norm=max_grad_norm, pp_mesh=pp_mesh, data_group=data_group,
                                        finite=finite)
    samples = batch.spec.batch_size * data_world
    state.samples_seen += samples
    state.tokens_seen += samples * batch.spec.sequence_length
    skipped = (~finite) if micro.closes else torch.zeros((), dtype=torch.bool, device=dev)
    as_scalar = lambda t: t.detach().to(torch.float32).reshape(())  # noqa: E731
    metrics = StepMetrics(loss=as_scalar(out.loss), video_loss=as_scalar(out.video_loss),
                          audio_loss=as_scalar(out.audio_loss), valid_video_tokens=out.valid_video_tokens,
                          valid_audio_tokens=out.valid_audio_tokens, grad_norm=norm.reshape(()),
                          nonfinite=(~finite).reshape(()), skipped=skipped.reshape(()))
    return state, metrics


def pipeline_train_step(state: TrainState, micro_batches: Sequence[MediaBatch], objective: Any, runner: Any, *,
                        patchifier: Patchifier, max_grad_norm: float | None = None,
                        cp_mesh: DeviceMesh | None = None, pp_mesh: DeviceMesh | None = None,
                        data_world: int = 1, data_group: Any = None) -> tuple[TrainState, StepMetrics]:
    """One optimizer step of a pipeline-parallel model: every stage prepares the same
    model inputs (same RNG streams on a data rank), ``runner`` (a
    :class:`~avgen_b200.parallel.pipeline.PipelineRunner`) drives the micro-batches
    through the stages, the last stage evaluates the loss, and the optimizer step
    (global norm summed over the stages) follows. Returns the step's mean metrics on
    every stage."""
    import torch.distributed as dist

    if not micro_batches:
        raise ValueError("pipeline_train_step needs at least one micro-batch")
    opt = state.optimizer
    if pp_mesh is not None and hasattr(opt, "norm_groups") and not opt.norm_groups:
        opt.norm_groups = (pp_mesh.get_group(),)  # the clip uses the norm over every stage's gradients
    _clear_gradients(opt)
    prepared = [objective.prepare(b, state.rng, patchifier=patchifier, cp_mesh=cp_mesh) for b in micro_batches]
    outcomes: list[ObjectiveOutput] = []

    def loss_fn(k: int, output: Any) -> torch.Tensor:
        out = objective.finish(output, prepared[k][0], prepared[k][1])
        outcomes.append(out)
        return out.loss / len(micro_batches)

    runner.run([p[0] for p in prepared], loss_fn)
    dev = micro_batches[0].device
    stats = torch.zeros(5, dtype=torch.float32, device=dev)  # loss, video, audio, valid video, valid audio
    for out in outcomes:
        stats += torch.stack([out.loss.detach().float(), out.video_loss.float(), out.audio_loss.float(),
                              out.valid_video_tokens.float(), out.valid_audio_tokens.float()])
    if pp_mesh is not None and dist.is_initialized():
        dist.all_reduce(stats, group=pp_mesh.get_group())  # only the last stage contributes
    stats[:3] /= len(micro_batches)
    finite = torch.isfinite(stats[0])
    norm, finite = optimizer_update(state, max_grad_norm=max_grad_norm, pp_mesh=pp_mesh, data_group=data_group,
                                    finite=finite)
    samples = sum(b.spec.batch_size for b in micro_batches) * data_world
    state.samples_seen += samples
    state.tokens_seen += samples * micro_batches[0].spec.sequence_length
    metrics = StepMetrics(loss=stats[0], video_loss=stats[1], audio_loss=stats[2],
                          valid_video_tokens=stats[3].to(torch.int64), valid_audio_tokens=stats[4].to(torch.int64),
                          grad_norm=norm.reshape(()), nonfinite=(~finite).reshape(()), skipped=(~finite).reshape(()))
    return state, metrics


@dataclass(slots=True)
class TrainerTelemetry:
    """What the fit loop measures besides the loss; every part is optional.

    ``accumulator`` averages step metrics over each log window (one collective and
    one host sync per log line); ``throughput`` times steps on the device (events,
    no per-step sync) and reports samples/s and MFU as the max over ranks;
    ``profiler`` is a torch profiler context (``telemetry.profile_steps``) stepped
    once per optimizer step; ``memory`` reports allocator peaks every
    ``memory_every`` steps."""

    accumulator: Any = None
    throughput: Any = None
    profiler: Any = None
    memory: Any = None
    memory_every: int = 0


class Trainer:
    """The fit loop: cadence callbacks, logging, telemetry, curriculum stage announcements."""

    def __init__(self, state: TrainState, objective: Objective, parallel: Any, config: TrainerConfig, *,
                 patchifier: Patchifier | None = None, callbacks: Sequence[TrainerCallback] = (),
                 logger: MetricSink | None = None, telemetry: TrainerTelemetry | None = None) -> None:
        self.state = state
        self.objective = objective
        self.parallel = parallel
        self.config = config
        self.patchifier = patchifier or _model_patchifier(state.model)
        self.callbacks = tuple(callbacks)
        self.logger = logger
        self.telemetry = telemetry or TrainerTelemetry()
        self._stage_name: str | None = None

    @property
    def device(self) -> torch.device:
        return next((p.device for p in self.state.model.parameters()), torch.device("cpu"))

    def train_step(self, batch: MediaBatch, *, microbatch_index: int = 0, accumulation: int | None = None,
                   ) -> StepMetrics:
        _, metrics = train_step(
            self.state, batch, self.objective, patchifier=self.patchifier,
            gradient_accumulation_steps=accumulation or self.config.gradient_accumulation_steps,
            microbatch_index=microbatch_index, max_grad_norm=self.config.max_grad_norm,
            cp_mesh=getattr(self.parallel, "cp_mesh", None), pp_mesh=getattr(self.parallel, "pp_mesh", None),
            autocast_dtype=self.config.torch_autocast_dtype, data_world=self.config.data_world,
            data_group=getattr(self.parallel, "data_group", None))
        return metrics

    def run_step(self, micro_batches: Sequence[MediaBatch]) -> StepMetrics:
        """One optimizer step over its micro-batches; returns the last micro-step's metrics
        (the step's means under pipeline parallelism)."""
        runner = getattr(self.parallel, "pipeline", None)
        if runner is not None:
            _, metrics = pipeline_train_step(
                self.state, micro_batches, self.objective, runner, patchifier=self.patchifier,
                max_grad_norm=self.config.max_grad_norm, cp_mesh=getattr(self.parallel, "cp_mesh", None),
                pp_mesh=getattr(self.parallel, "pp_mesh", None), data_world=self.config.data_world,
                data_group=getattr(self.parallel, "data_group", None))
            return metrics
        metrics = None
        for index, batch in enumerate(micro_batches):
            metrics = self.train_step(batch, microbatch_index=index, accumulation=len(micro_batches))
        assert metrics is not None
        return metrics

    def fit(self, loader: Iterable[MediaBatch], total_steps: int | None = None) -> None:
        if total_steps is not None and (isinstance(total_steps, bool) or total_steps < 1):
            raise ValueError(f"total_steps must be positive; got {total_steps!r}")
        tel = self.telemetry
        profiler = tel.profiler if tel.profiler is not None else nullcontext()
        with profiler:
            if tel.throughput is not None:
                tel.throughput.start()
            self._announce_stage(loader)
            for window in _step_windows(loader, self.config.gradient_accumulation_steps, self.device):
                metrics = self.run_step(window)
                self._measure(metrics, window)
                self._on_step_end(metrics)
                self._announce_stage(loader)
                if total_steps is not None and self.state.step >= total_steps:
                    return

    def _measure(self, metrics: StepMetrics, window: Sequence[MediaBatch]) -> None:
        tel = self.telemetry
        if tel.accumulator is not None:
            tel.accumulator.update(metrics)
        if tel.throughput is not None:
            samples = sum(b.spec.batch_size for b in window) * self.config.data_world
            tel.throughput.step(samples=samples, tokens=samples * window[0].spec.sequence_length)
        step = getattr(tel.profiler, "step", None)
        if callable(step):
            step()

    def _log_line(self, metrics: StepMetrics) -> dict[str, float]:
        tel = self.telemetry
        line = tel.accumulator.flush() if tel.accumulator is not None else metrics.to_mapping()
        line.update({f"progress/{k}": float(v) for k, v in self.state.progress().items()})
        if tel.throughput is not None:
            line.update(tel.throughput.report().to_mapping())
        step = self.state.step
        if tel.memory is not None and tel.memory_every and step % tel.memory_every == 0:
            report = tel.memory.report()
            if report is not None:
                line.update(report.to_mapping())
        if self.state.schedule is not None:
            line["lr"] = self.state.schedule.get_last_lr()[0]
        return line

    def _on_step_end(self, metrics: StepMetrics) -> None:
        step = self.state.step
        _dispatch(self.callbacks, "on_step_end", self, self.state, metrics)
        cadence = {"log": self.config.log_every, "eval": self.config.eval_every,
                   "checkpoint": self.config.checkpoint_every}
        due = {name for name, every in cadence.items() if every and step % every == 0}
        if "log" in due:
            line = self._log_line(metrics)
            if self.logger is not None:
                self.logger.log_metrics(line, step)
            else:
                _LOG.info("step %d %s", step, line)
        for hook in ("eval", "checkpoint"):
            if hook in due:
                _dispatch(self.callbacks, f"on_{hook}", self, self.state)

    def _announce_stage(self, loader: object) -> None:
        stage = self.config.curriculum.stage_for(self.state.step)
        if stage is None or stage.name == self._stage_name:
            return
        self._stage_name = stage.name
        setter = getattr(loader, "set_curriculum", None)
        if callable(setter):
            setter(stage)
        _LOG.info("curriculum stage %r active at step %d", stage.name, self.state.step)


def _step_windows(loader: Iterable[MediaBatch], size: int, device: torch.device) -> Iterator[list[MediaBatch]]:
    """The loader's batches on ``device``, grouped into optimizer steps of ``size``
    micro-batches (a trailing partial group is dropped: it cannot close a step)."""
    window: list[MediaBatch] = []
    for batch in loader:
        window.append(batch if batch.device == device else batch.to(device))
        if len(window) == size:
            yield window
            window = []


def _dispatch(callbacks: Sequence[Any], hook: str, *args: object) -> None:
    for cb in callbacks:
        method = getattr(cb, hook, None)
        if callable(method):
            method(*args)


def _model_patchifier(model: torch.nn.Module) -> Patchifier:
    inner = getattr(model, "module", model)
    cand = getattr(inner, "patchifier", None)
    return cand if isinstance(cand, Patchifier) else GridPatchifier()
