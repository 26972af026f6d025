"""Evaluation suite: metric bundles, prompt sharding across data ranks, exact
cross-rank merging and the pinned report (avgen/eval/suite.py:63-383 API)."""
from __future__ import annotations

from collections.abc import Callable, Iterable, Mapping, Sequence
from dataclasses import dataclass, field
from typing import Any

import torch

from avgen_b200.eval.learned import MissingBackendError, list_learned_metrics
from avgen_b200.eval.protocols import MetricError, RunningMetric, build_metric, list_metrics
from avgen_b200.eval.report import EvalPin, EvalReport, prompt_set_digest

__all__ = ["DEFAULT_PROMPTS", "EvalBatch", "MetricBundle", "build_metrics", "run_eval_suite", "shard_prompts",
           "torch_gather"]

DEFAULT_PROMPTS: tuple[str, ...] = (
    "a red balloon rising over a field", "waves breaking on a rocky shore", "a cat walking across a wooden floor",
    "steam rising from a cup of coffee", "a bicycle wheel spinning slowly", "leaves moving in the wind",
    "a candle flame flickering in a dark room", "traffic crossing a bridge at dusk")


@dataclass(slots=True)
class EvalBatch:
    video: torch.Tensor
    prompts: tuple[str, ...] = ()
    audio: torch.Tensor | None = None
    reference: torch.Tensor | None = None
    mask: torch.Tensor | None = None
    extra: dict[str, Any] = field(default_factory=dict)

    def as_inputs(self) -> dict[str, Any]:
        inputs: dict[str, Any] = {"video": self.video, **self.extra}
        if self.prompts:
            inputs["prompts"] = self.prompts
        for name in ("audio", "reference", "mask"):
            value = getattr(self, name)
            if value is not None:
                inputs[name] = value
        return inputs


@dataclass(slots=True)
class MetricBundle:
    metrics: dict[str, Any] = field(default_factory=dict)
    skipped: dict[str, str] = field(default_factory=dict)
    parameters: dict[str, str] = field(default_factory=dict)


_PIXEL_ON_LATENTS = ("pixel-space metric requested on latents; set eval.decode=true or drop it "
                     "(its value on latents would not measure what its name says)")


def _build_one(name: str, kwargs: dict[str, Any], decoded: bool) -> tuple[Any, str | None]:
    """(metric, None) when ``name`` can run here, else (None, why it is skipped)."""
    if name in list_learned_metrics():
        from avgen_b200.eval.learned import build_learned_metric

        try:
            return build_learned_metric(name, **kwargs), None
        except MissingBackendError as err:
            return None, str(err).splitlines()[0]
    if name not in list_metrics():
        raise MetricError(f"unknown metric {name!r}; built-ins: {', '.join(list_metrics())}; gated: "
                          f"{', '.join(list_learned_metrics())}")
    metric: RunningMetric = build_metric(name, **kwargs)
    if metric.pixel_space_only and not decoded:
        return None, _PIXEL_ON_LATENTS
    return metric, None


def build_metrics(names: Sequence[str], *, decoded: bool,
                  options: Mapping[str, Mapping[str, Any]] | None = None) -> MetricBundle:
    """Build each named metric; gated learned metrics whose backend is missing and
    pixel-space metrics on latents are recorded as skipped, with the reason."""
    bundle = MetricBundle()
    for name in names:
        kwargs = dict((options or {}).get(name, {}))
        metric, why = _build_one(name, kwargs, decoded)
        if metric is None:
            bundle.skipped[name] = why or "unavailable"
            continue
        bundle.metrics[name] = metric
        bundle.parameters[name] = ",".join(f"{k}={v!r}" for k, v in sorted(kwargs.items())) or "default"
    return bundle


def shard_prompts(prompts: Sequence[str], *, data_rank: int, data_world: int) -> tuple[str, ...]:
    if data_world < 1:
        raise ValueError(f"data_world must be >= 1; got {data_world!r}")
    if not 0 <= data_rank < data_world:
        raise ValueError(f"data_rank must be in [0, {data_world}); got {data_rank!r}")
    return tuple(prompts[data_rank::data_world])


def torch_gather(group: Any = None) -> Callable[[Any], list[Any]]:
    """A ``gather`` callable over ``torch.distributed`` (``all_gather_object``)."""
    import torch.distributed as dist

    def gather(obj: Any) -> list[Any]:
        if not (dist.is_available() and dist.is_initialized()):
            return [obj]
        out: list[Any] = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, obj, group=group)
        return out

    return gather


def _merge_remote(bundle: MetricBundle, gather: Callable[[Any], list[Any]] | None, data_rank: int) -> None:
    """Fold every other rank's running state into this rank's metrics (exact: states are sums)."""
    if gather is None:
        return
    for index, remote in enumerate(gather({name: m.state() for name, m in bundle.metrics.items()}) or ()):
        if index == data_rank or not isinstance(remote, dict):
            continue
        for name in remote.keys() & bundle.metrics.keys():
            bundle.metrics[name].merge(remote[name])


def _feed(bundle: MetricBundle, batches: Iterable[EvalBatch]) -> tuple[int, set[str]]:
    """Update every metric with every batch that carries its inputs; returns
    (samples seen, metrics that received at least one batch)."""
    samples, fed = 0, set()
    for batch in batches:
        inputs = batch.as_inputs()
        samples += int(batch.video.shape[0])
        for name, metric in bundle.metrics.items():
            lacking = [k for k in metric.required_inputs if k not in inputs]
            if lacking:
                bundle.skipped.setdefault(name, f"needs {', '.join(lacking)}, which this evaluation did not produce")
            else:
                metric.update(**inputs)
                fed.add(name)
    return samples, fed


def run_eval_suite(batches: Iterable[EvalBatch], *, metrics: Sequence[str] | MetricBundle, pin: EvalPin,
                   prompts: Sequence[str] = (), decoded: bool = False,
                   metric_options: Mapping[str, Mapping[str, Any]] | None = None,
                   gather: Callable[[Any], list[Any]] | None = None, data_rank: int = 0, run_name: str = "",
                   step: int = 0, notes: str = "") -> EvalReport:
    """Feed every batch to every metric that has its inputs, merge the ranks' running
    sums exactly, and return the pinned report (sample count summed over ranks)."""
    import dataclasses

    bundle = metrics if isinstance(metrics, MetricBundle) else build_metrics(metrics, decoded=decoded,
                                                                              options=metric_options)
    samples, fed = _feed(bundle, batches)
    for name in set(bundle.metrics) - fed:
        del bundle.metrics[name]
        bundle.skipped.setdefault(name, "no batch supplied its required inputs")
    _merge_remote(bundle, gather, data_rank)
    values: dict[str, float] = {}
    for name, metric in bundle.metrics.items():
        stats = metric.compute()
        if stats:
            values.update(stats)
        else:
            bundle.skipped.setdefault(name, "produced no statistics (every clip was too short for it)")
    total = sum(int(c) for c in gather(samples)) if gather is not None else samples
    resolved = dataclasses.replace(pin, num_samples=total, decoded=decoded, metrics=dict(bundle.parameters),
                                   prompt_digest=prompt_set_digest(prompts) if prompts else pin.prompt_digest)
    return EvalReport(pin=resolved, metrics=values, skipped=dict(bundle.skipped), run_name=run_name, step=step,
                      notes=notes)
