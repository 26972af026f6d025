"""Metric protocol, registry and the running-sum base class (avgen/eval/protocols.py:59-397 API).

A :class:`RunningMetric` turns each batch into named ``(sum, count)``
contributions; it keeps float64 sums on its device, so a distributed
evaluation merges ranks exactly by adding ``state()`` dictionaries and the
result does not depend on how prompts were sharded. Registered names are
unique: two runs never report different quantities under one label.
Third-party metrics register through the ``avgen.metrics`` entry-point group.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from collections.abc import Callable, Mapping
from typing import Any, Protocol, runtime_checkable

import torch

__all__ = ["METRIC_ENTRY_POINT_GROUP", "Metric", "MetricError", "RunningMetric", "build_metric", "describe_metrics",
           "list_metrics", "metric_class", "register_metric", "require_audio", "require_video"]

METRIC_ENTRY_POINT_GROUP = "avgen.metrics"


class MetricError(ValueError):
    """A metric was asked for something it cannot compute (bad name, shape or inputs)."""


@runtime_checkable
class Metric(Protocol):
    name: str

    def update(self, **inputs: Any) -> None: ...

    def compute(self) -> dict[str, float]: ...

    def reset(self) -> None: ...


_REGISTRY: dict[str, type[RunningMetric]] = {}


def register_metric(name: str) -> Callable[[type[RunningMetric]], type[RunningMetric]]:
    def deco(cls: type[RunningMetric]) -> type[RunningMetric]:
        if name in _REGISTRY:
            raise ValueError(f"metric {name!r} is already registered to {_REGISTRY[name].__name__}; choose another "
                             "name (one label must always mean one computation)")
        cls.name = name
        _REGISTRY[name] = cls
        return cls

    return deco


def _load_plugins() -> None:
    from avgen_b200._plugins import load_entry_points

    def accept(name: str, obj: object) -> None:
        if not isinstance(obj, type):
            raise TypeError(f"entry point {name!r} of {METRIC_ENTRY_POINT_GROUP!r} must be a RunningMetric class")
        if name not in _REGISTRY:
            register_metric(name)(obj)  # type: ignore[arg-type]

    load_entry_points(METRIC_ENTRY_POINT_GROUP, accept)


def list_metrics() -> tuple[str, ...]:
    _load_plugins()
    return tuple(sorted(_REGISTRY))


def metric_class(name: str) -> type[RunningMetric]:
    _load_plugins()
    if name not in _REGISTRY:
        raise MetricError(f"unknown metric {name!r}; available: {', '.join(sorted(_REGISTRY))}. Learned metrics "
                          "(fvd, fid, clip_score, ...) are declared in avgen_b200.eval.learned")
    return _REGISTRY[name]


def build_metric(name: str, **kwargs: Any) -> RunningMetric:
    cls = metric_class(name)
    try:
        return cls(**kwargs)
    except TypeError as err:
        raise MetricError(f"cannot build metric {name!r} with {kwargs!r}: {err}") from err


def describe_metrics() -> dict[str, str]:
    out: dict[str, str] = {}
    for name, cls in sorted(_REGISTRY.items()):
        doc = (cls.__doc__ or "").strip().splitlines()
        out[name] = doc[0] if doc else ""
    return out


class RunningMetric(ABC):
    """Base for metrics that average named per-batch contributions."""

    name: str = "unnamed"
    required_inputs: tuple[str, ...] = ("video",)
    pixel_space_only: bool = False

    def __init__(self, *, device: torch.device | str = "cpu") -> None:
        self._device = torch.device(device)
        self._sums: dict[str, torch.Tensor] = {}
        self._counts: dict[str, float] = {}

    @abstractmethod
    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        """``{statistic: (sum over items, item count)}`` for one batch."""

    def update(self, **inputs: Any) -> None:
        missing = [k for k in self.required_inputs if inputs.get(k) is None]
        if missing:
            raise MetricError(f"metric {self.name!r} requires {', '.join(missing)} but was given "
                              f"{', '.join(sorted(inputs)) or '<nothing>'}")
        for key, (value, count) in self.observe(**inputs).items():
            if count <= 0:
                continue
            v = value.detach().to(self._device, torch.float64)
            self._sums[key] = self._sums[key] + v if key in self._sums else v
            self._counts[key] = self._counts.get(key, 0.0) + float(count)

    def compute(self) -> dict[str, float]:
        return {f"{self.name}/{k}": float(s) / self._counts[k] for k, s in self._sums.items() if self._counts[k] > 0}

    def reset(self) -> None:
        self._sums.clear()
        self._counts.clear()

    def state(self) -> dict[str, tuple[float, float]]:
        return {k: (float(s), self._counts[k]) for k, s in self._sums.items()}

    def merge(self, other: Mapping[str, tuple[float, float]]) -> None:
        for key, (total, count) in other.items():
            v = torch.tensor(float(total), dtype=torch.float64, device=self._device)
            self._sums[key] = self._sums[key] + v if key in self._sums else v
            self._counts[key] = self._counts.get(key, 0.0) + float(count)


def _require(tensor: Any, ndim: int, *, metric: str, argument: str, layout: str) -> torch.Tensor:
    if not isinstance(tensor, torch.Tensor):
        raise MetricError(f"{metric}: {argument} must be a tensor; got {type(tensor).__name__}")
    if tensor.ndim != ndim:
        raise MetricError(f"{metric}: {argument} must be {layout}; got shape {tuple(tensor.shape)}")
    return tensor.detach().float()


def require_video(tensor: Any, *, metric: str, argument: str = "video") -> torch.Tensor:
    return _require(tensor, 5, metric=metric, argument=argument, layout="(batch, channels, frames, height, width)")


def require_audio(tensor: Any, *, metric: str, argument: str = "audio") -> torch.Tensor:
    return _require(tensor, 3, metric=metric, argument=argument, layout="(batch, channels, frames)")
