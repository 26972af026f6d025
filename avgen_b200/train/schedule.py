"""Learning-rate schedules through ``LambdaLR`` (avgen/train/schedule.py:93-326).

``constant``, ``linear``, ``cosine`` and ``wsd`` (warmup-stable-decay with a
1-sqrt, linear or cosine decay tail); all with linear warmup and an optional
``min_lr_ratio`` floor.
"""
from __future__ import annotations

import math
from collections.abc import Callable, Mapping
from typing import Any

from torch.optim import Optimizer
from torch.optim.lr_scheduler import LambdaLR

__all__ = ["build_schedule", "list_schedules", "register_schedule"]

Factory = Callable[[int, int, Mapping[str, Any]], Callable[[int], float]]
_SCHEDULES: dict[str, Factory] = {}


def register_schedule(name: str) -> Callable[[Factory], Factory]:
    def decorate(factory: Factory) -> Factory:
        if name in _SCHEDULES:
            raise ValueError(f"schedule {name!r} is already registered")
        _SCHEDULES[name] = factory
        return factory

    return decorate


def list_schedules() -> tuple[str, ...]:
    return tuple(sorted(_SCHEDULES))


def build_schedule(name: str, optimizer: Optimizer, *, total_steps: int, warmup_steps: int = 0,
                   **options: Any) -> LambdaLR:
    if name not in _SCHEDULES:
        raise KeyError(f"unknown schedule {name!r}; available: {', '.join(list_schedules())}")
    if isinstance(total_steps, bool) or total_steps < 1:
        raise ValueError(f"total_steps must be positive; got {total_steps!r}")
    if isinstance(warmup_steps, bool) or warmup_steps < 0:
        raise ValueError("warmup_steps must be non-negative")
    if warmup_steps >= total_steps:
        raise ValueError(f"warmup_steps={warmup_steps} must be below total_steps={total_steps}")
    return LambdaLR(optimizer, lr_lambda=_SCHEDULES[name](total_steps, warmup_steps, options))


def _warm(step: int, warmup: int) -> float:
    return float(step + 1) / float(max(warmup, 1))


def _floor(options: Mapping[str, Any]) -> float:
    ratio = float(options.get("min_lr_ratio", 0.0))
    if not 0.0 <= ratio <= 1.0:
        raise ValueError("min_lr_ratio must be in [0, 1]")
    return ratio


@register_schedule("constant")
def _constant(total: int, warmup: int, options: Mapping[str, Any]) -> Callable[[int], float]:
    return lambda step: _warm(step, warmup) if step < warmup else 1.0


@register_schedule("linear")
def _linear(total: int, warmup: int, options: Mapping[str, Any]) -> Callable[[int], float]:
    floor = _floor(options)
    span = max(total - warmup, 1)

    def f(step: int) -> float:
        if step < warmup:
            return _warm(step, warmup)
        return floor + (1.0 - floor) * (1.0 - min((step - warmup) / span, 1.0))

    return f


@register_schedule("cosine")
def _cosine(total: int, warmup: int, options: Mapping[str, Any]) -> Callable[[int], float]:
    floor = _floor(options)
    span = max(total - warmup, 1)

    def f(step: int) -> float:
        if step < warmup:
            return _warm(step, warmup)
        progress = min((step - warmup) / span, 1.0)
        return floor + (1.0 - floor) * 0.5 * (1.0 + math.cos(math.pi * progress))

    return f


@register_schedule("wsd")
def _wsd(total: int, warmup: int, options: Mapping[str, Any]) -> Callable[[int], float]:
    floor = _floor(options)
    fraction = float(options.get("decay_fraction", 0.1))
    if not 0.0 < fraction <= 1.0:
        raise ValueError("decay_fraction must be in (0, 1]")
    shape = str(options.get("decay_shape", "1-sqrt"))
    if shape not in {"1-sqrt", "linear", "cosine"}:
        raise ValueError("decay_shape must be one of 1-sqrt, linear, cosine")
    decay_steps = max(round(total * fraction), 1)
    start = max(total - decay_steps, warmup)
    span = max(total - start, 1)

    def f(step: int) -> float:
        if step < warmup:
            return _warm(step, warmup)
        if step < start:
            return 1.0
        p = min((step - start) / span, 1.0)
        rem = 1.0 - p if shape == "linear" else (0.5 * (1.0 + math.cos(math.pi * p)) if shape == "cosine"
                                                 else 1.0 - math.sqrt(p))
        return floor + (1.0 - floor) * rem

    return f
