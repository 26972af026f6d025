"""Timestep (noise-level) samplers with a registry (avgen/train/timestep.py:90-517).

``uniform``, ``logit_normal``, ``shifted_logit_normal`` (shift linear in the
sequence length between (base_seq_len, base_shift) and (max_seq_len, max_shift),
applied as t' = s t / (1 + (s - 1) t)) and ``mode`` (SD3 mode sampling).
"""
from __future__ import annotations

import math
from collections.abc import Callable, Mapping
from dataclasses import dataclass
from typing import Any, Protocol, TypeVar, runtime_checkable

import torch

from avgen_b200.core._validate import require_finite, require_positive
from avgen_b200.train._random import normal, uniform

__all__ = ["LogitNormalSampler", "ModeSampler", "ShiftedLogitNormalSampler", "TimestepSampler", "UniformSampler",
           "build_timestep_sampler", "list_timestep_samplers", "register_timestep_sampler", "resolution_shift",
           "shift_timesteps"]


@runtime_checkable
class TimestepSampler(Protocol):
    def sample(self, batch: int, *, device: torch.device | str, generator: torch.Generator,
               sequence_length: int | None = None) -> torch.Tensor: ...


_SAMPLERS: dict[str, Callable[..., TimestepSampler]] = {}
_T = TypeVar("_T", bound=Callable[..., TimestepSampler])


def register_timestep_sampler(name: str) -> Callable[[_T], _T]:
    def decorate(factory: _T) -> _T:
        if name in _SAMPLERS:
            raise ValueError(f"timestep sampler {name!r} is already registered")
        _SAMPLERS[name] = factory
        return factory

    return decorate


def build_timestep_sampler(name: str, config: Mapping[str, Any] | None = None) -> TimestepSampler:
    if name not in _SAMPLERS:
        raise KeyError(f"unknown timestep sampler {name!r}; available: {', '.join(list_timestep_samplers())}")
    return _SAMPLERS[name](**dict(config or {}))


def list_timestep_samplers() -> tuple[str, ...]:
    return tuple(sorted(_SAMPLERS))


def resolution_shift(sequence_length: int | None, *, base_seq_len: int, base_shift: float, max_seq_len: int,
                     max_shift: float) -> float:
    """Shift interpolated linearly in sequence length and clamped to its end points."""
    if sequence_length is None:
        return base_shift
    slope = (max_shift - base_shift) / (max_seq_len - base_seq_len)
    value = base_shift + slope * (sequence_length - base_seq_len)
    return min(max(value, min(base_shift, max_shift)), max(base_shift, max_shift))


def shift_timesteps(timesteps: torch.Tensor, shift: float) -> torch.Tensor:
    if not shift > 0.0:
        raise ValueError(f"shift must be positive; got {shift!r}")
    return shift * timesteps / (1.0 + (shift - 1.0) * timesteps)


@register_timestep_sampler("uniform")
@dataclass(frozen=True, slots=True)
class UniformSampler:
    low: float = 0.0
    high: float = 1.0

    def __post_init__(self) -> None:
        require_finite("low", self.low)
        require_finite("high", self.high)
        if not 0.0 <= self.low < self.high <= 1.0:
            raise ValueError("require 0 <= low < high <= 1")

    def sample(self, batch, *, device, generator, sequence_length=None):  # noqa: ANN001, ANN201
        return self.low + (self.high - self.low) * uniform((batch,), generator=generator, device=device)


@register_timestep_sampler("logit_normal")
@dataclass(frozen=True, slots=True)
class LogitNormalSampler:
    mean: float = 0.0
    std: float = 1.0

    def __post_init__(self) -> None:
        require_finite("mean", self.mean)
        require_finite("std", self.std)
        if self.std <= 0.0:
            raise ValueError("std must be positive")

    def sample(self, batch, *, device, generator, sequence_length=None):  # noqa: ANN001, ANN201
        return torch.sigmoid(self.mean + self.std * normal((batch,), generator=generator, device=device))


@register_timestep_sampler("shifted_logit_normal")
@dataclass(frozen=True, slots=True)
class ShiftedLogitNormalSampler:
    mean: float = 0.0
    std: float = 1.0
    base_seq_len: int = 1024
    base_shift: float = 0.95
    max_seq_len: int = 32768
    max_shift: float = 2.05

    def __post_init__(self) -> None:
        require_finite("mean", self.mean)
        require_finite("std", self.std)
        if self.std <= 0.0:
            raise ValueError("std must be positive")
        require_positive("base_seq_len", self.base_seq_len)
        require_positive("max_seq_len", self.max_seq_len)
        if self.base_seq_len >= self.max_seq_len:
            raise ValueError("base_seq_len must be below max_seq_len")
        for name in ("base_shift", "max_shift"):
            if float(getattr(self, name)) <= 0.0:
                raise ValueError(f"{name} must be positive")

    def shift_for(self, sequence_length: int | None) -> float:
        return resolution_shift(sequence_length, base_seq_len=self.base_seq_len, base_shift=self.base_shift,
                                max_seq_len=self.max_seq_len, max_shift=self.max_shift)

    def sample(self, batch, *, device, generator, sequence_length=None):  # noqa: ANN001, ANN201
        t = torch.sigmoid(self.mean + self.std * normal((batch,), generator=generator, device=device))
        return shift_timesteps(t, self.shift_for(sequence_length))


@register_timestep_sampler("mode")
@dataclass(frozen=True, slots=True)
class ModeSampler:
    scale: float = 1.29

    def __post_init__(self) -> None:
        require_finite("scale", self.scale)
        if not -1.0 <= self.scale <= 2.0 * math.pi / (math.pi - 2.0):
            raise ValueError("scale outside the monotone range")

    def sample(self, batch, *, device, generator, sequence_length=None):  # noqa: ANN001, ANN201
        u = uniform((batch,), generator=generator, device=device)
        c = torch.cos(0.5 * math.pi * u)
        return (1.0 - u - self.scale * (c.pow(2) - 1.0 + u)).clamp(0.0, 1.0)
