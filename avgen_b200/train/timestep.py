"""Noise-level (timestep) distributions for flow-matching training.

Every sampler here is one composition: a base variate in [0, 1] (uniform, or the
sigmoid of a normal draw) followed by an optional monotone warp of [0, 1] onto
itself (the sequence-length shift ``t' = s t / (1 + (s - 1) t)``, or the SD3 mode
warp ``t' = 1 - u - c (cos^2(pi u / 2) - 1 + u)``). A sampler states its base, its
warp and the limits of its fields; ``sample`` and validation are shared.

Registry names, class names and field names with their defaults are the
configuration interface of the reference (avgen/train/timestep.py:90-517): a
YAML ``train.timestep_sampler`` / ``timestep_sampler_kwargs`` pair selects the
same distribution in both frameworks.
"""
from __future__ import annotations

import math
from collections.abc import Callable, Mapping
from dataclasses import dataclass, fields
from typing import Any, ClassVar, Protocol, TypeVar, runtime_checkable

import torch

from avgen_b200.train._random import normal, uniform

__all__ = ["LogitNormalSampler", "ModeSampler", "ShiftedLogitNormalSampler", "TimestepSampler", "UniformSampler",
           "build_timestep_sampler", "list_timestep_samplers", "register_timestep_sampler", "resolution_shift",
           "shift_timesteps"]


@runtime_checkable
class TimestepSampler(Protocol):
    def sample(self, batch: int, *, device: torch.device | str, generator: torch.Generator,
               sequence_length: int | None = None) -> torch.Tensor: ...


_Factory = TypeVar("_Factory", bound=Callable[..., TimestepSampler])
_REGISTRY: dict[str, Callable[..., TimestepSampler]] = {}


def register_timestep_sampler(name: str) -> Callable[[_Factory], _Factory]:
    """Decorator adding a sampler factory under ``name`` (names are unique)."""

    def add(factory: _Factory) -> _Factory:
        if name in _REGISTRY:
            raise ValueError(f"timestep sampler {name!r} is already registered")
        _REGISTRY[name] = factory
        return factory

    return add


def list_timestep_samplers() -> tuple[str, ...]:
    return tuple(sorted(_REGISTRY))


def build_timestep_sampler(name: str, config: Mapping[str, Any] | None = None) -> TimestepSampler:
    factory = _REGISTRY.get(name)
    if factory is None:
        raise KeyError(f"unknown timestep sampler {name!r}; available: {', '.join(list_timestep_samplers())}")
    return factory(**dict(config or {}))


def resolution_shift(sequence_length: int | None, *, base_seq_len: int, base_shift: float, max_seq_len: int,
                     max_shift: float) -> float:
    """The shift at ``sequence_length`` on the line through (base_seq_len, base_shift)
    and (max_seq_len, max_shift), held at the nearer end point outside that span;
    ``base_shift`` when the length is unknown."""
    if sequence_length is None:
        return base_shift
    frac = (sequence_length - base_seq_len) / (max_seq_len - base_seq_len)
    lo, hi = sorted((base_shift, max_shift))
    return min(hi, max(lo, base_shift + frac * (max_shift - base_shift)))


def shift_timesteps(timesteps: torch.Tensor, shift: float) -> torch.Tensor:
    """Monotone map of [0, 1] onto itself; ``shift > 1`` moves mass toward 1 (more noise)."""
    if not shift > 0.0:
        raise ValueError(f"shift must be positive; got {shift!r}")
    return timesteps * shift / (1.0 + timesteps * (shift - 1.0))


# ----------------------------------------------------------------------------- the shared composition

_Rule = tuple[str, Callable[[Any], bool], str]


def _finite(v: Any) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(v)


class _NoiseLevels:
    """``sample`` = ``_warp(_base(...))``; ``_rules`` lists (field, predicate, message)."""

    __slots__ = ()
    _rules: ClassVar[tuple[_Rule, ...]] = ()

    def __post_init__(self) -> None:
        for name in (f.name for f in fields(self)):  # type: ignore[arg-type]
            if not _finite(getattr(self, name)):
                raise ValueError(f"{name} must be a finite number; got {getattr(self, name)!r}")
        for name, ok, message in self._rules:
            if not ok(self):
                raise ValueError(f"{name}: {message}")

    def _base(self, batch: int, device: torch.device | str, generator: torch.Generator) -> torch.Tensor:
        raise NotImplementedError

    def _warp(self, t: torch.Tensor, sequence_length: int | None) -> torch.Tensor:
        return t

    def sample(self, batch: int, *, device: torch.device | str, generator: torch.Generator,
               sequence_length: int | None = None) -> torch.Tensor:
        return self._warp(self._base(batch, device, generator), sequence_length)


def _sigmoid_normal(mean: float, std: float, batch: int, device: torch.device | str,
                    generator: torch.Generator) -> torch.Tensor:
    return torch.sigmoid(normal((batch,), generator=generator, device=device).mul(std).add(mean))


# ----------------------------------------------------------------------------- the registered samplers


@register_timestep_sampler("uniform")
@dataclass(frozen=True, slots=True)
class UniformSampler(_NoiseLevels):
    low: float = 0.0
    high: float = 1.0

    _rules = (("low/high", lambda s: 0.0 <= s.low < s.high <= 1.0, "require 0 <= low < high <= 1"),)

    def _base(self, batch, device, generator):  # noqa: ANN001, ANN202
        return uniform((batch,), generator=generator, device=device).mul(self.high - self.low).add(self.low)


@register_timestep_sampler("logit_normal")
@dataclass(frozen=True, slots=True)
class LogitNormalSampler(_NoiseLevels):
    mean: float = 0.0
    std: float = 1.0

    _rules = (("std", lambda s: s.std > 0.0, "must be positive"),)

    def _base(self, batch, device, generator):  # noqa: ANN001, ANN202
        return _sigmoid_normal(self.mean, self.std, batch, device, generator)


@register_timestep_sampler("shifted_logit_normal")
@dataclass(frozen=True, slots=True)
class ShiftedLogitNormalSampler(_NoiseLevels):
    """Logit-normal levels warped by the shift for the sample's token count."""

    mean: float = 0.0
    std: float = 1.0
    base_seq_len: int = 1024
    base_shift: float = 0.95
    max_seq_len: int = 32768
    max_shift: float = 2.05

    _rules = (("std", lambda s: s.std > 0.0, "must be positive"),
              ("base_seq_len", lambda s: s.base_seq_len > 0, "must be positive"),
              ("max_seq_len", lambda s: s.max_seq_len > s.base_seq_len, "must exceed base_seq_len"),
              ("base_shift", lambda s: s.base_shift > 0.0, "must be positive"),
              ("max_shift", lambda s: s.max_shift > 0.0, "must be positive"))

    def shift_for(self, sequence_length: int | None) -> float:
        return resolution_shift(sequence_length, base_seq_len=self.base_seq_len, base_shift=self.base_shift,
                                max_seq_len=self.max_seq_len, max_shift=self.max_shift)

    def _base(self, batch, device, generator):  # noqa: ANN001, ANN202
        return _sigmoid_normal(self.mean, self.std, batch, device, generator)

    def _warp(self, t, sequence_length):  # noqa: ANN001, ANN202
        return shift_timesteps(t, self.shift_for(sequence_length))


# The mode warp stays monotone on [0, 1] for scales in [-1, 2 pi / (pi - 2)].
_MODE_SCALE_MAX = 2.0 * math.pi / (math.pi - 2.0)


@register_timestep_sampler("mode")
@dataclass(frozen=True, slots=True)
class ModeSampler(_NoiseLevels):
    """SD3 mode sampling: uniform levels bent toward (scale > 0) or away from the middle."""

    scale: float = 1.29

    _rules = (("scale", lambda s: -1.0 <= s.scale <= _MODE_SCALE_MAX, "outside the monotone range"),)

    def _base(self, batch, device, generator):  # noqa: ANN001, ANN202
        return uniform((batch,), generator=generator, device=device)

    def _warp(self, u, sequence_length):  # noqa: ANN001, ANN202
        bend = torch.cos(u * (0.5 * math.pi)).square() - 1.0 + u
        return (1.0 - u - self.scale * bend).clamp(0.0, 1.0)
