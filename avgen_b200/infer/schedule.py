"""Sigma schedules for flow-matching sampling (avgen/infer/schedule.py:63-694 API).

A schedule is a strictly decreasing tensor of flow times from ``sigma_max`` (at
most 1) to exactly 0. Builders: ``linear``, ``karras`` (rho-spaced), and
``linear_quadratic`` (linear near 0 up to a threshold, quadratic above). A shift
``s`` warps every sigma through ``s t / (1 + (s - 1) t)``; with
``dynamic_shift`` the shift grows linearly with the token count between
``(base_length, base_shift)`` and ``(max_length, max_shift)`` (optionally
exponentiated), so long clips spend more steps at high noise.
"""
from __future__ import annotations

import math
from collections.abc import Callable, Iterator, Mapping
from dataclasses import asdict, dataclass, replace
from typing import Any

import torch

__all__ = ["ScheduleConfig", "SigmaSchedule", "apply_shift", "build_sigma_schedule", "karras_sigmas",
           "linear_quadratic_sigmas", "linear_sigmas", "list_sigma_schedules", "register_sigma_schedule",
           "resolution_shift"]


def apply_shift(sigmas: torch.Tensor, shift: float) -> torch.Tensor:
    if not (math.isfinite(shift) and shift > 0.0):
        raise ValueError(f"shift must be finite and positive; got {shift!r}")
    if shift == 1.0:
        return sigmas
    return (shift * sigmas / (1.0 + (shift - 1.0) * sigmas)).clamp(0.0, 1.0)


def resolution_shift(sequence_length: int, *, base_length: int = 256, base_shift: float = 1.0, max_length: int = 4096,
                     max_shift: float = 3.0, exponential: bool = False) -> float:
    for name, n in (("sequence_length", sequence_length), ("base_length", base_length), ("max_length", max_length)):
        if isinstance(n, bool) or n < 1:
            raise ValueError(f"{name} must be a positive integer; got {n!r}")
    if base_length == max_length:
        raise ValueError("base_length and max_length must differ")
    t = (sequence_length - base_length) / (max_length - base_length)
    value = base_shift + t * (max_shift - base_shift)
    value = min(max(value, min(base_shift, max_shift)), max(base_shift, max_shift))
    return math.exp(value) if exponential else value


@dataclass(frozen=True, slots=True)
class SigmaSchedule:
    sigmas: torch.Tensor
    shift: float = 1.0
    name: str = "linear"

    def __post_init__(self) -> None:
        s = self.sigmas
        if s.ndim != 1 or s.numel() < 2:
            raise ValueError(f"sigmas must be rank 1 with at least two entries; got {tuple(s.shape)}")
        if not s.is_floating_point() or not bool(torch.isfinite(s).all()):
            raise ValueError("sigmas must be finite floating point values")
        if not bool((s[1:] < s[:-1]).all()):
            raise ValueError(f"sigmas must strictly decrease; got {s.tolist()}")
        if float(s[0]) > 1.0 or float(s[-1]) != 0.0:
            raise ValueError(f"sigmas must start at or below 1 and end at exactly 0; got {float(s[0])} ... "
                             f"{float(s[-1])}")

    @property
    def num_steps(self) -> int:
        return int(self.sigmas.numel()) - 1

    @property
    def device(self) -> torch.device:
        return self.sigmas.device

    def __len__(self) -> int:
        return self.num_steps

    def __iter__(self) -> Iterator[tuple[int, float, float]]:
        vals = self.sigmas.tolist()
        for i in range(self.num_steps):
            yield i, float(vals[i]), float(vals[i + 1])

    def to(self, device: torch.device | str) -> SigmaSchedule:
        return replace(self, sigmas=self.sigmas.to(device))

    def timesteps(self) -> torch.Tensor:
        return self.sigmas[:-1]

    def tolist(self) -> list[float]:
        return [float(v) for v in self.sigmas.tolist()]


_BUILDERS: dict[str, Callable[..., torch.Tensor]] = {}


def register_sigma_schedule(name: str) -> Callable[[Callable[..., torch.Tensor]], Callable[..., torch.Tensor]]:
    if not name or name.strip() != name:
        raise ValueError(f"name must be a non-empty trimmed string; got {name!r}")
    if name in _BUILDERS:
        raise ValueError(f"sigma schedule {name!r} is already registered")

    def deco(fn: Callable[..., torch.Tensor]) -> Callable[..., torch.Tensor]:
        _BUILDERS[name] = fn
        return fn

    return deco


def list_sigma_schedules() -> tuple[str, ...]:
    return tuple(sorted(_BUILDERS))


def _steps_ok(steps: int) -> None:
    if isinstance(steps, bool) or steps < 1:
        raise ValueError(f"steps must be a positive integer; got {steps!r}")


def _range_ok(lo: float, hi: float) -> None:
    if not (math.isfinite(hi) and 0.0 < hi <= 1.0):
        raise ValueError(f"sigma_max must be in (0, 1] for a flow schedule; got {hi!r}")
    if not (math.isfinite(lo) and 0.0 < lo < hi):
        raise ValueError(f"sigma_min must be in (0, sigma_max={hi}); got {lo!r} (the final 0 is appended)")


def _with_zero(body: torch.Tensor) -> torch.Tensor:
    return torch.cat((body, torch.zeros(1, dtype=body.dtype, device=body.device)))


@register_sigma_schedule("linear")
def linear_sigmas(steps: int, *, sigma_max: float = 1.0, sigma_min: float | None = None,
                  device: torch.device | str = "cpu", **_: Any) -> torch.Tensor:
    _steps_ok(steps)
    if sigma_min is None and steps == 1:
        _range_ok(sigma_max / 2, sigma_max)
        return _with_zero(torch.tensor([sigma_max], dtype=torch.float32, device=device))
    lo = sigma_max / steps if sigma_min is None else sigma_min
    _range_ok(lo, sigma_max)
    return _with_zero(torch.linspace(sigma_max, lo, steps, dtype=torch.float32, device=device))


@register_sigma_schedule("karras")
def karras_sigmas(steps: int, *, sigma_max: float = 1.0, sigma_min: float | None = None, rho: float = 7.0,
                  device: torch.device | str = "cpu", **_: Any) -> torch.Tensor:
    _steps_ok(steps)
    lo = 0.002 if sigma_min is None else sigma_min
    _range_ok(lo, sigma_max)
    if not (math.isfinite(rho) and rho > 0.0):
        raise ValueError(f"rho must be finite and positive; got {rho!r}")
    u = torch.linspace(0.0, 1.0, steps, dtype=torch.float64, device=device)
    a, b = sigma_max ** (1.0 / rho), lo ** (1.0 / rho)
    return _with_zero(((a + u * (b - a)) ** rho).float())


@register_sigma_schedule("linear_quadratic")
def linear_quadratic_sigmas(steps: int, *, sigma_max: float = 1.0, linear_steps: int | None = None,
                            threshold_noise: float = 0.025, device: torch.device | str = "cpu",
                            **_: Any) -> torch.Tensor:
    _steps_ok(steps)
    _range_ok(sigma_max / (steps + 1), sigma_max)
    if steps == 1 and linear_steps is None:
        return _with_zero(torch.tensor([sigma_max], dtype=torch.float32, device=device))
    n_lin = max(steps // 2, 1) if linear_steps is None else linear_steps
    if isinstance(n_lin, bool) or not 0 < n_lin < steps:
        raise ValueError(f"linear_steps must be in (0, {steps}); got {n_lin!r}")
    if not 0.0 < threshold_noise < sigma_max:
        raise ValueError(f"threshold_noise must be in (0, {sigma_max}); got {threshold_noise!r}")
    n_quad = steps - n_lin
    rising = [threshold_noise * i / n_lin for i in range(n_lin)]
    rising += [threshold_noise + (sigma_max - threshold_noise) * (j / n_quad) ** 2 for j in range(n_quad + 1)]
    out = torch.tensor(rising[::-1], dtype=torch.float32, device=device)
    out[-1] = 0.0
    return out


@dataclass(frozen=True, slots=True)
class ScheduleConfig:
    name: str = "linear"
    steps: int = 30
    shift: float = 1.0
    dynamic_shift: bool = False
    base_length: int = 256
    base_shift: float = 1.0
    max_length: int = 4096
    max_shift: float = 3.0
    exponential_shift: bool = False
    sigma_max: float = 1.0
    sigma_min: float | None = None
    rho: float = 7.0
    linear_steps: int | None = None
    threshold_noise: float = 0.025

    def __post_init__(self) -> None:
        if not self.name or self.name.strip() != self.name:
            raise ValueError(f"name must be a non-empty trimmed string; got {self.name!r}")
        _steps_ok(self.steps)
        if not (math.isfinite(self.shift) and self.shift > 0.0):
            raise ValueError(f"shift must be finite and positive; got {self.shift!r}")

    def resolve_shift(self, sequence_length: int | None) -> float:
        if not self.dynamic_shift:
            return self.shift
        if sequence_length is None:
            raise ValueError("dynamic_shift needs the global token count of the sample (sequence_length=)")
        return resolution_shift(sequence_length, base_length=self.base_length, base_shift=self.base_shift,
                                max_length=self.max_length, max_shift=self.max_shift,
                                exponential=self.exponential_shift)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: Mapping[str, Any]) -> ScheduleConfig:
        names = set(cls.__dataclass_fields__)  # type: ignore[attr-defined]
        return cls(**{k: v for k, v in values.items() if k in names})


def build_sigma_schedule(config: ScheduleConfig, *, sequence_length: int | None = None,
                         device: torch.device | str = "cpu") -> SigmaSchedule:
    builder = _BUILDERS.get(config.name)
    if builder is None:
        raise KeyError(f"unknown sigma schedule {config.name!r}; registered: {', '.join(list_sigma_schedules())}")
    sig = builder(config.steps, sigma_max=config.sigma_max, sigma_min=config.sigma_min, rho=config.rho,
                  linear_steps=config.linear_steps, threshold_noise=config.threshold_noise, device=device)
    shift = config.resolve_shift(sequence_length)
    if shift != 1.0:
        sig = apply_shift(sig, shift).clone()
        sig[-1] = 0.0
    return SigmaSchedule(sigmas=sig, shift=shift, name=config.name)
