"""Field-named argument validation used across the contracts.

Mirrors the role of avgen/core/_validate.py:31-197: every check raises with the
offending field's name so a failure points at the caller's mistake.
"""
from __future__ import annotations

import math
from collections.abc import Iterable

import torch


def require_positive(name: str, value: int) -> None:
    if isinstance(value, bool) or not isinstance(value, int) or value < 1:
        raise ValueError(f"{name} must be a positive integer; got {value!r}")


def require_dimension(name: str, value: int, *, allow_zero: bool = False) -> None:
    low = 0 if allow_zero else 1
    if isinstance(value, bool) or not isinstance(value, int) or value < low:
        kind = "non-negative" if allow_zero else "positive"
        raise ValueError(f"{name} must be a {kind} integer; got {value!r}")


def require_finite(name: str, value: float) -> None:
    if not math.isfinite(float(value)):
        raise ValueError(f"{name} must be finite; got {value!r}")


def require_probability(name: str, value: float) -> None:
    require_finite(name, value)
    if not 0.0 <= float(value) <= 1.0:
        raise ValueError(f"{name} must lie in [0, 1]; got {value!r}")


def require_name(name: str, value: str) -> None:
    if not isinstance(value, str) or not value.strip():
        raise ValueError(f"{name} must be a non-empty string; got {value!r}")


def require_unique_names(name: str, values: Iterable[str]) -> None:
    seen: set[str] = set()
    for value in values:
        require_name(name, value)
        if value in seen:
            raise ValueError(f"{name} contains duplicate entry {value!r}")
        seen.add(value)


def require_shape(name: str, tensor: torch.Tensor, shape: tuple[int, ...]) -> None:
    if tuple(tensor.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}; got {tuple(tensor.shape)}")


def require_dtype(name: str, tensor: torch.Tensor, dtype: torch.dtype) -> None:
    if tensor.dtype is not dtype:
        raise TypeError(f"{name} must have dtype {dtype}; got {tensor.dtype}")


def require_floating(name: str, tensor: torch.Tensor) -> None:
    if not tensor.is_floating_point():
        raise TypeError(f"{name} must be floating point; got {tensor.dtype}")


def require_same_device(
    name: str, tensor: torch.Tensor, others: Iterable[tuple[str, torch.Tensor]]
) -> None:
    for other_name, other in others:
        if other.device != tensor.device:
            raise ValueError(f"{other_name} must be on {name} device {tensor.device}; got {other.device}")
