"""Declarative numeric limits for configuration dataclasses.

A config class states, once, the range each numeric field may take
(``Limit(lo=0, lo_open=True)`` is "positive", ``Limit(lo=1, integer=True)`` "a
positive integer"), and :func:`enforce` checks an instance against that table,
raising ``ValueError`` that names the field, the rule and the offending value.
"""
from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

__all__ = ["Limit", "enforce"]


@dataclass(frozen=True, slots=True)
class Limit:
    lo: float | None = None
    hi: float | None = None
    lo_open: bool = False
    hi_open: bool = False
    integer: bool = False
    optional: bool = False  # None is allowed

    def describe(self) -> str:
        kind = "an integer" if self.integer else "a finite number"
        parts = []
        if self.lo is not None:
            parts.append(f"{'>' if self.lo_open else '>='} {self.lo:g}")
        if self.hi is not None:
            parts.append(f"{'<' if self.hi_open else '<='} {self.hi:g}")
        return kind + (" " + " and ".join(parts) if parts else "")

    def admits(self, value: Any) -> bool:
        if value is None:
            return self.optional
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            return False
        if self.integer and not isinstance(value, int):
            return False
        if not math.isfinite(value):
            return False
        if self.lo is not None and (value < self.lo or (self.lo_open and value == self.lo)):
            return False
        return not (self.hi is not None and (value > self.hi or (self.hi_open and value == self.hi)))


def enforce(obj: Any, limits: Mapping[str, Limit]) -> None:
    """Raise ``ValueError`` for the first field of ``obj`` outside its limit."""
    for name, limit in limits.items():
        value = getattr(obj, name)
        if not limit.admits(value):
            raise ValueError(f"{type(obj).__name__}.{name} must be {limit.describe()}; got {value!r}")
