"""Training-state protocols and the mutable TrainState (avgen/core/state.py:35-170)."""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, field
from typing import Any, Protocol, runtime_checkable

from torch import nn

from avgen_b200.core.rng import RNGStreams

__all__ = ["EMA", "DataCursor", "LRSchedule", "Stateful", "TrainState"]


@runtime_checkable
class Stateful(Protocol):
    def state_dict(self) -> Mapping[str, Any]: ...

    def load_state_dict(self, state: Mapping[str, Any]) -> None: ...


@runtime_checkable
class LRSchedule(Stateful, Protocol):
    def step(self) -> object: ...

    def get_last_lr(self) -> list[float]: ...


@runtime_checkable
class EMA(Stateful, Protocol):
    def update(self, model: nn.Module) -> object: ...


@runtime_checkable
class DataCursor(Stateful, Protocol):
    def advance(self, samples: int) -> None: ...


_COUNTERS = ("step", "samples_seen", "tokens_seen", "epoch")


@dataclass(slots=True)
class TrainState:
    """Everything a step mutates, plus progress counters and checkpointable extras."""

    model: nn.Module
    optimizer: Any
    rng: RNGStreams
    schedule: LRSchedule | None = None
    ema: EMA | None = None
    step: int = 0
    samples_seen: int = 0
    tokens_seen: int = 0
    epoch: int = 0
    extras: dict[str, Stateful] = field(default_factory=dict)

    def validate(self) -> None:
        for name in _COUNTERS:
            v = getattr(self, name)
            if isinstance(v, bool) or not isinstance(v, int) or v < 0:
                raise ValueError(f"{name} must be a non-negative integer; got {v!r}")
        self.rng.validate()

    def progress(self) -> dict[str, int]:
        return {name: getattr(self, name) for name in _COUNTERS}

    def load_progress(self, values: Mapping[str, int]) -> None:
        for name in _COUNTERS:
            if name not in values:
                raise KeyError(f"missing progress counter {name!r}")
            setattr(self, name, int(values[name]))
