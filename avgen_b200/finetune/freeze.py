"""Freezing helpers and the trainable-parameter summary (avgen/finetune/freeze.py:117-232 API)."""
from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass

from torch import nn

from avgen_b200.finetune._match import matches_any, normalize_patterns

__all__ = ["TrainableSummary", "freeze_all", "freeze_except", "freeze_matching", "trainable_summary"]


@dataclass(frozen=True, slots=True)
class TrainableSummary:
    trainable: int
    frozen: int
    trainable_tensors: int
    total_tensors: int

    @property
    def total(self) -> int:
        return self.trainable + self.frozen

    @property
    def percentage(self) -> float:
        return 100.0 * self.trainable / self.total if self.total else 0.0

    @property
    def optimizer_state_bytes(self) -> int:
        """fp32 master + two AdamW moments per trainable parameter."""
        return 12 * self.trainable

    def describe(self) -> str:
        return (f"{_si(self.trainable)} trainable of {_si(self.total)} ({self.percentage:.2f}%), "
                f"{self.trainable_tensors}/{self.total_tensors} tensors, optimizer state "
                f"{_si(self.optimizer_state_bytes)}B")


def _si(v: float) -> str:
    for unit in ("", "K", "M", "G", "T"):
        if abs(v) < 1000:
            return f"{v:.1f}{unit}" if unit else f"{int(v)}"
        v /= 1000.0
    return f"{v:.1f}P"


def trainable_summary(model: nn.Module) -> TrainableSummary:
    t = f = tt = n = 0
    for p in model.parameters():
        n += 1
        if p.requires_grad:
            t += p.numel()
            tt += 1
        else:
            f += p.numel()
    return TrainableSummary(t, f, tt, n)


def freeze_all(model: nn.Module) -> int:
    count = 0
    for p in model.parameters():
        count += p.numel()
        p.requires_grad_(False)
    return count


def freeze_except(model: nn.Module, patterns: Iterable[str]) -> TrainableSummary:
    """Train only parameters whose names match one of ``patterns``."""
    pats = normalize_patterns(patterns)
    if not pats:
        raise ValueError("freeze_except needs at least one pattern")
    hits = 0
    for name, p in model.named_parameters():
        keep = matches_any(name, pats)
        hits += int(keep)
        p.requires_grad_(keep)
    if not hits:
        raise ValueError(f"no parameter matches {pats}")
    return trainable_summary(model)


def freeze_matching(model: nn.Module, patterns: Iterable[str]) -> TrainableSummary:
    """Freeze parameters whose names match one of ``patterns`` (others unchanged)."""
    pats = normalize_patterns(patterns)
    for name, p in model.named_parameters():
        if matches_any(name, pats):
            p.requires_grad_(False)
    return trainable_summary(model)
