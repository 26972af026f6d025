"""Pipeline parallelism: stage splitting and schedules (avgen/parallel/pipeline.py:64-301 API).

``balanced_split_points`` cuts the block list into contiguous stages minimising
the most expensive stage (blocks cost 1; the first stage also carries the input
embeddings and the last the output head, each weighted by a fraction of a
block). The min-max cut is found exactly by a binary search on the bottleneck
with a greedy feasibility check. ``split_model`` keeps one stage's blocks and
drops the embeddings / head it does not own; schedules come from
``torch.distributed.pipelining``.
"""
from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any, Literal

import torch
from torch import nn

__all__ = ["PipelineConfig", "ScheduleName", "balanced_split_points", "build_pipeline_schedule", "split_model",
           "stage_for_rank"]

ScheduleName = Literal["gpipe", "1f1b", "interleaved_1f1b", "zero_bubble"]
_NAMES = ("gpipe", "1f1b", "interleaved_1f1b", "zero_bubble")
_INPUT_MODULES = ("patch_embed", "time_embed", "text_proj", "text_refiner", "modulation")
_OUTPUT_MODULES = ("final_norm", "final_proj")


@dataclass(frozen=True, slots=True)
class PipelineConfig:
    schedule: ScheduleName = "1f1b"
    microbatches: int = 8
    stages_per_rank: int = 1
    embedding_weight: float = 0.5
    head_weight: float = 0.5

    def __post_init__(self) -> None:
        if self.schedule not in _NAMES:
            raise ValueError(f"unknown schedule {self.schedule!r}; available: {', '.join(_NAMES)}")
        for name in ("microbatches", "stages_per_rank"):
            v = getattr(self, name)
            if isinstance(v, bool) or v < 1:
                raise ValueError(f"{name} must be >= 1; got {v!r}")
        if self.stages_per_rank > 1 and self.schedule in ("gpipe", "1f1b"):
            raise ValueError(f"{self.schedule!r} runs one stage per rank; use interleaved_1f1b or zero_bubble")

    @property
    def is_interleaved(self) -> bool:
        return self.stages_per_rank > 1

    def bubble_fraction(self, stages: int) -> float:
        """Idle fraction of a step: (p - 1) / (m + p - 1) with p the effective depth."""
        if stages <= 1:
            return 0.0
        p = max(1, stages // self.stages_per_rank)
        if self.schedule == "zero_bubble":
            p = max(1, p // 2)
        return (p - 1) / (self.microbatches + p - 1)


def _fits(costs: list[float], stages: int, limit: float) -> list[int] | None:
    """Greedy cut with every stage under ``limit``; None if it needs more than ``stages``."""
    points, acc = [], 0.0
    for i, c in enumerate(costs):
        if c > limit:
            return None
        if acc + c > limit:
            points.append(i)
            acc = 0.0
        acc += c
    return points if len(points) <= stages - 1 else None


def balanced_split_points(num_blocks: int, num_stages: int, *, embedding_weight: float = 0.5,
                          head_weight: float = 0.5) -> list[int]:
    if num_stages < 1:
        raise ValueError(f"num_stages must be >= 1; got {num_stages!r}")
    if num_blocks < num_stages:
        raise ValueError(f"cannot split {num_blocks} blocks into {num_stages} stages")
    if num_stages == 1:
        return []
    costs = [1.0] * num_blocks
    costs[0] += embedding_weight
    costs[-1] += head_weight
    lo, hi = max(costs), sum(costs)
    best = _fits(costs, num_stages, hi)
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        found = _fits(costs, num_stages, mid)
        if found is None:
            lo = mid
        else:
            hi, best = mid, found
    assert best is not None
    points = list(best)
    # every stage needs at least one block: split the largest stages until there are num_stages
    while len(points) < num_stages - 1:
        bounds = [0, *points, num_blocks]
        sizes = [(bounds[i + 1] - bounds[i], i) for i in range(len(bounds) - 1)]
        size, i = max(sizes)
        points.insert(i, bounds[i] + size // 2)
        points.sort()
    return points


def split_model(model: nn.Module, *, stage_index: int, num_stages: int, split_points: Sequence[int],
                block_attribute: str = "blocks") -> nn.Module:
    if not 0 <= stage_index < num_stages:
        raise ValueError(f"stage_index must be in [0, {num_stages}); got {stage_index!r}")
    blocks = getattr(model, block_attribute, None)
    if not isinstance(blocks, nn.ModuleList):
        raise AttributeError(f"{type(model).__name__} has no nn.ModuleList {block_attribute!r}")
    if len(split_points) != num_stages - 1:
        raise ValueError(f"{num_stages} stages need {num_stages - 1} split points; got {len(split_points)}")
    bounds = [0, *split_points, len(blocks)]
    setattr(model, block_attribute, nn.ModuleList(list(blocks)[bounds[stage_index]:bounds[stage_index + 1]]))
    if stage_index > 0:
        for name in _INPUT_MODULES:
            if hasattr(model, name):
                setattr(model, name, None)
    if stage_index < num_stages - 1:
        for name in _OUTPUT_MODULES:
            if hasattr(model, name):
                setattr(model, name, None)
    return model


def build_pipeline_schedule(stages: Sequence[Any], config: PipelineConfig,
                            loss_fn: Callable[[Any, Any], torch.Tensor] | None = None) -> Any:
    from torch.distributed.pipelining import schedules as S

    cls = {"gpipe": S.ScheduleGPipe, "1f1b": S.Schedule1F1B, "interleaved_1f1b": S.ScheduleInterleaved1F1B,
           "zero_bubble": S.ScheduleInterleavedZeroBubble}[config.schedule]
    if config.is_interleaved:
        if len(stages) != config.stages_per_rank:
            raise ValueError(f"interleaved schedule expects {config.stages_per_rank} stages per rank; got "
                             f"{len(stages)}")
        return cls(list(stages), n_microbatches=config.microbatches, loss_fn=loss_fn)
    if len(stages) != 1:
        raise ValueError(f"{config.schedule!r} takes one stage per rank; got {len(stages)}")
    return cls(stages[0], n_microbatches=config.microbatches, loss_fn=loss_fn)


def stage_for_rank(mesh: Any) -> tuple[int, int]:
    """(stage index, number of stages) of this rank on the pipeline mesh."""
    return mesh.get_local_rank(), mesh.size()
