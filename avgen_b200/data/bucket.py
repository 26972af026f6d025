"""Resolution x duration buckets, largest-remainder quotas and curricula
(avgen/data/bucket.py:67-549).

A :class:`BucketSampler` turns per-bucket sample pools into an epoch of
same-shape batches: the number of batches per bucket follows the current
curriculum weights exactly (largest-remainder rounding), batches are shuffled
with a seeded permutation, and every data rank gets a disjoint slice.
"""
from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from dataclasses import dataclass

import torch

from avgen_b200.core.rng import mix_seed
from avgen_b200.data.protocols import BucketPlan

__all__ = ["BucketBatch", "BucketCurriculum", "BucketSampler", "CurriculumPhase", "largest_remainder"]


def largest_remainder(total: int, weights: Sequence[float]) -> tuple[int, ...]:
    """Integer quotas summing to ``total`` proportional to ``weights`` (Hamilton's method)."""
    if total < 0:
        raise ValueError("total must be non-negative")
    s = float(sum(weights))
    if s <= 0:
        raise ValueError("weights must contain a positive entry")
    if any(w < 0 for w in weights):
        raise ValueError("weights must be non-negative")
    exact = [total * w / s for w in weights]
    base = [math.floor(x) for x in exact]
    left = total - sum(base)
    order = sorted(range(len(weights)), key=lambda i: (-(exact[i] - base[i]), i))
    for i in order[:left]:
        base[i] += 1
    return tuple(base)


@dataclass(frozen=True, slots=True)
class CurriculumPhase:
    until_step: int
    weights: tuple[float, ...]

    def __post_init__(self) -> None:
        if self.until_step < 1:
            raise ValueError("until_step must be positive")
        if not self.weights or sum(self.weights) <= 0 or any(w < 0 for w in self.weights):
            raise ValueError("phase weights must be non-negative with a positive sum")


@dataclass(frozen=True, slots=True)
class BucketCurriculum:
    phases: tuple[CurriculumPhase, ...]
    interpolate: bool = False

    def __post_init__(self) -> None:
        if not self.phases:
            raise ValueError("a curriculum needs at least one phase")
        bounds = [p.until_step for p in self.phases]
        if bounds != sorted(set(bounds)):
            raise ValueError("phase until_step values must increase strictly")
        if len({len(p.weights) for p in self.phases}) != 1:
            raise ValueError("every phase must weight the same buckets")

    @property
    def bucket_count(self) -> int:
        return len(self.phases[0].weights)

    def weights_at(self, step: int) -> tuple[float, ...]:
        prev_end, prev_w = 0, self.phases[0].weights
        for p in self.phases:
            if step < p.until_step:
                if not self.interpolate or p is self.phases[0]:
                    return p.weights
                t = (step - prev_end) / max(1, p.until_step - prev_end)
                return tuple((1 - t) * a + t * b for a, b in zip(prev_w, p.weights))
            prev_end, prev_w = p.until_step, p.weights
        return self.phases[-1].weights


@dataclass(frozen=True, slots=True)
class BucketBatch:
    bucket_id: int
    indices: tuple[int, ...]


class BucketSampler:
    """Plans epochs of same-bucket batches for one data rank."""

    def __init__(self, plan: BucketPlan, assignments: Sequence[int], *, batch_size: int | None = None,
                 weights: Sequence[float] | None = None, curriculum: BucketCurriculum | None = None, seed: int = 0,
                 data_rank: int = 0, data_world: int = 1, drop_last: bool = True) -> None:
        if not 0 <= data_rank < data_world:
            raise ValueError("data_rank must be below data_world")
        self._plan = plan
        self._batch = batch_size
        self._seed = seed
        self._rank = data_rank
        self._world = data_world
        self._drop_last = drop_last
        self._pools: dict[int, list[int]] = {b.bucket_id: [] for b in plan.buckets}
        for i, bid in enumerate(assignments):
            if bid in self._pools:
                self._pools[bid].append(i)
        n = len(plan.buckets)
        if curriculum is not None and curriculum.bucket_count != n:
            raise ValueError("curriculum weights do not match the bucket plan")
        # without explicit weights a bucket is drawn as often as its pool fills whole batches on every
        # rank, so an epoch visits each sample at most once whatever the buckets' micro-batch sizes
        self._weights = tuple(weights) if weights is not None else tuple(
            float(len(self._pools[b.bucket_id]) // (self._bsz(b.bucket_id) * data_world)) for b in plan.buckets)
        self._curriculum = curriculum

    @property
    def plan(self) -> BucketPlan:
        return self._plan

    @property
    def batch_size(self) -> int:
        return self._batch or self._plan.buckets[0].micro_batch_size

    def _bsz(self, bucket_id: int) -> int:
        return self._batch or self._plan.get(bucket_id).micro_batch_size

    def pool_size(self, bucket_id: int) -> int:
        return len(self._pools[bucket_id])

    def batches_per_epoch(self) -> int:
        return sum(len(p) // (self._bsz(b) * self._world) for b, p in self._pools.items())

    def weights_at(self, step: int) -> tuple[float, ...]:
        w = self._curriculum.weights_at(step) if self._curriculum is not None else self._weights
        # a bucket without samples cannot be drawn
        return tuple(x if self._pools[b.bucket_id] else 0.0 for x, b in zip(w, self._plan.buckets))

    def quotas_at(self, step: int, *, batches: int | None = None) -> tuple[int, ...]:
        total = self.batches_per_epoch() if batches is None else batches
        weights = self.weights_at(step)
        if total == 0 or not any(weights):
            return tuple(0 for _ in weights)
        return largest_remainder(total, weights)

    def plan_epoch(self, *, epoch: int, step: int = 0) -> tuple[BucketBatch, ...]:
        """This rank's batches for ``epoch`` (identical plan on every rank, disjoint slices)."""
        quotas = self.quotas_at(step)
        out: list[BucketBatch] = []
        for bucket, quota in zip(self._plan.buckets, quotas):
            pool = self._pools[bucket.bucket_id]
            if not pool or quota == 0:
                continue
            g = torch.Generator().manual_seed(mix_seed(self._seed, epoch, bucket.bucket_id))
            perm = [pool[i] for i in torch.randperm(len(pool), generator=g).tolist()]
            bsz = self._bsz(bucket.bucket_id)
            need = quota * bsz * self._world
            while len(perm) < need:  # upsample a small pool to honour its weight
                perm += perm[: need - len(perm)]
            for q in range(quota):
                start = (q * self._world + self._rank) * bsz
                out.append(BucketBatch(bucket.bucket_id, tuple(perm[start:start + bsz])))
        g = torch.Generator().manual_seed(mix_seed(self._seed, epoch, "order"))
        order = torch.randperm(len(out), generator=g).tolist()
        return tuple(out[i] for i in order)

    def state_dict(self) -> Mapping[str, int]:
        return {"seed": self._seed, "data_rank": self._rank, "data_world": self._world}
