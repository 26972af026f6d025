"""Sequence packing: several token streams in one fixed-length row
(avgen/data/packing.py:75-526).

A :class:`PackedLayout` records where each segment sits in a row and exposes
``segment_ids``, ``cu_seqlens`` (varlen offsets), a block-diagonal attention
mask, per-token segment weights (so each sample contributes equally to the
loss regardless of its length) and the validity mask. ``plan_packing`` is a
first-fit-decreasing bin packer; ``pack_streams`` / ``split_packed`` move token
streams in and out of packed rows.
"""
from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch

from avgen_b200.core.tokens import PatchLayout, TokenStream

__all__ = ["PackPlan", "PackedLayout", "pack_streams", "plan_packing", "split_packed"]


@dataclass(frozen=True, slots=True)
class PackedLayout:
    capacity: int
    lengths: tuple[int, ...]
    sources: tuple[int, ...] = ()

    def __post_init__(self) -> None:
        if self.capacity < 1:
            raise ValueError("capacity must be positive")
        if any(n < 1 for n in self.lengths):
            raise ValueError("segment lengths must be positive")
        if sum(self.lengths) > self.capacity:
            raise ValueError(f"segments ({sum(self.lengths)} tokens) exceed the row capacity {self.capacity}")

    @property
    def segment_count(self) -> int:
        return len(self.lengths)

    @property
    def offsets(self) -> tuple[int, ...]:
        out, acc = [], 0
        for n in self.lengths:
            out.append(acc)
            acc += n
        return tuple(out)

    @property
    def used(self) -> int:
        return sum(self.lengths)

    @property
    def occupancy(self) -> float:
        return self.used / self.capacity

    def segment_ids(self, *, device: torch.device | str = "cpu") -> torch.Tensor:
        """``(capacity,)`` int64: segment index per token, ``-1`` for padding."""
        ids = torch.full((self.capacity,), -1, dtype=torch.int64, device=device)
        for i, (off, n) in enumerate(zip(self.offsets, self.lengths)):
            ids[off:off + n] = i
        return ids

    def cu_seqlens(self) -> torch.Tensor:
        """``(segments + 1,)`` int32 cumulative offsets (varlen attention layout)."""
        return torch.tensor([0, *torch.tensor(self.lengths).cumsum(0).tolist()], dtype=torch.int32)

    def attention_mask(self, *, device: torch.device | str = "cpu") -> torch.Tensor:
        """``(capacity, capacity)`` bool: tokens attend only within their segment."""
        ids = self.segment_ids(device=device)
        return (ids[:, None] == ids[None, :]) & (ids[:, None] >= 0)

    def segment_weights(self, *, device: torch.device | str = "cpu") -> torch.Tensor:
        """``(capacity,)`` fp32: ``1 / length`` of the token's segment (0 on padding)."""
        w = torch.zeros(self.capacity, dtype=torch.float32, device=device)
        for off, n in zip(self.offsets, self.lengths):
            w[off:off + n] = 1.0 / n
        return w

    def valid_mask(self, *, device: torch.device | str = "cpu") -> torch.Tensor:
        return self.segment_ids(device=device) >= 0


@dataclass(frozen=True, slots=True)
class PackPlan:
    rows: tuple[PackedLayout, ...]

    @property
    def occupancy(self) -> float:
        cap = sum(r.capacity for r in self.rows)
        return sum(r.used for r in self.rows) / cap if cap else 0.0

    def layout_for(self, row: int) -> PackedLayout:
        return self.rows[row]


def plan_packing(lengths: Sequence[int], capacity: int, *, max_segments: int | None = None) -> PackPlan:
    """First-fit decreasing: every length goes to the first row with room."""
    if any(n > capacity for n in lengths):
        raise ValueError("a stream is longer than the row capacity")
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    rows: list[list[int]] = []
    room: list[int] = []
    for i in order:
        for r, free in enumerate(room):
            if lengths[i] <= free and (max_segments is None or len(rows[r]) < max_segments):
                rows[r].append(i)
                room[r] -= lengths[i]
                break
        else:
            rows.append([i])
            room.append(capacity - lengths[i])
    return PackPlan(tuple(PackedLayout(capacity, tuple(lengths[i] for i in r), tuple(r)) for r in rows))


def pack_streams(streams: Sequence[TokenStream], layout: PackedLayout) -> TokenStream:
    """Concatenate single-sample streams into one packed row of ``layout.capacity`` tokens."""
    if len(streams) != layout.segment_count:
        raise ValueError("one stream per segment is required")
    width = streams[0].width
    dev = streams[0].device
    dtype = streams[0].tokens.dtype
    tokens = torch.zeros(1, layout.capacity, width, dtype=dtype, device=dev)
    coords = torch.zeros(1, layout.capacity, 3, dtype=torch.float32, device=dev)
    mask = torch.zeros(1, layout.capacity, dtype=torch.bool, device=dev)
    cond = torch.zeros_like(mask)
    noise = torch.zeros(1, layout.capacity, dtype=torch.float32, device=dev)
    for s, off, n in zip(streams, layout.offsets, layout.lengths):
        if s.batch_size != 1 or s.length != n:
            raise ValueError("each stream must be a single sample of its segment length")
        tokens[0, off:off + n] = s.tokens[0]
        coords[0, off:off + n] = s.coords[0]
        mask[0, off:off + n] = s.mask[0]
        cond[0, off:off + n] = s.conditioned[0]
        noise[0, off:off + n] = s.expanded_noise()[0]
    return TokenStream(tokens=tokens, coords=coords, mask=mask, noise_level=noise,
                       layout=PatchLayout.temporal(layout.capacity, width), conditioned=cond)


def split_packed(tensor: torch.Tensor, layout: PackedLayout) -> list[torch.Tensor]:
    """Per-segment slices ``(1, n, ...)`` of a packed ``(1, capacity, ...)`` tensor."""
    return [tensor[:, off:off + n] for off, n in zip(layout.offsets, layout.lengths)]
