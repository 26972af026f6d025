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

__all__ = ["InterleavedPipelineRunner", "PipelineConfig", "PipelineRunner", "ScheduleName", "StageBlocks",
           "balanced_split_points", "build_pipeline_schedule", "interleaved_order", "interleaved_timetable",
           "is_block_list", "split_model", "split_model_interleaved", "stage_for_rank"]

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


class StageBlocks(nn.ModuleDict):
    """One pipeline stage's blocks, registered under their indices in the full model
    (``blocks.12.attention...``), so parameter names, state dicts and DCP checkpoints
    of a stage match the unsplit model. Iterating yields the blocks in order."""

    def __iter__(self):  # noqa: ANN204 - the blocks, not their names
        return iter(self.values())

    def __getitem__(self, key):  # noqa: ANN001, ANN204 - position within the stage, or the global name
        if isinstance(key, int):
            return list(self.values())[key]
        return super().__getitem__(key)


def is_block_list(blocks: object) -> bool:
    """A model's block container: an ``nn.ModuleList`` or a pipeline stage's :class:`StageBlocks`."""
    return isinstance(blocks, (nn.ModuleList, StageBlocks))


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
    lo, hi = bounds[stage_index], bounds[stage_index + 1]
    setattr(model, block_attribute, StageBlocks({str(i): blocks[i] for i in range(lo, hi)}))
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


# --------------------------------------------------------------------------- execution
class _Carry:
    """The tensors one stage hands the next for a micro-batch: hidden states, the
    text context (or None) and the modulation rows. On the receiving side they are
    leaves that collect their gradients, sent back upstream in backward."""

    __slots__ = ("context", "hidden", "modulation")

    def __init__(self, hidden: torch.Tensor, context: torch.Tensor | None, modulation: torch.Tensor) -> None:
        self.hidden, self.context, self.modulation = hidden, context, modulation

    def tensors(self) -> list[torch.Tensor]:
        return [t for t in (self.hidden, self.context, self.modulation) if t is not None]


class PipelineRunner:
    """Runs one pipeline stage of a model that exposes ``stage_embed`` / ``stage_inputs``
    / ``stage_blocks`` / ``stage_head`` (:class:`~avgen_b200.models.VideoDiT`) through a
    1F1B or GPipe schedule, exchanging carries with the neighbouring stages by NCCL
    (or gloo) point-to-point operations.

    In the steady 1F1B state each stage batches "send my forward output, receive the
    gradient of an earlier micro-batch" (and the mirror operation downstream) into
    one grouped call, so the two neighbours' operations match and progress together,
    and the compute stream only waits on a transfer when it needs its data: the send
    of one micro-batch's activations overlaps the backward of another. The last stage
    evaluates ``loss_fn(micro_index, output)``; every stage accumulates its own
    parameters' gradients (the reference leaves its schedules unused:
    avgen/parallel/pipeline.py:254-289)."""

    def __init__(self, model: nn.Module, group: Any, *, schedule: str = "1f1b") -> None:
        import torch.distributed as dist

        if schedule not in ("1f1b", "gpipe"):
            raise ValueError(f"PipelineRunner runs the 1f1b and gpipe schedules; got {schedule!r}")
        for name in ("stage_embed", "stage_inputs", "stage_blocks", "stage_head"):
            if not callable(getattr(model, name, None)):
                raise TypeError(f"{type(model).__name__} has no {name}(): it cannot run as pipeline stages")
        self.model = model
        self.group = group
        self.schedule = schedule
        self.stage = dist.get_rank(group)
        self.stages = dist.get_world_size(group)
        ranks = dist.get_process_group_ranks(group)
        self._prev = ranks[self.stage - 1] if self.stage > 0 else None
        self._next = ranks[self.stage + 1] if self.stage < self.stages - 1 else None

    @property
    def first(self) -> bool:
        return self.stage == 0

    @property
    def last(self) -> bool:
        return self.stage == self.stages - 1

    # ---------------------------------------------------------------- communication
    def _exchange(self, sends: list[tuple[torch.Tensor, int]], recvs: list[tuple[torch.Tensor, int]]) -> None:
        """One grouped batch of point-to-point operations; the caller's stream (or the
        host, with gloo) waits for it before the received tensors are used."""
        import torch.distributed as dist

        ops = [dist.P2POp(dist.isend, t.contiguous(), peer, self.group) for t, peer in sends]
        ops += [dist.P2POp(dist.irecv, t, peer, self.group) for t, peer in recvs]
        if not ops:
            return
        for work in dist.batch_isend_irecv(ops):
            work.wait()

    def _carry_like(self, spec: list[tuple[tuple[int, ...], torch.dtype]], device: torch.device) -> list[torch.Tensor]:
        return [torch.empty(shape, dtype=dtype, device=device) for shape, dtype in spec]

    # ---------------------------------------------------------------- compute
    def _forward(self, k: int, inputs: Any, received: list[torch.Tensor] | None,
                 loss_fn: Callable[[int, Any], torch.Tensor]) -> tuple[Any, Any]:
        """Returns (what backward starts from, this micro-batch's received leaves)."""
        if self.first:
            carry = _Carry(*self.model(inputs, stage="embed"))
            leaves = None
        else:
            assert received is not None
            leaves = [t.requires_grad_() for t in received]
            it = iter(leaves)
            hidden = next(it)
            context = next(it) if self._has_context(inputs) else None
            carry = _Carry(hidden, context, next(it))
        hidden = self.model(inputs, stage="blocks", carry=(carry.hidden, carry.context, carry.modulation),
                            aux=self.model.stage_inputs(inputs))
        if self.last:
            return loss_fn(k, self.model(inputs, stage="head", hidden=hidden)), leaves
        return _Carry(hidden, carry.context, carry.modulation), leaves

    def _has_context(self, inputs: Any) -> bool:
        return (not inputs.text.is_empty) and bool(getattr(self.model.config, "cross_attention", True))

    def _spec(self, inputs: Any, like: Any) -> list[tuple[tuple[int, ...], torch.dtype]]:
        """Shapes and dtypes of a carry for ``inputs`` (every stage derives it alike)."""
        cfg = self.model.config
        video = inputs.video
        b, length = video.batch_size, video.length
        dtype = torch.bfloat16 if video.tokens.device.type == "cuda" else like.dtype
        spec = [((b, length, cfg.width), dtype)]
        if self._has_context(inputs):
            spec.append(((b, inputs.text.features.shape[1], cfg.width), dtype))
        if video.has_level_groups:
            rows = video.level_values.numel()
        elif video.per_token_noise:
            rows = b * length
        else:
            rows = b
        spec.append(((rows, 6, cfg.width), torch.float32))
        return spec

    def _backward(self, start: Any, grads: list[torch.Tensor] | None, leaves: list[torch.Tensor] | None
                  ) -> list[torch.Tensor] | None:
        if self.last:
            start.backward()
        else:
            outs = start.tensors()
            assert grads is not None and len(grads) == len(outs)
            torch.autograd.backward(outs, grads)
        if leaves is None:
            return None
        return [t.grad if t.grad is not None else torch.zeros_like(t) for t in leaves]

    # ---------------------------------------------------------------- schedule
    def run(self, micro_inputs: Sequence[Any], loss_fn: Callable[[int, Any], torch.Tensor]) -> list[torch.Tensor]:
        """Forward and backward of every micro-batch on this stage. Returns the losses
        (last stage only; empty elsewhere). Gradients accumulate in the parameters."""
        m = len(micro_inputs)
        if m == 0:
            return []
        like = next(self.model.parameters())
        device = like.device
        warmup = m if self.schedule == "gpipe" else min(self.stages - self.stage - 1, m)
        starts: dict[int, Any] = {}
        leaves: dict[int, Any] = {}
        losses: list[torch.Tensor] = []

        def recv_forward(k: int) -> list[torch.Tensor] | None:
            if self.first:
                return None
            bufs = self._carry_like(self._spec(micro_inputs[k], like), device)
            self._exchange([], [(t, self._prev) for t in bufs])
            return bufs

        def forward(k: int, received: list[torch.Tensor] | None) -> None:
            start, leaves[k] = self._forward(k, micro_inputs[k], received, loss_fn)
            starts[k] = start
            if self.last:
                losses.append(start.detach())

        def outgoing(k: int) -> list[tuple[torch.Tensor, int]]:
            if self.last:
                return []
            return [(t.detach(), self._next) for t in starts[k].tensors()]

        def grad_bufs(k: int) -> list[torch.Tensor]:
            return [] if self.last else self._carry_like(self._spec(micro_inputs[k], like), device)

        def backward(k: int, grads: list[torch.Tensor] | None) -> list[torch.Tensor] | None:
            out = self._backward(starts.pop(k), grads, leaves.pop(k))
            return out

        # warm-up forwards (all of them for GPipe)
        for k in range(warmup):
            forward(k, recv_forward(k))
            self._exchange(outgoing(k), [])
        # steady state: one forward, one backward
        received = recv_forward(warmup) if warmup < m else None
        for i in range(m - warmup):
            k = warmup + i
            forward(k, received)
            grads = grad_bufs(i)
            self._exchange(outgoing(k), [(g, self._next) for g in grads])
            upstream = backward(i, grads or None)
            nxt = k + 1
            if nxt < m:
                bufs = None if self.first else self._carry_like(self._spec(micro_inputs[nxt], like), device)
                sends = [] if upstream is None else [(g, self._prev) for g in upstream]
                self._exchange(sends, [] if bufs is None else [(t, self._prev) for t in bufs])
                received = bufs
            elif upstream is not None:
                self._exchange([(g, self._prev) for g in upstream], [])
        # cool-down backwards
        for i in range(m - warmup, m):
            grads = grad_bufs(i)
            self._exchange([], [(g, self._next) for g in grads])
            upstream = backward(i, grads or None)
            if upstream is not None:
                self._exchange([(g, self._prev) for g in upstream], [])
        return losses


# --------------------------------------------------------------------------- interleaved (virtual) stages
def split_model_interleaved(model: nn.Module, *, rank: int, ranks: int, chunks_per_rank: int,
                            split_points: Sequence[int], block_attribute: str = "blocks") -> nn.Module:
    """Keep this rank's ``chunks_per_rank`` chunks of an interleaved pipeline.

    The block list is cut into ``ranks * chunks_per_rank`` contiguous chunks; chunk
    ``g`` lives on rank ``g % ranks`` (rank ``r`` owns chunks ``r, r + ranks, ...``),
    so a micro-batch visits every rank ``chunks_per_rank`` times. The rank keeps its
    blocks under their global names (one :class:`StageBlocks`) and records each
    chunk's blocks in ``model.pipeline_chunks``; the input modules stay on the rank
    of chunk 0 (rank 0) and the output head on the rank of the last chunk."""
    chunks = ranks * chunks_per_rank
    if not 0 <= rank < ranks:
        raise ValueError(f"rank must be in [0, {ranks}); got {rank!r}")
    blocks = getattr(model, block_attribute, None)
    if not isinstance(blocks, nn.ModuleList):
        raise AttributeError(f"{type(model).__name__} has no nn.ModuleList {block_attribute!r}")
    if len(split_points) != chunks - 1:
        raise ValueError(f"{chunks} chunks need {chunks - 1} split points; got {len(split_points)}")
    bounds = [0, *split_points, len(blocks)]
    owned = [g for g in range(chunks) if g % ranks == rank]
    per_chunk = [StageBlocks({str(i): blocks[i] for i in range(bounds[g], bounds[g + 1])}) for g in owned]
    setattr(model, block_attribute, StageBlocks({k: m for chunk in per_chunk for k, m in chunk.items()}))
    model.pipeline_chunks = per_chunk  # plain attribute: the modules are registered once, above
    if rank != 0:
        for name in _INPUT_MODULES:
            if hasattr(model, name):
                setattr(model, name, None)
    if rank != (chunks - 1) % ranks:
        for name in _OUTPUT_MODULES:
            if hasattr(model, name):
                setattr(model, name, None)
    return model


def interleaved_order(rank: int, ranks: int, chunks_per_rank: int, microbatches: int) -> list[tuple[str, int, int]]:
    """Rank ``rank``'s actions ``(kind, local chunk, micro-batch)`` in interleaved 1F1B
    order: ``min(2 (ranks - rank - 1) + (chunks_per_rank - 1) ranks, total)`` warm-up
    forwards, then alternating forward / backward, then the remaining backwards.
    Forward ``k`` runs chunk ``(k // ranks) % v`` of micro-batch ``(k // (ranks v)) ranks + k % ranks``;
    backwards visit the chunks in reverse (the schedule of Narayanan et al., 2021)."""
    p, v, m = ranks, chunks_per_rank, microbatches
    if m % p:
        raise ValueError(f"the interleaved schedule needs the micro-batch count ({m}) to be a multiple of the "
                         f"pipeline size ({p})")
    total = m * v

    def mb(k: int) -> int:
        return (k // (p * v)) * p + k % p

    fwd = [("F", (k // p) % v, mb(k)) for k in range(total)]
    bwd = [("B", v - 1 - (k // p) % v, mb(k)) for k in range(total)]
    warm = min(2 * (p - rank - 1) + (v - 1) * p, total)
    order = fwd[:warm]
    for f, b in zip(fwd[warm:], bwd):
        order += [f, b]
    return order + bwd[total - warm:]


def interleaved_timetable(ranks: int, chunks_per_rank: int, microbatches: int) -> list[list[tuple[str, int, int] | None]]:
    """Lock-step ticks: ``table[t][r]`` is rank ``r``'s action at tick ``t`` (or None when
    it waits). Every rank derives the same table, so the point-to-point transfers of a
    tick (a finished forward's carry to the next chunk's rank, a finished backward's
    input gradients to the previous chunk's rank) are posted by both sides in the same
    tick and matched by construction. A rank runs its next action as soon as its input
    arrived in an earlier tick."""
    p, v = ranks, chunks_per_rank
    orders = [interleaved_order(r, p, v, microbatches) for r in range(p)]
    last = p * v - 1
    fwd_done: dict[tuple[int, int], int] = {}
    bwd_done: dict[tuple[int, int], int] = {}
    pos = [0] * p
    table: list[list[tuple[str, int, int] | None]] = []
    t = 0
    while any(pos[r] < len(orders[r]) for r in range(p)):
        row: list[tuple[str, int, int] | None] = [None] * p
        for r in range(p):
            if pos[r] >= len(orders[r]):
                continue
            kind, j, k = orders[r][pos[r]]
            g = j * p + r
            if kind == "F":
                ready = g == 0 or fwd_done.get((g - 1, k), t) < t
            else:
                ready = fwd_done.get((g, k), t) < t and (g == last or bwd_done.get((g + 1, k), t) < t)
            if ready:
                row[r] = (kind, j, k)
        if not any(row):
            raise RuntimeError("interleaved schedule stalled: no rank can make progress")
        for r, action in enumerate(row):
            if action is not None:
                kind, j, k = action
                (fwd_done if kind == "F" else bwd_done)[(j * p + r, k)] = t
                pos[r] += 1
        table.append(row)
        t += 1
    return table


class InterleavedPipelineRunner(PipelineRunner):
    """Interleaved 1F1B over ``chunks_per_rank`` virtual stages per rank (a model cut by
    :func:`split_model_interleaved`): the pipeline bubble shrinks by that factor at the
    cost of ``chunks_per_rank`` times as many carries crossing between ranks. Each tick
    of :func:`interleaved_timetable` runs at most one forward or backward chunk per
    rank, then one grouped exchange with the neighbours (the carry to the next chunk's
    rank, input gradients to the previous chunk's rank; chunk ``g``'s neighbours are
    ranks ``g - 1`` and ``g + 1`` mod ``ranks``)."""

    def __init__(self, model: nn.Module, group: Any, *, chunks_per_rank: int) -> None:
        super().__init__(model, group, schedule="1f1b")
        if self.stages < 2:
            raise ValueError("an interleaved pipeline needs at least two ranks")
        chunks = getattr(model, "pipeline_chunks", None)
        if chunks is None or len(chunks) != chunks_per_rank:
            raise ValueError(f"the model holds {0 if chunks is None else len(chunks)} pipeline chunks; expected "
                             f"{chunks_per_rank} (cut it with split_model_interleaved)")
        self.chunks_per_rank = chunks_per_rank
        import torch.distributed as dist

        self._ranks = dist.get_process_group_ranks(group)

    def _peer(self, rank: int) -> int:
        return self._ranks[rank % self.stages]

    def run(self, micro_inputs: Sequence[Any], loss_fn: Callable[[int, Any], torch.Tensor]) -> list[torch.Tensor]:
        m = len(micro_inputs)
        if m == 0:
            return []
        p, v, r = self.stages, self.chunks_per_rank, self.stage
        last = p * v - 1
        like = next(self.model.parameters())
        device = like.device
        table = interleaved_timetable(p, v, m)
        inputs: dict[tuple[int, int], list[torch.Tensor]] = {}   # received carries, by (global chunk, micro-batch)
        grads_in: dict[tuple[int, int], list[torch.Tensor]] = {}  # received output gradients
        starts: dict[tuple[int, int], Any] = {}
        leaves: dict[tuple[int, int], Any] = {}
        losses: dict[int, torch.Tensor] = {}

        def spec(k: int) -> list[tuple[tuple[int, ...], torch.dtype]]:
            return self._spec(micro_inputs[k], like)

        for row in table:
            sends: list[tuple[torch.Tensor, int]] = []
            mine = row[r]
            if mine is not None:
                kind, j, k = mine
                g = j * p + r
                if kind == "F":
                    start, leaf = self._chunk_forward(g, j, k, micro_inputs[k], inputs.pop((g, k), None), loss_fn,
                                                      last)
                    starts[(g, k)], leaves[(g, k)] = start, leaf
                    if g == last:
                        losses[k] = start.detach()
                    else:
                        sends += [(t.detach(), self._peer(r + 1)) for t in start.tensors()]
                else:
                    up = self._chunk_backward(starts.pop((g, k)), grads_in.pop((g, k), None), leaves.pop((g, k)),
                                              g == last)
                    if up is not None:
                        sends += [(t, self._peer(r - 1)) for t in up]
            recvs: list[tuple[torch.Tensor, int]] = []
            prev_rank, next_rank = (r - 1) % p, (r + 1) % p
            theirs = row[prev_rank]
            if theirs is not None and theirs[0] == "F":  # the previous chunk's carry, for my next chunk
                g = theirs[1] * p + prev_rank
                if g != last:
                    bufs = self._carry_like(spec(theirs[2]), device)
                    inputs[(g + 1, theirs[2])] = bufs
                    recvs += [(t, self._peer(prev_rank)) for t in bufs]
            theirs = row[next_rank]
            if theirs is not None and theirs[0] == "B":  # the next chunk's input gradients, for my chunk
                g = theirs[1] * p + next_rank
                if g != 0:
                    bufs = self._carry_like(spec(theirs[2]), device)
                    grads_in[(g - 1, theirs[2])] = bufs
                    recvs += [(t, self._peer(next_rank)) for t in bufs]
            self._exchange(sends, recvs)
        return [losses[k] for k in sorted(losses)]

    @staticmethod
    def _chunk_backward(start: Any, grads: list[torch.Tensor] | None, leaves: list[torch.Tensor] | None,
                        is_last: bool) -> list[torch.Tensor] | None:
        """Backward of one chunk from its loss (last chunk) or its output gradients;
        returns its input gradients (None for chunk 0)."""
        if is_last:
            start.backward()
        else:
            outs = start.tensors()
            assert grads is not None and len(grads) == len(outs), "output gradients did not arrive"
            torch.autograd.backward(outs, grads)
        if leaves is None:
            return None
        return [t.grad if t.grad is not None else torch.zeros_like(t) for t in leaves]

    def _chunk_forward(self, g: int, j: int, k: int, inputs: Any, received: list[torch.Tensor] | None,
                       loss_fn: Callable[[int, Any], torch.Tensor], last: int) -> tuple[Any, Any]:
        if g == 0:
            carry = _Carry(*self.model(inputs, stage="embed"))
            leaves = None
        else:
            assert received is not None, f"chunk {g}: no carry arrived for micro-batch {k}"
            leaves = [t.requires_grad_() for t in received]
            it = iter(leaves)
            hidden = next(it)
            context = next(it) if self._has_context(inputs) else None
            carry = _Carry(hidden, context, next(it))
        aux = dict(self.model.stage_inputs(inputs), blocks=self.model.pipeline_chunks[j])
        hidden = self.model(inputs, stage="blocks", carry=(carry.hidden, carry.context, carry.modulation), aux=aux)
        if g == last:
            return loss_fn(k, self.model(inputs, stage="head", hidden=hidden)), leaves
        return _Carry(hidden, carry.context, carry.modulation), leaves
