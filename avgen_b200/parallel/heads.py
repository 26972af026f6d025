"""Tensor parallelism by attention heads: uneven head splits and sequence parallelism.

The reference's tensor-parallel plan shards q/k/v by equal column chunks, which
needs the head count to divide by the degree (20 heads at tp=8 fails,
avgen/models/layers.py:496-504), and it has no working sequence-parallel
norms. Here each rank owns whole heads: ``head_partition(20, 8)`` is
``[3, 3, 3, 3, 2, 2, 2, 2]``. A rank keeps the q/k/v rows and out-projection
columns of its heads (self- and cross-attention) and a slice of the MLP's
hidden units, as plain local parameters.

Per block, the attention, cross-attention and MLP each enter and leave the
tensor-parallel region through one collective pair:

* without sequence parallelism the residual stream is replicated: entering is
  an identity whose backward all-reduces the input gradient, leaving is an
  all-reduce of the partial outputs (backward: identity);
* with sequence parallelism every rank holds ``L / tp`` tokens of the residual
  stream, so the norms, modulation and gated residuals run on local tokens:
  entering all-gathers the normalised tokens (backward: reduce-scatter),
  leaving reduce-scatters the partial outputs back to local tokens (backward:
  all-gather). Parameters that act on local tokens only (the block norms, the
  ``scale_shift_table``, the shared modulation rows and the text context feeding
  every rank's heads) have their gradients summed over the group.

With sequence parallelism and local attention the block runs as one fused
sm_100a node on its shards (the collectives sit between its kernels, see
:mod:`avgen_b200.models.fused`); without it the block runs module by module
through the enter / leave pairs above.

Checkpoints hold full tensors: each sharded weight's state-dict entry is
gathered from the ranks' (possibly uneven) slices on save and sliced on load.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

__all__ = ["HeadParallel", "apply_head_parallel", "head_partition", "tp_shard_group"]


def tp_shard_group(param: torch.Tensor) -> Any:
    """The tensor-parallel group whose ranks hold disjoint slices of ``param`` (None if replicated)."""
    return getattr(param, "_avgen_tp_group", None)


def head_partition(count: int, parts: int) -> list[int]:
    """``count`` units over ``parts`` ranks, the first ``count % parts`` ranks taking one more."""
    if parts < 1 or count < parts:
        raise ValueError(f"cannot split {count} heads / units over {parts} tensor-parallel ranks")
    base, extra = divmod(count, parts)
    return [base + (1 if r < extra else 0) for r in range(parts)]


def _span(sizes: list[int], rank: int) -> tuple[int, int]:
    start = sum(sizes[:rank])
    return start, sizes[rank]


# --------------------------------------------------------------------------- collectives with autograd
def _all_reduce(t: torch.Tensor, group: Any) -> torch.Tensor:
    t = t.contiguous().clone()
    dist.all_reduce(t, group=group)
    return t


def _gather_tokens(t: torch.Tensor, group: Any) -> torch.Tensor:
    world = dist.get_world_size(group)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.cat(parts, 1)


def _scatter_tokens_sum(t: torch.Tensor, group: Any) -> torch.Tensor:
    """Sum over ranks, keep this rank's token chunk (reduce-scatter along dim 1)."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if t.device.type == "cuda":
        chunks = [c.contiguous() for c in t.chunk(world, 1)]
        out = torch.empty_like(chunks[rank])
        dist.reduce_scatter(out, chunks, group=group)
        return out
    return _all_reduce(t, group).chunk(world, 1)[rank].contiguous()  # gloo: all-reduce, then slice


class _Enter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, sequence):  # noqa: ANN001, ANN205
        ctx.group, ctx.sequence = group, sequence
        return _gather_tokens(x, group) if sequence else x.view_as(x)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        if ctx.sequence:
            return _scatter_tokens_sum(g, ctx.group), None, None
        return _all_reduce(g, ctx.group), None, None


class _Leave(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, group, sequence):  # noqa: ANN001, ANN205
        ctx.group, ctx.sequence = group, sequence
        return _scatter_tokens_sum(y, group) if sequence else _all_reduce(y, group)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        if ctx.sequence:
            return _gather_tokens(g, ctx.group), None, None
        return g, None, None


class _Shared(torch.autograd.Function):
    """A replicated tensor feeding rank-local work: identity, gradients summed over ranks."""

    @staticmethod
    def forward(ctx, x, group):  # noqa: ANN001, ANN205
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return _all_reduce(g, ctx.group), None


class _SliceTokens(torch.autograd.Function):
    """Replicated -> this rank's token chunk (backward: all-gather the chunks' gradients)."""

    @staticmethod
    def forward(ctx, x, group):  # noqa: ANN001, ANN205
        ctx.group = group
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        return x.chunk(world, 1)[rank].contiguous()

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        return _gather_tokens(g, ctx.group), None


class _UnsliceTokens(torch.autograd.Function):
    """Token chunks -> the replicated sequence (backward: keep this rank's chunk)."""

    @staticmethod
    def forward(ctx, x, group):  # noqa: ANN001, ANN205
        ctx.group = group
        return _gather_tokens(x, group)

    @staticmethod
    def backward(ctx, g):  # noqa: ANN001, ANN205
        world, rank = dist.get_world_size(ctx.group), dist.get_rank(ctx.group)
        return g.chunk(world, 1)[rank].contiguous(), None


@dataclass(frozen=True)
class HeadParallel:
    """One tensor-parallel group's context, attached to the modules it shards."""

    group: Any
    rank: int
    world: int
    sequence_parallel: bool

    def enter(self, x: torch.Tensor) -> torch.Tensor:
        return _Enter.apply(x, self.group, self.sequence_parallel)

    def leave(self, y: torch.Tensor) -> torch.Tensor:
        return _Leave.apply(y, self.group, self.sequence_parallel)

    def shared(self, x: torch.Tensor) -> torch.Tensor:
        return _Shared.apply(x, self.group)

    def local_tokens(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[1] % self.world:
            raise ValueError(f"sequence parallelism needs the token count ({x.shape[1]}) divisible by tp={self.world}")
        return _SliceTokens.apply(x, self.group)

    def all_tokens(self, x: torch.Tensor) -> torch.Tensor:
        return _UnsliceTokens.apply(x, self.group)

    def token_slice(self, length: int) -> slice:
        chunk = length // self.world
        return slice(self.rank * chunk, (self.rank + 1) * chunk)


# --------------------------------------------------------------------------- sharding
def gather_slices(t: torch.Tensor, dim: int, sizes: list[int], group: Any) -> torch.Tensor:
    """Every rank's slice of a tensor split unevenly along ``dim`` (``sizes``, in rank
    order), concatenated into the full tensor on every rank (collective)."""
    biggest = max(sizes)
    pad = list(t.shape)
    pad[dim] = biggest
    padded = torch.zeros(pad, dtype=t.dtype, device=t.device)
    padded.narrow(dim, 0, t.shape[dim]).copy_(t)
    parts = [torch.empty_like(padded) for _ in sizes]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([part.narrow(dim, 0, n) for part, n in zip(parts, sizes)], dim)


def local_slice(t: torch.Tensor, dim: int, sizes: list[int], rank: int) -> torch.Tensor:
    """This rank's slice of a full tensor split along ``dim`` as ``sizes``."""
    start, length = _span(sizes, rank)
    return t.narrow(dim, start, length)


def _keep(linear: nn.Linear, dim: int, sizes: list[int], tp: HeadParallel) -> None:
    """Replace ``linear``'s weight (and bias along dim 0) by this rank's slice of ``sizes``
    (every rank's extent along ``dim``, the same list on every rank), and make its
    state-dict entries full tensors again (gathered on save, sliced on load)."""
    start, length = _span(sizes, tp.rank)
    full = sum(sizes)
    with torch.no_grad():
        weight = linear.weight.narrow(dim, start, length).detach().clone()
        linear.weight = nn.Parameter(weight, requires_grad=linear.weight.requires_grad)
        if linear.bias is not None and dim == 0:
            linear.bias = nn.Parameter(linear.bias.narrow(0, start, length).detach().clone(),
                                       requires_grad=linear.bias.requires_grad)
    if dim == 0:
        linear.out_features = length
    else:
        linear.in_features = length
    linear._avgen_tp_shard = (dim, list(sizes), full)  # type: ignore[attr-defined]
    # the parameters themselves carry their group: a global gradient norm sums their
    # squares over it (every rank holds a different slice), replicated ones count once
    linear.weight._avgen_tp_group = tp.group  # type: ignore[attr-defined]
    if linear.bias is not None and dim == 0:
        linear.bias._avgen_tp_group = tp.group  # type: ignore[attr-defined]

    def save_full(module: nn.Module, state: dict, prefix: str, _meta: Any) -> None:
        d, all_sizes, _ = module._avgen_tp_shard
        for name in ("weight", "bias"):
            key = prefix + name
            t = state.get(key)
            if t is None or (name == "bias" and d != 0):
                continue
            state[key] = gather_slices(t, d, all_sizes, tp.group)

    def load_local(state: dict, prefix: str, *_args: Any) -> None:
        d, all_sizes, full_size = linear._avgen_tp_shard
        for name in ("weight", "bias"):
            key = prefix + name
            t = state.get(key)
            if t is not None and t.dim() > d and t.shape[d] == full_size and (name == "weight" or d == 0):
                state[key] = local_slice(t, d, all_sizes, tp.rank)

    linear._register_state_dict_hook(save_full)
    linear._register_load_state_dict_pre_hook(load_local)


def _shard_attention(att: nn.Module, tp: HeadParallel) -> None:
    heads, kv, hd = att.num_heads, att.num_kv_heads, att.head_dim
    q_sizes = head_partition(heads, tp.world)
    if kv != heads:
        if kv % tp.world:
            raise ValueError(f"grouped-query attention with {kv} kv heads does not split over tp={tp.world}")
        kv_sizes = [kv // tp.world] * tp.world
        if any(q != (heads // kv) * k for q, k in zip(q_sizes, kv_sizes)):
            raise ValueError(f"{heads} query heads over {kv} kv heads cannot be split evenly by groups over "
                             f"tp={tp.world}")
    else:
        kv_sizes = q_sizes
    q_rows = [n * hd for n in q_sizes]
    kv_rows = [n * hd for n in kv_sizes]
    _keep(att.q_proj, 0, q_rows, tp)
    _keep(att.k_proj, 0, kv_rows, tp)
    _keep(att.v_proj, 0, kv_rows, tp)
    _keep(att.out_proj, 1, q_rows, tp)
    att.num_heads, att.num_kv_heads = q_sizes[tp.rank], kv_sizes[tp.rank]
    att.tp = tp
    # QK-norm weights are replicated but each rank applies them to its own heads only
    for norm in (getattr(att, "q_norm", None), getattr(att, "k_norm", None)):
        w = getattr(norm, "weight", None)
        if isinstance(w, nn.Parameter):
            w.register_hook(lambda g, _tp=tp: _all_reduce(g, _tp.group))


def _shard_mlp(ff: nn.Module, tp: HeadParallel) -> None:
    up = ff.up_proj
    hidden = up.out_features
    sizes = head_partition(hidden, tp.world)
    for name in ("gate_proj", "up_proj"):
        layer = getattr(ff, name, None)
        if layer is not None:
            _keep(layer, 0, sizes, tp)
    _keep(ff.down_proj, 1, sizes, tp)
    ff.tp = tp


def apply_head_parallel(model: nn.Module, mesh: Any, *, sequence_parallel: bool = False,
                        block_attribute: str = "blocks") -> HeadParallel:
    """Shard every DiT block of ``model`` by heads over the 1-D tensor-parallel ``mesh``."""
    from avgen_b200.models.blocks import DiTBlock

    group = mesh.get_group()
    tp = HeadParallel(group=group, rank=dist.get_rank(group), world=dist.get_world_size(group),
                      sequence_parallel=sequence_parallel)
    for block in getattr(model, block_attribute):
        if not isinstance(block, DiTBlock):
            raise TypeError(f"head-parallel sharding expects DiTBlocks; got {type(block).__name__}")
        _shard_attention(block.attention, tp)
        if block.cross_attention is not None:
            _shard_attention(block.cross_attention, tp)
        _shard_mlp(block.feed_forward, tp)
        block.tp = tp  # the fused block takes these shards when sequence parallel (models/fused.py)
        if sequence_parallel:  # these act on local tokens only: sum their gradients over the group
            for p in (block.attention_norm.weight, getattr(block.cross_norm, "weight", None),
                      block.ffn_norm.weight, block.scale_shift_table):
                if isinstance(p, nn.Parameter):
                    p.register_hook(lambda g, _tp=tp: _all_reduce(g, _tp.group))
    model.head_parallel = tp
    return tp
