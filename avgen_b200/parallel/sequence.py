"""Sequence-parallel tensor parallelism: trainable column / row linears whose
token all-gather and reduce-scatter are fused with their GEMMs.

With sequence parallelism the activations between tensor-parallel regions are
sharded along tokens (each rank holds ``T / tp`` rows), as the reference's
``SequenceParallel`` norms arrange (avgen/parallel/tensor.py:112-128):

* :func:`sp_column_linear` — column-parallel projection of token-sharded input:
  ``y = all_gather_tokens(x) . W_local^T (+ b_local)``, every token, this rank's
  output features. Forward runs :class:`~avgen_b200.parallel.collective_gemm.
  AllGatherGemm` (the gather overlapped with the GEMM tile by tile); backward
  reduce-scatters ``dY . W_local`` over tokens with
  :class:`~avgen_b200.parallel.collective_gemm.GemmReduceScatter` and re-gathers
  ``x`` for the weight gradient.
* :func:`sp_row_linear` — row-parallel projection back to token shards:
  ``y = reduce_scatter_tokens(x . W_local^T) (+ b)``; backward gathers ``dY``
  inside the input-gradient GEMM.

Tokens travel in rank-major order: row ``r * T_local + i`` of a gathered
tensor is row ``i`` of rank ``r``'s shard. The symmetric buffers are pooled per
(group, shape) and shared by every layer, so a gathered tensor is valid only
until the pool's next call but one; each function uses what it gathers right
away. On CPU process groups the same functions run NCCL-free reference
collectives (``all_gather_into_tensor`` / ``reduce_scatter_tensor``) so the
autograd logic is tested with ``gloo``.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

__all__ = ["sp_column_linear", "sp_row_linear"]

_POOL: dict[tuple, Any] = {}


def _allgather(group: Any, rows: int, cols: int, device: torch.device) -> Any:
    from avgen_b200.parallel.collective_gemm import AllGatherGemm

    key = ("ag", id(group), rows, cols, device)
    if key not in _POOL:
        _POOL[key] = AllGatherGemm(group, rows, cols, device, operand="a")
    return _POOL[key]


def _reducescatter(group: Any, m: int, n: int, device: torch.device) -> Any:
    from avgen_b200.parallel.collective_gemm import GemmReduceScatter

    key = ("rs", id(group), m, n, device)
    if key not in _POOL:
        _POOL[key] = GemmReduceScatter(group, m, n, device)
    return _POOL[key]


def _gather_cpu(x: torch.Tensor, group: Any) -> torch.Tensor:
    out = torch.empty((dist.get_world_size(group) * x.shape[0], *x.shape[1:]), dtype=x.dtype)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _scatter_cpu(x: torch.Tensor, group: Any) -> torch.Tensor:
    out = torch.empty((x.shape[0] // dist.get_world_size(group), *x.shape[1:]), dtype=x.dtype)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.bfloat16).contiguous()


def _weight_grad(dy: torch.Tensor, x: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """``dy^T . x`` in fp32 through the atomic-epilogue GEMM, cast like the weight."""
    from avgen_b200.ops import kernels as K

    grad = torch.zeros(like.shape, device=dy.device, dtype=torch.float32)
    K.linear_dw(dy, x, grad)
    return grad.to(like.dtype)


class _ColumnSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, group):  # noqa: ANN001, ANN205
        ctx.group, ctx.has_bias, ctx.x_dtype = group, bias is not None, x.dtype
        ctx.save_for_backward(x, weight)
        if x.device.type != "cuda":
            full = _gather_cpu(x, group)
            return torch.nn.functional.linear(full, weight, bias)
        ag = _allgather(group, x.shape[0], x.shape[1], x.device)
        b = bias.detach().float().contiguous() if bias is not None else None
        y, _ = ag(_bf16(x), _bf16(weight), bias=b)
        return y

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        x, weight = ctx.saved_tensors
        group = ctx.group
        db = dy.sum(0) if ctx.has_bias else None
        if x.device.type != "cuda":
            dx = _scatter_cpu(dy @ weight, group)
            dw = dy.t() @ _gather_cpu(x, group)
            return dx, dw, db, None
        dy2 = _bf16(dy)
        world = dist.get_world_size(group)
        rs = _reducescatter(group, dy2.shape[0], weight.shape[1], dy.device)
        dx = rs(dy2, _bf16(weight), b_mn=True)  # rows of dY . W summed over ranks, this rank's tokens
        ag = _allgather(group, x.shape[0], x.shape[1], x.device)
        full, _ = ag.gather(_bf16(x))
        torch.cuda.current_stream(x.device).wait_stream(ag._copy)  # the whole input is here
        assert full.shape[0] == world * x.shape[0]
        dw = _weight_grad(dy2, full, weight)
        return dx.to(ctx.x_dtype), dw, (db.to(dy.dtype) if db is not None else None), None


class _RowSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, group):  # noqa: ANN001, ANN205
        ctx.group, ctx.has_bias, ctx.x_dtype = group, bias is not None, x.dtype
        ctx.save_for_backward(x, weight)
        if x.device.type != "cuda":
            y = _scatter_cpu(torch.nn.functional.linear(x, weight), group)
        else:
            rs = _reducescatter(group, x.shape[0], weight.shape[0], x.device)
            y = rs(_bf16(x), _bf16(weight))
        return y + bias if bias is not None else y

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        x, weight = ctx.saved_tensors
        group = ctx.group
        db = None
        if ctx.has_bias:  # the bias is replicated: its gradient sums every rank's tokens
            db = dy.sum(0).float()
            dist.all_reduce(db, group=group)
            db = db.to(dy.dtype)
        if x.device.type != "cuda":
            dy_full = _gather_cpu(dy, group)
            return dy_full @ weight, dy_full.t() @ x, db, None
        ag = _allgather(group, dy.shape[0], dy.shape[1], dy.device)
        dx, dy_full = ag(_bf16(dy), _bf16(weight), b_mn=True)  # dX = all_gather(dY) . W
        dw = _weight_grad(dy_full, _bf16(x), weight)
        return dx.to(ctx.x_dtype), dw, db, None


def sp_column_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, group: Any) -> torch.Tensor:
    """``all_gather_tokens(x) . weight^T + bias`` for token-sharded ``x [T_local, K]``
    and this rank's output rows ``weight [N_local, K]``; returns ``[T, N_local]``."""
    if x.dim() != 2:
        raise ValueError("sp_column_linear takes [tokens, features]; flatten the batch first")
    return _ColumnSP.apply(x, weight, bias, group)


def sp_row_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, group: Any) -> torch.Tensor:
    """``reduce_scatter_tokens(x . weight^T) + bias`` for ``x [T, K_local]`` and this
    rank's input columns ``weight [N, K_local]``; returns this rank's ``[T / tp, N]``."""
    if x.dim() != 2:
        raise ValueError("sp_row_linear takes [tokens, features]; flatten the batch first")
    if x.shape[0] % dist.get_world_size(group):
        raise ValueError("the token count must divide by the group size")
    return _RowSP.apply(x, weight, bias, group)
