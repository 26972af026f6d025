"""Mesh-aware reductions, object collectives and gradient clipping.

Reductions run over the data mesh (``dp_cp``, never the whole world, so TP and
PP replicas are not double counted); clipping is DTensor- and PP-correct
(avgen/parallel/comm.py:51-245).
"""
from __future__ import annotations

from collections.abc import Iterable

from typing import Any

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh

from avgen_b200.parallel.dims import submesh

__all__ = ["all_gather_object", "all_reduce_max", "all_reduce_mean", "all_reduce_sum", "broadcast_object",
           "clip_grad_norm", "data_mesh", "gather_object", "global_grad_norm"]


def data_mesh(mesh: DeviceMesh | None) -> DeviceMesh | None:
    if mesh is None:
        return None
    for name in ("dp_cp", "dp_shard", "dp_replicate", "cp"):
        found = submesh(mesh, name)
        if found is not None:
            return found
    return None


def _live(mesh: DeviceMesh | None) -> bool:
    return mesh is not None and mesh.size() > 1 and dist.is_available() and dist.is_initialized()


def _reduce(value: torch.Tensor, mesh: DeviceMesh | None, op: dist.ReduceOp.RedOpType) -> torch.Tensor:
    if not _live(mesh):
        return value
    out = value.detach().clone()
    dist.all_reduce(out, op=op, group=mesh.get_group())
    return out


def all_reduce_sum(value: torch.Tensor, mesh: DeviceMesh | None) -> torch.Tensor:
    return _reduce(value, mesh, dist.ReduceOp.SUM)


def all_reduce_max(value: torch.Tensor, mesh: DeviceMesh | None) -> torch.Tensor:
    return _reduce(value, mesh, dist.ReduceOp.MAX)


def all_reduce_mean(value: torch.Tensor, mesh: DeviceMesh | None) -> torch.Tensor:
    if not _live(mesh):
        return value
    return all_reduce_sum(value, mesh) / mesh.size()


def clip_grad_norm(parameters: Iterable[torch.nn.Parameter], max_norm: float, *, pp_mesh: DeviceMesh | None = None,
                   foreach: bool = True, error_if_nonfinite: bool = False) -> torch.Tensor:
    """Clip by the global L2 norm (DTensor shards reduced, PP stages summed)."""
    params = [p for p in parameters if p.grad is not None]
    total = global_grad_norm(params, pp_mesh=pp_mesh, foreach=foreach, error_if_nonfinite=error_if_nonfinite)
    torch.nn.utils.clip_grads_with_norm_(params, max_norm, total, foreach=foreach)
    return total


def global_grad_norm(parameters: Iterable[torch.nn.Parameter], *, pp_mesh: DeviceMesh | None = None,
                     foreach: bool = True, error_if_nonfinite: bool = False) -> torch.Tensor:
    """The L2 norm of the whole model's gradient: DTensor shards reduced, head-parallel
    slices' squares summed over their group, pipeline stages' squares summed."""
    from torch.distributed.tensor import DTensor

    from avgen_b200.parallel.heads import tp_shard_group

    params = [p for p in parameters if p.grad is not None]
    replicated = [p.grad for p in params if tp_shard_group(p) is None]
    by_group: dict[Any, list[torch.Tensor]] = {}
    for p in params:
        if tp_shard_group(p) is not None:
            by_group.setdefault(tp_shard_group(p), []).append(p.grad)
    total = torch.nn.utils.get_total_norm(replicated, norm_type=2.0, error_if_nonfinite=error_if_nonfinite,
                                          foreach=foreach) if replicated else None
    if isinstance(total, DTensor):
        total = total.full_tensor()
    for group, grads in by_group.items():  # head-parallel slices: their squares sum over the group
        sq = torch.nn.utils.get_total_norm(grads, norm_type=2.0, foreach=foreach).pow(2)
        dist.all_reduce(sq, group=group)
        total = sq.sqrt() if total is None else (total.pow(2) + sq).sqrt()
    if total is None:
        total = torch.zeros((), device=params[0].grad.device if params else "cpu")
    if pp_mesh is not None and pp_mesh.size() > 1:
        sq = total.pow(2)
        dist.all_reduce(sq, op=dist.ReduceOp.SUM, group=pp_mesh.get_group())
        total = sq.sqrt()
    return total


def broadcast_object(obj: object, *, src: int = 0) -> object:
    if not (dist.is_available() and dist.is_initialized()):
        return obj
    payload = [obj if dist.get_rank() == src else None]
    dist.broadcast_object_list(payload, src=src)
    return payload[0]


def all_gather_object(obj: object) -> list[object]:
    if not (dist.is_available() and dist.is_initialized()):
        return [obj]
    out: list[object] = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def gather_object(obj: object, *, dst: int = 0) -> list[object] | None:
    if not (dist.is_available() and dist.is_initialized()):
        return [obj]
    out = [None] * dist.get_world_size() if dist.get_rank() == dst else None
    dist.gather_object(obj, out, dst=dst)
    return out
