"""Parallel topology: degrees, the fixed mesh order, flattened views.

Mesh dimensions are ordered ``(pp, dp_replicate, dp_shard, cp, tp)`` (outermost
to innermost, so tensor-parallel peers are adjacent ranks on NVSwitch) with the
flattened views ``dp_shard_cp`` (FSDP shard group), ``dp_cp`` (loss / metric
reductions) and ``hsdp`` (2-D replicate x shard). ``dp_shard=-1`` is inferred.
Same contract as avgen/parallel/dims.py:61-440.
"""
from __future__ import annotations

import os
import warnings
import weakref
from dataclasses import dataclass

import torch
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh

__all__ = ["MESH_DIM_ORDER", "ParallelDims", "submesh"]

MESH_DIM_ORDER: tuple[str, ...] = ("pp", "dp_replicate", "dp_shard", "cp", "tp")
_FLATTENED: weakref.WeakKeyDictionary = weakref.WeakKeyDictionary()


def submesh(mesh: DeviceMesh | None, name: str) -> DeviceMesh | None:
    """A named dimension or flattened view of ``mesh`` (``None`` if absent)."""
    if mesh is None:
        return None
    flat = _FLATTENED.get(mesh)
    if flat is not None and name in flat:
        return flat[name]
    if name in tuple(mesh.mesh_dim_names or ()):
        return mesh[name]
    return None


@dataclass(frozen=True, slots=True)
class ParallelDims:
    world_size: int
    dp_replicate: int = 1
    dp_shard: int = -1
    tensor: int = 1
    context: int = 1
    pipeline: int = 1
    enable_loss_parallel: bool = True

    def __post_init__(self) -> None:
        if isinstance(self.world_size, bool) or self.world_size < 1:
            raise ValueError(f"world_size must be positive; got {self.world_size!r}")
        for name in ("dp_replicate", "tensor", "context", "pipeline"):
            v = getattr(self, name)
            if isinstance(v, bool) or v < 1:
                raise ValueError(f"{name} must be >= 1; got {v!r}")
        if isinstance(self.dp_shard, bool) or (self.dp_shard < 1 and self.dp_shard != -1):
            raise ValueError(f"dp_shard must be >= 1 or -1; got {self.dp_shard!r}")
        others = self.dp_replicate * self.tensor * self.context * self.pipeline
        if self.dp_shard == -1:
            if self.world_size % others:
                raise ValueError(f"cannot infer dp_shard: world_size={self.world_size} is not divisible by "
                                 f"dp_replicate*tensor*context*pipeline={others}")
            object.__setattr__(self, "dp_shard", self.world_size // others)
        product = others * self.dp_shard
        if product != self.world_size:
            raise ValueError(f"parallelism degrees must multiply to world_size: dp_replicate={self.dp_replicate} * "
                             f"dp_shard={self.dp_shard} * tensor={self.tensor} * context={self.context} * "
                             f"pipeline={self.pipeline} = {product} != {self.world_size}")

    @property
    def dp_replicate_enabled(self) -> bool:
        return self.dp_replicate > 1

    @property
    def dp_shard_enabled(self) -> bool:
        return self.dp_shard > 1

    @property
    def dp_enabled(self) -> bool:
        return self.dp_replicate_enabled or self.dp_shard_enabled

    @property
    def tp_enabled(self) -> bool:
        return self.tensor > 1

    @property
    def cp_enabled(self) -> bool:
        return self.context > 1

    @property
    def pp_enabled(self) -> bool:
        return self.pipeline > 1

    @property
    def loss_parallel_enabled(self) -> bool:
        return self.tp_enabled and self.enable_loss_parallel

    @property
    def dp_size(self) -> int:
        return self.dp_replicate * self.dp_shard

    @property
    def sequence_shard_size(self) -> int:
        return self.context * self.tensor

    @property
    def model_shard_size(self) -> int:
        return self.dp_shard * self.context * self.tensor * self.pipeline

    def gradient_accumulation_for(self, *, global_batch_size: int, local_batch_size: int) -> int:
        den = self.dp_size * local_batch_size
        if global_batch_size % den:
            raise ValueError(f"global_batch_size={global_batch_size} must be divisible by dp_size*local_batch_size={den}")
        return global_batch_size // den

    @property
    def active_dims(self) -> tuple[tuple[str, int], ...]:
        deg = {"pp": self.pipeline, "dp_replicate": self.dp_replicate, "dp_shard": self.dp_shard, "cp": self.context,
               "tp": self.tensor}
        return tuple((n, deg[n]) for n in MESH_DIM_ORDER if deg[n] > 1)

    _active_dims = active_dims

    def build_mesh(self, device_type: str | None = None) -> DeviceMesh:
        """Build the device mesh over the active dimensions plus flattened views."""
        dev = device_type or ("cuda" if torch.cuda.is_available() else "cpu")
        active = self.active_dims
        if not active:
            raise RuntimeError("no parallelism dimension exceeds 1; run single-device without a mesh")
        names = tuple(n for n, _ in active)
        mesh = init_device_mesh(dev, tuple(s for _, s in active), mesh_dim_names=names)
        flat: dict[str, DeviceMesh] = {}
        shard = [n for n in ("dp_shard", "cp") if n in names]
        if len(shard) > 1:
            flat["dp_shard_cp"] = mesh[tuple(shard)]._flatten(mesh_dim_name="dp_shard_cp")
        data = [n for n in ("dp_replicate", "dp_shard", "cp") if n in names]
        if len(data) > 1:
            flat["dp_cp"] = mesh[tuple(data)]._flatten(mesh_dim_name="dp_cp")
        if "dp_replicate" in names and "dp_shard_cp" in flat:
            with warnings.catch_warnings():
                warnings.filterwarnings("ignore", message=".*flattened dim.*")
                flat["hsdp"] = mesh["dp_replicate", "dp_shard_cp"]
        elif "dp_replicate" in names and "dp_shard" in names:
            flat["hsdp"] = mesh["dp_replicate", "dp_shard"]
        if flat:
            _FLATTENED[mesh] = flat
        return mesh

    def data_coordinates(self, mesh: DeviceMesh | None) -> tuple[int, int]:
        """``(data_rank, data_world)``: CP and TP peers share a data rank."""
        if mesh is None:
            return (0, 1)
        names = tuple(mesh.mesh_dim_names or ())
        rank, world = 0, 1
        for name in ("dp_replicate", "dp_shard"):
            if name in names:
                m = mesh[name]
                rank = rank * m.size() + m.get_local_rank()
                world *= m.size()
        return rank, world

    def sequence_coordinates(self, mesh: DeviceMesh | None) -> tuple[int, int]:
        """``(cp_rank, cp_size)``."""
        if mesh is None or "cp" not in tuple(mesh.mesh_dim_names or ()):
            return (0, 1)
        cp = mesh["cp"]
        return cp.get_local_rank(), cp.size()

    def describe(self) -> str:
        parts = [f"world={self.world_size}"]
        for name, size in (("dp_replicate", self.dp_replicate), ("dp_shard", self.dp_shard), ("cp", self.context),
                           ("tp", self.tensor), ("pp", self.pipeline)):
            if size > 1:
                parts.append(f"{name}={size}")
        if len(parts) == 1:
            parts.append("single-device")
        return " ".join(parts)

    @classmethod
    def from_env(cls, **degrees: int | bool) -> ParallelDims:
        return cls(world_size=int(os.environ.get("WORLD_SIZE", "1")), **degrees)
