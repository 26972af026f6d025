"""Fake multi-rank worlds for planning without GPUs (avgen/simulate/world.py:30-280 API).

``fake_world`` opens PyTorch's ``fake`` process-group backend for one rank of
an N-rank world and builds the device mesh of a :class:`ParallelDims`, so
sharding plans can be applied to a meta-initialised model and inspected on
a CPU-only machine.
"""
from __future__ import annotations

import contextlib
import os
from collections.abc import Callable, Iterator
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
from torch import nn
from torch.distributed.device_mesh import DeviceMesh

from avgen_b200.parallel.dims import ParallelDims

__all__ = ["FakeWorld", "fake_tensors", "fake_world", "meta_init", "simulate_rank"]

_ENV = ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE")


@dataclass(slots=True)
class FakeWorld:
    dims: ParallelDims
    rank: int = 0
    device_type: str | None = None
    mesh: DeviceMesh | None = field(default=None, init=False)
    _entered: bool = field(default=False, init=False, repr=False)
    _saved: dict[str, str | None] = field(default_factory=dict, init=False, repr=False)

    def __post_init__(self) -> None:
        if not 0 <= self.rank < self.dims.world_size:
            raise ValueError(f"rank must be in [0, {self.dims.world_size}); got {self.rank!r}")
        if self.device_type is None:
            self.device_type = "cuda" if torch.cuda.is_available() else "cpu"

    def __enter__(self) -> FakeWorld:
        if dist.is_initialized():
            raise RuntimeError("a real process group is initialised; simulate in a fresh process")
        from torch.testing._internal.distributed.fake_pg import FakeStore

        values = (str(self.rank), str(self.dims.world_size), str(self.rank % 8), "8")
        for name, value in zip(_ENV, values):
            self._saved[name] = os.environ.get(name)
            os.environ[name] = value
        dist.init_process_group(backend="fake", store=FakeStore(), rank=self.rank, world_size=self.dims.world_size)
        self._entered = True
        self.mesh = self.dims.build_mesh(self.device_type)
        return self

    def __exit__(self, *_exc: object) -> None:
        if self._entered:
            with contextlib.suppress(Exception):
                dist.destroy_process_group()
            self._entered = False
        for name, value in self._saved.items():
            if value is None:
                os.environ.pop(name, None)
            else:
                os.environ[name] = value
        self._saved.clear()
        self.mesh = None

    @property
    def resolved_device_type(self) -> str:
        return self.device_type or "cpu"

    def require_mesh(self) -> DeviceMesh:
        if self.mesh is None:
            raise RuntimeError("use FakeWorld as a context manager")
        return self.mesh

    def describe(self) -> dict[str, Any]:
        mesh = self.require_mesh()
        names = tuple(mesh.mesh_dim_names or ())
        data_rank, data_world = self.dims.data_coordinates(mesh)
        seq, seqs = self.dims.sequence_coordinates(mesh)
        return {"world_size": self.dims.world_size, "rank": self.rank,
                "mesh_dims": {n: mesh[n].size() for n in names}, "mesh_order": list(names),
                "data_rank": data_rank, "data_world": data_world, "sequence_shard": seq, "sequence_shards": seqs,
                "dp_size": self.dims.dp_size, "model_shard_size": self.dims.model_shard_size}


@contextlib.contextmanager
def fake_world(dims: ParallelDims, *, rank: int = 0, device_type: str | None = None) -> Iterator[FakeWorld]:
    with FakeWorld(dims=dims, rank=rank, device_type=device_type) as world:
        yield world


@contextlib.contextmanager
def meta_init() -> Iterator[None]:
    with torch.device("meta"):
        yield


@contextlib.contextmanager
def fake_tensors(allow_fallback: bool = True) -> Iterator[Any]:
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode(allow_fallback_kernels=allow_fallback) as mode:
        yield mode


def simulate_rank(dims: ParallelDims, build: Callable[[], nn.Module],
                  apply_plan: Callable[[nn.Module, ParallelDims, DeviceMesh], nn.Module], *, rank: int = 0,
                  device_type: str | None = None) -> dict[str, Any]:
    """Apply ``apply_plan`` to a meta-built model in a fake world and report one rank's shard."""
    with fake_world(dims, rank=rank, device_type=device_type) as world:
        mesh = world.require_mesh()
        with meta_init():
            model = build()
        params = sum(p.numel() for p in model.parameters())
        model = apply_plan(model, dims, mesh)
        report = world.describe()
        report["global_parameters"] = params
        from avgen_b200.parallel.fsdp import summarize_sharding

        report.update(summarize_sharding(model))
        report["parameters_per_rank"] = report.pop("local_elements")
        per_rank = report["parameters_per_rank"]
        report["shard_efficiency"] = params / (per_rank * dims.model_shard_size) if per_rank else 0.0
        return report
