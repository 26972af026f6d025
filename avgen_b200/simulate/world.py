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

_GPUS_PER_NODE = 8


@contextlib.contextmanager
def _launcher_environ(rank: int, world: int) -> Iterator[None]:
    """Make the process look as if torchrun had started it as ``rank`` of ``world``
    (eight ranks per node), and put the previous environment back afterwards."""
    wanted = {"RANK": rank, "WORLD_SIZE": world, "LOCAL_RANK": rank % _GPUS_PER_NODE,
              "LOCAL_WORLD_SIZE": _GPUS_PER_NODE}
    previous = {name: os.environ.get(name) for name in wanted}
    os.environ.update({name: str(value) for name, value in wanted.items()})
    try:
        yield
    finally:
        for name, value in previous.items():
            if value is None:
                os.environ.pop(name, None)
            else:
                os.environ[name] = value


@contextlib.contextmanager
def _fake_process_group(rank: int, world: int) -> Iterator[None]:
    """PyTorch's ``fake`` backend: collectives return immediately and move no data."""
    if dist.is_initialized():
        raise RuntimeError("a real process group is initialised; simulate in a fresh process")
    from torch.testing._internal.distributed.fake_pg import FakeStore

    dist.init_process_group(backend="fake", store=FakeStore(), rank=rank, world_size=world)
    try:
        yield
    finally:
        with contextlib.suppress(Exception):
            dist.destroy_process_group()


@dataclass(slots=True)
class FakeWorld:
    """One rank of an N-rank world, for applying sharding plans on a CPU-only machine.

    Used as a context manager: entering installs the launcher environment and a
    fake process group and builds the mesh of ``dims``; leaving undoes both."""

    dims: ParallelDims
    rank: int = 0
    device_type: str | None = None
    mesh: DeviceMesh | None = field(default=None, init=False)
    _stack: contextlib.ExitStack | None = field(default=None, init=False, repr=False)

    def __post_init__(self) -> None:
        if not 0 <= self.rank < self.dims.world_size:
            raise ValueError(f"rank must be in [0, {self.dims.world_size}); got {self.rank!r}")
        self.device_type = self.device_type or ("cuda" if torch.cuda.is_available() else "cpu")

    def __enter__(self) -> FakeWorld:
        stack = contextlib.ExitStack()
        try:
            stack.enter_context(_launcher_environ(self.rank, self.dims.world_size))
            stack.enter_context(_fake_process_group(self.rank, self.dims.world_size))
            self.mesh = self.dims.build_mesh(self.device_type)
        except BaseException:
            stack.close()
            raise
        self._stack = stack
        return self

    def __exit__(self, *_exc: object) -> None:
        self.mesh = None
        stack, self._stack = self._stack, None
        if stack is not None:
            stack.close()

    @property
    def resolved_device_type(self) -> str:
        return self.device_type or "cpu"

    def require_mesh(self) -> DeviceMesh:
        if self.mesh is None:
            raise RuntimeError("use FakeWorld as a context manager")
        return self.mesh

    def describe(self) -> dict[str, Any]:
        """This rank's place in the mesh (sizes in mesh order, data and sequence coordinates)."""
        mesh = self.require_mesh()
        order = list(mesh.mesh_dim_names or ())
        coords = {"data": self.dims.data_coordinates(mesh), "sequence": self.dims.sequence_coordinates(mesh)}
        report: dict[str, Any] = {"world_size": self.dims.world_size, "rank": self.rank,
                                  "mesh_dims": {name: mesh[name].size() for name in order}, "mesh_order": order}
        report.update(data_rank=coords["data"][0], data_world=coords["data"][1],
                      sequence_shard=coords["sequence"][0], sequence_shards=coords["sequence"][1])
        report.update(dp_size=self.dims.dp_size, model_shard_size=self.dims.model_shard_size)
        return report


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
    """Apply ``apply_plan`` to a meta-built model in a fake world and report one rank's shard:
    its mesh coordinates, the parameters it holds and how evenly the plan divides them."""
    from avgen_b200.parallel.fsdp import summarize_sharding

    with fake_world(dims, rank=rank, device_type=device_type) as world:
        with meta_init():
            model = build()
        total = sum(p.numel() for p in model.parameters())
        sharding = summarize_sharding(apply_plan(model, dims, world.require_mesh()))
        held = sharding.pop("local_elements")
        ideal = held * dims.model_shard_size
        return {**world.describe(), "global_parameters": total, **sharding, "parameters_per_rank": held,
                "shard_efficiency": total / ideal if held else 0.0}
