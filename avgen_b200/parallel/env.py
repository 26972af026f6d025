"""Process-group lifecycle for one process per GPU (public API of avgen/parallel/env.py:54-318).

The launcher's environment (torchrun: ``RANK``, ``LOCAL_RANK``, ``WORLD_SIZE``,
``LOCAL_WORLD_SIZE``) is parsed once into an immutable :class:`_Launch`
record that validates itself. :func:`init_distributed` then binds the process
to its GPU before the process group exists, so NCCL creates its communicator
eagerly on that device (``device_id``), and uses one group for both device
types (``cpu:gloo,cuda:nccl``: object collectives and CPU tensors go through
gloo, device tensors through NCCL over NVLink). NCCL's flight recorder and
asynchronous error handling are switched on through environment defaults a
user's own settings override. A hung collective raises after ``timeout``
(10 min by default); ``collective_timeout`` changes that bound for a region
(checkpoint I/O), and ``init_timeout`` bounds the rendezvous (30 min).
"""
from __future__ import annotations

import os
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist
from torch import nn

__all__ = ["DEFAULT_INIT_TIMEOUT", "DEFAULT_TIMEOUT", "DistributedEnv", "barrier", "collective_timeout",
           "init_distributed", "is_distributed_launch", "local_rank_device", "shutdown_distributed", "unwrap_model"]

DEFAULT_TIMEOUT = timedelta(minutes=10)
DEFAULT_INIT_TIMEOUT = timedelta(minutes=30)
# the steady-state collective timeout the default group was created with; a
# temporary bound (collective_timeout) is undone back to this value
_group_timeout: timedelta = DEFAULT_TIMEOUT

# NCCL debugging aids on by default (a user's own environment wins): keep the last
# collectives of every communicator, dump them when a collective times out, and
# tear the communicator down on an asynchronous error instead of hanging.
_NCCL_DEFAULTS = {"TORCH_NCCL_DUMP_ON_TIMEOUT": "1", "TORCH_NCCL_ASYNC_ERROR_HANDLING": "1"}
# Wrapper attributes that hold the wrapped module: torch.compile, activation
# checkpointing, DistributedDataParallel.
_WRAPPER_ATTRS = ("_orig_mod", "_checkpoint_wrapped_module", "module")


@dataclass(frozen=True, slots=True)
class DistributedEnv:
    rank: int
    local_rank: int
    world_size: int
    local_world_size: int
    backend: str
    device: torch.device

    @property
    def is_main(self) -> bool:
        return self.rank == 0

    @property
    def is_local_main(self) -> bool:
        return self.local_rank == 0

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1

    @property
    def num_nodes(self) -> int:
        return max(1, self.world_size // max(1, self.local_world_size))


@dataclass(frozen=True, slots=True)
class _Launch:
    """What the launcher told this process, checked for consistency."""

    rank: int = 0
    local_rank: int = 0
    world_size: int = 1
    local_world_size: int = 1

    @classmethod
    def from_environ(cls) -> _Launch:
        values = {}
        for field_name, var in (("rank", "RANK"), ("local_rank", "LOCAL_RANK"), ("world_size", "WORLD_SIZE"),
                                ("local_world_size", "LOCAL_WORLD_SIZE")):
            raw = os.environ.get(var, "")
            if raw == "":
                continue
            try:
                values[field_name] = int(raw)
            except ValueError:
                raise ValueError(f"environment variable {var}={raw!r} is not an int") from None
        launch = cls(**values)
        if launch.world_size < 1 or not 0 <= launch.rank < launch.world_size:
            raise ValueError(f"bad RANK={launch.rank} / WORLD_SIZE={launch.world_size}")
        return launch

    def device(self) -> torch.device:
        if not torch.cuda.is_available():
            return torch.device("cpu")
        return torch.device("cuda", self.local_rank % max(1, torch.cuda.device_count()))


def is_distributed_launch() -> bool:
    """Whether a multi-process launcher (torchrun) started this process."""
    return all(var in os.environ for var in ("RANK", "WORLD_SIZE"))


def local_rank_device() -> torch.device:
    """This process's GPU (``LOCAL_RANK`` modulo the visible devices), or the CPU."""
    return _Launch.from_environ().device()


def init_distributed(*, backend: str | None = None, timeout: timedelta = DEFAULT_TIMEOUT,
                     init_timeout: timedelta = DEFAULT_INIT_TIMEOUT, enable_flight_recorder: bool = True,
                     trace_buffer_size: int = 2000) -> DistributedEnv:
    """Create the default process group from the launcher's environment.

    Without a launcher this is a single-process run: nothing is initialised and
    the returned environment has backend ``"none"``. Calling it again after the
    group exists returns the same description without re-initialising."""
    if not is_distributed_launch():
        return DistributedEnv(0, 0, 1, 1, "none", local_rank_device())
    launch = _Launch.from_environ()
    if enable_flight_recorder:
        for var, value in {**_NCCL_DEFAULTS, "TORCH_NCCL_TRACE_BUFFER_SIZE": str(trace_buffer_size)}.items():
            os.environ.setdefault(var, value)
    device = launch.device()
    if device.type == "cuda":
        torch.cuda.set_device(device)
        device = torch.device("cuda", launch.local_rank)
    chosen = backend or ("cpu:gloo,cuda:nccl" if device.type == "cuda" else "gloo")
    if not dist.is_initialized():
        # the TCP store reads its own timeout from the environment at creation
        os.environ["TORCH_DISTRIBUTED_STORE_TIMEOUT"] = str(int(init_timeout.total_seconds()))
        dist.init_process_group(backend=chosen, rank=launch.rank, world_size=launch.world_size, timeout=timeout,
                                device_id=device if device.type == "cuda" else None)
        global _group_timeout
        _group_timeout = timeout
    return DistributedEnv(rank=launch.rank, local_rank=launch.local_rank, world_size=launch.world_size,
                          local_world_size=launch.local_world_size, backend=chosen, device=device)


def barrier(env: DistributedEnv | None = None) -> None:
    """Block until every rank arrives (no-op without a process group)."""
    if not (dist.is_available() and dist.is_initialized()) or (env is not None and not env.is_distributed):
        return
    on_gpu = env.device.type == "cuda" if env is not None else False
    dist.barrier(device_ids=[env.local_rank]) if on_gpu else dist.barrier()


def shutdown_distributed() -> None:
    """Destroy the default process group if one exists."""
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


def _inner(module: nn.Module) -> nn.Module | None:
    """The module a wrapper holds, or None when ``module`` wraps nothing."""
    return next((m for m in (getattr(module, a, None) for a in _WRAPPER_ATTRS) if isinstance(m, nn.Module)), None)


def unwrap_model(model: nn.Module) -> nn.Module:
    """Peel off compile / activation-checkpoint / DDP wrappers down to the model itself."""
    seen = {id(model)}
    inner = _inner(model)
    while inner is not None and id(inner) not in seen:
        model = inner
        seen.add(id(model))
        inner = _inner(model)
    return model


@contextmanager
def collective_timeout(seconds: float) -> Iterator[None]:
    """Run the enclosed block with the default group's collective timeout set to
    ``seconds``; afterwards the timeout the group was created with (the
    ``timeout`` given to :func:`init_distributed`) applies again."""
    if not (dist.is_available() and dist.is_initialized()):
        yield
        return
    c10d = dist.distributed_c10d
    default = c10d._get_default_group()
    c10d._set_pg_timeout(timedelta(seconds=seconds), default)
    try:
        yield
    finally:
        c10d._set_pg_timeout(_group_timeout, default)
