"""Process-group lifecycle (avgen/parallel/env.py:54-318).

torchrun environment -> ``init_process_group`` with ``cpu:gloo,cuda:nccl`` (gloo
without CUDA), the NCCL flight recorder and async error handling switched on,
the local device bound (``device_id``), a 10 min collective timeout and a 30 min
rendezvous timeout (both overridable), ``collective_timeout`` to shorten them
temporarily (checkpoint I/O), and ``unwrap_model``.
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


def _env_int(name: str, default: int) -> int:
    raw = os.environ.get(name)
    if raw in (None, ""):
        return default
    try:
        return int(raw)
    except ValueError:
        raise ValueError(f"environment variable {name}={raw!r} is not an int") from None


def is_distributed_launch() -> bool:
    return "RANK" in os.environ and "WORLD_SIZE" in os.environ


def local_rank_device() -> torch.device:
    if not torch.cuda.is_available():
        return torch.device("cpu")
    return torch.device("cuda", _env_int("LOCAL_RANK", 0) % max(1, torch.cuda.device_count()))


def init_distributed(*, backend: str | None = None, timeout: timedelta = DEFAULT_TIMEOUT,
                     init_timeout: timedelta = DEFAULT_INIT_TIMEOUT, enable_flight_recorder: bool = True,
                     trace_buffer_size: int = 2000) -> DistributedEnv:
    """Initialise the default process group from torchrun's environment (no-op single-process)."""
    if not is_distributed_launch():
        return DistributedEnv(0, 0, 1, 1, "none", local_rank_device())
    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local = _env_int("LOCAL_RANK", 0)
    local_world = _env_int("LOCAL_WORLD_SIZE", 1)
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad RANK={rank} / WORLD_SIZE={world}")
    if enable_flight_recorder:
        os.environ.setdefault("TORCH_NCCL_TRACE_BUFFER_SIZE", str(trace_buffer_size))
        os.environ.setdefault("TORCH_NCCL_DUMP_ON_TIMEOUT", "1")
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    resolved = backend or ("cpu:gloo,cuda:nccl" if torch.cuda.is_available() else "gloo")
    if torch.cuda.is_available():
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
    else:
        device = torch.device("cpu")
    if not dist.is_initialized():
        os.environ["TORCH_DISTRIBUTED_STORE_TIMEOUT"] = str(int(init_timeout.total_seconds()))
        kwargs: dict[str, object] = {"backend": resolved, "rank": rank, "world_size": world, "timeout": timeout}
        if device.type == "cuda":
            kwargs["device_id"] = device
        dist.init_process_group(**kwargs)
    return DistributedEnv(rank, local, world, local_world, resolved, device)


def barrier(env: DistributedEnv | None = None) -> None:
    if env is not None and not env.is_distributed:
        return
    if not (dist.is_available() and dist.is_initialized()):
        return
    if env is not None and env.device.type == "cuda":
        dist.barrier(device_ids=[env.local_rank])
    else:
        dist.barrier()


def shutdown_distributed() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


def unwrap_model(model: nn.Module) -> nn.Module:
    """Strip compile / checkpoint / DDP wrappers."""
    current = model
    seen: set[int] = set()
    while id(current) not in seen:
        seen.add(id(current))
        for attr in ("_orig_mod", "_checkpoint_wrapped_module", "module"):
            inner = getattr(current, attr, None)
            if isinstance(inner, nn.Module):
                current = inner
                break
        else:
            break
    return current


@contextmanager
def collective_timeout(seconds: float) -> Iterator[None]:
    """Temporarily change the default group's collective timeout."""
    if not (dist.is_available() and dist.is_initialized()):
        yield
        return
    group = dist.distributed_c10d._get_default_group()
    try:
        dist.distributed_c10d._set_pg_timeout(timedelta(seconds=seconds), group)
        yield
    finally:
        dist.distributed_c10d._set_pg_timeout(DEFAULT_TIMEOUT, group)
