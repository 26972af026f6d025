"""Symmetric peer memory over NVLink for the fused context-parallel paths.

Each rank of a process group allocates one buffer of the same size outside
PyTorch's caching allocator, exports it as a CUDA IPC handle, and maps every
peer's buffer into its own address space after the handles are exchanged over
the group (``all_gather_object``). Inside an NVSwitch node every GPU then
reads and writes any peer's buffer directly: kernels with loads/stores, copy
engines with ``cudaMemcpyAsync``, the front end with stream memory operations.

The device calls go through a backend object (the in-tree extension by
default) so the exchange logic runs on CPU ``gloo`` ranks in tests with a fake
backend.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

__all__ = ["SymmetricBuffer"]


def _backend() -> Any:
    from avgen_b200.ops._ext import load

    return load()


class SymmetricBuffer:
    """``nbytes`` of device memory on every rank of ``group``, mapped into every peer.

    ``ptrs[r]`` is rank r's buffer as an address valid on this rank's device.
    Collective: every rank of ``group`` constructs it with the same size, in the
    same order relative to other collectives on the group.
    """

    def __init__(self, nbytes: int, group: Any, device: torch.device, *, backend: Any = None) -> None:
        if nbytes <= 0:
            raise ValueError(f"nbytes must be positive; got {nbytes}")
        self.backend = backend if backend is not None else _backend()
        self.group = group
        self.nbytes = int(nbytes)
        self.device = torch.device(device)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        dev = self.device.index if self.device.index is not None else 0
        self._dev = dev
        self.local = self.backend.p2p_alloc(self.nbytes, dev)
        handle = self.backend.p2p_export(self.local)
        handles: list[Any] = [None] * self.world
        dist.all_gather_object(handles, (handle, self.nbytes), group=group)
        sizes = {n for _, n in handles}
        if sizes != {self.nbytes}:
            self.backend.p2p_free(self.local)
            raise RuntimeError(f"symmetric allocation sizes differ across ranks: {sorted(sizes)}")
        self.ptrs: list[int] = []
        for r, (h, _) in enumerate(handles):
            self.ptrs.append(self.local if r == self.rank else self.backend.p2p_open(h, dev))
        self._closed = False

    def view(self, rank: int, offset: int, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        """A tensor over ``rank``'s buffer starting ``offset`` bytes in (no copy, no ownership)."""
        numel = 1
        for s in shape:
            numel *= s
        item = torch.empty((), dtype=dtype).element_size()
        if offset < 0 or offset % 16 or offset + numel * item > self.nbytes:
            raise ValueError(f"view [{offset}, {offset + numel * item}) is outside the {self.nbytes}-byte buffer "
                             "or not 16-byte aligned")
        return self.backend.tensor_at(self.ptrs[rank] + offset, list(shape), dtype, self._dev)

    def address(self, rank: int, offset: int = 0) -> int:
        return self.ptrs[rank] + offset

    def close(self, barrier: Any = None) -> None:
        """Unmap the peers and free this rank's buffer. Callers synchronise first so
        that no peer still reads or writes it. With ``barrier`` (a callable run by
        every rank), this rank frees its buffer only after every peer has unmapped
        it, as CUDA IPC requires of an exported allocation."""
        if self._closed:
            return
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self.backend.p2p_close(p)
        if barrier is not None:
            barrier()
        self.backend.p2p_free(self.local)
        self._closed = True
