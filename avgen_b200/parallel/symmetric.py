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

Canary guards: each allocation carries ``guard`` bytes before and after the
usable region, filled with a fixed pattern at allocation. Every writer into
peer memory here (copy engines, peer-store kernels) addresses the usable region
only, so :meth:`SymmetricBuffer.check_guards` finding a changed guard byte
means some write ran past its bounds; the multi-GPU tests call it after each
run. This stands in for a race/bounds sanitizer, which is not available on the
GPUs these tests run on.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

__all__ = ["GUARD_BYTES", "GUARD_PATTERN", "SymmetricBuffer"]

GUARD_BYTES = 4096
GUARD_PATTERN = 0xA5


def _backend() -> Any:
    from avgen_b200.ops._ext import load

    return load()


class SymmetricBuffer:
    """``nbytes`` of device memory on every rank of ``group``, mapped into every peer.

    ``ptrs[r]`` is rank r's buffer as an address valid on this rank's device.
    Collective: every rank of ``group`` constructs it with the same size, in the
    same order relative to other collectives on the group. ``guard`` canary
    bytes sit on both sides of each buffer (default :data:`GUARD_BYTES` when the
    backend can view device memory, else none).
    """

    def __init__(self, nbytes: int, group: Any, device: torch.device, *, backend: Any = None,
                 guard: int | None = None) -> None:
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
        if guard is None:
            guard = GUARD_BYTES if hasattr(self.backend, "tensor_at") else 0
        if guard < 0 or guard % 256:
            raise ValueError(f"guard must be a non-negative multiple of 256 bytes; got {guard}")
        self.guard = int(guard)
        self._base = self.backend.p2p_alloc(self.nbytes + 2 * self.guard, dev)
        self.local = self._base + self.guard
        if self.guard:
            for t in self._guards():
                t.fill_(GUARD_PATTERN)
        handle = self.backend.p2p_export(self._base)
        handles: list[Any] = [None] * self.world
        dist.all_gather_object(handles, (handle, self.nbytes), group=group)
        sizes = {n for _, n in handles}
        if sizes != {self.nbytes}:
            self.backend.p2p_free(self._base)
            raise RuntimeError(f"symmetric allocation sizes differ across ranks: {sorted(sizes)}")
        self.ptrs: list[int] = []
        for r, (h, _) in enumerate(handles):
            self.ptrs.append(self.local if r == self.rank else self.backend.p2p_open(h, dev) + self.guard)
        self._closed = False

    def _guards(self) -> list[torch.Tensor]:
        head = self.backend.tensor_at(self._base, [self.guard], torch.uint8, self._dev)
        tail = self.backend.tensor_at(self.local + self.nbytes, [self.guard], torch.uint8, self._dev)
        return [head, tail]

    def check_guards(self) -> list[tuple[str, int]]:
        """The guard bytes of this rank's allocation that no longer hold the pattern,
        as ``("head" | "tail", byte offset within the guard)``; empty when intact.
        Synchronises with the device."""
        bad: list[tuple[str, int]] = []
        if not self.guard or self._closed:
            return bad
        for name, t in zip(("head", "tail"), self._guards()):
            idx = torch.nonzero(t != GUARD_PATTERN).flatten().tolist()
            bad += [(name, int(i)) for i in idx[:16]]
        return bad

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
                self.backend.p2p_close(p - self.guard)
        if barrier is not None:
            barrier()
        self.backend.p2p_free(self._base)
        self._closed = True
