"""Collectives fused with their GEMMs over NVLink peer memory, inside one node.

Two hot patterns of sharded training pair a GEMM with a collective:

* all-gather → GEMM: FSDP gathers a block's weight rows before the first GEMM
  that reads them (the reference's FSDP2 wrapping, avgen/parallel/fsdp.py:75-124),
  and sequence-parallel tensor parallelism gathers the token rows of the
  activations before the column-parallel projections (avgen/parallel/tensor.py:
  112-128). :class:`AllGatherGemm` runs the gather on the copy engines into a
  symmetric buffer while the tcgen05 GEMM is already computing: a tile that
  reads a peer's rows waits (bounded) on that chunk's arrival flag, and the
  tiles of this rank's own rows go first.
* GEMM → reduce-scatter: the row-parallel projections (attention output,
  MLP down) produce partial sums that the reference reduce-scatters with
  DTensor/NCCL. :class:`GemmReduceScatter` writes each rank's partial product
  into a symmetric buffer and sums this rank's rows straight out of every
  peer's buffer with one peer-load kernel, with no NCCL data movement.

Synchronisation is the same as the fused ring attention's: a one-word NCCL
all-reduce marks every rank's input as written, the copy stream writes arrival
flags with stream memory operations (GPU front end, no SM), and the only waits
on flags are the GEMM's own bounded waits. Buffers are double-buffered by call
parity so that one barrier per call also orders the next overwrite of a buffer
after every peer's reads of it.

On CPU process groups (``gloo``) both classes compute the same result with
``all_gather_into_tensor`` / ``reduce_scatter`` so the host logic is testable
without a GPU.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
import torch.nn.functional as F

__all__ = ["AllGatherGemm", "GemmReduceScatter"]


def _on_cuda(device: torch.device) -> bool:
    return device.type == "cuda"


class AllGatherGemm:
    """``gemm(all_gather(shard), other)`` with the gather overlapped tile by tile.

    ``shard`` is this rank's ``[rows, cols]`` block of a matrix whose row blocks
    are spread over ``group`` in rank order. ``operand="b"`` gathers the
    right-hand operand (FSDP: weight rows, ``y = x . W^T``); ``operand="a"``
    gathers the left-hand operand (sequence parallel: token rows,
    ``y = X . W_local^T``). Collective: every rank calls it in the same order
    with the same shapes.
    """

    def __init__(self, group: Any, rows: int, cols: int, device: torch.device | str, *, operand: str = "b") -> None:
        if operand not in ("a", "b"):
            raise ValueError(f"operand must be 'a' or 'b'; got {operand!r}")
        if cols % 8 or rows <= 0:
            raise ValueError(f"shard must be [rows > 0, cols % 8 == 0]; got [{rows}, {cols}]")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 32:
            raise ValueError("at most 32 ranks per fused all-gather")
        self.rows, self.cols, self.operand = int(rows), int(cols), operand
        self.device = torch.device(device)
        self.calls = 0
        self.epoch = 0
        self.buf: Any = None
        if _on_cuda(self.device):
            from avgen_b200.parallel.symmetric import SymmetricBuffer

            self._full_bytes = self.world * self.rows * self.cols * 2
            self.buf = SymmetricBuffer(2 * self._full_bytes, group, self.device)
            self.flags = torch.zeros(self.world, dtype=torch.int32, device=self.device)
            self._token = torch.zeros(1, dtype=torch.float32, device=self.device)
            self._copy = torch.cuda.Stream(device=self.device)

    def _full(self, rank: int, parity: int) -> torch.Tensor:
        return self.buf.view(rank, parity * self._full_bytes, (self.world * self.rows, self.cols), torch.bfloat16)

    def shard_out(self) -> torch.Tensor | None:
        """This rank's rows of the next call's gather buffer: a producer that writes
        its shard here saves the local copy."""
        if self.buf is None:
            return None
        return self._full(self.rank, self.calls % 2)[self.rank * self.rows:(self.rank + 1) * self.rows]

    def gather(self, shard: torch.Tensor, out: torch.Tensor | None = None) -> tuple[torch.Tensor, int]:
        """Start the gather of ``shard``; returns the (filling) full matrix and the epoch
        its arrival flags reach. Pulls run on the copy stream, nearest-next rank first.
        The rows land in the symmetric buffer, or in ``out`` (a contiguous local
        ``[world * rows, cols]`` bf16 tensor the caller keeps) when given; peers read
        this rank's rows from the symmetric buffer either way."""
        from avgen_b200.ops._ext import load

        if tuple(shard.shape) != (self.rows, self.cols):
            raise ValueError(f"shard must be [{self.rows}, {self.cols}]; got {list(shard.shape)}")
        if out is not None and (tuple(out.shape) != (self.world * self.rows, self.cols) or not out.is_contiguous()
                                or out.dtype != torch.bfloat16 or out.device != self.device):
            raise ValueError(f"out must be a contiguous bf16 [{self.world * self.rows}, {self.cols}] tensor on "
                             f"{self.device}")
        parity = self.calls % 2
        self.calls += 1
        sym = self._full(self.rank, parity)
        own = sym[self.rank * self.rows:(self.rank + 1) * self.rows]
        if own.data_ptr() != shard.data_ptr():
            own.copy_(shard)
        full = sym if out is None else out
        if out is not None:
            out[self.rank * self.rows:(self.rank + 1) * self.rows].copy_(shard)
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF or 1
        main = torch.cuda.current_stream(self.device)
        dist.all_reduce(self._token, group=self.group)  # every rank's shard is written
        self._copy.wait_stream(main)
        ext = load()
        chunk = self.rows * self.cols * 2
        flag0 = self.flags.data_ptr()
        with torch.cuda.stream(self._copy):
            for step in range(1, self.world):
                r = (self.rank + step) % self.world
                ext.p2p_copy(full.data_ptr() + r * chunk, self.buf.address(r, parity * self._full_bytes) + r * chunk,
                             chunk)
                ext.stream_write(flag0 + 4 * r, self.epoch)
        return full, self.epoch

    def __call__(self, shard: torch.Tensor, other: torch.Tensor, *, gathered_out: torch.Tensor | None = None,
                 **gemm_kwargs: Any) -> tuple[torch.Tensor, torch.Tensor]:
        """Returns ``(y, gathered)``. ``gathered`` is ``gathered_out`` when given, else a
        view of the symmetric buffer that stays valid until the call after next."""
        if not _on_cuda(self.device):
            full = torch.empty(self.world * self.rows, self.cols, dtype=shard.dtype)
            dist.all_gather_into_tensor(full, shard.contiguous(), group=self.group)
            y = F.linear(other, full) if self.operand == "b" else F.linear(full, other)
            if gathered_out is not None:
                gathered_out.copy_(full)
                full = gathered_out
            return y, full
        from avgen_b200.ops import kernels as K

        full, epoch = self.gather(shard, gathered_out)
        a, b = (other, full) if self.operand == "b" else (full, other)
        y = K.gemm(a, b, gate_flags=self.flags, gate_epoch=epoch, gate_operand=self.operand, gate_chunk=self.rows,
                   gate_rank=self.rank, **gemm_kwargs)
        torch.cuda.current_stream(self.device).wait_stream(self._copy)
        return y, full

    def close(self) -> None:
        if self.buf is not None:
            torch.cuda.synchronize(self.device)
            bar = lambda: dist.barrier(group=self.group, device_ids=[self.device.index])  # noqa: E731
            bar()
            self.buf.close(barrier=bar)
            self.buf = None


class GemmReduceScatter:
    """``reduce_scatter(x . w^T)`` over rows: rank r receives rows ``[r*M/world,
    (r+1)*M/world)`` of the sum over ranks of each rank's partial product.

    Row-parallel tensor parallelism: ``x`` is ``[M, K_local]`` (this rank's
    slice of the reduction axis) and ``w`` is ``[N, K_local]``. Each rank's GEMM
    writes its partial ``[M, N]`` (bf16, fp32 accumulation inside the GEMM)
    into a symmetric buffer; after one barrier a peer-load kernel sums this
    rank's rows from every peer's buffer in fp32.
    """

    def __init__(self, group: Any, m: int, n: int, device: torch.device | str) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if m % self.world or n % 8:
            raise ValueError(f"M must divide by the group size and N by 8; got M={m}, N={n}, world={self.world}")
        self.m, self.n = int(m), int(n)
        self.device = torch.device(device)
        self.calls = 0
        self.buf: Any = None
        if _on_cuda(self.device):
            from avgen_b200.parallel.symmetric import SymmetricBuffer

            self._bytes = self.m * self.n * 2
            self.buf = SymmetricBuffer(2 * self._bytes, group, self.device)
            self._token = torch.zeros(1, dtype=torch.float32, device=self.device)

    def __call__(self, x: torch.Tensor, w: torch.Tensor, **gemm_kwargs: Any) -> torch.Tensor:
        rows = self.m // self.world
        if not _on_cuda(self.device):
            part = F.linear(x, w)
            out = torch.empty(rows, self.n, dtype=part.dtype)
            dist.reduce_scatter_tensor(out, part.contiguous(), group=self.group)
            return out
        from avgen_b200.ops import kernels as K

        parity = self.calls % 2
        self.calls += 1
        mine = self.buf.view(self.rank, parity * self._bytes, (self.m, self.n), torch.bfloat16)
        K.gemm(x, w, out=mine, **gemm_kwargs)
        dist.all_reduce(self._token, group=self.group)  # every rank's partial product is complete
        lo = self.rank * rows * self.n * 2
        sources = [self.buf.view(r, parity * self._bytes + lo, (rows, self.n), torch.bfloat16)
                   for r in [(self.rank + s) % self.world for s in range(self.world)]]
        return K.slab_sum(sources, torch.empty(rows, self.n, device=self.device, dtype=torch.bfloat16))

    def close(self) -> None:
        if self.buf is not None:
            torch.cuda.synchronize(self.device)
            bar = lambda: dist.barrier(group=self.group, device_ids=[self.device.index])  # noqa: E731
            bar()
            self.buf.close(barrier=bar)
            self.buf = None
