"""FSDP2's collectives over NVLink peer memory instead of NCCL.

The reference shards parameters with FSDP2, whose per-block parameter
all-gather and gradient reduce-scatter are NCCL kernels
(avgen/parallel/fsdp.py:123-135). On one NVSwitch node this module plugs two
communication objects into FSDP2's own hooks (``set_custom_all_gather`` /
``set_custom_reduce_scatter``), so sharding, DTensor parameters, DCP
checkpoints and resharding stay FSDP2's while the data moves as follows:

* :class:`PeerAllGather`: each rank copies its bf16 shard into its slot of a
  symmetric (CUDA IPC mapped) staging buffer, one one-word all-reduce marks
  every shard staged, and the copy engines pull every peer's shard straight
  into the gathered output over NVLink (nearest-next rank first). No SM and no
  NCCL data movement; FSDP2 issues it one block ahead on its all-gather stream,
  so it overlaps the previous block's compute.
* :class:`PeerReduceScatter`: FSDP2 writes the block's full fp32 gradient
  (its reduce-scatter input) directly into a symmetric buffer that this object
  hands out; one one-word all-reduce marks every rank's gradient written, and
  one pull-reduce kernel (``peer_reduce``) reads this rank's shard from every
  peer over NVLink, sums in fp32 and applies the data-parallel average in the
  same pass. FSDP2 runs it on its reduce-scatter stream right after the
  block's backward, overlapped with the backward of the blocks before it.

Both buffers are double-buffered. A slot is written again only after a later
call's one-word all-reduce, which every peer reaches after its pulls from that
slot completed (the pulls and the all-reduce are ordered on each rank's
stream), so no rank overwrites memory a peer is still reading.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
from torch.distributed.fsdp._fully_shard._fsdp_api import AllGather, ReduceScatter

__all__ = ["PeerAllGather", "PeerReduceScatter", "install_peer_collectives", "peer_collectives_available"]

_MIN_SLOT = 1 << 20


def _ext() -> Any:
    from avgen_b200.ops._ext import load

    return load()


def _count() -> None:
    from avgen_b200.ops import kernels as K

    K._count()


def peer_collectives_available(group: Any) -> bool:
    """Whether every rank of ``group`` is a CUDA device of this node (NVLink peer access)."""
    import os

    if not (dist.is_available() and dist.is_initialized() and torch.cuda.is_available()):
        return False
    if os.environ.get("AVGEN_FSDP_PEER", "1") == "0":
        return False
    if dist.get_backend(group) != "nccl":
        return False
    world = dist.get_world_size(group)
    local = int(os.environ.get("LOCAL_WORLD_SIZE", torch.cuda.device_count()))
    ranks = dist.get_process_group_ranks(group)
    return world <= 16 and len({r // max(1, local) for r in ranks}) == 1


class _Slots:
    """A symmetric buffer split into two equal slots, grown collectively on demand."""

    def __init__(self, group: Any, device: torch.device) -> None:
        self.group = group
        self.device = device
        self.buf: Any = None
        self.slot_bytes = 0
        self.token = torch.zeros(1, dtype=torch.float32, device=device)

    def ensure(self, nbytes: int) -> None:
        from avgen_b200.parallel.symmetric import SymmetricBuffer

        if nbytes <= self.slot_bytes:
            return
        # Every rank asks for the same size at the same call (FSDP2 pads shards evenly),
        # so the reallocation is collective. Drain the device first: peers may still
        # read the old buffer, and a barrier after the drain orders every rank's free.
        size = max(_MIN_SLOT, -(-nbytes // 4096) * 4096)
        if self.buf is not None:
            torch.cuda.synchronize(self.device)
            bar = lambda: dist.barrier(group=self.group, device_ids=[self.device.index])  # noqa: E731
            bar()
            self.buf.close(barrier=bar)
        self.buf = SymmetricBuffer(2 * size, self.group, self.device)
        self.slot_bytes = size

    def barrier(self) -> None:
        """One-word all-reduce on the current stream: every rank reached this point of its stream."""
        dist.all_reduce(self.token, group=self.group)

    def address(self, rank: int, slot: int, offset: int = 0) -> int:
        return self.buf.address(rank, slot * self.slot_bytes + offset)


class PeerAllGather(AllGather):
    """FSDP2 parameter all-gather: stage, one barrier, copy-engine pulls from every peer."""

    def __init__(self, group: Any, device: torch.device) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.slots = _Slots(group, device)
        self.calls = 0

    def allocate(self, size: Any, *, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        return torch.empty(size, dtype=dtype, device=device)

    def __call__(self, output_tensor: torch.Tensor, input_tensor: torch.Tensor, group: Any,
                 async_op: bool = False) -> None:
        del async_op  # the copies are ordered on the calling (all-gather) stream; FSDP2 waits on its event
        if group is not self.group and dist.get_process_group_ranks(group) != dist.get_process_group_ranks(self.group):
            raise ValueError("PeerAllGather was built for another process group")
        n = input_tensor.numel() * input_tensor.element_size()
        if output_tensor.numel() * output_tensor.element_size() != n * self.world:
            raise ValueError("all-gather output must hold world x input bytes")
        if not (input_tensor.is_contiguous() and output_tensor.is_contiguous()):
            raise ValueError("all-gather tensors must be contiguous")
        ext = _ext()
        self.slots.ensure(n)
        slot = self.calls % 2
        self.calls += 1
        staged = self.slots.buf.view(self.rank, slot * self.slots.slot_bytes, (n,), torch.uint8)
        staged.copy_(input_tensor.view(-1).view(torch.uint8))
        self.slots.barrier()  # every rank's shard is staged (and every pull of this slot's last use is done)
        out = output_tensor.data_ptr()
        mine = out + self.rank * n
        if input_tensor.data_ptr() != mine:
            ext.p2p_copy(mine, input_tensor.data_ptr(), n)
        for step in range(1, self.world):
            r = (self.rank + step) % self.world
            ext.p2p_copy(out + r * n, self.slots.address(r, slot), n)
        return None


class PeerReduceScatter(ReduceScatter):
    """FSDP2 gradient reduce-scatter: inputs live in symmetric memory; one barrier,
    then one pull-reduce kernel over NVLink per call."""

    def __init__(self, group: Any, device: torch.device) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.slots = _Slots(group, device)
        self.device = device
        self.calls = 0
        self._next_is_input = True
        self._input_slot: int | None = None
        self._free: list[torch.cuda.Event | None] = [None, None]
        self.norm_acc: torch.Tensor | None = None  # optional fp32 [1]: sum of squares of every reduced shard

    def allocate(self, size: Any, *, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        # FSDP2 asks for the input (world x shard) first, then for the output (shard).
        if not self._next_is_input:
            self._next_is_input = True
            return torch.empty(size, dtype=dtype, device=device)
        self._next_is_input = False
        numel = 1
        for s in size:
            numel *= int(s)
        item = torch.empty((), dtype=dtype).element_size()
        self.slots.ensure(numel * item)
        slot = self.calls % 2
        event = self._free[slot]
        if event is not None:  # every peer finished reading this slot's previous contents
            torch.cuda.current_stream(device).wait_event(event)
        self._input_slot = slot
        return self.slots.buf.view(self.rank, slot * self.slots.slot_bytes, (numel,), dtype)

    def __call__(self, output_tensor: torch.Tensor, input_tensor: torch.Tensor, group: Any, op: Any,
                 async_op: bool = False) -> None:
        del async_op
        if op == dist.ReduceOp.AVG:
            scale = 1.0 / self.world
        elif op == dist.ReduceOp.SUM:
            scale = 1.0
        else:
            raise NotImplementedError(f"PeerReduceScatter supports SUM and AVG, not {op}")
        slot = self.calls % 2
        if self._input_slot != slot:
            raise RuntimeError("reduce-scatter input was not allocated by this PeerReduceScatter")
        expected = self.slots.address(self.rank, slot)
        if input_tensor.data_ptr() != expected:
            raise RuntimeError("reduce-scatter input is not the symmetric slot handed out by allocate()")
        if input_tensor.dtype not in (torch.float32, torch.bfloat16) or output_tensor.dtype != torch.float32:
            raise TypeError("PeerReduceScatter reduces fp32 or bf16 gradients into an fp32 shard")
        self.calls += 1
        self._input_slot = None
        shard = output_tensor.numel()
        if input_tensor.numel() != shard * self.world:
            raise ValueError("reduce-scatter input must hold world x output elements")
        self.slots.barrier()  # every rank's gradient is in its slot; every pull from the other slot is done
        self._free[(slot + 1) % 2] = torch.cuda.current_stream(self.device).record_event()
        srcs = [self.slots.address(r, slot) for r in range(self.world)]
        _ext().peer_reduce(srcs, self.rank, self.rank * shard, output_tensor, input_tensor.dtype == torch.bfloat16,
                           scale, self.norm_acc)
        _count()
        return None


def install_peer_collectives(model: torch.nn.Module, mesh: Any) -> int:
    """Give every FSDP2 module of ``model`` the peer all-gather and reduce-scatter
    (one shared pair per process group). Returns how many modules got them, 0
    when the group does not qualify (not one node of CUDA ranks)."""
    from torch.distributed.fsdp import FSDPModule

    if mesh is None or mesh.ndim != 1:
        return 0  # HSDP (2-D) meshes keep NCCL
    group = mesh.get_group()
    if not peer_collectives_available(group):
        return 0
    device = torch.device("cuda", torch.cuda.current_device())
    gather = PeerAllGather(group, device)
    reduce = PeerReduceScatter(group, device)
    count = 0
    for module in model.modules():
        if isinstance(module, FSDPModule):
            module.set_custom_all_gather(gather)
            module.set_custom_reduce_scatter(reduce)
            count += 1
    model._avgen_peer_collectives = (gather, reduce)
    return count
