"""Context parallelism: contiguous sequence sharding and global attention over shards.

Sharding (avgen/parallel/context.py:58-229): the token axis is split into
contiguous equal shards (balanced because attention is bidirectional);
``pad_to_multiple`` makes padding explicit and masked; ``gather_stream`` /
``gather_tokens`` reassemble.

Unlike the reference, whose ``context_parallel_region`` is never entered (each
rank attends only within its shard), attention here is global:

* :class:`ContextParallelAttention` is the fused-block implementation on
  B200s: every rank's K/V shard is exchanged over NVLink and the local queries
  attend to the whole sequence with the tcgen05 flash kernels; backward
  reduce-scatters dK/dV back to their owners.
* :func:`cp_attention` is the eager / CPU path (gloo): K/V all-gathered with
  autograd, then the reference attention; it is the oracle for the fused path.
"""
from __future__ import annotations

from collections.abc import Iterator, Sequence
from contextlib import contextmanager, nullcontext
from dataclasses import replace
import weakref
from typing import Any

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh

from avgen_b200.core.tokens import TokenStream
from avgen_b200.telemetry.comm import comm_span, counter as comm_counter, enabled as comm_enabled

__all__ = ["ContextParallelAttention", "RingAttention", "context_parallel_region", "cp_attention", "gather_stream", "gather_tokens",
           "maybe_context_parallel", "pad_to_multiple", "shard_bounds", "shard_stream", "sharded_length"]


def sharded_length(total: int, shards: int) -> int:
    if total % shards:
        raise ValueError(f"sequence length {total} is not divisible by context-parallel degree {shards}; pad with "
                         "pad_to_multiple() at the data boundary so the padding is explicit and masked")
    return total // shards


def shard_bounds(total: int, shards: int, index: int) -> tuple[int, int]:
    local = sharded_length(total, shards)
    return index * local, (index + 1) * local


def pad_to_multiple(stream: TokenStream, multiple: int) -> TokenStream:
    """Pad the token axis with masked, unconditioned, zero tokens to a multiple."""
    if multiple < 1:
        raise ValueError(f"multiple must be positive; got {multiple!r}")
    rem = stream.length % multiple
    if rem == 0:
        return stream
    pad = multiple - rem
    b = stream.batch_size

    def padt(t: torch.Tensor) -> torch.Tensor:
        shape = list(t.shape)
        shape[1] = pad
        return torch.cat((t, torch.zeros(shape, dtype=t.dtype, device=t.device)), 1)

    noise = padt(stream.noise_level) if stream.per_token_noise else stream.noise_level
    values, index = stream.level_values, stream.level_index
    if stream.has_level_groups:  # padding tokens sit at level 0: give them a group of their own
        g = values.shape[1]
        values = torch.cat((values, torch.zeros((b, 1), dtype=values.dtype, device=values.device)), 1)
        index = torch.cat((index, torch.full((b, pad), g, dtype=index.dtype, device=index.device)), 1)
    return TokenStream(tokens=padt(stream.tokens), coords=padt(stream.coords), mask=padt(stream.mask),
                       noise_level=noise, layout=stream.layout, conditioned=padt(stream.conditioned),
                       level_values=values, level_index=index)


def _cp(mesh: DeviceMesh | None) -> tuple[int, int]:
    if mesh is None or mesh.size() == 1:
        return 0, 1
    return mesh.get_local_rank(), mesh.size()


def shard_stream(stream: TokenStream, mesh: DeviceMesh | None) -> TokenStream:
    """This rank's contiguous shard of a stream."""
    index, shards = _cp(mesh)
    if shards == 1:
        return stream
    lo, hi = shard_bounds(stream.length, shards, index)
    noise = stream.noise_level[:, lo:hi] if stream.per_token_noise else stream.noise_level
    index = stream.level_index[:, lo:hi] if stream.has_level_groups else stream.level_index
    return replace(stream, tokens=stream.tokens[:, lo:hi], coords=stream.coords[:, lo:hi], mask=stream.mask[:, lo:hi],
                   noise_level=noise, conditioned=stream.conditioned[:, lo:hi], level_index=index)


def _gather_dim1(t: torch.Tensor, mesh: DeviceMesh) -> torch.Tensor:
    parts = [torch.empty_like(t) for _ in range(mesh.size())]
    dist.all_gather(parts, t.contiguous(), group=mesh.get_group())
    return torch.cat(parts, 1)


def gather_stream(stream: TokenStream, mesh: DeviceMesh | None) -> TokenStream:
    if mesh is None or mesh.size() == 1 or not (dist.is_available() and dist.is_initialized()):
        return stream
    noise = _gather_dim1(stream.noise_level, mesh) if stream.per_token_noise else stream.noise_level
    index = _gather_dim1(stream.level_index, mesh) if stream.has_level_groups else stream.level_index
    return replace(stream, tokens=_gather_dim1(stream.tokens, mesh), coords=_gather_dim1(stream.coords, mesh),
                   mask=_gather_dim1(stream.mask, mesh), noise_level=noise,
                   conditioned=_gather_dim1(stream.conditioned, mesh), level_index=index)


def gather_tokens(tensor: torch.Tensor, mesh: DeviceMesh | None) -> torch.Tensor:
    if mesh is None or mesh.size() == 1 or not (dist.is_available() and dist.is_initialized()):
        return tensor
    return _gather_dim1(tensor, mesh)


class _AllGatherSeq(torch.autograd.Function):
    """All-gather along the sequence axis (dim 2 of [B, H, L, D]); backward reduce-scatters."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, group) -> torch.Tensor:  # noqa: ANN001, ANN205
        world = dist.get_world_size(group)
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous(), group=group)
        ctx.group = group
        ctx.world = world
        ctx.rank = dist.get_rank(group)
        return torch.cat(parts, 2)

    @staticmethod
    def backward(ctx, grad: torch.Tensor):  # noqa: ANN205
        chunks = [c.contiguous() for c in grad.chunk(ctx.world, 2)]
        out = torch.empty_like(chunks[0])
        if grad.device.type == "cpu":
            # gloo has no reduce_scatter: all-reduce then slice.
            full = grad.contiguous().clone()
            dist.all_reduce(full, group=ctx.group)
            out = full.chunk(ctx.world, 2)[ctx.rank].contiguous()
        else:
            dist.reduce_scatter(out, chunks, group=ctx.group)
        return out, None


def cp_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, mesh: DeviceMesh | None,
                 key_mask: torch.Tensor | None = None, scale: float | None = None) -> torch.Tensor:
    """Global attention for sequence-sharded q/k/v ``[B, H, L_local, D]`` (returns ``[B, H, L_local, D]``).

    ``key_mask`` is the *global* ``(B, L_global)`` key validity (or ``None``).
    """
    from avgen_b200.models.attention import attention

    if mesh is None or mesh.size() == 1:
        return attention(q, k, v, key_mask=key_mask, scale=scale)
    group = mesh.get_group()
    kf = _AllGatherSeq.apply(k, group)
    vf = _AllGatherSeq.apply(v, group)
    return attention(q, kf, vf, key_mask=key_mask, scale=scale)


class ContextParallelAttention:
    """Fused-block self-attention over a context-parallel group.

    Forward exchanges K/V shards over NVLink (NCCL all-gather into one
    ``[B, Hk, L_global, D]`` buffer) and runs the tcgen05 flash kernel with the
    local queries against the whole sequence; backward runs the flash backward
    against the same buffer and reduce-scatters dK/dV to their owners.
    """

    def __init__(self, mesh: DeviceMesh) -> None:
        self.mesh = mesh
        self.group = mesh.get_group()
        self.world = mesh.size()

    def _gather(self, t: torch.Tensor) -> torch.Tensor:
        b, h, length, d = t.shape
        # rank-major rows, dim 0 a multiple of the input's (the layout every backend accepts)
        buf = torch.empty((self.world * b, h, length, d), device=t.device, dtype=t.dtype)
        dist.all_gather_into_tensor(buf, t.contiguous(), group=self.group)
        return buf.view(self.world, b, h, length, d).permute(1, 2, 0, 3, 4).reshape(b, h, self.world * length, d)

    def forward(self, q, k, v, kmask, scale):  # noqa: ANN001, ANN201
        from avgen_b200.ops import kernels as K

        kf = self._gather(k)
        vf = self._gather(v)
        out, lse = K.attention_fwd(q, kf, vf, kmask=kmask, scale=scale)
        return out, lse, (kf, vf)

    def backward(self, q, k, v, o, do, lse, kmask, scale, state):  # noqa: ANN001, ANN201
        from avgen_b200.ops import kernels as K

        kf, vf = state
        dq, dkf, dvf = K.attention_bwd(q, kf, vf, o, do, lse, kmask=kmask, scale=scale)
        b, h, length, d = k.shape

        def scatter(full: torch.Tensor) -> torch.Tensor:
            parts = full.view(b, h, self.world, length, d).permute(2, 0, 1, 3, 4).reshape(self.world * b, h, length, d)
            out = torch.empty((b, h, length, d), device=full.device, dtype=full.dtype)
            dist.reduce_scatter_tensor(out, parts, group=self.group)
            return out

        return dq, scatter(dkf), scatter(dvf)


_RING_INSTANCES: "weakref.WeakSet[RingAttention]" = weakref.WeakSet()


def ring_buffers_pending(b: int, hk: int, length: int, d: int) -> int:
    """Bytes of ring K/V buffers that live :class:`RingAttention` instances have yet to
    allocate for this shape (they allocate lazily, on their block's first forward)."""
    total = 0
    for inst in list(_RING_INSTANCES):
        shape = (inst.world, b, hk, length, d)
        if inst.shape != shape and RingAttention.supported((b, hk, length, d)):
            total += 2 * inst.world * b * hk * length * d * 2
    return total


class RingAttention:
    """Fused context-parallel self-attention over NVLink peer memory, for one DiT block.

    Every rank keeps, per block, a persistent symmetric buffer holding K and V
    of the whole sequence in the ring layout ``[world, B, Hk, L_local, D]``
    (slab r = rank r's keys), mapped into every peer with CUDA IPC. Forward:

    1. the block's QK-norm + RoPE kernel writes this rank's K/V straight into
       its own slab (:meth:`kv_out`);
    2. a one-word all-reduce over the CP group marks every rank's slab as
       written (the only synchronisation; the streams never wait on flags);
    3. a copy stream pulls each peer's slab over NVLink with the copy engines,
       nearest-next rank first, and after each slab writes ``arrived[r]`` with a
       stream memory operation (GPU front end, no SM);
    4. meanwhile the tcgen05 flash kernel runs the local queries against the
       local slab first and gates each remote slab on ``arrived[r]`` with a
       bounded wait, so the transfer of slab r overlaps the softmax/MMA work on
       the slabs before it.

    Backward runs the one-pass flash backward on the same buffer, launched once
    per slab with the remote slabs first and this rank's own slab last. As each
    remote slab's partial dK/dV completes, the copy engines push it into the
    owner's receive buffer (one per CP group, double-buffered across
    backward calls) while the next slab computes; one word all-reduce then
    marks every push landed and a summing kernel forms this rank's dK/dV from
    its own partial and the pushed ones. That barrier also orders the next
    step's overwrite of a K/V slab after every peer's copy of it.
    """

    def __init__(self, mesh: DeviceMesh, index: int) -> None:
        self.mesh = mesh
        self.group = mesh.get_group()
        self.world = mesh.size()
        self.rank = mesh.get_local_rank()
        self.index = index
        self.epoch = 0
        self.kv: Any = None      # SymmetricBuffer: K then V, ring layout
        self.flags: torch.Tensor | None = None  # int32 arrived[world], written by this rank's copy stream
        self.shape: tuple[int, ...] | None = None
        self._token: torch.Tensor | None = None
        self._copy_stream: torch.cuda.Stream | None = None
        self._nccl = ContextParallelAttention(mesh)  # shapes the ring kernels do not take
        _RING_INSTANCES.add(self)

    @staticmethod
    def supported(k_shape: tuple[int, ...]) -> bool:
        return k_shape[2] % 128 == 0 and k_shape[3] == 128

    def _ensure(self, b: int, hk: int, length: int, d: int, device: torch.device) -> None:
        from avgen_b200.parallel.symmetric import SymmetricBuffer

        shape = (self.world, b, hk, length, d)
        if self.shape == shape:
            return
        if self.kv is not None:  # shape changed: every rank reallocates at the same call
            torch.cuda.synchronize(device)
            bar = lambda: dist.barrier(group=self.group, device_ids=[device.index])  # noqa: E731
            bar()
            self.kv.close(barrier=bar)
        self.kv = SymmetricBuffer(2 * self.world * b * hk * length * d * 2, self.group, device)
        self.flags = torch.zeros(self.world, dtype=torch.int32, device=device)
        self._token = torch.zeros(1, dtype=torch.float32, device=device)
        self._copy_stream = torch.cuda.Stream(device=device)
        self.shape = shape
        self.epoch = 0

    def _slabs(self, rank: int) -> tuple[torch.Tensor, torch.Tensor]:
        assert self.shape is not None
        half = self.kv.nbytes // 2
        return (self.kv.view(rank, 0, self.shape, torch.bfloat16), self.kv.view(rank, half, self.shape, torch.bfloat16))

    def kv_out(self, b: int, hk: int, length: int, d: int, device: torch.device,
               ) -> tuple[torch.Tensor, torch.Tensor] | None:
        """This rank's slabs, for the QK-norm + RoPE kernel to write K and V into."""
        if not self.supported((b, hk, length, d)):
            return None
        self._ensure(b, hk, length, d, device)
        k_all, v_all = self._slabs(self.rank)
        return k_all[self.rank], v_all[self.rank]

    def forward(self, q, k, v, kmask, scale):  # noqa: ANN001, ANN201
        from avgen_b200.ops import kernels as K
        from avgen_b200.ops._ext import load

        if not self.supported(tuple(k.shape)):
            return self._nccl.forward(q, k, v, kmask, scale)
        b, hk, length, d = k.shape
        self._ensure(b, hk, length, d, k.device)
        ext = load()
        k_all, v_all = self._slabs(self.rank)
        if k.data_ptr() != k_all[self.rank].data_ptr():
            k_all[self.rank].copy_(k)
        if v.data_ptr() != v_all[self.rank].data_ptr():
            v_all[self.rank].copy_(v)
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF or 1
        epoch = self.epoch
        main = torch.cuda.current_stream(k.device)
        assert self._token is not None and self.flags is not None
        with comm_span("ring_ready_barrier"):
            dist.all_reduce(self._token, group=self.group)  # every rank's slab is written
        copy = self._copy_stream
        assert copy is not None
        copy.wait_stream(main)
        slab_bytes = k_all[0].numel() * k_all.element_size()
        flag0 = self.flags.data_ptr()
        with torch.cuda.stream(copy):
            for step in range(1, self.world):
                r = (self.rank + step) % self.world
                pk, pv = self._slabs(r)
                ext.p2p_copy(k_all[r].data_ptr(), pk[r].data_ptr(), slab_bytes)
                ext.p2p_copy(v_all[r].data_ptr(), pv[r].data_ptr(), slab_bytes)
                ext.stream_write(flag0 + 4 * r, epoch)
        wait = None
        if comm_enabled():
            sms = torch.cuda.get_device_properties(q.device).multi_processor_count
            wait = comm_counter("ring_kv_wait", q.device, sms)
        out, lse = K.attention_fwd(q, k_all, v_all, kmask=kmask, scale=scale, ring_rank=self.rank,
                                   ring_flags=self.flags, ring_epoch=epoch, ring_wait=wait)
        with comm_span("ring_copy_tail"):
            main.wait_stream(copy)
        return out, lse, (k_all, v_all)

    # receive buffers for dK/dV partials pushed by peers: one pair per (group, shape),
    # shared by every block, double-buffered by backward parity
    _recv_pool: dict[tuple[int, tuple[int, ...]], Any] = {}

    def _recv(self, device: torch.device) -> Any:
        from avgen_b200.parallel.symmetric import SymmetricBuffer

        assert self.shape is not None
        key = (id(self.group), self.shape)
        buf = RingAttention._recv_pool.get(key)
        if buf is None:
            n = 1
            for s_ in self.shape:
                n *= s_
            buf = SymmetricBuffer(2 * 2 * n * 2, self.group, device)  # parity x (dK, dV) x ring layout, bf16
            RingAttention._recv_pool[key] = buf
        return buf

    def backward(self, q, k, v, o, do, lse, kmask, scale, state):  # noqa: ANN001, ANN201
        from avgen_b200.ops import kernels as K
        from avgen_b200.ops._ext import load

        if not isinstance(state, tuple) or state[0].dim() != 5:
            return self._nccl.backward(q, k, v, o, do, lse, kmask, scale, state)
        k_all, v_all = state
        ext = load()
        recv = self._recv(q.device)
        assert self.shape is not None and self._copy_stream is not None and self._token is not None
        parity = RingAttention._bwd_calls % 2
        RingAttention._bwd_calls += 1
        part = recv.nbytes // 4  # bytes of one ring-layout tensor
        slab = part // self.world

        def base(rank: int, which: int) -> int:  # which: 0 = dK, 1 = dV
            return recv.address(rank, (2 * parity + which) * part)

        main = torch.cuda.current_stream(q.device)
        copy = self._copy_stream

        def push(r: int, dk_all: torch.Tensor, dv_all: torch.Tensor) -> None:
            if r == self.rank:
                return
            copy.wait_stream(main)  # slab r's partials are complete
            with torch.cuda.stream(copy):
                ext.p2p_copy(base(r, 0) + self.rank * slab, dk_all[r].data_ptr(), slab)
                ext.p2p_copy(base(r, 1) + self.rank * slab, dv_all[r].data_ptr(), slab)

        order = [(self.rank + s_) % self.world for s_ in range(1, self.world)] + [self.rank]
        dq, dk_all, dv_all = K.attention_bwd_slabs(q, k_all, v_all, o, do, lse, order=order, kmask=kmask,
                                                   scale=scale, on_slab=push)
        with comm_span("ring_dkdv_barrier"):
            main.wait_stream(copy)
            dist.all_reduce(self._token, group=self.group)  # every peer's pushes into this rank have landed
        shape = self.shape[1:]
        sources_k = [dk_all[self.rank]] + [recv.view(self.rank, (2 * parity) * part + s_ * slab, shape, torch.bfloat16)
                                           for s_ in range(self.world) if s_ != self.rank]
        sources_v = [dv_all[self.rank]] + [recv.view(self.rank, (2 * parity + 1) * part + s_ * slab, shape,
                                                     torch.bfloat16) for s_ in range(self.world) if s_ != self.rank]
        with comm_span("ring_dkdv_sum"):
            dk = K.slab_sum(sources_k, torch.empty(shape, device=q.device, dtype=torch.bfloat16))
            dv = K.slab_sum(sources_v, torch.empty(shape, device=q.device, dtype=torch.bfloat16))
        return dq, dk, dv

    _bwd_calls = 0


@contextmanager
def context_parallel_region(mesh: DeviceMesh | None, *, buffers: Sequence[torch.Tensor] | None = None,
                            buffer_seq_dims: Sequence[int] | None = None) -> Iterator[None]:
    """Compatibility region: attention in this framework is always global under CP,
    so entering the region only validates its arguments."""
    if buffers is not None and buffer_seq_dims is not None and len(buffers) != len(buffer_seq_dims):
        raise ValueError("buffers and buffer_seq_dims must have the same length")
    del mesh
    yield


def maybe_context_parallel(mesh: DeviceMesh | None, **kwargs: object):  # noqa: ANN201
    if mesh is None or mesh.size() == 1:
        return nullcontext()
    return context_parallel_region(mesh, **kwargs)


def ring_attention_available(mesh: DeviceMesh | None) -> bool:
    """The fused NVLink ring needs CUDA ranks in one node with peer access to each other."""
    import os

    if mesh is None or mesh.size() == 1 or not torch.cuda.is_available():
        return False
    if os.environ.get("AVGEN_CP_RING", "1") == "0":
        return False
    if mesh.device_type != "cuda":
        return False
    local = torch.cuda.device_count()
    ranks = mesh.mesh.flatten().tolist()
    world_local = int(os.environ.get("LOCAL_WORLD_SIZE", local))
    # every rank of the group on this node (same node index)
    nodes = {r // max(1, world_local) for r in ranks}
    return len(nodes) == 1


def apply_context_parallel(model: torch.nn.Module, mesh: DeviceMesh | None, *, ring: bool | None = None,
                           ) -> torch.nn.Module:
    """Make every self-attention of ``model`` global over the CP group ``mesh``.

    Fused DiT blocks get :class:`RingAttention` (one per block: K/V exchanged
    over NVLink peer memory inside the attention kernel's schedule) when the
    group lives on one NVSwitch node, else :class:`ContextParallelAttention`
    (NCCL all-gather / reduce-scatter). Eager ``SelfAttention`` modules get the
    all-gather attention; the model gathers key masks across shards.
    """
    if mesh is None or mesh.size() == 1:
        return model
    from avgen_b200.models.blocks import DiTBlock
    from avgen_b200.models.layers import SelfAttention

    use_ring = ring_attention_available(mesh) if ring is None else ring
    shared = ContextParallelAttention(mesh)
    count = 0
    for module in model.modules():
        if isinstance(module, DiTBlock):
            module.attention_impl = RingAttention(mesh, count) if use_ring else shared
            count += 1
        if isinstance(module, SelfAttention):
            module.cp_mesh = mesh
    model.cp_mesh = mesh
    # text-refiner self-attention runs on replicated text tokens: keep it local (a
    # pipeline stage without the embedding holds no refiner)
    for refiner in getattr(model, "text_refiner", None) or []:
        refiner.attention.cp_mesh = None
    return model


__all__ += ["apply_context_parallel", "ring_attention_available"]
