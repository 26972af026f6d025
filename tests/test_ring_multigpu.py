"""Fused ring attention over real NVLink peer memory: 2 and 4 ranks, one GPU
each, CUDA IPC buffers, copy-engine pulls (forward) and pushes (backward) with
front-end flag writes, and the flash kernel gating each remote slab on its flag.
Forward and backward must match attention over the whole sequence computed on
one device, over three repeated steps (epochs, double-buffered receive buffers)."""
from __future__ import annotations

import math
import os
import socket

import pytest
import torch
from multigpu_util import leave_on_failure

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, masked: bool) -> None:
    from datetime import timedelta

    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), LOCAL_WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from avgen_b200.ops import kernels as K
        from avgen_b200.ops._ext import check_errors
        from avgen_b200.parallel.context import RingAttention, ring_attention_available

        mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("cp",))
        assert ring_attention_available(mesh)
        b, h, hk, length, d = 1, 4, 2, 256, 128
        g = torch.Generator().manual_seed(0)
        q_all = torch.randn(world, b, h, length, d, generator=g).bfloat16()
        k_all = torch.randn(world, b, hk, length, d, generator=g).bfloat16()
        v_all = torch.randn(world, b, hk, length, d, generator=g).bfloat16()
        do_all = torch.randn(world, b, length, h, d, generator=g).bfloat16()
        kmask = None
        packed = None
        if masked:
            kmask = torch.ones(b, world * length, dtype=torch.bool)
            kmask[:, 200:330] = False
            packed = K.pack_key_mask(kmask.to(dev))
        impl = RingAttention(mesh, 0)
        scale = 1.0 / math.sqrt(d)
        for step in range(3):  # repeated calls exercise the epochs and buffer reuse
            kb, vb = impl.kv_out(b, hk, length, d, dev)
            kb.copy_(k_all[rank])
            vb.copy_(v_all[rank])
            q = q_all[rank].to(dev)
            out, lse, state = impl.forward(q, kb, vb, packed, scale)
            dq, dk, dv = impl.backward(q, kb, vb, out, do_all[rank].to(dev), lse, packed, scale, state)
            torch.cuda.synchronize()
            assert check_errors(dev) == 0, "a bounded wait timed out"
        assert not impl.kv.check_guards(), f"rank {rank}: K/V buffer guard bytes changed"
        for buf in RingAttention._recv_pool.values():  # pushed dK/dV partials stayed in bounds
            assert not buf.check_guards(), f"rank {rank}: receive buffer guard bytes changed"
        # reference on this device: the whole sequence
        kf = k_all.permute(1, 2, 0, 3, 4).reshape(b, hk, world * length, d).float().to(dev).requires_grad_()
        vf = v_all.permute(1, 2, 0, 3, 4).reshape(b, hk, world * length, d).float().to(dev).requires_grad_()
        qf = q_all[rank].float().to(dev).requires_grad_()
        rep = h // hk
        s = torch.einsum("bhqd,bhkd->bhqk", qf, kf.repeat_interleave(rep, 1)) * scale
        if kmask is not None:
            s = s.masked_fill(~kmask.to(dev)[:, None, None, :], float("-inf"))
        ref = torch.einsum("bhqk,bhkd->bhqd", s.softmax(-1), vf.repeat_interleave(rep, 1))
        ref.backward(do_all[rank].permute(0, 2, 1, 3).float().to(dev))
        # dK/dV of this rank's keys sum over every rank's queries
        gk = kf.grad.contiguous()
        gv = vf.grad.contiguous()
        dist.all_reduce(gk)
        dist.all_reduce(gv)
        lo, hi = rank * length, (rank + 1) * length

        def close(a: torch.Tensor, r: torch.Tensor, tol: float = 3e-2) -> None:
            err = (a.float() - r.float()).abs().max().item()
            assert err <= tol * (1 + r.abs().max().item()), f"rank {rank}: max err {err}"

        close(out.permute(0, 2, 1, 3), ref)
        close(dq, qf.grad)
        close(dk, gk[:, :, lo:hi])
        close(dv, gv[:, :, lo:hi])
    except BaseException:
        leave_on_failure()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.parametrize("world,masked", [(2, False), (2, True), (4, True)])
def test_ring_attention_multi_gpu(world: int, masked: bool) -> None:
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port(), masked), nprocs=world, join=True)
