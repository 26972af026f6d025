"""All-gather fused into the GEMM and GEMM followed by a peer-load
reduce-scatter, over real NVLink peer memory: 2 ranks, one GPU each. Results
must match the NCCL collective + GEMM computed on each rank, over repeated
calls (double-buffered symmetric buffers, rising epochs); the timings of both
paths are printed for the record."""
from __future__ import annotations

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


def _time(fn, iters: int = 10) -> float:  # noqa: ANN001
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def _worker(rank: int, world: int, port: int) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from avgen_b200.ops import kernels as K
        from avgen_b200.ops._ext import check_errors
        from avgen_b200.parallel.collective_gemm import AllGatherGemm, GemmReduceScatter

        g = torch.Generator().manual_seed(0)
        m, n, k = 8192, 2560, 2560
        rows = n // world
        w_all = (torch.randn(n, k, generator=g) * 0.05).bfloat16().to(dev)
        x = torch.randn(m, k, generator=g).bfloat16().to(dev)
        shard = w_all[rank * rows:(rank + 1) * rows].contiguous()
        ag = AllGatherGemm(dist.group.WORLD, rows, k, dev, operand="b")
        for _ in range(3):
            y, full = ag(shard, x)
        torch.cuda.synchronize()
        assert check_errors(dev) == 0, "a bounded wait timed out"
        assert torch.equal(full, w_all)
        ref = K.gemm(x, w_all)
        assert (y.float() - ref.float()).abs().max().item() <= 1e-2 * (1 + ref.float().abs().max().item())

        # sequence parallel: token rows gathered, column-parallel weight local
        xr = m // world
        sp = AllGatherGemm(dist.group.WORLD, xr, k, dev, operand="a")
        w_loc = w_all[: n // world].contiguous()
        y2, xf = sp(x[rank * xr:(rank + 1) * xr].contiguous(), w_loc)
        torch.cuda.synchronize()
        assert torch.equal(xf, x)
        ref2 = K.gemm(x, w_loc)
        assert (y2.float() - ref2.float()).abs().max().item() <= 1e-2 * (1 + ref2.float().abs().max().item())

        # row parallel: reduction axis split, rows of the sum scattered
        kc = k // world
        xs = x[:, rank * kc:(rank + 1) * kc].contiguous()
        ws = w_all[:, rank * kc:(rank + 1) * kc].contiguous()
        rs = GemmReduceScatter(dist.group.WORLD, m, n, dev)
        for _ in range(3):
            part = rs(xs, ws)
        torch.cuda.synchronize()
        full_sum = (x.float() @ w_all.float().t())[rank * (m // world):(rank + 1) * (m // world)]
        assert (part.float() - full_sum).abs().max().item() <= 2e-2 * (1 + full_sum.abs().max().item())
        assert check_errors(dev) == 0

        def nccl_ag() -> None:
            buf = torch.empty(n, k, device=dev, dtype=torch.bfloat16)
            dist.all_gather_into_tensor(buf, shard)
            K.gemm(x, buf)

        def nccl_rs() -> None:
            p = K.gemm(xs, ws)
            out = torch.empty(m // world, n, device=dev, dtype=torch.bfloat16)
            dist.reduce_scatter_tensor(out, p)

        times = torch.tensor([_time(lambda: ag(shard, x)), _time(nccl_ag), _time(lambda: K.gemm(x, w_all)),
                              _time(lambda: rs(xs, ws)), _time(nccl_rs)], device=dev)
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        if rank == 0:
            print(f"\n[collective-gemm world={world} M={m} N={n} K={k}] ms (max over ranks): "
                  f"fused AG+GEMM {times[0]:.3f}  NCCL AG + GEMM {times[1]:.3f}  GEMM alone {times[2]:.3f}  "
                  f"fused GEMM+RS {times[3]:.3f}  GEMM + NCCL RS {times[4]:.3f}", flush=True)
        for prim in (ag, sp, rs):  # no write ran past a symmetric buffer's bounds
            assert not prim.buf.check_guards(), f"rank {rank}: guard bytes changed"
        ag.close()
        sp.close()
        rs.close()
    except BaseException:
        leave_on_failure()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_collective_gemms_multi_gpu(world: int) -> None:
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _free_port()), nprocs=world, join=True)


def _sp_worker(rank: int, world: int, port: int) -> None:
    """A sequence-parallel MLP (column-parallel up with the token all-gather fused,
    row-parallel down with the reduce-scatter fused) against the unsharded MLP."""
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        import torch.nn.functional as F

        from avgen_b200.ops._ext import check_errors
        from avgen_b200.parallel.sequence import _POOL, sp_column_linear, sp_row_linear

        g = torch.Generator().manual_seed(1)
        t, k, f = 4096, 1024, 2048
        x = torch.randn(t, k, generator=g).to(dev)
        w1 = (torch.randn(f, k, generator=g) * 0.03).to(dev)
        w2 = (torch.randn(k, f, generator=g) * 0.03).to(dev)
        up = torch.randn(t, k, generator=g).to(dev)
        ref = [p.clone().requires_grad_() for p in (x, w1, w2)]
        y_ref = F.linear(F.gelu(F.linear(ref[0], ref[1])), ref[2])
        (y_ref * up).sum().backward()
        tl, fl = t // world, f // world
        rows, cols = slice(rank * tl, (rank + 1) * tl), slice(rank * fl, (rank + 1) * fl)
        xs = x[rows].clone().requires_grad_()
        w1s = w1[cols].clone().requires_grad_()
        w2s = w2[:, cols].contiguous().requires_grad_()
        for _ in range(2):  # repeated steps reuse the pooled symmetric buffers
            for p in (xs, w1s, w2s):
                p.grad = None
            y = sp_row_linear(F.gelu(sp_column_linear(xs, w1s, None, dist.group.WORLD).float()), w2s, None,
                              dist.group.WORLD)
            (y.float() * up[rows]).sum().backward()
        torch.cuda.synchronize()
        assert check_errors(dev) == 0

        def close(a: torch.Tensor, r: torch.Tensor, tol: float = 3e-2) -> None:
            err = (a.float() - r.float()).abs().max().item()
            assert err <= tol * (1 + r.abs().max().item()), f"rank {rank}: max err {err}"

        close(y, y_ref[rows])
        close(xs.grad, ref[0].grad[rows])
        close(w1s.grad, ref[1].grad[cols])
        close(w2s.grad, ref[2].grad[:, cols])
        for prim in _POOL.values():
            assert not prim.buf.check_guards()
            prim.close()
    except BaseException:
        leave_on_failure()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_sequence_parallel_mlp_multi_gpu() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_sp_worker, args=(2, _free_port()), nprocs=2, join=True)
