"""Device-timed microbenchmarks of the sm_100a kernels.

    python -m avgen_b200.ops.bench attention --L 16384 --H 20 [--bwd split]
    python -m avgen_b200.ops.bench gemm --m 16384 --n 7680 --k 2560
    python -m avgen_b200.ops.bench gemm --m 16384 --n 7680 --k 2560 --gated 4   # all-gather gating on, flags set
    python -m avgen_b200.ops.bench attention --L 4096 --H 37 --once   # one call each (for ncu -k/-c)
    python -m avgen_b200.ops.bench trace --L 16384 --H 20 --pass bwd   # SM-clock timeline of CTA 0
    python -m avgen_b200.ops.bench ring --L 16384 --world 4          # one CP rank's ring attention, emulated
    python -m avgen_b200.ops.bench zero --numel 268435456            # sharded AdamW step on a one-rank group

Times come from CUDA events on the launching stream after warm-up, with a
synchronize on both sides; each line also reports the library equivalent
(cuBLAS through ``torch.matmul``, cuDNN/flash SDPA) on the same inputs.
"""
from __future__ import annotations

import argparse
import os
from collections.abc import Callable

import torch


def _time(fn: Callable[[], object], iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def bench_attention(length: int, heads: int, iters: int, once: bool) -> None:
    from avgen_b200.ops import kernels as K

    q = torch.randn(1, heads, length, 128, device="cuda").bfloat16()
    k, v = torch.randn_like(q), torch.randn_like(q)
    out, lse = K.attention_fwd(q, k, v)
    dout = torch.randn_like(out)
    if once:
        K.attention_fwd(q, k, v)
        K.attention_bwd(q, k, v, out, dout, lse)
        torch.cuda.synchronize()
        return
    flops = 4.0 * heads * length * length * 128
    t_fwd = _time(lambda: K.attention_fwd(q, k, v), iters)
    t_bwd = _time(lambda: K.attention_bwd(q, k, v, out, dout, lse), iters)
    dense = K.pack_key_mask(torch.ones(1, length, dtype=torch.bool, device="cuda"))  # what the model passes
    t_fwd_m = _time(lambda: K.attention_fwd(q, k, v, kmask=dense), iters)
    t_bwd_m = _time(lambda: K.attention_bwd(q, k, v, out, dout, lse, kmask=dense), iters)
    qt, kt, vt = (t.requires_grad_() for t in (q.clone(), k.clone(), v.clone()))
    ref = torch.nn.functional.scaled_dot_product_attention
    t_lf = _time(lambda: ref(qt, kt, vt), iters)
    o = ref(qt, kt, vt)
    g = torch.randn_like(o)
    t_lb = _time(lambda: torch.autograd.grad(o, (qt, kt, vt), g, retain_graph=True), iters)
    print(f"attention L={length} H={heads}: fwd {t_fwd:.3f} ms ({flops / t_fwd / 1e9:.0f} TF/s) | "
          f"bwd {t_bwd:.3f} ms ({2.5 * flops / t_bwd / 1e9:.0f} TF/s counted) | "
          f"torch SDPA fwd {t_lf:.3f} ms, bwd {t_lb:.3f} ms | with an all-valid key mask: fwd {t_fwd_m:.3f} ms, "
          f"bwd {t_bwd_m:.3f} ms")


def trace_attention(length: int, heads: int, which: str) -> None:
    """Print the SM-clock timeline of CTA 0 (one row per tile), from the kernels' ``trace`` slots."""
    from avgen_b200.ops import kernels as K

    q = torch.randn(1, heads, length, 128, device="cuda").bfloat16()
    k, v = torch.randn_like(q), torch.randn_like(q)
    tr = torch.zeros(64 * 24, dtype=torch.int64, device="cuda")
    if which == "fwd":
        for _ in range(3):
            K.attention_fwd(q, k, v, trace=tr)
    else:
        out, lse = K.attention_fwd(q, k, v)
        dout = torch.randn_like(out)
        for _ in range(3):
            K.attention_bwd(q, k, v, out, dout, lse, trace=tr)
    torch.cuda.synchronize()
    t = tr.view(64, 24).cpu().tolist()
    rows = range(4, 24)
    if which == "fwd":
        print("cycles relative to the MMA thread passing p_full[0] of tile j")
        print("tile period | g0: S seen  loaded  max  rescaled  exp  arrive | PV0 done | g1: S seen  loaded  max  "
              "rescaled  exp  arrive | MMA passes p_full[1] | PV1 done")
        for j in rows:
            b = t[j][0]
            g0 = " ".join(f"{t[j][s] - b:6d}" for s in range(3, 9))
            g1 = " ".join(f"{t[j][s] - b:6d}" for s in range(9, 15))
            print(f"{j:4d} {b - t[j - 1][0]:6d} | {g0} | {t[j][16] - b:6d} | {g1} | {t[j][2] - b:6d} | {t[j][18] - b:6d}")
    else:
        print("cycles relative to the MMA thread passing p_full(i)")
        print("iter period | dV dK dQ^T S(i+2) dP(i+2) complete | MMA passes dq_empty | softmax start, last arrive "
              "(of i) | drain sees dQ^T, releases it")
        for i in rows:
            b = t[i][0]
            ends = max(t[i][s] for s in range(8, 16))
            mma = " ".join(f"{t[i][s] - b:6d}" for s in (5, 6, 7, 20, 21))
            print(f"{i:4d} {b - t[i - 1][0]:6d} | {mma} | {t[i][1] - b:6d} | {t[i][2] - b:6d} {ends - b:6d} | "
                  f"{t[i][4] - b:6d} {max(t[i][s] for s in range(16, 20)) - b:6d}")


def bench_gemm(m: int, n: int, k: int, iters: int, once: bool = False, gated: int = 0) -> None:
    from avgen_b200.ops import kernels as K

    if gated:
        bench_gemm_gated(m, n, k, iters, once, gated)
        return

    a = torch.randn(m, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    dy = torch.randn(m, n, device="cuda").bfloat16()
    grad = torch.zeros(n, k, device="cuda")
    flops = 2.0 * m * n * k
    if once:  # one launch of each (SwiGLU-epilogue forward, dX, dW) for a profiler
        K.gemm(a, b, epilogue="swiglu", aux=torch.empty(m, n, device="cuda", dtype=torch.bfloat16))
        K.linear_dx(dy, b)
        K.linear_dw(dy, a, grad)
        torch.cuda.synchronize()
        return
    aux = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    resid = torch.randn(m, n, device="cuda").bfloat16()
    gate = torch.randn(1, n, device="cuda")
    rows = [("fwd", lambda: K.gemm(a, b), lambda: a @ b.t()),
            ("fwd+swiglu", lambda: K.gemm(a, b, epilogue="swiglu", aux=aux), lambda: a @ b.t()),
            ("fwd+gate_resid", lambda: K.gemm(a, b, epilogue="gate_resid", resid=resid, gate=gate, rows_per_batch=m),
             lambda: a @ b.t()),
            ("dx", lambda: K.linear_dx(dy, b), lambda: dy @ b),
            ("dw", lambda: K.linear_dw(dy, a, grad), lambda: dy.t() @ a)]
    for name, ours, lib in rows:
        t_o, t_l = _time(ours, iters), _time(lib, iters)
        print(f"gemm {m}x{n}x{k} {name}: {t_o:.3f} ms ({flops / t_o / 1e9:.0f} TF/s) | "
              f"cuBLAS {t_l:.3f} ms ({flops / t_l / 1e9:.0f} TF/s)")


def bench_gemm_gated(m: int, n: int, k: int, iters: int, once: bool, world: int) -> None:
    """The GEMM in gated-operand mode as one rank of a ``world``-way all-gather:
    B's rows in ``world`` chunks whose arrival flags are already set, so the
    difference to the plain GEMM is the cost of the rotation and the flag checks."""
    from avgen_b200.ops import kernels as K

    a = torch.randn(m, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    flags = torch.ones(world, dtype=torch.int32, device="cuda")
    gated = dict(gate_flags=flags, gate_epoch=1, gate_operand="b", gate_chunk=-(-n // world), gate_rank=world // 2)
    if once:
        K.gemm(a, b, **gated)
        torch.cuda.synchronize()
        return
    flops = 2.0 * m * n * k
    for name, fn in (("fwd", lambda: K.gemm(a, b)), (f"fwd gated {world} chunks", lambda: K.gemm(a, b, **gated))):
        t = _time(fn, iters)
        print(f"gemm {m}x{n}x{k} {name}: {t:.3f} ms ({flops / t / 1e9:.0f} TF/s)")


def bench_zero(numel: int, iters: int, once: bool) -> None:
    """One optimizer step over ``numel`` fp32 parameters: :class:`ShardedAdamW` on a
    one-rank NCCL group (the gradient pull-reduce kernel, the norm all-reduce and
    the AdamW-with-push kernel, with no peer traffic) against the replicated
    :class:`FusedAdamW`. Bandwidth counts the bytes each must move: 36 B per
    parameter sharded (gradient read, reduced shard written and read, parameter
    and both moments read and written), 32 B replicated (gradient read by the norm
    and the update, parameter and both moments read and written)."""
    import socket

    import torch.distributed as dist

    from avgen_b200.train.optimizer import FusedAdamW, ShardedAdamW

    if not dist.is_initialized():
        with socket.socket() as sock:
            sock.bind(("127.0.0.1", 0))
            port = sock.getsockname()[1]
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(port))
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    p = torch.nn.Parameter(torch.randn(numel, device="cuda"))
    o_sh = ShardedAdamW([p], lr=1e-4, weight_decay=0.1)
    p.grad.normal_()
    if once:
        o_sh.step(max_grad_norm=1.0)
        torch.cuda.synchronize()
        dist.destroy_process_group()
        return
    q = torch.nn.Parameter(p.detach().clone())
    o_f = FusedAdamW([q], lr=1e-4, weight_decay=0.1)
    q.grad.normal_()
    for name, opt, per in (("sharded (1 rank)", o_sh, 36), ("replicated", o_f, 32)):
        t = _time(lambda opt=opt: opt.step(max_grad_norm=1.0), iters)
        print(f"adamw step {numel} params {name}: {t:.3f} ms ({per * numel / (t * 1e-3) / 1e9:.0f} GB/s)")
    dist.destroy_process_group()


def bench_ring(length: int, heads: int, world: int, iters: int, once: bool) -> None:
    """Ring-layout attention as one rank of a ``world``-way context-parallel group
    sees it, emulated on one GPU: the kernels in ring mode (rotated slab order,
    per-slab flag checks, per-slab backward launches) with every slab already
    resident and its flag set. On one GPU the slab copies would be same-device
    copies, which the driver may run as kernels that cannot start while the
    attention kernel holds every SM; across GPUs they run on copy engines."""
    from avgen_b200.ops import kernels as K
    from avgen_b200.ops._ext import load

    ext = load()
    q = torch.randn(1, heads, length, 128, device="cuda").bfloat16()
    src = torch.randn(2, world, 1, heads, length, 128, device="cuda").bfloat16()
    k_all, v_all = torch.zeros_like(src[0]), torch.zeros_like(src[1])
    flags = torch.zeros(world, dtype=torch.int32, device="cuda")
    copy = torch.cuda.Stream()
    slab = src[0, 0].numel() * 2
    epoch = [0]

    for r in range(world):
        ext.p2p_copy(k_all[r].data_ptr(), src[0, r].data_ptr(), slab)
        ext.p2p_copy(v_all[r].data_ptr(), src[1, r].data_ptr(), slab)
    flags.fill_(1)
    torch.cuda.synchronize()
    del copy, epoch

    def forward() -> tuple[torch.Tensor, torch.Tensor]:
        return K.attention_fwd(q, k_all, v_all, ring_rank=0, ring_flags=flags, ring_epoch=1)

    out, lse = forward()
    dout = torch.randn_like(out)
    order = list(range(1, world)) + [0]

    def backward() -> object:
        return K.attention_bwd_slabs(q, k_all, v_all, out, dout, lse, order=order)

    if once:
        forward()
        backward()
        torch.cuda.synchronize()
        return
    flops = 4.0 * heads * length * world * length * 128
    t_f, t_b = _time(forward, iters), _time(backward, iters)
    print(f"ring attention Lq={length} Lk={world}x{length} H={heads}: fwd {t_f:.3f} ms ({flops / t_f / 1e9:.0f} TF/s) "
          f"| bwd ({world} launches) {t_b:.3f} ms ({2.5 * flops / t_b / 1e9:.0f} TF/s counted)")


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="op", required=True)
    a = sub.add_parser("attention")
    a.add_argument("--L", type=int, default=16384)
    a.add_argument("--H", type=int, default=20)
    a.add_argument("--bwd", choices=("fused", "split"), default=None)
    a.add_argument("--once", action="store_true")
    t = sub.add_parser("trace")
    t.add_argument("--L", type=int, default=16384)
    t.add_argument("--H", type=int, default=20)
    t.add_argument("--pass", dest="which", choices=("fwd", "bwd"), default="bwd")
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=16384)
    g.add_argument("--n", type=int, default=7680)
    g.add_argument("--k", type=int, default=2560)
    g.add_argument("--once", action="store_true")
    g.add_argument("--gated", type=int, default=0, help="chunks of a gated (all-gathered) B operand")
    r = sub.add_parser("ring")
    r.add_argument("--L", type=int, default=4096, help="keys and queries per rank")
    r.add_argument("--H", type=int, default=20)
    r.add_argument("--world", type=int, default=4)
    r.add_argument("--once", action="store_true")
    z = sub.add_parser("zero")
    z.add_argument("--numel", type=int, default=268435456)
    z.add_argument("--once", action="store_true")
    for s in (a, g, r, z):
        s.add_argument("--iters", type=int, default=10)
    args = p.parse_args()
    if getattr(args, "bwd", None):
        os.environ["AVGEN_ATTN_BWD"] = args.bwd
        from avgen_b200.ops import kernels as K

        K._ATTN_BWD = args.bwd
    if args.op == "attention":
        bench_attention(args.L, args.H, args.iters, args.once)
    elif args.op == "trace":
        trace_attention(args.L, args.H, args.which)
    elif args.op == "ring":
        bench_ring(args.L, args.H, args.world, args.iters, args.once)
    elif args.op == "zero":
        bench_zero(args.numel, args.iters, args.once)
    else:
        bench_gemm(args.m, args.n, args.k, args.iters, args.once, args.gated)
    from avgen_b200.ops._ext import check_errors

    code = check_errors()
    if code:
        raise SystemExit(f"a kernel recorded error code {code}")


if __name__ == "__main__":
    main()
