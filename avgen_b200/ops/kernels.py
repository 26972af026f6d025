"""Functional wrappers over the sm_100a kernels of ``avgen_b200._C``.

Every function here launches a hand-written kernel on the current CUDA stream;
outputs are allocated by the caller or here with ``torch.empty``. Shapes follow
the conventions of the kernels:

* GEMM: ``D[M, N] = A[M, K] . B[N, K]^T``; ``a_mn`` / ``b_mn`` say an operand is
  given transposed (``[K, M]`` / ``[K, N]``) so backward GEMMs need no copies.
* attention: ``q`` ``[B, H, Lq, D]``, ``k``/``v`` ``[B, Hk, Lk, D]`` (head-major),
  output token-major ``[B, Lq, H, D]``, ``lse`` fp32 ``[B, H, Lq]`` in the base-2
  domain of the scaled scores.
"""
from __future__ import annotations

import math
import os
import sys
import time

import torch

from avgen_b200.ops._ext import load

EPILOGUES = {"store": 0, "gate_resid": 1, "swiglu": 2, "gelu": 3, "atomic": 4}

# Running count of kernel launches issued through this module (benchmarks read it).
LAUNCHES = [0]
# AVGEN_KERNEL_DEBUG=1: synchronise after every wrapper call, report its device time
# and stop at the first call that leaves a timed-out wait in the device error word.
_DEBUG = os.environ.get("AVGEN_KERNEL_DEBUG") == "1"
_ATTN_BWD = os.environ.get("AVGEN_ATTN_BWD", "fused")


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n
    if _DEBUG:
        _debug_check(sys._getframe(1).f_code.co_name)


def _debug_check(name: str) -> None:
    from avgen_b200.ops._ext import check_errors

    t0 = time.perf_counter()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    code = check_errors(clear=False)
    if dt > 0.5 or code:
        print(f"[avgen kernel debug] {name}: {dt * 1e3:.1f} ms after launch, error word {code}", flush=True)
    if code:
        raise RuntimeError(f"kernel wrapper {name} left error code {code}")


def launch_count() -> int:
    """Kernels launched through :mod:`avgen_b200.ops.kernels` so far in this process."""
    return LAUNCHES[0]


# Deterministic weight gradients: the weight-gradient GEMM splits its reduction over
# CTAs that add into the fp32 gradient with atomics, in whatever order they finish.
# In deterministic mode (``AVGEN_DETERMINISTIC=1`` or ``set_deterministic(True)``)
# it runs unsplit: each output element gets exactly one add per call, so repeated
# runs agree bitwise. Attention's dQ accumulation and the norm reductions keep their
# order-dependent sums.
_DETERMINISTIC = [os.environ.get("AVGEN_DETERMINISTIC", "0") == "1"]


def set_deterministic(on: bool = True) -> None:
    _DETERMINISTIC[0] = bool(on)


def deterministic() -> bool:
    return _DETERMINISTIC[0]


_BF16 = torch.bfloat16
_F32 = torch.float32


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    epilogue: str = "store",
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = _BF16,
    bias: torch.Tensor | None = None,
    resid: torch.Tensor | None = None,
    gate: torch.Tensor | None = None,
    rows_per_batch: int = 1,
    aux: torch.Tensor | None = None,
    k_splits: int = 1,
    groups: torch.Tensor | None = None,
    a2: torch.Tensor | None = None,
    b2: torch.Tensor | None = None,
    gate_flags: torch.Tensor | None = None,
    gate_epoch: int = 0,
    gate_operand: str = "",
    gate_chunk: int = 0,
    gate_rank: int = 0,
) -> torch.Tensor:
    """tcgen05 GEMM with a fused epilogue (see ``csrc/gemm.cu``).

    ``gate`` rows are picked per output row by ``groups`` (int32, one entry per
    row) when given, else by ``row // rows_per_batch``. An appended pair
    ``(a2, b2)``, laid out like ``(a, b)``, extends the reduction:
    ``D = [a | a2] . [b | b2]^T`` in one accumulator.

    Gated operand (an all-gather fused into the GEMM): with ``gate_flags``, the
    rows of ``a`` (``gate_operand="a"``, the M axis) or of ``b`` (``"b"``, the N
    axis) form chunks of ``gate_chunk`` rows; a tile that reads chunk ``c`` other
    than ``gate_rank`` first waits (bounded; error code 5 on timeout) until
    ``gate_flags[c] >= gate_epoch``. Tiles of the own chunk run first.
    """
    m = a.shape[1] if a_mn else a.shape[0]
    n = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        cols = n // 2 if epilogue == "swiglu" else n
        if epilogue == "atomic":
            out = torch.zeros((m, cols), device=a.device, dtype=_F32)
        else:
            out = torch.empty((m, cols), device=a.device, dtype=out_dtype)
    load().gemm(
        a, b, out, a_mn, b_mn, EPILOGUES[epilogue], bias, resid, gate, rows_per_batch, aux, k_splits, groups, a2, b2,
        gate_flags, gate_epoch, {"": 0, "a": 1, "b": 2}[gate_operand], gate_chunk, gate_rank,
    )
    _count()
    return out


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x[M, K] @ w[N, K]^T (+ bias)`` in bf16 with fp32 accumulation."""
    return gemm(x, w, bias=bias)


def linear_dx(dy: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype = _BF16, *,
              a2: torch.Tensor | None = None, b2: torch.Tensor | None = None) -> torch.Tensor:
    """Input gradient ``dy[M, N] @ w[N, K]`` (``+ a2[M, R] @ b2[R, K]`` when given)."""
    return gemm(dy, w, b_mn=True, out_dtype=out_dtype, a2=a2, b2=b2)


def linear_dw(dy: torch.Tensor, x: torch.Tensor, grad: torch.Tensor, *, k_splits: int = 0) -> torch.Tensor:
    """Accumulate the weight gradient ``grad[N, K] += dy[M, N]^T @ x[M, K]`` (fp32)."""
    n, k = grad.shape
    if k_splits <= 0 and _DETERMINISTIC[0]:
        k_splits = 1
    if k_splits <= 0:
        tiles = -(-n // 128) * -(-k // 256)
        sms = torch.cuda.get_device_properties(dy.device).multi_processor_count
        k_splits = max(1, min(8, (2 * sms) // max(1, tiles)))
    return gemm(dy, x, a_mn=True, b_mn=True, epilogue="atomic", out=grad, k_splits=k_splits)


def rmsnorm_mod(
    x: torch.Tensor,
    weight: torch.Tensor | None,
    scale: torch.Tensor | None = None,
    shift: torch.Tensor | None = None,
    *,
    rows_per_batch: int = 1,
    eps: float = 1e-6,
    out: torch.Tensor | None = None,
    want_rstd: bool = True,
    groups: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``rmsnorm(x) * weight * (1 + scale[g]) + shift[g]`` over rows of ``x[R, W]``, with
    ``g = groups[row]`` when a per-row group index is given, else ``row // rows_per_batch``."""
    y = out if out is not None else torch.empty_like(x)
    rstd = torch.empty(x.shape[0], device=x.device, dtype=_F32) if want_rstd else None
    load().rmsnorm_mod_fwd(x, y, rstd, weight, scale, shift, rows_per_batch, eps, groups)
    _count()
    return y, rstd


def rmsnorm_mod_bwd(
    x: torch.Tensor,
    rstd: torch.Tensor,
    dy: torch.Tensor,
    weight: torch.Tensor | None,
    scale: torch.Tensor | None = None,
    shift: torch.Tensor | None = None,
    *,
    dres: torch.Tensor | None = None,
    dweight: torch.Tensor | None = None,
    dscale: torch.Tensor | None = None,
    dshift: torch.Tensor | None = None,
    rows_per_batch: int = 1,
    dx: torch.Tensor | None = None,
    groups: torch.Tensor | None = None,
) -> torch.Tensor:
    """Backward of :func:`rmsnorm_mod`; parameter grads accumulate (fp32)."""
    dx = dx if dx is not None else torch.empty_like(x)
    load().rmsnorm_mod_bwd(
        x, rstd, dy, dx, dres, weight, scale, shift, dweight, dscale, dshift, rows_per_batch, groups
    )
    _count(2 if (dweight is not None or dscale is not None or dshift is not None) else 1)
    return dx


def gate_bwd(
    dx: torch.Tensor, a: torch.Tensor, gate: torch.Tensor, dgate: torch.Tensor, *, rows_per_batch: int,
    groups: torch.Tensor | None = None,
) -> torch.Tensor:
    """``da = dx * gate[g]`` and ``dgate[g] += sum_rows(dx * a)`` (``g`` as in :func:`rmsnorm_mod`)."""
    da = torch.empty_like(dx)
    load().gate_bwd(dx, a, gate, da, dgate, rows_per_batch, groups)
    _count()
    return da


def rope_frequencies(
    head_dim: int,
    *,
    theta: float = 10000.0,
    time_scale: float = 1.0,
    mode: str = "none",
    time_factor: float = 1.0,
    spatial_factor: float = 1.0,
    device: torch.device | str = "cpu",
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-pair angular frequency and coordinate axis for 3-D axial RoPE.

    Pairs are split over (time, row, column) as ``(P - 2 floor(P/3), floor(P/3),
    floor(P/3))`` (reference: avgen/models/rope.py:128-157); time scaling and
    linear / NTK scaling fold into the frequencies so the kernel computes
    ``angle = coords[axis] * freq`` (reference: avgen/models/rope.py:218-294).
    """
    pairs = head_dim // 2
    spatial = pairs // 3
    budgets = (pairs - 2 * spatial, spatial, spatial)
    factors = (time_factor, spatial_factor, spatial_factor)
    freqs: list[torch.Tensor] = []
    axes: list[torch.Tensor] = []
    for axis, (count, factor) in enumerate(zip(budgets, factors, strict=True)):
        axis_theta = theta
        mult = 1.0
        if axis == 0 and time_scale != 1.0:
            mult *= time_scale
        if mode == "linear" and factor != 1.0:
            mult /= factor
        elif mode == "ntk" and factor != 1.0:
            dim = 2 * count
            if dim > 2:
                axis_theta = theta * factor ** (dim / (dim - 2))
        exponent = torch.arange(count, dtype=_F32) / count
        inv = torch.pow(torch.tensor(axis_theta, dtype=_F32), -exponent) * mult
        freqs.append(inv)
        axes.append(torch.full((count,), axis, dtype=torch.int32))
    return torch.cat(freqs).to(device), torch.cat(axes).to(device)


def qkv_rope(
    qkv: torch.Tensor,
    *,
    batch: int,
    length: int,
    heads: int,
    kv_heads: int,
    head_dim: int,
    q_weight: torch.Tensor | None,
    k_weight: torch.Tensor | None,
    coords: torch.Tensor | None,
    freq: torch.Tensor | None,
    axis: torch.Tensor | None,
    eps: float = 1e-6,
    k_out: torch.Tensor | None = None,
    v_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor | None, torch.Tensor | None, torch.Tensor | None]:
    """QK-RMSNorm + RoPE + relayout of ``qkv[B*L, (H + 2Hk) * D]`` into head-major q, k, v.

    ``k_out``/``v_out`` (dense ``[B, Hk, L, D]`` bf16) receive k and v in place,
    e.g. this rank's slab of a context-parallel ring buffer."""
    dev = qkv.device
    q = torch.empty((batch, heads, length, head_dim), device=dev, dtype=_BF16) if heads else None
    shape = (batch, kv_heads, length, head_dim)
    for t in (k_out, v_out):
        if t is not None and (tuple(t.shape) != shape or t.dtype != _BF16 or not t.is_contiguous()):
            raise ValueError(f"k_out/v_out must be dense bf16 {shape}")
    k = (k_out if k_out is not None else torch.empty(shape, device=dev, dtype=_BF16)) if kv_heads else None
    v = (v_out if v_out is not None else torch.empty(shape, device=dev, dtype=_BF16)) if kv_heads else None
    load().qkv_rope_fwd(
        qkv, batch, length, heads, kv_heads, head_dim, eps, q_weight, k_weight, coords, freq, axis, q, k, v
    )
    _count()
    return q, k, v


def qkv_rope_bwd(
    qkv: torch.Tensor,
    dq: torch.Tensor | None,
    dk: torch.Tensor | None,
    dv: torch.Tensor | None,
    *,
    batch: int,
    length: int,
    heads: int,
    kv_heads: int,
    head_dim: int,
    q_weight: torch.Tensor | None,
    k_weight: torch.Tensor | None,
    coords: torch.Tensor | None,
    freq: torch.Tensor | None,
    axis: torch.Tensor | None,
    dq_weight: torch.Tensor | None = None,
    dk_weight: torch.Tensor | None = None,
    eps: float = 1e-6,
) -> torch.Tensor:
    """Backward of :func:`qkv_rope`: returns ``dqkv`` in the GEMM layout."""
    dqkv = torch.empty_like(qkv)
    load().qkv_rope_bwd(
        qkv, dqkv, batch, length, heads, kv_heads, head_dim, eps, q_weight, k_weight, coords, freq, axis,
        dq, dk, dv, dq_weight, dk_weight,
    )
    _count()
    return dqkv


def pack_key_mask(mask: torch.Tensor | None) -> torch.Tensor | None:
    """Pack a boolean key mask ``[B, L]`` into int32 bit words ``[B, ceil(L/32)]``."""
    if mask is None:
        return None
    b, length = mask.shape
    words = -(-length // 32)
    padded = torch.zeros((b, words * 32), device=mask.device, dtype=torch.int64)
    padded[:, :length] = mask.to(torch.int64)
    weights = torch.bitwise_left_shift(torch.ones(32, device=mask.device, dtype=torch.int64),
                                       torch.arange(32, device=mask.device, dtype=torch.int64))
    packed = (padded.view(b, words, 32) * weights).sum(-1)
    packed = torch.where(packed >= 2**31, packed - 2**32, packed)
    return packed.to(torch.int32).contiguous()


def row_stats(b: int, h: int, length: int, device: torch.device) -> torch.Tensor:
    """An fp32 ``[b, h, length]`` tensor whose ``(b, h)`` rows are padded to 16 bytes
    (the attention backward streams these rows with TMA)."""
    padded = -(-length // 4) * 4
    return torch.empty((b, h, padded), device=device, dtype=_F32)[..., :length]


def attention_fwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    kmask: torch.Tensor | None = None,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    want_lse: bool = True,
    trace: torch.Tensor | None = None,
    ring_rank: int = 0,
    ring_flags: torch.Tensor | None = None,
    ring_epoch: int = 0,
    ring_wait: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Flash attention forward. Returns ``(out [B, Lq, H, D], lse [B, H, Lq])``.

    ``trace`` (int64, >= 1536 entries, diagnostics) receives SM clock stamps of
    CTA 0 per key tile: the MMA thread's waits, each softmax group's phases and
    the completion of its S and PV products (slot map in ``attention.cu``).

    Context-parallel ring: ``k``/``v`` given as ``[world, B, Hk, L, D]`` (rank r's
    keys in slab r, ``L`` a multiple of 128). Every CTA starts at slab
    ``ring_rank`` and reads slab r only after ``ring_flags[r]`` (int32, written
    by a copy stream or a peer) has reached ``ring_epoch``. ``ring_wait`` (int64
    [1], optional) accumulates the SM clock cycles the CTAs spent in those waits.
    """
    b, h, lq, d = q.shape
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    if out is None:
        out = torch.empty((b, lq, h, d), device=q.device, dtype=_BF16)
    lse = row_stats(b, h, lq, q.device) if want_lse else None
    load().attn_fwd(q, k, v, out, lse, kmask, scale, trace, ring_rank, ring_flags, ring_epoch & 0xFFFFFFFF, ring_wait)
    _count()
    return out, lse


def attention_bwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    dout: torch.Tensor,
    lse: torch.Tensor,
    *,
    kmask: torch.Tensor | None = None,
    scale: float | None = None,
    trace: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Flash attention backward. Returns ``(dq, dk, dv)`` (bf16, shapes of q, k, v).

    With ``k``/``v`` in the ring layout ``[world, B, Hk, L, D]``, ``dk``/``dv``
    come back in it too: slab r holds this rank's partial gradients for rank r's keys.

    ``trace`` (int64, >= 1536 entries, diagnostics) receives per-role SM clock
    stamps of the first CTA of the one-pass kernel.

    The default is the one-pass kernel (five GEMM-shaped products per tile pair,
    dQ summed in an fp32 scratch by TMA reduce-add); ``AVGEN_ATTN_BWD=split``
    selects the two-kernel variant (dK/dV and dQ passes, no reduction, two extra
    products per tile pair).
    """
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    delta = torch.empty_strided(lse.shape, lse.stride(), device=lse.device, dtype=_F32)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    acc = None
    if _ATTN_BWD != "split" or k.dim() == 5:  # the ring layout [world, B, Hk, L, D] needs the one-pass kernel
        acc = torch.empty(q.shape[0] * q.shape[1] * d * (-(-q.shape[2] // 4) * 4), device=q.device, dtype=_F32)
    load().attn_bwd(q, k, v, o, dout, lse, delta, dq, dk, dv, kmask, scale, acc, trace)
    _count(4 if acc is not None else 3)
    return dq, dk, dv


def attention_bwd_slabs(
    q: torch.Tensor,
    k_all: torch.Tensor,
    v_all: torch.Tensor,
    o: torch.Tensor,
    dout: torch.Tensor,
    lse: torch.Tensor,
    *,
    order: list[int],
    kmask: torch.Tensor | None = None,
    scale: float | None = None,
    on_slab=None,  # noqa: ANN001
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Ring-layout backward launched once per key slab, in ``order``.

    ``k_all``/``v_all`` are ``[world, B, Hk, L, D]``; slab r's partial dK/dV land
    in ``dk_all[r]``/``dv_all[r]`` when its launch completes, and ``on_slab(r,
    dk_all, dv_all)`` runs right after that launch is enqueued (to start moving
    the slab while the next one computes). dQ accumulates across the launches
    and is converted after the last.
    """
    world, _, _, length, d = k_all.shape
    if length % 128:
        raise ValueError("ring slabs must hold a multiple of 128 keys")
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    tiles = length // 128
    delta = torch.empty_strided(lse.shape, lse.stride(), device=lse.device, dtype=_F32)
    dq = torch.empty_like(q)
    dk_all = torch.empty_like(k_all)
    dv_all = torch.empty_like(v_all)
    acc = torch.empty(q.shape[0] * q.shape[1] * d * (-(-q.shape[2] // 4) * 4), device=q.device, dtype=_F32)
    ext = load()
    for i, r in enumerate(order):
        ext.attn_bwd(q, k_all, v_all, o, dout, lse, delta, dq, dk_all, dv_all, kmask, scale, acc, None,
                     r * tiles, tiles, i > 0, i < len(order) - 1)
        _count(1 + (i == 0) + (i == len(order) - 1))
        if on_slab is not None:
            on_slab(r, dk_all, dv_all)
    return dq, dk_all, dv_all


def slab_sum(sources: list[torch.Tensor], out: torch.Tensor) -> torch.Tensor:
    """``out = sum(sources)`` for bf16 tensors shaped like ``out`` (fp32 accumulation)."""
    ptrs = torch.tensor([t.data_ptr() for t in sources], dtype=torch.int64, device=out.device)
    load().slab_sum(ptrs, out)
    _count()
    return out


def swiglu_bwd(dh: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    """Backward of the interleaved SwiGLU epilogue: returns ``dgu`` like ``gu``."""
    dgu = torch.empty_like(gu)
    load().swiglu_bwd(dh, gu, dgu)
    _count()
    return dgu


def gelu_bwd(dh: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    """Backward of GELU(tanh): returns the gradient w.r.t. the pre-activation."""
    dpre = torch.empty_like(pre)
    load().gelu_bwd(dh, pre, dpre)
    _count()
    return dpre


def flow_loss_stats(
    pred: torch.Tensor,
    target: torch.Tensor,
    loss_mask: torch.Tensor,
    weight: torch.Tensor | None,
    *,
    rows_per_batch: int,
) -> torch.Tensor:
    """``[sum(w*mse*m), sum(mse*m), sum(m)]`` over token rows (fp32, device)."""
    stats = torch.zeros(3, device=pred.device, dtype=_F32)
    load().flow_loss_fwd(pred.contiguous(), target.contiguous(), loss_mask.contiguous(), weight, rows_per_batch, stats)
    _count()
    return stats


def flow_loss_grad(
    pred: torch.Tensor,
    target: torch.Tensor,
    loss_mask: torch.Tensor,
    weight: torch.Tensor | None,
    scale: torch.Tensor,
    *,
    rows_per_batch: int,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Gradient of ``scale * sum(w * mse * m)`` w.r.t. ``pred``."""
    dpred = torch.empty(pred.shape, device=pred.device, dtype=out_dtype or pred.dtype)
    load().flow_loss_bwd(pred.contiguous(), target.contiguous(), loss_mask.contiguous(), weight, rows_per_batch,
                         scale, dpred)
    _count()
    return dpred


def noise_interp(
    clean: torch.Tensor,
    t: torch.Tensor,
    *,
    seed: int,
    offset: int = 0,
    row_base: int = 0,
    rows_per_sample: int | None = None,
    global_rows_per_sample: int | None = None,
    want_noise: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """Counter-based noise and ``noisy = x + t(eps - x)``, ``target = eps - x``."""
    rows = clean.numel() // clean.shape[-1]
    rps = rows_per_sample or clean.shape[-2]
    grps = global_rows_per_sample or rps
    noisy = torch.empty(clean.shape, device=clean.device, dtype=_F32)
    target = torch.empty_like(noisy)
    noise = torch.empty_like(noisy) if want_noise else None
    del rows
    load().noise_interp(clean.contiguous(), t.contiguous(), seed & ((1 << 63) - 1), offset, row_base, rps, grps,
                        noisy, target, noise)
    _count()
    return noisy, target, noise


def adamw_step(
    param: torch.Tensor,
    grad: torch.Tensor,
    exp_avg: torch.Tensor,
    exp_avg_sq: torch.Tensor,
    *,
    lr: float,
    betas: tuple[float, float],
    eps: float,
    weight_decay: float,
    step: int,
    param_bf16: torch.Tensor | None = None,
    grad_scale: torch.Tensor | None = None,
    skip: torch.Tensor | None = None,
) -> None:
    """Fused AdamW over flat fp32 buffers (optionally writing a bf16 copy)."""
    load().adamw(param, grad, exp_avg, exp_avg_sq, lr, betas[0], betas[1], eps, weight_decay, step, param_bf16,
                 grad_scale, skip)
    _count()


def sq_norm_(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``out += sum(x ** 2)`` for a flat fp32 buffer."""
    load().sq_norm(x, out)
    _count()
    return out


def ema_(param: torch.Tensor, shadow: torch.Tensor, decay: float) -> None:
    """``shadow += (1 - decay) * (param - shadow)``."""
    load().ema(param, shadow, decay)
    _count()


def guided_euler(cond: torch.Tensor, uncond: torch.Tensor | None, x: torch.Tensor, sigma: torch.Tensor,
                 sigma_next: torch.Tensor, *, scale: float = 1.0, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """One Euler step with classifier-free guidance fused in:
    ``x + (sigma_next - sigma) * (uncond + scale * (cond - uncond))`` per sample
    (``uncond=None``: plain Euler). ``sigma``/``sigma_next`` are fp32 ``[batch]``."""
    out = torch.empty(x.shape, device=x.device, dtype=out_dtype or x.dtype)
    load().guided_euler(cond.contiguous(), None if uncond is None else uncond.contiguous(), x.contiguous(),
                        sigma.to(_F32).contiguous(), sigma_next.to(_F32).contiguous(), float(scale), out)
    _count()
    return out


def sde_step(v: torch.Tensor, x: torch.Tensor, sigma: torch.Tensor, sigma_next: torch.Tensor, g: torch.Tensor, *,
             floor: float, noise: torch.Tensor | None = None, prev: torch.Tensor | None = None,
             mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Flow-GRPO SDE transition: returns ``(sample, mean, log_prob)``. Rollout mode takes
    a standard-normal ``noise``; update mode scores the stored ``prev`` instead."""
    xf = x.to(_F32).contiguous()
    mean = torch.empty_like(xf)
    log_prob = torch.zeros(x.shape[0], device=x.device, dtype=_F32)
    sample = torch.empty_like(xf) if prev is None else None
    load().sde_step(v.contiguous(), xf, sigma.to(_F32).contiguous(), sigma_next.to(_F32).contiguous(),
                    g.to(_F32).contiguous(), float(floor), mean, log_prob,
                    None if noise is None else noise.to(_F32).contiguous(),
                    None if prev is None else prev.to(_F32).contiguous(),
                    None if mask is None else mask.to(torch.bool).contiguous(), sample)
    _count()
    return (sample if prev is None else prev), mean, log_prob
