"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
from __future__ import annotations

import math
import os

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from avgen_b200.ops import kernels

    return kernels


def _close(got: torch.Tensor, ref: torch.Tensor, rtol: float = 2e-2, atol: float = 2e-2) -> None:
    got = got.float()
    ref = ref.float()
    err = (got - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= atol + rtol * scale, f"max err {err:.4g} vs scale {scale:.4g}"


def _errors_clear() -> None:
    from avgen_b200.ops._ext import check_errors

    assert check_errors() == 0, "a kernel recorded a timed-out wait"


@pytest.mark.parametrize("m,n,k", [(256, 256, 128), (300, 264, 200), (1024, 2560, 2560), (129, 8, 64)])
def test_gemm_store(m: int, n: int, k: int) -> None:
    ops = _ops()
    torch.manual_seed(0)
    a = torch.randn(m, k, device=DEV).bfloat16()
    b = torch.randn(n, k, device=DEV).bfloat16()
    bias = torch.randn(n, device=DEV)
    ref = a.float() @ b.float().t() + bias
    got = ops.gemm(a, b, bias=bias)
    _close(got, ref)
    got32 = ops.gemm(a, b, out_dtype=torch.float32)
    _close(got32, a.float() @ b.float().t(), rtol=1e-3, atol=1e-2)
    _errors_clear()


@pytest.mark.parametrize("m,n,k", [(512, 384, 256), (200, 136, 72)])
def test_gemm_transposed_operands(m: int, n: int, k: int) -> None:
    ops = _ops()
    torch.manual_seed(1)
    dy = torch.randn(m, n, device=DEV).bfloat16()
    w = torch.randn(n, k, device=DEV).bfloat16()
    x = torch.randn(m, k, device=DEV).bfloat16()
    # dX = dY . W  (B given as [K_red, N_out])
    _close(ops.linear_dx(dy, w), dy.float() @ w.float())
    # dW += dY^T . X (both operands MN-major), split-K atomics, accumulating
    grad = torch.ones(n, k, device=DEV)
    ops.linear_dw(dy, x, grad, k_splits=3)
    _close(grad, 1.0 + dy.float().t() @ x.float(), rtol=1e-3, atol=5e-2)
    _errors_clear()


def test_gemm_fused_epilogues() -> None:
    ops = _ops()
    torch.manual_seed(2)
    bsz, rows, k, n = 2, 192, 256, 512
    m = bsz * rows
    a = torch.randn(m, k, device=DEV).bfloat16()
    w = torch.randn(n, k, device=DEV).bfloat16() * 0.1
    acc = a.float() @ w.float().t()
    resid = torch.randn(m, n, device=DEV).bfloat16()
    gate = torch.randn(bsz, n, device=DEV)
    aux = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    got = ops.gemm(a, w, epilogue="gate_resid", resid=resid, gate=gate, rows_per_batch=rows, aux=aux)
    ref = resid.float() + gate.repeat_interleave(rows, 0) * acc
    _close(got, ref)
    _close(aux, acc)
    sw = ops.gemm(a, w, epilogue="swiglu")
    g, u = acc[:, 0::2], acc[:, 1::2]
    _close(sw, F.silu(g) * u)
    ge = ops.gemm(a, w, epilogue="gelu")
    _close(ge, F.gelu(acc, approximate="tanh"))
    _errors_clear()


def test_rmsnorm_mod_fwd_bwd() -> None:
    ops = _ops()
    torch.manual_seed(3)
    bsz, rows, w_ = 2, 100, 2560
    x = torch.randn(bsz * rows, w_, device=DEV).bfloat16()
    weight = torch.rand(w_, device=DEV) + 0.5
    scale = torch.randn(bsz, w_, device=DEV) * 0.1
    shift = torch.randn(bsz, w_, device=DEV) * 0.1
    y, rstd = ops.rmsnorm_mod(x, weight, scale, shift, rows_per_batch=rows)
    xr = x.float().requires_grad_()
    wr, sr, tr = (t.clone().requires_grad_() for t in (weight, scale, shift))
    ref = F.rms_norm(xr, (w_,), wr, 1e-6) * (1 + sr.repeat_interleave(rows, 0)) + tr.repeat_interleave(rows, 0)
    _close(y, ref)
    dy = torch.randn_like(ref).bfloat16()
    ref.backward(dy.float())
    dw = torch.zeros(w_, device=DEV)
    ds = torch.zeros(bsz, w_, device=DEV)
    dt = torch.zeros(bsz, w_, device=DEV)
    dx = ops.rmsnorm_mod_bwd(x, rstd, dy, weight, scale, shift, dweight=dw, dscale=ds, dshift=dt, rows_per_batch=rows)
    _close(dx, xr.grad)
    _close(dw, wr.grad, rtol=1e-2, atol=1e-2)
    _close(ds, sr.grad, rtol=1e-2, atol=1e-2)
    _close(dt, tr.grad, rtol=1e-2, atol=1e-2)
    _errors_clear()


def test_gate_bwd() -> None:
    ops = _ops()
    torch.manual_seed(4)
    bsz, rows, w_ = 2, 64, 256
    dx = torch.randn(bsz * rows, w_, device=DEV).bfloat16()
    a = torch.randn_like(dx)
    gate = torch.randn(bsz, w_, device=DEV)
    dgate = torch.zeros(bsz, w_, device=DEV)
    da = ops.gate_bwd(dx, a, gate, dgate, rows_per_batch=rows)
    _close(da, dx.float() * gate.repeat_interleave(rows, 0))
    _close(dgate, (dx.float() * a.float()).view(bsz, rows, w_).sum(1), rtol=1e-2, atol=1e-2)


def _rope_ref(x: torch.Tensor, coords: torch.Tensor, freq: torch.Tensor, axis: torch.Tensor) -> torch.Tensor:
    # x [B, H, L, D] fp32, coords [B, L, 3]
    ang = coords[..., axis.long()] * freq  # [B, L, D/2]
    cos, sin = torch.cos(ang)[:, None], torch.sin(ang)[:, None]
    pairs = x.unflatten(-1, (-1, 2))
    e, o = pairs[..., 0], pairs[..., 1]
    return torch.stack((e * cos - o * sin, e * sin + o * cos), -1).flatten(-2)


def test_qkv_rope_fwd_bwd() -> None:
    ops = _ops()
    torch.manual_seed(5)
    bsz, length, h, d = 2, 40, 3, 128
    qkv = torch.randn(bsz * length, 3 * h * d, device=DEV).bfloat16()
    qw = torch.rand(d, device=DEV) + 0.5
    kw = torch.rand(d, device=DEV) + 0.5
    coords = torch.rand(bsz, length, 3, device=DEV) * 10
    freq, axis = ops.rope_frequencies(d, device=DEV)
    q, k, v = ops.qkv_rope(qkv, batch=bsz, length=length, heads=h, kv_heads=h, head_dim=d, q_weight=qw,
                           k_weight=kw, coords=coords, freq=freq, axis=axis)
    xr = qkv.float().view(bsz, length, 3, h, d).permute(2, 0, 3, 1, 4).requires_grad_()
    qr = _rope_ref(F.rms_norm(xr[0], (d,), qw, 1e-6), coords, freq, axis)
    kr = _rope_ref(F.rms_norm(xr[1], (d,), kw, 1e-6), coords, freq, axis)
    vr = xr[2]
    _close(q, qr)
    _close(k, kr)
    _close(v, vr)
    dq, dk, dv = (torch.randn(t.shape, device=DEV).bfloat16() for t in (qr, kr, vr))
    (qr * dq.float()).sum().add((kr * dk.float()).sum()).add((vr * dv.float()).sum()).backward()
    dqw = torch.zeros(d, device=DEV)
    dkw = torch.zeros(d, device=DEV)
    dqkv = ops.qkv_rope_bwd(qkv, dq, dk, dv, batch=bsz, length=length, heads=h, kv_heads=h, head_dim=d,
                            q_weight=qw, k_weight=kw, coords=coords, freq=freq, axis=axis, dq_weight=dqw,
                            dk_weight=dkw)
    ref_grad = xr.grad.permute(1, 3, 0, 2, 4).reshape(bsz * length, 3 * h * d)
    _close(dqkv, ref_grad)
    _errors_clear()


def _attn_ref(q, k, v, kmask, scale):
    qf, kf, vf = q.float(), k.float(), v.float()
    rep = q.shape[1] // k.shape[1]
    kf = kf.repeat_interleave(rep, 1)
    vf = vf.repeat_interleave(rep, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if kmask is not None:
        s = s.masked_fill(~kmask[:, None, None, :], float("-inf"))
    p = torch.softmax(s, -1)
    return (p @ vf).transpose(1, 2)  # [B, Lq, H, D]


@pytest.mark.parametrize("b,h,hk,lq,lk,masked", [(1, 2, 2, 256, 256, False), (2, 2, 1, 300, 333, True),
                                                   (1, 1, 1, 1024, 2048, False)])
def test_attention_fwd_bwd(b: int, h: int, hk: int, lq: int, lk: int, masked: bool) -> None:
    ops = _ops()
    torch.manual_seed(6)
    d = 128
    scale = 1.0 / math.sqrt(d)
    q = torch.randn(b, h, lq, d, device=DEV).bfloat16()
    k = torch.randn(b, hk, lk, d, device=DEV).bfloat16()
    v = torch.randn(b, hk, lk, d, device=DEV).bfloat16()
    kmask = None
    if masked:
        kmask = torch.rand(b, lk, device=DEV) > 0.3
        kmask[:, 0] = True
    packed = ops.pack_key_mask(kmask)
    out, lse = ops.attention_fwd(q, k, v, kmask=packed)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    ref = _attn_ref(qr, kr, vr, kmask, scale)
    _close(out, ref, rtol=2e-2, atol=2e-2)
    dout = torch.randn_like(ref).bfloat16()
    ref.backward(dout.float())
    dq, dk, dv = ops.attention_bwd(q, k, v, out, dout.contiguous(), lse, kmask=packed)
    _close(dq, qr.grad, rtol=3e-2, atol=3e-2)
    _close(dk, kr.grad, rtol=3e-2, atol=3e-2)
    _close(dv, vr.grad, rtol=3e-2, atol=3e-2)
    _errors_clear()


def test_flow_loss_and_noise() -> None:
    ops = _ops()
    torch.manual_seed(7)
    bsz, length, p = 2, 50, 64
    pred = torch.randn(bsz, length, p, device=DEV)
    target = torch.randn(bsz, length, p, device=DEV)
    mask = torch.rand(bsz, length, device=DEV) > 0.2
    weight = torch.rand(bsz, device=DEV)
    stats = ops.flow_loss_stats(pred, target, mask, weight, rows_per_batch=length)
    mse = (pred - target).pow(2).mean(-1)
    m = mask.float()
    ref = torch.stack(((mse * m * weight[:, None]).sum(), (mse * m).sum(), m.sum()))
    _close(stats, ref, rtol=1e-4, atol=1e-3)
    scale = torch.tensor([0.5], device=DEV)
    grad = ops.flow_loss_grad(pred, target, mask, weight, scale, rows_per_batch=length)
    pr = pred.clone().requires_grad_()
    (0.5 * ((pr - target).pow(2).mean(-1) * m * weight[:, None]).sum()).backward()
    _close(grad, pr.grad, rtol=1e-4, atol=1e-5)
    clean = torch.randn(bsz, length, p, device=DEV)
    t = torch.rand(bsz, length, device=DEV)
    noisy, tgt, noise = ops.noise_interp(clean, t, seed=123, want_noise=True)
    assert abs(noise.mean().item()) < 0.05 and abs(noise.std().item() - 1) < 0.05
    _close(noisy, clean + t[..., None] * (noise - clean), rtol=1e-5, atol=1e-5)
    _close(tgt, noise - clean, rtol=1e-5, atol=1e-5)
    # a shard drawn with its global row base equals the slice of the full draw
    half = length // 2
    _, _, shard = ops.noise_interp(clean[:, half:].contiguous(), t[:, half:].contiguous(), seed=123, row_base=half,
                                   rows_per_sample=length - half, global_rows_per_sample=length, want_noise=True)
    torch.testing.assert_close(shard, noise[:, half:])


def test_adamw_matches_torch() -> None:
    ops = _ops()
    torch.manual_seed(8)
    n = 1000
    p = torch.randn(n, device=DEV)
    ref = p.clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    pb = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    for step in range(1, 4):
        g = torch.randn(n, device=DEV)
        ref.grad = g.clone()
        opt.step()
        ops.adamw_step(p, g, m, v, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, step=step, param_bf16=pb)
    torch.testing.assert_close(p, ref.detach(), rtol=1e-5, atol=1e-6)
    _close(pb, p, rtol=1e-2, atol=1e-2)
    out = torch.zeros(1, device=DEV)
    ops.sq_norm_(p, out)
    torch.testing.assert_close(out[0], p.pow(2).sum(), rtol=1e-4, atol=1e-4)


def _piecewise_groups(rows: int, groups: int, gen: torch.Generator) -> torch.Tensor:
    """Row -> modulation row, constant over random runs (like clean / noisy frames)."""
    cuts = torch.sort(torch.randint(0, rows, (groups * 2,), generator=gen)).values.tolist()
    out = torch.zeros(rows, dtype=torch.int32)
    g = 0
    for i, c in enumerate(cuts):
        out[c:] = (g + i) % groups
    return out


def test_grouped_modulation_kernels() -> None:
    ops = _ops()
    gen = torch.Generator().manual_seed(11)
    rows, w_, ng = 777, 384, 5
    groups_cpu = _piecewise_groups(rows, ng, gen)
    groups = groups_cpu.to(DEV)
    gl = groups_cpu.long().to(DEV)
    x = torch.randn(rows, w_, generator=gen).to(DEV).bfloat16()
    weight = (torch.rand(w_, generator=gen) + 0.5).to(DEV)
    mod = (torch.randn(ng, 3, w_, generator=gen) * 0.1).to(DEV)
    scale, shift, gate = mod[:, 0], mod[:, 1], mod[:, 2]
    y, rstd = ops.rmsnorm_mod(x, weight, scale, shift, groups=groups)
    xr = x.float().requires_grad_()
    modr = mod.clone().requires_grad_()
    wr = weight.clone().requires_grad_()
    ref = F.rms_norm(xr, (w_,), wr, 1e-6) * (1 + modr[:, 0][gl]) + modr[:, 1][gl]
    _close(y, ref)
    dy = torch.randn(rows, w_, generator=gen).to(DEV).bfloat16()
    ref.backward(dy.float())
    dmod = torch.zeros_like(mod)
    dw = torch.zeros(w_, device=DEV)
    dx = ops.rmsnorm_mod_bwd(x, rstd, dy, weight, scale, shift, dweight=dw, dscale=dmod[:, 0], dshift=dmod[:, 1],
                             groups=groups)
    _close(dx, xr.grad)
    _close(dw, wr.grad, rtol=1e-2, atol=1e-2)
    _close(dmod[:, :2], modr.grad[:, :2], rtol=1e-2, atol=1e-2)
    # gate backward and the gated-residual GEMM epilogue with the same groups
    a = torch.randn(rows, w_, generator=gen).to(DEV).bfloat16()
    da = ops.gate_bwd(dy, a, gate, dmod[:, 2], rows_per_batch=1, groups=groups)
    _close(da, dy.float() * gate[gl])
    ref_dg = torch.zeros(ng, w_, device=DEV).index_add_(0, gl, dy.float() * a.float())
    _close(dmod[:, 2], ref_dg, rtol=1e-2, atol=1e-2)
    wt = (torch.randn(w_, 256, generator=gen) * 0.05).to(DEV).bfloat16()
    resid = torch.randn(rows, w_, generator=gen).to(DEV).bfloat16()
    inp = torch.randn(rows, 256, generator=gen).to(DEV).bfloat16()
    got = ops.gemm(inp, wt, epilogue="gate_resid", resid=resid, gate=gate, groups=groups)
    _close(got, resid.float() + gate[gl] * (inp.float() @ wt.float().t()))
    _errors_clear()


@pytest.mark.parametrize("lq,lk", [(77, 16), (5, 130)])
def test_attention_odd_lengths(lq: int, lk: int) -> None:
    """Short and unaligned sequence lengths (text tokens): padded row statistics."""
    ops = _ops()
    torch.manual_seed(12)
    b, h, d = 2, 2, 128
    q = torch.randn(b, h, lq, d, device=DEV).bfloat16()
    k = torch.randn(b, h, lk, d, device=DEV).bfloat16()
    v = torch.randn(b, h, lk, d, device=DEV).bfloat16()
    out, lse = ops.attention_fwd(q, k, v)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    ref = _attn_ref(qr, kr, vr, None, 1.0 / math.sqrt(d))
    _close(out, ref)
    dout = torch.randn_like(ref).bfloat16()
    ref.backward(dout.float())
    dq, dk, dv = ops.attention_bwd(q, k, v, out, dout.contiguous(), lse)
    _close(dq, qr.grad, rtol=3e-2, atol=3e-2)
    _close(dk, kr.grad, rtol=3e-2, atol=3e-2)
    _close(dv, vr.grad, rtol=3e-2, atol=3e-2)
    _errors_clear()


@pytest.mark.parametrize("mode", ["fused", "split"])
def test_attention_bwd_variants_agree(mode: str, monkeypatch: pytest.MonkeyPatch) -> None:
    """Both backward variants (one-pass with dQ reduce-add, and two-pass) against fp32."""
    ops = _ops()
    monkeypatch.setattr(ops, "_ATTN_BWD", mode)
    torch.manual_seed(13)
    b, h, hk, lq, lk, d = 2, 4, 2, 517, 389, 128
    q = torch.randn(b, h, lq, d, device=DEV).bfloat16()
    k = torch.randn(b, hk, lk, d, device=DEV).bfloat16()
    v = torch.randn(b, hk, lk, d, device=DEV).bfloat16()
    kmask = torch.rand(b, lk, device=DEV) > 0.25
    kmask[1] = False  # a sample with no valid key: its rows attend to nothing
    packed = ops.pack_key_mask(kmask)
    out, lse = ops.attention_fwd(q, k, v, kmask=packed)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    ref = _attn_ref(qr, kr, vr, kmask, 1.0 / math.sqrt(d))
    ref = torch.where(kmask.any(-1)[:, None, None, None], ref, torch.zeros_like(ref))
    _close(out, ref)
    dout = torch.randn_like(ref).bfloat16()
    ref.backward(dout.float())
    dq, dk, dv = ops.attention_bwd(q, k, v, out, dout.contiguous(), lse, kmask=packed)
    for got, want in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        assert torch.isfinite(got.float()).all()
        _close(got, torch.nan_to_num(want), rtol=3e-2, atol=3e-2)
    _errors_clear()


def test_norm_column_reductions_many_rows() -> None:
    """More rows than a grid dimension holds, with and without modulation (per-token rows)."""
    ops = _ops()
    torch.manual_seed(14)
    rows, w_ = 70000, 256
    x = torch.randn(rows, w_, device=DEV).bfloat16()
    weight = torch.rand(w_, device=DEV) + 0.5
    y, rstd = ops.rmsnorm_mod(x, weight)
    dy = torch.randn(rows, w_, device=DEV).bfloat16()
    dw = torch.zeros(w_, device=DEV)
    dx = ops.rmsnorm_mod_bwd(x, rstd, dy, weight, dweight=dw)
    xr, wr = x.float().requires_grad_(), weight.clone().requires_grad_()
    ref = F.rms_norm(xr, (w_,), wr, 1e-6)
    ref.backward(dy.float())
    _close(y, ref)
    _close(dx, xr.grad)
    _close(dw, wr.grad, rtol=1e-2, atol=1e-2)
    # per-token modulation rows (rows_per_batch = 1)
    scale = torch.randn(rows, w_, device=DEV) * 0.1
    gate = torch.randn(rows, w_, device=DEV)
    ds = torch.zeros_like(scale)
    ops.rmsnorm_mod_bwd(x, rstd, dy, weight, scale, None, dscale=ds, rows_per_batch=1)
    _close(ds, dy.float() * F.rms_norm(x.float(), (w_,), weight, 1e-6), rtol=2e-2, atol=2e-2)
    dg = torch.zeros_like(gate)
    ops.gate_bwd(dy, x, gate, dg, rows_per_batch=1)
    _close(dg, dy.float() * x.float(), rtol=1e-2, atol=1e-2)
    _errors_clear()


def test_attention_trace_diagnostics_leave_results_unchanged() -> None:
    """The ``trace`` diagnostics only add clock stamps: outputs match an untraced call bit for bit."""
    ops = _ops()
    torch.manual_seed(0)
    q = torch.randn(1, 2, 512, 128, device=DEV).bfloat16()
    k, v = torch.randn_like(q), torch.randn_like(q)
    out, lse = ops.attention_fwd(q, k, v)
    tr = torch.zeros(64 * 24, dtype=torch.int64, device=DEV)
    out_t, lse_t = ops.attention_fwd(q, k, v, trace=tr)
    torch.cuda.synchronize()
    assert torch.equal(out, out_t) and torch.equal(lse, lse_t)
    assert int(tr.view(64, 24)[:4, 0].min()) > 0, "forward stamps missing"
    dout = torch.randn_like(out)
    ref = ops.attention_bwd(q, k, v, out, dout, lse)
    tr.zero_()
    got = ops.attention_bwd(q, k, v, out, dout, lse, trace=tr)
    torch.cuda.synchronize()
    for a, b in zip(ref, got):
        _close(b, a, rtol=1e-3, atol=1e-3)
    assert int(tr.view(64, 24)[:4, 0].min()) > 0, "backward stamps missing"
    _errors_clear()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_guided_euler_matches_torch(dtype: torch.dtype) -> None:
    ops = _ops()
    torch.manual_seed(0)
    b = 3
    x = torch.randn(b, 4, 3, 8, 8, device=DEV)
    cond = torch.randn_like(x).to(dtype)
    uncond = torch.randn_like(x).to(dtype)
    s = torch.tensor([0.9, 0.5, 0.2], device=DEV)
    sn = torch.tensor([0.7, 0.4, 0.0], device=DEV)
    got = ops.guided_euler(cond, uncond, x, s, sn, scale=5.0)
    v = uncond.float() + 5.0 * (cond.float() - uncond.float())
    ref = x + (sn - s).view(b, 1, 1, 1, 1) * v
    _close(got, ref, rtol=1e-5, atol=1e-5)
    plain = ops.guided_euler(cond, None, x, s, sn)
    _close(plain, x + (sn - s).view(b, 1, 1, 1, 1) * cond.float(), rtol=1e-5, atol=1e-5)


def test_sde_step_matches_torch_oracle() -> None:
    from avgen_b200.rl.sde import diffusion_coefficient

    ops = _ops()
    torch.manual_seed(0)
    b = 4
    x = torch.randn(b, 16, 4, 16, 16, device=DEV)
    v = torch.randn_like(x)
    s = torch.tensor([0.95, 0.6, 0.3, 0.1], device=DEV)
    sn = torch.tensor([0.9, 0.5, 0.2, 0.0], device=DEV)
    g = diffusion_coefficient(s, noise_level=0.7)
    z = torch.randn_like(x)
    sample, mean, logp = ops.sde_step(v, x, s, sn, g, floor=1e-3, noise=z)
    sb = s.clamp_min(1e-3).view(b, 1, 1, 1, 1)
    ref_mean = x + (v + (g * g).view(b, 1, 1, 1, 1) / (2 * sb) * (x + (1 - sb) * v)) * (sn - s).view(b, 1, 1, 1, 1)
    std = g * (s - sn).abs().sqrt()
    ref_sample = ref_mean + std.view(b, 1, 1, 1, 1) * z
    zz = ((ref_sample - ref_mean) / std.view(b, 1, 1, 1, 1)).flatten(1).double()
    n = x[0].numel()
    ref_logp = -0.5 * (zz ** 2).sum(1) - n * torch.log(std.double()) - n * 0.5 * math.log(2 * math.pi)
    _close(mean, ref_mean, rtol=1e-5, atol=1e-5)
    _close(sample, ref_sample, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(logp.double(), ref_logp, rtol=1e-4, atol=1.0)
    # update mode scores a stored state; a mask drops elements from the sum
    mask = torch.rand_like(x) > 0.3
    _, mean2, logp2 = ops.sde_step(v, x, s, sn, g, floor=1e-3, prev=ref_sample, mask=mask)
    _close(mean2, ref_mean, rtol=1e-5, atol=1e-5)
    per = -0.5 * ((ref_sample - ref_mean) / std.view(b, 1, 1, 1, 1)) ** 2 - torch.log(std).view(b, 1, 1, 1, 1) \
        - 0.5 * math.log(2 * math.pi)
    torch.testing.assert_close(logp2.double(), (per * mask).flatten(1).sum(1).double(), rtol=1e-4, atol=1.0)
    _errors_clear()


def _ring_reference(q, k_all, v_all, kmask, scale):  # noqa: ANN001, ANN202
    """Plain fp32 attention over the concatenated ring slabs ([world, B, Hk, L, D] -> [B, Hk, world*L, D])."""
    world, b, hk, length, d = k_all.shape
    kf = k_all.permute(1, 2, 0, 3, 4).reshape(b, hk, world * length, d).float()
    vf = v_all.permute(1, 2, 0, 3, 4).reshape(b, hk, world * length, d).float()
    rep = q.shape[1] // hk
    kf, vf = kf.repeat_interleave(rep, 1), vf.repeat_interleave(rep, 1)
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), kf) * scale
    if kmask is not None:
        s = s.masked_fill(~kmask[:, None, None, :], float("-inf"))
    return torch.einsum("bhqk,bhkd->bhqd", s.softmax(-1), vf)


@pytest.mark.parametrize("masked", [False, True])
def test_ring_attention_gates_on_copied_slabs(masked: bool) -> None:
    """World 3 emulated on one GPU: slabs 1 and 2 arrive by copy engine behind a
    large unrelated copy on the copy stream, each followed by a front-end flag
    write, while the kernel (launched at once) gates each slab on its flag;
    results match attention over the whole sequence, forward and backward
    (dK/dV come back per slab). No stream waits on a flag."""
    from avgen_b200.ops._ext import load

    ops, ext = _ops(), load()
    torch.manual_seed(0)
    world, b, h, hk, length, d = 3, 1, 4, 2, 256, 128
    me = 0
    q = torch.randn(b, h, length, d, device=DEV).bfloat16()
    src_k = torch.randn(world, b, hk, length, d, device=DEV).bfloat16()
    src_v = torch.randn(world, b, hk, length, d, device=DEV).bfloat16()
    k_all = torch.zeros_like(src_k)
    v_all = torch.zeros_like(src_v)
    k_all[me].copy_(src_k[me])
    v_all[me].copy_(src_v[me])
    flags = torch.zeros(world, dtype=torch.int32, device=DEV)
    kmask = packed = None
    if masked:
        kmask = torch.ones(b, world * length, dtype=torch.bool, device=DEV)
        kmask[:, 300:400] = False
        packed = ops.pack_key_mask(kmask)
    ballast = torch.empty(1 << 28, dtype=torch.uint8, device=DEV)  # 256 MB: delays the slab copies
    ballast2 = torch.empty_like(ballast)
    torch.cuda.synchronize()
    epoch = 7
    copy = torch.cuda.Stream()
    slab = src_k[0].numel() * 2
    with torch.cuda.stream(copy):
        ext.p2p_copy(ballast2.data_ptr(), ballast.data_ptr(), ballast.numel())
        for r in (1, 2):
            ext.p2p_copy(k_all[r].data_ptr(), src_k[r].data_ptr(), slab)
            ext.p2p_copy(v_all[r].data_ptr(), src_v[r].data_ptr(), slab)
            ext.stream_write(flags.data_ptr() + 4 * r, epoch)
    scale = 1.0 / math.sqrt(d)
    out, lse = ops.attention_fwd(q, k_all, v_all, kmask=packed, scale=scale, ring_rank=me, ring_flags=flags,
                                 ring_epoch=epoch)
    torch.cuda.synchronize()
    _errors_clear()
    ref = _ring_reference(q, src_k, src_v, kmask, scale)
    _close(out.permute(0, 2, 1, 3), ref)
    # backward against autograd on the fp32 reference
    do = torch.randn(b, length, h, d, device=DEV).bfloat16()
    dq, dk_all, dv_all = ops.attention_bwd(q, k_all, v_all, out, do, lse, kmask=packed, scale=scale)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, src_k, src_v))
    ref2 = _ring_reference(qr, kr, vr, kmask, scale)
    ref2.backward(do.permute(0, 2, 1, 3).float())
    _close(dq, qr.grad, rtol=3e-2, atol=3e-2)
    assert dk_all.shape == src_k.shape
    _close(dk_all, kr.grad, rtol=3e-2, atol=3e-2)
    _close(dv_all, vr.grad, rtol=3e-2, atol=3e-2)
    # the same backward split into one launch per slab (remote slabs first)
    seen = []
    dq2, dk2, dv2 = ops.attention_bwd_slabs(q, k_all, v_all, out, do, lse, order=[1, 2, 0], kmask=packed,
                                            scale=scale, on_slab=lambda r, a, b_: seen.append(r))
    torch.cuda.synchronize()
    assert seen == [1, 2, 0]
    _close(dq2, dq, rtol=1e-2, atol=1e-2)
    _close(dk2, dk_all, rtol=1e-2, atol=1e-2)
    _close(dv2, dv_all, rtol=1e-2, atol=1e-2)
    _errors_clear()


def test_slab_sum_matches_fp32() -> None:
    ops = _ops()
    torch.manual_seed(0)
    parts = [torch.randn(2, 3, 256, 128, device=DEV).bfloat16() for _ in range(4)]
    out = ops.slab_sum(parts, torch.empty_like(parts[0]))
    _close(out, sum(p.float() for p in parts), rtol=1e-2, atol=1e-2)


def test_ring_attention_times_out_without_its_slab() -> None:
    """A slab whose flag never arrives makes the kernel give up after its bounded
    wait and report it in the error word; the context stays usable."""
    from avgen_b200.ops._ext import check_errors

    ops = _ops()
    world, b, h, length, d = 2, 1, 2, 128, 128
    q = torch.randn(b, h, length, d, device=DEV).bfloat16()
    k_all = torch.randn(world, b, h, length, d, device=DEV).bfloat16()
    flags = torch.zeros(world, dtype=torch.int32, device=DEV)
    ops.attention_fwd(q, k_all, k_all.clone(), ring_rank=0, ring_flags=flags, ring_epoch=1)
    torch.cuda.synchronize()
    assert check_errors(clear=True) == 5  # timed out waiting on a peer's slab
    out, _ = ops.attention_fwd(q, k_all[0], k_all[0])  # the device still works
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    _errors_clear()


@pytest.mark.skipif(os.environ.get("AVGEN_LORA_FUSED", "0") != "1",
                    reason="opt-in fused LoRA path: a host crash at 8192 rows is not yet explained")
@pytest.mark.parametrize("m,n,k,r", [(384, 512, 256, 16), (200, 264, 136, 8), (256, 256, 128, 72)])
def test_gemm_appended_pair_and_fused_lora_linear(m: int, n: int, k: int, r: int) -> None:
    """``[a | a2] . [b | b2]^T`` in one accumulator (K-major and dX layouts), and a
    LoRA layer on that path matching the fp32 eager adapter, forward and backward."""
    ops = _ops()
    torch.manual_seed(11)
    a = torch.randn(m, k, device=DEV).bfloat16()
    b = torch.randn(n, k, device=DEV).bfloat16() * 0.1
    a2 = torch.randn(m, r, device=DEV).bfloat16()
    b2 = torch.randn(n, r, device=DEV).bfloat16() * 0.1
    bias = torch.randn(n, device=DEV)
    ref = a.float() @ b.float().t() + a2.float() @ b2.float().t() + bias
    _close(ops.gemm(a, b, bias=bias, a2=a2, b2=b2), ref)
    dy = torch.randn(m, n, device=DEV).bfloat16()
    u = torch.randn(m, r, device=DEV).bfloat16()
    sa = torch.randn(r, k, device=DEV).bfloat16() * 0.1
    _close(ops.linear_dx(dy, b, a2=u, b2=sa), dy.float() @ b.float() + u.float() @ sa.float())
    with pytest.raises(RuntimeError):
        ops.gemm(a, b, a2=a2)  # a2 without b2

    from avgen_b200.finetune.lora import LoRALinear
    from avgen_b200.models.linear import _lora_fusable, linear

    base = torch.nn.Linear(k, n, device=DEV)
    layer = LoRALinear.from_linear(base, rank=r, alpha=2.0 * r)
    with torch.no_grad():
        layer.lora_b.normal_(0, 0.05)
    layer.weight.requires_grad_(False)
    assert _lora_fusable(layer)
    x = torch.randn(2, m // 2, k, device=DEV, requires_grad=True)
    g = torch.randn(2, m // 2, n, device=DEV)
    y = linear(x.bfloat16(), layer)
    y.float().backward(g)
    got = (y.detach(), x.grad.clone(), layer.lora_a.grad.clone(), layer.lora_b.grad.clone())
    xr = x.detach().clone().requires_grad_()
    ar = layer.lora_a.detach().clone().requires_grad_()
    br = layer.lora_b.detach().clone().requires_grad_()
    yr = xr @ layer.weight.t() + layer.bias + (xr @ ar.t()) @ br.t() * layer.scaling
    yr.backward(g)
    _close(got[0], yr)
    _close(got[1], xr.grad)
    _close(got[2], ar.grad, rtol=3e-2, atol=3e-2)
    _close(got[3], br.grad, rtol=3e-2, atol=3e-2)
    assert layer.weight.grad is None
    _errors_clear()


@pytest.mark.parametrize("operand,world,rows,rank", [("b", 4, 200, 2), ("b", 2, 512, 1), ("a", 4, 192, 3),
                                                     ("a", 8, 128, 5)])
def test_gemm_gated_operand_rotation_and_chunks(operand: str, world: int, rows: int, rank: int) -> None:
    """Gated-operand GEMM with every peer chunk already arrived: the tile rotation
    and the per-chunk waits (chunks that straddle tiles) leave the product exact."""
    ops = _ops()
    torch.manual_seed(5)
    k = 320
    full = torch.randn(world * rows, k, device=DEV).bfloat16()
    other = torch.randn(264 if operand == "b" else 392, k, device=DEV).bfloat16()
    flags = torch.full((world,), 7, dtype=torch.int32, device=DEV)
    flags[rank] = 0  # the own chunk is never waited on
    a, b = (other, full) if operand == "b" else (full, other)
    got = ops.gemm(a, b, gate_flags=flags, gate_epoch=7, gate_operand=operand, gate_chunk=rows, gate_rank=rank)
    _close(got, a.float() @ b.float().t())
    _errors_clear()


def test_gemm_gated_operand_times_out_without_its_chunk() -> None:
    """A chunk whose flag never arrives: the tiles reading it give up after the
    bounded wait, the error word says so, and the device stays usable."""
    from avgen_b200.ops._ext import check_errors

    ops = _ops()
    x = torch.randn(256, 128, device=DEV).bfloat16()
    w = torch.randn(2 * 256, 128, device=DEV).bfloat16()
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)
    ops.gemm(x, w, gate_flags=flags, gate_epoch=1, gate_operand="b", gate_chunk=256, gate_rank=0)
    torch.cuda.synchronize()
    assert check_errors(clear=True) == 5
    _close(ops.gemm(x, w), x.float() @ w.float().t())
    _errors_clear()


def test_deterministic_weight_gradient_is_bitwise_repeatable() -> None:
    """The weight-gradient GEMM unsplit (deterministic mode) gives bitwise-identical
    results on repeated runs and agrees with the split-K atomic form to fp32 rounding."""
    from avgen_b200.ops import kernels as K

    torch.manual_seed(4)
    dy = torch.randn(8192, 512, device=DEV).bfloat16()
    x = torch.randn(8192, 768, device=DEV).bfloat16()
    try:
        K.set_deterministic(True)
        runs = []
        for _ in range(3):
            g = torch.zeros(512, 768, device=DEV)
            K.linear_dw(dy, x, g)
            runs.append(g)
    finally:
        K.set_deterministic(False)
    assert torch.equal(runs[0], runs[1]) and torch.equal(runs[0], runs[2])
    split = torch.zeros(512, 768, device=DEV)
    K.linear_dw(dy, x, split, k_splits=8)
    ref = dy.float().T @ x.float()
    _close(runs[0], ref)
    _close(split, ref)
    _errors_clear()
