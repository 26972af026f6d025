"""PyTorch stand-ins for the sm_100a kernel wrappers the fused DiT block calls.

Each function restates, in fp32 PyTorch on whatever device its inputs live, the
contract documented on the wrapper it replaces in ``avgen_b200.ops.kernels``
(shapes, layouts, dtypes of the outputs, which arguments accumulate). With
:func:`emulate_kernels` active the fused block's own orchestration -- packed
weights, recompute versus kept intermediates, modulation rows, weight-gradient
routing (dense, low-rank LoRA, adapters' effective weights), the tensor-parallel
collectives and the gradient order handed back to autograd -- runs on CPU, so it
can be checked against the eager block without a GPU. The kernels themselves are
checked against fp32 on the GPU by the ``gpu``-marked tests.
"""
from __future__ import annotations

import contextlib
import math
from collections.abc import Iterator

import torch
import torch.nn.functional as F

_BF16 = torch.bfloat16
_F32 = torch.float32


def _rows(t: torch.Tensor, count: int, rows_per_batch: int, groups: torch.Tensor | None) -> torch.Tensor:
    """Row ``i`` of the result is ``t[groups[i]]`` or ``t[i // rows_per_batch]``."""
    if groups is not None:
        idx = groups.long()
    else:
        idx = torch.arange(count, device=t.device) // max(1, rows_per_batch)
    return t.float()[idx]


def _group_index(count: int, rows_per_batch: int, groups: torch.Tensor | None, device: torch.device) -> torch.Tensor:
    if groups is not None:
        return groups.long()
    return torch.arange(count, device=device) // max(1, rows_per_batch)


def gemm(a, b, *, a_mn=False, b_mn=False, epilogue="store", out=None, out_dtype=_BF16, bias=None, resid=None,  # noqa: ANN001, ANN201, C901
         gate=None, rows_per_batch=1, aux=None, k_splits=1, groups=None, a2=None, b2=None, gate_flags=None,
         gate_epoch=0, gate_operand="", gate_chunk=0, gate_rank=0):
    mat_a = (a.t() if a_mn else a).float()
    mat_b = (b.t() if b_mn else b).float()
    acc = mat_a @ mat_b.t()
    if a2 is not None:
        acc = acc + (a2.t() if a_mn else a2).float() @ (b2.t() if b_mn else b2).float().t()
    if bias is not None:
        acc = acc + bias.float()
    if epilogue == "atomic":
        out.add_(acc)
        return out
    if aux is not None:
        aux.copy_(acc)
    if epilogue == "store":
        res = acc
    elif epilogue == "gate_resid":
        g = _rows(gate, acc.shape[0], rows_per_batch, groups) if gate is not None else 1.0
        res = resid.float() + g * acc
    elif epilogue == "swiglu":
        res = F.silu(acc[:, 0::2]) * acc[:, 1::2]
    elif epilogue == "gelu":
        res = F.gelu(acc, approximate="tanh")
    else:
        raise ValueError(epilogue)
    if out is None:
        out = torch.empty(res.shape, device=res.device, dtype=out_dtype)
    out.copy_(res)
    return out


def linear_dx(dy, w, out_dtype=_BF16, *, a2=None, b2=None):  # noqa: ANN001, ANN201
    return gemm(dy, w, b_mn=True, out_dtype=out_dtype, a2=a2, b2=b2)


def linear_dw(dy, x, grad, *, k_splits=0):  # noqa: ANN001, ANN201
    return gemm(dy, x, a_mn=True, b_mn=True, epilogue="atomic", out=grad)


def _norm_mod(xf, rstd, weight, scale, shift, rows_per_batch, groups):  # noqa: ANN001, ANN202
    y = xf * rstd[:, None]
    if weight is not None:
        y = y * weight.float()
    if scale is not None:
        y = y * (1.0 + _rows(scale, xf.shape[0], rows_per_batch, groups))
    if shift is not None:
        y = y + _rows(shift, xf.shape[0], rows_per_batch, groups)
    return y


def rmsnorm_mod(x, weight, scale=None, shift=None, *, rows_per_batch=1, eps=1e-6, out=None, want_rstd=True,  # noqa: ANN001, ANN201
                groups=None):
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    y = _norm_mod(xf, rstd, weight, scale, shift, rows_per_batch, groups)
    out = out if out is not None else torch.empty_like(x)
    out.copy_(y)
    return out, (rstd if want_rstd else None)


def rmsnorm_mod_bwd(x, rstd, dy, weight, scale=None, shift=None, *, dres=None, dweight=None, dscale=None,  # noqa: ANN001, ANN201
                    dshift=None, rows_per_batch=1, dx=None, groups=None):
    xf, dyf = x.float(), dy.float()
    n = xf.shape[0]
    xhat = xf * rstd[:, None]
    mult = torch.ones_like(xf)
    if weight is not None:
        mult = mult * weight.float()
    if scale is not None:
        mult = mult * (1.0 + _rows(scale, n, rows_per_batch, groups))
    g = dyf * mult
    grad = rstd[:, None] * (g - xhat * (g * xhat).mean(-1, keepdim=True))
    if dres is not None:
        grad = grad + dres.float()
    idx = _group_index(n, rows_per_batch, groups, x.device)
    if dweight is not None:
        pre = 1.0 + _rows(scale, n, rows_per_batch, groups) if scale is not None else 1.0
        dweight.add_((dyf * xhat * pre).sum(0))
    if dscale is not None:
        w = weight.float() if weight is not None else 1.0
        dscale.index_add_(0, idx, dyf * xhat * w)
    if dshift is not None:
        dshift.index_add_(0, idx, dyf)
    dx = dx if dx is not None else torch.empty_like(x)
    dx.copy_(grad)
    return dx


def gate_bwd(dx, a, gate, dgate, *, rows_per_batch, groups=None):  # noqa: ANN001, ANN201
    n = dx.shape[0]
    da = torch.empty_like(dx)
    da.copy_(dx.float() * _rows(gate, n, rows_per_batch, groups))
    dgate.index_add_(0, _group_index(n, rows_per_batch, groups, dx.device), dx.float() * a.float())
    return da


def _head_norm(t: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    if weight is None:
        return t
    return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * weight


def _rotate(t: torch.Tensor, coords, freq, axis) -> torch.Tensor:  # noqa: ANN001
    """Rotate interleaved channel pairs of ``t [B, L, H, D]`` by ``coords[..., axis] * freq``."""
    if coords is None:
        return t
    phase = coords.float()[..., axis.long()] * freq.float()  # [B, L, P]
    cos, sin = torch.cos(phase)[:, :, None], torch.sin(phase)[:, :, None]
    pairs = t.unflatten(-1, (-1, 2))
    even, odd = pairs[..., 0], pairs[..., 1]
    return torch.stack((even * cos - odd * sin, even * sin + odd * cos), -1).flatten(-2)


def _qkv_parts(qkv_f, batch, length, heads, kv_heads, head_dim, q_weight, k_weight, coords, freq, axis, eps):  # noqa: ANN001, ANN202
    x = qkv_f.view(batch, length, heads + 2 * kv_heads, head_dim)
    q = x[:, :, :heads]
    k = x[:, :, heads:heads + kv_heads]
    v = x[:, :, heads + kv_heads:]
    q = _rotate(_head_norm(q, q_weight, eps), coords, freq, axis) if heads else None
    k = _rotate(_head_norm(k, k_weight, eps), coords, freq, axis) if kv_heads else None
    return (q.transpose(1, 2) if heads else None, k.transpose(1, 2) if kv_heads else None,
            v.transpose(1, 2) if kv_heads else None)


def qkv_rope(qkv, *, batch, length, heads, kv_heads, head_dim, q_weight, k_weight, coords, freq, axis, eps=1e-6,  # noqa: ANN001, ANN201
             k_out=None, v_out=None):
    q, k, v = _qkv_parts(qkv.float(), batch, length, heads, kv_heads, head_dim, q_weight, k_weight, coords, freq,
                         axis, eps)
    q = q.to(_BF16).contiguous() if q is not None else None
    if k is not None:
        k = k_out.copy_(k) if k_out is not None else k.to(_BF16).contiguous()
        v = v_out.copy_(v) if v_out is not None else v.to(_BF16).contiguous()
    return q, k, v


def qkv_rope_bwd(qkv, dq, dk, dv, *, batch, length, heads, kv_heads, head_dim, q_weight, k_weight, coords, freq,  # noqa: ANN001, ANN201
                 axis, dq_weight=None, dk_weight=None, eps=1e-6):
    with torch.enable_grad():
        x = qkv.detach().float().requires_grad_(True)
        qw = q_weight.detach().float().requires_grad_(True) if q_weight is not None else None
        kw = k_weight.detach().float().requires_grad_(True) if k_weight is not None else None
        q, k, v = _qkv_parts(x, batch, length, heads, kv_heads, head_dim, qw, kw, coords, freq, axis, eps)
        outs, grads = [], []
        for t, g in ((q, dq), (k, dk), (v, dv)):
            if t is not None and g is not None:
                outs.append(t)
                grads.append(g.float())
        inputs = [x] + [w for w in (qw, kw) if w is not None]
        got = torch.autograd.grad(outs, inputs, grads, allow_unused=True)
    i = 1
    if qw is not None:
        if dq_weight is not None and got[i] is not None:
            dq_weight.add_(got[i])
        i += 1
    if kw is not None and dk_weight is not None and got[i] is not None:
        dk_weight.add_(got[i])
    dqkv = torch.empty_like(qkv)
    dqkv.copy_(got[0])
    return dqkv


def _unpack_mask(kmask: torch.Tensor | None, length: int) -> torch.Tensor | None:
    if kmask is None:
        return None
    bits = torch.arange(32, device=kmask.device, dtype=torch.int64)
    words = kmask.to(torch.int64) & 0xFFFFFFFF
    flat = ((words[..., None] >> bits) & 1).flatten(-2)
    return flat[:, :length].bool()


def _attend(q, k, v, kmask, scale):  # noqa: ANN001, ANN202
    """q [B, H, Lq, D], k/v [B, Hk, Lk, D] in fp32 -> (out [B, Lq, H, D], lse base 2 [B, H, Lq])."""
    rep = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    s = (q @ k.transpose(-1, -2)) * scale
    keep = _unpack_mask(kmask, k.shape[2])
    if keep is not None:
        s = s.masked_fill(~keep[:, None, None, :], float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.exp(s - lse[..., None])
    return (p @ v).transpose(1, 2), lse / math.log(2.0)


def attention_fwd(q, k, v, *, kmask=None, scale=None, out=None, want_lse=True, **_ring):  # noqa: ANN001, ANN003, ANN201
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    o, lse = _attend(q.float(), k.float(), v.float(), kmask, scale)
    out = out if out is not None else torch.empty(o.shape, device=q.device, dtype=_BF16)
    out.copy_(o)
    return out, (lse if want_lse else None)


def attention_bwd(q, k, v, o, dout, lse, *, kmask=None, scale=None, trace=None):  # noqa: ANN001, ANN201
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    with torch.enable_grad():
        qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
        out, _ = _attend(qf, kf, vf, kmask, scale)
        dq, dk, dv = torch.autograd.grad(out, (qf, kf, vf), dout.float())
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def swiglu_bwd(dh, gu):  # noqa: ANN001, ANN201
    g, u = gu.float()[:, 0::2], gu.float()[:, 1::2]
    d = dh.float()
    sig = torch.sigmoid(g)
    dg = d * u * sig * (1.0 + g * (1.0 - sig))
    du = d * g * sig
    dgu = torch.empty_like(gu)
    dgu[:, 0::2] = dg.to(gu.dtype)
    dgu[:, 1::2] = du.to(gu.dtype)
    return dgu


def gelu_bwd(dh, pre):  # noqa: ANN001, ANN201
    with torch.enable_grad():
        x = pre.detach().float().requires_grad_(True)
        (g,) = torch.autograd.grad(F.gelu(x, approximate="tanh"), x, dh.float())
    return g.to(pre.dtype)


_REPLACED = ("gemm", "linear_dx", "linear_dw", "rmsnorm_mod", "rmsnorm_mod_bwd", "gate_bwd", "qkv_rope",
             "qkv_rope_bwd", "attention_fwd", "attention_bwd", "swiglu_bwd", "gelu_bwd")


@contextlib.contextmanager
def emulate_kernels() -> Iterator[None]:
    """Replace the kernel wrappers the fused block calls with the functions above."""
    from avgen_b200.ops import kernels as K

    saved = {name: getattr(K, name) for name in _REPLACED}
    here = globals()
    try:
        for name in _REPLACED:
            setattr(K, name, here[name])
        yield
    finally:
        for name, fn in saved.items():
            setattr(K, name, fn)
