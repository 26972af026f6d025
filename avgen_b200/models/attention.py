"""The single attention entry point.

On a B200 every attention (self, cross, text refiner, AV fusion) runs the
hand-written tcgen05 flash-attention kernels (``csrc/attention.cu``) through the
:class:`FlashAttention` autograd function. On the CPU it is the plain fp32
PyTorch reference used as the numerics oracle. The reference framework's
equivalent is avgen/models/attention.py:98-273 (an SDPA call with a
cuDNN-first backend list); its key-padding helper (``key_padding_mask``) keeps
the same semantics here.
"""
from __future__ import annotations

import math

import torch

__all__ = ["FlashAttention", "attention", "attention_backends", "device_arch", "key_padding_mask",
           "reference_attention", "sdpa_context"]

_ARCH_BY_MAJOR = ((10, "blackwell"), (9, "hopper"), (8, "ampere"), (0, "legacy"))


def device_arch(device: torch.device | str | None = None) -> str:
    """``"blackwell"`` on sm_100, ``"cpu"`` without CUDA, etc."""
    dev = torch.device(device) if device is not None else torch.device("cuda" if torch.cuda.is_available() else "cpu")
    if dev.type != "cuda" or not torch.cuda.is_available():
        return "cpu"
    major, _ = torch.cuda.get_device_capability(dev)
    return next(name for floor, name in _ARCH_BY_MAJOR if major >= floor)


def key_padding_mask(mask: torch.Tensor | None, *, assume_dense: bool = False) -> torch.Tensor | None:
    """``(B, L)`` bool validity, or ``None`` when every key is known to be valid.

    On CUDA the mask is returned as given, without testing whether every key is
    valid: that test reads a device value on the host and so waits for the
    device to drain its queue. The kernels apply an all-valid mask at the cost of
    a few bit loads per key tile. On the CPU an all-valid mask becomes ``None``."""
    if mask is None or assume_dense:
        return None
    if mask.ndim != 2:
        raise ValueError(f"key mask must have rank 2 (batch, keys); got {tuple(mask.shape)}")
    if mask.dtype is not torch.bool:
        raise TypeError(f"key mask must be bool; got {mask.dtype}")
    if mask.numel() == 0:
        return None
    if mask.is_cuda:
        return mask
    if bool(mask.all()):
        return None
    return mask


class FlashAttention(torch.autograd.Function):
    """tcgen05 flash attention with a key-padding bitmask; q ``[B,H,L,D]`` in, ``[B,L,H,D]`` out."""

    @staticmethod
    def forward(ctx, q, k, v, key_mask, scale):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        packed = K.pack_key_mask(key_mask) if key_mask is not None else None
        qb, kb, vb = (t.to(torch.bfloat16).contiguous() for t in (q, k, v))
        out, lse = K.attention_fwd(qb, kb, vb, kmask=packed, scale=scale)
        ctx.save_for_backward(qb, kb, vb, out, lse, packed if packed is not None else torch.empty(0))
        ctx.scale = scale
        ctx.has_mask = packed is not None
        ctx.dtypes = (q.dtype, k.dtype, v.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        qb, kb, vb, out, lse, packed = ctx.saved_tensors
        dq, dk, dv = K.attention_bwd(qb, kb, vb, out, dout.to(torch.bfloat16).contiguous(), lse,
                                     kmask=packed if ctx.has_mask else None, scale=ctx.scale)
        return dq.to(ctx.dtypes[0]), dk.to(ctx.dtypes[1]), dv.to(ctx.dtypes[2]), None, None


def attention_backends(device: torch.device | str | None = None, *, allow_flash: bool = True) -> tuple:
    """Priority list of ``torch.nn.functional.scaled_dot_product_attention`` backends for
    SDPA calls made outside this framework's kernels (user code, plugins): cuDNN first
    on Blackwell and Hopper, then flash, memory-efficient and math; math alone on the
    CPU. The framework's own attention never calls SDPA (see :func:`attention`)."""
    from torch.nn.attention import SDPBackend

    if device_arch(device) == "cpu":
        return (SDPBackend.MATH,)
    order = [SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]
    if device_arch(device) not in ("blackwell", "hopper"):
        order.remove(SDPBackend.CUDNN_ATTENTION)
    if not allow_flash:
        order.remove(SDPBackend.FLASH_ATTENTION)
    return tuple(order)


def sdpa_context(device: torch.device | str | None = None, *, backends=None):  # noqa: ANN001, ANN201
    """A context pinning SDPA's backend priority (``backends`` or
    :func:`attention_backends`) on CUDA; a no-op on the CPU, which has one kernel."""
    import contextlib

    if device_arch(device) == "cpu":
        return contextlib.nullcontext()
    from torch.nn.attention import sdpa_kernel

    chosen = list(backends) if backends is not None else list(attention_backends(device))
    try:
        return sdpa_kernel(chosen, set_priority=True)
    except TypeError:  # builds without priority ordering take the set only
        return sdpa_kernel(chosen)


def reference_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, key_mask: torch.Tensor | None,
                        scale: float) -> torch.Tensor:
    """fp32 oracle with the kernels' semantics (a query with no valid key gets 0).

    Returns the token-major ``(B, Lq, H, D)`` layout.
    """
    rep = q.shape[1] // k.shape[1]
    if rep > 1:
        k = k.repeat_interleave(rep, 1)
        v = v.repeat_interleave(rep, 1)
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    if key_mask is not None:
        s = s.masked_fill(~key_mask[:, None, None, :], float("-inf"))
    m = s.amax(-1, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(s - m)
    den = p.sum(-1, keepdim=True)
    out = (p @ v.float()) / torch.where(den > 0, den, torch.ones_like(den))
    return out.to(q.dtype).transpose(1, 2)


def attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *,
              key_mask: torch.Tensor | None = None, scale: float | None = None,
              layout: str = "bhld") -> torch.Tensor:
    """Bidirectional attention with an optional key-padding mask and GQA.

    Args:
        query: ``(B, H, Lq, D)``.
        key, value: ``(B, Hk, Lk, D)`` with ``H % Hk == 0``.
        key_mask: ``(B, Lk)`` bool validity or ``None``.
        scale: softmax scale, default ``1/sqrt(D)``.
        layout: ``"bhld"`` returns ``(B, H, Lq, D)``; ``"blhd"`` returns the
            token-major ``(B, Lq, H, D)`` the kernels produce natively.
    """
    if query.shape[-2] == 0 or key.shape[-2] == 0:
        out = torch.zeros_like(query)
        return out if layout == "bhld" else out.transpose(1, 2)
    d = query.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    if query.device.type == "cuda":
        if d != 128:
            raise NotImplementedError(f"the sm_100a attention kernels support head_dim 128; got {d}")
        out = FlashAttention.apply(query, key, value, key_mask, scale).to(query.dtype)
    else:
        out = reference_attention(query, key, value, key_mask, scale)
    return out.transpose(1, 2) if layout == "bhld" else out
