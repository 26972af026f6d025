"""Linear layers on the tcgen05 GEMM.

``linear(x, layer)`` runs ``x @ W^T + b`` through the sm_100a GEMM kernel on CUDA
(bf16 operands, fp32 accumulation, fp32 master weights cast once per optimizer
step through :func:`bf16_weight`), and through ``F.linear`` on the CPU (the fp32
oracle). Weight gradients accumulate in fp32 with the GEMM's atomic epilogue.

With ``AVGEN_LORA_FUSED=1``, a plain LoRA layer (no DoRA, not merged, no
adapter dropout, rank a multiple of 8) runs as one GEMM with an appended rank-r
reduction pair instead of materialising ``W + s B A`` (see
:class:`LoRAKernelLinear`). It is opt-in: a microbenchmark of it at 8192 rows
ended in a host segmentation fault inside the GEMM launch of its backward whose
cause is not yet found; by default LoRA layers run one GEMM on the effective
weight.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F
from torch import nn

__all__ = ["KernelLinear", "LoRAKernelLinear", "bf16_weight", "bump_weight_epoch", "linear", "weight_epoch"]

_CACHE_ATTR = "_avgen_bf16_cache"
_EPOCH = [0]


def bump_weight_epoch() -> None:
    """Invalidate every cached bf16 weight copy (called after optimizer kernels
    update parameters through raw pointers, which does not bump version counters)."""
    _EPOCH[0] += 1


def weight_epoch() -> int:
    return _EPOCH[0]


def bf16_weight(param: torch.Tensor, *, key: str = "w", build=None) -> torch.Tensor:  # noqa: ANN001
    """A bf16 copy of ``param`` (or of ``build(param)``), rebuilt only when it changes.

    The cache is keyed on the parameter's version counter, which in-place
    optimizer updates bump, so the cast costs one pass per optimizer step rather
    than one per forward / recompute.
    """
    cache = getattr(param, _CACHE_ATTR, None)
    if cache is None:
        cache = {}
        try:
            setattr(param, _CACHE_ATTR, cache)
        except (AttributeError, RuntimeError):
            pass
    version = (param._version, param.data_ptr(), tuple(param.shape), _EPOCH[0])
    hit = cache.get(key)
    if hit is not None and hit[0] == version:
        return hit[1]
    with torch.no_grad():
        value = build(param) if build is not None else param.detach().to(torch.bfloat16).contiguous()
    cache[key] = (version, value)
    return value


def _weight_grad_buffer(weight: torch.Tensor) -> torch.Tensor:
    return torch.zeros(weight.shape, device=weight.device, dtype=torch.float32)


class KernelLinear(torch.autograd.Function):
    """``y = x W^T + b`` on the tcgen05 GEMM with fp32 weight-gradient accumulation."""

    @staticmethod
    def forward(ctx, x, weight, bias):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        w = bf16_weight(weight)
        b = bias.detach().float().contiguous() if bias is not None else None
        y = K.gemm(x2, w, bias=b)
        ctx.save_for_backward(x2, weight)
        ctx.has_bias = bias is not None
        ctx.in_dtype = x.dtype
        ctx.shape = shape
        return y.view(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        x2, weight = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16).contiguous()
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = K.linear_dx(dy2, bf16_weight(weight)).view(*ctx.shape).to(ctx.in_dtype)
        if ctx.needs_input_grad[1]:
            dw = _weight_grad_buffer(weight)
            K.linear_dw(dy2, x2, dw)
            dw = dw.to(weight.dtype)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = dy2.float().sum(0)
        return dx, dw, db


class LoRAKernelLinear(torch.autograd.Function):
    """``y = x W^T + b + s (x A^T) B^T`` with the low-rank term appended to the dense GEMM.

    Forward: ``t = x (s A)^T`` ([M, r]), then one GEMM over ``[x | t] . [W | B]^T``.
    Backward: ``u = dy B`` ([M, r]); ``dx = [dy | u] . [W ; s A]`` in one GEMM;
    ``dA = s u^T x`` and ``dB = dy^T t`` through the fp32 atomic epilogue; ``dW``
    only when the base weight trains. The reference computes the base and adapter
    products separately in eager PyTorch (avgen/finetune/lora.py:692-715).
    """

    @staticmethod
    def forward(ctx, x, weight, bias, lora_a, lora_b, scaling):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        w = bf16_weight(weight)
        sa = (lora_a.detach().float() * scaling).to(torch.bfloat16).contiguous()
        bb = lora_b.detach().to(torch.bfloat16).contiguous()
        t = K.gemm(x2, sa)
        b = bias.detach().float().contiguous() if bias is not None else None
        y = K.gemm(x2, w, bias=b, a2=t, b2=bb)
        ctx.save_for_backward(x2, weight, t, sa, bb)
        ctx.has_bias = bias is not None
        ctx.in_dtype = x.dtype
        ctx.shape = shape
        ctx.scaling = scaling
        ctx.ab_dtypes = (lora_a.dtype, lora_b.dtype)
        return y.view(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        x2, weight, t, sa, bb = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16).contiguous()
        dx = dw = db = da = dbb = None
        u = K.gemm(dy2, bb, b_mn=True)  # [M, r] = dy B
        if ctx.needs_input_grad[0]:
            dx = K.linear_dx(dy2, bf16_weight(weight), a2=u, b2=sa).view(*ctx.shape).to(ctx.in_dtype)
        if ctx.needs_input_grad[1]:
            dw = _weight_grad_buffer(weight)
            K.linear_dw(dy2, x2, dw)
            dw = dw.to(weight.dtype)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = dy2.float().sum(0)
        if ctx.needs_input_grad[3]:
            da = torch.zeros(sa.shape, device=dy.device, dtype=torch.float32)
            K.linear_dw(u, x2, da)
            da = (da * ctx.scaling).to(ctx.ab_dtypes[0])
        if ctx.needs_input_grad[4]:
            dbb = torch.zeros(bb.shape, device=dy.device, dtype=torch.float32)
            K.linear_dw(dy2, t, dbb)
            dbb = dbb.to(ctx.ab_dtypes[1])
        return dx, dw, db, da, dbb, None


def _lora_fusable(layer: nn.Module) -> bool:
    """A plain LoRA adapter the appended-pair GEMM covers exactly."""
    a = getattr(layer, "lora_a", None)
    return (os.environ.get("AVGEN_LORA_FUSED", "0") == "1" and a is not None
            and getattr(layer, "lora_magnitude", None) is None and not getattr(layer, "merged", True)
            and isinstance(getattr(layer, "lora_dropout", None), nn.Identity) and a.shape[0] % 8 == 0
            and not _is_dtensor(a) and not _is_dtensor(layer.lora_b))


def _kernel_ok(x: torch.Tensor, layer: nn.Linear) -> bool:
    return (x.device.type == "cuda" and layer.in_features % 8 == 0 and layer.out_features % 8 == 0
            and x.numel() > 0)


def _is_dtensor(t: torch.Tensor) -> bool:
    from torch.distributed.tensor import DTensor

    return isinstance(t, DTensor)


def linear(x: torch.Tensor, layer: nn.Linear) -> torch.Tensor:
    """Apply ``layer`` with the sm_100a GEMM on CUDA (bf16 output), ``F.linear`` on CPU.

    A tensor-parallel layer (DTensor weight) runs its own forward so its parallel
    style's hooks move activations between local shards and DTensors.
    """
    if _is_dtensor(layer.weight):
        return layer(x)
    adapted = getattr(layer, "adapted_weight", None)
    if callable(adapted):
        if _kernel_ok(x, layer) and _lora_fusable(layer):  # plain LoRA: rank-r pair appended to the GEMM
            return LoRAKernelLinear.apply(x, layer.weight, layer.bias, layer.lora_a, layer.lora_b, layer.scaling)
        # DoRA, merged or dropout adapters: one GEMM on the effective weight, autograd reaches the adapters
        if _kernel_ok(x, layer):
            return KernelLinear.apply(x, adapted(), layer.bias)
        return layer(x)
    if _kernel_ok(x, layer):
        return KernelLinear.apply(x, layer.weight, layer.bias)
    if x.device.type == "cuda":
        raise NotImplementedError(
            f"linear {layer.in_features}->{layer.out_features}: the GEMM kernel needs feature sizes that are "
            "multiples of 8"
        )
    w = layer.weight
    b = layer.bias
    if w.dtype != x.dtype:
        w = w.to(x.dtype)
        b = b.to(x.dtype) if b is not None else None
    return F.linear(x, w, b)
