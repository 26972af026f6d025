"""DiT building blocks with the reference's module and parameter names.

FusedRMSNorm, ``modulate`` (x * (1 + scale) + shift), the sinusoidal timestep
embedding (scale 1000), TimestepEmbedding, AdaLNModulation (6 chunks,
zero-init), SwiGLU, a GELU(tanh) MLP variant, SelfAttention (QK-RMSNorm, GQA,
RoPE) and CrossAttention (zero-init output). Reference:
avgen/models/layers.py:70-686. These eager forwards are the CPU oracle; on CUDA
their linears run the tcgen05 GEMM and attention runs the flash kernels, and
the DiT block itself uses the fused path in :mod:`avgen_b200.models.fused`.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from avgen_b200.models.attention import attention
from avgen_b200.models.linear import linear
from avgen_b200.models.rope import RotaryTables, apply_rotary

__all__ = ["MODULATION_CHUNKS", "AdaLNModulation", "CrossAttention", "FusedRMSNorm", "GeluMLP", "SelfAttention",
           "SwiGLU", "TimestepEmbedding", "init_linear", "init_norm", "match_dtype", "modulate", "rms_norm",
           "sinusoidal_embedding"]

MODULATION_CHUNKS = 6


class FusedRMSNorm(nn.RMSNorm):
    """RMSNorm whose weight follows the input dtype."""

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        w = self.weight
        if w is not None and w.dtype != hidden.dtype:
            w = w.to(hidden.dtype)
        return F.rms_norm(hidden, self.normalized_shape, w, self.eps)


def match_dtype(tensor: torch.Tensor, module: nn.Module) -> torch.Tensor:
    w = getattr(module, "weight", None)
    if w is None:
        raise AttributeError(f"{type(module).__name__} has no weight")
    return tensor if tensor.dtype == w.dtype or tensor.device.type == "cuda" else tensor.to(w.dtype)


def rms_norm(width: int, *, eps: float = 1e-6) -> FusedRMSNorm:
    return FusedRMSNorm(width, eps=eps)


def init_linear(layer: nn.Linear, *, std: float = 0.02, zero: bool = False) -> None:
    if zero:
        nn.init.zeros_(layer.weight)
    else:
        nn.init.trunc_normal_(layer.weight, std=std, a=-2 * std, b=2 * std)
    if layer.bias is not None:
        nn.init.zeros_(layer.bias)


def init_norm(norm: nn.Module) -> None:
    if isinstance(getattr(norm, "weight", None), torch.Tensor):
        nn.init.ones_(norm.weight)
    if isinstance(getattr(norm, "bias", None), torch.Tensor):
        nn.init.zeros_(norm.bias)


def modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return x * (1.0 + scale) + shift


def sinusoidal_embedding(values: torch.Tensor, dim: int, *, max_period: float = 10000.0,
                         scale: float = 1000.0) -> torch.Tensor:
    """``[cos(a), sin(a)]`` with ``a = values * scale * max_period^(-i/half)``."""
    if dim < 2 or dim % 2:
        raise ValueError(f"embedding dim must be a positive even integer; got {dim!r}")
    half = dim // 2
    exponent = torch.arange(half, device=values.device, dtype=torch.float32) / half
    freqs = torch.exp(-math.log(max_period) * exponent)
    angles = values.float()[..., None] * scale * freqs
    return torch.cat((torch.cos(angles), torch.sin(angles)), -1)


class TimestepEmbedding(nn.Module):
    def __init__(self, width: int, *, frequency_dim: int = 256, max_period: float = 10000.0,
                 scale: float = 1000.0) -> None:
        super().__init__()
        self.frequency_dim = frequency_dim
        self.max_period = max_period
        self.scale = scale
        self.in_proj = nn.Linear(frequency_dim, width, bias=True)
        self.out_proj = nn.Linear(width, width, bias=True)

    def forward(self, noise_level: torch.Tensor) -> torch.Tensor:
        feats = sinusoidal_embedding(noise_level, self.frequency_dim, max_period=self.max_period, scale=self.scale)
        feats = feats.to(self.in_proj.weight.dtype)
        return linear(F.silu(linear(feats, self.in_proj)), self.out_proj)

    def init_weights(self) -> None:
        init_linear(self.in_proj)
        init_linear(self.out_proj)


class AdaLNModulation(nn.Module):
    """Shared adaLN-single projection: ``proj(silu(cond))`` split into 6 chunks."""

    def __init__(self, cond_width: int, width: int, *, chunks: int = MODULATION_CHUNKS) -> None:
        super().__init__()
        self.width = width
        self.chunks = chunks
        self.proj = nn.Linear(cond_width, chunks * width, bias=True)

    def forward(self, cond: torch.Tensor) -> torch.Tensor:
        return linear(F.silu(cond), self.proj).float().unflatten(-1, (self.chunks, self.width))

    def init_weights(self) -> None:
        init_linear(self.proj, zero=True)


class SwiGLU(nn.Module):
    def __init__(self, width: int, hidden: int, *, bias: bool = False) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(width, hidden, bias=bias)
        self.up_proj = nn.Linear(width, hidden, bias=bias)
        self.down_proj = nn.Linear(hidden, width, bias=bias)
        self.tp = None  # set by head-parallel sharding: this rank's slice of the hidden units

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        if self.tp is not None:
            hidden = self.tp.enter(hidden)
        out = linear(F.silu(linear(hidden, self.gate_proj)) * linear(hidden, self.up_proj), self.down_proj)
        return self.tp.leave(out) if self.tp is not None else out

    def init_weights(self, *, std: float = 0.02, out_std: float | None = None) -> None:
        init_linear(self.gate_proj, std=std)
        init_linear(self.up_proj, std=std)
        init_linear(self.down_proj, std=out_std if out_std is not None else std)


class GeluMLP(nn.Module):
    """``down(gelu_tanh(up(x)))`` (the "GELU MLP" variant; names up_proj/down_proj)."""

    def __init__(self, width: int, hidden: int, *, bias: bool = False) -> None:
        super().__init__()
        self.up_proj = nn.Linear(width, hidden, bias=bias)
        self.down_proj = nn.Linear(hidden, width, bias=bias)
        self.tp = None  # set by head-parallel sharding

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        if self.tp is not None:
            hidden = self.tp.enter(hidden)
        out = linear(F.gelu(linear(hidden, self.up_proj), approximate="tanh"), self.down_proj)
        return self.tp.leave(out) if self.tp is not None else out

    def init_weights(self, *, std: float = 0.02, out_std: float | None = None) -> None:
        init_linear(self.up_proj, std=std)
        init_linear(self.down_proj, std=out_std if out_std is not None else std)


def _head_dim(width: int, num_heads: int, head_dim: int | None) -> int:
    if head_dim is not None:
        return head_dim
    if width % num_heads:
        raise ValueError(f"width {width} must be divisible by num_heads {num_heads}")
    return width // num_heads


class SelfAttention(nn.Module):
    def __init__(self, width: int, num_heads: int, *, head_dim: int | None = None, num_kv_heads: int | None = None,
                 qk_norm: bool = True, eps: float = 1e-6, bias: bool = False) -> None:
        super().__init__()
        head_dim = _head_dim(width, num_heads, head_dim)
        kv = num_kv_heads if num_kv_heads is not None else num_heads
        if num_heads % kv:
            raise ValueError(f"num_heads {num_heads} must be divisible by num_kv_heads {kv}")
        self.num_heads = num_heads
        self.num_kv_heads = kv
        self.head_dim = head_dim
        self.q_proj = nn.Linear(width, num_heads * head_dim, bias=bias)
        self.k_proj = nn.Linear(width, kv * head_dim, bias=bias)
        self.v_proj = nn.Linear(width, kv * head_dim, bias=bias)
        self.out_proj = nn.Linear(num_heads * head_dim, width, bias=bias)
        self.q_norm = rms_norm(head_dim, eps=eps) if qk_norm else nn.Identity()
        self.k_norm = rms_norm(head_dim, eps=eps) if qk_norm else nn.Identity()
        self.cp_mesh = None  # set by context parallelism: attention becomes global over the shards
        self.tp = None  # set by head-parallel sharding: this rank's heads, collectives in and out

    def _heads(self, x: torch.Tensor) -> torch.Tensor:
        return x.unflatten(-1, (-1, self.head_dim)).transpose(1, 2)

    def forward(self, hidden: torch.Tensor, rope: RotaryTables | None = None, *,
                key_mask: torch.Tensor | None = None) -> torch.Tensor:
        if self.tp is not None:
            hidden = self.tp.enter(hidden)
        q = self.q_norm(self._heads(linear(hidden, self.q_proj)))
        k = self.k_norm(self._heads(linear(hidden, self.k_proj)))
        v = self._heads(linear(hidden, self.v_proj))
        if rope is not None:
            q = apply_rotary(q, rope)
            k = apply_rotary(k, rope)
        if self.cp_mesh is not None:
            from avgen_b200.parallel.context import cp_attention

            out = cp_attention(q, k, v, mesh=self.cp_mesh, key_mask=key_mask).transpose(1, 2)
        else:
            out = attention(q, k, v, key_mask=key_mask, layout="blhd")
        out = linear(out.flatten(2), self.out_proj)
        return self.tp.leave(out) if self.tp is not None else out

    def init_weights(self, *, std: float = 0.02, out_std: float | None = None) -> None:
        for layer in (self.q_proj, self.k_proj, self.v_proj):
            init_linear(layer, std=std)
        init_linear(self.out_proj, std=out_std if out_std is not None else std)
        init_norm(self.q_norm)
        init_norm(self.k_norm)


class CrossAttention(nn.Module):
    def __init__(self, width: int, num_heads: int, *, context_width: int | None = None, head_dim: int | None = None,
                 num_kv_heads: int | None = None, qk_norm: bool = True, eps: float = 1e-6,
                 bias: bool = False) -> None:
        super().__init__()
        head_dim = _head_dim(width, num_heads, head_dim)
        kv = num_kv_heads if num_kv_heads is not None else num_heads
        if num_heads % kv:
            raise ValueError(f"num_heads {num_heads} must be divisible by num_kv_heads {kv}")
        ctx_w = context_width if context_width is not None else width
        self.num_heads = num_heads
        self.num_kv_heads = kv
        self.head_dim = head_dim
        self.q_proj = nn.Linear(width, num_heads * head_dim, bias=bias)
        self.k_proj = nn.Linear(ctx_w, kv * head_dim, bias=bias)
        self.v_proj = nn.Linear(ctx_w, kv * head_dim, bias=bias)
        self.out_proj = nn.Linear(num_heads * head_dim, width, bias=bias)
        self.q_norm = rms_norm(head_dim, eps=eps) if qk_norm else nn.Identity()
        self.k_norm = rms_norm(head_dim, eps=eps) if qk_norm else nn.Identity()
        self.tp = None  # set by head-parallel sharding

    def _heads(self, x: torch.Tensor) -> torch.Tensor:
        return x.unflatten(-1, (-1, self.head_dim)).transpose(1, 2)

    def forward(self, hidden: torch.Tensor, context: torch.Tensor, context_mask: torch.Tensor | None = None,
                ) -> torch.Tensor:
        if context.shape[1] == 0:
            return torch.zeros_like(hidden)
        if self.tp is not None:
            hidden = self.tp.enter(hidden)
            context = self.tp.shared(context)  # every rank's heads read the same text tokens
        q = self.q_norm(self._heads(linear(hidden, self.q_proj)))
        k = self.k_norm(self._heads(linear(context, self.k_proj)))
        v = self._heads(linear(context, self.v_proj))
        mask = context_mask
        if mask is not None and mask.ndim != 2:
            raise ValueError("cross-attention context mask must be (batch, keys)")
        out = attention(q, k, v, key_mask=mask, layout="blhd")
        out = linear(out.flatten(2), self.out_proj)
        return self.tp.leave(out) if self.tp is not None else out

    def init_weights(self, *, std: float = 0.02, zero_output: bool = True) -> None:
        for layer in (self.q_proj, self.k_proj, self.v_proj):
            init_linear(layer, std=std)
        init_linear(self.out_proj, std=std, zero=zero_output)
        init_norm(self.q_norm)
        init_norm(self.k_norm)
