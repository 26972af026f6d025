"""3-D axial rotary embeddings on physical coordinates.

Head channel pairs are split over (time, row, column) as
``(P - 2 floor(P/3), floor(P/3), floor(P/3))`` with ``P = head_dim / 2``; pairs are
interleaved (even, odd) channels; tables are fp32; linear and NTK scaling per
axis (reference: avgen/models/rope.py:61-401). On CUDA the fused DiT block
computes the same angles inside the QK-norm/RoPE kernel from ``coords`` and the
per-pair frequencies returned by :meth:`RotaryEmbedding.kernel_frequencies`.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

__all__ = ["RoPEScaling", "RotaryEmbedding", "RotaryTables", "apply_rotary", "build_rotary_tables", "rope_axis_pairs"]

ROPE_SCALING_MODES = ("none", "linear", "ntk")


@dataclass(frozen=True, slots=True)
class RoPEScaling:
    mode: str = "none"
    time_factor: float = 1.0
    spatial_factor: float = 1.0

    def __post_init__(self) -> None:
        if self.mode not in ROPE_SCALING_MODES:
            raise ValueError(f"mode must be one of {ROPE_SCALING_MODES}; got {self.mode!r}")
        for name in ("time_factor", "spatial_factor"):
            if not float(getattr(self, name)) > 0.0:
                raise ValueError(f"{name} must be positive")

    @property
    def is_identity(self) -> bool:
        return self.mode == "none" or (self.time_factor == 1.0 and self.spatial_factor == 1.0)

    def factors(self) -> tuple[float, float, float]:
        return (self.time_factor, self.spatial_factor, self.spatial_factor)


def rope_axis_pairs(head_dim: int) -> tuple[int, int, int]:
    """Channel pairs given to (time, row, column)."""
    if head_dim < 6 or head_dim % 2:
        raise ValueError(f"head_dim must be even and >= 6; got {head_dim!r}")
    pairs = head_dim // 2
    spatial = pairs // 3
    return (pairs - 2 * spatial, spatial, spatial)


@dataclass(frozen=True, slots=True)
class RotaryTables:
    cos: torch.Tensor
    sin: torch.Tensor

    @property
    def pairs(self) -> int:
        return int(self.cos.shape[-1])

    @property
    def length(self) -> int:
        return int(self.cos.shape[-2])

    @property
    def device(self) -> torch.device:
        return self.cos.device

    def validate(self) -> None:
        if self.cos.ndim != 4 or self.cos.shape != self.sin.shape:
            raise ValueError("rotary tables must be matching (batch, 1, length, pairs) tensors")
        if self.cos.dtype is not torch.float32 or self.sin.dtype is not torch.float32:
            raise TypeError("rotary tables must be float32")


def axis_frequencies(head_dim: int, *, theta: float = 10000.0, time_scale: float = 1.0,
                     scaling: RoPEScaling | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-pair frequency (with all scalings folded in) and coordinate axis."""
    plan = scaling or RoPEScaling()
    freqs, axes = [], []
    for axis, (count, factor) in enumerate(zip(rope_axis_pairs(head_dim), plan.factors())):
        axis_theta, mult = theta, 1.0
        if axis == 0 and time_scale != 1.0:
            mult *= time_scale
        if plan.mode == "linear" and factor != 1.0:
            mult /= factor
        elif plan.mode == "ntk" and factor != 1.0 and count > 1:
            dim = 2 * count
            axis_theta = theta * factor ** (dim / (dim - 2))
        exponent = torch.arange(count, dtype=torch.float32) / count
        freqs.append(torch.pow(torch.tensor(axis_theta, dtype=torch.float32), -exponent) * mult)
        axes.append(torch.full((count,), axis, dtype=torch.int32))
    return torch.cat(freqs), torch.cat(axes)


def build_rotary_tables(coords: torch.Tensor, *, head_dim: int, theta: float = 10000.0, time_scale: float = 1.0,
                        scaling: RoPEScaling | None = None) -> RotaryTables:
    """cos/sin tables ``(B, 1, L, head_dim/2)`` from ``coords (B, L, 3)``."""
    if coords.ndim != 3 or coords.shape[-1] != 3:
        raise ValueError(f"coords must be (batch, length, 3); got {tuple(coords.shape)}")
    if coords.dtype is not torch.float32:
        raise TypeError(f"coords must be float32; got {coords.dtype}")
    freq, axis = axis_frequencies(head_dim, theta=theta, time_scale=time_scale, scaling=scaling)
    freq = freq.to(coords.device)
    phase = coords[..., axis.long().to(coords.device)] * freq
    phase = phase[:, None]
    return RotaryTables(cos=torch.cos(phase), sin=torch.sin(phase))


def apply_rotary(x: torch.Tensor, tables: RotaryTables) -> torch.Tensor:
    """Rotate interleaved channel pairs of ``x (B, H, L, D)`` in fp32."""
    if x.ndim != 4:
        raise ValueError(f"rotary input must be (batch, heads, length, head_dim); got {tuple(x.shape)}")
    if x.shape[-1] != 2 * tables.pairs:
        raise ValueError("head_dim does not match the rotary tables")
    if x.shape[-2] != tables.length:
        raise ValueError("sequence length does not match the rotary tables (build them from the local shard)")
    pairs = x.float().unflatten(-1, (tables.pairs, 2))
    even, odd = pairs[..., 0], pairs[..., 1]
    rotated = torch.stack((even * tables.cos - odd * tables.sin, even * tables.sin + odd * tables.cos), -1)
    return rotated.flatten(-2).to(x.dtype)


class RotaryEmbedding(nn.Module):
    """Builds rotary tables from coordinates (and the kernel frequency table)."""

    def __init__(self, head_dim: int, *, theta: float = 10000.0, time_scale: float = 1.0,
                 scaling: RoPEScaling | None = None) -> None:
        super().__init__()
        rope_axis_pairs(head_dim)
        self.head_dim = head_dim
        self.theta = theta
        self.time_scale = time_scale
        self.scaling = scaling or RoPEScaling()
        self._kernel_cache: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}

    def forward(self, coords: torch.Tensor) -> RotaryTables:
        return build_rotary_tables(coords, head_dim=self.head_dim, theta=self.theta, time_scale=self.time_scale,
                                   scaling=self.scaling)

    def kernel_frequencies(self, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        """``(freq fp32 [D/2], axis int32 [D/2])`` on ``device`` (cached)."""
        if device not in self._kernel_cache:
            freq, axis = axis_frequencies(self.head_dim, theta=self.theta, time_scale=self.time_scale,
                                          scaling=self.scaling)
            self._kernel_cache[device] = (freq.to(device), axis.to(device))
        return self._kernel_cache[device]

    def extra_repr(self) -> str:
        return (f"head_dim={self.head_dim}, pairs(t,h,w)={rope_axis_pairs(self.head_dim)}, theta={self.theta}, "
                f"time_scale={self.time_scale}, scaling={self.scaling.mode}")
