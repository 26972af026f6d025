"""Per-channel latent normalisation (avgen/codecs/normalization.py:51-330 API).

``normalize_latents`` maps codec latents to the unit-variance space the model is
trained in; ``denormalize_latents`` inverts it before decoding.
"""
from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import torch

__all__ = ["LatentStatistics", "denormalize_latents", "normalize_latents", "resolve_latent_normalization"]


@dataclass(frozen=True, slots=True)
class LatentStatistics:
    mean: tuple[float, ...]
    std: tuple[float, ...]
    channel_dim: int = 1

    def __post_init__(self) -> None:
        object.__setattr__(self, "mean", tuple(float(v) for v in self.mean))
        object.__setattr__(self, "std", tuple(float(v) for v in self.std))
        if not self.mean or len(self.mean) != len(self.std):
            raise ValueError(f"mean and std need the same non-zero length; got {len(self.mean)} and {len(self.std)}")
        if not all(math.isfinite(v) for v in self.mean):
            raise ValueError("mean must be finite")
        if not all(math.isfinite(v) and v > 0.0 for v in self.std):
            raise ValueError("std must be finite and positive")

    @property
    def channels(self) -> int:
        return len(self.mean)

    @property
    def is_identity(self) -> bool:
        return all(m == 0.0 for m in self.mean) and all(s == 1.0 for s in self.std)

    def tensors(self, *, ndim: int, device: torch.device | str = "cpu",
                dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
        """Mean and std shaped to broadcast against a rank-``ndim`` latent."""
        dim = self.channel_dim % ndim
        shape = [1] * ndim
        shape[dim] = self.channels
        mean = torch.tensor(self.mean, device=device, dtype=dtype).view(shape)
        std = torch.tensor(self.std, device=device, dtype=dtype).view(shape)
        return mean, std

    def to_dict(self) -> dict[str, Any]:
        return {"mean": list(self.mean), "std": list(self.std), "channel_dim": self.channel_dim}

    @classmethod
    def from_dict(cls, values: Mapping[str, Any]) -> LatentStatistics:
        return cls(mean=tuple(values["mean"]), std=tuple(values["std"]), channel_dim=int(values.get("channel_dim", 1)))

    @classmethod
    def identity(cls, channels: int, *, channel_dim: int = 1) -> LatentStatistics:
        return cls((0.0,) * channels, (1.0,) * channels, channel_dim)

    @classmethod
    def from_scalar(cls, channels: int, *, mean: float = 0.0, std: float = 1.0,
                    channel_dim: int = 1) -> LatentStatistics:
        return cls((mean,) * channels, (std,) * channels, channel_dim)

    @classmethod
    def from_latents(cls, latents: torch.Tensor, *, channel_dim: int = 1) -> LatentStatistics:
        """Per-channel statistics measured on a batch of latents (fp64 accumulation)."""
        x = latents.detach().double().movedim(channel_dim, 0).reshape(latents.shape[channel_dim], -1)
        std = x.std(dim=1, unbiased=False).clamp_min(1e-6)
        return cls(tuple(x.mean(dim=1).tolist()), tuple(std.tolist()), channel_dim)


def _check(latents: torch.Tensor, stats: LatentStatistics) -> None:
    got = latents.shape[stats.channel_dim % latents.ndim]
    if got != stats.channels:
        raise ValueError(f"latents have {got} channels along dim {stats.channel_dim}; statistics have {stats.channels}")


def normalize_latents(latents: torch.Tensor, statistics: LatentStatistics) -> torch.Tensor:
    _check(latents, statistics)
    if statistics.is_identity:
        return latents
    mean, std = statistics.tensors(ndim=latents.ndim, device=latents.device, dtype=latents.dtype)
    return (latents - mean) / std


def denormalize_latents(latents: torch.Tensor, statistics: LatentStatistics) -> torch.Tensor:
    _check(latents, statistics)
    if statistics.is_identity:
        return latents
    mean, std = statistics.tensors(ndim=latents.ndim, device=latents.device, dtype=latents.dtype)
    return latents * std + mean


def _as_floats(values: object) -> tuple[float, ...]:
    if isinstance(values, torch.Tensor):
        return tuple(float(v) for v in values.flatten().tolist())
    if isinstance(values, (int, float)):
        return (float(values),)
    return tuple(float(v) for v in values)  # type: ignore[union-attr]


def resolve_latent_normalization(source: object, *, channels: int | None = None,
                                 channel_dim: int = 1) -> LatentStatistics:
    """Statistics from a codec, a mapping (``mean``/``std``, or ``shift_factor``/``scaling_factor``
    as in diffusers configs), an existing :class:`LatentStatistics`, or ``None`` (identity)."""
    if isinstance(source, LatentStatistics):
        return source
    if source is None:
        if channels is None:
            raise ValueError("identity normalisation needs the channel count")
        return LatentStatistics.identity(channels, channel_dim=channel_dim)
    stats = getattr(source, "latent_statistics", None)
    if stats is not None:
        return stats() if callable(stats) else stats
    if isinstance(source, Mapping):
        if "mean" in source and "std" in source:
            mean, std = _as_floats(source["mean"]), _as_floats(source["std"])
        elif "latents_mean" in source and "latents_std" in source:
            mean, std = _as_floats(source["latents_mean"]), _as_floats(source["latents_std"])
        elif "scaling_factor" in source:
            scale = float(source["scaling_factor"])
            shift = float(source.get("shift_factor") or 0.0)
            mean, std = (shift,), (1.0 / scale,)
        else:
            raise KeyError("mapping needs mean/std, latents_mean/latents_std or scaling_factor")
        if len(mean) == 1 and channels:
            mean, std = mean * channels, std * channels
        if channels is not None and len(mean) != channels:
            raise ValueError(f"statistics have {len(mean)} channels; expected {channels}")
        return LatentStatistics(mean, std, channel_dim)
    raise TypeError(f"cannot derive latent statistics from {type(source).__name__}")
