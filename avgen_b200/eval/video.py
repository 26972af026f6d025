"""Reference-free video metrics (avgen/eval/video.py:68-435 behaviour).

Every statistic is normalised by the clip's own standard deviation where it
measures a difference, so latents and pixels of any scale give comparable
numbers. Each contribution is a per-item sum plus its count.
"""
from __future__ import annotations

from collections.abc import Mapping
from typing import Any

import torch
import torch.nn.functional as F

from avgen_b200.eval.protocols import RunningMetric, register_metric, require_video

__all__ = ["FlickerIndex", "MotionMagnitude", "SaturationClipping", "SharpnessProxy", "StaticFrameRatio",
           "TemporalConsistency"]

_EPS = 1e-8


def _frame_vectors(video: torch.Tensor) -> torch.Tensor:
    return video.transpose(1, 2).flatten(2)  # [B, T, C*H*W]


def _clip_std(video: torch.Tensor) -> torch.Tensor:
    return video.flatten(1).std(1).clamp_min(_EPS)


def _frame_deltas(video: torch.Tensor) -> torch.Tensor:
    """Mean absolute difference of consecutive frames, ``[B, T-1]``."""
    return (video[:, :, 1:] - video[:, :, :-1]).abs().mean((1, 3, 4))


@register_metric("temporal_consistency")
class TemporalConsistency(RunningMetric):
    """Cosine similarity of frames ``stride`` apart (mean, and the worst pair per clip)."""

    def __init__(self, *, stride: int = 1, device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        if stride < 1:
            raise ValueError(f"stride must be >= 1; got {stride!r}")
        self._stride = stride

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        f = _frame_vectors(require_video(inputs["video"], metric=self.name))
        if f.shape[1] <= self._stride:
            return {}
        sim = F.cosine_similarity(f[:, self._stride:], f[:, :-self._stride], dim=-1, eps=_EPS)
        worst = sim.min(1).values
        return {"cosine": (sim.sum(), sim.numel()), "worst_pair": (worst.sum(), worst.numel())}


@register_metric("motion_magnitude")
class MotionMagnitude(RunningMetric):
    """Frame-to-frame change relative to the clip's spread (mean and per-clip peak)."""

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        if v.shape[2] < 2:
            return {}
        d = _frame_deltas(v) / _clip_std(v)[:, None]
        peak = d.max(1).values
        return {"mean": (d.sum(), d.numel()), "peak": (peak.sum(), peak.numel())}


@register_metric("flicker_index")
class FlickerIndex(RunningMetric):
    """Energy of the temporal second difference over that of the first difference
    (high for frame-to-frame oscillation, low for smooth motion)."""

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        if v.shape[2] < 3:
            return {}
        d1 = v[:, :, 1:] - v[:, :, :-1]
        d2 = d1[:, :, 1:] - d1[:, :, :-1]
        e1 = d1[:, :, 1:].pow(2).flatten(1).mean(1)
        e2 = d2.pow(2).flatten(1).mean(1)
        ratio = e2 / e1.clamp_min(_EPS)
        return {"index": (ratio.sum(), ratio.numel()),
                "second_difference": ((e2 / _clip_std(v).pow(2)).sum(), e2.numel())}


@register_metric("static_frames")
class StaticFrameRatio(RunningMetric):
    """Share of consecutive-frame pairs (and of whole clips) that barely change."""

    def __init__(self, *, threshold: float = 0.02, device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        if threshold <= 0.0:
            raise ValueError(f"threshold must be > 0; got {threshold!r}")
        self._threshold = threshold

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        if v.shape[2] < 2:
            return {}
        still = ((_frame_deltas(v) / _clip_std(v)[:, None]) < self._threshold).float()
        clips = still.min(1).values
        return {"pair_rate": (still.sum(), still.numel()), "clip_rate": (clips.sum(), clips.numel())}


@register_metric("saturation")
class SaturationClipping(RunningMetric):
    """Share of pixels at the ends of the value range, and outside it (pixel space only)."""

    pixel_space_only = True

    def __init__(self, *, value_range: tuple[float, float] = (-1.0, 1.0), tolerance: float = 1e-3,
                 device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        lo, hi = value_range
        if not hi > lo:
            raise ValueError(f"value_range must be increasing; got {value_range!r}")
        self._lo, self._hi, self._margin = lo, hi, tolerance * (hi - lo)

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        n = v.numel()
        at_edge = (v <= self._lo + self._margin) | (v >= self._hi - self._margin)
        outside = (v < self._lo) | (v > self._hi)
        return {"clipped_fraction": (at_edge.float().sum(), n), "out_of_range_fraction": (outside.float().sum(), n)}


_LAPLACIAN = torch.tensor([[0.0, 1.0, 0.0], [1.0, -4.0, 1.0], [0.0, 1.0, 0.0]])


@register_metric("sharpness")
class SharpnessProxy(RunningMetric):
    """Variance of the per-frame Laplacian response relative to the clip's variance,
    and its tail-over-head ratio across the clip (blur creeping in over time)."""

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        b, c, t, h, w = v.shape
        if h < 3 or w < 3:
            return {}
        k = _LAPLACIAN.to(v.device).view(1, 1, 3, 3).repeat(c, 1, 1, 1)
        resp = F.conv2d(v.transpose(1, 2).reshape(b * t, c, h, w), k, groups=c)
        per = resp.flatten(1).var(1).view(b, t) / _clip_std(v).pow(2)[:, None]
        out: dict[str, tuple[torch.Tensor, int]] = {"mean": (per.sum(), per.numel())}
        third = t // 3
        if third >= 1:
            decay = per[:, -third:].mean(1) / per[:, :third].mean(1).clamp_min(_EPS)
            out["decay"] = (decay.sum(), decay.numel())
        return out
