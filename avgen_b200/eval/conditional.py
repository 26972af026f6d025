"""Metrics for conditioned generation: image-to-video, continuation and inpainting
(avgen/eval/conditional.py:49-318 behaviour)."""
from __future__ import annotations

from collections.abc import Mapping
from typing import Any

import torch
import torch.nn.functional as F

from avgen_b200.eval.protocols import MetricError, RunningMetric, register_metric, require_video

__all__ = ["FirstFrameFidelity", "InpaintBoundaryConsistency", "SeamContinuity"]

_EPS = 1e-8


@register_metric("first_frame_fidelity")
class FirstFrameFidelity(RunningMetric):
    """How closely the anchored frame reproduces the reference: MSE, PSNR over the
    reference's range, and cosine similarity."""

    required_inputs = ("video", "reference")

    def __init__(self, *, frame_index: int = 0, device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        if frame_index < 0:
            raise ValueError(f"frame_index must be >= 0; got {frame_index!r}")
        self._index = frame_index

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        r = require_video(inputs["reference"], metric=self.name, argument="reference")
        if v.shape != r.shape:
            raise MetricError(f"{self.name}: video {tuple(v.shape)} and reference {tuple(r.shape)} differ in shape")
        if self._index >= v.shape[2]:
            raise MetricError(f"{self.name}: frame_index={self._index} is out of range for {v.shape[2]} frames")
        g, t = v[:, :, self._index].flatten(1), r[:, :, self._index].flatten(1)
        mse = (g - t).pow(2).mean(1)
        span = (t.max(1).values - t.min(1).values).clamp_min(_EPS)
        psnr = 10.0 * torch.log10(span.pow(2) / mse.clamp_min(_EPS))
        cos = F.cosine_similarity(g, t, dim=1)
        n = mse.numel()
        return {"mse": (mse.sum(), n), "psnr_db": (psnr.sum(), n), "cosine": (cos.sum(), n)}


@register_metric("seam_continuity")
class SeamContinuity(RunningMetric):
    """Change across the context/continuation boundary relative to the change between
    other consecutive frames (1 = seamless), and relative to the clip's spread."""

    def __init__(self, *, context_frames: int = 1, device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        if context_frames < 1:
            raise ValueError(f"context_frames must be >= 1; got {context_frames!r}")
        self._context = context_frames

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        ctx = int(inputs.get("context_frames", self._context))
        t = v.shape[2]
        if ctx < 1 or ctx >= t:
            raise MetricError(f"{self.name}: context_frames={ctx} leaves no continuation in a clip of {t} frames")
        if t < 4:
            return {}
        d = (v[:, :, 1:] - v[:, :, :-1]).abs().mean((1, 3, 4))
        seam = d[:, ctx - 1]
        rest = torch.cat((d[:, :ctx - 1], d[:, ctx:]), 1)
        if rest.shape[1] == 0:
            return {}
        n = seam.numel()
        return {"ratio": ((seam / rest.mean(1).clamp_min(_EPS)).sum(), n),
                "seam_delta": ((seam / v.flatten(1).std(1).clamp_min(_EPS)).sum(), n)}


@register_metric("inpaint_boundary")
class InpaintBoundaryConsistency(RunningMetric):
    """Spatial-gradient energy on the one-pixel ring around the inpainting mask over
    that inside/outside it (1 = invisible boundary); with a reference, also the
    change leaked into the preserved region."""

    required_inputs = ("video", "mask")

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        mask = inputs["mask"]
        if not isinstance(mask, torch.Tensor) or mask.ndim != 5:
            raise MetricError(f"{self.name}: mask must be a (batch, 1, frames, height, width) tensor; got "
                              f"{type(mask).__name__} {tuple(getattr(mask, 'shape', ()))}")
        mask = mask.detach().float()
        if mask.shape[0] != v.shape[0] or mask.shape[2:] != v.shape[2:]:
            raise MetricError(f"{self.name}: mask {tuple(mask.shape)} does not align with video {tuple(v.shape)}")
        b, _, t, h, w = v.shape
        if h < 3 or w < 3:
            return {}
        gy = F.pad((v[:, :, :, 1:] - v[:, :, :, :-1]).abs(), (0, 0, 0, 1))
        gx = F.pad((v[..., 1:] - v[..., :-1]).abs(), (0, 1))
        grad = (gx + gy).mean(1, keepdim=True)
        flat = mask.reshape(b * t, 1, h, w)
        ring = (F.max_pool2d(flat, 3, 1, 1) + F.max_pool2d(-flat, 3, 1, 1)).reshape(b, 1, t, h, w)
        inner = 1.0 - ring
        rw, iw = ring.flatten(1).sum(1), inner.flatten(1).sum(1)
        ok = (rw > 0) & (iw > 0)
        if not bool(ok.any()):
            return {}
        e_ring = (grad * ring).flatten(1).sum(1) / rw.clamp_min(_EPS)
        e_in = (grad * inner).flatten(1).sum(1) / iw.clamp_min(_EPS)
        ratio = (e_ring / e_in.clamp_min(_EPS))[ok]
        out: dict[str, tuple[torch.Tensor, int]] = {"gradient_ratio": (ratio.sum(), ratio.numel())}
        ref = inputs.get("reference")
        if isinstance(ref, torch.Tensor) and ref.shape == v.shape:
            keep = 1.0 - mask
            diff = (v - ref.detach().float()).abs().mean(1, keepdim=True)
            leak = (diff * keep).flatten(1).sum(1) / keep.flatten(1).sum(1).clamp_min(_EPS) \
                / v.flatten(1).std(1).clamp_min(_EPS)
            out["leakage"] = (leak.sum(), leak.numel())
        return out
