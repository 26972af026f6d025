"""Audio and audio-visual metrics (avgen/eval/av.py:72-329 behaviour)."""
from __future__ import annotations

from collections.abc import Mapping
from typing import Any

import torch
import torch.nn.functional as F

from avgen_b200.eval.protocols import RunningMetric, register_metric, require_audio, require_video

__all__ = ["AVSyncProxy", "AudioBandwidth", "AudioSilence"]

_EPS = 1e-8


def _zscore(x: torch.Tensor) -> torch.Tensor:
    x = x - x.mean(-1, keepdim=True)
    return x / x.std(-1, keepdim=True).clamp_min(_EPS)


def _to_length(x: torch.Tensor, n: int) -> torch.Tensor:
    return x if x.shape[-1] == n else F.interpolate(x[:, None], size=n, mode="linear", align_corners=False)[:, 0]


@register_metric("av_sync_proxy")
class AVSyncProxy(RunningMetric):
    """Lagged correlation of visual motion with the audio RMS envelope: the peak over
    lags up to ``max_lag`` frames, the zero-lag value and the lag of the peak."""

    required_inputs = ("video", "audio")

    def __init__(self, *, max_lag: int = 4, video_fps: float = 0.0, device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        if max_lag < 1:
            raise ValueError(f"max_lag must be >= 1; got {max_lag!r}")
        if video_fps < 0.0:
            raise ValueError(f"video_fps must be >= 0; got {video_fps!r}")
        self._max_lag, self._fps = max_lag, video_fps

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        v = require_video(inputs["video"], metric=self.name)
        a = require_audio(inputs["audio"], metric=self.name)
        if v.shape[2] < 3 or a.shape[2] < 3:
            return {}
        motion = (v[:, :, 1:] - v[:, :, :-1]).abs().mean((1, 3, 4))
        n = motion.shape[-1]
        lim = min(self._max_lag, n - 1)
        if lim < 1:
            return {}
        m = _zscore(motion)
        e = _zscore(_to_length(a.pow(2).mean(1).sqrt(), n))
        corr = []
        for lag in range(-lim, lim + 1):
            x, y = (m[:, -lag:], e[:, :n + lag]) if lag < 0 else (m[:, :n - lag], e[:, lag:])
            corr.append((x * y).sum(-1) / max(1, x.shape[-1]))
        c = torch.stack(corr, 1)
        peak, idx = c.max(1)
        lag = (idx - lim).float().abs()
        bsz = peak.numel()
        out = {"peak_correlation": (peak.sum(), bsz), "zero_lag_correlation": (c[:, lim].sum(), bsz),
               "lag_frames": (lag.sum(), bsz)}
        if self._fps > 0.0:
            out["lag_seconds"] = (lag.sum() / self._fps, bsz)
        return out


@register_metric("audio_silence")
class AudioSilence(RunningMetric):
    """Share of near-silent frames (relative to the clip's loudest), of entirely
    silent clips, and of clipped samples."""

    required_inputs = ("audio",)

    def __init__(self, *, silence_threshold: float = 0.01, clip_threshold: float = 0.999,
                 device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        if not 0.0 < silence_threshold < 1.0:
            raise ValueError(f"silence_threshold must be in (0, 1); got {silence_threshold!r}")
        if clip_threshold <= 0.0:
            raise ValueError(f"clip_threshold must be > 0; got {clip_threshold!r}")
        self._silence, self._clip = silence_threshold, clip_threshold

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        a = require_audio(inputs["audio"], metric=self.name)
        rms = a.pow(2).mean(1).sqrt()
        loudest = rms.max(-1, keepdim=True).values
        silent = (rms / loudest.clamp_min(_EPS) < self._silence).float()
        dead = (loudest[:, 0] < _EPS).float()
        clipped = (a.abs() >= self._clip).float()
        return {"frame_rate": (silent.sum(), silent.numel()), "clip_rate": (dead.sum(), dead.numel()),
                "clipped_fraction": (clipped.sum(), clipped.numel())}


@register_metric("audio_bandwidth")
class AudioBandwidth(RunningMetric):
    """Spectral centroid and roll-off of the mono mix, as fractions of Nyquist (and Hz
    when the sample rate is known)."""

    required_inputs = ("audio",)

    def __init__(self, *, rolloff_fraction: float = 0.95, sample_rate: float = 0.0,
                 device: torch.device | str = "cpu") -> None:
        super().__init__(device=device)
        if not 0.0 < rolloff_fraction < 1.0:
            raise ValueError(f"rolloff_fraction must be in (0, 1); got {rolloff_fraction!r}")
        if sample_rate < 0.0:
            raise ValueError(f"sample_rate must be >= 0; got {sample_rate!r}")
        self._fraction, self._rate = rolloff_fraction, sample_rate

    def observe(self, **inputs: Any) -> Mapping[str, tuple[torch.Tensor, int]]:
        a = require_audio(inputs["audio"], metric=self.name)
        if a.shape[2] < 4:
            return {}
        power = torch.fft.rfft(a.mean(1), dim=-1).abs().pow(2)
        bins = power.shape[-1]
        power = power[:, 1:]  # drop DC
        if power.shape[-1] < 2:
            return {}
        freq = torch.linspace(1.0 / (bins - 1), 1.0, power.shape[-1], device=a.device)
        total = power.sum(-1, keepdim=True).clamp_min(_EPS)
        centroid = (power * freq).sum(-1) / total[:, 0]
        rolloff = freq[((power.cumsum(-1) / total) >= self._fraction).float().argmax(-1)]
        bsz = centroid.numel()
        out = {"centroid": (centroid.sum(), bsz), "rolloff": (rolloff.sum(), bsz)}
        if self._rate > 0.0:
            nyq = self._rate / 2.0
            out["centroid_hz"] = (centroid.sum() * nyq, bsz)
            out["rolloff_hz"] = (rolloff.sum() * nyq, bsz)
        return out
