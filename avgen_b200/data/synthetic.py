"""Deterministic procedural latents: a learnable, resumable, rank-sharded source.

Same API and role as avgen/data/synthetic.py:85-864. Every sample is a pure
function of ``(seed, index)``: its parameters come from a SplitMix64 hash of
the pair, so any rank can regenerate any sample and a resumed run sees the same
stream. Samples carry structure a model can learn:

* a *drive* waveform ``d(t) = sin(2 pi f t + phase) + g sin(4 pi f t + 2 phase)``
  (per-sample frequency with jitter, optional harmonic);
* video channel ``video_drive_channel`` is the drive (plus a static texture);
  the other channels are a plane wave travelling at a per-sample velocity;
* audio channel ``audio_drive_channel`` is the drive delayed by
  ``audio_lag_seconds`` (other channels: a second waveform);
* the text embedding encodes the sample's frequency, phase and velocity
  through a fixed random projection, so conditioning is informative.

:class:`AlignmentTruth` measures the video/audio correlation of the drive, the
ground truth an AV-sync metric should recover. Rank ``r`` of ``w`` owns indices
``r, r + w, ...``.
"""
from __future__ import annotations

import math
from collections.abc import Iterator, Mapping
from dataclasses import dataclass
from typing import Any

import torch

from avgen_b200.core._validate import require_dimension, require_finite, require_name, require_positive
from avgen_b200.core.batch import MediaBatch
from avgen_b200.core.rng import mix_seed
from avgen_b200.data.protocols import LatentSample, SampleDescriptor, collate_samples

__all__ = ["AlignmentTruth", "SyntheticConfig", "SyntheticSource"]


@dataclass(frozen=True, slots=True)
class SyntheticConfig:
    seed: int = 0
    num_samples: int = 64
    video_channels: int = 4
    frames: int = 8
    height: int = 8
    width: int = 8
    audio_channels: int = 2
    audio_frames: int = 32
    text_tokens: int = 4
    text_width: int = 16
    video_timebase_num: int = 8
    video_timebase_den: int = 1
    audio_timebase_num: int = 32
    audio_timebase_den: int = 1
    drive_frequency_hz: float = 0.5
    drive_frequency_jitter: float = 0.6
    drive_harmonic_gain: float = 0.6
    audio_lag_seconds: float = 0.0
    motion_scale: float = 1.0
    audio_gain: float = 1.0
    texture_scale: float = 0.25
    dtype: torch.dtype = torch.float32
    video_codec_id: str = "synthetic-video-v1"
    audio_codec_id: str = "synthetic-audio-v1"

    def __post_init__(self) -> None:
        require_dimension("seed", self.seed, allow_zero=True)
        for n in ("num_samples", "video_channels", "frames", "height", "width", "audio_channels", "text_width",
                  "video_timebase_num", "video_timebase_den", "audio_timebase_num", "audio_timebase_den"):
            require_positive(n, getattr(self, n))
        for n in ("audio_frames", "text_tokens"):
            require_dimension(n, getattr(self, n), allow_zero=True)
        for n in ("drive_frequency_hz", "drive_frequency_jitter", "drive_harmonic_gain", "audio_lag_seconds",
                  "motion_scale", "audio_gain", "texture_scale"):
            require_finite(n, getattr(self, n))
        if self.drive_frequency_hz <= 0:
            raise ValueError("drive_frequency_hz must be positive")
        if not 0.0 <= self.drive_frequency_jitter < 1.0:
            raise ValueError("drive_frequency_jitter must be in [0, 1)")
        if self.drive_harmonic_gain < 0:
            raise ValueError("drive_harmonic_gain must be non-negative")
        require_name("video_codec_id", self.video_codec_id)
        require_name("audio_codec_id", self.audio_codec_id)
        if self.has_audio and self.max_drive_frequency_hz * 4.0 > self.video_fps:
            raise ValueError(f"the drive reaches {self.max_drive_frequency_hz} Hz but the video rate is "
                             f"{self.video_fps} fps: need four samples per period")

    @property
    def max_drive_frequency_hz(self) -> float:
        top = self.drive_frequency_hz * (1.0 + self.drive_frequency_jitter)
        return top * 2.0 if self.drive_harmonic_gain > 0 else top

    @property
    def video_fps(self) -> float:
        return self.video_timebase_num / self.video_timebase_den

    @property
    def audio_fps(self) -> float:
        return self.audio_timebase_num / self.audio_timebase_den

    @property
    def has_audio(self) -> bool:
        return self.audio_frames > 0


@dataclass(frozen=True, slots=True)
class AlignmentTruth:
    """Where the shared drive lives and how well video and audio should correlate."""

    drive_frequency_hz: float
    audio_lag_seconds: float
    video_drive_channel: int
    audio_drive_channel: int
    expected_correlation: float = 1.0
    tolerance: float = 0.01

    def video_drive(self, video: torch.Tensor) -> torch.Tensor:
        return video[:, self.video_drive_channel].mean(dim=(-2, -1)).float()

    def audio_drive_at(self, audio: torch.Tensor, video_positions: torch.Tensor, *,
                       audio_fps: float) -> tuple[torch.Tensor, torch.Tensor]:
        """Audio drive linearly interpolated at the (lagged) video frame times."""
        if audio.shape[-1] == 0:
            raise ValueError("cannot measure alignment on a batch with no audio frames")
        track = audio[:, self.audio_drive_channel].float()
        last = track.shape[-1] - 1
        pos = (video_positions.float() + self.audio_lag_seconds) * audio_fps
        covered = (pos >= 0) & (pos <= last)
        pos = pos.clamp(0, last)
        lo = pos.floor().long()
        hi = (lo + 1).clamp(max=last)
        w = pos - lo.float()
        a = torch.gather(track, 1, lo)
        return a + (torch.gather(track, 1, hi) - a) * w, covered

    def correlation(self, batch: MediaBatch) -> torch.Tensor:
        v = self.video_drive(batch.video)
        a, covered = self.audio_drive_at(batch.audio, batch.video_positions, audio_fps=batch.spec.audio_fps)
        wts = covered.float()
        n = wts.sum(1, keepdim=True).clamp(min=1)
        vc = (v - (v * wts).sum(1, True) / n) * wts
        ac = (a - (a * wts).sum(1, True) / n) * wts
        den = vc.norm(dim=1) * ac.norm(dim=1)
        ok = (den > 0) & (wts.sum(1) >= 3)
        return torch.where(ok, (vc * ac).sum(1) / den.clamp(min=1e-12), torch.zeros_like(den))

    def holds(self, batch: MediaBatch) -> bool:
        return float(self.correlation(batch).min()) >= self.expected_correlation - self.tolerance


def _unit(seed: int, *labels: int | str) -> float:
    return (mix_seed(seed, *labels) >> 11) / float(1 << 52)


class SyntheticSource:
    """Iterator of :class:`MediaBatch` over this rank's procedural samples."""

    def __init__(self, config: SyntheticConfig | None = None, *, batch_size: int = 1, data_rank: int = 0,
                 data_world: int = 1, bucket_id: int = 0) -> None:
        self._config = config or SyntheticConfig()
        require_positive("batch_size", batch_size)
        require_positive("data_world", data_world)
        if not 0 <= data_rank < data_world:
            raise ValueError(f"data_rank={data_rank} must be below data_world={data_world}")
        self._batch_size = batch_size
        self._data_rank = data_rank
        self._data_world = data_world
        self._bucket_id = bucket_id
        self._local = tuple(range(data_rank, self._config.num_samples, data_world))
        if not self._local:
            raise ValueError("num_samples is smaller than data_world")
        self._cursor = 0
        self._epoch = 0
        g = torch.Generator().manual_seed(mix_seed(self._config.seed, "text-projection"))
        self._text_proj = torch.randn(6, self._config.text_tokens, self._config.text_width, generator=g)

    @property
    def config(self) -> SyntheticConfig:
        return self._config

    @property
    def batch_size(self) -> int:
        return self._batch_size

    def __len__(self) -> int:
        return len(self._local) // self._batch_size

    def alignment_truth(self) -> AlignmentTruth:
        c = self._config
        return AlignmentTruth(drive_frequency_hz=c.drive_frequency_hz, audio_lag_seconds=c.audio_lag_seconds,
                              video_drive_channel=0, audio_drive_channel=0)

    def sample_params(self, index: int) -> dict[str, float]:
        c = self._config
        f = c.drive_frequency_hz * (1.0 + c.drive_frequency_jitter * (2.0 * _unit(c.seed, index, "f") - 1.0))
        return {"frequency": f, "phase": 2 * math.pi * _unit(c.seed, index, "phase"),
                "vx": 2.0 * _unit(c.seed, index, "vx") - 1.0, "vy": 2.0 * _unit(c.seed, index, "vy") - 1.0,
                "kx": 1.0 + 3.0 * _unit(c.seed, index, "kx"), "ky": 1.0 + 3.0 * _unit(c.seed, index, "ky")}

    def _drive(self, t: torch.Tensor, p: Mapping[str, float]) -> torch.Tensor:
        c = self._config
        w = 2 * math.pi * p["frequency"]
        return torch.sin(w * t + p["phase"]) + c.drive_harmonic_gain * torch.sin(2 * w * t + 2 * p["phase"])

    def descriptor(self, index: int) -> SampleDescriptor:
        """Metadata of sample ``index`` without generating it: every synthetic sample has the
        configured geometry, so only the id varies. ``index`` must lie in ``[0, num_samples)``."""
        c = self._config
        if not 0 <= index < c.num_samples:
            raise IndexError(f"sample {index} is outside the synthetic corpus of {c.num_samples}")
        audio = c.has_audio
        return SampleDescriptor(sample_id=index, frames=c.frames, height=c.height, width=c.width,
                                channels=c.video_channels, audio_frames=c.audio_frames,
                                audio_channels=c.audio_channels if audio else 0, text_tokens=c.text_tokens,
                                text_width=c.text_width, video_timebase_num=c.video_timebase_num,
                                video_timebase_den=c.video_timebase_den, audio_timebase_num=c.audio_timebase_num,
                                audio_timebase_den=c.audio_timebase_den, video_codec_id=c.video_codec_id,
                                audio_codec_id=c.audio_codec_id if audio else "none")

    def sample(self, index: int) -> LatentSample:
        """Sample ``index`` (a pure function of the seed and the index)."""
        c = self._config
        p = self.sample_params(index)
        tv = torch.arange(c.frames, dtype=torch.float64) / c.video_fps
        drive_v = self._drive(tv, p).float()
        g = torch.Generator().manual_seed(mix_seed(c.seed, index, "texture"))
        texture = c.texture_scale * torch.randn(c.video_channels, c.height, c.width, generator=g)
        yy = torch.linspace(0, 1, c.height)[:, None]
        xx = torch.linspace(0, 1, c.width)[None, :]
        video = torch.empty(c.video_channels, c.frames, c.height, c.width)
        video[0] = c.motion_scale * drive_v[:, None, None] + texture[0]
        for ch in range(1, c.video_channels):
            shift = tv.float()[:, None, None] * c.motion_scale
            phase = 2 * math.pi * (p["kx"] * (xx - p["vx"] * shift) + p["ky"] * (yy - p["vy"] * shift)) + ch
            video[ch] = torch.sin(phase) + texture[ch]
        if c.has_audio:
            ta = torch.arange(c.audio_frames, dtype=torch.float64) / c.audio_fps
            audio = torch.empty(c.audio_channels, c.audio_frames)
            audio[0] = c.audio_gain * self._drive(ta - c.audio_lag_seconds, p).float()
            for ch in range(1, c.audio_channels):
                audio[ch] = torch.cos(2 * math.pi * p["frequency"] * (ch + 1) * ta).float()
        else:
            audio = torch.zeros(c.audio_channels, 0)
        coeff = torch.tensor([p["frequency"], math.sin(p["phase"]), math.cos(p["phase"]), p["vx"], p["vy"], 1.0])
        text = torch.einsum("k,ktd->td", coeff, self._text_proj)
        return LatentSample(descriptor=self.descriptor(index), video=video.to(c.dtype), audio=audio.to(c.dtype), text=text,
                            text_mask=torch.ones(c.text_tokens, dtype=torch.bool))

    def __iter__(self) -> Iterator[MediaBatch]:
        while True:
            if self._cursor + self._batch_size > len(self._local):
                self._cursor = 0
                self._epoch += 1
            idx = self._local[self._cursor:self._cursor + self._batch_size]
            self._cursor += self._batch_size
            yield collate_samples([self.sample(i) for i in idx], bucket_id=self._bucket_id,
                                  text_tokens=self._config.text_tokens)

    def advance(self, samples: int) -> None:
        self._cursor += samples

    def state_dict(self) -> dict[str, Any]:
        return {"cursor": self._cursor, "epoch": self._epoch, "data_rank": self._data_rank,
                "data_world": self._data_world, "seed": self._config.seed}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        if int(state.get("data_world", self._data_world)) != self._data_world:
            raise ValueError("cannot resume a synthetic stream on a different data_world")
        self._cursor = int(state["cursor"])
        self._epoch = int(state.get("epoch", 0))
