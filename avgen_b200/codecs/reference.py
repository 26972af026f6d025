"""Dependency-free reference codecs (avgen/codecs/reference.py:100-519 API).

Exact, invertible stand-ins for a VAE, an audio codec and a text encoder, used
by tests, the synthetic data path and smoke runs:

* video: space-time-to-depth folding (``temporal x spatial x spatial`` blocks
  into channels) followed by a seeded orthogonal channel rotation;
* audio: ``hop_length`` samples folded into channels, then the same rotation;
* text: UTF-8 bytes through a seeded byte-embedding table plus a sinusoidal
  position code, with a validity mask (an empty prompt is the null text).

The rotation is the Q factor of the QR decomposition of a seeded Gaussian
matrix (sign-fixed so it is unique), so decode(encode(x)) == x up to rounding.
"""
from __future__ import annotations

import math
from collections.abc import Sequence
from dataclasses import dataclass
from functools import lru_cache

import torch

from avgen_b200.codecs.normalization import LatentStatistics
from avgen_b200.codecs.protocols import codec_fingerprint

__all__ = ["ReferenceAudioCodec", "ReferenceTextEncoder", "ReferenceVideoCodec"]


@lru_cache(maxsize=32)
def _rotation(width: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(0x5EED0000 + seed)
    q, r = torch.linalg.qr(torch.randn((width, width), generator=g, dtype=torch.float64))
    return q * torch.sign(torch.diagonal(r)).where(torch.diagonal(r) != 0, torch.ones(()))[None, :]


def _rotate(t: torch.Tensor, seed: int, *, inverse: bool = False) -> torch.Tensor:
    m = _rotation(t.shape[1], seed).to(device=t.device, dtype=t.dtype)
    return torch.movedim(torch.movedim(t, 1, -1) @ (m.t() if inverse else m), -1, 1)


def _positive(name: str, value: int) -> None:
    if isinstance(value, bool) or int(value) < 1:
        raise ValueError(f"{name} must be a positive integer; got {value!r}")


def _positive_scale(scale: float) -> None:
    if not math.isfinite(scale) or scale <= 0.0:
        raise ValueError(f"scale must be finite and positive; got {scale!r}")


@dataclass(frozen=True, slots=True)
class ReferenceVideoCodec:
    channels: int = 3
    temporal_compression: int = 1
    spatial_compression: int = 2
    scale: float = 1.0
    seed: int = 0

    def __post_init__(self) -> None:
        for name in ("channels", "temporal_compression", "spatial_compression"):
            _positive(name, getattr(self, name))
        _positive_scale(self.scale)

    @property
    def fingerprint(self) -> str:
        return codec_fingerprint("video", "avgen_b200.reference",
                                 {"channels": self.channels, "tc": self.temporal_compression,
                                  "sc": self.spatial_compression, "scale": self.scale, "seed": self.seed})

    @property
    def latent_channels(self) -> int:
        return self.channels * self.temporal_compression * self.spatial_compression ** 2

    @property
    def latent_statistics(self) -> LatentStatistics:
        return LatentStatistics.from_scalar(self.latent_channels, std=self.scale)

    def latent_shape(self, pixel_shape: Sequence[int]) -> tuple[int, int, int, int, int]:
        shape = tuple(int(v) for v in pixel_shape)
        if len(shape) != 5:
            raise ValueError(f"pixel shape must be (batch, channels, frames, height, width); got {shape}")
        b, c, t, h, w = shape
        if c != self.channels:
            raise ValueError(f"expected {self.channels} pixel channels; got {c}")
        tc, sc = self.temporal_compression, self.spatial_compression
        for name, n, f in (("frames", t, tc), ("height", h, sc), ("width", w, sc)):
            if n % f:
                raise ValueError(f"{name}={n} is not divisible by its compression {f}; pad or crop first")
        return b, self.latent_channels, t // tc, h // sc, w // sc

    def pixel_shape(self, latent_shape: Sequence[int]) -> tuple[int, int, int, int, int]:
        shape = tuple(int(v) for v in latent_shape)
        if len(shape) != 5:
            raise ValueError(f"latent shape must be rank 5; got {shape}")
        b, c, t, h, w = shape
        if c != self.latent_channels:
            raise ValueError(f"expected {self.latent_channels} latent channels; got {c}")
        return b, self.channels, t * self.temporal_compression, h * self.spatial_compression, w * self.spatial_compression

    def encode(self, pixels: torch.Tensor) -> torch.Tensor:
        if not pixels.is_floating_point():
            raise TypeError(f"pixels must be floating point; got {pixels.dtype}")
        b, lc, t, h, w = self.latent_shape(pixels.shape)
        tc, sc = self.temporal_compression, self.spatial_compression
        x = pixels.reshape(b, self.channels, t, tc, h, sc, w, sc).permute(0, 3, 5, 7, 1, 2, 4, 6)
        return _rotate(x.reshape(b, lc, t, h, w), self.seed) * self.scale

    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        if not latents.is_floating_point():
            raise TypeError(f"latents must be floating point; got {latents.dtype}")
        b, c, t, h, w = self.pixel_shape(latents.shape)
        tc, sc = self.temporal_compression, self.spatial_compression
        x = _rotate(latents / self.scale, self.seed, inverse=True)
        x = x.reshape(b, tc, sc, sc, c, t // tc, h // sc, w // sc).permute(0, 4, 5, 1, 6, 2, 7, 3)
        return x.reshape(b, c, t, h, w)


@dataclass(frozen=True, slots=True)
class ReferenceAudioCodec:
    channels: int = 1
    hop_length: int = 256
    sample_rate: int = 24000
    scale: float = 1.0
    seed: int = 1

    def __post_init__(self) -> None:
        for name in ("channels", "hop_length", "sample_rate"):
            _positive(name, getattr(self, name))
        _positive_scale(self.scale)

    @property
    def fingerprint(self) -> str:
        return codec_fingerprint("audio", "avgen_b200.reference",
                                 {"channels": self.channels, "hop": self.hop_length, "sr": self.sample_rate,
                                  "scale": self.scale, "seed": self.seed})

    @property
    def latent_channels(self) -> int:
        return self.channels * self.hop_length

    @property
    def latent_rate(self) -> float:
        return self.sample_rate / self.hop_length

    @property
    def latent_statistics(self) -> LatentStatistics:
        return LatentStatistics.from_scalar(self.latent_channels, std=self.scale)

    def latent_frames(self, samples: int) -> int:
        if isinstance(samples, bool) or samples < 0:
            raise ValueError(f"samples must be non-negative; got {samples!r}")
        if samples % self.hop_length:
            raise ValueError(f"samples={samples} is not a multiple of hop_length={self.hop_length}; pad first")
        return samples // self.hop_length

    def num_samples(self, frames: int) -> int:
        return int(frames) * self.hop_length

    def encode(self, waveform: torch.Tensor) -> torch.Tensor:
        if not waveform.is_floating_point():
            raise TypeError(f"waveform must be floating point; got {waveform.dtype}")
        if waveform.ndim != 3 or waveform.shape[1] != self.channels:
            raise ValueError(f"waveform must be (batch, {self.channels}, samples); got {tuple(waveform.shape)}")
        b, c, n = waveform.shape
        f = self.latent_frames(n)
        x = waveform.reshape(b, c, f, self.hop_length).permute(0, 3, 1, 2).reshape(b, self.latent_channels, f)
        return _rotate(x, self.seed) * self.scale

    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        if not latents.is_floating_point():
            raise TypeError(f"latents must be floating point; got {latents.dtype}")
        if latents.ndim != 3 or latents.shape[1] != self.latent_channels:
            raise ValueError(f"latents must be (batch, {self.latent_channels}, frames); got {tuple(latents.shape)}")
        b, _, f = latents.shape
        x = _rotate(latents / self.scale, self.seed, inverse=True)
        x = x.reshape(b, self.hop_length, self.channels, f).permute(0, 2, 3, 1)
        return x.reshape(b, self.channels, f * self.hop_length)


@lru_cache(maxsize=8)
def _byte_embeddings(width: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(0x7E47 + seed)
    return torch.randn((256, width), generator=g) / math.sqrt(width)


@lru_cache(maxsize=16)
def _position_code(length: int, width: int) -> torch.Tensor:
    pos = torch.arange(length, dtype=torch.float64)[:, None]
    half = max(1, width // 2)
    freq = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
    code = torch.cat((torch.sin(pos * freq), torch.cos(pos * freq)), 1)[:, :width]
    if code.shape[1] < width:
        code = torch.cat((code, torch.zeros(length, width - code.shape[1], dtype=code.dtype)), 1)
    return (0.1 * code).float()


@dataclass(frozen=True, slots=True)
class ReferenceTextEncoder:
    width: int = 64
    max_length: int = 32
    seed: int = 2
    device: str = "cpu"

    def __post_init__(self) -> None:
        _positive("width", self.width)
        _positive("max_length", self.max_length)

    @property
    def fingerprint(self) -> str:
        return codec_fingerprint("text", "avgen_b200.reference",
                                 {"width": self.width, "max_length": self.max_length, "seed": self.seed})

    def encode(self, prompts: Sequence[str]) -> tuple[torch.Tensor, torch.Tensor]:
        if isinstance(prompts, str):
            prompts = [prompts]
        n = self.max_length
        ids = torch.zeros((len(prompts), n), dtype=torch.long)
        mask = torch.zeros((len(prompts), n), dtype=torch.bool)
        for i, p in enumerate(prompts):
            raw = list(p.encode("utf-8"))[:n]
            if raw:
                ids[i, :len(raw)] = torch.tensor(raw)
                mask[i, :len(raw)] = True
        feats = _byte_embeddings(self.width, self.seed)[ids] + _position_code(n, self.width)[None]
        feats = feats * mask[..., None]
        return feats.to(self.device), mask.to(self.device)
