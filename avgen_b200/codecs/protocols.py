"""Codec protocols (avgen/codecs/protocols.py:56-337 API).

Video latents are ``(B, C, T, H, W)``; audio latents ``(B, C, T)``; a text
encoder returns features ``(B, N, D)`` and a boolean mask ``(B, N)``. Every
codec exposes a ``fingerprint``: a stable hash of its identity and
configuration, stored with shards and checkpoints so that latents are never
decoded with a different codec than the one that made them.
"""
from __future__ import annotations

import hashlib
import json
from collections.abc import Mapping, Sequence
from typing import Any, Protocol, runtime_checkable

import torch

from avgen_b200.codecs.normalization import LatentStatistics

__all__ = ["AudioCodec", "TextEncoder", "VideoCodec", "Vocoder", "codec_fingerprint"]


def codec_fingerprint(kind: str, identity: str, config: Mapping[str, Any] | None = None) -> str:
    """``kind:identity:sha256(config)[:16]`` with the config serialised canonically."""
    if not kind or not identity:
        raise ValueError("kind and identity must be non-empty")
    blob = json.dumps(dict(config or {}), sort_keys=True, separators=(",", ":"), default=str)
    return f"{kind}:{identity}:{hashlib.sha256(blob.encode()).hexdigest()[:16]}"


@runtime_checkable
class VideoCodec(Protocol):
    @property
    def fingerprint(self) -> str: ...
    @property
    def latent_channels(self) -> int: ...
    @property
    def temporal_compression(self) -> int: ...
    @property
    def spatial_compression(self) -> int: ...
    @property
    def latent_statistics(self) -> LatentStatistics: ...
    def latent_shape(self, pixel_shape: Sequence[int]) -> tuple[int, int, int, int, int]: ...
    def pixel_shape(self, latent_shape: Sequence[int]) -> tuple[int, int, int, int, int]: ...
    def encode(self, pixels: torch.Tensor) -> torch.Tensor: ...
    def decode(self, latents: torch.Tensor) -> torch.Tensor: ...


@runtime_checkable
class AudioCodec(Protocol):
    @property
    def fingerprint(self) -> str: ...
    @property
    def latent_channels(self) -> int: ...
    @property
    def sample_rate(self) -> int: ...
    @property
    def hop_length(self) -> int: ...
    @property
    def latent_statistics(self) -> LatentStatistics: ...
    def latent_frames(self, samples: int) -> int: ...
    def encode(self, waveform: torch.Tensor) -> torch.Tensor: ...
    def decode(self, latents: torch.Tensor) -> torch.Tensor: ...


@runtime_checkable
class Vocoder(Protocol):
    @property
    def fingerprint(self) -> str: ...
    @property
    def sample_rate(self) -> int: ...
    @property
    def mel_bins(self) -> int: ...
    def decode(self, mel: torch.Tensor) -> torch.Tensor: ...


@runtime_checkable
class TextEncoder(Protocol):
    @property
    def fingerprint(self) -> str: ...
    @property
    def width(self) -> int: ...
    @property
    def max_length(self) -> int: ...
    def encode(self, prompts: Sequence[str]) -> tuple[torch.Tensor, torch.Tensor]: ...
