"""Multi-task conditioning plans (avgen/train/conditioning.py:64-399).

Per sample: a ConditionMode drawn from a weighted mixture (joint .55, V2A .05,
A2V .05, continuation .10, inpaint .05, I2V .20 by default), the clean-anchor
masks it implies (temporal prefix, first frame(s), random inpaint tokens, a
whole modality), anchor dropout, and text dropout for CFG.
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, field
from typing import Protocol, runtime_checkable

import torch

from avgen_b200.core._validate import require_dtype, require_probability, require_shape
from avgen_b200.core.batch import ConditionMode, MediaBatch
from avgen_b200.core.rng import RNGStreams
from avgen_b200.train._random import bernoulli, categorical, uniform

__all__ = ["ConditioningPlan", "ConditioningSampler", "MultiTaskConditioning", "default_mode_weights"]

_AUDIO_MODES = frozenset({ConditionMode.VIDEO_TO_AUDIO, ConditionMode.AUDIO_TO_VIDEO})


def default_mode_weights() -> tuple[tuple[ConditionMode, float], ...]:
    return ((ConditionMode.JOINT, 0.55), (ConditionMode.VIDEO_TO_AUDIO, 0.05), (ConditionMode.AUDIO_TO_VIDEO, 0.05),
            (ConditionMode.CONTINUATION, 0.10), (ConditionMode.INPAINT, 0.05), (ConditionMode.IMAGE_TO_VIDEO, 0.20))


@dataclass(frozen=True, slots=True)
class ConditioningPlan:
    condition_mode: torch.Tensor
    video_conditioned: torch.Tensor
    audio_conditioned: torch.Tensor
    drop_text: torch.Tensor

    @property
    def batch_size(self) -> int:
        return int(self.condition_mode.shape[0])

    def validate(self, batch: MediaBatch) -> None:
        size = batch.spec.batch_size
        _, _, t, h, w = batch.spec.video_shape
        require_shape("condition_mode", self.condition_mode, (size,))
        require_shape("video_conditioned", self.video_conditioned, (size, t, h, w))
        require_shape("audio_conditioned", self.audio_conditioned, (size, batch.spec.audio_tokens))
        require_shape("drop_text", self.drop_text, (size,))
        require_dtype("condition_mode", self.condition_mode, torch.int64)
        for name in ("video_conditioned", "audio_conditioned", "drop_text"):
            require_dtype(name, getattr(self, name), torch.bool)


@runtime_checkable
class ConditioningSampler(Protocol):
    def sample(self, batch: MediaBatch, *, rng: RNGStreams) -> ConditioningPlan: ...


@dataclass(frozen=True, slots=True)
class MultiTaskConditioning:
    mode_weights: tuple[tuple[ConditionMode, float], ...] = field(default_factory=default_mode_weights)
    continuation_prefix: tuple[float, float] = (0.125, 0.5)
    inpaint_ratio: tuple[float, float] = (0.1, 0.6)
    image_frames: int = 1
    text_dropout: float = 0.1
    video_anchor_dropout: float = 0.1
    audio_anchor_dropout: float = 0.1

    def __post_init__(self) -> None:
        if not self.mode_weights:
            raise ValueError("mode_weights must contain at least one entry")
        seen: set[ConditionMode] = set()
        for mode, weight in self.mode_weights:
            if not isinstance(mode, ConditionMode):
                raise TypeError(f"mode_weights key must be a ConditionMode; got {mode!r}")
            if mode in seen:
                raise ValueError(f"mode_weights contains {mode.name} twice")
            seen.add(mode)
            if weight < 0.0:
                raise ValueError(f"weight for {mode.name} must be >= 0")
        if sum(w for _, w in self.mode_weights) <= 0.0:
            raise ValueError("mode_weights must contain a positive weight")
        for name in ("continuation_prefix", "inpaint_ratio"):
            lo, hi = getattr(self, name)
            require_probability(f"{name}[0]", lo)
            require_probability(f"{name}[1]", hi)
            if lo > hi:
                raise ValueError(f"{name} must be ordered (low, high)")
        if isinstance(self.image_frames, bool) or self.image_frames < 1:
            raise ValueError("image_frames must be >= 1")
        for name in ("text_dropout", "video_anchor_dropout", "audio_anchor_dropout"):
            require_probability(name, getattr(self, name))

    @classmethod
    def from_weights(cls, weights: Mapping[ConditionMode | str | int, float], **options) -> MultiTaskConditioning:  # noqa: ANN003
        resolved = []
        for key, weight in weights.items():
            if isinstance(key, ConditionMode):
                mode = key
            elif isinstance(key, int):
                mode = ConditionMode(key)
            else:
                try:
                    mode = ConditionMode[key.upper()]
                except KeyError:
                    raise KeyError(f"unknown condition mode {key!r}") from None
            resolved.append((mode, float(weight)))
        resolved.sort(key=lambda p: int(p[0]))
        return cls(mode_weights=tuple(resolved), **options)

    def sample(self, batch: MediaBatch, *, rng: RNGStreams) -> ConditioningPlan:
        dev = batch.device
        g = rng.conditioning
        size = batch.spec.batch_size
        _, _, frames, height, width = batch.spec.video_shape
        a_frames = batch.spec.audio_tokens
        modes = self._draw_modes(size, batch=batch, generator=g, device=dev)
        video = torch.zeros((size, frames, height, width), dtype=torch.bool, device=dev)
        audio = torch.zeros((size, a_frames), dtype=torch.bool, device=dev)
        frame_index = torch.arange(frames, device=dev)[None]
        lo, hi = self.continuation_prefix
        ratio = lo + (hi - lo) * uniform((size,), generator=g, device=dev)
        cont = (ratio * frames).to(torch.int64).clamp(1, max(frames - 1, 1))
        prefix = torch.zeros((size,), dtype=torch.int64, device=dev)
        image = torch.full_like(prefix, min(self.image_frames, max(frames - 1, 1)))
        prefix = torch.where(modes == int(ConditionMode.CONTINUATION), cont, prefix)
        prefix = torch.where(modes == int(ConditionMode.IMAGE_TO_VIDEO), image, prefix)
        video |= (frame_index < prefix[:, None])[:, :, None, None]
        lo, hi = self.inpaint_ratio
        keep = lo + (hi - lo) * uniform((size,), generator=g, device=dev)
        draw = uniform((size, frames, height, width), generator=g, device=dev)
        video |= (draw < keep[:, None, None, None]) & (modes == int(ConditionMode.INPAINT))[:, None, None, None]
        video |= (modes == int(ConditionMode.VIDEO_TO_AUDIO))[:, None, None, None]
        audio |= (modes == int(ConditionMode.AUDIO_TO_VIDEO))[:, None]
        video &= ~bernoulli((size,), self.video_anchor_dropout, generator=g, device=dev)[:, None, None, None]
        audio &= ~bernoulli((size,), self.audio_anchor_dropout, generator=g, device=dev)[:, None]
        video &= batch.video_mask
        audio &= batch.audio_mask
        drop_text = bernoulli((size,), self.text_dropout, generator=g, device=dev)
        return ConditioningPlan(condition_mode=modes, video_conditioned=video, audio_conditioned=audio,
                                drop_text=drop_text)

    def _draw_modes(self, size: int, *, batch: MediaBatch, generator: torch.Generator,
                    device: torch.device) -> torch.Tensor:
        modes = [m for m, _ in self.mode_weights]
        weights = [w for _, w in self.mode_weights]
        if not batch.spec.has_audio:
            weights = [0.0 if m in _AUDIO_MODES else w for m, w in zip(modes, weights)]
        idx = categorical(torch.tensor(weights, dtype=torch.float32), size, generator=generator, device=device)
        lookup = torch.tensor([int(m) for m in modes], dtype=torch.int64, device=device)
        return lookup[idx]
