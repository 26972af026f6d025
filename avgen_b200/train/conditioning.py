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


def _resolve_mode(key: ConditionMode | str | int) -> ConditionMode:
    """A condition mode from itself, its integer value or its (case-insensitive) name."""
    if isinstance(key, ConditionMode):
        return key
    if isinstance(key, int):
        return ConditionMode(key)
    mode = ConditionMode.__members__.get(str(key).upper())
    if mode is None:
        raise KeyError(f"unknown condition mode {key!r}")
    return mode


@dataclass(frozen=True, slots=True)
class _Draws:
    """Every random quantity one plan needs, drawn up front from the conditioning stream."""

    modes: torch.Tensor           # int64 [B]
    prefix_fraction: torch.Tensor  # [B] continuation prefix as a fraction of the frames
    keep_fraction: torch.Tensor    # [B] inpaint: share of tokens kept clean
    keep_draw: torch.Tensor        # [B, T, H, W] uniform draw per token for inpainting
    drop_video: torch.Tensor       # bool [B] anchor dropout
    drop_audio: torch.Tensor
    drop_text: torch.Tensor


def _no_anchor(cfg, draws, frames, video_shape, audio_len):  # noqa: ANN001, ANN202
    return None, None


def _prefix_anchor(frames_kept: torch.Tensor, frames: int, video_shape: tuple[int, ...]) -> torch.Tensor:
    index = torch.arange(frames, device=frames_kept.device)
    return (index[None, :] < frames_kept[:, None])[:, :, None, None].expand(video_shape)


def _continuation_anchor(cfg, draws, frames, video_shape, audio_len):  # noqa: ANN001, ANN202
    kept = (draws.prefix_fraction * frames).to(torch.int64).clamp(1, max(frames - 1, 1))
    return _prefix_anchor(kept, frames, video_shape), None


def _image_anchor(cfg, draws, frames, video_shape, audio_len):  # noqa: ANN001, ANN202
    kept = torch.full_like(draws.modes, min(cfg.image_frames, max(frames - 1, 1)))
    return _prefix_anchor(kept, frames, video_shape), None


def _inpaint_anchor(cfg, draws, frames, video_shape, audio_len):  # noqa: ANN001, ANN202
    return draws.keep_draw < draws.keep_fraction[:, None, None, None], None


def _video_to_audio_anchor(cfg, draws, frames, video_shape, audio_len):  # noqa: ANN001, ANN202
    return torch.ones(video_shape, dtype=torch.bool, device=draws.modes.device), None


def _audio_to_video_anchor(cfg, draws, frames, video_shape, audio_len):  # noqa: ANN001, ANN202
    return None, torch.ones((video_shape[0], audio_len), dtype=torch.bool, device=draws.modes.device)


# Which clean anchors each task gives the model (the mode's definition): a
# continuation keeps a random prefix of frames, image-to-video the first frame(s),
# inpainting a random share of tokens, V2A the whole video, A2V the whole audio.
_ANCHORS = {
    ConditionMode.JOINT: _no_anchor,
    ConditionMode.CONTINUATION: _continuation_anchor,
    ConditionMode.IMAGE_TO_VIDEO: _image_anchor,
    ConditionMode.INPAINT: _inpaint_anchor,
    ConditionMode.VIDEO_TO_AUDIO: _video_to_audio_anchor,
    ConditionMode.AUDIO_TO_VIDEO: _audio_to_video_anchor,
}


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
        modes = [m for m, _ in self.mode_weights]
        bad = [m for m in modes if not isinstance(m, ConditionMode)]
        if not modes:
            raise ValueError("mode_weights must contain at least one entry")
        if bad:
            raise TypeError(f"mode_weights key must be a ConditionMode; got {bad[0]!r}")
        repeated = {m for m in modes if modes.count(m) > 1}
        if repeated:
            raise ValueError(f"mode_weights contains {sorted(repeated)[0].name} twice")
        negative = [m for m, w in self.mode_weights if w < 0.0]
        if negative:
            raise ValueError(f"weight for {negative[0].name} must be >= 0")
        if not any(w > 0.0 for _, w in self.mode_weights):
            raise ValueError("mode_weights must contain a positive weight")
        for name in ("continuation_prefix", "inpaint_ratio"):
            bounds = getattr(self, name)
            for i, value in enumerate(bounds):
                require_probability(f"{name}[{i}]", value)
            if bounds[0] > bounds[1]:
                raise ValueError(f"{name} must be ordered (low, high)")
        if isinstance(self.image_frames, bool) or self.image_frames < 1:
            raise ValueError("image_frames must be >= 1")
        for name in ("text_dropout", "video_anchor_dropout", "audio_anchor_dropout"):
            require_probability(name, getattr(self, name))

    @classmethod
    def from_weights(cls, weights: Mapping[ConditionMode | str | int, float], **options) -> MultiTaskConditioning:  # noqa: ANN003
        """Build from a mapping keyed by mode, mode name or mode value (ordered by mode value)."""
        table = sorted(((_resolve_mode(k), float(w)) for k, w in weights.items()), key=lambda mw: int(mw[0]))
        return cls(mode_weights=tuple(table), **options)

    def _draw(self, batch: MediaBatch, generator: torch.Generator) -> _Draws:
        dev = batch.device
        size = batch.spec.batch_size
        _, _, frames, height, width = batch.spec.video_shape

        def between(bounds: tuple[float, float]) -> torch.Tensor:
            return bounds[0] + (bounds[1] - bounds[0]) * uniform((size,), generator=generator, device=dev)

        modes = self._draw_modes(size, batch=batch, generator=generator, device=dev)
        prefix = between(self.continuation_prefix)
        keep = between(self.inpaint_ratio)
        keep_draw = uniform((size, frames, height, width), generator=generator, device=dev)
        drop_video = bernoulli((size,), self.video_anchor_dropout, generator=generator, device=dev)
        drop_audio = bernoulli((size,), self.audio_anchor_dropout, generator=generator, device=dev)
        drop_text = bernoulli((size,), self.text_dropout, generator=generator, device=dev)
        return _Draws(modes, prefix, keep, keep_draw, drop_video, drop_audio, drop_text)

    def sample(self, batch: MediaBatch, *, rng: RNGStreams) -> ConditioningPlan:
        """Draw a task per sample and the clean anchors it implies (masked by validity and anchor dropout)."""
        draws = self._draw(batch, rng.conditioning)
        size = batch.spec.batch_size
        _, _, frames, height, width = batch.spec.video_shape
        video_shape = (size, frames, height, width)
        audio_len = batch.spec.audio_tokens
        video = torch.zeros(video_shape, dtype=torch.bool, device=batch.device)
        audio = torch.zeros((size, audio_len), dtype=torch.bool, device=batch.device)
        for mode, anchor in _ANCHORS.items():
            chosen = draws.modes == int(mode)
            v, a = anchor(self, draws, frames, video_shape, audio_len)
            if v is not None:
                video |= v & chosen[:, None, None, None]
            if a is not None:
                audio |= a & chosen[:, None]
        video &= batch.video_mask & ~draws.drop_video[:, None, None, None]
        audio &= batch.audio_mask & ~draws.drop_audio[:, None]
        return ConditioningPlan(condition_mode=draws.modes, video_conditioned=video, audio_conditioned=audio,
                                drop_text=draws.drop_text)

    def _draw_modes(self, size: int, *, batch: MediaBatch, generator: torch.Generator,
                    device: torch.device) -> torch.Tensor:
        """Modes by weight; the audio tasks get weight 0 when the batch carries no audio."""
        usable = [(m, 0.0 if (m in _AUDIO_MODES and not batch.spec.has_audio) else w) for m, w in self.mode_weights]
        weights = torch.tensor([w for _, w in usable], dtype=torch.float32)
        values = torch.tensor([int(m) for m, _ in usable], dtype=torch.int64, device=device)
        return values[categorical(weights, size, generator=generator, device=device)]
