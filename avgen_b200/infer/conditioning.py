"""Inference-time conditioning (avgen/infer/conditioning.py:80-720 API).

A :class:`StreamState` is one modality's latent grid during sampling plus its
frame rate and optional clean anchors (a first frame, a temporal prefix, an
inpainting mask, or a whole other modality). :func:`build_model_input` turns
the states into the model's token contract at flow time ``sigma``: anchored
positions are replaced by their clean values at noise level 0 and flagged
``conditioned``; everything else sits at ``sigma``. When the anchors are
patch-aligned the per-token levels take two values per sample, which the
stream records as level groups so the model computes adaLN modulation once per
level.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import cast

import torch

from avgen_b200.core.batch import ConditionMode
from avgen_b200.core.model_input import ModelInput
from avgen_b200.core.patchify import GridPatchifier, Patchifier
from avgen_b200.core.tokens import PatchLayout, TextContext, TokenStream

__all__ = ["StreamState", "build_model_input", "condition_first_frame", "condition_mask", "condition_stream",
           "condition_temporal_prefix", "default_audio_patchifier", "first_frame_mask", "temporal_prefix_mask",
           "unconditional_input"]


def default_audio_patchifier() -> GridPatchifier:
    return GridPatchifier(patch_frames=1, patch_height=1, patch_width=1)


@dataclass(frozen=True, slots=True)
class StreamState:
    """Latents ``(B, C, T, H, W)`` (video) or ``(B, C, T)`` (audio) during sampling."""

    latents: torch.Tensor
    fps: float
    anchor: torch.Tensor | None = None
    anchor_mask: torch.Tensor | None = None
    start_seconds: float = 0.0
    valid_mask: torch.Tensor | None = None

    def __post_init__(self) -> None:
        if not (math.isfinite(self.fps) and self.fps > 0.0):
            raise ValueError(f"fps must be finite and positive; got {self.fps!r}")
        if not math.isfinite(self.start_seconds):
            raise ValueError(f"start_seconds must be finite; got {self.start_seconds!r}")
        if self.latents.ndim not in (3, 5):
            raise ValueError(f"latents must be rank 5 (video) or rank 3 (audio); got {tuple(self.latents.shape)}")
        if (self.anchor is None) != (self.anchor_mask is None):
            raise ValueError("anchor and anchor_mask go together")
        if self.anchor is not None and tuple(self.anchor.shape) != tuple(self.latents.shape):
            raise ValueError(f"anchor must have shape {tuple(self.latents.shape)}; got {tuple(self.anchor.shape)}")
        for name in ("anchor_mask", "valid_mask"):
            m = getattr(self, name)
            if m is None:
                continue
            if tuple(m.shape) != self.element_shape:
                raise ValueError(f"{name} must have shape {self.element_shape}; got {tuple(m.shape)}")
            if m.dtype is not torch.bool:
                raise TypeError(f"{name} must be bool; got {m.dtype}")

    @property
    def is_audio(self) -> bool:
        return cast("bool", self.latents.ndim == 3)

    @property
    def batch_size(self) -> int:
        return int(self.latents.shape[0])

    @property
    def frames(self) -> int:
        return int(self.latents.shape[2])

    @property
    def element_shape(self) -> tuple[int, ...]:
        """Shape of a per-position mask: the latents without the channel axis."""
        s = tuple(int(v) for v in self.latents.shape)
        return (s[0], *s[2:])

    @property
    def has_anchor(self) -> bool:
        return self.anchor_mask is not None

    def grid(self) -> torch.Tensor:
        """A 5-D view (audio gets unit height and width)."""
        return self.latents[..., None, None] if self.is_audio else self.latents

    def with_latents(self, latents: torch.Tensor) -> StreamState:
        return replace(self, latents=latents)

    def positions(self) -> torch.Tensor:
        """Start time in seconds of every latent frame, ``(B, T)``."""
        t = self.start_seconds + torch.arange(self.frames, device=self.latents.device, dtype=torch.float32) / self.fps
        return t[None].expand(self.batch_size, self.frames)


def first_frame_mask(state: StreamState, *, frames: int = 1, device: torch.device | None = None) -> torch.Tensor:
    if isinstance(frames, bool) or not 1 <= frames <= state.frames:
        raise ValueError(f"frames must be in [1, {state.frames}]; got {frames!r}")
    mask = torch.zeros(state.element_shape, dtype=torch.bool, device=device or state.latents.device)
    mask[:, :frames] = True
    return mask


def temporal_prefix_mask(state: StreamState, *, frames: int, device: torch.device | None = None) -> torch.Tensor:
    return first_frame_mask(state, frames=frames, device=device)


def _sigma_ok(name: str, v: float) -> None:
    if not (math.isfinite(v) and 0.0 <= v <= 1.0):
        raise ValueError(f"{name} must be a flow time in [0, 1]; got {v!r}")


def _to_stream(state: StreamState, sigma: float, patchifier: Patchifier) -> TokenStream:
    grid = state.grid()
    b, dev = state.batch_size, grid.device
    eshape = (grid.shape[0], *grid.shape[2:])
    valid = torch.ones(eshape, dtype=torch.bool, device=dev) if state.valid_mask is None else \
        state.valid_mask.reshape(eshape)
    if state.anchor is None or state.anchor_mask is None:
        level = torch.full((b,), float(sigma), dtype=torch.float32, device=dev)
        return patchifier.to_tokens(grid, positions=state.positions(), mask=valid, noise_level=level)
    amask = state.anchor_mask.reshape(eshape)
    mixed = torch.where(amask[:, None], state.anchor.reshape(grid.shape).to(grid.dtype), grid)
    level_grid = torch.where(amask, 0.0, float(sigma)).to(torch.float32)
    stream = patchifier.to_tokens(mixed, positions=state.positions(), mask=valid, noise_level=level_grid,
                                  conditioned=amask)
    # patch-aligned anchors: per-token levels are exactly {sigma, 0}; record them as two groups
    index = stream.conditioned.to(torch.int32)
    values = torch.tensor([float(sigma), 0.0], dtype=torch.float32, device=dev).expand(b, 2).contiguous()
    if torch.equal(values.gather(1, index.long()), stream.noise_level):
        stream = replace(stream, level_values=values, level_index=index)
    return stream


def build_model_input(*, video: StreamState, sigma: float, text: TextContext, patchifier: Patchifier,
                      condition_mode: ConditionMode = ConditionMode.JOINT, audio: StreamState | None = None,
                      audio_patchifier: Patchifier | None = None, audio_sigma: float | None = None) -> ModelInput:
    _sigma_ok("sigma", sigma)
    a_sigma = sigma if audio_sigma is None else audio_sigma
    _sigma_ok("audio_sigma", a_sigma)
    vstream = _to_stream(video, sigma, patchifier)
    if audio is None:
        astream = TokenStream.empty_like(video.batch_size, PatchLayout.empty().patch_dim, device=video.latents.device,
                                         dtype=video.latents.dtype)
    else:
        if audio.batch_size != video.batch_size:
            raise ValueError(f"audio batch {audio.batch_size} must match video batch {video.batch_size}")
        astream = _to_stream(audio, a_sigma, audio_patchifier or default_audio_patchifier())
    modes = torch.full((video.batch_size,), int(condition_mode), dtype=torch.int64, device=video.latents.device)
    inputs = ModelInput(video=vstream, audio=astream, text=text, condition_mode=modes)
    inputs.validate()
    return inputs


def unconditional_input(video: StreamState, *, sigma: float, text: TextContext, patchifier: Patchifier,
                        audio: StreamState | None = None, audio_patchifier: Patchifier | None = None) -> ModelInput:
    """No anchors and the given (typically null) text."""
    mode = ConditionMode.JOINT if audio is not None else ConditionMode.VIDEO_ONLY
    bare = replace(video, anchor=None, anchor_mask=None)
    bare_audio = replace(audio, anchor=None, anchor_mask=None) if audio is not None else None
    return build_model_input(video=bare, sigma=sigma, text=text, patchifier=patchifier, condition_mode=mode,
                             audio=bare_audio, audio_patchifier=audio_patchifier)


def _with_prefix(state: StreamState, anchor: torch.Tensor, frames: int) -> StreamState:
    if anchor.ndim == 4:
        anchor = anchor[:, :, None]
    if anchor.ndim != 5:
        raise ValueError(f"anchor must be a single frame (rank 4) or a grid (rank 5); got {tuple(anchor.shape)}")
    want = (state.latents.shape[0], state.latents.shape[1], frames, *state.latents.shape[3:])
    if tuple(anchor.shape) != tuple(want):
        raise ValueError(f"anchor must have shape {tuple(want)}; got {tuple(anchor.shape)}")
    canvas = state.latents.clone()
    canvas[:, :, :frames] = anchor.to(canvas.dtype)
    return replace(state, anchor=canvas, anchor_mask=first_frame_mask(state, frames=frames))


def condition_first_frame(video: StreamState, first_frame: torch.Tensor, *, sigma: float, text: TextContext,
                          patchifier: Patchifier, latent_frames: int = 1, audio: StreamState | None = None,
                          audio_patchifier: Patchifier | None = None) -> ModelInput:
    return build_model_input(video=_with_prefix(video, first_frame, latent_frames), sigma=sigma, text=text,
                             patchifier=patchifier, condition_mode=ConditionMode.IMAGE_TO_VIDEO, audio=audio,
                             audio_patchifier=audio_patchifier)


def condition_temporal_prefix(video: StreamState, prefix: torch.Tensor, *, sigma: float, text: TextContext,
                              patchifier: Patchifier, audio: StreamState | None = None,
                              audio_patchifier: Patchifier | None = None) -> ModelInput:
    if prefix.ndim != 5:
        raise ValueError(f"prefix must be a rank-5 latent grid; got {tuple(prefix.shape)}")
    return build_model_input(video=_with_prefix(video, prefix, int(prefix.shape[2])), sigma=sigma, text=text,
                             patchifier=patchifier, condition_mode=ConditionMode.CONTINUATION, audio=audio,
                             audio_patchifier=audio_patchifier)


def condition_mask(video: StreamState, known: torch.Tensor, mask: torch.Tensor, *, sigma: float, text: TextContext,
                   patchifier: Patchifier, audio: StreamState | None = None,
                   audio_patchifier: Patchifier | None = None) -> ModelInput:
    return build_model_input(video=replace(video, anchor=known, anchor_mask=mask), sigma=sigma, text=text,
                             patchifier=patchifier, condition_mode=ConditionMode.INPAINT, audio=audio,
                             audio_patchifier=audio_patchifier)


def _anchor_all(state: StreamState) -> StreamState:
    return replace(state, anchor=state.latents,
                   anchor_mask=torch.ones(state.element_shape, dtype=torch.bool, device=state.latents.device))


def condition_stream(*, video: StreamState, audio: StreamState, generate: str, sigma: float, text: TextContext,
                     patchifier: Patchifier, audio_patchifier: Patchifier | None = None) -> ModelInput:
    """Generate one modality with the other fully given (video-to-audio or audio-to-video)."""
    if generate == "audio":
        return build_model_input(video=_anchor_all(video), sigma=0.0, text=text, patchifier=patchifier,
                                 condition_mode=ConditionMode.VIDEO_TO_AUDIO, audio=audio,
                                 audio_patchifier=audio_patchifier, audio_sigma=sigma)
    if generate == "video":
        return build_model_input(video=video, sigma=sigma, text=text, patchifier=patchifier,
                                 condition_mode=ConditionMode.AUDIO_TO_VIDEO, audio=_anchor_all(audio),
                                 audio_patchifier=audio_patchifier, audio_sigma=0.0)
    raise ValueError(f"generate must be 'audio' or 'video'; got {generate!r}")
