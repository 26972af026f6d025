"""Sequence-first token contracts: PatchLayout, TokenStream, TextContext.

Every model interior works on token sequences ``(batch, length, width)`` with
explicit per-token physical coordinates ``(seconds, row, column)``, a validity
mask, a per-sample or per-token noise level and a clean-conditioning mask.
Dimension 1 is the axis context parallelism shards. Same contract as
avgen/core/tokens.py:42-476 (PatchLayout 42-165, TokenStream 167-361,
TextContext 363-443, pytree registration 470-476).
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

import torch
from torch.utils import _pytree

from avgen_b200.core._validate import require_dtype, require_positive, require_shape

__all__ = ["PatchLayout", "TextContext", "TokenStream"]


@dataclass(frozen=True, slots=True)
class PatchLayout:
    """Static grid geometry needed to fold tokens back into a latent grid.

    Args:
        frames, height, width: latent extent before patching.
        patch_frames, patch_height, patch_width: patch size per axis.
        channels: latent channels.
    """

    frames: int
    height: int
    width: int
    patch_frames: int = 1
    patch_height: int = 2
    patch_width: int = 2
    channels: int = 1

    def __post_init__(self) -> None:
        for name in ("frames", "height", "width", "patch_frames", "patch_height", "patch_width", "channels"):
            require_positive(name, getattr(self, name))
        for axis, patch in (("frames", "patch_frames"), ("height", "patch_height"), ("width", "patch_width")):
            if getattr(self, axis) % getattr(self, patch):
                raise ValueError(
                    f"{axis}={getattr(self, axis)} must be divisible by {patch}={getattr(self, patch)}; "
                    "pad or crop at the data boundary"
                )

    @property
    def grid(self) -> tuple[int, int, int]:
        """Post-patch grid ``(frames, height, width)``."""
        return (self.frames // self.patch_frames, self.height // self.patch_height, self.width // self.patch_width)

    @property
    def num_tokens(self) -> int:
        f, h, w = self.grid
        return f * h * w

    @property
    def patch_dim(self) -> int:
        return self.channels * self.patch_frames * self.patch_height * self.patch_width

    def is_temporal_only(self) -> bool:
        return self.height == 1 and self.width == 1

    @classmethod
    def temporal(cls, frames: int, channels: int, patch_frames: int = 1) -> PatchLayout:
        """1-D layout of an audio-like stream."""
        return cls(frames=frames, height=1, width=1, patch_frames=patch_frames, patch_height=1, patch_width=1,
                   channels=channels)

    @classmethod
    def empty(cls) -> PatchLayout:
        """Layout of an absent stream (all patch sizes one)."""
        return cls(frames=1, height=1, width=1, patch_frames=1, patch_height=1, patch_width=1, channels=1)


def _empty_bool() -> torch.Tensor:
    return torch.empty(0, dtype=torch.bool)


@dataclass(frozen=True, slots=True)
class TokenStream:
    """One modality's tokens with coordinates, mask and noise state.

    Args:
        tokens: ``(B, L, W)`` features.
        coords: ``(B, L, 3)`` fp32 ``(seconds, row, column)``.
        mask: ``(B, L)`` validity.
        noise_level: ``(B,)`` per-sample or ``(B, L)`` per-token, fp32 in [0, 1].
        layout: static geometry.
        conditioned: ``(B, L)`` clean anchors (attended, excluded from the loss).
        level_values: optional ``(B, G)`` fp32 distinct noise levels of each sample.
        level_index: optional ``(B, L)`` int32 with ``noise_level[b, l] ==
            level_values[b, level_index[b, l]]``. Producers that know their per-token
            levels take few values (clean conditioning frames at 0, the rest at
            ``t``) set both, so the model computes adaLN modulation once per level
            instead of once per token. Empty when absent.
    """

    tokens: torch.Tensor
    coords: torch.Tensor
    mask: torch.Tensor
    noise_level: torch.Tensor
    layout: PatchLayout
    conditioned: torch.Tensor = field(default_factory=_empty_bool)
    level_values: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    level_index: torch.Tensor = field(default_factory=lambda: torch.empty(0, dtype=torch.int32))

    def __post_init__(self) -> None:
        if self.conditioned.numel() == 0:
            object.__setattr__(
                self, "conditioned", torch.zeros(self.tokens.shape[:2], dtype=torch.bool, device=self.tokens.device)
            )

    @property
    def batch_size(self) -> int:
        return int(self.tokens.shape[0])

    @property
    def length(self) -> int:
        """Local length (the CP shard length under context parallelism)."""
        return int(self.tokens.shape[1])

    @property
    def width(self) -> int:
        return int(self.tokens.shape[2])

    @property
    def device(self) -> torch.device:
        return self.tokens.device

    @property
    def is_empty(self) -> bool:
        return self.tokens.shape[1] == 0 or not bool(self.mask.any())

    @property
    def per_token_noise(self) -> bool:
        return self.noise_level.ndim == 2

    @property
    def has_level_groups(self) -> bool:
        return self.level_values.numel() > 0

    def expanded_noise(self) -> torch.Tensor:
        """Noise level broadcast to ``(B, L)``."""
        if self.per_token_noise:
            return self.noise_level
        return self.noise_level[:, None].expand(self.tokens.shape[:2])

    def with_tokens(self, tokens: torch.Tensor) -> TokenStream:
        return replace(self, tokens=tokens)

    def masked(self) -> torch.Tensor:
        """Tokens with padding positions zeroed."""
        return self.tokens * self.mask.unsqueeze(-1).to(self.tokens.dtype)

    def loss_mask(self) -> torch.Tensor:
        """Valid and not clean-conditioned: the tokens the objective supervises."""
        return self.mask & ~self.conditioned

    def validate(self) -> None:
        if self.tokens.ndim != 3:
            raise ValueError(f"tokens must have rank 3 (batch, length, width); got {tuple(self.tokens.shape)}")
        batch, length, _ = self.tokens.shape
        require_shape("coords", self.coords, (batch, length, 3))
        require_shape("mask", self.mask, (batch, length))
        require_shape("conditioned", self.conditioned, (batch, length))
        if tuple(self.noise_level.shape) not in {(batch,), (batch, length)}:
            raise ValueError(f"noise_level must be ({batch},) or ({batch}, {length}); got {tuple(self.noise_level.shape)}")
        if not self.tokens.is_floating_point():
            raise TypeError(f"tokens must be floating point; got {self.tokens.dtype}")
        require_dtype("coords", self.coords, torch.float32)
        require_dtype("mask", self.mask, torch.bool)
        require_dtype("conditioned", self.conditioned, torch.bool)
        require_dtype("noise_level", self.noise_level, torch.float32)
        for name in ("coords", "mask", "conditioned", "noise_level"):
            if getattr(self, name).device != self.tokens.device:
                raise ValueError(f"{name} must be on tokens device {self.tokens.device}")
        if self.level_index.numel():
            require_shape("level_index", self.level_index, (batch, length))
            require_dtype("level_index", self.level_index, torch.int32)
            require_dtype("level_values", self.level_values, torch.float32)
            if self.level_values.ndim != 2 or self.level_values.shape[0] != batch:
                raise ValueError(f"level_values must be ({batch}, G); got {tuple(self.level_values.shape)}")
            expanded = self.level_values.gather(1, self.level_index.long())
            if not torch.equal(expanded, self.expanded_noise()):
                raise ValueError("level_values[level_index] must equal noise_level")

    @classmethod
    def empty_like(cls, batch: int, width: int, *, device: torch.device | str = "cpu",
                   dtype: torch.dtype = torch.float32) -> TokenStream:
        """Zero-length stream standing in for an absent modality."""
        dev = torch.device(device)
        return cls(
            tokens=torch.zeros((batch, 0, width), dtype=dtype, device=dev),
            coords=torch.zeros((batch, 0, 3), dtype=torch.float32, device=dev),
            mask=torch.zeros((batch, 0), dtype=torch.bool, device=dev),
            noise_level=torch.zeros((batch,), dtype=torch.float32, device=dev),
            layout=PatchLayout.empty(),
            conditioned=torch.zeros((batch, 0), dtype=torch.bool, device=dev),
        )


@dataclass(frozen=True, slots=True)
class TextContext:
    """Frozen text-encoder features for cross-attention (never CP-sharded)."""

    features: torch.Tensor
    mask: torch.Tensor

    @property
    def is_empty(self) -> bool:
        return self.features.shape[1] == 0

    def validate(self) -> None:
        if self.features.ndim != 3:
            raise ValueError(f"text features must have rank 3; got {tuple(self.features.shape)}")
        batch, tokens, _ = self.features.shape
        require_shape("text mask", self.mask, (batch, tokens))
        require_dtype("text mask", self.mask, torch.bool)
        if self.mask.device != self.features.device:
            raise ValueError("text mask must be on the features device")

    def nullified(self) -> TextContext:
        """Zero features and mask: the unconditional context of CFG."""
        return TextContext(features=torch.zeros_like(self.features), mask=torch.zeros_like(self.mask))

    @classmethod
    def empty(cls, batch: int, width: int, *, device: torch.device | str = "cpu",
              dtype: torch.dtype = torch.float32) -> TextContext:
        dev = torch.device(device)
        return cls(features=torch.zeros((batch, 0, width), dtype=dtype, device=dev),
                   mask=torch.zeros((batch, 0), dtype=torch.bool, device=dev))


def _flatten_stream(stream: TokenStream) -> tuple[list[torch.Tensor], PatchLayout]:
    return [stream.tokens, stream.coords, stream.mask, stream.noise_level, stream.conditioned, stream.level_values,
            stream.level_index], stream.layout


def _unflatten_stream(values: list[torch.Tensor], layout: PatchLayout) -> TokenStream:
    tokens, coords, mask, noise, cond, lv, li = values
    return TokenStream(tokens=tokens, coords=coords, mask=mask, noise_level=noise, layout=layout, conditioned=cond,
                       level_values=lv, level_index=li)


_pytree.register_pytree_node(TokenStream, _flatten_stream, _unflatten_stream,
                             serialized_type_name="avgen_b200.TokenStream")
_pytree.register_dataclass(TextContext, serialized_type_name="avgen_b200.TextContext")
