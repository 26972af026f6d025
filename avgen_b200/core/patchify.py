"""Grid <-> token boundary (time-major, then row, then column).

Same behaviour as avgen/core/patchify.py:45-422: patches are flattened as
(channel, patch_t, patch_h, patch_w); token coordinates are the mean frame time
of the patch in seconds and the patch origin in latent pixels (or normalised to
[0, 1]); the validity mask reduces with *any* over a patch, the conditioning
mask with *all*, per-token noise with the patch mean.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol, runtime_checkable

import torch

from avgen_b200.core.tokens import PatchLayout, TokenStream

__all__ = ["GridPatchifier", "Patchifier", "build_spatial_coords", "build_temporal_coords", "patchify_grid",
           "unpatchify_grid"]


def build_temporal_coords(positions: torch.Tensor, layout: PatchLayout, *, normalize_space: bool = False) -> torch.Tensor:
    """Per-token ``(seconds, row, column)`` from per-frame times ``positions[B, T]``."""
    batch, frames = positions.shape
    if frames != layout.frames:
        raise ValueError(f"positions has {frames} frames but layout declares {layout.frames}")
    gf, gh, gw = layout.grid
    dev = positions.device
    time = positions.reshape(batch, gf, layout.patch_frames).mean(2)
    rows = torch.arange(gh, device=dev, dtype=torch.float32)
    cols = torch.arange(gw, device=dev, dtype=torch.float32)
    if normalize_space:
        rows = rows / max(gh - 1, 1)
        cols = cols / max(gw - 1, 1)
    else:
        rows = rows * layout.patch_height
        cols = cols * layout.patch_width
    shape = (batch, gf, gh, gw)
    t = time[:, :, None, None].expand(shape).reshape(batch, -1)
    r = rows[None, None, :, None].expand(shape).reshape(batch, -1)
    c = cols[None, None, None, :].expand(shape).reshape(batch, -1)
    return torch.stack((t, r, c), -1).to(torch.float32)


def build_spatial_coords(layout: PatchLayout, *, batch: int, fps: float, device: torch.device | str = "cpu",
                         start_seconds: float = 0.0) -> torch.Tensor:
    """Coordinates of a uniformly sampled clip at ``fps``."""
    if fps <= 0.0:
        raise ValueError(f"fps must be positive; got {fps!r}")
    frames = torch.arange(layout.frames, device=device, dtype=torch.float32)
    positions = (start_seconds + frames / fps)[None].expand(batch, layout.frames)
    return build_temporal_coords(positions, layout)


def patchify_grid(grid: torch.Tensor, layout: PatchLayout) -> torch.Tensor:
    """``(B, C, T, H, W)`` -> ``(B, L, C*pt*ph*pw)``."""
    expected = (grid.shape[0], layout.channels, layout.frames, layout.height, layout.width)
    if tuple(grid.shape) != expected:
        raise ValueError(f"grid shape must be {expected}; got {tuple(grid.shape)}")
    b = grid.shape[0]
    gf, gh, gw = layout.grid
    x = grid.reshape(b, layout.channels, gf, layout.patch_frames, gh, layout.patch_height, gw, layout.patch_width)
    return x.permute(0, 2, 4, 6, 1, 3, 5, 7).reshape(b, layout.num_tokens, layout.patch_dim)


def unpatchify_grid(tokens: torch.Tensor, layout: PatchLayout) -> torch.Tensor:
    """Inverse of :func:`patchify_grid`."""
    expected = (tokens.shape[0], layout.num_tokens, layout.patch_dim)
    if tuple(tokens.shape) != expected:
        raise ValueError(f"tokens shape must be {expected}; got {tuple(tokens.shape)}")
    b = tokens.shape[0]
    gf, gh, gw = layout.grid
    x = tokens.reshape(b, gf, gh, gw, layout.channels, layout.patch_frames, layout.patch_height, layout.patch_width)
    return x.permute(0, 4, 1, 5, 2, 6, 3, 7).reshape(b, layout.channels, layout.frames, layout.height, layout.width)


@runtime_checkable
class Patchifier(Protocol):
    def to_tokens(self, grid: torch.Tensor, *, positions: torch.Tensor, mask: torch.Tensor,
                  noise_level: torch.Tensor, conditioned: torch.Tensor | None = None) -> TokenStream: ...

    def to_grid(self, stream: TokenStream) -> torch.Tensor: ...

    def layout_for(self, grid_shape: tuple[int, ...]) -> PatchLayout: ...


@dataclass(frozen=True, slots=True)
class GridPatchifier:
    """Default patchifier over ``(B, C, T, H, W)`` latents."""

    patch_frames: int = 1
    patch_height: int = 2
    patch_width: int = 2
    normalize_space: bool = False

    def layout_for(self, grid_shape: tuple[int, ...]) -> PatchLayout:
        if len(grid_shape) != 5:
            raise ValueError(f"grid shape must be rank 5; got {grid_shape}")
        _, c, t, h, w = grid_shape
        return PatchLayout(frames=t, height=h, width=w, patch_frames=self.patch_frames,
                           patch_height=self.patch_height, patch_width=self.patch_width, channels=c)

    def to_tokens(self, grid: torch.Tensor, *, positions: torch.Tensor, mask: torch.Tensor,
                  noise_level: torch.Tensor, conditioned: torch.Tensor | None = None) -> TokenStream:
        layout = self.layout_for(tuple(grid.shape))
        b = grid.shape[0]
        tokens = patchify_grid(grid, layout)
        coords = build_temporal_coords(positions, layout, normalize_space=self.normalize_space)
        token_mask = self._reduce(mask, layout, b).any(-1)
        if conditioned is not None:
            token_cond = self._reduce(conditioned, layout, b).all(-1)
        else:
            token_cond = torch.zeros((b, layout.num_tokens), dtype=torch.bool, device=grid.device)
        if noise_level.ndim == 1:
            noise = noise_level
        else:
            noise = self._reduce(noise_level, layout, b).mean(-1).to(torch.float32)
        return TokenStream(tokens=tokens, coords=coords, mask=token_mask, noise_level=noise, layout=layout,
                           conditioned=token_cond)

    def to_grid(self, stream: TokenStream) -> torch.Tensor:
        return unpatchify_grid(stream.tokens, stream.layout)

    @staticmethod
    def _reduce(values: torch.Tensor, layout: PatchLayout, batch: int) -> torch.Tensor:
        expected = (batch, layout.frames, layout.height, layout.width)
        if tuple(values.shape) != expected:
            raise ValueError(f"per-pixel tensor must have shape {expected}; got {tuple(values.shape)}")
        gf, gh, gw = layout.grid
        v = values.reshape(batch, gf, layout.patch_frames, gh, layout.patch_height, gw, layout.patch_width)
        return v.permute(0, 1, 3, 5, 2, 4, 6).reshape(batch, layout.num_tokens, -1)
