"""Adapters for pretrained codecs from ``diffusers`` / ``transformers``
(avgen/codecs/adapters.py:53-669 API). Both libraries are optional and loaded on
first use; weights come from a local path or the HF cache (no network here).

Tiled decode/encode splits long or large latents into overlapping windows and
blends them with linear ramps, so arbitrary resolutions fit in memory.
"""
from __future__ import annotations

import importlib
from collections.abc import Callable, Sequence
from dataclasses import asdict, dataclass
from typing import Any

import torch

from avgen_b200.codecs.normalization import LatentStatistics, resolve_latent_normalization
from avgen_b200.codecs.protocols import codec_fingerprint

__all__ = ["DiffusersVideoCodec", "TilingConfig", "TransformersTextEncoder", "blend_tiles"]


@dataclass(frozen=True, slots=True)
class TilingConfig:
    enabled: bool = False
    tile_size: int = 512
    tile_overlap: int = 128
    temporal_chunk: int = 0
    temporal_overlap: int = 0

    def __post_init__(self) -> None:
        for name in ("tile_size", "tile_overlap", "temporal_chunk", "temporal_overlap"):
            v = getattr(self, name)
            if isinstance(v, bool) or v < 0:
                raise ValueError(f"{name} must be a non-negative integer; got {v!r}")
        if self.enabled and self.tile_size < 1:
            raise ValueError("tile_size must be positive when tiling is enabled")
        if self.enabled and self.tile_overlap >= self.tile_size:
            raise ValueError("tile_overlap must be smaller than tile_size")
        if self.temporal_chunk and self.temporal_overlap >= self.temporal_chunk:
            raise ValueError("temporal_overlap must be smaller than temporal_chunk")

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def blend_tiles(total: int, tile: int, overlap: int) -> list[tuple[int, int]]:
    """``[start, stop)`` windows of ``tile`` covering ``total`` with ``overlap`` shared elements."""
    if total <= 0:
        return []
    if tile <= 0 or tile >= total:
        return [(0, total)]
    stride = max(1, tile - overlap)
    starts = list(range(0, max(1, total - tile) + 1, stride))
    if starts[-1] + tile < total:
        starts.append(total - tile)
    return [(s, min(total, s + tile)) for s in starts]


def _ramp_weights(n: int, ramp_in: int, ramp_out: int, device: torch.device) -> torch.Tensor:
    w = torch.ones(n, device=device, dtype=torch.float32)
    if ramp_in > 0:
        w[:ramp_in] = torch.linspace(0.0, 1.0, ramp_in + 2, device=device)[1:-1]
    if ramp_out > 0:
        w[n - ramp_out:] = torch.minimum(w[n - ramp_out:],
                                         torch.linspace(1.0, 0.0, ramp_out + 2, device=device)[1:-1])
    return w


def _tiled(x: torch.Tensor, fn: Callable[[torch.Tensor], torch.Tensor], tiling: TilingConfig, t_scale: float,
           s_scale: float) -> torch.Tensor:
    """Apply ``fn`` to overlapping (time, height, width) windows of ``x`` ``(B, C, T, H, W)``
    and blend; output extents are the input's times ``t_scale`` / ``s_scale``."""
    _, _, t, h, w = x.shape
    tw = blend_tiles(t, tiling.temporal_chunk, tiling.temporal_overlap) if tiling.temporal_chunk else [(0, t)]
    hw = blend_tiles(h, tiling.tile_size, tiling.tile_overlap)
    ww = blend_tiles(w, tiling.tile_size, tiling.tile_overlap)
    out = weight = None
    for t0, t1 in tw:
        for h0, h1 in hw:
            for w0, w1 in ww:
                y = fn(x[:, :, t0:t1, h0:h1, w0:w1]).float()
                if out is None:
                    shape = (y.shape[0], y.shape[1], round(t * t_scale), round(h * s_scale), round(w * s_scale))
                    out = torch.zeros(shape, device=y.device)
                    weight = torch.zeros(shape[2:], device=y.device)
                ot0, oh0, ow0 = round(t0 * t_scale), round(h0 * s_scale), round(w0 * s_scale)
                nt, nh, nw = y.shape[2:]
                ov_t = round(tiling.temporal_overlap * t_scale) if t0 > 0 else 0
                ov_h = round(tiling.tile_overlap * s_scale) if h0 > 0 else 0
                ov_w = round(tiling.tile_overlap * s_scale) if w0 > 0 else 0
                wt = _ramp_weights(nt, min(ov_t, nt), 0, y.device)
                wh = _ramp_weights(nh, min(ov_h, nh), 0, y.device)
                wv = _ramp_weights(nw, min(ov_w, nw), 0, y.device)
                wgt = wt[:, None, None] * wh[None, :, None] * wv[None, None, :]
                out[:, :, ot0:ot0 + nt, oh0:oh0 + nh, ow0:ow0 + nw] += y * wgt
                weight[ot0:ot0 + nt, oh0:oh0 + nh, ow0:ow0 + nw] += wgt
    assert out is not None and weight is not None
    return out / weight.clamp_min(1e-6)


def _require(module: str, extra: str) -> Any:
    try:
        return importlib.import_module(module)
    except ImportError as exc:
        raise RuntimeError(f"{module} is needed for this codec; install the '{extra}' extra") from exc


_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


class DiffusersVideoCodec:
    """A diffusers video autoencoder (``AutoencoderKL*``) as a :class:`VideoCodec`."""

    def __init__(self, model_id: str, *, subfolder: str | None = "vae", dtype: str = "float32", device: str = "cpu",
                 tiling: TilingConfig | None = None, statistics: LatentStatistics | None = None,
                 revision: str | None = None) -> None:
        self.model_id, self.subfolder, self.revision = model_id, subfolder, revision
        self.dtype, self.device = _DTYPES[dtype], torch.device(device)
        self.tiling = tiling or TilingConfig()
        self._statistics = statistics
        self._module: Any = None

    @property
    def module(self) -> Any:
        if self._module is None:
            diffusers = _require("diffusers", "codecs")
            loaders = [getattr(diffusers, n) for n in ("AutoencoderKLWan", "AutoencoderKLHunyuanVideo",
                                                       "AutoencoderKLCogVideoX", "AutoencoderKL")
                       if hasattr(diffusers, n)]
            last: Exception | None = None
            for cls in loaders:
                try:
                    self._module = cls.from_pretrained(self.model_id, subfolder=self.subfolder,
                                                       revision=self.revision, torch_dtype=self.dtype)
                    break
                except Exception as exc:  # noqa: BLE001 - try the next family
                    last = exc
            if self._module is None:
                raise RuntimeError(f"could not load a video autoencoder from {self.model_id!r}") from last
            self._module.to(self.device).eval().requires_grad_(False)
        return self._module

    @property
    def fingerprint(self) -> str:
        return codec_fingerprint("video", f"diffusers:{self.model_id}",
                                 {"subfolder": self.subfolder, "revision": self.revision})

    def _config(self) -> Any:
        return self.module.config

    @property
    def latent_channels(self) -> int:
        c = self._config()
        return int(getattr(c, "latent_channels", None) or getattr(c, "z_dim"))

    @property
    def temporal_compression(self) -> int:
        c = self._config()
        return int(getattr(c, "temporal_compression_ratio", None) or getattr(c, "scale_factor_temporal", 4) or 4)

    @property
    def spatial_compression(self) -> int:
        c = self._config()
        return int(getattr(c, "spatial_compression_ratio", None) or getattr(c, "scale_factor_spatial", 8) or 8)

    @property
    def latent_statistics(self) -> LatentStatistics:
        if self._statistics is None:
            self._statistics = resolve_latent_normalization(dict(self._config()), channels=self.latent_channels)
        return self._statistics

    def latent_shape(self, pixel_shape: Sequence[int]) -> tuple[int, int, int, int, int]:
        b, _, t, h, w = (int(v) for v in pixel_shape)
        tc, sc = self.temporal_compression, self.spatial_compression
        return b, self.latent_channels, (t - 1) // tc + 1, h // sc, w // sc

    def pixel_shape(self, latent_shape: Sequence[int]) -> tuple[int, int, int, int, int]:
        b, _, t, h, w = (int(v) for v in latent_shape)
        tc, sc = self.temporal_compression, self.spatial_compression
        return b, 3, (t - 1) * tc + 1, h * sc, w * sc

    @torch.no_grad()
    def encode(self, pixels: torch.Tensor) -> torch.Tensor:
        def run(x: torch.Tensor) -> torch.Tensor:
            out = self.module.encode(x.to(self.device, self.dtype))
            dist = getattr(out, "latent_dist", out)
            return dist.mode() if hasattr(dist, "mode") else dist[0]

        if self.tiling.enabled:
            return _tiled(pixels, run, self.tiling, 1.0 / self.temporal_compression, 1.0 / self.spatial_compression)
        return run(pixels).float()

    @torch.no_grad()
    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        def run(z: torch.Tensor) -> torch.Tensor:
            out = self.module.decode(z.to(self.device, self.dtype))
            return getattr(out, "sample", out)

        if self.tiling.enabled:
            return _tiled(latents, run, self.tiling, float(self.temporal_compression), float(self.spatial_compression))
        return run(latents).float()


class TransformersTextEncoder:
    """A ``transformers`` encoder (T5/UMT5/CLIP text) as a :class:`TextEncoder`."""

    def __init__(self, model_id: str, *, max_length: int = 226, dtype: str = "float32", device: str = "cpu",
                 revision: str | None = None, subfolder: str | None = None) -> None:
        self.model_id, self.revision, self.subfolder = model_id, revision, subfolder
        self._max_length = max_length
        self.dtype, self.device = _DTYPES[dtype], torch.device(device)
        self._tok: Any = None
        self._model: Any = None

    @property
    def fingerprint(self) -> str:
        return codec_fingerprint("text", f"transformers:{self.model_id}",
                                 {"max_length": self._max_length, "revision": self.revision})

    @property
    def max_length(self) -> int:
        return self._max_length

    @property
    def tokenizer(self) -> Any:
        if self._tok is None:
            tf = _require("transformers", "codecs")
            kw = {"subfolder": self.subfolder} if self.subfolder else {}
            self._tok = tf.AutoTokenizer.from_pretrained(self.model_id, revision=self.revision, **kw)
        return self._tok

    @property
    def model(self) -> Any:
        if self._model is None:
            tf = _require("transformers", "codecs")
            kw = {"subfolder": self.subfolder} if self.subfolder else {}
            try:
                m = tf.T5EncoderModel.from_pretrained(self.model_id, revision=self.revision, torch_dtype=self.dtype,
                                                      **kw)
            except Exception:  # noqa: BLE001 - not a T5 checkpoint
                m = tf.AutoModel.from_pretrained(self.model_id, revision=self.revision, torch_dtype=self.dtype, **kw)
                m = getattr(m, "text_model", None) or getattr(m, "encoder", None) or m
            self._model = m.to(self.device).eval().requires_grad_(False)
        return self._model

    @property
    def width(self) -> int:
        c = self.model.config
        return int(getattr(c, "d_model", None) or getattr(c, "hidden_size"))

    @torch.no_grad()
    def encode(self, prompts: Sequence[str]) -> tuple[torch.Tensor, torch.Tensor]:
        if isinstance(prompts, str):
            prompts = [prompts]
        tok = self.tokenizer(list(prompts), padding="max_length", truncation=True, max_length=self._max_length,
                             return_tensors="pt")
        ids = tok["input_ids"].to(self.device)
        mask = tok["attention_mask"].to(self.device).bool()
        empty = torch.tensor([len(p) == 0 for p in prompts], device=self.device)
        mask = mask & ~empty[:, None]
        hidden = self.model(input_ids=ids, attention_mask=mask.long()).last_hidden_state.float()
        return hidden * mask[..., None], mask
