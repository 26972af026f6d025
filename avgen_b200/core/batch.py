"""Dense data-edge batch contract (MediaBatch) and conditioning modes.

Dense grids live at the data / codec boundary only: video ``(B, C, T, H, W)``,
audio ``(B, C, T)``, text ``(B, N, D)``, masks, physical frame positions in
seconds, CPU-resident ``sample_ids`` and exact rational timebases. Same contract
as avgen/core/batch.py:59-476.
"""
from __future__ import annotations

from collections.abc import Sequence
from dataclasses import asdict, dataclass, field, replace
from enum import IntEnum

import torch
from torch.utils import _pytree

from avgen_b200.core._validate import (require_dimension, require_dtype, require_floating, require_name,
                                       require_same_device, require_shape)
from avgen_b200.core.tensors import TensorBundle, TensorBundleSpec

__all__ = ["ConditionMode", "MediaBatch", "MediaBatchSpec", "null_text_conditioning", "stack_batches"]


class ConditionMode(IntEnum):
    """Per-sample conditioning task (values are part of the data format)."""

    JOINT = 0
    VIDEO_TO_AUDIO = 1
    AUDIO_TO_VIDEO = 2
    VIDEO_ONLY = 3
    CONTINUATION = 4
    INPAINT = 5
    IMAGE_TO_VIDEO = 6
    VIDEO_TO_VIDEO = 7


@dataclass(frozen=True, slots=True)
class MediaBatchSpec:
    """Static description of a batch: shapes, timebases, codec ids, targets."""

    schema_version: int
    bucket_id: int
    video_shape: tuple[int, ...]
    audio_shape: tuple[int, ...]
    text_shape: tuple[int, ...]
    video_timebase_num: int
    video_timebase_den: int
    audio_timebase_num: int
    audio_timebase_den: int
    video_codec_id: str
    audio_codec_id: str
    target_spec: TensorBundleSpec = field(default_factory=TensorBundleSpec)

    def __post_init__(self) -> None:
        require_dimension("schema_version", self.schema_version)
        require_dimension("bucket_id", self.bucket_id, allow_zero=True)
        self._check("video_shape", self.video_shape, 5, None)
        self._check("audio_shape", self.audio_shape, 3, 2)
        self._check("text_shape", self.text_shape, 3, 1)
        if len({self.video_shape[0], self.audio_shape[0], self.text_shape[0]}) != 1:
            raise ValueError("video, audio, and text batch dimensions must match")
        for name in ("video_timebase_num", "video_timebase_den", "audio_timebase_num", "audio_timebase_den"):
            require_dimension(name, getattr(self, name))
        require_name("video_codec_id", self.video_codec_id)
        require_name("audio_codec_id", self.audio_codec_id)

    @staticmethod
    def _check(name: str, shape: tuple[int, ...], rank: int, zero_ok: int | None) -> None:
        if len(shape) != rank:
            raise ValueError(f"{name} must have rank {rank}; got {shape}")
        for i, v in enumerate(shape):
            require_dimension(f"{name}[{i}]", v, allow_zero=i == zero_ok)

    @property
    def batch_size(self) -> int:
        return self.video_shape[0]

    @property
    def video_fps(self) -> float:
        return self.video_timebase_num / self.video_timebase_den

    @property
    def audio_fps(self) -> float:
        return self.audio_timebase_num / self.audio_timebase_den

    @property
    def has_audio(self) -> bool:
        return self.audio_shape[2] > 0

    @property
    def has_text(self) -> bool:
        return self.text_shape[1] > 0

    @property
    def video_tokens(self) -> int:
        _, _, t, h, w = self.video_shape
        return t * h * w

    @property
    def audio_tokens(self) -> int:
        return self.audio_shape[2]

    @property
    def sequence_length(self) -> int:
        return self.video_tokens + self.audio_tokens

    def to_dict(self) -> dict[str, object]:
        values = asdict(self)
        for key in ("video_shape", "audio_shape", "text_shape"):
            values[key] = list(values[key])
        values["target_spec"] = self.target_spec.to_dict()
        return values

    @classmethod
    def from_dict(cls, values: dict) -> MediaBatchSpec:
        v = dict(values)
        for key in ("video_shape", "audio_shape", "text_shape"):
            v[key] = tuple(v[key])
        v["target_spec"] = TensorBundleSpec.from_dict(v["target_spec"]) if "target_spec" in v else TensorBundleSpec()
        return cls(**v)


def _empty_bool() -> torch.Tensor:
    return torch.empty(0, dtype=torch.bool)


@dataclass(frozen=True, slots=True)
class MediaBatch:
    """A dense batch at the data edge."""

    video: torch.Tensor
    audio: torch.Tensor
    text: torch.Tensor
    video_mask: torch.Tensor
    audio_mask: torch.Tensor
    video_positions: torch.Tensor
    audio_positions: torch.Tensor
    sample_ids: torch.Tensor
    spec: MediaBatchSpec
    text_mask: torch.Tensor = field(default_factory=_empty_bool)
    targets: TensorBundle = field(default_factory=TensorBundle)

    def __post_init__(self) -> None:
        if self.text_mask.numel() == 0:
            object.__setattr__(self, "text_mask",
                               torch.ones(self.spec.text_shape[:2], dtype=torch.bool, device=self.text.device))

    @property
    def device(self) -> torch.device:
        return self.video.device

    def to(self, device: torch.device | str, *, non_blocking: bool = True) -> MediaBatch:
        """Move every tensor but ``sample_ids`` (pinned sources copy asynchronously)."""
        dev = torch.device(device)

        def mv(t: torch.Tensor) -> torch.Tensor:
            return t.to(dev, non_blocking=non_blocking)

        return MediaBatch(video=mv(self.video), audio=mv(self.audio), text=mv(self.text),
                          video_mask=mv(self.video_mask), audio_mask=mv(self.audio_mask),
                          video_positions=mv(self.video_positions), audio_positions=mv(self.audio_positions),
                          sample_ids=self.sample_ids, spec=self.spec, text_mask=mv(self.text_mask),
                          targets=TensorBundle(tuple(mv(v) for v in self.targets.values)))

    def pin_memory(self) -> MediaBatch:
        """Page-locked copy of every host tensor (for async H2D copies)."""
        def pin(t: torch.Tensor) -> torch.Tensor:
            return t.pin_memory() if t.device.type == "cpu" and torch.cuda.is_available() else t

        return MediaBatch(video=pin(self.video), audio=pin(self.audio), text=pin(self.text),
                          video_mask=pin(self.video_mask), audio_mask=pin(self.audio_mask),
                          video_positions=pin(self.video_positions), audio_positions=pin(self.audio_positions),
                          sample_ids=self.sample_ids, spec=self.spec, text_mask=pin(self.text_mask),
                          targets=TensorBundle(tuple(pin(v) for v in self.targets.values)))

    def nbytes(self) -> int:
        """Bytes of the tensors that :meth:`to` copies."""
        tensors = [self.video, self.audio, self.text, self.video_mask, self.audio_mask, self.video_positions,
                   self.audio_positions, self.text_mask, *self.targets.values]
        return int(sum(t.numel() * t.element_size() for t in tensors))

    def validate(self) -> None:
        batch, _, vt, h, w = self.spec.video_shape
        at = self.spec.audio_shape[2]
        require_shape("video", self.video, self.spec.video_shape)
        require_shape("audio", self.audio, self.spec.audio_shape)
        require_shape("text", self.text, self.spec.text_shape)
        require_shape("video_mask", self.video_mask, (batch, vt, h, w))
        require_shape("audio_mask", self.audio_mask, (batch, at))
        require_shape("text_mask", self.text_mask, (batch, self.spec.text_shape[1]))
        require_shape("video_positions", self.video_positions, (batch, vt))
        require_shape("audio_positions", self.audio_positions, (batch, at))
        require_shape("sample_ids", self.sample_ids, (batch,))
        for name in ("video", "audio", "text"):
            require_floating(name, getattr(self, name))
        for name in ("video_mask", "audio_mask", "text_mask"):
            require_dtype(name, getattr(self, name), torch.bool)
        for name in ("video_positions", "audio_positions"):
            require_dtype(name, getattr(self, name), torch.float32)
        require_dtype("sample_ids", self.sample_ids, torch.int64)
        if self.sample_ids.device.type != "cpu":
            raise ValueError("sample_ids must remain on CPU")
        require_same_device("video", self.video, ((n, getattr(self, n)) for n in (
            "audio", "text", "video_mask", "audio_mask", "text_mask", "video_positions", "audio_positions")))
        self.targets.validate(self.spec.target_spec, device=self.video.device)


def stack_batches(batches: Sequence[MediaBatch]) -> MediaBatch:
    """Concatenate batches with identical specs along the batch axis."""
    if not batches:
        raise ValueError("stack_batches requires at least one batch")
    if len(batches) == 1:
        return batches[0]
    base = batches[0].spec
    if any(b.spec != base for b in batches[1:]):
        raise ValueError("stack_batches requires an identical MediaBatchSpec")
    widths = {len(b.targets) for b in batches}
    if len(widths) != 1:
        raise ValueError("stack_batches requires matching target bundles")
    total = sum(b.spec.batch_size for b in batches)
    spec = replace(base, video_shape=(total, *base.video_shape[1:]), audio_shape=(total, *base.audio_shape[1:]),
                   text_shape=(total, *base.text_shape[1:]), target_spec=base.target_spec.with_batch_size(total))

    def cat(name: str) -> torch.Tensor:
        return torch.cat([getattr(b, name) for b in batches], 0)

    targets = TensorBundle(tuple(torch.cat([b.targets.values[i] for b in batches], 0) for i in range(widths.pop())))
    return MediaBatch(video=cat("video"), audio=cat("audio"), text=cat("text"), video_mask=cat("video_mask"),
                      audio_mask=cat("audio_mask"), text_mask=cat("text_mask"),
                      video_positions=cat("video_positions"), audio_positions=cat("audio_positions"),
                      sample_ids=cat("sample_ids"), targets=targets, spec=spec)


def null_text_conditioning(text: torch.Tensor, text_mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The exact null text the model is trained on for CFG dropout."""
    return torch.zeros_like(text), torch.zeros_like(text_mask)


def _flatten_batch(b: MediaBatch) -> tuple[list[torch.Tensor], MediaBatchSpec]:
    return ([b.video, b.audio, b.text, b.video_mask, b.audio_mask, b.text_mask, b.video_positions,
             b.audio_positions, b.sample_ids, *b.targets.values], b.spec)


def _unflatten_batch(values, spec) -> MediaBatch:
    t = list(values)
    return MediaBatch(video=t[0], audio=t[1], text=t[2], video_mask=t[3], audio_mask=t[4], text_mask=t[5],
                      video_positions=t[6], audio_positions=t[7], sample_ids=t[8], targets=TensorBundle(tuple(t[9:])),
                      spec=spec)


_pytree.register_pytree_node(MediaBatch, _flatten_batch, _unflatten_batch, serialized_type_name="avgen_b200.MediaBatch",
                             to_dumpable_context=MediaBatchSpec.to_dict, from_dumpable_context=MediaBatchSpec.from_dict)
