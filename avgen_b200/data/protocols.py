"""Data-edge protocols: buckets, bucket plans, sample descriptors, latent samples,
stores, sources and collation (avgen/data/protocols.py:64-758).

A *bucket* is a (frames, height, width[, audio_frames]) latent shape with a
micro-batch size; a *plan* is the ordered set of buckets a run trains on. A
*latent sample* is one encoded clip; collation stacks same-bucket samples into
a :class:`~avgen_b200.core.batch.MediaBatch`.
"""
from __future__ import annotations

from collections.abc import Iterator, Mapping, Sequence
from dataclasses import dataclass, field
from typing import Any, Protocol, runtime_checkable

import torch

from avgen_b200.core._validate import require_dimension, require_name, require_positive
from avgen_b200.core.batch import MediaBatch, MediaBatchSpec

__all__ = ["DATA_SCHEMA_VERSION", "Bucket", "BucketPlan", "DataSource", "LatentSample", "SampleDescriptor",
           "SampleStore", "collate_samples"]

DATA_SCHEMA_VERSION = 1


@dataclass(frozen=True, slots=True)
class Bucket:
    bucket_id: int
    frames: int
    height: int
    width: int
    micro_batch_size: int = 1
    audio_frames: int = 0
    patch_frames: int = 1
    patch_height: int = 2
    patch_width: int = 2
    name: str = ""

    def __post_init__(self) -> None:
        require_dimension("bucket_id", self.bucket_id, allow_zero=True)
        for n in ("frames", "height", "width", "micro_batch_size", "patch_frames", "patch_height", "patch_width"):
            require_positive(n, getattr(self, n))
        require_dimension("audio_frames", self.audio_frames, allow_zero=True)
        for axis, patch in (("frames", "patch_frames"), ("height", "patch_height"), ("width", "patch_width")):
            if getattr(self, axis) % getattr(self, patch):
                raise ValueError(f"bucket {self.bucket_id}: {axis} must be divisible by {patch}")

    @property
    def aspect_ratio(self) -> float:
        return self.width / self.height

    @property
    def latent_cells(self) -> int:
        return self.frames * self.height * self.width

    @property
    def video_tokens(self) -> int:
        return (self.frames // self.patch_frames) * (self.height // self.patch_height) * (
            self.width // self.patch_width)

    @property
    def audio_tokens(self) -> int:
        return self.audio_frames

    @property
    def tokens(self) -> int:
        return self.video_tokens + self.audio_tokens

    @property
    def has_audio(self) -> bool:
        return self.audio_frames > 0

    def duration_seconds(self, *, timebase_num: int, timebase_den: int) -> float:
        return self.frames * timebase_den / timebase_num

    def describe(self) -> str:
        audio = f"+a{self.audio_frames}" if self.audio_frames else ""
        return f"{self.name or self.bucket_id}:{self.frames}x{self.height}x{self.width}{audio} (mb {self.micro_batch_size})"


@dataclass(frozen=True, slots=True)
class BucketPlan:
    buckets: tuple[Bucket, ...]

    def __post_init__(self) -> None:
        if not self.buckets:
            raise ValueError("a bucket plan needs at least one bucket")
        ids = [b.bucket_id for b in self.buckets]
        if len(set(ids)) != len(ids):
            raise ValueError(f"bucket ids must be unique; got {ids}")

    def index_of(self, bucket_id: int) -> int:
        for i, b in enumerate(self.buckets):
            if b.bucket_id == bucket_id:
                return i
        raise KeyError(f"no bucket with id {bucket_id}")

    def get(self, bucket_id: int) -> Bucket:
        return self.buckets[self.index_of(bucket_id)]

    @property
    def token_budget(self) -> int:
        return max(b.tokens * b.micro_batch_size for b in self.buckets)

    def nearest(self, *, frames: int, height: int, width: int) -> Bucket:
        """Bucket minimising log-aspect and log-duration distance to a clip."""
        import math

        def cost(b: Bucket) -> float:
            return abs(math.log(b.aspect_ratio) - math.log(width / height)) + abs(math.log(b.frames / frames))

        return min(self.buckets, key=cost)

    def describe(self) -> str:
        return ", ".join(b.describe() for b in self.buckets)


@dataclass(frozen=True, slots=True)
class SampleDescriptor:
    """Metadata of one stored sample (no tensors)."""

    sample_id: int
    frames: int
    height: int
    width: int
    channels: int
    audio_frames: int = 0
    audio_channels: int = 0
    text_tokens: int = 0
    text_width: int = 0
    video_timebase_num: int = 24
    video_timebase_den: int = 1
    audio_timebase_num: int = 1
    audio_timebase_den: int = 1
    video_codec_id: str = "unknown"
    audio_codec_id: str = "none"
    caption: str = ""

    def __post_init__(self) -> None:
        require_dimension("sample_id", self.sample_id, allow_zero=True)
        for n in ("frames", "height", "width", "channels", "video_timebase_num", "video_timebase_den",
                  "audio_timebase_num", "audio_timebase_den"):
            require_positive(n, getattr(self, n))
        require_name("video_codec_id", self.video_codec_id)

    def codec_key(self) -> tuple[str, str, int, int, int, int]:
        return (self.video_codec_id, self.audio_codec_id, self.video_timebase_num, self.video_timebase_den,
                self.audio_timebase_num, self.audio_timebase_den)


@dataclass(frozen=True, slots=True)
class LatentSample:
    """One encoded clip: video ``(C, T, H, W)``, audio ``(Ca, Ta)``, text ``(N, D)``."""

    descriptor: SampleDescriptor
    video: torch.Tensor
    audio: torch.Tensor = field(default_factory=lambda: torch.zeros(1, 0))
    text: torch.Tensor = field(default_factory=lambda: torch.zeros(0, 1))
    text_mask: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=torch.bool))

    @property
    def sample_id(self) -> int:
        return self.descriptor.sample_id

    def validate(self) -> None:
        d = self.descriptor
        if tuple(self.video.shape) != (d.channels, d.frames, d.height, d.width):
            raise ValueError(f"video shape {tuple(self.video.shape)} does not match its descriptor")
        if self.audio.shape[-1] != d.audio_frames:
            raise ValueError("audio frames do not match the descriptor")
        if self.text.ndim != 2 or self.text_mask.shape[0] != self.text.shape[0]:
            raise ValueError("text must be (tokens, width) with a matching mask")


@runtime_checkable
class SampleStore(Protocol):
    def __len__(self) -> int: ...

    def descriptor(self, index: int) -> SampleDescriptor: ...

    def __getitem__(self, index: int) -> LatentSample: ...


@runtime_checkable
class DataSource(Protocol):
    def __iter__(self) -> Iterator[MediaBatch]: ...

    def state_dict(self) -> Mapping[str, Any]: ...

    def load_state_dict(self, state: Mapping[str, Any]) -> None: ...


def collate_samples(samples: Sequence[LatentSample], *, bucket_id: int = 0, text_tokens: int | None = None,
                    pin: bool = False) -> MediaBatch:
    """Stack same-shape samples into a MediaBatch (text padded / cropped to ``text_tokens``)."""
    if not samples:
        raise ValueError("collate_samples needs at least one sample")
    d0 = samples[0].descriptor
    for s in samples[1:]:
        d = s.descriptor
        if (d.channels, d.frames, d.height, d.width, d.audio_frames) != (d0.channels, d0.frames, d0.height,
                                                                          d0.width, d0.audio_frames):
            raise ValueError("collate_samples requires samples of one bucket shape")
        if d.codec_key() != d0.codec_key():
            raise ValueError("collate_samples requires one codec / timebase")
    n = len(samples)
    t_tokens = text_tokens if text_tokens is not None else max(s.text.shape[0] for s in samples)
    t_width = max((s.text.shape[1] for s in samples if s.text.numel()), default=max(1, d0.text_width))
    text = torch.zeros(n, t_tokens, t_width)
    tmask = torch.zeros(n, t_tokens, dtype=torch.bool)
    for i, s in enumerate(samples):
        k = min(t_tokens, s.text.shape[0])
        if k:
            text[i, :k] = s.text[:k].float()
            tmask[i, :k] = s.text_mask[:k]
    video = torch.stack([s.video.float() for s in samples])
    ac = max(1, d0.audio_channels)
    audio = torch.stack([s.audio.float().reshape(-1, d0.audio_frames) if d0.audio_frames else torch.zeros(ac, 0)
                         for s in samples])
    fps_v = d0.video_timebase_num / d0.video_timebase_den
    fps_a = d0.audio_timebase_num / d0.audio_timebase_den
    vpos = (torch.arange(d0.frames, dtype=torch.float32) / fps_v)[None].expand(n, -1).contiguous()
    apos = (torch.arange(d0.audio_frames, dtype=torch.float32) / fps_a)[None].expand(n, -1).contiguous()
    spec = MediaBatchSpec(schema_version=DATA_SCHEMA_VERSION, bucket_id=bucket_id, video_shape=tuple(video.shape),
                          audio_shape=tuple(audio.shape), text_shape=tuple(text.shape),
                          video_timebase_num=d0.video_timebase_num, video_timebase_den=d0.video_timebase_den,
                          audio_timebase_num=d0.audio_timebase_num, audio_timebase_den=d0.audio_timebase_den,
                          video_codec_id=d0.video_codec_id, audio_codec_id=d0.audio_codec_id or "none")
    batch = MediaBatch(video=video, audio=audio, text=text,
                       video_mask=torch.ones((n, d0.frames, d0.height, d0.width), dtype=torch.bool),
                       audio_mask=torch.ones((n, d0.audio_frames), dtype=torch.bool), video_positions=vpos,
                       audio_positions=apos, sample_ids=torch.tensor([s.sample_id for s in samples]), spec=spec,
                       text_mask=tmask)
    return batch.pin_memory() if pin else batch
