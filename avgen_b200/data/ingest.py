"""Offline ingest: clip probing, a quality gate, fingerprints, clip planning and
latent-sample building (avgen/data/ingest.py:73-972).

Probing a media file needs the optional ``av`` (PyAV) package and clip tables
need ``pyarrow``; both are imported only when used and fail with an install
hint otherwise. Everything else (the gate, fingerprints, clip specs, building a
:class:`~avgen_b200.data.protocols.LatentSample` from encoder outputs) is
dependency-free.
"""
from __future__ import annotations

import hashlib
import importlib
from collections.abc import Iterator, Sequence
from dataclasses import dataclass, field
from enum import Enum
from typing import Any

import torch

from avgen_b200.data.protocols import LatentSample, SampleDescriptor

__all__ = ["ClipProbe", "ClipQA", "ClipReport", "ClipSpec", "IngestSummary", "QualityGate", "RejectionReason",
           "build_latent_sample", "content_fingerprint", "iter_clip_table", "plan_clip_spec", "probe_clip",
           "summarise_reports", "tensor_fingerprint"]


def _require(name: str, extra: str) -> Any:
    try:
        return importlib.import_module(name)
    except ImportError as exc:
        raise RuntimeError(f"{name} is required for this step; install the '{extra}' extra (pip install {name})") from exc


class RejectionReason(str, Enum):
    TOO_SHORT = "too_short"
    TOO_LONG = "too_long"
    LOW_RESOLUTION = "low_resolution"
    BAD_ASPECT = "bad_aspect"
    LOW_FRAME_RATE = "low_frame_rate"
    NO_AUDIO = "no_audio"
    SILENT_AUDIO = "silent_audio"
    DUPLICATE = "duplicate"


@dataclass(frozen=True, slots=True)
class ClipProbe:
    path: str
    width: int
    height: int
    frames: int
    frame_rate_num: int
    frame_rate_den: int
    duration_seconds: float
    has_audio: bool = False
    audio_sample_rate: int = 0
    audio_rms_dbfs: float = float("-inf")
    fingerprint: str = ""

    @property
    def frame_rate(self) -> float:
        return self.frame_rate_num / self.frame_rate_den

    @property
    def aspect_ratio(self) -> float:
        return self.width / self.height

    @property
    def short_side(self) -> int:
        return min(self.width, self.height)


@dataclass(frozen=True, slots=True)
class ClipQA:
    min_seconds: float = 1.0
    max_seconds: float = 60.0
    min_short_side: int = 256
    min_aspect: float = 0.4
    max_aspect: float = 2.5
    min_frame_rate: float = 12.0
    require_audio: bool = False
    min_audio_dbfs: float = -60.0
    deduplicate: bool = True


@dataclass(frozen=True, slots=True)
class ClipReport:
    probe: ClipProbe
    admitted: bool
    reasons: tuple[RejectionReason, ...] = ()


class QualityGate:
    """Admits or rejects probed clips, with de-duplication by content fingerprint."""

    def __init__(self, config: ClipQA | None = None) -> None:
        self._config = config or ClipQA()
        self._seen: set[str] = set()
        self._admitted = 0

    @property
    def config(self) -> ClipQA:
        return self._config

    @property
    def admitted(self) -> int:
        return self._admitted

    def reset(self) -> None:
        self._seen.clear()
        self._admitted = 0

    def evaluate(self, probe: ClipProbe) -> ClipReport:
        c = self._config
        r: list[RejectionReason] = []
        if probe.duration_seconds < c.min_seconds:
            r.append(RejectionReason.TOO_SHORT)
        if probe.duration_seconds > c.max_seconds:
            r.append(RejectionReason.TOO_LONG)
        if probe.short_side < c.min_short_side:
            r.append(RejectionReason.LOW_RESOLUTION)
        if not c.min_aspect <= probe.aspect_ratio <= c.max_aspect:
            r.append(RejectionReason.BAD_ASPECT)
        if probe.frame_rate < c.min_frame_rate:
            r.append(RejectionReason.LOW_FRAME_RATE)
        if c.require_audio and not probe.has_audio:
            r.append(RejectionReason.NO_AUDIO)
        if probe.has_audio and probe.audio_rms_dbfs < c.min_audio_dbfs:
            r.append(RejectionReason.SILENT_AUDIO)
        if c.deduplicate and probe.fingerprint:
            if probe.fingerprint in self._seen:
                r.append(RejectionReason.DUPLICATE)
        ok = not r
        if ok:
            self._admitted += 1
            if probe.fingerprint:
                self._seen.add(probe.fingerprint)
        return ClipReport(probe=probe, admitted=ok, reasons=tuple(r))


def content_fingerprint(payload: bytes | Sequence[bytes]) -> str:
    h = hashlib.sha256()
    for chunk in ([payload] if isinstance(payload, (bytes, bytearray)) else payload):
        h.update(chunk)
    return h.hexdigest()


def tensor_fingerprint(tensor: torch.Tensor) -> str:
    t = tensor.detach().contiguous().cpu()
    h = hashlib.sha256(str((tuple(t.shape), str(t.dtype))).encode())
    h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return h.hexdigest()


@dataclass(frozen=True, slots=True)
class ClipSpec:
    start_frame: int
    frames: int
    frame_rate_num: int
    frame_rate_den: int
    height: int
    width: int

    @property
    def frame_rate(self) -> float:
        return self.frame_rate_num / self.frame_rate_den

    @property
    def duration_seconds(self) -> float:
        return self.frames / self.frame_rate


def plan_clip_spec(probe: ClipProbe, *, frames: int, height: int, width: int, temporal_multiple: int = 4,
                   spatial_multiple: int = 16, stride: int = 1) -> ClipSpec:
    """A centred window of ``frames`` frames at a size divisible by the codec's strides."""
    usable = (probe.frames - 1) // stride + 1
    n = min(frames, usable)
    n = max(1, (n - 1) // temporal_multiple * temporal_multiple + 1)
    start = max(0, (probe.frames - (n - 1) * stride - 1) // 2)
    h = max(spatial_multiple, height // spatial_multiple * spatial_multiple)
    w = max(spatial_multiple, width // spatial_multiple * spatial_multiple)
    return ClipSpec(start, n, probe.frame_rate_num, probe.frame_rate_den * stride, h, w)


def build_latent_sample(sample_id: int, *, video_latent: torch.Tensor, text: torch.Tensor,
                        text_mask: torch.Tensor | None = None, audio_latent: torch.Tensor | None = None,
                        video_timebase: tuple[int, int] = (24, 1), audio_timebase: tuple[int, int] = (1, 1),
                        video_codec_id: str = "video", audio_codec_id: str = "none",
                        caption: str = "") -> LatentSample:
    """Wrap encoder outputs ``(C, T, H, W)`` / ``(Ca, Ta)`` / ``(N, D)`` as a stored sample."""
    c, t, h, w = video_latent.shape
    audio = audio_latent if audio_latent is not None else torch.zeros(1, 0)
    tm = text_mask if text_mask is not None else torch.ones(text.shape[0], dtype=torch.bool)
    desc = SampleDescriptor(sample_id=sample_id, frames=t, height=h, width=w, channels=c,
                            audio_frames=audio.shape[-1], audio_channels=audio.shape[0] if audio.shape[-1] else 0,
                            text_tokens=text.shape[0], text_width=text.shape[1],
                            video_timebase_num=video_timebase[0], video_timebase_den=video_timebase[1],
                            audio_timebase_num=audio_timebase[0], audio_timebase_den=audio_timebase[1],
                            video_codec_id=video_codec_id, audio_codec_id=audio_codec_id, caption=caption)
    sample = LatentSample(descriptor=desc, video=video_latent.detach().cpu(), audio=audio.detach().cpu(),
                          text=text.detach().cpu(), text_mask=tm.cpu())
    sample.validate()
    return sample


def probe_clip(path: str) -> ClipProbe:
    """Probe a media file with PyAV (optional dependency)."""
    av = _require("av", "data")
    with av.open(path) as container:
        vs = container.streams.video[0]
        rate = vs.average_rate or vs.base_rate
        frames = vs.frames or int(float(vs.duration * vs.time_base * rate)) if vs.duration else vs.frames
        duration = float(container.duration / 1e6) if container.duration else frames / float(rate)
        has_audio = bool(container.streams.audio)
        sr = container.streams.audio[0].rate if has_audio else 0
    with open(path, "rb") as fh:
        fp = content_fingerprint(fh.read(1 << 20))
    return ClipProbe(path=path, width=vs.width, height=vs.height, frames=int(frames or 0),
                     frame_rate_num=rate.numerator, frame_rate_den=rate.denominator, duration_seconds=duration,
                     has_audio=has_audio, audio_sample_rate=sr, fingerprint=fp)


def iter_clip_table(path: str, *, columns: Sequence[str] = ("path", "caption")) -> Iterator[dict[str, Any]]:
    """Rows of a parquet clip table (optional ``pyarrow`` dependency)."""
    pq = _require("pyarrow.parquet", "data")
    table = pq.read_table(path, columns=list(columns))
    yield from table.to_pylist()


@dataclass(frozen=True, slots=True)
class IngestSummary:
    total: int
    admitted: int
    rejections: dict[str, int] = field(default_factory=dict)

    @property
    def acceptance_rate(self) -> float:
        return self.admitted / self.total if self.total else 0.0

    def describe(self) -> str:
        parts = ", ".join(f"{k}={v}" for k, v in sorted(self.rejections.items()))
        return f"{self.admitted}/{self.total} admitted ({self.acceptance_rate:.1%}); rejected: {parts or 'none'}"


def summarise_reports(reports: Sequence[ClipReport]) -> IngestSummary:
    rej: dict[str, int] = {}
    for r in reports:
        for reason in r.reasons:
            rej[reason.value] = rej.get(reason.value, 0) + 1
    return IngestSummary(total=len(reports), admitted=sum(r.admitted for r in reports), rejections=rej)
