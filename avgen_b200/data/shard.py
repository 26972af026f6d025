"""Latent shards: a directory of ``data.safetensors`` + ``manifest.json`` + ``COMMIT``.

The 3-file layout is the on-disk format shared with avgen
(avgen/data/shard.py:1-1036): tensors for every sample live in one safetensors
file under keys ``<sample_id>/video``, ``/audio``, ``/text``, ``/text_mask``; the
manifest lists records (descriptor, caption, sha256 of each tensor's bytes) and
the codec / timebase; ``COMMIT`` is written last, after an fsync of everything
else, so a partially written shard is never read. Readers memory-map the
safetensors file; :class:`ConcatShardReader` indexes many shards as one store.
"""
from __future__ import annotations

import bisect
import hashlib
import json
import os
from collections.abc import Iterable, Mapping, Sequence
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

import torch

from avgen_b200.data.protocols import DATA_SCHEMA_VERSION, LatentSample, SampleDescriptor

__all__ = ["COMMIT_NAME", "DATA_NAME", "MANIFEST_NAME", "ConcatShardReader", "ShardCorruptionError", "ShardManifest",
           "ShardReader", "ShardRecord", "validate_shard", "write_shard"]

DATA_NAME = "data.safetensors"
MANIFEST_NAME = "manifest.json"
COMMIT_NAME = "COMMIT"
_FIELDS = ("video", "audio", "text", "text_mask")


class ShardCorruptionError(RuntimeError):
    """A shard is incomplete, inconsistent, or its bytes fail their checksum."""


@dataclass(frozen=True, slots=True)
class ShardRecord:
    descriptor: SampleDescriptor
    checksums: dict[str, str] = field(default_factory=dict)

    def to_dict(self) -> dict[str, Any]:
        return {"descriptor": asdict(self.descriptor), "checksums": dict(self.checksums)}

    @classmethod
    def from_dict(cls, values: Mapping[str, Any]) -> ShardRecord:
        return cls(descriptor=SampleDescriptor(**values["descriptor"]), checksums=dict(values.get("checksums", {})))


@dataclass(frozen=True, slots=True)
class ShardManifest:
    schema_version: int
    records: tuple[ShardRecord, ...]
    video_codec_id: str
    audio_codec_id: str
    video_timebase: tuple[int, int]
    audio_timebase: tuple[int, int]
    extra: dict[str, Any] = field(default_factory=dict)

    def __len__(self) -> int:
        return len(self.records)

    def codec_key(self) -> tuple[str, str, int, int, int, int]:
        return (self.video_codec_id, self.audio_codec_id, *self.video_timebase, *self.audio_timebase)

    def to_dict(self) -> dict[str, Any]:
        return {"schema_version": self.schema_version, "records": [r.to_dict() for r in self.records],
                "video_codec_id": self.video_codec_id, "audio_codec_id": self.audio_codec_id,
                "video_timebase": list(self.video_timebase), "audio_timebase": list(self.audio_timebase),
                "extra": self.extra}

    @classmethod
    def from_dict(cls, values: Mapping[str, Any]) -> ShardManifest:
        return cls(schema_version=int(values["schema_version"]),
                   records=tuple(ShardRecord.from_dict(r) for r in values["records"]),
                   video_codec_id=values["video_codec_id"], audio_codec_id=values["audio_codec_id"],
                   video_timebase=tuple(values["video_timebase"]), audio_timebase=tuple(values["audio_timebase"]),
                   extra=dict(values.get("extra", {})))


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().numpy().tobytes()).hexdigest()


def _fsync_dir(path: Path) -> None:
    try:
        fd = os.open(path, os.O_RDONLY)
    except OSError:
        return
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def write_shard(path: str | Path, samples: Iterable[LatentSample], *, extra: Mapping[str, Any] | None = None,
                overwrite: bool = False) -> ShardManifest:
    """Write samples atomically (data, manifest, fsync, then ``COMMIT``)."""
    from safetensors.torch import save_file

    root = Path(path)
    if (root / COMMIT_NAME).exists() and not overwrite:
        raise FileExistsError(f"shard {root} already committed")
    root.mkdir(parents=True, exist_ok=True)
    (root / COMMIT_NAME).unlink(missing_ok=True)
    items = list(samples)
    if not items:
        raise ValueError("a shard needs at least one sample")
    key = items[0].descriptor.codec_key()
    tensors: dict[str, torch.Tensor] = {}
    records = []
    seen: set[int] = set()
    for s in items:
        s.validate()
        if s.descriptor.codec_key() != key:
            raise ValueError("all samples of a shard must share codec ids and timebases")
        if s.sample_id in seen:
            raise ValueError(f"duplicate sample id {s.sample_id}")
        seen.add(s.sample_id)
        sums = {}
        for name in _FIELDS:
            t = getattr(s, name).contiguous().cpu()
            tensors[f"{s.sample_id}/{name}"] = t
            sums[name] = _sha(t)
        records.append(ShardRecord(descriptor=s.descriptor, checksums=sums))
    d0 = items[0].descriptor
    manifest = ShardManifest(schema_version=DATA_SCHEMA_VERSION, records=tuple(records),
                             video_codec_id=d0.video_codec_id, audio_codec_id=d0.audio_codec_id,
                             video_timebase=(d0.video_timebase_num, d0.video_timebase_den),
                             audio_timebase=(d0.audio_timebase_num, d0.audio_timebase_den), extra=dict(extra or {}))
    tmp = root / (DATA_NAME + ".tmp")
    save_file(tensors, str(tmp))
    with open(tmp, "rb") as fh:
        os.fsync(fh.fileno())
    tmp.replace(root / DATA_NAME)
    mtmp = root / (MANIFEST_NAME + ".tmp")
    with open(mtmp, "w", encoding="utf-8") as fh:
        json.dump(manifest.to_dict(), fh)
        fh.flush()
        os.fsync(fh.fileno())
    mtmp.replace(root / MANIFEST_NAME)
    _fsync_dir(root)
    with open(root / COMMIT_NAME, "w", encoding="utf-8") as fh:
        fh.write(f"{len(records)}\n")
        fh.flush()
        os.fsync(fh.fileno())
    _fsync_dir(root)
    return manifest


def _read_manifest(root: Path) -> ShardManifest:
    if not (root / COMMIT_NAME).exists():
        raise ShardCorruptionError(f"shard {root} has no {COMMIT_NAME}: it was never completely written")
    try:
        return ShardManifest.from_dict(json.loads((root / MANIFEST_NAME).read_text(encoding="utf-8")))
    except (OSError, ValueError, KeyError) as exc:
        raise ShardCorruptionError(f"shard {root}: unreadable manifest ({exc})") from exc


def validate_shard(path: str | Path, *, check_data: bool = True) -> ShardManifest:
    """Check COMMIT, manifest, tensor presence / shapes and (optionally) checksums."""
    root = Path(path)
    manifest = _read_manifest(root)
    if manifest.schema_version > DATA_SCHEMA_VERSION:
        raise ShardCorruptionError(f"shard {root} has a newer schema version")
    reader = ShardReader(root)
    try:
        for i in range(len(reader)):
            s = reader[i]
            try:
                s.validate()
            except ValueError as exc:
                raise ShardCorruptionError(f"shard {root}: sample {s.sample_id}: {exc}") from exc
            if check_data:
                rec = manifest.records[i]
                for name in _FIELDS:
                    if rec.checksums.get(name) and _sha(getattr(s, name)) != rec.checksums[name]:
                        raise ShardCorruptionError(f"shard {root}: sample {s.sample_id} {name} fails its checksum")
    finally:
        reader.close()
    return manifest


class ShardReader:
    """Memory-mapped random access to one committed shard."""

    def __init__(self, path: str | Path) -> None:
        from safetensors import safe_open

        self._path = Path(path)
        self._manifest = _read_manifest(self._path)
        try:
            self._file = safe_open(str(self._path / DATA_NAME), framework="pt", device="cpu")
        except Exception as exc:  # noqa: BLE001
            raise ShardCorruptionError(f"shard {self._path}: cannot open {DATA_NAME} ({exc})") from exc
        keys = set(self._file.keys())
        for rec in self._manifest.records:
            for name in _FIELDS:
                if f"{rec.descriptor.sample_id}/{name}" not in keys:
                    raise ShardCorruptionError(f"shard {self._path}: missing tensor for sample "
                                               f"{rec.descriptor.sample_id} field {name}")

    @property
    def path(self) -> Path:
        return self._path

    @property
    def manifest(self) -> ShardManifest:
        return self._manifest

    def __len__(self) -> int:
        return len(self._manifest.records)

    def close(self) -> None:
        self._file = None

    def descriptor(self, index: int) -> SampleDescriptor:
        return self._manifest.records[index].descriptor

    def record(self, index: int) -> ShardRecord:
        return self._manifest.records[index]

    def __getitem__(self, index: int) -> LatentSample:
        if self._file is None:
            raise RuntimeError("reader is closed")
        d = self.descriptor(index)
        get = self._file.get_tensor
        return LatentSample(descriptor=d, video=get(f"{d.sample_id}/video"), audio=get(f"{d.sample_id}/audio"),
                            text=get(f"{d.sample_id}/text"), text_mask=get(f"{d.sample_id}/text_mask"))


class ConcatShardReader:
    """Many shards indexed as one store (all must share a codec key)."""

    def __init__(self, readers: Sequence[ShardReader]) -> None:
        if not readers:
            raise ValueError("ConcatShardReader needs at least one shard")
        key = readers[0].manifest.codec_key()
        if any(r.manifest.codec_key() != key for r in readers[1:]):
            raise ValueError("shards disagree on codec ids / timebases")
        self._readers = tuple(readers)
        self._starts = [0]
        for r in readers:
            self._starts.append(self._starts[-1] + len(r))

    @classmethod
    def from_paths(cls, paths: Iterable[str | Path]) -> ConcatShardReader:
        return cls([ShardReader(p) for p in sorted(Path(p) for p in paths)])

    @classmethod
    def from_root(cls, root: str | Path) -> ConcatShardReader:
        dirs = [p for p in Path(root).iterdir() if p.is_dir() and (p / COMMIT_NAME).exists()]
        return cls.from_paths(dirs)

    @property
    def readers(self) -> tuple[ShardReader, ...]:
        return self._readers

    def __len__(self) -> int:
        return self._starts[-1]

    def close(self) -> None:
        for r in self._readers:
            r.close()

    def locate(self, index: int) -> tuple[int, int]:
        if not 0 <= index < len(self):
            raise IndexError(index)
        shard = bisect.bisect_right(self._starts, index) - 1
        return shard, index - self._starts[shard]

    def descriptor(self, index: int) -> SampleDescriptor:
        s, i = self.locate(index)
        return self._readers[s].descriptor(i)

    def __getitem__(self, index: int) -> LatentSample:
        s, i = self.locate(index)
        return self._readers[s][i]
