"""Checkpoint manager: DCP save / load with async upload, completion markers,
retention and resharding resume (avgen/checkpoint/manager.py:186-945).

Layout (the format): ``<root>/step_<10 digits>/`` holds one DCP file per rank
(``single_file_per_rank``) plus ``avgen_checkpoint.json``, written atomically
(tmp + rename) only after the upload finished, followed by a barrier. A
directory without the marker is invisible to resume and swept by retention.
The marker records format_version 1, step, progress, keys, world_size,
data_world and the parallel layout. Load reshards to any rank count; per-rank
RNG state is skipped (with a warning) when the data-parallel width changed.
"""
from __future__ import annotations

import json
import logging
import os
import shutil
import time
from concurrent.futures import Future
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch import nn
from torch.distributed.checkpoint.api import CheckpointException

from avgen_b200.checkpoint.stateful import (EMA_KEY, EXTRAS_KEY, MODEL_OPTIMIZER_KEY, PROGRESS_KEY, RNG_KEY,
                                            SCHEDULE_KEY, build_stateful)
from avgen_b200.core.state import TrainState
from avgen_b200.parallel.env import collective_timeout

__all__ = ["CHECKPOINT_DIR_PREFIX", "CHECKPOINT_FORMAT_VERSION", "MARKER_FILENAME", "CheckpointEntry",
           "CheckpointManager", "load", "load_ema", "load_model", "save"]

_LOG = logging.getLogger("avgen_b200.checkpoint")
CHECKPOINT_DIR_PREFIX = "step_"
MARKER_FILENAME = "avgen_checkpoint.json"
CHECKPOINT_FORMAT_VERSION = 1


@dataclass(frozen=True, slots=True)
class CheckpointEntry:
    step: int
    path: Path
    metadata: dict[str, Any]

    @property
    def data_world(self) -> int:
        return int(self.metadata.get("data_world", 1))

    @property
    def world_size(self) -> int:
        return int(self.metadata.get("world_size", 1))


def step_dirname(step: int) -> str:
    return f"{CHECKPOINT_DIR_PREFIX}{step:010d}"


def _parse_step(name: str) -> int | None:
    if not name.startswith(CHECKPOINT_DIR_PREFIX):
        return None
    tail = name[len(CHECKPOINT_DIR_PREFIX):]
    return int(tail) if tail.isdigit() else None


def _world() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _main() -> bool:
    return not (dist.is_available() and dist.is_initialized()) or dist.get_rank() == 0


def _barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def _data_coords(parallel: Any) -> tuple[int, int]:
    if parallel is None or getattr(parallel, "mesh", None) is None:
        return 0, 1
    return parallel.dims.data_coordinates(parallel.mesh)


class CheckpointManager:
    def __init__(self, root: str | os.PathLike[str], *, keep_last_n: int = 3, keep_every_n_steps: int = 0,
                 save_timeout_s: float = 600.0, strict: bool = True, include_rng: bool = True,
                 cpu_offload: bool = False, thread_count: int = 1) -> None:
        if keep_last_n < 0 or keep_every_n_steps < 0:
            raise ValueError("retention counts must be non-negative")
        if save_timeout_s <= 0 or thread_count < 1:
            raise ValueError("save_timeout_s must be positive and thread_count >= 1")
        self._root = Path(root)
        self._keep_last_n = keep_last_n
        self._keep_every = keep_every_n_steps
        self._timeout = save_timeout_s
        self._strict = strict
        self._include_rng = include_rng
        self._cpu_offload = cpu_offload
        self._threads = thread_count
        self._pending: Future | None = None
        self._pending_step: int | None = None
        self._pending_marker: dict[str, Any] | None = None

    @property
    def root(self) -> Path:
        return self._root

    @property
    def has_pending_save(self) -> bool:
        return self._pending is not None

    def save(self, step: int, state: TrainState, *, parallel: Any = None, async_save: bool = True,
             extras: dict[str, Any] | None = None) -> Path:
        if isinstance(step, bool) or step < 0:
            raise ValueError(f"step must be a non-negative integer; got {step!r}")
        self.wait()
        data_rank, data_world = _data_coords(parallel)
        directory = self._root / step_dirname(step)
        if _main():
            directory.mkdir(parents=True, exist_ok=True)
        _barrier()
        entries = build_stateful(state, data_rank=data_rank, include_rng=self._include_rng, strict=self._strict,
                                 cpu_offload=self._cpu_offload)
        marker = self._marker(step, state, entries, data_world, parallel, extras)
        writer = dcp.FileSystemWriter(directory, thread_count=self._threads, single_file_per_rank=True,
                                      overwrite=True)
        t0 = time.monotonic()
        if async_save:
            with collective_timeout(self._timeout):
                result = dcp.async_save(entries, storage_writer=writer)
            self._pending = getattr(result, "upload_completion", result)
            self._pending_step = step
            self._pending_marker = marker
            _LOG.info("checkpoint step=%d staged in %.2fs -> %s", step, time.monotonic() - t0, directory)
        else:
            with collective_timeout(self._timeout):
                dcp.save(entries, storage_writer=writer)
            self._finalize(step, directory, marker)
            _LOG.info("checkpoint step=%d written in %.2fs -> %s", step, time.monotonic() - t0, directory)
        return directory

    def wait(self) -> None:
        fut = self._pending
        if fut is None:
            return
        step, marker = self._pending_step, self._pending_marker
        self._pending = self._pending_step = self._pending_marker = None
        try:
            fut.result(timeout=self._timeout)
        except TimeoutError as exc:
            raise TimeoutError(f"checkpoint upload for step {step} exceeded {self._timeout}s; left unmarked") from exc
        if step is not None and marker is not None:
            self._finalize(step, self._root / step_dirname(step), marker)

    def _finalize(self, step: int, directory: Path, marker: dict[str, Any]) -> None:
        if _main():
            payload = dict(marker, completed_at=time.time())
            tmp = directory / f".{MARKER_FILENAME}.tmp"
            tmp.write_text(json.dumps(payload, indent=2, sort_keys=True))
            tmp.replace(directory / MARKER_FILENAME)
            self._prune(keep_step=step)
        _barrier()

    def _marker(self, step: int, state: TrainState, entries: dict[str, Any], data_world: int, parallel: Any,
                extras: dict[str, Any] | None) -> dict[str, Any]:
        m: dict[str, Any] = {"format_version": CHECKPOINT_FORMAT_VERSION, "step": step,
                             "progress": dict(state.progress()), "keys": sorted(entries), "world_size": _world(),
                             "data_world": data_world, "torch_version": torch.__version__}
        if parallel is not None and getattr(parallel, "dims", None) is not None:
            d = parallel.dims
            m["parallel"] = {"describe": d.describe(), "dp_replicate": d.dp_replicate, "dp_shard": d.dp_shard,
                             "context": d.context, "tensor": d.tensor, "pipeline": d.pipeline,
                             "applied": list(getattr(parallel, "applied", ()))}
        if extras:
            m["extras"] = dict(extras)
        return m

    def _scan(self, path: str | os.PathLike[str] | None = None) -> list[tuple[int, Path]]:
        root = Path(path) if path is not None else self._root
        if not root.is_dir():
            return []
        found = [(s, c) for c in root.iterdir() if c.is_dir() and (s := _parse_step(c.name)) is not None]
        return sorted(found, key=lambda x: x[0])

    def list_checkpoints(self, path: str | os.PathLike[str] | None = None) -> tuple[CheckpointEntry, ...]:
        out = []
        for step, d in self._scan(path):
            marker = d / MARKER_FILENAME
            if not marker.is_file():
                continue
            try:
                meta = json.loads(marker.read_text())
            except (OSError, json.JSONDecodeError):
                _LOG.warning("unreadable checkpoint marker at %s; skipping", marker)
                continue
            if isinstance(meta, dict):
                out.append(CheckpointEntry(step, d, meta))
        return tuple(out)

    def latest_step(self, path: str | os.PathLike[str] | None = None) -> int | None:
        entries = self.list_checkpoints(path)
        return entries[-1].step if entries else None

    def _prune(self, *, keep_step: int) -> None:
        entries = self.list_checkpoints()
        if not entries:
            return
        keep = {keep_step, entries[-1].step}
        keep.update(e.step for e in (entries[-self._keep_last_n:] if self._keep_last_n > 0 else entries))
        if self._keep_every > 0:
            keep.update(e.step for e in entries if e.step % self._keep_every == 0)
        for e in entries:
            if e.step not in keep:
                shutil.rmtree(e.path, ignore_errors=True)
        newest = entries[-1].step
        for step, d in self._scan():
            if step < newest and step != keep_step and not (d / MARKER_FILENAME).exists():
                shutil.rmtree(d, ignore_errors=True)
                _LOG.warning("removed incomplete checkpoint step=%d at %s", step, d)

    def load(self, state: TrainState, *, parallel: Any = None, step: int | None = None) -> int | None:
        self.wait()
        entries = self.list_checkpoints()
        if step is None:
            if not entries:
                _LOG.info("no complete checkpoint under %s; starting fresh", self._root)
                return None
            entry = entries[-1]
        else:
            match = [e for e in entries if e.step == step]
            if not match:
                raise FileNotFoundError(f"no complete checkpoint for step {step} under {self._root}")
            entry = match[0]
        if int(entry.metadata.get("format_version", 0)) > CHECKPOINT_FORMAT_VERSION:
            raise ValueError(f"checkpoint at {entry.path} uses a newer format version")
        data_rank, data_world = _data_coords(parallel)
        saved = set(entry.metadata.get("keys", ()))
        include_rng = self._include_rng and RNG_KEY in saved
        if include_rng and entry.data_world != data_world:
            _LOG.warning("resuming at data-parallel width %d from a checkpoint written at %d: RNG state is "
                         "re-derived from the seed", data_world, entry.data_world)
            include_rng = False
        to_load = build_stateful(state, data_rank=data_rank, include_rng=include_rng, strict=self._strict,
                                 cpu_offload=self._cpu_offload)
        for key in (SCHEDULE_KEY, EMA_KEY, EXTRAS_KEY, RNG_KEY):
            if key in to_load and saved and key not in saved:
                _LOG.warning("component %r is absent from the checkpoint; it keeps its fresh state", key)
                to_load.pop(key)
        extra = saved - set(to_load) - {MODEL_OPTIMIZER_KEY, PROGRESS_KEY}
        if extra:
            _LOG.warning("checkpoint contains %s which this run does not use; skipped", sorted(extra))
        try:
            with collective_timeout(self._timeout):
                dcp.load(to_load, storage_reader=dcp.FileSystemReader(entry.path))
        except CheckpointException as exc:  # a BaseException in DCP: surface it as an ordinary error
            raise RuntimeError(f"checkpoint {entry.path} could not be read (truncated or corrupt data, or a "
                               f"state layout this run cannot take): {str(exc).splitlines()[0]}") from exc
        return entry.step

    def close(self) -> None:
        self.wait()

    def __enter__(self) -> CheckpointManager:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()


def save(path: str | os.PathLike[str], state: TrainState, *, parallel: Any = None, async_save: bool = True,
         extras: dict[str, Any] | None = None) -> Path:
    mgr = CheckpointManager(path, keep_last_n=0)
    d = mgr.save(state.step, state, parallel=parallel, async_save=async_save, extras=extras)
    mgr.close()
    return d


def load(path: str | os.PathLike[str], state: TrainState, *, parallel: Any = None, step: int | None = None) -> int | None:
    return CheckpointManager(path, keep_last_n=0).load(state, parallel=parallel, step=step)


def load_model(path: str | Path, model: nn.Module, *, strict: bool = True) -> None:
    """Load only the model weights of one checkpoint directory (any rank count)."""
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict, set_model_state_dict

    d = Path(path)
    if not d.is_dir():
        raise FileNotFoundError(f"no checkpoint directory at {d}")
    opts = StateDictOptions(full_state_dict=False, strict=strict)
    holder = {MODEL_OPTIMIZER_KEY: {"model": get_model_state_dict(model, options=opts)}}
    try:
        dcp.load(holder, checkpoint_id=str(d))
    except (Exception, CheckpointException) as exc:  # noqa: BLE001 - DCP's error is a BaseException
        raise RuntimeError(f"could not read model weights from {d}: {str(exc).splitlines()[0]}") from exc
    set_model_state_dict(model, holder[MODEL_OPTIMIZER_KEY]["model"], options=opts)
    from avgen_b200.models.linear import bump_weight_epoch

    bump_weight_epoch()


def load_ema(path: str | Path, model: nn.Module, *, decay: float = 0.9999) -> None:
    """Load the EMA shadow of a checkpoint into ``model``'s weights."""
    from avgen_b200.train.ema import ShardedEMA

    d = Path(path)
    if not d.is_dir():
        raise FileNotFoundError(f"no checkpoint directory at {d}")
    ema = ShardedEMA(model, decay=decay)
    holder = {EMA_KEY: ema.state_dict()}
    try:
        dcp.load(holder, checkpoint_id=str(d))
    except (Exception, CheckpointException) as exc:  # noqa: BLE001 - DCP's error is a BaseException
        raise RuntimeError(f"could not read EMA weights from {d}: {str(exc).splitlines()[0]}") from exc
    ema.load_state_dict(holder[EMA_KEY])
    ema.copy_to(model)
