"""Profiling and hang forensics (avgen/telemetry/profiler.py:63-320) plus device timing.

* ``profile_steps``: a rank-gated ``torch.profiler`` schedule writing
  ``trace_rank{r}_step{n}.json.gz`` Chrome traces.
* ``memory_snapshot``: CUDA caching-allocator history to a pickle for the
  memory visualiser.
* ``flight_recorder_dump``: the NCCL flight recorder (enabled by
  ``init_distributed``) written to disk for hang analysis.
* ``DeviceTimer`` / ``nvtx_range``: CUDA-event timing of named regions (max over
  ranks on request) and NVTX ranges for external profilers.
"""
from __future__ import annotations

import contextlib
import os
import pickle
from collections import defaultdict
from collections.abc import Iterator
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

__all__ = ["DeviceTimer", "flight_recorder_dump", "memory_snapshot", "nvtx_range", "profile_steps",
           "should_profile_rank"]


def _rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else int(os.environ.get("RANK", "0"))


def should_profile_rank(*, mode: str = "global_zero") -> bool:
    """``global_zero``: rank 0 only; ``local_zero``: local rank 0 of each node; ``all``."""
    if mode == "all":
        return True
    if mode == "local_zero":
        return int(os.environ.get("LOCAL_RANK", "0")) == 0
    if mode == "global_zero":
        return _rank() == 0
    raise ValueError(f"unknown profiling mode {mode!r}")


class _NullProfiler:
    def step(self) -> None:
        pass

    def export_chrome_trace(self, path: str) -> None:
        del path

    def __enter__(self) -> _NullProfiler:
        return self

    def __exit__(self, *exc: object) -> None:
        pass


def profile_steps(output_dir: str | os.PathLike[str], *, active: int = 3, warmup: int = 5, wait: int = 0,
                  repeat: int = 1, mode: str = "global_zero", record_shapes: bool = False,
                  with_stack: bool = False) -> Any:
    """A profiler context; call ``.step()`` once per training step."""
    if active <= 0 or not should_profile_rank(mode=mode):
        return _NullProfiler()
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    rank = _rank()
    acts = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(torch.profiler.ProfilerActivity.CUDA)

    def handler(prof: torch.profiler.profile) -> None:
        prof.export_chrome_trace(str(out / f"trace_rank{rank}_step{prof.step_num}.json.gz"))

    return torch.profiler.profile(activities=acts,
                                  schedule=torch.profiler.schedule(wait=wait, warmup=warmup, active=active,
                                                                   repeat=repeat),
                                  on_trace_ready=handler, record_shapes=record_shapes, with_stack=with_stack)


@contextlib.contextmanager
def memory_snapshot(path: str | os.PathLike[str], *, max_entries: int = 100_000) -> Iterator[None]:
    """Record allocator history inside the block and dump it on exit."""
    if not torch.cuda.is_available():
        yield
        return
    torch.cuda.memory._record_memory_history(max_entries=max_entries)
    try:
        yield
    finally:
        p = Path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        torch.cuda.memory._dump_snapshot(str(p))
        torch.cuda.memory._record_memory_history(enabled=None)


def flight_recorder_dump(path: str | os.PathLike[str]) -> Path | None:
    """Write this rank's NCCL flight-recorder buffer (``None`` if unavailable)."""
    try:
        from torch._C._distributed_c10d import _dump_nccl_trace
    except ImportError:
        return None
    try:
        payload = _dump_nccl_trace()
    except RuntimeError:
        return None
    p = Path(path)
    target = p / f"flight_recorder_rank{_rank()}.pkl" if p.suffix == "" else p  # a directory, or a file name
    target.parent.mkdir(parents=True, exist_ok=True)
    with open(target, "wb") as fh:
        fh.write(payload if isinstance(payload, bytes) else pickle.dumps(payload))
    return target


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class DeviceTimer:
    """Accumulates CUDA-event durations of named regions on the current stream."""

    def __init__(self) -> None:
        self._open: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self.totals_ms: dict[str, float] = defaultdict(float)

    @contextlib.contextmanager
    def region(self, name: str) -> Iterator[None]:
        if not torch.cuda.is_available():
            yield
            return
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self._open.append((name, start, end))

    def collect(self, *, max_over_ranks: bool = False) -> dict[str, float]:
        if not self._open and not self.totals_ms:
            return {}
        torch.cuda.synchronize()
        for name, s, e in self._open:
            self.totals_ms[name] += s.elapsed_time(e)
        self._open.clear()
        out = dict(self.totals_ms)
        if max_over_ranks and dist.is_initialized() and out:
            keys = sorted(out)
            t = torch.tensor([out[k] for k in keys], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out = dict(zip(keys, t.tolist()))
        return out
