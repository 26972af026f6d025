"""On-device metric accumulation, throughput / MFU and memory reporting
(avgen/telemetry/metrics.py:58-659).

* :class:`MetricAccumulator` sums :class:`StepMetrics` in float64 on the device;
  a flush is one all-reduce over the data mesh plus one device->host copy.
* :class:`ThroughputMeter` times steps with CUDA events (device time, not host
  wall clock), reports p50 / p99 step time, samples/s, tokens/s, MFU and HFU,
  and can take the max over ranks.
* :class:`MemoryReporter` reports current / peak / reserved memory and
  fragmentation, warns near capacity, and reduces the peak across ranks.
"""
from __future__ import annotations

import logging
import statistics
import time
from dataclasses import dataclass, fields

from typing import Any

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh

from avgen_b200.core.metrics import StepMetrics

__all__ = ["MemoryReport", "MemoryReporter", "MetricAccumulator", "ThroughputMeter", "ThroughputReport",
           "merge_metrics"]

_LOG = logging.getLogger("avgen_b200.telemetry")
_NAMES = tuple(f.name for f in fields(StepMetrics))


class MetricAccumulator:
    def __init__(self, *, mesh: DeviceMesh | None = None, device: torch.device | str | None = None) -> None:
        self._mesh = mesh
        self._device = torch.device(device) if device is not None else None
        self._sums: torch.Tensor | None = None
        self._count: torch.Tensor | None = None

    @property
    def device(self) -> torch.device:
        return self._device or torch.device("cpu")

    @property
    def is_empty(self) -> bool:
        return self._sums is None

    def update(self, metrics: StepMetrics, *, weight: float = 1.0) -> None:
        vec = torch.stack([getattr(metrics, n).detach().to(torch.float64) for n in _NAMES])
        if self._sums is None:
            self._device = vec.device
            self._sums = torch.zeros_like(vec)
            self._count = torch.zeros((), dtype=torch.float64, device=vec.device)
        self._sums += vec * weight
        self._count += weight

    def reset(self) -> None:
        self._sums = None
        self._count = None

    def flush(self, *, reset: bool = True) -> dict[str, float]:
        """Means over accumulated steps (and data ranks): one collective, one sync."""
        if self._sums is None:
            return {}
        packed = torch.cat((self._sums, self._count.reshape(1)))
        if self._mesh is not None and self._mesh.size() > 1 and dist.is_initialized():
            dist.all_reduce(packed, group=self._mesh.get_group())
        host = packed.cpu().tolist()
        n = max(host[-1], 1e-12)
        out = {name: v / n for name, v in zip(_NAMES, host[:-1])}
        for k in ("valid_video_tokens", "valid_audio_tokens", "nonfinite", "skipped"):
            out[k] = out[k] * n  # counts are totals
        if reset:
            self.reset()
        return out


@dataclass(frozen=True, slots=True)
class ThroughputReport:
    steps: int
    step_time_p50: float
    step_time_p99: float
    samples_per_second: float
    tokens_per_second: float
    mfu: float
    hfu: float

    def to_mapping(self) -> dict[str, float]:
        return {f"throughput/{f.name}": float(getattr(self, f.name)) for f in fields(self)}


class ThroughputMeter:
    """Device-timed step throughput and model FLOPs utilisation.

    With CUDA, each ``step()`` records an event on the current stream and
    returns at once (no host synchronisation); step times are read from the
    events when ``report()`` is called, which synchronises once. Without CUDA
    the host clock is used. ``report()`` takes the max over ``mesh``'s ranks of
    the window's total time (the slowest rank sets the pace)."""

    def __init__(self, *, flops_per_sample: float = 0.0, hardware_flops_per_sample: float | None = None,
                 peak_flops: float = 2.25e15, world_size: int = 1, mesh: DeviceMesh | None = None,
                 use_cuda_events: bool | None = None, group: Any = None) -> None:
        self._group = mesh.get_group() if mesh is not None and mesh.size() > 1 else group
        self._fps = flops_per_sample
        self._hfps = hardware_flops_per_sample if hardware_flops_per_sample is not None else flops_per_sample
        self._peak = peak_flops
        self._world = world_size
        self._mesh = mesh
        self._events = torch.cuda.is_available() if use_cuda_events is None else use_cuda_events
        self._marks: list[object] = []  # window start, then one mark per step (events or host times)
        self._samples = 0
        self._tokens = 0

    def _mark(self) -> object:
        if not self._events:
            return time.perf_counter()
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def start(self) -> None:
        self._marks = [self._mark()]

    def step(self, *, samples: int = 0, tokens: int = 0) -> None:
        """Close the current step."""
        if not self._marks:
            self.start()
            return
        self._marks.append(self._mark())
        self._samples += samples
        self._tokens += tokens

    def _step_times(self) -> list[float]:
        if len(self._marks) < 2:
            return []
        if not self._events:
            return [b - a for a, b in zip(self._marks, self._marks[1:])]  # type: ignore[operator]
        self._marks[-1].synchronize()  # type: ignore[union-attr]
        return [a.elapsed_time(b) / 1000.0 for a, b in zip(self._marks, self._marks[1:])]  # type: ignore[union-attr]

    def report(self, *, reset: bool = True) -> ThroughputReport:
        step_times = self._step_times()
        times = sorted(step_times) or [float("nan")]
        total = sum(step_times)
        if self._group is not None and dist.is_initialized() and dist.get_world_size(self._group) > 1:
            t = torch.tensor([total], dtype=torch.float64, device="cuda" if self._events else "cpu")
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self._group)
            total = float(t.item())
        sps = self._samples / total if total > 0 else 0.0
        tps = self._tokens / total if total > 0 else 0.0
        p99 = times[min(len(times) - 1, int(round(0.99 * (len(times) - 1))))]
        rep = ThroughputReport(steps=len(step_times), step_time_p50=statistics.median(times), step_time_p99=p99,
                               samples_per_second=sps, tokens_per_second=tps,
                               mfu=sps * self._fps / (self._peak * self._world) if self._peak else 0.0,
                               hfu=sps * self._hfps / (self._peak * self._world) if self._peak else 0.0)
        if reset:
            self._marks = self._marks[-1:]
            self._samples = self._tokens = 0
        return rep


@dataclass(frozen=True, slots=True)
class MemoryReport:
    allocated_gib: float
    peak_allocated_gib: float
    reserved_gib: float
    peak_reserved_gib: float
    total_gib: float
    fragmentation: float

    def to_mapping(self) -> dict[str, float]:
        return {f"memory/{f.name}": float(getattr(self, f.name)) for f in fields(self)}


class MemoryReporter:
    def __init__(self, device: torch.device | str | None = None, *, warn_fraction: float = 0.92) -> None:
        self._device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        self._warn = warn_fraction
        self._warned = False

    @property
    def available(self) -> bool:
        return self._device.type == "cuda" and torch.cuda.is_available()

    def reset_peaks(self) -> None:
        if self.available:
            torch.cuda.reset_peak_memory_stats(self._device)

    def report(self) -> MemoryReport | None:
        if not self.available:
            return None
        g = 1024 ** 3
        alloc = torch.cuda.memory_allocated(self._device) / g
        peak = torch.cuda.max_memory_allocated(self._device) / g
        res = torch.cuda.memory_reserved(self._device) / g
        peak_res = torch.cuda.max_memory_reserved(self._device) / g
        total = torch.cuda.get_device_properties(self._device).total_memory / g
        frag = 1.0 - alloc / res if res > 0 else 0.0
        if not self._warned and peak_res > self._warn * total:
            self._warned = True
            _LOG.warning("peak reserved memory %.1f GiB is within %.0f%% of the %.1f GiB capacity", peak_res,
                         100 * (1 - self._warn), total)
        return MemoryReport(alloc, peak, res, peak_res, total, frag)

    def clear_warning(self) -> None:
        self._warned = False

    def peak_across(self, mesh: DeviceMesh | None) -> MemoryReport | None:
        rep = self.report()
        if rep is None or mesh is None or mesh.size() == 1 or not dist.is_initialized():
            return rep
        t = torch.tensor([getattr(rep, f.name) for f in fields(rep)], dtype=torch.float64, device=self._device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=mesh.get_group())
        return MemoryReport(*t.tolist())


def merge_metrics(*parts: dict[str, float]) -> dict[str, float]:
    out: dict[str, float] = {}
    for p in parts:
        out.update(p)
    return out
