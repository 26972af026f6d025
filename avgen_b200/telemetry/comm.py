"""Exposed communication: device time the compute stream spends waiting on communication.

Communication that overlaps compute costs nothing; what the north-star target
(ring attention's exposed communication under 5 % of step time) counts is the
part the compute stream waits for. Three sources are measured, all on the
device:

* spans: CUDA events recorded on the compute stream around an operation that
  is pure communication or waits for it (the ring's one-word readiness
  all-reduce, its wait for the copy stream, the dK/dV barrier and owner-side
  sum; FSDP's parameter unshard before each block's forward);
* in-kernel waits: the ring attention kernel adds the SM cycles its CTAs spend
  waiting for peer K/V slabs into a device counter; the total divided by the
  CTAs resident at once (one per SM) and the SM clock is the time the kernel
  was held up;
* nothing else is counted: FSDP's reduce-scatter and the ring copies run on
  their own streams and appear here only if the compute stream waits for them.

Accounting is off by default (``enable()`` turns it on; recording costs two
events per span). ``summary(sm_mhz)`` synchronises and returns milliseconds
per source since the last ``reset()``.
"""
from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager
from typing import Any, Iterator

import torch

__all__ = ["comm_span", "counter", "enable", "enabled", "instrument_fsdp", "reset", "summary"]

_STATE: dict[str, Any] = {"on": False, "spans": [], "counters": {}}


def enable(on: bool = True) -> None:
    _STATE["on"] = bool(on)


def enabled() -> bool:
    return bool(_STATE["on"])


def reset() -> None:
    _STATE["spans"].clear()
    for t, _ in _STATE["counters"].values():
        t.zero_()


@contextmanager
def comm_span(name: str, device: torch.device | None = None) -> Iterator[None]:
    """Record the device time of the enclosed stream work under ``name`` (when enabled)."""
    if not _STATE["on"] or not torch.cuda.is_available():
        yield
        return
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    start.record(stream)
    try:
        yield
    finally:
        end.record(stream)
        _STATE["spans"].append((name, start, end))


def counter(name: str, device: torch.device, concurrency: int) -> torch.Tensor:
    """An int64 device word that kernels add wait cycles into; ``concurrency`` is how
    many waiting CTAs run at once (their waits overlap in time)."""
    entry = _STATE["counters"].get((name, device))
    if entry is None:
        entry = (torch.zeros(1, dtype=torch.int64, device=device), max(1, int(concurrency)))
        _STATE["counters"][(name, device)] = entry
    return entry[0]


def summary(sm_mhz: float | None = None) -> dict[str, float]:
    """Milliseconds per source since ``reset()`` (synchronises the device)."""
    out: dict[str, float] = defaultdict(float)
    if _STATE["spans"]:
        torch.cuda.synchronize()
    for name, start, end in _STATE["spans"]:
        out[name] += start.elapsed_time(end)
    if _STATE["counters"]:
        mhz = sm_mhz or 0.0
        if not mhz and torch.cuda.is_available():
            mhz = torch.cuda.get_device_properties(torch.cuda.current_device()).clock_rate / 1e3
        for (name, _), (t, conc) in _STATE["counters"].items():
            cycles = float(t.item())
            out[name] += cycles / conc / (mhz * 1e3) if mhz else 0.0
    return dict(out)


def instrument_fsdp(model: torch.nn.Module) -> int:
    """Bracket every FSDP2 module's pre-forward (parameter unshard: the wait for its
    all-gather and the copy-out) with a ``fsdp_unshard`` span. Returns the count."""
    from torch.distributed.fsdp import FSDPModule

    count = 0
    for module in model.modules():
        if not isinstance(module, FSDPModule):
            continue
        pending: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []

        def before(mod: torch.nn.Module, args: Any, _pending=pending) -> None:  # noqa: ANN001
            if _STATE["on"]:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                _pending.append((ev, ev))

        def after(mod: torch.nn.Module, args: Any, _pending=pending) -> None:  # noqa: ANN001
            if _STATE["on"] and _pending:
                start, _ = _pending.pop()
                end = torch.cuda.Event(enable_timing=True)
                end.record()
                _STATE["spans"].append(("fsdp_unshard", start, end))

        module.register_forward_pre_hook(before, prepend=True)
        module.register_forward_pre_hook(after)
        count += 1
    return count
