"""Execution-trace capture for network simulators (avgen/simulate/chakra.py:20-205 API).

Captures a PyTorch execution trace (and a Kineto timing trace) of a few steps;
the MLCommons Chakra tools convert them for ASTRA-sim. The conversion itself
runs outside this package (no network here to fetch the tools).
"""
from __future__ import annotations

import json
from collections.abc import Callable, Iterator
from contextlib import contextmanager
from dataclasses import dataclass
from pathlib import Path
from typing import Any

__all__ = ["CONVERSION_STEPS", "TraceArtifacts", "capture_execution_trace", "capture_with_timing"]

CONVERSION_STEPS = """Convert the captured traces for ASTRA-sim:
  1. install the MLCommons Chakra tools (chakra_trace_link, chakra_converter)
  2. chakra_trace_link --chakra-host-trace {et} --chakra-device-trace {kineto} --output-file linked.json
  3. chakra_converter PyTorch --input linked.json --output chakra.et --num-ranks {world}
  4. astra-sim --workload-configuration=chakra --system-configuration=system.json \\
        --network-configuration=network.yml --remote-memory-configuration=memory.json
"""
_COLLECTIVE_HINTS = ("c10d", "nccl", "all_gather", "all_reduce", "reduce_scatter", "all_to_all", "broadcast")


@dataclass(frozen=True, slots=True)
class TraceArtifacts:
    execution_trace: Path
    kineto_trace: Path | None
    world_size: int

    def conversion_commands(self) -> str:
        return CONVERSION_STEPS.format(et=self.execution_trace,
                                       kineto=self.kineto_trace or "<capture_with_timing writes one>",
                                       world=self.world_size)

    def summarize(self) -> dict[str, Any]:
        data = json.loads(self.execution_trace.read_text())
        nodes = data.get("nodes", []) if isinstance(data, dict) else []
        counts: dict[str, int] = {}
        collectives = 0
        for node in nodes:
            name = str(node.get("name", "?"))
            counts[name] = counts.get(name, 0) + 1
            low = name.lower()
            collectives += any(h in low for h in _COLLECTIVE_HINTS)
        top = dict(sorted(counts.items(), key=lambda kv: kv[1], reverse=True)[:10])
        return {"total_nodes": len(nodes), "distinct_ops": len(counts), "collective_nodes": collectives,
                "top_operators": top}


@contextmanager
def capture_execution_trace(output: str | Path) -> Iterator[Path]:
    from torch.profiler import ExecutionTraceObserver

    path = Path(output)
    path.parent.mkdir(parents=True, exist_ok=True)
    obs = ExecutionTraceObserver()
    obs.register_callback(str(path))
    obs.start()
    try:
        yield path
    finally:
        obs.stop()
        obs.unregister_callback()


def capture_with_timing(step: Callable[[], Any], output_dir: str | Path, *, world_size: int, warmup_steps: int = 3,
                        active_steps: int = 1) -> TraceArtifacts:
    import torch
    from torch.profiler import ProfilerActivity, profile, schedule

    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    et, kineto = out / "execution_trace.json", out / "kineto_trace.json"
    for _ in range(warmup_steps):
        step()
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    with capture_execution_trace(et), profile(activities=acts, record_shapes=True,
                                              schedule=schedule(wait=0, warmup=0, active=active_steps)) as prof:
        for _ in range(active_steps):
            step()
            prof.step()
    prof.export_chrome_trace(str(kineto))
    return TraceArtifacts(execution_trace=et, kineto_trace=kineto, world_size=world_size)
