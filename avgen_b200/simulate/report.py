"""One-configuration simulation report (avgen/simulate/report.py:40-371 API)."""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from avgen_b200.parallel.activation import ActivationCheckpointConfig
from avgen_b200.parallel.dims import ParallelDims
from avgen_b200.simulate.comms import INFINIBAND_NDR, NVLINK5, CommunicationEstimate, Interconnect, \
    estimate_step_communication
from avgen_b200.simulate.compute import B200, Accelerator, ComputeEstimate, estimate_compute, transformer_flops
from avgen_b200.simulate.memory import MemoryEstimate, ModelShape, estimate_memory
from avgen_b200.simulate.plan import attention_seconds_per_layer

__all__ = ["SimulationReport", "simulate_config"]


@dataclass(frozen=True, slots=True)
class SimulationReport:
    shape: ModelShape
    dims: ParallelDims
    activation_checkpoint: ActivationCheckpointConfig
    accelerator: Accelerator
    memory: MemoryEstimate
    compute: ComputeEstimate
    communication: CommunicationEstimate
    gradient_accumulation: int = 1
    notes: tuple[str, ...] = field(default_factory=tuple)

    @property
    def fits(self) -> bool:
        return self.memory.fits_in(self.accelerator.memory_gib)

    @property
    def step_seconds(self) -> float:
        return self.communication.estimated_step_seconds * self.gradient_accumulation

    @property
    def global_batch_size(self) -> int:
        return self.dims.dp_size * self.shape.micro_batch_size * self.gradient_accumulation

    @property
    def tokens_per_second(self) -> float:
        t = self.step_seconds
        return self.global_batch_size * self.shape.sequence_length / t if t > 0 else 0.0

    @property
    def mfu(self) -> float:
        return self.compute.mfu(self.step_seconds / max(1, self.gradient_accumulation), self.accelerator.peak_flops())

    def days_for_tokens(self, target_tokens: float) -> float:
        r = self.tokens_per_second
        return target_tokens / (r * 86400.0) if r > 0 else float("inf")

    def to_dict(self) -> dict[str, Any]:
        comm = self.communication
        return {"plan": self.dims.describe(), "world_size": self.dims.world_size, "accelerator": self.accelerator.name,
                "sequence_length": self.shape.sequence_length, "parameters": self.shape.parameters,
                "micro_batch_size": self.shape.micro_batch_size, "gradient_accumulation": self.gradient_accumulation,
                "global_batch_size": self.global_batch_size, "activation_checkpoint": self.activation_checkpoint.mode,
                "fits": self.fits, "memory_gib": round(self.memory.total_gib, 3),
                "memory_breakdown_gib": {k: round(v, 3) for k, v in self.memory.breakdown_gib().items()},
                "dominant_memory_term": self.memory.dominant_term(), "step_seconds": round(self.step_seconds, 5),
                "compute_seconds": round(self.compute.seconds, 5),
                "exposed_comm_seconds": round(comm.exposed_seconds, 5),
                "comm_gib_per_step": round(comm.total_wire_gib, 4),
                "comm_by_label_seconds": {k: round(v, 5) for k, v in comm.by_label().items()},
                "comm_bottleneck": comm.bottleneck(), "scaling_efficiency": round(comm.scaling_efficiency, 4),
                "mfu": round(self.mfu, 4), "tokens_per_second": round(self.tokens_per_second, 1),
                "recompute_overhead": round(self.compute.recompute_overhead, 4), "notes": list(self.notes)}

    def save(self, path: str | Path) -> Path:
        dest = Path(path)
        dest.parent.mkdir(parents=True, exist_ok=True)
        dest.write_text(json.dumps(self.to_dict(), indent=2, sort_keys=True))
        return dest

    def render(self) -> str:
        local = self.shape.sequence_length // max(1, self.dims.sequence_shard_size)
        bar = "=" * 72
        out = [bar, f"avgen_b200 simulation - {self.dims.describe()}", bar,
               f"  device                {self.accelerator.name} ({self.accelerator.memory_gib:.0f} GiB)",
               f"  parameters            {self.shape.parameters / 1e9:.2f} B",
               f"  depth x width         {self.shape.depth} x {self.shape.width}",
               f"  sequence length       {self.shape.sequence_length:,} tokens ({local:,} per rank)",
               f"  global batch          {self.global_batch_size} (micro {self.shape.micro_batch_size} x accum "
               f"{self.gradient_accumulation} x dp {self.dims.dp_size})", "",
               f"MEMORY  {self.memory.total_gib:.1f} GiB per rank   {'FITS' if self.fits else 'DOES NOT FIT'}"]
        for name, gib in self.memory.breakdown_gib().items():
            if gib > 0.01:
                out.append(f"    {name.removesuffix('_bytes'):<20} {gib:8.2f} GiB")
        out += ["", f"COMPUTE  {self.compute.seconds * 1e3:.1f} ms/microbatch   MFU {self.mfu:.1%}   recompute "
                    f"overhead {self.compute.recompute_overhead:.1%}", "",
                f"COMMUNICATION  {self.communication.total_wire_gib:.2f} GiB/step   exposed "
                f"{self.communication.exposed_seconds * 1e3:.1f} ms   scaling efficiency "
                f"{self.communication.scaling_efficiency:.1%}"]
        out += [f"    {label:<32} {sec * 1e3:8.2f} ms" for label, sec in self.communication.by_label().items()]
        out += ["", f"THROUGHPUT  {self.step_seconds:.3f} s/step   {self.tokens_per_second / 1e6:.2f} M tokens/s"]
        if self.notes:
            out += ["", "NOTES", *(f"    - {n}" for n in self.notes)]
        out.append(bar)
        return "\n".join(out)

    def assert_no_regression(self, baseline: dict[str, Any], *, mfu_tolerance: float = 0.05,
                             memory_tolerance_gib: float = 2.0) -> None:
        cur = self.to_dict()
        if baseline.get("fits") and not cur["fits"]:
            raise AssertionError(f"configuration no longer fits: {cur['memory_gib']:.1f} GiB > "
                                 f"{self.accelerator.memory_gib:.0f} GiB (was {baseline.get('memory_gib')} GiB); "
                                 f"dominant term {cur['dominant_memory_term']}")
        grew = cur["memory_gib"] - float(baseline.get("memory_gib", 0.0))
        if grew > memory_tolerance_gib:
            raise AssertionError(f"per-rank memory grew by {grew:.2f} GiB (tolerance {memory_tolerance_gib} GiB); "
                                 f"dominant term {cur['dominant_memory_term']}")
        base_mfu = float(baseline.get("mfu", 0.0))
        if base_mfu > 0 and (base_mfu - cur["mfu"]) / base_mfu > mfu_tolerance:
            raise AssertionError(f"predicted MFU fell {(base_mfu - cur['mfu']) / base_mfu:.1%} ({base_mfu:.3f} -> "
                                 f"{cur['mfu']:.3f}); communication bottleneck {cur['comm_bottleneck']}")


def _advisories(shape: ModelShape, dims: ParallelDims, memory: MemoryEstimate, comm: CommunicationEstimate,
                accel: Accelerator, policy: ActivationCheckpointConfig) -> tuple[str, ...]:
    notes: list[str] = []
    if dims.tensor > 8:
        notes.append(f"tensor parallel degree {dims.tensor} spans NVLink domains; TP sits on the critical path twice "
                     "per block and belongs inside one NVSwitch domain")
    if dims.pp_enabled and dims.pipeline > shape.depth // 4:
        notes.append(f"pipeline degree {dims.pipeline} leaves fewer than 4 blocks per stage; the bubble dominates")
    if not memory.fits_in(accel.memory_gib):
        notes.append(f"does not fit: {memory.total_gib:.1f} GiB needed, {accel.memory_gib:.0f} GiB available; "
                     f"largest term {memory.dominant_term()}")
    if comm.scaling_efficiency < 0.8:
        notes.append(f"scaling efficiency {comm.scaling_efficiency:.0%}: {comm.bottleneck()} is not hidden")
    frac = transformer_flops(shape)["attention_fraction"]
    if frac > 0.5:
        notes.append(f"attention is {frac:.0%} of forward FLOPs at {shape.sequence_length:,} tokens; the attention "
                     "kernel and context parallelism matter more than parameter sharding")
    if dims.cp_enabled and shape.sequence_length % dims.sequence_shard_size:
        notes.append(f"sequence length {shape.sequence_length} does not divide by cp*tp = {dims.sequence_shard_size}; "
                     "pad at the data boundary")
    if policy.mode != "fused" and accel.name == "B200":
        notes.append(f"policy {policy.mode!r} runs the eager block; the fused B200 block saves only x, O and lse")
    return tuple(notes)


def simulate_config(shape: ModelShape, dims: ParallelDims, *, accelerator: Accelerator = B200,
                    activation_checkpoint: ActivationCheckpointConfig | None = None,
                    intra_node: Interconnect = NVLINK5, inter_node: Interconnect = INFINIBAND_NDR,
                    achieved_fraction: float | None = None, gradient_accumulation: int = 1) -> SimulationReport:
    policy = activation_checkpoint or ActivationCheckpointConfig(mode="fused")
    memory = estimate_memory(shape, dims, activation_checkpoint=policy)
    compute = estimate_compute(shape, dims, accelerator=accelerator, activation_checkpoint=policy,
                               achieved_fraction=achieved_fraction)
    comm = estimate_step_communication(shape, dims, intra_node=intra_node, inter_node=inter_node,
                                       compute_seconds=compute.seconds,
                                       attention_seconds_per_layer=attention_seconds_per_layer(shape, dims,
                                                                                               accelerator))
    return SimulationReport(shape, dims, policy, accelerator, memory, compute, comm, gradient_accumulation,
                            _advisories(shape, dims, memory, comm, accelerator, policy))
