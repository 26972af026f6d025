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
        """A plain-text summary: one headline, then one aligned table per concern."""
        d = self.to_dict()
        local = self.shape.sequence_length // max(1, self.dims.sequence_shard_size)
        verdict = "fits" if d["fits"] else "DOES NOT FIT"
        head = (f"{d['plan']} on {self.accelerator.name}: {self.step_seconds:.3f} s/step, "
                f"{d['tokens_per_second'] / 1e6:.2f} M tok/s, MFU {d['mfu']:.1%}, {d['memory_gib']:.1f} GiB/rank "
                f"({verdict})")
        sections = [
            ("model", [("parameters", f"{self.shape.parameters / 1e9:.2f} B ({self.shape.depth} x {self.shape.width})"),
                       ("tokens", f"{self.shape.sequence_length:,} per sample, {local:,} per rank"),
                       ("global batch", f"{d['global_batch_size']} = dp {self.dims.dp_size} x micro "
                                        f"{self.shape.micro_batch_size} x accumulation {self.gradient_accumulation}")]),
            ("memory per rank (GiB)", [(k.removesuffix("_bytes"), f"{v:.2f}")
                                       for k, v in d["memory_breakdown_gib"].items() if v > 0.01]
             + [("device", f"{self.accelerator.memory_gib:.0f}")]),
            ("compute", [("per micro-batch", f"{d['compute_seconds'] * 1e3:.1f} ms"),
                         ("recompute", f"{d['recompute_overhead']:.1%}")]),
            ("communication (exposed ms)", [(k, f"{v * 1e3:.2f}") for k, v in d["comm_by_label_seconds"].items()]
             + [("total on the wire", f"{d['comm_gib_per_step']:.2f} GiB/step"),
                ("scaling efficiency", f"{d['scaling_efficiency']:.1%}")]),
        ]
        lines = [head]
        for title, rows in sections:
            width = max((len(k) for k, _ in rows), default=0)
            lines.append(f"[{title}]")
            lines += [f"  {k.ljust(width)}  {v}" for k, v in rows]
        if self.notes:
            lines.append("[advice]")
            lines += [f"  * {n}" for n in self.notes]
        return "\n".join(lines)

    def assert_no_regression(self, baseline: dict[str, Any], *, mfu_tolerance: float = 0.05,
                             memory_tolerance_gib: float = 2.0) -> None:
        """Compare against a pinned report; raise one AssertionError naming every
        metric that moved past its tolerance (fit lost, memory up, MFU down)."""
        now = self.to_dict()
        problems: list[str] = []
        if bool(baseline.get("fits")) and not now["fits"]:
            problems.append(f"fit lost: {now['memory_gib']:.1f} GiB on a {self.accelerator.memory_gib:.0f} GiB device")
        pinned_mem = float(baseline.get("memory_gib", 0.0))
        if now["memory_gib"] - pinned_mem > memory_tolerance_gib:
            problems.append(f"memory {pinned_mem:.2f} -> {now['memory_gib']:.2f} GiB "
                            f"(+{now['memory_gib'] - pinned_mem:.2f} > {memory_tolerance_gib})")
        pinned_mfu = float(baseline.get("mfu", 0.0))
        if pinned_mfu > 0.0 and now["mfu"] < pinned_mfu * (1.0 - mfu_tolerance):
            problems.append(f"MFU {pinned_mfu:.3f} -> {now['mfu']:.3f} (more than {mfu_tolerance:.0%} lower)")
        if problems:
            raise AssertionError(f"{self.dims.describe()} regressed: " + "; ".join(problems)
                                 + f" [largest memory term {now['dominant_memory_term']}, "
                                   f"communication bottleneck {now['comm_bottleneck']}]")


# Advisory rules: each looks at the estimate and returns a sentence or None. They
# encode B200 / NVLink 5 facts: an HGX B200 node is one NVSwitch domain of 8 GPUs,
# the ring attention kernel takes key tiles of 128 tokens, and exposed
# communication above 5 % of a step is worth restructuring.
_NODE_GPUS = 8


def _rule_memory(shape, dims, memory, comm, accel, policy):  # noqa: ANN001, ANN202
    need, have = memory.total_gib, accel.memory_gib
    if need > have:
        return f"needs {need:.1f} of {have:.0f} GiB: shrink {memory.dominant_term()} (more sharding or recompute)"
    if need > 0.95 * have:
        return f"{need:.1f} of {have:.0f} GiB leaves under 5 % headroom for allocator fragmentation"
    return None


def _rule_ring_tiles(shape, dims, memory, comm, accel, policy):  # noqa: ANN001, ANN202
    if not dims.cp_enabled:
        return None
    if shape.sequence_length % dims.sequence_shard_size:
        return (f"{shape.sequence_length} tokens do not split over cp x tp = {dims.sequence_shard_size}: pad the "
                "sequence at the data boundary")
    if (shape.sequence_length // dims.sequence_shard_size) % 128:
        return "tokens per context-parallel rank are not a multiple of 128: the NVLink ring kernel falls back to NCCL"
    return None


def _rule_domains(shape, dims, memory, comm, accel, policy):  # noqa: ANN001, ANN202
    inner = dims.tensor * (dims.context if dims.cp_enabled else 1)
    if dims.tensor > _NODE_GPUS:
        return f"tp={dims.tensor} leaves the {_NODE_GPUS}-GPU NVSwitch domain: keep tensor parallelism inside a node"
    if inner > _NODE_GPUS:
        return f"tp x cp = {inner} > {_NODE_GPUS}: ring steps cross InfiniBand; prefer cp inside a node"
    return None


def _rule_exposed(shape, dims, memory, comm, accel, policy):  # noqa: ANN001, ANN202
    step = comm.estimated_step_seconds
    if step > 0 and comm.exposed_seconds / step > 0.05:
        return f"{comm.exposed_seconds / step:.0%} of the step waits on {comm.bottleneck()}"
    return None


def _rule_pipeline(shape, dims, memory, comm, accel, policy):  # noqa: ANN001, ANN202
    if dims.pp_enabled and shape.depth < 4 * dims.pipeline:
        return f"{shape.depth} blocks over pp={dims.pipeline} stages: under 4 blocks per stage, the bubble dominates"
    return None


def _rule_attention(shape, dims, memory, comm, accel, policy):  # noqa: ANN001, ANN202
    frac = transformer_flops(shape)["attention_fraction"]
    if frac > 0.5:
        return f"attention is {frac:.0%} of forward FLOPs: its kernel speed sets the step time"
    return None


def _rule_policy(shape, dims, memory, comm, accel, policy):  # noqa: ANN001, ANN202
    if accel.name == "B200" and policy.mode != "fused":
        return f"activation policy {policy.mode!r} takes the per-layer path; 'fused' keeps only x, O and lse"
    return None


_RULES = (_rule_memory, _rule_domains, _rule_ring_tiles, _rule_exposed, _rule_attention, _rule_pipeline,
          _rule_policy)


def _advisories(shape: ModelShape, dims: ParallelDims, memory: MemoryEstimate, comm: CommunicationEstimate,
                accel: Accelerator, policy: ActivationCheckpointConfig) -> tuple[str, ...]:
    notes = (rule(shape, dims, memory, comm, accel, policy) for rule in _RULES)
    return tuple(n for n in notes if n)


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
