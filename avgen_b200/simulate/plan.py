"""Parallel-plan search (avgen/simulate/plan.py:40-371 API).

Enumerates (tensor, pipeline, context, replicate, shard) factorisations of the
world, keeps the first activation policy of each that fits in memory (the
fused B200 block first), prices compute and communication, and ranks plans by
throughput with near-ties broken by memory headroom.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

from avgen_b200.parallel.activation import ActivationCheckpointConfig
from avgen_b200.parallel.dims import ParallelDims
from avgen_b200.simulate.comms import INFINIBAND_NDR, NVLINK5, CommunicationEstimate, Interconnect, \
    estimate_step_communication
from avgen_b200.simulate.compute import B200, Accelerator, ComputeEstimate, estimate_compute, transformer_flops
from avgen_b200.simulate.memory import MemoryEstimate, ModelShape, estimate_memory

__all__ = ["PlanCandidate", "SearchSpace", "render_plan_table", "search_parallel_plan"]


def _divisors(n: int, *, maximum: int | None = None) -> list[int]:
    top = n if maximum is None else min(n, maximum)
    return [d for d in range(1, top + 1) if n % d == 0]


def _default_policies() -> tuple[ActivationCheckpointConfig, ...]:
    return (ActivationCheckpointConfig(mode="fused"), ActivationCheckpointConfig(mode="none"),
            ActivationCheckpointConfig(mode="selective_op", save_op_frequency=1),
            ActivationCheckpointConfig(mode="selective_op", save_op_frequency=2),
            ActivationCheckpointConfig(mode="full"))


@dataclass(frozen=True, slots=True)
class SearchSpace:
    world_size: int
    gpus_per_node: int = 8
    max_tensor: int = 8
    max_context: int = 16
    max_pipeline: int = 1
    allow_hsdp: bool = True
    global_batch_size: int | None = None
    min_blocks_per_stage: int = 4
    activation_policies: tuple[ActivationCheckpointConfig, ...] = field(default_factory=_default_policies)

    def __post_init__(self) -> None:
        if self.world_size < 1:
            raise ValueError(f"world_size must be positive; got {self.world_size!r}")
        if self.gpus_per_node < 1:
            raise ValueError(f"gpus_per_node must be positive; got {self.gpus_per_node!r}")


@dataclass(frozen=True, slots=True)
class PlanCandidate:
    dims: ParallelDims
    activation_checkpoint: ActivationCheckpointConfig
    memory: MemoryEstimate
    compute: ComputeEstimate
    communication: CommunicationEstimate
    micro_batch_size: int
    gradient_accumulation: int = 1

    @property
    def step_seconds(self) -> float:
        return self.communication.estimated_step_seconds * self.gradient_accumulation

    @property
    def samples_per_second(self) -> float:
        t = self.step_seconds
        return self.dims.dp_size * self.micro_batch_size * self.gradient_accumulation / t if t > 0 else 0.0

    def mfu(self, accelerator: Accelerator, *, use_fp8: bool = False) -> float:
        return self.compute.mfu(self.step_seconds / max(1, self.gradient_accumulation),
                                accelerator.peak_flops(fp8=use_fp8))

    def summary(self, accelerator: Accelerator) -> dict[str, Any]:
        return {"plan": self.dims.describe(), "activation_checkpoint": self.activation_checkpoint.mode,
                "micro_batch": self.micro_batch_size, "grad_accum": self.gradient_accumulation,
                "memory_gib": round(self.memory.total_gib, 2),
                "memory_headroom_gib": round(accelerator.memory_gib - self.memory.total_gib, 2),
                "step_seconds": round(self.step_seconds, 4), "samples_per_second": round(self.samples_per_second, 3),
                "mfu": round(self.mfu(accelerator), 4),
                "scaling_efficiency": round(self.communication.scaling_efficiency, 4),
                "comm_gib_per_step": round(self.communication.total_wire_gib, 3),
                "bottleneck": self.communication.bottleneck(), "dominant_memory": self.memory.dominant_term()}


def attention_seconds_per_layer(shape: ModelShape, dims: ParallelDims, accelerator: Accelerator) -> float:
    """Forward attention time of one layer on one rank (what a fused K/V stream hides under)."""
    f = transformer_flops(shape, include_backward=False)
    per_layer = f["attention"] / max(1, shape.depth) / max(1, dims.context * dims.tensor)
    return per_layer / (accelerator.peak_flops() * accelerator.kernels.attention_fwd)


def search_parallel_plan(shape: ModelShape, space: SearchSpace, *, accelerator: Accelerator = B200,
                         intra_node: Interconnect = NVLINK5, inter_node: Interconnect = INFINIBAND_NDR,
                         achieved_fraction: float | None = None, headroom: float = 0.1, top_k: int = 10,
                         throughput_tie_tolerance: float = 0.02) -> list[PlanCandidate]:
    found: list[PlanCandidate] = []
    tp_cap = min(space.max_tensor, space.gpus_per_node, space.world_size)
    for tp in _divisors(space.world_size, maximum=tp_cap):
        for pp in _divisors(space.world_size // tp, maximum=space.max_pipeline):
            if shape.depth % pp or shape.depth // pp < space.min_blocks_per_stage:
                continue
            rest = space.world_size // (tp * pp)
            for cp in _divisors(rest, maximum=space.max_context):
                if shape.sequence_length % (cp * tp):
                    continue
                dp = rest // cp
                for rep in (_divisors(dp) if space.allow_hsdp else [1]):
                    shard = dp // rep
                    if rep > 1 and shard == 1:
                        continue
                    try:
                        dims = ParallelDims(world_size=space.world_size, dp_replicate=rep, dp_shard=shard, tensor=tp,
                                            context=cp, pipeline=pp)
                    except ValueError:
                        continue
                    accum = 1
                    if space.global_batch_size is not None:
                        try:
                            accum = dims.gradient_accumulation_for(global_batch_size=space.global_batch_size,
                                                                   local_batch_size=shape.micro_batch_size)
                        except ValueError:
                            continue
                    for policy in space.activation_policies:
                        mem = estimate_memory(shape, dims, activation_checkpoint=policy)
                        if not mem.fits_in(accelerator.memory_gib, headroom=headroom):
                            continue
                        comp = estimate_compute(shape, dims, accelerator=accelerator, activation_checkpoint=policy,
                                                achieved_fraction=achieved_fraction)
                        comm = estimate_step_communication(
                            shape, dims, intra_node=intra_node, inter_node=inter_node, compute_seconds=comp.seconds,
                            attention_seconds_per_layer=attention_seconds_per_layer(shape, dims, accelerator))
                        found.append(PlanCandidate(dims, policy, mem, comp, comm, shape.micro_batch_size, accum))
                        break
    if not found:
        return []
    best = max(c.samples_per_second for c in found)
    tied_above = best * (1.0 - throughput_tie_tolerance)

    def rank(c: PlanCandidate) -> tuple[int, float, float]:
        tied = c.samples_per_second >= tied_above
        return (0 if tied else 1, c.memory.total_gib if tied else -c.samples_per_second, -c.samples_per_second)

    return sorted(found, key=rank)[:top_k]


_COLUMNS = (("plan", 34), ("activation_checkpoint", 20), ("memory_gib", 11), ("step_seconds", 13),
            ("samples_per_second", 19), ("mfu", 7), ("scaling_efficiency", 19), ("bottleneck", 26))


def render_plan_table(candidates: list[PlanCandidate], accelerator: Accelerator) -> str:
    if not candidates:
        return ("No configuration fits. In order of effect:\n"
                "  1. more context parallelism (sequence length usually binds first for video);\n"
                "  2. a shorter clip or a lower resolution;\n"
                "  3. a device with more memory;\n"
                "  4. a shallower or narrower model.")
    rows = [c.summary(accelerator) for c in candidates]
    widths = {n: max(m, len(n), *(len(str(r[n])) for r in rows)) for n, m in _COLUMNS}
    head = " ".join(n.ljust(widths[n]) for n, _ in _COLUMNS)
    return "\n".join([head, "-" * len(head)] + [" ".join(str(r[n]).ljust(widths[n]) for n, _ in _COLUMNS)
                                                 for r in rows])
