"""Interconnect tiers and per-step collective costs (avgen/simulate/comms.py:60-470 API).

NVLink 5 is calibrated to this pool's measurements: an 8-rank all-reduce bus
bandwidth of 725 GB/s and 770 GB/s per direction for a peer copy (900 GB/s
nominal). Collective wire bytes use the ring formulas. Context parallelism is
modelled as the framework runs it: every rank receives the other ranks' K/V
once per layer in the forward (``cp - 1`` shards) and returns dK/dV partials
once in the backward; both overlap the attention kernel, so only the part that
exceeds the attention time of that layer is exposed.
"""
from __future__ import annotations

import functools
import math

import contextlib
from collections.abc import Callable
from dataclasses import dataclass
from typing import Any

from avgen_b200.simulate.memory import ModelShape

__all__ = ["ETHERNET_200G", "INFINIBAND_NDR", "NVLINK4", "NVLINK5", "CollectiveCost", "CommunicationEstimate",
           "Interconnect", "calibrate_from_busbw", "count_collectives", "estimate_step_communication"]

_GIB = 1024.0 ** 3


@dataclass(frozen=True, slots=True)
class Interconnect:
    name: str
    peak_gbps: float
    efficiency: float = 0.8
    latency_us: float = 5.0
    ranks_per_group: int = 8

    def __post_init__(self) -> None:
        if self.peak_gbps <= 0:
            raise ValueError("peak_gbps must be positive")
        if not 0.0 < self.efficiency <= 1.0:
            raise ValueError("efficiency must be in (0, 1]")

    @property
    def achievable_bytes_per_second(self) -> float:
        return self.peak_gbps * 1e9 * self.efficiency

    def transfer_seconds(self, byte_count: float) -> float:
        return self.latency_us * 1e-6 + byte_count / self.achievable_bytes_per_second


NVLINK4 = Interconnect("NVLink 4 (H100)", peak_gbps=450.0, efficiency=0.85, latency_us=3.0)
NVLINK5 = Interconnect("NVLink 5 (B200)", peak_gbps=900.0, efficiency=770.0 / 900.0, latency_us=3.0)
INFINIBAND_NDR = Interconnect("InfiniBand NDR 400G", peak_gbps=50.0, efficiency=0.75, latency_us=8.0)
ETHERNET_200G = Interconnect("RoCE 200G", peak_gbps=25.0, efficiency=0.6, latency_us=15.0)


def calibrate_from_busbw(name: str, *, measured_busbw_gbps: float, peak_gbps: float, latency_us: float = 5.0,
                         ranks_per_group: int = 8) -> Interconnect:
    return Interconnect(name, peak_gbps, min(1.0, measured_busbw_gbps / peak_gbps), latency_us, ranks_per_group)


@dataclass(frozen=True, slots=True)
class CollectiveCost:
    label: str
    kind: str
    payload_bytes: float
    wire_bytes: float
    ranks: int
    count: int
    tier: str
    seconds: float
    overlappable_with: float = 0.0  # seconds of compute this collective can hide under
    synchronising: bool = False  # a wait for the slowest rank: never hidden under compute


def _wire(kind: str, payload: float, ranks: int) -> float:
    if ranks <= 1:
        return 0.0
    f = (ranks - 1) / ranks
    return 2.0 * payload * f if kind == "all_reduce" else payload * f


@dataclass(frozen=True, slots=True)
class CommunicationEstimate:
    collectives: tuple[CollectiveCost, ...]
    compute_seconds: float = 0.0
    overlap_efficiency: float = 0.8

    @property
    def total_seconds(self) -> float:
        return sum(c.seconds for c in self.collectives)

    @property
    def total_wire_gib(self) -> float:
        return sum(c.wire_bytes * c.count for c in self.collectives) / _GIB

    @property
    def exposed_seconds(self) -> float:
        exposed = 0.0
        general = 0.0
        for c in self.collectives:
            if c.synchronising:
                exposed += c.seconds
            elif c.overlappable_with > 0:  # fused with its compute: only the excess is exposed
                exposed += max(0.0, c.seconds - c.overlappable_with)
            else:
                general += c.seconds
        hidden = min(general * self.overlap_efficiency, self.compute_seconds)
        return exposed + max(0.0, general - hidden)

    @property
    def estimated_step_seconds(self) -> float:
        return self.compute_seconds + self.exposed_seconds

    @property
    def scaling_efficiency(self) -> float:
        t = self.estimated_step_seconds
        return self.compute_seconds / t if t > 0 else 1.0

    def by_label(self) -> dict[str, float]:
        out: dict[str, float] = {}
        for c in self.collectives:
            out[c.label] = out.get(c.label, 0.0) + c.seconds
        return dict(sorted(out.items(), key=lambda kv: kv[1], reverse=True))

    def bottleneck(self) -> str:
        return next(iter(self.by_label()), "none")


def estimate_step_communication(shape: ModelShape, dims: Any, *, intra_node: Interconnect = NVLINK5,
                                inter_node: Interconnect = INFINIBAND_NDR, param_dtype_bytes: int = 2,
                                reduce_dtype_bytes: int = 4, compute_seconds: float = 0.0,
                                overlap_efficiency: float = 0.8,
                                attention_seconds_per_layer: float = 0.0) -> CommunicationEstimate:
    items: list[CollectiveCost] = []
    per_node = intra_node.ranks_per_group

    def add(label: str, kind: str, payload: float, ranks: int, count: int, overlap: float = 0.0) -> None:
        if ranks <= 1 or count <= 0 or payload <= 0:
            return
        tier = intra_node if ranks <= per_node else inter_node
        wire = _wire(kind, payload, ranks)
        items.append(CollectiveCost(label, kind, payload, wire, ranks, count, tier.name,
                                    tier.transfer_seconds(wire) * count, overlap * count))

    per_block = shape.parameters / max(1, shape.depth)
    depth = max(1, shape.depth // max(1, dims.pipeline))
    seq = shape.sequence_length / max(1, dims.sequence_shard_size)
    if dims.cp_enabled:
        head_dim = shape.width // max(1, shape.num_heads)
        kv = shape.micro_batch_size * seq * shape.num_heads * head_dim * 2.0 * param_dtype_bytes / max(1, dims.tensor)
        # K/V of the other shards in, dK/dV partials out: (cp - 1) shards each way per layer
        full_payload = kv * dims.context
        add("context_parallel.ring_kv", "all_gather", full_payload, dims.context, depth,
            overlap=attention_seconds_per_layer)
        add("context_parallel.ring_dkv", "reduce_scatter", full_payload * 2.0, dims.context, depth,
            overlap=attention_seconds_per_layer * 2.5)
    if dims.dp_shard_enabled:
        ranks = dims.dp_shard * dims.context
        add("fsdp.all_gather", "all_gather", per_block * param_dtype_bytes / max(1, dims.tensor), ranks, depth * 2)
        add("fsdp.reduce_scatter", "reduce_scatter", per_block * reduce_dtype_bytes / max(1, dims.tensor), ranks,
            depth)
    elif dims.cp_enabled:
        local = shape.parameters / max(1, dims.tensor * dims.pipeline)
        add("data_parallel.all_reduce", "all_reduce", local * reduce_dtype_bytes, dims.context, 1)
    if dims.dp_replicate_enabled:
        local = shape.parameters / max(1, dims.dp_shard * dims.context * dims.tensor * dims.pipeline)
        add("hsdp.all_reduce", "all_reduce", local * reduce_dtype_bytes, dims.dp_replicate, 1)
    if dims.tp_enabled:
        act = shape.micro_batch_size * seq * shape.width * param_dtype_bytes
        add("tensor_parallel.activation", "reduce_scatter" if dims.sequence_shard_size > 1 else "all_reduce", act,
            dims.tensor, depth * 4)
    if dims.pp_enabled:
        boundary = shape.micro_batch_size * seq * shape.width * param_dtype_bytes
        add("pipeline.p2p", "all_gather", boundary, 2, dims.pipeline - 1)
    if dims.cp_enabled and compute_seconds > 0:
        # The ring's per-block barriers (K/V readiness before each block's attention,
        # dK/dV arrival after its backward) wait for the slowest rank of the ranks that
        # step together: the expected maximum of their block-time jitter.
        ranks = dims.context * (dims.dp_shard if dims.dp_shard_enabled else 1)
        per_block_seconds = compute_seconds / depth
        wait = RING_SKEW_FRACTION * per_block_seconds * expected_max_normal(ranks)
        items.append(CollectiveCost("context_parallel.rank_skew", "barrier", 0.0, 0.0, ranks, 2 * depth,
                                    intra_node.name, wait * 2 * depth, synchronising=True))
    return CommunicationEstimate(tuple(items), compute_seconds, overlap_efficiency)


# Standard deviation of one block's time across ranks, as a fraction of the block
# time, fitted to the barrier waits this framework measured on B200 at cp=2 and at
# dp_shard 2 x cp 4 (``measured_b200.json``).
RING_SKEW_FRACTION = 0.013

@functools.lru_cache(maxsize=256)
def expected_max_normal(n: int) -> float:
    """Expected maximum of ``n`` independent standard normal draws,
    ``integral x n phi(x) Phi(x)^(n-1) dx``, by the trapezoid rule on [-9, 9]
    (0 for n <= 1; 0.5642 for 2, 1.0294 for 4, 1.4236 for 8)."""
    if n <= 1:
        return 0.0
    steps, lo, hi = 6000, -9.0, 9.0
    h = (hi - lo) / steps
    total = 0.0
    for i in range(steps + 1):
        x = lo + i * h
        pdf = math.exp(-0.5 * x * x) / math.sqrt(2.0 * math.pi)
        cdf = 0.5 * (1.0 + math.erf(x / math.sqrt(2.0)))
        w = 0.5 if i in (0, steps) else 1.0
        total += w * x * n * pdf * cdf ** (n - 1)
    return total * h


def count_collectives(step: Callable[[], Any], *, trace_file: str | None = None) -> dict[str, Any]:
    """Collectives issued by ``step`` per module (``CommDebugMode``)."""
    from torch.distributed.tensor.debug import CommDebugMode

    mode = CommDebugMode()
    with mode:
        step()
    out: dict[str, Any] = {"total_counts": {str(k): v for k, v in mode.get_total_counts().items()}
                           if callable(getattr(mode, "get_total_counts", None)) else {},
                           "module_counts": {str(m): {str(op): n for op, n in ops.items()}
                                             for m, ops in mode.get_comm_counts().items()}}
    with contextlib.suppress(Exception):
        out["sharding"] = {str(k): str(v) for k, v in mode.get_sharding_info().items()}
    if trace_file is not None:
        mode.log_comm_debug_tracing_table_to_file(file_name=trace_file)
        out["trace_file"] = trace_file
    return out
