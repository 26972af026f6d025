"""The analytic simulator's models on CPU, by their invariants: memory falls
with sharding and rises with the kept activations, FLOP counts scale as the
formulas say, collective wire bytes follow ring algebra, overlap only hides what
compute covers, and the plan search returns valid, ranked layouts (reference
test strategy: tests/test_simulate*.py -- monotonicity, closed forms, ranking)."""
from __future__ import annotations

import math

import pytest

from avgen_b200.parallel.activation import ActivationCheckpointConfig
from avgen_b200.parallel.dims import ParallelDims
from avgen_b200.simulate.comms import (NVLINK4, NVLINK5, CollectiveCost, CommunicationEstimate, Interconnect,
                                       _wire, calibrate_from_busbw, estimate_step_communication)
from avgen_b200.simulate.compute import B200, H100_SXM, estimate_compute, suggest_activation_policy, transformer_flops
from avgen_b200.simulate.memory import OPTIMIZER_BYTES, ModelShape, estimate_memory
from avgen_b200.simulate.plan import SearchSpace, render_plan_table, search_parallel_plan

SHAPE_2B = ModelShape(parameters=4_252_429_888, depth=32, width=2560, sequence_length=65536, num_heads=20,
                      text_tokens=512)
SMALL = ModelShape(parameters=300_000_000, depth=24, width=1024, sequence_length=4096, num_heads=8)


def _dims(world: int = 8, **kw) -> ParallelDims:  # noqa: ANN003
    return ParallelDims(world_size=world, **kw)


# ----------------------------------------------------------------------------- memory


@pytest.mark.parametrize("shard", [1, 2, 4, 8])
def test_parameter_state_memory_falls_with_sharding(shard: int) -> None:
    one = estimate_memory(SMALL, _dims(1))
    many = estimate_memory(SMALL, _dims(shard, dp_shard=shard))
    assert many.parameter_bytes == pytest.approx(one.parameter_bytes / shard)
    assert many.optimizer_bytes == pytest.approx(one.optimizer_bytes / shard)
    assert many.gradient_bytes == pytest.approx(one.gradient_bytes / shard)
    if shard > 1:
        assert many.gather_bytes > 0  # FSDP holds gathered blocks
    else:
        assert many.gather_bytes == 0


@pytest.mark.parametrize("optimizer", sorted(OPTIMIZER_BYTES))
def test_optimizer_state_bytes_per_parameter(optimizer: str) -> None:
    est = estimate_memory(SMALL, _dims(1), optimizer=optimizer)
    assert est.optimizer_bytes == pytest.approx(SMALL.parameters * OPTIMIZER_BYTES[optimizer])


def test_unknown_optimizer_rejected() -> None:
    with pytest.raises(KeyError):
        estimate_memory(SMALL, _dims(1), optimizer="lion")


def test_activation_policies_order() -> None:
    acts = {m: estimate_memory(SHAPE_2B, _dims(1), policy=m).activation_bytes
            for m in ("none", "selective_layer", "full", "fused")}
    assert acts["none"] > acts["selective_layer"] > acts["full"]
    assert acts["fused"] < acts["none"]
    f1 = estimate_memory(SHAPE_2B, _dims(1), activation_checkpoint=ActivationCheckpointConfig(
        mode="selective_op", save_op_frequency=1)).activation_bytes
    f2 = estimate_memory(SHAPE_2B, _dims(1), activation_checkpoint=ActivationCheckpointConfig(
        mode="selective_op", save_op_frequency=2)).activation_bytes
    assert acts["none"] > f1 > f2 > acts["full"]


@pytest.mark.parametrize("cp", [1, 2, 4, 8])
def test_context_parallel_divides_activation_memory(cp: int) -> None:
    base = estimate_memory(SHAPE_2B, _dims(1), policy="none").activation_bytes
    sharded = estimate_memory(SHAPE_2B, _dims(cp, context=cp, dp_shard=1), policy="none").activation_bytes
    assert sharded == pytest.approx(base / cp, rel=0.02)


def test_memory_estimate_helpers() -> None:
    est = estimate_memory(SHAPE_2B, _dims(1), policy="none")
    assert est.total_gib == pytest.approx(est.total_bytes / 1024 ** 3)
    parts = est.breakdown_gib()
    assert list(parts.values()) == sorted(parts.values(), reverse=True)
    assert est.dominant_term() == next(iter(parts))
    assert not est.fits_in(80.0) and est.fits_in(est.total_gib * 2, headroom=0.1)


def test_memory_matches_the_measured_flagship_roughly() -> None:
    # the 2B model at 64k tokens on one B200 keeps fused activations: measured peak 172 GiB
    est = estimate_memory(SHAPE_2B, _dims(1), policy="fused")
    assert 60.0 < est.total_gib < 178.0


def test_shape_hidden_defaults() -> None:
    assert SMALL.hidden == 4 * 1024
    assert ModelShape(parameters=1, depth=1, width=64, sequence_length=1, ffn_hidden=100).hidden == 100


# ----------------------------------------------------------------------------- compute


def test_flop_formulas() -> None:
    f = transformer_flops(SMALL, include_backward=False)
    s, w, d = SMALL.sequence_length, SMALL.width, SMALL.depth
    assert f["projections"] == pytest.approx(d * 8 * s * w * w)
    assert f["attention"] == pytest.approx(d * 4 * s * s * w)
    assert f["feed_forward"] == pytest.approx(d * 6 * s * w * SMALL.hidden)
    assert f["cross_attention"] == 0.0
    train = transformer_flops(SMALL)
    assert train["total"] == pytest.approx(3 * f["total"])
    assert f["head_dim"] == 128


@pytest.mark.parametrize("factor", [2, 4])
def test_attention_flops_are_quadratic_in_length(factor: int) -> None:
    from dataclasses import replace

    a = transformer_flops(SMALL)
    b = transformer_flops(replace(SMALL, sequence_length=SMALL.sequence_length * factor))
    assert b["attention"] == pytest.approx(a["attention"] * factor * factor)
    assert b["projections"] == pytest.approx(a["projections"] * factor)
    assert b["attention_fraction"] > a["attention_fraction"]


def test_compute_recompute_overheads() -> None:
    dims = _dims(1)
    none = estimate_compute(SHAPE_2B, dims, policy="none")
    full = estimate_compute(SHAPE_2B, dims, policy="full")
    fused = estimate_compute(SHAPE_2B, dims, policy="fused")
    # without checkpointing the only extra hardware work is the flash backward's recomputed
    # scores: 2.5x the attention forward against the 2x that model FLOPs count
    f = transformer_flops(SHAPE_2B, include_backward=False)
    lin = f["projections"] + f["feed_forward"] + f["cross_attention"]
    assert none.recompute_overhead == pytest.approx(0.5 * f["attention"] / (3 * (lin + f["attention"])))
    assert full.recompute_overhead > fused.recompute_overhead > 0
    assert full.seconds > fused.seconds > none.seconds
    assert none.model_flops == pytest.approx(full.model_flops)
    step = fused.seconds
    assert 0 < fused.mfu(step, B200.peak_flops()) <= fused.hfu(step, B200.peak_flops())


@pytest.mark.parametrize("cp,tp", [(2, 1), (4, 1), (1, 2), (2, 2)])
def test_compute_splits_over_model_parallel_ranks(cp: int, tp: int) -> None:
    one = estimate_compute(SHAPE_2B, _dims(1), policy="none")
    split = estimate_compute(SHAPE_2B, _dims(cp * tp, context=cp, tensor=tp, dp_shard=1), policy="none")
    assert split.seconds == pytest.approx(one.seconds / (cp * tp))


def test_accelerator_peaks_and_policy_suggestion() -> None:
    assert B200.peak_flops(fp8=True) == pytest.approx(2 * B200.peak_flops())
    assert B200.peak_flops(sustained=True) <= B200.peak_flops()
    assert H100_SXM.peak_flops() < B200.peak_flops()
    assert suggest_activation_policy(SMALL, _dims(1)) == "fused"
    huge = ModelShape(parameters=14_000_000_000, depth=40, width=5120, sequence_length=262144, num_heads=40)
    assert suggest_activation_policy(huge, _dims(1)) == "full"


# ----------------------------------------------------------------------------- communication


@pytest.mark.parametrize("kind,ranks,expect", [("all_reduce", 8, 2 * 7 / 8), ("all_gather", 8, 7 / 8),
                                               ("reduce_scatter", 4, 3 / 4), ("all_reduce", 2, 1.0),
                                               ("all_gather", 1, 0.0)])
def test_ring_wire_bytes(kind: str, ranks: int, expect: float) -> None:
    assert _wire(kind, 1.0, ranks) == pytest.approx(expect)


def test_interconnect_validation_and_calibration() -> None:
    with pytest.raises(ValueError):
        Interconnect("x", peak_gbps=0.0)
    with pytest.raises(ValueError):
        Interconnect("x", peak_gbps=1.0, efficiency=1.5)
    cal = calibrate_from_busbw("nvl", measured_busbw_gbps=725.0, peak_gbps=900.0)
    assert cal.efficiency == pytest.approx(725 / 900)
    assert calibrate_from_busbw("nvl", measured_busbw_gbps=1000.0, peak_gbps=900.0).efficiency == 1.0
    assert NVLINK5.transfer_seconds(1e9) < NVLINK4.transfer_seconds(1e9)
    assert NVLINK5.transfer_seconds(0) == pytest.approx(NVLINK5.latency_us * 1e-6)


def test_single_rank_has_no_collectives() -> None:
    est = estimate_step_communication(SHAPE_2B, _dims(1), compute_seconds=1.0)
    assert est.collectives == () and est.exposed_seconds == 0.0 and est.scaling_efficiency == 1.0
    assert est.bottleneck() == "none"


def test_flagship_layout_collectives() -> None:
    dims = _dims(8, dp_shard=2, context=4)
    est = estimate_step_communication(SHAPE_2B, dims, compute_seconds=7.0, attention_seconds_per_layer=0.05)
    labels = {c.label: c for c in est.collectives}
    assert {"context_parallel.ring_kv", "context_parallel.ring_dkv", "fsdp.all_gather",
            "fsdp.reduce_scatter"} <= set(labels)
    assert labels["fsdp.all_gather"].count == 2 * SHAPE_2B.depth  # forward and backward re-gather
    assert labels["fsdp.reduce_scatter"].count == SHAPE_2B.depth
    assert labels["fsdp.all_gather"].ranks == 8
    assert est.total_wire_gib > 0 and 0 < est.scaling_efficiency <= 1.0
    assert est.estimated_step_seconds >= est.compute_seconds


def test_overlap_hides_only_what_compute_covers() -> None:
    fused = CollectiveCost("ring", "all_gather", 1.0, 1.0, 4, 1, "nvl", seconds=2.0, overlappable_with=1.5)
    general = CollectiveCost("fsdp", "all_gather", 1.0, 1.0, 4, 1, "nvl", seconds=1.0)
    est = CommunicationEstimate((fused, general), compute_seconds=10.0, overlap_efficiency=0.8)
    assert est.exposed_seconds == pytest.approx(0.5 + 0.2)
    short = CommunicationEstimate((general,), compute_seconds=0.1, overlap_efficiency=1.0)
    assert short.exposed_seconds == pytest.approx(0.9)
    assert est.by_label() == {"ring": 2.0, "fsdp": 1.0} and est.bottleneck() == "ring"


@pytest.mark.parametrize("tp,sp", [(2, True), (4, True), (8, False)])
def test_tensor_parallel_activation_collectives(tp: int, sp: bool) -> None:
    dims = _dims(tp, tensor=tp, dp_shard=1)
    est = estimate_step_communication(SHAPE_2B, dims)
    (act,) = [c for c in est.collectives if c.label == "tensor_parallel.activation"]
    assert act.count == 4 * SHAPE_2B.depth and act.ranks == tp


# ----------------------------------------------------------------------------- plan search


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_search_returns_valid_ranked_layouts(world: int) -> None:
    space = SearchSpace(world_size=world, max_pipeline=1)
    plans = search_parallel_plan(SHAPE_2B, space, top_k=5)
    assert plans, "the 2B model at 64k tokens fits at every world size"
    for p in plans:
        d = p.dims
        assert d.dp_replicate * d.dp_shard * d.context * d.tensor * d.pipeline == world
        assert SHAPE_2B.sequence_length % (d.context * d.tensor) == 0
        assert p.memory.fits_in(B200.memory_gib, headroom=0.1)
        assert p.samples_per_second > 0 and 0 < p.mfu(B200) < 1
    best = max(p.samples_per_second for p in plans)
    assert plans[0].samples_per_second >= best * 0.98
    table = render_plan_table(plans, B200)
    assert table.splitlines()[0].startswith("plan") and len(table.splitlines()) == len(plans) + 2


def test_plan_search_with_global_batch_and_no_fit() -> None:
    space = SearchSpace(world_size=8, global_batch_size=8)
    plans = search_parallel_plan(SHAPE_2B, space)
    assert all(p.dims.dp_size * p.micro_batch_size * p.gradient_accumulation == 8 for p in plans)
    impossible = ModelShape(parameters=10**12, depth=100, width=16384, sequence_length=1 << 20, num_heads=128)
    assert search_parallel_plan(impossible, SearchSpace(world_size=1)) == []
    assert "No configuration fits" in render_plan_table([], B200)
    for bad in ({"world_size": 0}, {"world_size": 8, "gpus_per_node": 0}):
        with pytest.raises(ValueError):
            SearchSpace(**bad)


def test_plan_summary_keys() -> None:
    (plan, *_) = search_parallel_plan(SMALL, SearchSpace(world_size=2))
    summary = plan.summary(B200)
    for key in ("plan", "activation_checkpoint", "memory_gib", "step_seconds", "samples_per_second", "mfu",
                "scaling_efficiency", "bottleneck", "dominant_memory"):
        assert key in summary
    assert math.isfinite(summary["step_seconds"])
