"""Single-process checks of the parallel library: plans, pipeline splits, precision, simulator."""
from __future__ import annotations

import pytest
import torch

from avgen_b200.parallel import (ActivationCheckpointConfig, ParallelDims, PipelineConfig, PrecisionConfig,
                                 balanced_split_points, split_model, standard_block_plan)


def test_balanced_split_points_minimise_the_bottleneck() -> None:
    assert balanced_split_points(32, 4) == [8, 16, 24]
    assert balanced_split_points(10, 3) == [3, 7]
    assert balanced_split_points(4, 1) == []
    pts = balanced_split_points(8, 8)
    assert pts == list(range(1, 8))
    with pytest.raises(ValueError):
        balanced_split_points(3, 4)


def test_pipeline_config_and_split_model() -> None:
    from dataclasses import asdict

    from avgen_b200.models import build_model, preset

    cfg = PipelineConfig(schedule="1f1b", microbatches=8)
    assert cfg.bubble_fraction(4) == pytest.approx(3 / 11)
    with pytest.raises(ValueError):
        PipelineConfig(schedule="1f1b", stages_per_rank=2)
    m = build_model("video_dit", {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"})
    n = len(m.blocks)
    first = split_model(m, stage_index=0, num_stages=2, split_points=[n // 2])
    assert len(first.blocks) == n // 2 and first.final_proj is None and first.patch_embed is not None


def test_block_plan_and_precision() -> None:
    plan = standard_block_plan(cross_attention_prefix=None, ffn_projections=("up_proj",))
    assert "attention.q_proj" in plan and "feed_forward.up_proj" in plan and "feed_forward.gate_proj" not in plan
    with pytest.raises(NotImplementedError):
        standard_block_plan(sequence_parallel=True)
    p = PrecisionConfig()
    assert p.param is torch.bfloat16 and p.reduce is torch.float32
    assert p.fsdp_policy().cast_forward_inputs is False
    with pytest.raises(KeyError):
        PrecisionConfig(param_dtype="int8")  # type: ignore[arg-type]
    with pytest.raises(ValueError):
        PrecisionConfig(float8_min_features=0)
    assert PrecisionConfig(param_dtype="float32").autocast_dtype() is None


def test_float8_targets_skip_small_unaligned_and_kept_linears() -> None:
    model = torch.nn.ModuleDict({"patch_embed": torch.nn.Linear(2048, 2048), "big": torch.nn.Linear(2048, 4096),
                                 "small": torch.nn.Linear(512, 2048), "odd": torch.nn.Linear(2048, 2050),
                                 "final_proj": torch.nn.Linear(2048, 2048)})
    assert PrecisionConfig().float8_targets(model) == ["big"]
    assert PrecisionConfig(float8_min_features=256, float8_exclude=()).float8_targets(model) == [
        "patch_embed", "big", "small", "final_proj"]


def test_activation_policies_preserve_checkpoint_keys() -> None:
    from dataclasses import asdict

    from avgen_b200.models import build_model, preset
    from avgen_b200.parallel import apply_activation_checkpointing

    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    ref = build_model("video_dit", cfg)
    keys = set(ref.state_dict())
    for mode in ("full", "selective_op", "selective_layer"):
        m = build_model("video_dit", cfg)
        apply_activation_checkpointing(m, ActivationCheckpointConfig(mode=mode))
        assert set(m.state_dict()) == keys
        m.load_state_dict(ref.state_dict())
    assert not ActivationCheckpointConfig(mode="fused").enabled


def test_simulator_plans_for_b200() -> None:
    from avgen_b200.simulate import B200, ModelShape, SearchSpace, search_parallel_plan, simulate_config

    shape = ModelShape(parameters=4_200_000_000, depth=32, width=2560, sequence_length=65536, num_heads=20,
                       text_tokens=512)
    report = simulate_config(shape, ParallelDims(world_size=8, dp_shard=2, context=4))
    d = report.to_dict()
    assert d["fits"] and 0 < d["mfu"] < 1 and d["comm_bottleneck"].startswith(("context", "fsdp"))
    plans = search_parallel_plan(shape, SearchSpace(world_size=8))
    assert plans and all(p.memory.total_gib < B200.memory_gib for p in plans)
    report.assert_no_regression(d)
    with pytest.raises(AssertionError):
        report.assert_no_regression({**d, "mfu": d["mfu"] * 2})
