"""Configuration and the analytic simulator on CPU: YAML ``_base_`` composition,
``${env:...}`` interpolation, dotted overrides with list indices, fatal unknown
keys, config diffs; parallel dims (mesh order, inference, data and sequence
coordinates) and the mesh built at large world sizes on the fake process group;
memory / compute / comms estimates and plan search (reference test strategy:
tests/test_config.py, tests/test_simulate.py, tests/test_distributed_stress.py)."""
from __future__ import annotations

import multiprocessing as mp
from pathlib import Path

import pytest

from avgen_b200.config import load_config
from avgen_b200.config.diff import config_diff
from avgen_b200.config.loader import ConfigError, apply_overrides, deep_merge, parse_override
from avgen_b200.parallel.dims import ParallelDims


def test_base_composition_env_and_overrides(tmp_path: Path, monkeypatch: pytest.MonkeyPatch) -> None:
    base = tmp_path / "base.yaml"
    base.write_text("model:\n  depth: 4\n  width: 64\n  num_heads: 2\ntrain:\n  lr: 0.001\n  steps: 10\n  warmup_steps: 1\n"
                    "data:\n  buckets: [{name: a, frames: 2, height: 8, width: 8}, {name: b, frames: 4, height: 8, width: 8}]\n")
    child = tmp_path / "run.yaml"
    child.write_text("_base_: base.yaml\nmodel:\n  depth: 6\ntrain:\n  steps: ${env:AVGEN_TEST_STEPS:7}\n"
                     "run_name: ${env:AVGEN_TEST_NAME:fallback}\n")
    monkeypatch.setenv("AVGEN_TEST_STEPS", "12")
    cfg = load_config(child, ["train.lr=0.01", "data.buckets[1].frames=8"])
    assert cfg.model.depth == 6 and cfg.model.width == 64  # child overrides, base fills
    assert cfg.train.steps == 12 and isinstance(cfg.train.steps, int)  # env value coerced by annotation
    assert cfg.run_name == "fallback"
    assert cfg.train.lr == pytest.approx(0.01)
    assert cfg.data.buckets[1].frames == 8 and cfg.data.buckets[0].frames == 2


def test_unknown_keys_and_bad_values_are_fatal() -> None:
    with pytest.raises((ConfigError, ValueError, KeyError)) as err:
        load_config(None, ["model.dpeth=3"])
    assert "dpeth" in str(err.value)
    with pytest.raises((ConfigError, ValueError)):
        load_config(None, ["train.steps=-1"])
    with pytest.raises((ConfigError, ValueError)):
        load_config(None, ["train.lr=fast"])


def test_override_parsing_merge_and_diff() -> None:
    path, value = parse_override("data.buckets[0].frames=16")
    assert path == ["data", "buckets", 0, "frames"] and value == 16
    merged = deep_merge({"a": {"b": 1, "l": [1, 2]}}, {"a": {"c": 2, "l": [3]}})
    assert merged == {"a": {"b": 1, "c": 2, "l": [3]}}  # lists replace
    out = apply_overrides({"train": {"lr": 0.1}}, ["train.lr=0.2", "train.betas=[0.9, 0.95]"])
    assert out["train"]["lr"] == 0.2 and out["train"]["betas"] == [0.9, 0.95]
    a = load_config(None, ["train.lr=0.001"])
    b = load_config(None, ["train.lr=0.002", "model.depth=3"])
    d = config_diff(a, b)
    assert "train.lr" in d and "model.depth" in d and d["train.lr"] == (0.001, 0.002)


@pytest.mark.parametrize("world,kw,expect", [
    (8, {"context": 4}, {"dp_shard": 2}),
    (16, {"dp_replicate": 2, "context": 2, "tensor": 2}, {"dp_shard": 2}),
    (512, {"dp_replicate": 8, "context": 4, "tensor": 8}, {"dp_shard": 2}),
    (4096, {"dp_replicate": 4, "context": 8, "tensor": 8, "pipeline": 2}, {"dp_shard": 8}),
])
def test_parallel_dims_inference(world: int, kw: dict, expect: dict) -> None:
    d = ParallelDims(world_size=world, **kw)
    for k, v in expect.items():
        assert getattr(d, k) == v
    names = [n for n, _ in d.active_dims]
    order = ("pp", "dp_replicate", "dp_shard", "cp", "tp")
    assert names == [n for n in order if n in names]
    with pytest.raises(ValueError):
        ParallelDims(world_size=world + 1, **kw)


def _mesh_probe(world: int, kw: dict, rank: int) -> tuple:
    from avgen_b200.simulate.world import fake_world

    dims = ParallelDims(world_size=world, **kw)
    with fake_world(dims, rank=rank, device_type="cpu") as w:
        mesh = w.mesh
        return (tuple(mesh.mesh_dim_names), tuple(mesh.shape), dims.data_coordinates(mesh),
                dims.sequence_coordinates(mesh))


@pytest.mark.parametrize("world,kw,rank", [(64, {"dp_replicate": 2, "context": 4, "tensor": 2}, 37),
                                           (1024, {"dp_replicate": 8, "context": 8, "tensor": 4}, 1000)])
def test_fake_world_mesh_and_coordinates(world: int, kw: dict, rank: int) -> None:
    ctx = mp.get_context("spawn")
    with ctx.Pool(1) as pool:
        names, shape, (data_rank, data_world), (seq_rank, seq_world) = pool.apply(_mesh_probe, (world, kw, rank))
    dims = ParallelDims(world_size=world, **kw)
    assert names == tuple(n for n in ("pp", "dp_replicate", "dp_shard", "cp", "tp") if n in names)
    assert int(__import__("math").prod(shape)) == world
    assert data_world == dims.dp_replicate * dims.dp_shard and 0 <= data_rank < data_world
    assert seq_world == dims.context and 0 <= seq_rank < seq_world
    # ranks that differ only in cp / tp see the same data; the cp index is the sequence shard
    _, _, (data_rank2, _), (seq_rank2, _) = _mesh_probe_pair(world, kw, rank)
    assert data_rank2 == data_rank and seq_rank2 != seq_rank


def _mesh_probe_pair(world: int, kw: dict, rank: int) -> tuple:
    tp = kw.get("tensor", 1)
    ctx = mp.get_context("spawn")
    with ctx.Pool(1) as pool:  # the neighbouring cp index of the same data shard
        other = rank + tp if (rank // tp) % kw.get("context", 1) + 1 < kw.get("context", 1) else rank - tp
        return pool.apply(_mesh_probe, (world, kw, other))


def test_simulator_estimates_and_plan_search() -> None:
    from avgen_b200.simulate import B200, H100_SXM, ModelShape, SearchSpace, search_parallel_plan, simulate_config

    shape = ModelShape(parameters=4_252_429_888, depth=32, width=2560, sequence_length=65536, num_heads=20,
                       text_tokens=512)
    one = simulate_config(shape, ParallelDims(world_size=1))
    cp4 = simulate_config(shape, ParallelDims(world_size=8, dp_shard=2, context=4))
    assert cp4.memory.total_gib < one.memory.total_gib  # activations shard over cp, states over dp_shard x cp
    assert 0.0 < cp4.mfu < 1.0 and cp4.fits
    slow = simulate_config(shape, ParallelDims(world_size=8, dp_shard=2, context=4), accelerator=H100_SXM)
    assert slow.step_seconds > cp4.step_seconds  # B200 predicts a faster step than H100
    d = cp4.to_dict()
    assert {"plan", "memory_gib", "mfu", "scaling_efficiency", "comm_by_label_seconds"} <= set(d)
    plans = search_parallel_plan(shape, SearchSpace(world_size=8), accelerator=B200)
    assert plans and all(p.memory.fits_in(B200.memory_gib) for p in plans[:3])
