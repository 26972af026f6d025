"""Checkpoint manager, model-only / EMA loads and export paths on CPU
(reference test strategy: tests/test_checkpoint*.py -- directory naming,
retention rules, explicit-step loads, format guards, marker contents, model
and EMA restores, export dtype / sharding / metadata, conversions)."""
from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from avgen_b200.checkpoint import CheckpointManager, convert, export_safetensors, import_safetensors
from avgen_b200.checkpoint.export import export_huggingface, read_safetensors_dir
from avgen_b200.checkpoint.manager import _parse_step, load, load_ema, load_model, save, step_dirname
from avgen_b200.core import RNGStreams, TrainState
from avgen_b200.data.synthetic_batch import random_batch
from avgen_b200.models import build_model
from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, ShardedEMA,
                              build_optimizer, build_schedule, build_timestep_sampler, train_step)

TINY = {"width": 64, "depth": 2, "num_heads": 4, "ffn_hidden": 128, "in_channels": 4, "text_width": 32,
        "text_context_length": 8, "cond_width": 64, "time_frequency_dim": 32}


def _state(seed: int = 0, *, ema: bool = True) -> TrainState:
    torch.manual_seed(seed)
    model = build_model("video_dit", TINY)
    model.init_weights()
    torch.nn.init.normal_(model.final_proj.weight, std=0.02)
    opt = build_optimizer(model, lr=1e-3, weight_decay=0.01, fused=True)
    return TrainState(model=model, optimizer=opt, rng=RNGStreams.from_seed(0),
                      schedule=build_schedule("cosine", opt, total_steps=100, warmup_steps=2),
                      ema=ShardedEMA(model, decay=0.5, optimizer=opt) if ema else None)


def _step(state: TrainState) -> float:
    batch = random_batch(batch=2, channels=4, frames=2, height=8, width=8, text_tokens=8, text_width=32,
                         generator=torch.Generator().manual_seed(state.step))
    obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    _, m = train_step(state, batch, obj, patchifier=state.model.patchifier, max_grad_norm=1.0)
    return m.to_mapping()["loss"]


@pytest.mark.parametrize("step", [0, 1, 42, 10**9])
def test_step_dirname_round_trip(step: int) -> None:
    name = step_dirname(step)
    assert _parse_step(name) == step and len(name) == len(step_dirname(0))


@pytest.mark.parametrize("name", ["step_abc", "ckpt_0000000001", "step_", "step_-1", "step_12a"])
def test_parse_step_rejects_foreign_names(name: str) -> None:
    assert _parse_step(name) is None


@pytest.mark.parametrize("kw", [{"keep_last_n": -1}, {"keep_every_n_steps": -1}, {"save_timeout_s": 0.0},
                                {"thread_count": 0}])
def test_manager_rejects_bad_settings(tmp_path: Path, kw: dict) -> None:
    with pytest.raises(ValueError):
        CheckpointManager(tmp_path, **kw)


def test_manager_rejects_negative_step(tmp_path: Path) -> None:
    with pytest.raises(ValueError):
        CheckpointManager(tmp_path).save(-1, _state(), async_save=False)


@pytest.mark.parametrize("keep_last,keep_every,expect", [(1, 0, [6]), (2, 0, [5, 6]), (1, 2, [2, 4, 6]),
                                                         (0, 0, [1, 2, 3, 4, 5, 6]), (2, 3, [3, 5, 6])])
def test_retention_rules(tmp_path: Path, keep_last: int, keep_every: int, expect: list[int]) -> None:
    s = _state(ema=False)
    mgr = CheckpointManager(tmp_path, keep_last_n=keep_last, keep_every_n_steps=keep_every)
    for step in range(1, 7):
        mgr.save(step, s, async_save=False)
    assert [e.step for e in mgr.list_checkpoints()] == expect
    assert mgr.latest_step() == 6


def test_empty_root_and_explicit_step_loads(tmp_path: Path) -> None:
    mgr = CheckpointManager(tmp_path / "none")
    assert mgr.load(_state()) is None and mgr.latest_step() is None and mgr.list_checkpoints() == ()
    s = _state()
    mgr = CheckpointManager(tmp_path / "ck", keep_last_n=0)
    _step(s)
    mgr.save(s.step, s, async_save=False)
    first = {n: p.detach().clone() for n, p in s.model.named_parameters()}
    _step(s)
    mgr.save(s.step, s, async_save=False)
    fresh = _state(seed=5)
    assert mgr.load(fresh, step=1) == 1
    for n, p in fresh.model.named_parameters():
        torch.testing.assert_close(p, first[n], msg=n)
    assert fresh.step == 1
    with pytest.raises(FileNotFoundError):
        mgr.load(fresh, step=7)


def test_newer_format_and_unreadable_marker_are_handled(tmp_path: Path) -> None:
    s = _state(ema=False)
    mgr = CheckpointManager(tmp_path, keep_last_n=0)
    d = mgr.save(0, s, async_save=False)
    marker = d / "avgen_checkpoint.json"
    meta = json.loads(marker.read_text())
    meta["format_version"] = 99
    marker.write_text(json.dumps(meta))
    with pytest.raises(ValueError, match="newer format"):
        mgr.load(_state(ema=False))
    marker.write_text("{broken")
    assert mgr.list_checkpoints() == ()  # an unreadable marker is skipped, not trusted


def test_marker_records_progress_keys_and_extras(tmp_path: Path) -> None:
    s = _state()
    _step(s)
    d = save(tmp_path, s, async_save=False, extras={"note": "x", "tokens_seen": 123})
    meta = json.loads((d / "avgen_checkpoint.json").read_text())
    assert meta["step"] == 1 and meta["world_size"] == 1 and meta["data_world"] == 1
    assert meta["extras"] == {"note": "x", "tokens_seen": 123}
    assert {"model_optimizer", "ema"} <= set(meta["keys"])
    assert meta["progress"]["step"] == 1 and "completed_at" in meta
    assert not list(d.glob(".*.tmp"))


def test_async_save_waits_before_the_next_save_and_on_close(tmp_path: Path) -> None:
    s = _state(ema=False)
    with CheckpointManager(tmp_path, keep_last_n=0) as mgr:
        mgr.save(0, s, async_save=True)
        assert mgr.has_pending_save
        mgr.save(1, s, async_save=True)  # finalises step 0 first
        assert [e.step for e in mgr.list_checkpoints()] == [0]
    assert [e.step for e in CheckpointManager(tmp_path).list_checkpoints()] == [0, 1]


def test_module_level_save_load(tmp_path: Path) -> None:
    s = _state()
    _step(s)
    save(tmp_path, s, async_save=False)
    other = _state(seed=3)
    assert load(tmp_path, other) == 1
    for (n, p), (_, q) in zip(s.model.named_parameters(), other.model.named_parameters()):
        torch.testing.assert_close(p, q, msg=n)


def test_load_model_only_and_errors(tmp_path: Path) -> None:
    s = _state()
    _step(s)
    d = save(tmp_path, s, async_save=False)
    model = build_model("video_dit", TINY)
    load_model(d, model)
    for (n, p), (_, q) in zip(s.model.named_parameters(), model.named_parameters()):
        torch.testing.assert_close(p, q, msg=n)
    with pytest.raises(FileNotFoundError):
        load_model(tmp_path / "missing", model)
    wrong = build_model("video_dit", dict(TINY, width=32, num_heads=2, cond_width=32))
    with pytest.raises(RuntimeError):
        load_model(d, wrong)


def test_load_ema_restores_the_shadow(tmp_path: Path) -> None:
    s = _state()
    for _ in range(3):
        _step(s)
    d = save(tmp_path, s, async_save=False)
    model = build_model("video_dit", TINY)
    load_ema(d, model, decay=0.5)
    shadow = ShardedEMA(build_model("video_dit", TINY), decay=0.5)
    shadow_state = s.ema.state_dict()
    shadow.load_state_dict(shadow_state)
    reference = build_model("video_dit", TINY)
    shadow.copy_to(reference)
    for (n, p), (_, q) in zip(reference.named_parameters(), model.named_parameters()):
        torch.testing.assert_close(p, q, msg=n)
    # the EMA differs from the live weights after a few steps with decay 0.5
    assert any(not torch.allclose(p, q) for p, q in zip(s.model.parameters(), model.parameters()))
    with pytest.raises(FileNotFoundError):
        load_ema(tmp_path / "missing", model)


@pytest.mark.parametrize("dtype", [None, torch.bfloat16, torch.float16])
def test_export_dtype_and_round_trip(tmp_path: Path, dtype: torch.dtype | None) -> None:
    s = _state(ema=False)
    export_safetensors(tmp_path / "e", s.model, dtype=dtype)
    tensors = read_safetensors_dir(tmp_path / "e")
    assert set(tensors) == set(dict(s.model.named_parameters())) | set(dict(s.model.named_buffers())) or \
        set(dict(s.model.named_parameters())) <= set(tensors)
    for name, p in s.model.named_parameters():
        assert tensors[name].dtype == (dtype or p.dtype)
        torch.testing.assert_close(tensors[name].float(), p.detach().to(dtype or p.dtype).float())


@pytest.mark.parametrize("shard_bytes", [10_000, 100_000, 10**9])
def test_export_sharding_index(tmp_path: Path, shard_bytes: int) -> None:
    s = _state(ema=False)
    export_safetensors(tmp_path / "e", s.model, max_shard_bytes=shard_bytes)
    files = sorted(p.name for p in (tmp_path / "e").glob("*.safetensors"))
    index_path = tmp_path / "e" / "model.safetensors.index.json"
    if len(files) > 1:
        index = json.loads(index_path.read_text())
        assert set(index["weight_map"].values()) == set(files)
        assert set(index["weight_map"]) == set(read_safetensors_dir(tmp_path / "e"))
    other = _state(seed=2, ema=False)
    import_safetensors(tmp_path / "e", other.model)
    for (n, p), (_, q) in zip(s.model.named_parameters(), other.model.named_parameters()):
        torch.testing.assert_close(p, q, msg=n)


def test_export_rejects_and_import_strictness(tmp_path: Path) -> None:
    s = _state(ema=False)
    with pytest.raises(ValueError):
        export_safetensors(tmp_path / "e", s.model, max_shard_bytes=0)
    with pytest.raises(FileNotFoundError):
        read_safetensors_dir(tmp_path / "nothing")
    export_safetensors(tmp_path / "e", s.model)
    bigger = build_model("video_dit", dict(TINY, depth=3))
    with pytest.raises(RuntimeError):
        import_safetensors(tmp_path / "e", bigger)
    import_safetensors(tmp_path / "e", bigger, strict=False)  # the shared prefix loads


def test_export_huggingface_layout(tmp_path: Path) -> None:
    s = _state(ema=False)
    export_huggingface(tmp_path / "hf", s.model)
    files = {p.name for p in (tmp_path / "hf").iterdir()}
    assert any(f.endswith(".safetensors") for f in files)
    tensors = read_safetensors_dir(tmp_path / "hf")
    for name, p in s.model.named_parameters():
        torch.testing.assert_close(tensors[name], p.detach(), msg=name)


def test_convert_to_dcp_and_back(tmp_path: Path) -> None:
    s = _state(ema=False)
    save(tmp_path / "ck", s, async_save=False)
    src = tmp_path / "ck" / step_dirname(0)
    convert(src, tmp_path / "st", to="safetensors")
    convert(tmp_path / "st", tmp_path / "dcp", to="dcp")
    model = build_model("video_dit", TINY)
    load_model(tmp_path / "dcp", model)
    for (n, p), (_, q) in zip(s.model.named_parameters(), model.named_parameters()):
        torch.testing.assert_close(p, q, msg=n)
    with pytest.raises(ValueError):
        convert(src, tmp_path / "x", to="onnx")
