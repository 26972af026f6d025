"""Checkpoint: DCP save/resume reproduces the next step; markers; retention; export round trip."""
from __future__ import annotations

import json

import torch

from avgen_b200.checkpoint import CheckpointManager, convert, export_safetensors, import_safetensors
from avgen_b200.core import RNGStreams, TrainState
from avgen_b200.data.synthetic_batch import random_batch
from avgen_b200.models import build_model
from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, ShardedEMA,
                              build_optimizer, build_schedule, build_timestep_sampler, train_step)

TINY = {"width": 64, "depth": 2, "num_heads": 4, "ffn_hidden": 128, "in_channels": 4, "text_width": 32,
        "text_context_length": 8, "cond_width": 64, "time_frequency_dim": 32}


def _state(seed: int = 0) -> TrainState:
    torch.manual_seed(seed)
    model = build_model("video_dit", TINY)
    model.init_weights()
    torch.nn.init.normal_(model.final_proj.weight, std=0.02)
    opt = build_optimizer(model, lr=1e-3, weight_decay=0.01, fused=True)
    return TrainState(model=model, optimizer=opt, rng=RNGStreams.from_seed(0),
                      schedule=build_schedule("cosine", opt, total_steps=100, warmup_steps=2),
                      ema=ShardedEMA(model, decay=0.9, optimizer=opt))


def _step(state: TrainState) -> float:
    batch = random_batch(batch=2, channels=4, frames=2, height=8, width=8, text_tokens=8, text_width=32,
                         generator=torch.Generator().manual_seed(state.step))
    obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    _, m = train_step(state, batch, obj, patchifier=state.model.patchifier, max_grad_norm=1.0)
    return m.to_mapping()["loss"]


def test_resume_reproduces_next_step(tmp_path) -> None:
    a = _state()
    _step(a)
    _step(a)
    mgr = CheckpointManager(tmp_path, keep_last_n=2)
    mgr.save(a.step, a, async_save=False)
    want = _step(a)
    b = _state(seed=123)
    assert mgr.load(b) == 2
    assert b.step == 2
    got = _step(b)
    assert abs(got - want) < 1e-5, (got, want)
    marker = json.loads((tmp_path / "step_0000000002" / "avgen_checkpoint.json").read_text())
    assert marker["format_version"] == 1 and "model_optimizer" in marker["keys"] and "ema" in marker["keys"]


def test_retention_and_unmarked_dirs(tmp_path) -> None:
    s = _state()
    mgr = CheckpointManager(tmp_path, keep_last_n=2)
    (tmp_path / "step_0000000000").mkdir(parents=True)  # an interrupted save: no marker
    for _ in range(4):
        _step(s)
        mgr.save(s.step, s, async_save=True)
    mgr.close()
    steps = [e.step for e in mgr.list_checkpoints()]
    assert steps == [3, 4]
    assert not (tmp_path / "step_0000000000").exists()


def test_export_import_and_convert(tmp_path) -> None:
    s = _state()
    export_safetensors(tmp_path / "export", s.model, max_shard_bytes=40_000)
    index = json.loads((tmp_path / "export" / "model.safetensors.index.json").read_text())
    assert len(set(index["weight_map"].values())) > 1
    other = _state(seed=7)
    import_safetensors(tmp_path / "export", other.model)
    for (n, p), (_, q) in zip(s.model.named_parameters(), other.model.named_parameters()):
        torch.testing.assert_close(p, q, msg=n)
    mgr = CheckpointManager(tmp_path / "ck")
    mgr.save(0, s, async_save=False)
    convert(tmp_path / "ck" / "step_0000000000", tmp_path / "conv", to="safetensors")
    third = _state(seed=9)
    import_safetensors(tmp_path / "conv", third.model)
    torch.testing.assert_close(third.model.final_proj.weight, s.model.final_proj.weight)
