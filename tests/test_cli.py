"""The ``avgen-b200`` command line end to end on CPU: plan, simulate, train (with resume),
checkpoint inspect / export, generate, data, info, and the exit codes."""
from __future__ import annotations

import json
from pathlib import Path

import pytest

from avgen_b200.cli.main import main

TINY = ["model.depth=1", "model.width=64", "model.num_heads=2", "model.in_channels=4", "data.latent_channels=4",
        "data.text_tokens=4", "data.text_width=16", "data.buckets=[{frames: 2, height: 8, width: 8}]",
        "train.warmup_steps=1", "train.global_batch_size=1", "telemetry.log_every=1",
        "telemetry.loggers=[jsonl]", "checkpoint.async_save=false"]


def test_version_usage_and_config_errors(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["--version"]) == 0
    assert "avgen-b200" in capsys.readouterr().out
    assert main([]) == 2
    assert main(["plan"]) == 2  # --world-size is required
    assert main(["train", "--dry-run", "no_such_section.key=1"]) == 3


def test_plan_and_simulate_json(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["plan", "--world-size", "8", "--gpu", "b200", "--json"]) == 0
    plans = json.loads(capsys.readouterr().out)
    assert plans and {"plan", "memory_gib", "mfu"} <= set(plans[0])
    assert main(["simulate", "--json", "--gpu", "b200", "--world-size", "8", "parallel.dp_shard=8"]) == 0
    rep = json.loads(capsys.readouterr().out)
    assert rep["world_size"] == 8 and rep["fits"]


def test_train_resume_export_generate(tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    out = tmp_path / "run"
    assert main(["train", *TINY, "train.steps=2", "checkpoint.save_every=1", f"output_dir={out}"]) == 0
    ckpts = sorted((out / "checkpoints").iterdir())
    assert [c.name for c in ckpts] == ["step_0000000001", "step_0000000002"]
    lines = (out / "metrics.jsonl").read_text().splitlines()
    assert len(lines) == 2 and json.loads(lines[-1])["step"] == 2
    # the training loop drives the metric accumulator and the throughput meter
    last = json.loads(lines[-1])
    flat = {**last, **last.get("metrics", {})}
    assert "loss" in flat and "progress/samples_seen" in flat
    assert flat["throughput/steps"] == 1 and flat["throughput/samples_per_second"] > 0 and flat["throughput/mfu"] > 0
    # resume continues from step 2 to step 3
    assert main(["train", *TINY, "train.steps=3", "checkpoint.save_every=10", f"output_dir={out}",
                 "--resume", "latest"]) == 0
    assert (out / "checkpoints" / "step_0000000003").is_dir()
    capsys.readouterr()
    assert main(["checkpoint", "inspect", "--json", str(out / "checkpoints" / "step_0000000003")]) == 0
    info = json.loads(capsys.readouterr().out)
    assert info["complete"] and info["step"] == 3
    export = tmp_path / "export"
    assert main(["checkpoint", "export", str(out / "checkpoints" / "step_0000000003"), str(export)]) == 0
    assert (export / "model.safetensors.index.json").is_file()
    samples = tmp_path / "samples"
    assert main(["generate", "--checkpoint", str(export), "--config", str(out / "config.yaml"), "--prompt", "kite",
                 "--steps", "2", "--frames", "2", "--height", "8", "--width", "8", "--seed", "4",
                 "--output", str(samples)]) == 0
    assert (samples / "sample_00000.pt").is_file()


def test_data_commands(tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    root = tmp_path / "data"
    assert main(["data", "synthesize", "--output", str(root), "--samples", "6", "--samples-per-shard", "4"]) == 0
    assert main(["data", "validate", str(root)]) == 0
    assert "2 shards, 6 samples" in capsys.readouterr().out
    (root / "shard_00001" / "manifest.json").write_text("{}")
    assert main(["data", "validate", str(root)]) == 1


def test_info(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["info"]) == 0
    assert "torch" in capsys.readouterr().out


def test_finetune_lora_from_exported_base(tmp_path: Path) -> None:
    base = tmp_path / "base"
    assert main(["train", *TINY, "train.steps=2", "checkpoint.save_every=2", f"output_dir={base}"]) == 0
    export = tmp_path / "export"
    assert main(["checkpoint", "export", str(base / "checkpoints" / "step_0000000002"), str(export)]) == 0
    out = tmp_path / "ft"
    assert main(["finetune", *TINY, "train.steps=2", "--base", str(export), f"output_dir={out}",
                 "finetune.lora_rank=4"]) == 0
    from avgen_b200.finetune import LoRAConfig, apply_lora, load_adapter

    from avgen_b200.config import load_config
    from avgen_b200.config.resolve import build_model

    model = build_model(load_config(out / "config.yaml"))
    apply_lora(model, LoRAConfig(rank=4, alpha=32.0))
    meta = load_adapter(out / "adapter.safetensors", model)
    assert meta["base_checkpoint"] == str(export)
