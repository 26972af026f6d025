"""More of the ``avgen-b200`` command line on CPU: the data subcommands
(synthesize, shard, inspect, validate, and corruption), info, plan tables,
simulate text output, checkpoint usage errors, override placement, and the exit
codes of each failure class (reference test strategy: tests/test_cli.py)."""
from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from avgen_b200.cli.main import _overrides_last, main


def test_data_synthesize_inspect_validate(tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    out = tmp_path / "ds"
    assert main(["data", "synthesize", "--output", str(out), "--samples", "5", "--samples-per-shard", "2"]) == 0
    shards = sorted(p.name for p in out.iterdir())
    assert shards == ["shard_00000", "shard_00001", "shard_00002"]
    capsys.readouterr()
    assert main(["data", "inspect", str(out)]) == 0
    text = capsys.readouterr().out
    assert "5" in text
    assert main(["data", "validate", str(out)]) == 0
    assert main(["data", "validate", str(out / "shard_00001")]) == 0  # a single shard directory


def test_data_validate_detects_corruption_and_empty_roots(tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    out = tmp_path / "ds"
    assert main(["data", "synthesize", "--output", str(out), "--samples", "2", "--samples-per-shard", "2"]) == 0
    shard = out / "shard_00000"
    payload = [p for p in shard.iterdir() if p.suffix in (".safetensors", ".pt", ".bin")][0]
    raw = bytearray(payload.read_bytes())
    raw[-3] ^= 0xFF
    payload.write_bytes(bytes(raw))
    assert main(["data", "validate", str(out)]) != 0
    empty = tmp_path / "empty"
    empty.mkdir()
    assert main(["data", "inspect", str(empty)]) == 1
    assert main(["data"]) == 2


def test_data_shard_packs_sample_files(tmp_path: Path) -> None:
    from avgen_b200.data.synthetic import SyntheticConfig, SyntheticSource

    src = SyntheticSource(SyntheticConfig(num_samples=3, audio_frames=0))
    raw = tmp_path / "raw"
    raw.mkdir()
    for i in range(3):
        torch.save(src.sample(i), raw / f"s{i}.pt")
    assert main(["data", "shard", str(raw), str(tmp_path / "packed"), "--samples-per-shard", "2"]) == 0
    assert len(list((tmp_path / "packed").iterdir())) == 2
    assert main(["data", "shard", str(tmp_path / "nothing_here"), str(tmp_path / "x")]) == 1


def test_info_lists_versions_and_metrics(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["info", "--metrics"]) == 0
    out = capsys.readouterr().out
    assert "torch" in out and "kernels" in out and "metric       temporal_consistency" in out


def test_plan_table_and_errors(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["plan", "--world-size", "8", "--gpu", "b200"]) == 0
    lines = capsys.readouterr().out.splitlines()
    assert "B200" in lines[0]  # a header naming the problem, then the ranked table
    assert any(line.startswith("plan") for line in lines)
    assert main(["plan", "--world-size", "8", "--gpu", "tpu"]) != 0


def test_simulate_text_and_config_errors(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["simulate", "--gpu", "b200", "--world-size", "8", "parallel.dp_shard=8"]) == 0
    assert capsys.readouterr().out.strip()
    assert main(["simulate", "--world-size", "8", "model.width=100", "model.num_heads=3"]) == 3
    assert main(["simulate", "--world-size", "8", "no.such=1"]) == 3


def test_checkpoint_usage_errors(tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["checkpoint"]) == 2
    assert main(["checkpoint", "inspect", "--json", str(tmp_path)]) == 0
    info = json.loads(capsys.readouterr().out)
    assert not info["complete"]


@pytest.mark.parametrize("argv,expect", [
    (["train", "--dry-run", "train.lr=0.1"], ["train", "--dry-run", "train.lr=0.1"]),
    (["train", "train.lr=0.1", "--dry-run"], ["train", "--dry-run", "train.lr=0.1"]),
    (["train", "--config", "a=b.yaml", "x.y=1"], ["train", "--config", "a=b.yaml", "x.y=1"]),
    (["plan", "--world-size", "8", "model.depth=4", "--json"], ["plan", "--world-size", "8", "--json", "model.depth=4"]),
])
def test_overrides_move_behind_options(argv: list[str], expect: list[str]) -> None:
    assert _overrides_last(argv) == expect


def test_train_dry_run_prints_the_plan(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["train", "--dry-run", "model.depth=2", "model.width=64", "model.num_heads=2",
                 "data.buckets=[{frames: 2, height: 8, width: 8}]", "train.warmup_steps=1"]) == 0
    assert capsys.readouterr().out.strip()


def test_unknown_command_and_help(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["frobnicate"]) == 2
    assert main(["--help"]) == 0
    assert "exit codes" in capsys.readouterr().out


def test_eval_is_an_alias_of_evaluate(capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["eval", "--help"]) == 0  # the reference's subcommand name
    assert capsys.readouterr().out.startswith("usage: avgen-b200 evaluate")
