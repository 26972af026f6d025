"""Profiler and hang-forensics helpers on CPU: rank gating, a torch-profiler
schedule that writes one Chrome trace per active window, and the no-op forms of
the CUDA-only tools when no device is present (reference test strategy:
tests/test_telemetry.py -- profiler section)."""
from __future__ import annotations

from pathlib import Path

import pytest
import torch

from avgen_b200.telemetry.profiler import (DeviceTimer, flight_recorder_dump, memory_snapshot, nvtx_range,
                                           profile_steps, should_profile_rank)


@pytest.mark.parametrize("rank,local,mode,expect", [("0", "0", "global_zero", True), ("3", "0", "global_zero", False),
                                                    ("3", "0", "local_zero", True), ("3", "2", "local_zero", False),
                                                    ("5", "1", "all", True)])
def test_rank_gating(monkeypatch: pytest.MonkeyPatch, rank: str, local: str, mode: str, expect: bool) -> None:
    monkeypatch.setenv("RANK", rank)
    monkeypatch.setenv("LOCAL_RANK", local)
    assert should_profile_rank(mode=mode) is expect


def test_unknown_mode_rejected() -> None:
    with pytest.raises(ValueError):
        should_profile_rank(mode="odd_ranks")


def test_profile_steps_writes_a_trace_per_window(tmp_path: Path, monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("RANK", "0")
    x = torch.randn(64, 64)
    with profile_steps(tmp_path, active=2, warmup=1, wait=0, repeat=1) as prof:
        for _ in range(5):
            (x @ x).sum()
            prof.step()
    traces = sorted(tmp_path.glob("trace_rank0_step*.json.gz"))
    assert len(traces) == 1 and traces[0].stat().st_size > 0


def test_profile_steps_is_a_no_op_off_rank_or_inactive(tmp_path: Path, monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("RANK", "1")
    with profile_steps(tmp_path / "a") as prof:
        prof.step()
    assert not (tmp_path / "a").exists()
    monkeypatch.setenv("RANK", "0")
    with profile_steps(tmp_path / "b", active=0) as prof:
        prof.step()
        prof.export_chrome_trace(str(tmp_path / "never.json"))
    assert not (tmp_path / "b").exists() and not (tmp_path / "never.json").exists()


def test_cuda_only_tools_are_no_ops_without_a_device(tmp_path: Path) -> None:
    if torch.cuda.is_available():
        pytest.skip("checks the CPU-only behaviour")
    with memory_snapshot(tmp_path / "snap.pickle"):
        torch.ones(3).sum()
    assert not (tmp_path / "snap.pickle").exists()
    with nvtx_range("region"):
        pass
    timer = DeviceTimer()
    with timer.region("step"):
        torch.ones(3).sum()
    assert timer.collect() == {}


def test_flight_recorder_dump_without_a_process_group(tmp_path: Path) -> None:
    out = flight_recorder_dump(tmp_path / "fr")
    assert out is None or out.exists()
