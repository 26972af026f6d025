"""Telemetry units on CPU: metric accumulation (weighted means, counts kept as
totals, one flush), host-clock throughput with MFU arithmetic and percentiles,
rank-gated loggers, the JSONL format, fan-out that survives a failing backend,
and the exposed-communication accounting's off-by-default contract (reference
test strategy: tests/test_telemetry*.py)."""
from __future__ import annotations

import io
import json
import time
from pathlib import Path

import pytest
import torch

from avgen_b200.core.metrics import StepMetrics
from avgen_b200.telemetry import comm as exposed
from avgen_b200.telemetry.logger import (ConsoleLogger, JSONLLogger, MultiLogger, NoOpLogger, RankGatedLogger,
                                         build_logger)
from avgen_b200.telemetry.metrics import MemoryReporter, MetricAccumulator, ThroughputMeter, merge_metrics


def _metrics(loss: float, tokens: int = 10, skipped: bool = False, nonfinite: bool = False) -> StepMetrics:
    f = lambda v: torch.tensor(v, dtype=torch.float32)  # noqa: E731
    return StepMetrics(loss=f(loss), video_loss=f(loss * 0.5), audio_loss=f(0.0),
                       valid_video_tokens=torch.tensor(tokens), valid_audio_tokens=torch.tensor(0),
                       grad_norm=f(2.0 * loss), nonfinite=torch.tensor(nonfinite), skipped=torch.tensor(skipped))


def test_step_metrics_contract() -> None:
    m = _metrics(1.5)
    m.validate()
    assert m.to_mapping()["loss"] == 1.5
    z = StepMetrics.zeros()
    z.validate()
    assert all(v == 0.0 for v in z.to_mapping().values())
    from dataclasses import replace

    with pytest.raises(TypeError):
        replace(m, skipped=torch.tensor(1.0)).validate()  # a flag must be bool
    with pytest.raises(TypeError):
        replace(m, valid_video_tokens=torch.tensor(1.0)).validate()  # a count must be int64
    with pytest.raises(ValueError):
        replace(m, loss=torch.ones(2)).validate()  # every field is a scalar
    with pytest.raises(ValueError):
        replace(m, loss=torch.ones((), requires_grad=True)).validate()  # and detached


@pytest.mark.parametrize("weights", [(1.0, 1.0, 1.0), (1.0, 2.0, 3.0), (0.5, 0.25, 0.25)])
def test_accumulator_weighted_means_and_totals(weights: tuple[float, ...]) -> None:
    acc = MetricAccumulator()
    assert acc.is_empty and acc.flush() == {}
    losses = (1.0, 2.0, 4.0)
    for loss, w in zip(losses, weights):
        acc.update(_metrics(loss, tokens=10, skipped=loss == 4.0), weight=w)
    out = acc.flush()
    mean = sum(l * w for l, w in zip(losses, weights)) / sum(weights)
    assert out["loss"] == pytest.approx(mean)
    assert out["grad_norm"] == pytest.approx(2 * mean)
    # counts come back as totals (weighted), not means
    assert out["valid_video_tokens"] == pytest.approx(10 * sum(weights))
    assert out["skipped"] == pytest.approx(weights[2])
    assert acc.is_empty  # flush resets by default


def test_accumulator_flush_without_reset() -> None:
    acc = MetricAccumulator()
    acc.update(_metrics(1.0))
    first = acc.flush(reset=False)
    acc.update(_metrics(3.0))
    assert acc.flush()["loss"] == pytest.approx(2.0) and first["loss"] == 1.0
    assert acc.device.type == "cpu"


def test_throughput_meter_host_clock() -> None:
    meter = ThroughputMeter(flops_per_sample=1e12, peak_flops=1e13, world_size=2, use_cuda_events=False)
    meter.step()  # the first call only opens the window
    for _ in range(4):
        time.sleep(0.01)
        meter.step(samples=2, tokens=100)
    rep = meter.report()
    assert rep.steps == 4
    assert 0.005 < rep.step_time_p50 < 0.5 and rep.step_time_p99 >= rep.step_time_p50
    total = rep.samples_per_second and 8 / rep.samples_per_second
    assert rep.tokens_per_second == pytest.approx(400 / total)
    assert rep.mfu == pytest.approx(rep.samples_per_second * 1e12 / (1e13 * 2))
    assert rep.hfu == pytest.approx(rep.mfu)
    keys = rep.to_mapping()
    assert set(keys) == {f"throughput/{k}" for k in ("steps", "step_time_p50", "step_time_p99", "samples_per_second",
                                                    "tokens_per_second", "mfu", "hfu")}
    again = meter.report()  # the window was reset: no steps since
    assert again.steps == 0 and again.samples_per_second == 0.0


def test_throughput_meter_hardware_flops_and_explicit_start() -> None:
    meter = ThroughputMeter(flops_per_sample=1.0, hardware_flops_per_sample=1.5, peak_flops=10.0,
                            use_cuda_events=False)
    meter.start()
    time.sleep(0.005)
    meter.step(samples=1)
    rep = meter.report()
    assert rep.steps == 1 and rep.hfu == pytest.approx(1.5 * rep.mfu)


def test_memory_reporter_without_cuda() -> None:
    rep = MemoryReporter(device="cpu")
    assert not rep.available and rep.report() is None and rep.peak_across(None) is None
    rep.reset_peaks()
    assert merge_metrics({"a": 1.0}, {"b": 2.0}, {"a": 3.0}) == {"a": 3.0, "b": 2.0}


# ----------------------------------------------------------------------------- loggers


def test_rank_gating() -> None:
    assert ConsoleLogger(rank=0, stream=io.StringIO()).enabled
    quiet = ConsoleLogger(rank=3, stream=io.StringIO())
    assert not quiet.enabled
    quiet.log_metrics({"loss": 1.0}, 1)
    assert quiet._stream.getvalue() == ""  # noqa: SLF001
    loud = ConsoleLogger(rank=3, all_ranks=True, stream=io.StringIO())
    loud.log_metrics({"loss": 1.0}, 1)
    assert "loss 1" in loud._stream.getvalue()  # noqa: SLF001


def test_console_format_and_key_selection() -> None:
    buf = io.StringIO()
    lg = ConsoleLogger(rank=0, stream=buf, keys=("train/loss", "throughput/mfu"))
    lg.log_metrics({"train/loss": 0.123456, "throughput/mfu": 0.35, "ignored": 9.0, }, 42)
    lg.log_metrics({"train/loss": 2.5e6}, 43)
    lines = buf.getvalue().splitlines()
    assert lines[0].startswith("step      42") and "loss 0.1235" in lines[0] and "mfu 0.35" in lines[0]
    assert "ignored" not in lines[0] and "e+06" in lines[1]


def test_jsonl_logger_round_trip_and_close(tmp_path: Path) -> None:
    path = tmp_path / "sub" / "m.jsonl"
    lg = JSONLLogger(path, rank=0)
    lg.log_config({"model": {"depth": 2}, "path": Path("/x")})
    lg.log_metrics({"loss": 1.0, "n": 3}, 7)
    lg.close()
    lg.close()  # idempotent
    lg.log_metrics({"loss": 2.0}, 8)  # ignored after close
    rows = [json.loads(x) for x in path.read_text().splitlines()]
    assert rows[0]["config"]["model"]["depth"] == 2 and rows[0]["config"]["path"] == "/x"
    assert rows[1]["step"] == 7 and rows[1]["loss"] == 1.0 and rows[1]["n"] == 3.0 and "time" in rows[1]
    assert len(rows) == 2
    other = JSONLLogger(tmp_path / "r1.jsonl", rank=1)
    other.log_metrics({"loss": 1.0}, 1)
    assert not (tmp_path / "r1.jsonl").exists()  # non-zero ranks never open the file


def test_multilogger_survives_a_failing_backend(caplog: pytest.LogCaptureFixture) -> None:
    class Broken(RankGatedLogger):
        calls = 0

        def _metrics(self, metrics, step):  # noqa: ANN001, ANN202
            Broken.calls += 1
            raise OSError("disk full")

    buf = io.StringIO()
    multi = MultiLogger([Broken(rank=0), ConsoleLogger(rank=0, stream=buf)])
    multi.log_metrics({"loss": 1.0}, 1)
    multi.log_metrics({"loss": 2.0}, 2)
    assert Broken.calls == 1  # disabled after its first failure
    assert buf.getvalue().count("step") == 2
    multi.log_config({"a": 1})
    multi.log_artifact("x")
    multi.close()
    assert len(multi.loggers) == 2


def test_build_logger(tmp_path: Path) -> None:
    lg = build_logger(["noop", "jsonl"], output_dir=tmp_path)
    assert isinstance(lg.loggers[0], NoOpLogger) and isinstance(lg.loggers[1], JSONLLogger)
    lg.log_metrics({"x": 1.0}, 0)
    lg.close()
    assert (tmp_path / "metrics.jsonl").exists()
    with pytest.raises(ValueError):
        build_logger(["mlflow"])


def test_base_logger_requires_metrics_override() -> None:
    with pytest.raises(NotImplementedError):
        RankGatedLogger(rank=0).log_metrics({"a": 1.0}, 0)
    with RankGatedLogger(rank=0) as lg:
        lg.log_config({"a": 1})
    assert not lg.enabled


# ----------------------------------------------------------------------------- exposed communication


def test_exposed_comm_accounting_is_off_by_default_and_free_on_cpu() -> None:
    exposed.enable(False)
    assert not exposed.enabled()
    with exposed.comm_span("ring_ready_barrier"):
        pass
    assert exposed.summary() == {}
    exposed.enable(True)
    try:
        with exposed.comm_span("ring_ready_barrier"):  # no CUDA: nothing is recorded
            pass
        assert exposed.summary() == {}
    finally:
        exposed.enable(False)
        exposed.reset()


def test_instrument_fsdp_ignores_plain_modules() -> None:
    model = torch.nn.Sequential(torch.nn.Linear(4, 4), torch.nn.ReLU())
    assert exposed.instrument_fsdp(model) == 0
