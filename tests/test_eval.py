"""Evaluation on CPU: metric semantics, exact cross-rank merging, pinned reports
and their comparison guard, and ``avgen-b200 evaluate`` end to end
(reference test strategy: tests/test_eval.py)."""
from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from avgen_b200.eval import (EvalBatch, EvalPin, EvalReport, IncomparableReports, MetricError, MissingBackendError,
                             build_learned_metric, build_metric, build_metrics, compare_reports, frechet_distance,
                             list_metrics, prompt_set_digest, run_eval_suite, shard_prompts)


def _clip(seed: int, b: int = 3, t: int = 6) -> torch.Tensor:
    return torch.randn(b, 3, t, 8, 8, generator=torch.Generator().manual_seed(seed))


def test_registry_and_semantics() -> None:
    assert {"temporal_consistency", "motion_magnitude", "flicker_index", "static_frames", "saturation", "sharpness",
            "av_sync_proxy", "audio_silence", "audio_bandwidth", "first_frame_fidelity", "seam_continuity",
            "inpaint_boundary"} <= set(list_metrics())
    with pytest.raises(MetricError):
        build_metric("nope")
    still = _clip(0, t=1).expand(-1, -1, 5, -1, -1)
    m = build_metric("static_frames")
    m.update(video=still)
    assert m.compute()["static_frames/clip_rate"] == 1.0
    tc = build_metric("temporal_consistency")
    tc.update(video=still)
    assert tc.compute()["temporal_consistency/cosine"] == pytest.approx(1.0)
    ff = build_metric("first_frame_fidelity")
    v = _clip(1)
    ff.update(video=v, reference=v)
    assert ff.compute()["first_frame_fidelity/cosine"] == pytest.approx(1.0)
    # a clip whose motion follows a beeping audio envelope correlates with it
    t = torch.arange(24.0)
    env = (torch.sin(t / 2) > 0).float()
    video = torch.cumsum(env[None, None, :, None, None].expand(2, 1, 24, 4, 4) * torch.randn(2, 1, 1, 4, 4), 2)
    audio = (env.repeat_interleave(100) * torch.randn(2400))[None, None].expand(2, 1, 2400)
    av = build_metric("av_sync_proxy")
    av.update(video=video, audio=audio)
    assert av.compute()["av_sync_proxy/peak_correlation"] > 0.5
    with pytest.raises(MetricError):
        build_metric("av_sync_proxy").update(video=video)


def test_sharded_evaluation_merges_exactly() -> None:
    clips = [_clip(i) for i in range(4)]
    names = ["temporal_consistency", "motion_magnitude", "flicker_index", "sharpness"]
    pin = EvalPin(steps=4)
    whole = run_eval_suite([EvalBatch(video=c) for c in clips], metrics=names, pin=pin)
    # rank 1 measured the odd batches; rank 0 runs the suite on the even ones and merges
    remote = build_metrics(names, decoded=False)
    for c in clips[1::2]:
        for m in remote.metrics.values():
            m.update(video=c)
    remote_state = {n: m.state() for n, m in remote.metrics.items()}

    def gather(obj):  # noqa: ANN001, ANN202
        return [obj, remote_state] if isinstance(obj, dict) else [obj, 6]

    rep = run_eval_suite([EvalBatch(video=c) for c in clips[0::2]], metrics=names, pin=pin, gather=gather,
                         data_rank=0)
    assert rep.pin.num_samples == whole.pin.num_samples == 12
    for k, v in whole.metrics.items():
        assert rep.metrics[k] == pytest.approx(v, rel=1e-12)
    assert shard_prompts(list("abcde"), data_rank=1, data_world=2) == ("b", "d")


def test_reports_round_trip_and_comparison_guard(tmp_path: Path) -> None:
    prompts = ["a", "b"]
    rep = run_eval_suite([EvalBatch(video=_clip(0))], metrics=["motion_magnitude", "saturation", "fvd"],
                         pin=EvalPin(checkpoint="x", steps=8, seed=1), prompts=prompts)
    assert "saturation" in rep.skipped and "fvd" in rep.skipped  # latent space; no FVD extractor ships
    assert rep.pin.prompt_digest == prompt_set_digest(prompts)
    path = rep.save(tmp_path / "r.json")
    back = EvalReport.load(path)
    assert back.metrics == rep.metrics and back.pin == rep.pin
    other = EvalReport(pin=EvalPin(checkpoint="y", steps=8, seed=2, prompt_digest=rep.pin.prompt_digest,
                                   num_samples=rep.pin.num_samples, metrics=rep.pin.metrics),
                       metrics={k: v * 2 for k, v in rep.metrics.items()})
    with pytest.raises(IncomparableReports):
        compare_reports(rep, other)
    table = compare_reports(rep, other, allow=("seed",))
    key = next(iter(table))
    assert table[key]["delta"] == pytest.approx(rep.metrics[key])
    with pytest.raises(ValueError):
        EvalReport.from_dict({**rep.to_dict(), "report_version": 99})
    assert "METRICS" in rep.render()


def test_frechet_distance_and_gating() -> None:
    g = torch.Generator().manual_seed(0)
    a = torch.randn(500, 4, generator=g)
    assert frechet_distance(a, a) == pytest.approx(0.0, abs=1e-6)
    b = a + 3.0
    assert frechet_distance(a, b) == pytest.approx(36.0, rel=1e-6)  # only the mean moved: |3 * 1|^2 * 4
    with pytest.raises(MissingBackendError):
        build_learned_metric("fvd")


def test_cli_evaluate_and_compare(tmp_path: Path, capsys: pytest.CaptureFixture[str]) -> None:
    from avgen_b200.cli.main import main

    tiny = ["model.depth=1", "model.width=32", "model.num_heads=2", "model.in_channels=4", "data.latent_channels=4",
            "data.text_tokens=3", "data.text_width=8", "data.buckets=[{frames: 2, height: 8, width: 8}]",
            "train.warmup_steps=1", "train.global_batch_size=1", "checkpoint.async_save=false"]
    out = tmp_path / "run"
    assert main(["train", *tiny, "train.steps=2", f"output_dir={out}"]) == 0
    export = tmp_path / "export"
    assert main(["checkpoint", "export", str(out / "checkpoints" / "step_0000000002"), str(export)]) == 0
    ev = ["eval.steps=2", "eval.frames=4", "eval.height=8", "eval.width=8", "eval.num_prompts=3",
          "eval.metrics=[temporal_consistency, motion_magnitude, flicker_index]"]
    r1, r2 = tmp_path / "a.json", tmp_path / "b.json"
    assert main(["evaluate", "--checkpoint", str(export), "--config", str(out / "config.yaml"), "--output", str(r1),
                 *ev]) == 0
    assert main(["evaluate", "--checkpoint", str(export), "--config", str(out / "config.yaml"), "--output", str(r2),
                 *ev, "eval.seed=5"]) == 0
    rep = json.loads(r1.read_text())
    assert rep["pin"]["num_samples"] == 3 and "temporal_consistency/cosine" in rep["metrics"]
    capsys.readouterr()
    assert main(["evaluate", "--baseline", str(r1), "--report", str(r2)]) == 1  # seeds differ
    assert main(["evaluate", "--baseline", str(r1), "--report", str(r2), "--allow", "seed"]) == 0
    assert "temporal_consistency/cosine" in capsys.readouterr().out
