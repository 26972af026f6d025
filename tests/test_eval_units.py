"""Evaluation metrics on CPU against constructed clips with known answers:
temporal consistency, motion, flicker, static frames, saturation, sharpness,
the conditional-generation metrics and the audio metrics; running-metric
merging across shards; the Frechet distance against the Gaussian closed form
(reference test strategy: tests/test_eval*.py)."""
from __future__ import annotations

import math

import pytest
import torch

from avgen_b200.eval.learned import frechet_distance, list_learned_metrics, learned_metric_available
from avgen_b200.eval.protocols import MetricError, RunningMetric, build_metric, list_metrics, require_video


def _static(b: int = 2, t: int = 6, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(b, 3, 1, 8, 8, generator=g) * 1.6 - 0.8).repeat(1, 1, t, 1, 1)


def _moving(b: int = 2, t: int = 6, step: float = 0.1) -> torch.Tensor:
    base = _static(b, 1)
    return torch.cat([(base + step * i).clamp(-1, 1) for i in range(t)], dim=2)


def test_registry_lists_the_builtin_metrics() -> None:
    names = set(list_metrics())
    assert {"temporal_consistency", "motion_magnitude", "flicker_index", "static_frames", "saturation",
            "sharpness"} <= names
    with pytest.raises((KeyError, MetricError)):
        build_metric("fvd_magic")


def test_static_clip_scores() -> None:
    video = _static()
    tc = build_metric("temporal_consistency")
    tc.update(video=video)
    assert tc.compute()["temporal_consistency/cosine"] == pytest.approx(1.0, abs=1e-6)
    mm = build_metric("motion_magnitude")
    mm.update(video=video)
    assert mm.compute()["motion_magnitude/mean"] == pytest.approx(0.0, abs=1e-7)
    sf = build_metric("static_frames")
    sf.update(video=video)
    out = sf.compute()
    assert out["static_frames/pair_rate"] == pytest.approx(1.0) and out["static_frames/clip_rate"] == pytest.approx(1.0)


@pytest.mark.parametrize("step", [0.05, 0.1, 0.2])
def test_motion_magnitude_measures_the_frame_delta(step: float) -> None:
    base = torch.zeros(1, 3, 1, 4, 4)
    video = torch.cat([base + step * i for i in range(5)], dim=2)
    mm = build_metric("motion_magnitude")
    mm.update(video=video)
    # the mean absolute frame delta, relative to the clip's spread
    assert mm.compute()["motion_magnitude/mean"] == pytest.approx(step / float(video.flatten(1).std(1)), rel=1e-5)
    sf = build_metric("static_frames", threshold=step / 2)
    sf.update(video=video)
    assert sf.compute()["static_frames/pair_rate"] == pytest.approx(0.0)


def test_flicker_is_higher_for_alternating_frames() -> None:
    smooth = _moving(step=0.02)
    base = _static(t=1)
    alternating = torch.cat([base + (0.3 if i % 2 else -0.3) for i in range(6)], dim=2)
    a, b = build_metric("flicker_index"), build_metric("flicker_index")
    a.update(video=smooth)
    b.update(video=alternating)
    assert b.compute()["flicker_index/index"] > a.compute()["flicker_index/index"]


def test_saturation_fractions() -> None:
    video = torch.zeros(1, 1, 2, 2, 2)
    video[0, 0, 0, 0, 0] = 1.0  # at the edge
    video[0, 0, 0, 0, 1] = 1.5  # outside and at the edge
    m = build_metric("saturation")
    m.update(video=video)
    out = m.compute()
    assert out["saturation/clipped_fraction"] == pytest.approx(2 / 8)
    assert out["saturation/out_of_range_fraction"] == pytest.approx(1 / 8)


def test_sharpness_prefers_detail() -> None:
    g = torch.Generator().manual_seed(3)
    noisy = torch.rand(1, 3, 2, 16, 16, generator=g)
    flat = torch.full((1, 3, 2, 16, 16), 0.5)
    a, b = build_metric("sharpness"), build_metric("sharpness")
    a.update(video=noisy)
    b.update(video=flat)
    ka = next(k for k in a.compute())
    assert a.compute()[ka] > b.compute().get(ka, 0.0)


def test_running_metric_merge_equals_one_pass() -> None:
    videos = [_moving(step=s) for s in (0.05, 0.1, 0.2)]
    whole = build_metric("motion_magnitude")
    for v in videos:
        whole.update(video=v)
    shards = [build_metric("motion_magnitude") for _ in range(3)]
    for m, v in zip(shards, videos):
        m.update(video=v)
    merged = build_metric("motion_magnitude")
    for m in shards:
        merged.merge(m.state())
    assert merged.compute() == pytest.approx(whole.compute())
    merged.reset()
    assert merged.compute() == {}


def test_required_inputs_and_layouts() -> None:
    m = build_metric("temporal_consistency")
    with pytest.raises(MetricError, match="requires video"):
        m.update(audio=torch.zeros(1, 1, 4))
    with pytest.raises(MetricError):
        require_video(torch.zeros(2, 3, 4), metric="x")
    with pytest.raises(MetricError):
        require_video([1, 2], metric="x")

    class Counting(RunningMetric):
        name = "counting"

        def observe(self, **inputs):  # noqa: ANN003, ANN201
            return {"n": (torch.tensor(float(inputs["video"].shape[0])), 1), "skip": (torch.tensor(5.0), 0)}

    c = Counting()
    c.update(video=torch.zeros(3, 1, 1, 1, 1))
    assert c.compute() == {"counting/n": 3.0}  # zero-count statistics are dropped


def test_single_frame_clips_contribute_nothing_to_temporal_metrics() -> None:
    one = _static(t=1)
    for name in ("temporal_consistency", "motion_magnitude", "flicker_index", "static_frames"):
        m = build_metric(name)
        m.update(video=one)
        assert m.compute() == {}, name


# ----------------------------------------------------------------------------- conditional and audio metrics


def test_first_frame_fidelity_and_seam_continuity() -> None:
    video = _moving(step=0.05)
    m = build_metric("first_frame_fidelity")
    m.update(video=video, reference=video.clone())
    out = m.compute()
    assert out["first_frame_fidelity/mse"] == pytest.approx(0.0, abs=1e-12)
    assert out["first_frame_fidelity/cosine"] == pytest.approx(1.0, abs=1e-6)
    off = build_metric("first_frame_fidelity")
    off.update(video=video, reference=video + 0.1)
    assert off.compute()["first_frame_fidelity/mse"] == pytest.approx(0.01, rel=1e-4)
    with pytest.raises(MetricError):
        off.update(video=video, reference=video[:, :, :2])
    base = torch.zeros(1, 1, 1, 4, 4)
    steady = torch.cat([base + 0.1 * i for i in range(6)], dim=2)
    seam = build_metric("seam_continuity", context_frames=2)
    seam.update(video=steady)
    assert seam.compute()["seam_continuity/ratio"] == pytest.approx(1.0, rel=1e-5)  # a seamless continuation
    jump = steady.clone()
    jump[:, :, 2:] += 1.0
    cut = build_metric("seam_continuity", context_frames=2)
    cut.update(video=jump)
    assert cut.compute()["seam_continuity/ratio"] > 5.0
    with pytest.raises(MetricError):
        build_metric("seam_continuity", context_frames=6).update(video=steady)


def test_audio_metrics_on_silence_and_tone() -> None:
    names = set(list_metrics())
    t = torch.arange(1600, dtype=torch.float32) / 16000
    tone = torch.sin(2 * math.pi * 440 * t)[None, None].repeat(2, 1, 1)
    silence = torch.zeros(2, 1, 1600)
    if "audio_silence" in names:
        quiet, loud = build_metric("audio_silence"), build_metric("audio_silence")
        quiet.update(video=_static(), audio=silence)
        loud.update(video=_static(), audio=tone)
        kq = next(iter(quiet.compute()))
        assert quiet.compute()[kq] > loud.compute()[kq]
    if "audio_bandwidth" in names:
        m = build_metric("audio_bandwidth", sample_rate=16000.0)
        m.update(video=_static(), audio=tone)
        assert all(math.isfinite(v) for v in m.compute().values())


# ----------------------------------------------------------------------------- Frechet distance


def test_frechet_distance_gaussian_closed_form() -> None:
    g = torch.Generator().manual_seed(0)
    n, d = 20000, 4
    a = torch.randn(n, d, generator=g, dtype=torch.float64)
    b = torch.randn(n, d, generator=g, dtype=torch.float64) * 2.0 + 1.0
    # N(0, I) vs N(1, 4I): |mu|^2 + tr(I) + tr(4I) - 2 tr(2I) = d + d + 4d - 4d = 2d
    assert frechet_distance(a, b) == pytest.approx(2 * d, rel=0.05)
    assert frechet_distance(a, a) == pytest.approx(0.0, abs=1e-6)
    for bad in ((a[:, :3], b), (a[:1], b), (a[0], b)):
        with pytest.raises(MetricError):
            frechet_distance(*bad)


def test_learned_metric_registry_reports_backends() -> None:
    names = list_learned_metrics()
    assert names
    for name in names:
        assert isinstance(learned_metric_available(name), bool)
