"""Samplers, schedules, guidance, conditioning and the pipeline (CPU)."""
from __future__ import annotations

import math
from dataclasses import asdict

import pytest
import torch

from avgen_b200.infer import (GuidanceConfig, ScheduleConfig, SigmaSchedule, StreamState, adaptive_projected_guidance,
                              apply_guidance, apply_modality_guidance, apply_shift, build_model_input, build_sampler,
                              build_sigma_schedule, classifier_free_guidance, condition_first_frame, list_samplers,
                              list_sigma_schedules, rescale_guidance, resolution_shift)


@pytest.mark.parametrize("name", ["euler", "heun", "dpmpp_2m", "res_multistep", "euler_ancestral"])
def test_samplers_exact_on_straight_flows(name: str) -> None:
    """With a constant velocity (a straight rectified-flow path) every consistent solver is exact."""
    g = torch.Generator().manual_seed(0)
    x0, noise = torch.randn(3, 7, generator=g), torch.randn(3, 7, generator=g)
    v = noise - x0
    s = build_sampler(name)
    s.reset()
    sig = build_sigma_schedule(ScheduleConfig(steps=6, shift=3.0))
    x = x0 + float(sig.sigmas[0]) * v
    for _, a, b in sig:
        x = s.step(v, x, a, b, denoise=lambda p, t: v)
    assert torch.allclose(x, x0, atol=1e-5)


def test_sampler_registry_and_validation() -> None:
    assert {"euler", "heun", "dpmpp_2m", "res_multistep", "euler_ancestral"} <= set(list_samplers())
    with pytest.raises(KeyError):
        build_sampler("nope")
    with pytest.raises(ValueError):
        build_sampler("euler").step(torch.zeros(1), torch.zeros(1), 0.3, 0.5)
    with pytest.raises(ValueError):
        build_sampler("heun").step(torch.zeros(1), torch.zeros(1), 0.5, 0.3)  # needs denoise


def test_ancestral_noise_split() -> None:
    from avgen_b200.infer import EulerAncestralSampler, SamplerConfig

    s = EulerAncestralSampler(SamplerConfig(name="euler_ancestral", eta=1.0))
    down, up = s.ancestral_split(0.8, 0.5)
    assert math.isclose(down * down + up * up, 0.25, rel_tol=1e-9) and up > 0
    x, noise, scale = s.step_with_noise(torch.zeros(4), torch.ones(4), 0.8, 0.5, generator=torch.Generator())
    assert scale == up and noise.shape == (4,)
    assert s.is_stochastic


def test_schedules() -> None:
    assert set(list_sigma_schedules()) >= {"linear", "karras", "linear_quadratic"}
    for name in ("linear", "karras", "linear_quadratic"):
        sched = build_sigma_schedule(ScheduleConfig(name=name, steps=10))
        s = sched.sigmas
        assert s.numel() == 11 and float(s[-1]) == 0.0 and bool((s[1:] < s[:-1]).all())
    shifted = apply_shift(torch.tensor([0.0, 0.5, 1.0]), 3.0)
    assert torch.allclose(shifted, torch.tensor([0.0, 0.75, 1.0]))
    assert resolution_shift(256) == 1.0 and resolution_shift(4096) == 3.0 and resolution_shift(10**6) == 3.0
    dyn = ScheduleConfig(steps=4, dynamic_shift=True)
    assert build_sigma_schedule(dyn, sequence_length=4096).shift == 3.0
    with pytest.raises(ValueError):
        build_sigma_schedule(dyn)
    with pytest.raises(ValueError):
        SigmaSchedule(torch.tensor([1.0, 0.5, 0.6, 0.0]))


def test_guidance_math() -> None:
    g = torch.Generator().manual_seed(1)
    c, u = torch.randn(2, 5, 6, generator=g), torch.randn(2, 5, 6, generator=g)
    assert torch.allclose(classifier_free_guidance(c, u, 4.0), u + 4.0 * (c - u), atol=1e-6)
    r = rescale_guidance(u + 4 * (c - u), c, 1.0)
    assert torch.allclose(r.std(dim=(1, 2)), c.std(dim=(1, 2)), rtol=1e-5)
    apg = adaptive_projected_guidance(c, u, 3.0, eta=1.0)  # eta=1 keeps the parallel part: plain CFG
    assert torch.allclose(apg, classifier_free_guidance(c, u, 3.0), atol=1e-5)
    cfg = GuidanceConfig(scale=5.0, schedule="linear", min_scale=1.0)
    assert cfg.scale_at(0.0) == 5.0 and cfg.scale_at(1.0) == 1.0
    assert GuidanceConfig(scale=3.0, schedule="interval", start_fraction=0.2, end_fraction=0.5).scale_at(0.9) == 1.0
    assert torch.equal(apply_guidance(c, None, config=GuidanceConfig()), c)
    with pytest.raises(ValueError):
        apply_guidance(c, None, config=GuidanceConfig(scale=2.0))
    chained = apply_modality_guidance([("text", u), ("text", c)], config=GuidanceConfig(scale=2.0))
    assert torch.allclose(chained, classifier_free_guidance(c, u, 2.0), atol=1e-6)


def test_conditioning_records_level_groups() -> None:
    from avgen_b200.core.patchify import GridPatchifier
    from avgen_b200.core.tokens import TextContext

    lat = torch.randn(2, 4, 3, 4, 4)
    state = StreamState(latents=lat, fps=8.0)
    text = TextContext.empty(2, 8)
    inputs = condition_first_frame(state, torch.zeros(2, 4, 4, 4), sigma=0.7, text=text, patchifier=GridPatchifier())
    v = inputs.video
    assert v.has_level_groups
    assert torch.equal(v.level_values.gather(1, v.level_index.long()), v.noise_level)
    assert bool(v.conditioned[:, :4].all()) and not bool(v.conditioned[:, 4:].any())
    plain = build_model_input(video=state, sigma=0.4, text=text, patchifier=GridPatchifier())
    assert plain.video.noise_level.shape == (2,)


def _tiny_pipeline():  # noqa: ANN202
    from avgen_b200.codecs import ReferenceTextEncoder, ReferenceVideoCodec
    from avgen_b200.infer import GenerationPipeline
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    codec = ReferenceVideoCodec(channels=1, spatial_compression=2)
    cfg["in_channels"] = codec.latent_channels
    model = build_model("video_dit", cfg)
    model.init_weights()
    with torch.no_grad():
        for p in model.parameters():
            p.add_(0.02 * torch.randn_like(p))
    model.eval()
    return GenerationPipeline(model, video_codec=codec, text_encoder=ReferenceTextEncoder(width=cfg["text_width"]))


def test_pipeline_batched_guidance_matches_two_forwards() -> None:
    pipe = _tiny_pipeline()
    kw = dict(steps=3, guidance=GuidanceConfig(scale=4.0, rescale=0.5), height=16, width=16, num_frames=2, seed=3,
              return_latents=True)
    pipe.batch_guidance = True
    a = pipe(["a cat", "rain on a window"], **kw)
    pipe.batch_guidance = False
    b = pipe(["a cat", "rain on a window"], **kw)
    assert a.video.shape == (2, 1, 2, 16, 16)
    assert torch.allclose(a.latents, b.latents, atol=1e-4)
    assert a.config["resolved_shift"] == 1.0 and a.config["sequence_length"] == 2 * 4 * 4
    pipe.batch_guidance = True
    c = pipe(["a cat", "rain on a window"], **kw)
    assert torch.equal(a.latents, c.latents)  # seeded
