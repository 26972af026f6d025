"""Sampler, sigma-schedule and guidance mathematics on CPU, checked against
closed forms (reference test strategy: tests/test_infer.py -- per-sampler
convergence, schedule invariants, guidance identities, config round trips).

The convergence tests integrate the probability-flow ODE of a 1-D Gaussian:
data ~ N(0, c^2) on the path x_t = (1 - t) x0 + t n has the exact velocity
v(x, t) = (t - (1 - t) c^2) x / V(t) with V(t) = (1 - t)^2 c^2 + t^2, and the
flow maps x_1 to x_0 = c x_1 exactly, so every solver's error is measurable.
"""
from __future__ import annotations

import math

import pytest
import torch

from avgen_b200.infer.guidance import (GuidanceConfig, adaptive_projected_guidance, apply_guidance,
                                       apply_modality_guidance, classifier_free_guidance, rescale_guidance)
from avgen_b200.infer.sampler import (EulerAncestralSampler, SamplerConfig, build_sampler, list_samplers,
                                      register_sampler, to_epsilon, to_x0)
from avgen_b200.infer.schedule import (ScheduleConfig, SigmaSchedule, apply_shift, build_sigma_schedule,
                                       karras_sigmas, linear_quadratic_sigmas, linear_sigmas, list_sigma_schedules,
                                       register_sigma_schedule, resolution_shift)

C = 0.5  # data standard deviation of the Gaussian test flow


def _velocity(x: torch.Tensor, t: float, c: float = C) -> torch.Tensor:
    var = (1.0 - t) ** 2 * c * c + t * t
    return (t - (1.0 - t) * c * c) * x / var


def _integrate(name: str, steps: int, schedule: str = "linear") -> float:
    sampler = build_sampler(name)
    sig = build_sigma_schedule(ScheduleConfig(name=schedule, steps=steps))
    x1 = torch.linspace(-2.0, 2.0, 9, dtype=torch.float64)
    x = x1.clone()
    for _, s, s_next in sig:
        x = sampler.step(_velocity(x, s), x, s, s_next, denoise=lambda y, t: _velocity(y, t))
    return float((x - C * x1).abs().max())


@pytest.mark.parametrize("name", ["euler", "heun", "dpmpp_2m", "res_multistep"])
@pytest.mark.parametrize("steps", [8, 32])
def test_deterministic_samplers_converge_on_gaussian_flow(name: str, steps: int) -> None:
    err = _integrate(name, steps)
    first_order = name == "euler"
    bound = {8: 0.2 if first_order else 0.05, 32: 0.05 if first_order else 0.012}[steps]
    assert err < bound, err


@pytest.mark.parametrize("name", ["euler", "heun", "dpmpp_2m", "res_multistep"])
def test_sampler_error_shrinks_with_steps(name: str) -> None:
    errs = [_integrate(name, n) for n in (4, 16, 64)]
    assert errs[0] > errs[1] > errs[2]


@pytest.mark.parametrize("name", ["heun", "dpmpp_2m", "res_multistep"])
def test_second_order_samplers_beat_euler(name: str) -> None:
    assert _integrate(name, 16) < _integrate("euler", 16)


def test_euler_is_first_order() -> None:
    e1, e2 = _integrate("euler", 32), _integrate("euler", 64)
    assert 1.7 < e1 / e2 < 2.3


def test_heun_is_second_order() -> None:
    # halving the step should cut the error by ~4 (allow 2.5: the final step drops to first order)
    e1, e2 = _integrate("heun", 16), _integrate("heun", 32)
    assert e1 / e2 > 2.5


@pytest.mark.parametrize("schedule", ["linear", "karras", "linear_quadratic"])
def test_euler_converges_on_every_schedule(schedule: str) -> None:
    assert _integrate("euler", 48, schedule) < 0.08


@pytest.mark.parametrize("name", ["euler", "heun", "dpmpp_2m", "res_multistep", "euler_ancestral"])
def test_point_mass_flow_is_exact_for_first_step_forms(name: str) -> None:
    # data is a single point x0: the velocity (x - x0) / t is exact and every solver lands on x0
    x0 = torch.tensor([0.3, -1.2, 2.0], dtype=torch.float64)
    sampler = build_sampler(name)
    x = torch.tensor([1.0, 0.5, -0.7], dtype=torch.float64)
    for _, s, s_next in build_sigma_schedule(ScheduleConfig(steps=6)):
        v = (x - x0) / s
        x = sampler.step(v, x, s, s_next, denoise=lambda y, t: (y - x0) / t)
    torch.testing.assert_close(x, x0, atol=1e-9, rtol=0)


@pytest.mark.parametrize("name", ["dpmpp_2m", "res_multistep"])
def test_multistep_reset_restarts_history(name: str) -> None:
    sampler = build_sampler(name)
    x = torch.ones(4, dtype=torch.float64)
    first = sampler.step(_velocity(x, 0.9), x, 0.9, 0.8)
    sampler.step(_velocity(first, 0.8), first, 0.8, 0.7)
    sampler.reset()
    again = sampler.step(_velocity(x, 0.9), x, 0.9, 0.8)
    torch.testing.assert_close(first, again)


@pytest.mark.parametrize("name", ["euler", "heun", "dpmpp_2m", "res_multistep", "euler_ancestral"])
@pytest.mark.parametrize("sigmas", [(0.5, 0.5), (0.3, 0.6), (float("nan"), 0.1), (0.5, float("inf"))])
def test_samplers_reject_non_decreasing_or_non_finite_steps(name: str, sigmas: tuple[float, float]) -> None:
    x = torch.zeros(2)
    with pytest.raises(ValueError):
        build_sampler(name).step(x, x, *sigmas, denoise=lambda y, t: y)


def test_heun_needs_denoiser_except_on_final_step() -> None:
    heun = build_sampler("heun")
    x = torch.ones(3)
    with pytest.raises(ValueError, match="denoise"):
        heun.step(x, x, 0.5, 0.25)
    torch.testing.assert_close(heun.step(x, x, 0.5, 0.0), x - 0.5 * x)
    assert heun.evaluations_per_step == 2
    assert build_sampler("euler").evaluations_per_step == 1


@pytest.mark.parametrize("eta", [0.0, 0.3, 1.0])
@pytest.mark.parametrize("s,s_next", [(1.0, 0.5), (0.8, 0.7), (0.4, 0.1), (0.5, 0.0)])
def test_ancestral_split_preserves_marginal_scale(eta: float, s: float, s_next: float) -> None:
    sampler = EulerAncestralSampler(SamplerConfig(name="euler_ancestral", eta=eta))
    down, up = sampler.ancestral_split(s, s_next)
    assert math.isclose(down * down + up * up, s_next * s_next, rel_tol=1e-9, abs_tol=1e-12)
    assert 0.0 <= up <= s_next and 0.0 <= down <= s_next + 1e-12
    if eta == 0.0 or s_next == 0.0:
        assert up == 0.0 and down == s_next
    assert sampler.is_stochastic == (eta > 0.0)


def test_ancestral_noise_is_reproducible_and_reported() -> None:
    sampler = EulerAncestralSampler(SamplerConfig(name="euler_ancestral", eta=1.0))
    x = torch.zeros(16)
    v = torch.ones(16)
    a, noise_a, up = sampler.step_with_noise(v, x, 0.8, 0.5, generator=torch.Generator().manual_seed(3))
    b, noise_b, _ = sampler.step_with_noise(v, x, 0.8, 0.5, generator=torch.Generator().manual_seed(3))
    torch.testing.assert_close(a, b)
    torch.testing.assert_close(noise_a, noise_b)
    down, up2 = sampler.ancestral_split(0.8, 0.5)
    assert up == up2 > 0
    torch.testing.assert_close(a, x + (down - 0.8) * v + up * noise_a)
    with pytest.raises(ValueError, match="Generator"):
        sampler.step_with_noise(v, x, 0.8, 0.5)
    given = torch.full((16,), 2.0)
    c, n, _ = sampler.step_with_noise(v, x, 0.8, 0.5, noise=given)
    assert n is given


@pytest.mark.parametrize("sigma", [0.0, 0.25, 0.5, 1.0])
def test_x0_and_epsilon_invert_the_path(sigma: float) -> None:
    g = torch.Generator().manual_seed(1)
    x0, eps = torch.randn(8, generator=g, dtype=torch.float64), torch.randn(8, generator=g, dtype=torch.float64)
    x_t = (1 - sigma) * x0 + sigma * eps
    v = eps - x0
    torch.testing.assert_close(to_x0(x_t, v, sigma), x0)
    torch.testing.assert_close(to_epsilon(x_t, v, sigma), eps)


@pytest.mark.parametrize("kw", [{"name": ""}, {"name": " euler"}, {"eta": -0.1}, {"eta": 1.5},
                                {"eta": float("nan")}, {"s_noise": -1.0}, {"s_noise": float("inf")}])
def test_sampler_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        SamplerConfig(**kw)


def test_sampler_config_round_trip_and_registry() -> None:
    cfg = SamplerConfig(name="euler_ancestral", eta=0.5, s_noise=0.9, lower_order_final=False)
    assert SamplerConfig.from_dict({**cfg.to_dict(), "ignored": 1}) == cfg
    names = list_samplers()
    for n in ("euler", "heun", "dpmpp_2m", "res_multistep", "euler_ancestral"):
        assert n in names
    with pytest.raises(KeyError, match="unknown sampler"):
        build_sampler("plms")
    with pytest.raises(ValueError, match="already registered"):
        register_sampler("euler")
    with pytest.raises(ValueError):
        register_sampler(" padded")


# ----------------------------------------------------------------------------- schedules


@pytest.mark.parametrize("name", ["linear", "karras", "linear_quadratic"])
@pytest.mark.parametrize("steps", [1, 2, 5, 30, 100])
def test_schedule_invariants(name: str, steps: int) -> None:
    sig = build_sigma_schedule(ScheduleConfig(name=name, steps=steps))
    s = sig.sigmas
    assert s.numel() == steps + 1 and len(sig) == steps == sig.num_steps
    assert float(s[-1]) == 0.0 and float(s[0]) <= 1.0
    assert bool((s[1:] < s[:-1]).all())
    assert sig.timesteps().numel() == steps
    assert [i for i, _, _ in sig] == list(range(steps))
    assert sig.tolist() == pytest.approx(s.tolist())


@pytest.mark.parametrize("shift", [0.5, 1.0, 2.0, 3.0, 7.0])
def test_shift_is_monotone_and_fixes_endpoints(shift: float) -> None:
    t = torch.linspace(0.0, 1.0, 101, dtype=torch.float64)
    out = apply_shift(t, shift)
    assert float(out[0]) == 0.0 and float(out[-1]) == pytest.approx(1.0)
    assert bool((out[1:] > out[:-1]).all())
    if shift > 1.0:
        assert bool((out[1:-1] > t[1:-1]).all())  # more time at high noise
    elif shift < 1.0:
        assert bool((out[1:-1] < t[1:-1]).all())


@pytest.mark.parametrize("shift", [0.0, -1.0, float("nan"), float("inf")])
def test_shift_rejects(shift: float) -> None:
    with pytest.raises(ValueError):
        apply_shift(torch.linspace(0, 1, 5), shift)


@pytest.mark.parametrize("length,expect", [(256, 1.0), (4096, 3.0), (2176, 2.0), (64, 1.0), (100000, 3.0)])
def test_resolution_shift_linear_and_clamped(length: int, expect: float) -> None:
    assert resolution_shift(length) == pytest.approx(expect)


def test_resolution_shift_exponential_and_errors() -> None:
    assert resolution_shift(4096, base_shift=0.5, max_shift=1.15, exponential=True) == pytest.approx(math.exp(1.15))
    for kw in ({"sequence_length": 0}, {"sequence_length": 10, "base_length": 0},
               {"sequence_length": 10, "base_length": 5, "max_length": 5}):
        with pytest.raises(ValueError):
            resolution_shift(**kw)


def test_dynamic_shift_grows_with_tokens() -> None:
    cfg = ScheduleConfig(steps=10, dynamic_shift=True)
    short = build_sigma_schedule(cfg, sequence_length=256)
    long = build_sigma_schedule(cfg, sequence_length=4096)
    assert long.shift > short.shift
    assert bool((long.sigmas[1:-1] >= short.sigmas[1:-1]).all())
    with pytest.raises(ValueError, match="sequence_length"):
        build_sigma_schedule(cfg)
    assert float(long.sigmas[-1]) == 0.0


def test_linear_sigmas_forms() -> None:
    torch.testing.assert_close(linear_sigmas(4), torch.tensor([1.0, 0.75, 0.5, 0.25, 0.0]))
    torch.testing.assert_close(linear_sigmas(1), torch.tensor([1.0, 0.0]))
    torch.testing.assert_close(linear_sigmas(2, sigma_max=0.8, sigma_min=0.2), torch.tensor([0.8, 0.2, 0.0]))
    for kw in ({"steps": 0}, {"steps": 3, "sigma_max": 1.5}, {"steps": 3, "sigma_min": 0.0},
               {"steps": 3, "sigma_max": 0.5, "sigma_min": 0.6}):
        with pytest.raises(ValueError):
            linear_sigmas(**kw)


@pytest.mark.parametrize("rho", [1.0, 3.0, 7.0])
def test_karras_sigmas_endpoints_and_rho(rho: float) -> None:
    s = karras_sigmas(10, sigma_min=0.01, rho=rho)
    assert float(s[0]) == pytest.approx(1.0) and float(s[-2]) == pytest.approx(0.01, rel=1e-5)
    if rho == 1.0:
        torch.testing.assert_close(s[:-1], torch.linspace(1.0, 0.01, 10))
    with pytest.raises(ValueError):
        karras_sigmas(5, rho=0.0)


def test_karras_concentrates_steps_at_low_noise() -> None:
    lin = linear_sigmas(20, sigma_min=0.002)
    kar = karras_sigmas(20)
    assert int((kar < 0.1).sum()) > int((lin < 0.1).sum())


@pytest.mark.parametrize("steps,linear", [(10, None), (10, 3), (4, 1), (30, 29)])
def test_linear_quadratic_sigmas(steps: int, linear: int | None) -> None:
    s = linear_quadratic_sigmas(steps, linear_steps=linear, threshold_noise=0.05)
    assert s.numel() == steps + 1 and float(s[0]) == pytest.approx(1.0) and float(s[-1]) == 0.0
    n_lin = linear if linear is not None else steps // 2
    tail = s.flip(0)[:n_lin + 1]  # the first n_lin + 1 rising values are the linear ramp to the threshold
    torch.testing.assert_close(tail, torch.linspace(0.0, 0.05, n_lin + 1), atol=1e-6, rtol=0)


@pytest.mark.parametrize("kw", [{"linear_steps": 0}, {"linear_steps": 10}, {"threshold_noise": 0.0},
                                {"threshold_noise": 1.0}])
def test_linear_quadratic_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        linear_quadratic_sigmas(10, **kw)


@pytest.mark.parametrize("values", [[1.0], [1.0, 0.5], [1.0, 0.5, 0.5, 0.0], [1.2, 0.5, 0.0], [1.0, 0.5, 0.1],
                                    [1.0, float("nan"), 0.0]])
def test_sigma_schedule_rejects(values: list[float]) -> None:
    with pytest.raises(ValueError):
        SigmaSchedule(torch.tensor(values))


def test_sigma_schedule_rejects_integer_and_2d() -> None:
    with pytest.raises(ValueError):
        SigmaSchedule(torch.tensor([1, 0]))
    with pytest.raises(ValueError):
        SigmaSchedule(torch.tensor([[1.0, 0.0]]))


def test_schedule_config_round_trip_registry_and_device() -> None:
    cfg = ScheduleConfig(name="karras", steps=12, shift=2.0, rho=5.0, sigma_min=0.01)
    assert ScheduleConfig.from_dict({**cfg.to_dict(), "extra": 1}) == cfg
    sig = build_sigma_schedule(cfg)
    assert sig.shift == 2.0 and sig.name == "karras" and sig.to("cpu").device.type == "cpu"
    assert set(list_sigma_schedules()) >= {"linear", "karras", "linear_quadratic"}
    with pytest.raises(KeyError):
        build_sigma_schedule(ScheduleConfig(name="cosine"))
    with pytest.raises(ValueError):
        register_sigma_schedule("linear")
    for kw in ({"name": ""}, {"steps": 0}, {"shift": 0.0}):
        with pytest.raises(ValueError):
            ScheduleConfig(**kw)


# ----------------------------------------------------------------------------- guidance


def _pair(seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(3, 4, 5, generator=g, dtype=torch.float64), torch.randn(3, 4, 5, generator=g,
                                                                                 dtype=torch.float64)


@pytest.mark.parametrize("scale", [0.0, 1.0, 2.5, 7.5])
def test_cfg_formula(scale: float) -> None:
    c, u = _pair()
    torch.testing.assert_close(classifier_free_guidance(c, u, scale), u + scale * (c - u))


def test_cfg_rejects_mismatched_branches() -> None:
    c, _ = _pair()
    with pytest.raises(ValueError, match="shape"):
        classifier_free_guidance(c, c[:1], 3.0)


@pytest.mark.parametrize("factor", [0.0, 0.5, 1.0])
def test_rescale_matches_conditional_std(factor: float) -> None:
    c, u = _pair(1)
    guided = classifier_free_guidance(c, u, 5.0)
    out = rescale_guidance(guided, c, factor)
    dims = (1, 2)
    if factor == 1.0:
        torch.testing.assert_close(out.std(dim=dims), c.std(dim=dims))
    elif factor == 0.0:
        torch.testing.assert_close(out, guided)
    else:
        lo, hi = sorted((float(c.std()), float(guided.std())))
        assert lo - 1e-6 <= float(out.std()) <= hi + 1e-6
    with pytest.raises(ValueError):
        rescale_guidance(guided, c, 1.5)


def test_apg_orthogonal_decomposition() -> None:
    c, u = _pair(2)
    diff = c - u
    dims = (1, 2)
    coef = (diff * c).sum(dims, keepdim=True) / (c * c).sum(dims, keepdim=True)
    parallel, orth = coef * c, diff - coef * c
    torch.testing.assert_close((orth * c).sum(dims), torch.zeros(3, dtype=torch.float64), atol=1e-10, rtol=0)
    # eta = 1 keeps both parts: plain CFG
    torch.testing.assert_close(adaptive_projected_guidance(c, u, 4.0, eta=1.0), classifier_free_guidance(c, u, 4.0))
    torch.testing.assert_close(adaptive_projected_guidance(c, u, 4.0, eta=0.0), c + 3.0 * orth)
    torch.testing.assert_close(adaptive_projected_guidance(c, u, 1.0), c)
    assert parallel.shape == c.shape


def test_apg_norm_threshold_caps_the_update() -> None:
    c, u = _pair(3)
    capped = adaptive_projected_guidance(c, u, 2.0, eta=1.0, norm_threshold=0.1)
    update = capped - c
    norms = torch.linalg.vector_norm(update, dim=(1, 2))
    assert bool((norms <= 0.1 + 1e-9).all())
    with pytest.raises(ValueError):
        adaptive_projected_guidance(c, u, 2.0, norm_threshold=-1.0)


@pytest.mark.parametrize("schedule,progress,expect", [
    ("constant", 0.7, 6.0), ("linear", 0.0, 6.0), ("linear", 1.0, 1.0), ("linear", 0.5, 3.5),
    ("cosine", 0.0, 6.0), ("cosine", 1.0, 1.0), ("cosine", 0.5, 3.5), ("power", 0.5, 1.0 + 5.0 * 0.25),
    ("interval", 0.1, 1.0), ("interval", 0.5, 6.0), ("interval", 0.95, 1.0),
])
def test_guidance_scale_schedules(schedule: str, progress: float, expect: float) -> None:
    cfg = GuidanceConfig(scale=6.0, schedule=schedule, schedule_power=2.0, start_fraction=0.2, end_fraction=0.8)
    assert cfg.scale_at(progress) == pytest.approx(expect)


@pytest.mark.parametrize("kw", [{"scale": 0.0}, {"scale": -1.0}, {"text_scale": 0.0}, {"rescale": 1.5},
                                {"projection_eta": float("nan")}, {"projection_threshold": -1.0},
                                {"schedule": "step"}, {"start_fraction": 1.5}, {"start_fraction": 0.5,
                                                                               "end_fraction": 0.5},
                                {"schedule_power": 0.0}])
def test_guidance_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        GuidanceConfig(**kw)


def test_guidance_config_enabled_modalities_and_round_trip() -> None:
    assert not GuidanceConfig().is_enabled
    assert GuidanceConfig(scale=2.0).is_enabled
    assert GuidanceConfig(audio_scale=1.5).is_enabled
    cfg = GuidanceConfig(scale=4.0, text_scale=1.5, audio_scale=0.5)
    assert cfg.modality_scale("text") == pytest.approx(6.0)
    assert cfg.modality_scale("audio") == pytest.approx(2.0)
    assert cfg.modality_scale("video") == pytest.approx(4.0)
    with pytest.raises(ValueError):
        cfg.modality_scale("depth")
    with pytest.raises(ValueError):
        cfg.scale_at(1.5)
    assert GuidanceConfig.from_dict({**cfg.to_dict(), "junk": 1}) == cfg


def test_apply_guidance_paths() -> None:
    c, u = _pair(4)
    assert apply_guidance(c) is c
    assert apply_guidance(c, u, config=GuidanceConfig()) is c
    cfg = GuidanceConfig(scale=3.0)
    torch.testing.assert_close(apply_guidance(c, u, config=cfg), classifier_free_guidance(c, u, 3.0))
    with pytest.raises(ValueError, match="unconditional"):
        apply_guidance(c, None, config=cfg)
    assert apply_guidance(c, u, config=cfg, scale=1.0) is c
    proj = GuidanceConfig(scale=3.0, projection=True, projection_eta=0.0)
    torch.testing.assert_close(apply_guidance(c, u, config=proj), adaptive_projected_guidance(c, u, 3.0))
    res = GuidanceConfig(scale=3.0, rescale=1.0)
    torch.testing.assert_close(apply_guidance(c, u, config=res).std(dim=(1, 2)), c.std(dim=(1, 2)))


def test_modality_guidance_chains_conditions() -> None:
    g = torch.Generator().manual_seed(5)
    base, text, both = (torch.randn(2, 6, generator=g, dtype=torch.float64) for _ in range(3))
    cfg = GuidanceConfig(scale=2.0, text_scale=1.5, audio_scale=0.5)
    out = apply_modality_guidance([("none", base), ("text", text), ("audio", both)], config=cfg)
    torch.testing.assert_close(out, base + 3.0 * (text - base) + 1.0 * (both - text))
    with pytest.raises(ValueError):
        apply_modality_guidance([("text", base)], config=cfg)
