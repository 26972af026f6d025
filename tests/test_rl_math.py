"""Post-training mathematics on CPU against closed forms: the marginal-preserving
SDE (its Gaussian log-density, its ODE limit, marginal preservation on an exact
Gaussian flow), the GRPO surrogate, KL estimator, advantages, MixGRPO windows,
the DPO losses and the reward normalisers (reference test strategy:
tests/test_rl.py -- per-formula cases and config validation)."""
from __future__ import annotations

import math

import pytest
import torch

from avgen_b200.rl.dpo import DPOConfig, dpo_loss
from avgen_b200.rl.grpo import GRPOConfig, WindowSchedule, clipped_surrogate, kl_penalty, regulated_log_ratio
from avgen_b200.rl.rewards import (AVSyncProxyReward, CompositeReward, MotionMagnitudeReward, RunningNormalizer,
                                   TemporalConsistencyReward, build_reward, list_rewards, media_tensors,
                                   register_reward)
from avgen_b200.rl.rollout import RolloutBuffer, distribute_prompts, gather_rewards, group_advantages
from avgen_b200.rl.sde import SDEStep, diffusion_coefficient, gaussian_log_prob, ode_step, to_sde

# ----------------------------------------------------------------------------- SDE


@pytest.mark.parametrize("level", [0.1, 0.5, 0.9])
@pytest.mark.parametrize("a", [0.3, 0.7, 1.0])
def test_diffusion_coefficient_forms(level: float, a: float) -> None:
    s = torch.tensor([level])
    torch.testing.assert_close(diffusion_coefficient(s, noise_level=a), torch.tensor([a * math.sqrt(level / (1 - level))]))
    torch.testing.assert_close(diffusion_coefficient(s, noise_level=a, schedule="constant"), torch.tensor([a]))


def test_diffusion_coefficient_clamps_and_rejects() -> None:
    g = diffusion_coefficient(torch.tensor([0.0, 1.0]), noise_level=1.0, floor=0.01)
    assert bool(torch.isfinite(g).all()) and float(g[0]) == pytest.approx(math.sqrt(0.01 / 0.99))
    for kw in ({"noise_level": -0.1}, {"noise_level": 0.5, "floor": 0.0}, {"noise_level": 0.5, "floor": 1.0},
               {"noise_level": 0.5, "schedule": "cosine"}):
        with pytest.raises(ValueError):
            diffusion_coefficient(torch.tensor([0.5]), **kw)


@pytest.mark.parametrize("std", [0.1, 1.0, 3.0])
def test_gaussian_log_prob_matches_torch_normal(std: float) -> None:
    g = torch.Generator().manual_seed(0)
    value = torch.randn(3, 4, 5, generator=g, dtype=torch.float64)
    mean = torch.randn(3, 4, 5, generator=g, dtype=torch.float64)
    sig = torch.full((3,), std, dtype=torch.float64)
    ref = torch.distributions.Normal(mean, std).log_prob(value).flatten(1).sum(1)
    torch.testing.assert_close(gaussian_log_prob(value, mean, sig), ref)
    mask = torch.zeros(3, 4, 5, dtype=torch.float64)
    mask[:, :2] = 1
    ref_masked = torch.distributions.Normal(mean, std).log_prob(value)[:, :2].flatten(1).sum(1)
    torch.testing.assert_close(gaussian_log_prob(value, mean, sig, mask=mask), ref_masked)
    with pytest.raises(ValueError):
        gaussian_log_prob(value, mean[:, :1], sig)


def test_ode_step_is_euler() -> None:
    v, x = torch.ones(2, 3), torch.zeros(2, 3)
    out = ode_step(v, x, torch.tensor([0.8, 0.5]), torch.tensor([0.6, 0.1]))
    torch.testing.assert_close(out, torch.tensor([[-0.2] * 3, [-0.4] * 3]))


def test_sde_noise_level_zero_is_the_ode() -> None:
    g = torch.Generator().manual_seed(1)
    v, x = torch.randn(2, 8, generator=g), torch.randn(2, 8, generator=g)
    s, sn = torch.tensor([0.7, 0.7]), torch.tensor([0.6, 0.6])
    step = to_sde(v, x, s, sn, noise_level=0.0)
    assert step.deterministic and isinstance(step, SDEStep)
    torch.testing.assert_close(step.sample, ode_step(v, x, s, sn))
    assert bool((step.log_prob == 0).all())


def test_sde_scores_its_own_draw_and_rescoring_matches() -> None:
    g = torch.Generator().manual_seed(2)
    v, x = torch.randn(4, 16, generator=g), torch.randn(4, 16, generator=g)
    s, sn = torch.full((4,), 0.6), torch.full((4,), 0.5)
    step = to_sde(v, x, s, sn, generator=torch.Generator().manual_seed(3))
    again = to_sde(v, x, s, sn, prev_sample=step.sample)
    torch.testing.assert_close(again.log_prob, step.log_prob)
    assert again.sample is step.sample
    ref = torch.distributions.Normal(step.mean, step.std[:, None]).log_prob(step.sample).sum(1)
    torch.testing.assert_close(step.log_prob, ref, rtol=1e-5, atol=1e-4)
    # a different velocity scores the same sample lower on average (the draw came from the first policy)
    other = to_sde(v + 0.5, x, s, sn, prev_sample=step.sample)
    assert float(other.log_prob.mean()) < float(step.log_prob.mean())


def test_sde_validates_inputs() -> None:
    x = torch.zeros(2, 4)
    with pytest.raises(ValueError, match="sigma_next"):
        to_sde(x, x, torch.tensor([0.5, 0.5]), torch.tensor([0.6, 0.4]))
    with pytest.raises(ValueError, match="prev_sample"):
        to_sde(x, x, torch.tensor([0.5, 0.5]), torch.tensor([0.4, 0.4]), prev_sample=torch.zeros(2, 5))


@pytest.mark.parametrize("s,s_next", [(0.8, 0.79), (0.5, 0.49), (0.3, 0.29)])
def test_sde_preserves_gaussian_marginals(s: float, s_next: float) -> None:
    # data ~ N(0, c^2): x_s ~ N(0, V(s)); one SDE step with the exact velocity keeps the variance on V(s_next)
    c = 0.5
    n = 200_000
    g = torch.Generator().manual_seed(4)

    def var(t: float) -> float:
        return (1 - t) ** 2 * c * c + t * t

    x = torch.randn(n, 1, generator=g, dtype=torch.float64) * math.sqrt(var(s))
    v = (s - (1 - s) * c * c) * x / var(s)
    step = to_sde(v.float(), x.float(), torch.full((n,), s), torch.full((n,), s_next), noise_level=0.7,
                  generator=torch.Generator().manual_seed(5))
    got = float(step.sample.double().var())
    assert got == pytest.approx(var(s_next), rel=0.02)
    # the ODE step keeps it as well (to first order in the step)
    ode = ode_step(v, x, torch.full((n,), s, dtype=torch.float64), torch.full((n,), s_next, dtype=torch.float64))
    assert float(ode.var()) == pytest.approx(var(s_next), rel=0.02)


# ----------------------------------------------------------------------------- GRPO


@pytest.mark.parametrize("log_ratio,adv,expect_clipped", [
    (0.0, 1.0, False), (0.5, 1.0, True), (-0.5, -1.0, True), (0.05, 1.0, False), (-0.05, 2.0, False),
])
def test_clipped_surrogate_formula(log_ratio: float, adv: float, expect_clipped: bool) -> None:
    lr, a = torch.tensor([log_ratio]), torch.tensor([adv])
    loss, frac, ratio = clipped_surrogate(lr, a, clip_low=0.2, clip_high=0.2)
    r = math.exp(log_ratio)
    expect = -min(r * adv, min(max(r, 0.8), 1.2) * adv)
    assert float(loss) == pytest.approx(expect)
    assert bool(frac > 0) == expect_clipped
    torch.testing.assert_close(ratio, torch.exp(lr))


def test_clipped_surrogate_weights_and_gradient() -> None:
    lr = torch.zeros(4, requires_grad=True)
    adv = torch.tensor([1.0, -1.0, 2.0, 0.5])
    w = torch.tensor([1.0, 2.0, 0.5, 1.0])
    loss, _, _ = clipped_surrogate(lr, adv, clip_low=0.1, clip_high=0.3, weights=w)
    loss.backward()
    # at ratio 1 (inside the clip range) d(-mean(r A w))/d log r = -A w / n
    torch.testing.assert_close(lr.grad, -(adv * w) / 4)


def test_clipped_surrogate_stops_gradient_outside_the_range() -> None:
    lr = torch.tensor([1.0], requires_grad=True)  # ratio e, beyond 1 + 0.2 with a positive advantage
    loss, frac, _ = clipped_surrogate(lr, torch.tensor([1.0]), clip_low=0.2, clip_high=0.2)
    loss.backward()
    assert float(lr.grad) == 0.0 and float(frac) == 1.0


@pytest.mark.parametrize("d", [-2.0, -0.5, 0.0, 0.3, 1.5])
def test_kl_k3_estimator(d: float) -> None:
    k = kl_penalty(torch.tensor([0.0]), torch.tensor([d]))
    assert float(k) == pytest.approx(math.exp(d) - d - 1.0)
    assert float(k) >= 0.0
    assert (float(k) == 0.0) == (d == 0.0)


def test_kl_k3_is_unbiased_for_gaussians() -> None:
    # E_{x ~ p}[exp(log q - log p) - (log q - log p) - 1] = KL(p || q)
    g = torch.Generator().manual_seed(6)
    x = torch.randn(400_000, generator=g, dtype=torch.float64)
    p, q = torch.distributions.Normal(0.0, 1.0), torch.distributions.Normal(0.3, 1.2)
    est = float(kl_penalty(p.log_prob(x), q.log_prob(x)).mean())
    exact = float(torch.distributions.kl_divergence(p, q))
    assert est == pytest.approx(exact, rel=0.03)


def test_regulated_log_ratio_properties() -> None:
    g = torch.Generator().manual_seed(7)
    mean_old = torch.randn(3, 6, generator=g)
    std = torch.full((3,), 0.5)
    sample = mean_old + 0.5 * torch.randn(3, 6, generator=g)
    torch.testing.assert_close(regulated_log_ratio(mean_old, mean_old, std, sample), torch.zeros(3))
    shift = torch.randn(3, 6, generator=g)
    z = (sample - mean_old) / 0.5
    torch.testing.assert_close(regulated_log_ratio(mean_old + shift, mean_old, std, sample), (shift * z).sum(1))
    mask = torch.zeros(3, 6)
    mask[:, :3] = 1
    torch.testing.assert_close(regulated_log_ratio(mean_old + shift, mean_old, std, sample, mask=mask),
                               (shift * z)[:, :3].sum(1))


@pytest.mark.parametrize("kw", [{"group_size": 1}, {"clip_range": 0.0}, {"clip_range_high": -1.0},
                                {"kl_coefficient": -0.1}, {"noise_level": 0.0}, {"inner_epochs": 0},
                                {"minibatch_size": 0}, {"max_grad_norm": 0.0}])
def test_grpo_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        GRPOConfig(**kw)


def test_grpo_config_high_clip() -> None:
    assert GRPOConfig(clip_range=0.1).high == 0.1
    assert GRPOConfig(clip_range=0.1, clip_range_high=0.3).high == 0.3


@pytest.mark.parametrize("step,start", [(0, 0), (24, 0), (25, 1), (49, 1), (50, 2), (100, 4), (10_000, 6)])
def test_window_schedule_linear(step: int, start: int) -> None:
    w = WindowSchedule(window=4, stride=1, interval=25, total_steps=10)
    assert w.start_for(step) == start
    assert w.steps_for(step) == tuple(range(start, start + 4))


def test_window_schedule_stride_and_exponential() -> None:
    w = WindowSchedule(window=2, stride=3, interval=10, total_steps=10)
    assert [w.start_for(s) for s in (0, 10, 20, 30, 40)] == [0, 3, 6, 8, 8]
    e = WindowSchedule(window=2, stride=1, interval=10, total_steps=8, exponential=True, decay=0.5)
    # moves at steps 10, 15, 17.5, 18.75, 19.75, 20.75 (intervals 10, 5, 2.5, 1.25, then 1)
    assert [e.start_for(s) for s in (9, 10, 14, 15, 17, 18, 19, 20, 21)] == [0, 1, 1, 2, 2, 3, 4, 5, 6]
    assert e.start_for(1000) == 6
    with pytest.raises(ValueError):
        w.start_for(-1)


@pytest.mark.parametrize("kw", [{"window": 0}, {"stride": 0}, {"interval": 0}, {"total_steps": 0},
                                {"window": 5, "total_steps": 4}, {"decay": 0.0}, {"decay": 1.5}])
def test_window_schedule_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        WindowSchedule(**kw)


@pytest.mark.parametrize("group", [2, 4, 8])
def test_group_advantages_are_centred_and_scaled(group: int) -> None:
    g = torch.Generator().manual_seed(group)
    r = torch.randn(3 * group, generator=g) * 3 + 1
    adv = group_advantages(r, group, clip=None).reshape(3, group)
    torch.testing.assert_close(adv.mean(1), torch.zeros(3), atol=1e-5, rtol=0)
    torch.testing.assert_close(adv.std(1, unbiased=False), torch.ones(3), atol=1e-3, rtol=0)
    raw = group_advantages(r, group, normalize_by_std=False, clip=None).reshape(3, group)
    torch.testing.assert_close(raw, r.reshape(3, group) - r.reshape(3, group).mean(1, keepdim=True))


def test_group_advantages_clip_constant_groups_and_errors() -> None:
    r = torch.tensor([0.0, 0.0, 0.0, 100.0, 1.0, 1.0, 1.0, 1.0])
    adv = group_advantages(r, 4, clip=1.5)
    assert float(adv.abs().max()) <= 1.5
    torch.testing.assert_close(adv[4:], torch.zeros(4))  # a constant group carries no signal
    with pytest.raises(ValueError):
        group_advantages(r, 1)
    with pytest.raises(ValueError):
        group_advantages(r, 3)


def test_rollout_buffer_flow() -> None:
    buf = RolloutBuffer(group_size=2)
    assert len(buf) == 0 and buf.num_samples == 0
    x = torch.zeros(4, 3)
    for i in range(3):
        step = SDEStep(sample=x + i + 1, log_prob=torch.zeros(4), mean=x, std=torch.ones(4))
        buf.add_step(step_index=i, sample_before=x + i, step=step, sigma=torch.full((4,), 0.5),
                     sigma_next=torch.full((4,), 0.4))
    assert len(buf) == 3 and buf.num_samples == 4
    with pytest.raises(RuntimeError):
        buf.compute_advantages()
    with pytest.raises(ValueError):
        buf.set_rewards(torch.zeros(3), media=None)
    buf.set_rewards(torch.tensor([1.0, 0.0, 2.0, 4.0]), media=None)
    with pytest.raises(RuntimeError):
        next(buf.iter_minibatches(2))
    adv = buf.compute_advantages(clip=None)
    assert adv.shape == (4,)
    batches = list(buf.iter_minibatches(5, shuffle=False))
    assert [b.size for b in batches] == [5, 5, 2]
    allidx = torch.cat([b.step_index for b in batches])
    assert sorted(allidx.tolist()) == [0] * 4 + [1] * 4 + [2] * 4
    prompt_index = torch.cat([b.prompt_index for b in batches])
    assert prompt_index.tolist()[:4] == [0, 0, 1, 1]
    with pytest.raises(ValueError):
        next(buf.iter_minibatches(0))
    with pytest.raises(ValueError):
        RolloutBuffer(group_size=1)


def test_rollout_buffer_arenas_grow_and_keep_every_step() -> None:
    """Without a capacity hint the arenas double when full; stored rows survive every regrowth
    and a minibatch row maps back to its (step, sample) pair."""
    buf = RolloutBuffer(group_size=2)
    for i in range(5):
        x = torch.full((4, 2), float(i))
        step = SDEStep(sample=x + 0.5, log_prob=torch.full((4,), -float(i)), mean=x, std=torch.ones(4))
        buf.add_step(step_index=10 + i, sample_before=x, step=step, sigma=torch.full((4,), 1.0 - 0.1 * i),
                     sigma_next=torch.full((4,), 0.9 - 0.1 * i))
    assert len(buf) == 5 and buf.transitions("sample_before").shape == (5, 4, 2)
    torch.testing.assert_close(buf.transitions("sample_before")[:, 0, 0], torch.arange(5.0))
    with pytest.raises(KeyError):
        buf.transitions("advantage")
    with pytest.raises(ValueError):  # a step over a different sample count
        buf.add_step(step_index=0, sample_before=torch.zeros(3, 2),
                     step=SDEStep(sample=torch.zeros(3, 2), log_prob=torch.zeros(3), mean=torch.zeros(3, 2),
                                  std=torch.ones(3)), sigma=torch.ones(3), sigma_next=torch.ones(3))
    buf.set_rewards(torch.tensor([0.0, 1.0, 3.0, 5.0]), media=None)
    adv = buf.compute_advantages(clip=None)
    for batch in buf.iter_minibatches(3, generator=torch.Generator().manual_seed(1)):
        step = batch.step_index - 10
        torch.testing.assert_close(batch.sample_before[:, 0], step.float())
        torch.testing.assert_close(batch.log_prob_old, -step.float())
        torch.testing.assert_close(batch.sigma, 1.0 - 0.1 * step.float())
        assert set(batch.prompt_index.tolist()) <= {0, 1}
        assert all(float(a) in adv.tolist() for a in batch.advantage)


def test_rollout_buffer_from_empty_has_no_transitions() -> None:
    with pytest.raises(RuntimeError):
        RolloutBuffer(group_size=3).transitions("sample_before")


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_distribute_prompts_is_a_partition(world: int) -> None:
    prompts = [f"p{i}" for i in range(10)]
    seen: list[int] = []
    for rank in range(world):
        shard, idx = distribute_prompts(prompts, data_rank=rank, data_world=world)
        assert list(shard) == [prompts[i] for i in idx]
        seen += idx
    assert sorted(seen) == list(range(10))
    with pytest.raises(ValueError):
        distribute_prompts(prompts, data_rank=world, data_world=world)


def test_gather_rewards_without_a_group_is_identity() -> None:
    r = torch.arange(3.0)
    assert gather_rewards(r) is r


# ----------------------------------------------------------------------------- DPO


@pytest.mark.parametrize("loss_type", ["sigmoid", "hinge", "ipo"])
@pytest.mark.parametrize("gap", [-0.01, 0.0, 0.01])
def test_dpo_loss_forms(loss_type: str, gap: float) -> None:
    cfg = DPOConfig(beta=100.0, loss_type=loss_type, center_loss=False)
    pw, pl = torch.tensor([0.5 + gap]), torch.tensor([0.5])
    rw, rl = torch.tensor([0.5]), torch.tensor([0.5])
    loss, margin = dpo_loss(pw, pl, rw, rl, cfg)
    m = -100.0 * gap
    assert float(margin) == pytest.approx(m, abs=1e-5)
    expect = {"sigmoid": -math.log(1 / (1 + math.exp(-m))), "hinge": max(0.0, 1.0 - m), "ipo": (m - 0.5) ** 2}
    assert float(loss) == pytest.approx(expect[loss_type], abs=1e-5)


def test_dpo_centering_smoothing_and_beta_scaling() -> None:
    z = torch.zeros(3)
    loss, _ = dpo_loss(z, z, z, z, DPOConfig())
    assert float(loss) == pytest.approx(0.0, abs=1e-6)  # centred at margin 0
    smooth = DPOConfig(beta=1.0, label_smoothing=0.2, center_loss=False)
    m = torch.tensor([2.0])
    loss, _ = dpo_loss(-m, torch.zeros(1), torch.zeros(1), torch.zeros(1), smooth)
    expect = -(0.8 * math.log(1 / (1 + math.exp(-2.0))) + 0.2 * math.log(1 / (1 + math.exp(2.0))))
    assert float(loss) == pytest.approx(expect, rel=1e-5)
    assert DPOConfig(beta=2.0, beta_scales_with_steps=True, timestep_count=10).effective_beta == 20.0
    assert DPOConfig(beta=2.0).effective_beta == 2.0


def test_dpo_policy_matching_reference_has_zero_margin_gradient_direction() -> None:
    pw = torch.tensor([0.3], requires_grad=True)
    pl = torch.tensor([0.3], requires_grad=True)
    loss, _ = dpo_loss(pw, pl, torch.tensor([0.3]), torch.tensor([0.3]), DPOConfig(beta=10.0))
    loss.backward()
    # lowering the winner's error and raising the loser's both reduce the loss
    assert float(pw.grad) > 0 and float(pl.grad) < 0


@pytest.mark.parametrize("kw", [{"beta": 0.0}, {"loss_type": "kto"}, {"label_smoothing": 0.5},
                                {"label_smoothing": -0.1}, {"timestep_count": 0}])
def test_dpo_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        DPOConfig(**kw)


# ----------------------------------------------------------------------------- rewards


def test_running_normalizer_matches_pooled_statistics() -> None:
    g = torch.Generator().manual_seed(8)
    chunks = [torch.randn(n, generator=g) * 2 + 3 for n in (5, 17, 40)]
    norm = RunningNormalizer()
    for c in chunks:
        norm.update(c)
    allv = torch.cat(chunks)
    st = norm.state_dict()
    assert st["count"] == 62
    assert st["mean"] == pytest.approx(float(allv.mean()), rel=1e-5)
    assert st["variance"] == pytest.approx(float(allv.var(unbiased=False)), rel=1e-4)
    out = norm.normalize(allv)
    assert float(out.mean()) == pytest.approx(0.0, abs=1e-4)
    fresh = RunningNormalizer()
    fresh.load_state_dict(st)
    torch.testing.assert_close(fresh.normalize(allv), out)
    with pytest.raises(KeyError):
        fresh.load_state_dict({"count": 1})
    norm.update(torch.empty(0))
    assert norm.state_dict()["count"] == 62


def test_running_normalizer_ema_and_validation() -> None:
    n = RunningNormalizer(momentum=0.5)
    assert torch.equal(n.normalize(torch.ones(2)), torch.ones(2))  # no statistics yet
    n.update(torch.tensor([2.0, 2.0]))
    assert n.state_dict()["mean"] == pytest.approx(1.0)
    for kw in ({"momentum": 0.0}, {"momentum": 1.0}, {"epsilon": 0.0}):
        with pytest.raises(ValueError):
            RunningNormalizer(**kw)


def _video(b: int = 2, t: int = 4, seed: int = 0) -> torch.Tensor:
    return torch.randn(b, 3, t, 4, 4, generator=torch.Generator().manual_seed(seed))


def test_temporal_consistency_reward() -> None:
    static = _video(t=1).repeat(1, 1, 4, 1, 1)
    r = TemporalConsistencyReward().score(static, ["a", "b"])
    torch.testing.assert_close(r, torch.ones(2))
    noisy = TemporalConsistencyReward().score(_video(), ["a", "b"])
    assert bool((noisy < 0.9).all())
    torch.testing.assert_close(TemporalConsistencyReward().score(_video(t=1), ["a", "b"]), torch.ones(2))
    with pytest.raises(ValueError):
        TemporalConsistencyReward().score(_video(), ["a"])


def test_motion_magnitude_reward_peaks_at_target() -> None:
    base = _video(t=1)
    frames = torch.cat([base + 0.1 * i for i in range(4)], dim=2)  # mean |frame difference| is exactly 0.1
    r = MotionMagnitudeReward(target=0.1, tolerance=0.05).score(frames, ["a", "b"])
    torch.testing.assert_close(r, torch.ones(2))
    far = MotionMagnitudeReward(target=1.0, tolerance=0.05).score(frames, ["a", "b"])
    assert bool((far < 1e-3).all())
    with pytest.raises(ValueError):
        MotionMagnitudeReward(tolerance=0.0)
    with pytest.raises(ValueError):
        MotionMagnitudeReward(target=-1.0)


def test_av_sync_proxy_reward() -> None:
    video = _video(b=1, t=9)
    motion = (video[:, :, 1:] - video[:, :, :-1]).abs().mean((1, 3, 4))  # [1, 8]
    audio = motion[:, None, :].repeat(1, 2, 1)  # [B, channels, time] following the motion exactly
    r = AVSyncProxyReward().score({"video": video, "audio": audio}, ["x"])
    assert float(r) == pytest.approx(1.0, abs=1e-4)
    inverse = (motion.max() - motion)[:, None, :].repeat(1, 2, 1)  # loud where the picture is still
    anti = AVSyncProxyReward().score({"video": video, "audio": inverse}, ["x"])
    assert float(anti) == pytest.approx(-1.0, abs=1e-4)
    assert float(AVSyncProxyReward().score(video, ["x"])) == 0.0  # no audio


def test_media_tensors_forms() -> None:
    v = _video()
    assert media_tensors(v)[0] is v
    assert media_tensors({"video": v})[0] is v

    class M:
        video = v
        audio = None

    assert media_tensors(M())[1] is None
    with pytest.raises(TypeError):
        media_tensors({"audio": v})
    with pytest.raises(ValueError):
        media_tensors(v[0])


def test_reward_registry_and_composite() -> None:
    names = list_rewards()
    for n in ("temporal_consistency", "motion_magnitude", "av_sync_proxy", "mlp_scorer"):
        assert n in names
    with pytest.raises(KeyError):
        build_reward("aesthetic_v9")
    with pytest.raises(KeyError):
        register_reward("temporal_consistency")(TemporalConsistencyReward)
    comp = CompositeReward(((TemporalConsistencyReward(), 1.0), (MotionMagnitudeReward(), 2.0)), normalization="none")
    v = _video()
    parts = comp.component_scores(v, ["a", "b"])
    torch.testing.assert_close(comp.score(v, ["a", "b"]), parts["temporal_consistency"] + 2 * parts["motion_magnitude"])
    batch = CompositeReward(((TemporalConsistencyReward(), 1.0),), normalization="batch")
    out = batch.score(torch.cat([_video(seed=i) for i in range(4)]), list("abcdefgh"))
    assert float(out.mean()) == pytest.approx(0.0, abs=1e-5)
    running = CompositeReward(((TemporalConsistencyReward(), 1.0),), normalization="running")
    running.score(v, ["a", "b"])
    st = running.state_dict()
    assert st["component_0"]["count"] == 2
    running.load_state_dict(st)
    with pytest.raises(KeyError):
        running.load_state_dict({})
    with pytest.raises(ValueError):
        CompositeReward(())
    with pytest.raises(ValueError):
        CompositeReward(((TemporalConsistencyReward(), 1.0),), normalization="rank")
