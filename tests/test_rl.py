"""RL post-training on CPU: SDE transitions, advantages, GRPO / DPO losses and
updates on a tiny model, rewards, and ``avgen-b200 rl`` end to end
(reference test strategy: tests/test_rl.py:185, :258, :1555)."""
from __future__ import annotations

import json
import math
from dataclasses import asdict
from pathlib import Path

import pytest
import torch

from avgen_b200.rl import (CompositeReward, DPOConfig, GRPOConfig, GRPOTrainer, MLPScorerReward, RunningNormalizer,
                           WindowSchedule, build_reward, clipped_surrogate, diffusion_coefficient, dpo_loss,
                           gaussian_log_prob, generate_group, group_advantages, kl_penalty, list_rewards,
                           model_velocity_fn, ode_step, regulated_log_ratio, to_sde)


def test_sde_reduces_to_ode_and_scores_its_own_draw() -> None:
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 4, 2, 4, 4, generator=g)
    v = torch.randn(3, 4, 2, 4, 4, generator=g)
    s, sn = torch.tensor([0.9, 0.5, 0.3]), torch.tensor([0.8, 0.45, 0.1])
    det = to_sde(v, x, s, sn, noise_level=0.0)
    assert det.deterministic and torch.equal(det.sample, ode_step(v, x, s, sn))
    assert torch.count_nonzero(det.log_prob) == 0
    roll = to_sde(v, x, s, sn, noise_level=0.7, generator=torch.Generator().manual_seed(1))
    upd = to_sde(v, x, s, sn, noise_level=0.7, prev_sample=roll.sample)
    torch.testing.assert_close(upd.log_prob, roll.log_prob, rtol=1e-5, atol=1e-3)
    torch.testing.assert_close(upd.mean, roll.mean)
    # mean: x + (v + g^2/(2s) (x + (1-s) v)) ds ; log-density of an isotropic Gaussian
    gc = diffusion_coefficient(s, noise_level=0.7)
    sb = s.view(3, 1, 1, 1, 1)
    mean = x + (v + (gc ** 2).view(3, 1, 1, 1, 1) / (2 * sb) * (x + (1 - sb) * v)) * (sn - s).view(3, 1, 1, 1, 1)
    torch.testing.assert_close(roll.mean, mean)
    std = gc * (s - sn).sqrt()
    n = x[0].numel()
    z = ((roll.sample - mean) / std.view(3, 1, 1, 1, 1)).flatten(1)
    want = -0.5 * (z ** 2).sum(1) - n * torch.log(std) - n * 0.5 * math.log(2 * math.pi)
    torch.testing.assert_close(roll.log_prob, want, rtol=1e-5, atol=1e-3)
    torch.testing.assert_close(gaussian_log_prob(roll.sample, mean, std), want, rtol=1e-5, atol=1e-3)
    with pytest.raises(ValueError):
        to_sde(v, x, sn, s)


def test_advantages_window_surrogate_kl() -> None:
    r = torch.tensor([1.0, 2.0, 3.0, 4.0, 0.0, 0.0, 0.0, 0.0])
    a = group_advantages(r, 4)
    torch.testing.assert_close(a[:4].mean(), torch.tensor(0.0), atol=1e-6, rtol=0)
    assert torch.all(a[4:] == 0)
    with pytest.raises(ValueError):
        group_advantages(r, 3)
    w = WindowSchedule(window=4, stride=1, interval=2, total_steps=10)
    assert w.steps_for(0) == (0, 1, 2, 3) and w.steps_for(5) == (2, 3, 4, 5) and w.steps_for(100) == (6, 7, 8, 9)
    assert WindowSchedule(window=2, interval=4, total_steps=6, exponential=True, decay=0.5).start_for(7) == 3
    lr = torch.log(torch.tensor([0.5, 1.0, 2.0]))
    adv = torch.tensor([1.0, 1.0, -1.0])
    loss, frac, ratio = clipped_surrogate(lr, adv, clip_low=0.2, clip_high=0.2)
    assert float(loss) == pytest.approx(-(0.5 + 1.0 - 2.0) / 3)
    torch.testing.assert_close(frac, torch.tensor(2 / 3))
    assert float(kl_penalty(torch.tensor(0.3), torch.tensor(0.3))) == 0.0
    x = torch.randn(2, 8)
    assert torch.all(regulated_log_ratio(x, x, torch.ones(2), x + 1) == 0)


def _tiny_model() -> torch.nn.Module:
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    cfg.update(depth=1, width=32, num_heads=2, in_channels=4, text_width=8)
    m = build_model("video_dit", cfg)
    m.init_weights()
    with torch.no_grad():  # non-zero output head so the policy is not identically zero
        for p in m.final_proj.parameters():
            p.normal_(0, 0.02)
    return m


def test_grpo_rollout_and_update_with_reference_snapshot() -> None:
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.train import build_optimizer

    model = _tiny_model()
    ref = GRPOTrainer.snapshot_reference(model)
    assert not any(p.requires_grad for p in ref.parameters())
    opt = build_optimizer(model, lr=1e-3)
    state = TrainState(model=model, optimizer=opt, rng=RNGStreams.from_seed(0))
    feats = torch.randn(2, 3, 8)
    tmask = torch.ones(2, 3, dtype=torch.bool)
    common = dict(patchifier=model.patchifier, positions=torch.arange(2.0)[None] / 8, mask=torch.ones(1, 2, 8, 8,
                  dtype=torch.bool), text_features=feats, text_mask=tmask, guidance=3.0)
    vel = model_velocity_fn(model, **common)
    cfg = GRPOConfig(group_size=4, clip_range=0.2, kl_coefficient=0.04, minibatch_size=4,
                     window=WindowSchedule(window=2, total_steps=4))
    trainer = GRPOTrainer(state, vel, cfg, reference_velocity_fn=model_velocity_fn(ref, **common))
    with pytest.raises(ValueError):
        GRPOTrainer(state, vel, cfg)
    sig = torch.linspace(1.0, 0.0, 5)
    before = [p.detach().clone() for p in model.parameters()]
    buf = trainer.rollout(["a", "b"], sigmas=sig, latent_shape=(4, 2, 8, 8), reward=MLPScorerReward(channels=4))
    assert len(buf) == 2 and buf.num_samples == 8  # window of 2 SDE steps stored
    assert buf.media is not None and torch.isfinite(buf.media).all()
    metrics = trainer.update(buf)
    assert len(metrics) == 4 and state.step == 4
    m = metrics[0].to_mapping()
    assert all(math.isfinite(v) for v in m.values())
    assert abs(m["grpo/ratio_mean"] - 1.0) < 1e-3  # first minibatch is on-policy
    assert any(not torch.equal(a, b.detach()) for a, b in zip(before, model.parameters()))


def test_generate_group_shares_seed_noise_per_prompt() -> None:
    def vel(x, s, *, prompt_index):  # noqa: ANN001, ANN202
        return -x

    buf = generate_group(vel, prompts=["p", "q"], group_size=3, sigmas=torch.linspace(1, 0, 4), latent_shape=(2, 3),
                         generator=torch.Generator().manual_seed(0), noise_level=0.5)
    first = buf.transitions("sample_before")[0]
    assert torch.equal(first[0], first[2]) and not torch.equal(first[0], first[3])


def test_dpo_loss_forms() -> None:
    e = torch.tensor([0.3, 0.4])
    loss, margin = dpo_loss(e, e, e, e, DPOConfig(beta=10.0))
    assert float(loss) == pytest.approx(0.0, abs=1e-7) and torch.all(margin == 0)
    loss, _ = dpo_loss(e - 0.1, e, e, e, DPOConfig(beta=10.0, center_loss=False))
    assert float(loss) == pytest.approx(-math.log(1 / (1 + math.exp(-1.0))), rel=1e-5)
    assert float(dpo_loss(e, e, e, e, DPOConfig(loss_type="hinge"))[0]) == 1.0
    assert float(dpo_loss(e, e, e, e, DPOConfig(loss_type="ipo"))[0]) == 0.25


def test_dpo_objective_policy_equals_reference() -> None:
    from avgen_b200.core import RNGStreams
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.rl import DPOObjective

    model = _tiny_model()
    obj = DPOObjective(DPOConfig(beta=100.0), GRPOTrainer.snapshot_reference(model))
    batch = random_batch(batch=2, channels=4, frames=2, height=8, width=8, text_tokens=3, text_width=8)
    out = obj(model, batch, RNGStreams.from_seed(0), patchifier=model.patchifier)
    assert float(out.loss.detach()) == pytest.approx(0.0, abs=1e-5)
    out.loss.backward()
    assert obj.last_margin is not None and obj.last_margin.shape == (1,)


def test_rewards_registry_and_normalisation() -> None:
    names = list_rewards()
    assert {"temporal_consistency", "motion_magnitude", "av_sync_proxy", "mlp_scorer", "hps_v2"} <= set(names)
    with pytest.raises(RuntimeError):
        build_reward("hps_v2")
    with pytest.raises(KeyError):
        build_reward("nope")
    video = torch.randn(4, 3, 5, 4, 4)
    prompts = ["x"] * 4
    tc = build_reward("temporal_consistency").score(video, prompts)
    assert tc.shape == (4,) and torch.all(tc.abs() <= 1)
    static = video[:, :, :1].expand(-1, -1, 5, -1, -1)
    torch.testing.assert_close(build_reward("temporal_consistency").score(static, prompts), torch.ones(4))
    s1 = MLPScorerReward(channels=3, seed=7).score(video, prompts)
    s2 = MLPScorerReward(channels=3, seed=7).score(video, prompts)
    assert torch.equal(s1, s2)
    n = RunningNormalizer()
    n.update(torch.tensor([1.0, 3.0]))
    n.update(torch.tensor([5.0]))
    assert n.state_dict()["mean"] == pytest.approx(3.0) and n.state_dict()["variance"] == pytest.approx(8 / 3)
    comp = CompositeReward(((build_reward("temporal_consistency"), 1.0), (build_reward("motion_magnitude"), 0.5)))
    assert comp.score(video, prompts).shape == (4,)
    assert set(comp.state_dict()) == {"component_0", "component_1"}


TINY = ["model.depth=1", "model.width=32", "model.num_heads=2", "model.in_channels=4", "data.latent_channels=4",
        "data.text_tokens=3", "data.text_width=8", "data.buckets=[{frames: 2, height: 8, width: 8}]",
        "train.warmup_steps=1", "telemetry.log_every=1", "telemetry.loggers=[jsonl]",
        "checkpoint.async_save=false"]


def test_cli_rl_grpo_and_dpo(tmp_path: Path) -> None:
    from avgen_b200.cli.main import main

    out = tmp_path / "grpo"
    assert main(["rl", *TINY, "train.steps=2", "train.global_batch_size=4", "rl.group_size=4",
                 "rl.sampler_steps=3", "rl.mixgrpo_window=2", "rl.kl_coefficient=0.04", "rl.guidance=2.0",
                 "rl.timestep_shift=true", "rl.rewards=[mlp_scorer, temporal_consistency]",
                 "rl.reward_weights=[1.0, 0.5]", f"output_dir={out}"]) == 0
    rows = [json.loads(x) for x in (out / "metrics.jsonl").read_text().splitlines()]
    assert rows and "grpo/loss" in rows[-1]
    assert (out / "checkpoints").is_dir()
    out = tmp_path / "dpo"
    assert main(["rl", *TINY, "train.steps=2", "train.global_batch_size=2", "data.buckets=[{frames: 2, height: 8, "
                 "width: 8, micro_batch_size: 2}]", "rl.algorithm=dpo", "rl.dpo_beta=10", f"output_dir={out}"]) == 0
