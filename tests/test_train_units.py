"""Training units on CPU against closed forms: learning-rate schedules at their
landmark steps, timestep samplers' distributions and shifts, parameter groups,
the flat-buffer AdamW against torch's AdamW (with clipping and the non-finite
skip), and the EMA's decay arithmetic and restore paths (reference test
strategy: tests/test_train*.py -- schedule tables, sampler statistics,
optimizer equivalence)."""
from __future__ import annotations

import math

import pytest
import torch
from torch import nn

from avgen_b200.train.ema import ShardedEMA
from avgen_b200.train.optimizer import FusedAdamW, build_optimizer, build_param_groups
from avgen_b200.train.schedule import build_schedule, list_schedules, register_schedule
from avgen_b200.train.timestep import (ModeSampler, ShiftedLogitNormalSampler, UniformSampler, build_timestep_sampler,
                                       list_timestep_samplers, register_timestep_sampler, resolution_shift,
                                       shift_timesteps)


def _opt(lr: float = 1.0) -> torch.optim.Optimizer:
    return torch.optim.SGD([nn.Parameter(torch.zeros(1))], lr=lr)


def _lrs(name: str, total: int, warmup: int, **kw) -> list[float]:  # noqa: ANN003
    opt = _opt()
    sched = build_schedule(name, opt, total_steps=total, warmup_steps=warmup, **kw)
    out = []
    for _ in range(total):
        out.append(opt.param_groups[0]["lr"])
        opt.step()
        sched.step()
    return out


# ----------------------------------------------------------------------------- schedules


@pytest.mark.parametrize("name", ["constant", "linear", "cosine", "wsd"])
def test_warmup_is_linear(name: str) -> None:
    lrs = _lrs(name, 100, 10)
    assert lrs[:10] == pytest.approx([(i + 1) / 10 for i in range(10)])
    assert lrs[10] == pytest.approx(1.0)


def test_constant_linear_cosine_landmarks() -> None:
    assert _lrs("constant", 20, 0) == pytest.approx([1.0] * 20)
    lin = _lrs("linear", 101, 1, min_lr_ratio=0.1)
    assert lin[1] == pytest.approx(1.0) and lin[51] == pytest.approx(0.1 + 0.9 * 0.5) and lin[-1] > 0.1
    cos = _lrs("cosine", 101, 1)
    assert cos[1] == pytest.approx(1.0) and cos[51] == pytest.approx(0.5) and cos[-1] < 0.01
    floored = _lrs("cosine", 101, 1, min_lr_ratio=0.2)
    assert min(floored) >= 0.2 - 1e-9 and floored[51] == pytest.approx(0.6)


@pytest.mark.parametrize("shape", ["1-sqrt", "linear", "cosine"])
def test_wsd_stable_then_decay(shape: str) -> None:
    lrs = _lrs("wsd", 100, 5, decay_fraction=0.2, decay_shape=shape)
    assert lrs[5:80] == pytest.approx([1.0] * 75)  # stable phase
    tail = lrs[80:]
    assert all(a >= b for a, b in zip(tail, tail[1:])) and tail[-1] < 0.3
    mid = lrs[90]
    expect = {"1-sqrt": 1 - math.sqrt(0.5), "linear": 0.5, "cosine": 0.5}[shape]
    assert mid == pytest.approx(expect, abs=1e-6)


@pytest.mark.parametrize("kw", [{"total_steps": 0}, {"total_steps": 10, "warmup_steps": 10},
                                {"total_steps": 10, "warmup_steps": -1}])
def test_schedule_argument_errors(kw: dict) -> None:
    with pytest.raises(ValueError):
        build_schedule("cosine", _opt(), **kw)


def test_schedule_option_errors_and_registry() -> None:
    with pytest.raises(ValueError):
        build_schedule("cosine", _opt(), total_steps=10, min_lr_ratio=1.5)
    with pytest.raises(ValueError):
        build_schedule("wsd", _opt(), total_steps=10, decay_fraction=0.0)
    with pytest.raises(ValueError):
        build_schedule("wsd", _opt(), total_steps=10, decay_shape="exp")
    with pytest.raises(KeyError):
        build_schedule("step", _opt(), total_steps=10)
    assert set(list_schedules()) >= {"constant", "linear", "cosine", "wsd"}
    with pytest.raises(ValueError):
        register_schedule("cosine")(lambda *a: (lambda s: 1.0))


# ----------------------------------------------------------------------------- timestep samplers


def _draw(sampler, n: int = 200_000, length: int | None = None) -> torch.Tensor:  # noqa: ANN001
    return sampler.sample(n, device="cpu", generator=torch.Generator().manual_seed(0), sequence_length=length)


@pytest.mark.parametrize("low,high", [(0.0, 1.0), (0.2, 0.8), (0.5, 0.6)])
def test_uniform_sampler_moments(low: float, high: float) -> None:
    t = _draw(UniformSampler(low, high))
    assert float(t.min()) >= low and float(t.max()) <= high
    assert float(t.mean()) == pytest.approx((low + high) / 2, abs=3e-3)
    assert float(t.var()) == pytest.approx((high - low) ** 2 / 12, rel=0.02)


@pytest.mark.parametrize("mean,std", [(0.0, 1.0), (0.5, 1.0), (-0.5, 0.5)])
def test_logit_normal_median_and_logit_moments(mean: float, std: float) -> None:
    t = _draw(build_timestep_sampler("logit_normal", {"mean": mean, "std": std}))
    logit = torch.log(t / (1 - t))
    assert float(logit.mean()) == pytest.approx(mean, abs=0.01)
    assert float(logit.std()) == pytest.approx(std, rel=0.01)
    assert float(t.median()) == pytest.approx(1 / (1 + math.exp(-mean)), abs=0.005)


@pytest.mark.parametrize("length,expect", [(None, 0.95), (1024, 0.95), (32768, 2.05), (16896, 1.5),
                                           (10, 0.95), (10**6, 2.05)])
def test_resolution_shift_interpolates_and_clamps(length: int | None, expect: float) -> None:
    s = resolution_shift(length, base_seq_len=1024, base_shift=0.95, max_seq_len=32768, max_shift=2.05)
    assert s == pytest.approx(expect, rel=1e-6)


def test_shifted_sampler_moves_mass_to_high_noise_with_length() -> None:
    s = ShiftedLogitNormalSampler()
    short, long = _draw(s, length=1024), _draw(s, length=65536)
    assert float(long.mean()) > float(short.mean())
    # the shift is an increasing bijection of (0, 1): same draws, shifted
    raw = _draw(build_timestep_sampler("logit_normal"))
    torch.testing.assert_close(long, shift_timesteps(raw, s.shift_for(65536)))


@pytest.mark.parametrize("shift", [0.5, 1.0, 3.0])
def test_shift_timesteps_properties(shift: float) -> None:
    t = torch.linspace(0, 1, 11, dtype=torch.float64)
    out = shift_timesteps(t, shift)
    assert float(out[0]) == 0.0 and float(out[-1]) == pytest.approx(1.0)
    assert bool((out[1:] > out[:-1]).all())
    with pytest.raises(ValueError):
        shift_timesteps(t, 0.0)


@pytest.mark.parametrize("scale", [-1.0, 0.0, 1.29, 3.0])
def test_mode_sampler_range_and_zero_scale_is_uniform(scale: float) -> None:
    t = _draw(ModeSampler(scale))
    assert float(t.min()) >= 0.0 and float(t.max()) <= 1.0
    if scale == 0.0:  # t = 1 - u
        assert float(t.mean()) == pytest.approx(0.5, abs=3e-3)


@pytest.mark.parametrize("factory,kw", [(UniformSampler, {"low": 0.6, "high": 0.5}), (UniformSampler, {"low": -0.1}),
                                        (ShiftedLogitNormalSampler, {"std": 0.0}),
                                        (ShiftedLogitNormalSampler, {"base_seq_len": 10, "max_seq_len": 5}),
                                        (ShiftedLogitNormalSampler, {"max_shift": 0.0}), (ModeSampler, {"scale": 9.0})])
def test_sampler_validation(factory, kw: dict) -> None:  # noqa: ANN001
    with pytest.raises(ValueError):
        factory(**kw)


def test_sampler_registry() -> None:
    assert set(list_timestep_samplers()) >= {"uniform", "logit_normal", "shifted_logit_normal", "mode"}
    with pytest.raises(KeyError):
        build_timestep_sampler("beta")
    with pytest.raises(ValueError):
        register_timestep_sampler("uniform")(UniformSampler)
    a = _draw(build_timestep_sampler("uniform"), n=16)
    b = _draw(build_timestep_sampler("uniform"), n=16)
    torch.testing.assert_close(a, b)  # same generator seed, same draws


# ----------------------------------------------------------------------------- optimizer


class _Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.proj = nn.Linear(6, 5)
        self.norm = nn.LayerNorm(5)
        self.scale_shift_table = nn.Parameter(torch.randn(2, 5))
        self.frozen = nn.Linear(5, 5)
        self.frozen.requires_grad_(False)


def test_param_groups_split_decay() -> None:
    net = _Net()
    groups = build_param_groups(net, weight_decay=0.1)
    decayed = {id(p) for p in groups[0]["params"]}
    assert groups[0]["weight_decay"] == 0.1 and groups[1]["weight_decay"] == 0.0
    assert id(net.proj.weight) in decayed
    assert id(net.proj.bias) not in decayed and id(net.norm.weight) not in decayed
    assert id(net.frozen.weight) not in decayed
    with pytest.raises(ValueError):
        build_param_groups(nn.Linear(2, 2).requires_grad_(False), weight_decay=0.1)


@pytest.mark.parametrize("kw", [{"lr": 0.0}, {"lr": 1e-3, "weight_decay": -1.0}, {"lr": 1e-3, "betas": (1.0, 0.9)},
                                {"lr": 1e-3, "eps": 0.0}, {"lr": 1e-3, "name": "lamb"}])
def test_build_optimizer_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        build_optimizer(_Net(), **kw)


def _pair(seed: int = 0) -> tuple[nn.Module, nn.Module]:
    torch.manual_seed(seed)
    a = _Net()
    b = _Net()
    b.load_state_dict(a.state_dict())
    return a, b


def _grads(model: nn.Module, seed: int, scale: float = 1.0) -> None:
    g = torch.Generator().manual_seed(seed)
    for p in model.parameters():
        if p.requires_grad:
            value = torch.randn(p.shape, generator=g) * scale
            if p.grad is None:
                p.grad = value
            else:  # the flat-buffer optimizer's gradients are views into its flat buffer: write in place
                p.grad.copy_(value)


@pytest.mark.parametrize("clip", [None, 0.5])
def test_fused_adamw_matches_torch_adamw(clip: float | None) -> None:
    ours_model, ref_model = _pair()
    ours = build_optimizer(ours_model, lr=1e-2, weight_decay=0.1, fused=True)
    assert isinstance(ours, FusedAdamW)
    ref = torch.optim.AdamW(build_param_groups(ref_model, weight_decay=0.1), lr=1e-2, betas=(0.9, 0.95), eps=1e-8)
    for step in range(4):
        ours.zero_grad()
        _grads(ours_model, step)
        _grads(ref_model, step)
        if clip is not None:
            torch.nn.utils.clip_grad_norm_([p for p in ref_model.parameters() if p.requires_grad], clip)
        ours.step(max_grad_norm=clip)
        ref.step()
    for (n, p), (_, q) in zip(ours_model.named_parameters(), ref_model.named_parameters()):
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6, msg=n)


def test_fused_adamw_skips_non_finite_steps() -> None:
    model, _ = _pair()
    opt = build_optimizer(model, lr=1e-2, fused=True)
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    opt.zero_grad()
    _grads(model, 0)
    next(model.parameters()).grad[0, 0] = float("nan")
    opt.step(max_grad_norm=1.0)
    assert bool(opt.last_nonfinite)
    for n, p in model.named_parameters():
        torch.testing.assert_close(p, before[n], msg=n)
    opt.zero_grad()
    _grads(model, 1)
    opt.step()
    assert not bool(opt.last_nonfinite)
    assert any(not torch.equal(p, before[n]) for n, p in model.named_parameters())


def test_fused_adamw_grad_norm_and_state_round_trip() -> None:
    model, _ = _pair()
    opt = build_optimizer(model, lr=1e-2, fused=True)
    opt.zero_grad()
    _grads(model, 3)
    want = torch.sqrt(sum((p.grad.double() ** 2).sum() for p in model.parameters() if p.requires_grad))
    assert float(opt.grad_norm()) == pytest.approx(float(want), rel=1e-5)
    opt.step()
    sd = opt.state_dict()
    group = sd["param_groups"][0]
    for key in ("lr", "betas", "eps", "weight_decay", "amsgrad", "maximize", "foreach", "capturable"):
        assert key in group
    torch_opt = torch.optim.AdamW(build_param_groups(model, weight_decay=0.0), lr=1e-2)
    torch_opt.load_state_dict(sd)  # the state dict is torch AdamW's format
    fresh = build_optimizer(model, lr=1e-2, fused=True)
    fresh.load_state_dict(sd)
    s0 = next(iter(fresh.state.values()))
    assert set(s0) >= {"exp_avg", "exp_avg_sq", "step"}


# ----------------------------------------------------------------------------- EMA


@pytest.mark.parametrize("step,warmup,expect", [(0, 0, 1 / 10), (80, 0, 0.9), (10**6, 0, 0.99), (3, 5, 0.0)])
def test_ema_effective_decay(step: int, warmup: int, expect: float) -> None:
    ema = ShardedEMA(nn.Linear(2, 2), decay=0.99, warmup_steps=warmup)
    assert ema.effective_decay(step) == pytest.approx(expect, rel=1e-3)


def test_ema_tracks_lerp_and_restores() -> None:
    torch.manual_seed(0)
    model = nn.Linear(3, 3)
    ema = ShardedEMA(model, decay=0.5, storage_dtype=torch.float32)
    start = {n: p.detach().clone() for n, p in model.named_parameters()}
    with torch.no_grad():
        for p in model.parameters():
            p.add_(1.0)
    for _ in range(30):
        ema.update(model)  # decay warms up toward 0.5: the shadow converges to the new weights
    assert ema.num_updates == 30 and ema.decay == 0.5
    live = {n: p.detach().clone() for n, p in model.named_parameters()}
    with ema.apply_to(model):
        for n, p in model.named_parameters():
            torch.testing.assert_close(p, live[n], rtol=0, atol=1e-6)
    for n, p in model.named_parameters():
        torch.testing.assert_close(p, live[n])  # restored after the context
        assert not torch.allclose(p, start[n])
    state = ema.state_dict()
    other = ShardedEMA(nn.Linear(3, 3), decay=0.5, storage_dtype=torch.float32)
    other.load_state_dict(state)
    assert other.num_updates == 30
    with pytest.raises(KeyError):
        other.load_state_dict({"num_updates": 1})


@pytest.mark.parametrize("kw", [{"decay": 0.0}, {"decay": 1.0}, {"warmup_steps": -1}, {"update_every": 0}])
def test_ema_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        ShardedEMA(nn.Linear(2, 2), **kw)


def test_ema_update_every_skips_steps() -> None:
    model = nn.Linear(2, 2)
    ema = ShardedEMA(model, decay=0.9, update_every=3, storage_dtype=torch.float32)
    snap = {k: v.clone() for k, v in ema.state_dict().items() if isinstance(v, torch.Tensor)}
    with torch.no_grad():
        for p in model.parameters():
            p.add_(1.0)
    ema.update(model)  # step 0 updates
    after0 = {k: v.clone() for k, v in ema.state_dict().items() if isinstance(v, torch.Tensor)}
    ema.update(model)  # step 1 is skipped
    after1 = {k: v for k, v in ema.state_dict().items() if isinstance(v, torch.Tensor)}
    assert any(not torch.equal(snap[k], after0[k]) for k in snap)
    assert all(torch.equal(after0[k], after1[k]) for k in after0)
