"""Flow-GRPO policy optimisation for flow models (avgen/rl/grpo.py:89-714 API).

The objective per stored transition is PPO's clipped surrogate on the
importance ratio of the SDE transition (:mod:`avgen_b200.rl.sde`), optionally

* regulated (GRPO-Guard): the log-ratio is expressed through the difference of
  transition means scored against the stored noise, so it does not drift with
  the noise level;
* reweighted per timestep by ``1/|ds|`` (renormalised to mean one);
* penalised by the k3 KL estimator ``exp(d) - d - 1`` against a frozen
  reference policy;
* restricted to a MixGRPO sliding window of denoising steps.

Unlike the reference (avgen/rl/grpo.py:491-495 with avgen/rl/entry.py:232,
which raise when ``kl_coefficient > 0``), :meth:`GRPOTrainer.snapshot_reference`
freezes a copy of the current policy so the KL term always has a reference.
"""
from __future__ import annotations

import bisect
import copy
import functools
from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

import torch

from avgen_b200.core.limits import Limit, enforce
from avgen_b200.rl.rollout import RolloutBatch, RolloutBuffer, VelocityFn, generate_group
from avgen_b200.rl.sde import to_sde

__all__ = ["GRPOConfig", "GRPOMetrics", "GRPOTrainer", "WindowSchedule", "clipped_surrogate", "kl_penalty",
           "regulated_log_ratio"]


@functools.lru_cache(maxsize=64)
def _move_times(interval: int, stride: int, limit: int, exponential: bool, decay: float) -> tuple[float, ...]:
    """Optimizer steps at which the window moves, ascending: every ``interval`` steps,
    or (``exponential``) after intervals that shrink by ``decay`` down to one step.
    The window stops once it reaches ``limit``, after ceil(limit / stride) moves."""
    moves = -(-limit // stride) if limit > 0 else 0
    if not exponential:
        return tuple(float(interval * (k + 1)) for k in range(moves))
    times, at, span = [], 0.0, float(interval)
    for _ in range(moves):
        at += span
        times.append(at)
        span = max(span * decay, 1.0)
    return tuple(times)


@dataclass(frozen=True, slots=True)
class WindowSchedule:
    """MixGRPO window: ``window`` SDE steps starting at the high-noise end and
    moving ``stride`` steps every ``interval`` optimizer steps (geometrically
    shrinking intervals when ``exponential``)."""

    window: int = 4
    stride: int = 1
    interval: int = 25
    total_steps: int = 25
    exponential: bool = False
    decay: float = 0.8

    def __post_init__(self) -> None:
        enforce(self, _WINDOW_LIMITS)
        enforce(self, {"window": Limit(lo=1, hi=self.total_steps, integer=True)})  # fits in the trajectory

    def start_for(self, optimizer_step: int) -> int:
        """First SDE step of the window after ``optimizer_step`` optimizer steps."""
        if optimizer_step < 0:
            raise ValueError(f"optimizer_step must be non-negative; got {optimizer_step}")
        last = self.total_steps - self.window
        times = _move_times(self.interval, self.stride, last, self.exponential, self.decay)
        return min(self.stride * bisect.bisect_right(times, optimizer_step), last)

    def steps_for(self, optimizer_step: int) -> tuple[int, ...]:
        first = self.start_for(optimizer_step)
        return tuple(first + i for i in range(self.window))


_WINDOW_LIMITS = {name: Limit(lo=1, integer=True) for name in ("window", "stride", "interval", "total_steps")} | {
    "decay": Limit(lo=0.0, hi=1.0, lo_open=True)}


@dataclass(frozen=True, slots=True)
class GRPOConfig:
    group_size: int = 12
    clip_range: float = 2e-6
    clip_range_high: float | None = None
    regulated_clip: bool = True
    timestep_weighting: bool = True
    kl_coefficient: float = 0.0
    advantage_epsilon: float = 1e-4
    advantage_clip: float | None = 5.0
    normalize_advantage_by_std: bool = True
    noise_level: float = 0.7
    sde_schedule: str = "flow_grpo"
    inner_epochs: int = 1
    minibatch_size: int = 4
    max_grad_norm: float = 1.0
    window: WindowSchedule | None = None

    def __post_init__(self) -> None:
        # a group of one has no baseline; a deterministic policy (noise 0) has no policy gradient
        enforce(self, _GRPO_LIMITS)

    @property
    def high(self) -> float:
        return self.clip_range if self.clip_range_high is None else self.clip_range_high


_POSITIVE = Limit(lo=0.0, lo_open=True)
_GRPO_LIMITS = {"group_size": Limit(lo=2, integer=True), "clip_range": _POSITIVE,
                "clip_range_high": Limit(lo=0.0, lo_open=True, optional=True), "kl_coefficient": Limit(lo=0.0),
                "noise_level": _POSITIVE, "inner_epochs": Limit(lo=1, integer=True),
                "minibatch_size": Limit(lo=1, integer=True), "max_grad_norm": _POSITIVE}


@dataclass(frozen=True, slots=True)
class GRPOMetrics:
    loss: torch.Tensor
    policy_loss: torch.Tensor
    kl: torch.Tensor
    clip_fraction: torch.Tensor
    ratio_mean: torch.Tensor
    advantage_mean: torch.Tensor
    advantage_std: torch.Tensor

    def to_mapping(self) -> dict[str, float]:
        vals = torch.stack([t.detach().float().reshape(()) for t in (
            self.loss, self.policy_loss, self.kl, self.clip_fraction, self.ratio_mean, self.advantage_mean,
            self.advantage_std)]).cpu().tolist()  # one host sync
        keys = ("loss", "policy_loss", "kl", "clip_fraction", "ratio_mean", "advantage_mean", "advantage_std")
        return {f"grpo/{k}": float(v) for k, v in zip(keys, vals)}


def regulated_log_ratio(mean_new: torch.Tensor, mean_old: torch.Tensor, std_old: torch.Tensor, sample: torch.Tensor,
                        *, mask: torch.Tensor | None = None) -> torch.Tensor:
    """GRPO-Guard's normalised log-ratio: ``-sum((mean_old - mean_new) * z_old)``,
    ``z_old = (sample - mean_old) / std_old``."""
    sigma = std_old.reshape(-1, *((1,) * (sample.ndim - 1))).clamp_min(1e-12)
    prod = -((mean_old - mean_new) * ((sample - mean_old) / sigma))
    if mask is not None:
        prod = prod * mask.to(prod.dtype)
    return prod.flatten(1).sum(1)


def clipped_surrogate(log_ratio: torch.Tensor, advantage: torch.Tensor, *, clip_low: float, clip_high: float,
                      weights: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(-mean(min(r A, clip(r) A) * w), clipped fraction, r)``."""
    ratio = torch.exp(log_ratio)
    surrogate = torch.minimum(ratio * advantage, ratio.clamp(1.0 - clip_low, 1.0 + clip_high) * advantage)
    if weights is not None:
        surrogate = surrogate * weights
    clipped = (ratio < 1.0 - clip_low) | (ratio > 1.0 + clip_high)
    return -surrogate.mean(), clipped.float().mean(), ratio


def kl_penalty(log_prob_new: torch.Tensor, log_prob_reference: torch.Tensor) -> torch.Tensor:
    """k3 estimator of KL(pi || pi_ref): ``exp(d) - d - 1`` with ``d = log pi_ref - log pi``."""
    d = log_prob_reference - log_prob_new
    return torch.exp(d) - d - 1.0


class GRPOTrainer:
    """Rollout -> rewards -> group advantages -> clipped-surrogate updates."""

    def __init__(self, state: Any, velocity_fn: VelocityFn, config: GRPOConfig, *,
                 reference_velocity_fn: VelocityFn | None = None, cp_mesh: Any = None, pp_mesh: Any = None,
                 data_group: Any = None) -> None:
        if config.kl_coefficient > 0.0 and reference_velocity_fn is None:
            raise ValueError("kl_coefficient is non-zero but no reference policy was given; pass "
                             "reference_velocity_fn or build one with GRPOTrainer.snapshot_reference()")
        self.state = state
        self.velocity_fn = velocity_fn
        self.config = config
        self.reference_velocity_fn = reference_velocity_fn
        self.cp_mesh = cp_mesh
        self.pp_mesh = pp_mesh
        self.data_group = data_group

    @staticmethod
    def snapshot_reference(model: torch.nn.Module) -> torch.nn.Module:
        """A frozen deep copy of ``model`` (eval mode, no grads) to serve as the KL reference."""
        ref = copy.deepcopy(model)
        ref.eval()
        for p in ref.parameters():
            p.requires_grad_(False)
        return ref

    def gradient_steps(self) -> tuple[int, ...] | None:
        w = self.config.window
        return None if w is None else w.steps_for(int(self.state.step))

    def _step_weights(self, batch: RolloutBatch) -> torch.Tensor | None:
        if not self.config.timestep_weighting:
            return None
        w = 1.0 / (batch.sigma - batch.sigma_next).abs().clamp_min(1e-8)
        return w / w.mean().clamp_min(1e-12)

    def _transition(self, velocity_fn: VelocityFn, batch: RolloutBatch) -> Any:
        """The SDE transition ``velocity_fn`` assigns to each stored step (scored on the stored next state)."""
        c = self.config
        v = velocity_fn(batch.sample_before, batch.sigma, prompt_index=batch.prompt_index)
        return to_sde(v, batch.sample_before, batch.sigma, batch.sigma_next, noise_level=c.noise_level,
                      schedule=c.sde_schedule, prev_sample=batch.sample_after)

    def _log_ratio(self, step: Any, batch: RolloutBatch) -> torch.Tensor:
        if not self.config.regulated_clip:
            return step.log_prob - batch.log_prob_old
        return regulated_log_ratio(step.mean.float(), batch.mean_old.float(), batch.std_old.float(),
                                   batch.sample_after.float())

    def _kl(self, step: Any, batch: RolloutBatch, like: torch.Tensor) -> torch.Tensor:
        if self.config.kl_coefficient <= 0.0 or self.reference_velocity_fn is None:
            return torch.zeros((), device=like.device, dtype=like.dtype)
        with torch.no_grad():
            reference = self._transition(self.reference_velocity_fn, batch)
        return kl_penalty(step.log_prob, reference.log_prob).mean()

    def loss(self, batch: RolloutBatch) -> tuple[torch.Tensor, GRPOMetrics]:
        """Clipped surrogate of the policy's transitions plus the weighted KL term."""
        c = self.config
        step = self._transition(self.velocity_fn, batch)
        policy_loss, clip_fraction, ratio = clipped_surrogate(self._log_ratio(step, batch), batch.advantage,
                                                              clip_low=c.clip_range, clip_high=c.high,
                                                              weights=self._step_weights(batch))
        kl = self._kl(step, batch, policy_loss)
        total = policy_loss + c.kl_coefficient * kl
        adv = batch.advantage.detach()
        summary = {"loss": total, "policy_loss": policy_loss, "kl": kl, "clip_fraction": clip_fraction,
                   "ratio_mean": ratio.mean(), "advantage_mean": adv.mean(), "advantage_std": adv.std(unbiased=False)}
        return total, GRPOMetrics(**{k: v.detach() for k, v in summary.items()})

    def train_step(self, batch: RolloutBatch) -> GRPOMetrics:
        """Backward of one minibatch, then a clipped optimizer step (skipped on device if non-finite)."""
        from avgen_b200.train.optimizer import FusedAdamW
        from avgen_b200.train.trainer import optimizer_update

        opt = self.state.optimizer
        opt.zero_grad(set_to_none=not isinstance(opt, FusedAdamW))
        loss, metrics = self.loss(batch)
        loss.backward()
        optimizer_update(self.state, max_grad_norm=self.config.max_grad_norm, pp_mesh=self.pp_mesh,
                         data_group=self.data_group, finite=torch.isfinite(loss.detach()))
        return metrics

    def update(self, buffer: RolloutBuffer) -> list[GRPOMetrics]:
        if buffer.rewards is None:
            raise RuntimeError("attach rewards with set_rewards() before updating")
        c = self.config
        buffer.compute_advantages(epsilon=c.advantage_epsilon, normalize_by_std=c.normalize_advantage_by_std,
                                  clip=c.advantage_clip)
        out: list[GRPOMetrics] = []
        for _ in range(c.inner_epochs):
            for batch in buffer.iter_minibatches(c.minibatch_size, generator=self.state.rng.sampler):
                out.append(self.train_step(batch))
        return out

    def rollout(self, prompts: Sequence[str], *, sigmas: torch.Tensor, latent_shape: tuple[int, ...], reward: Any,
                device: torch.device | str = "cpu", dtype: torch.dtype = torch.float32,
                initial_latents: torch.Tensor | None = None) -> RolloutBuffer:
        c = self.config
        gen = self.state.rng.sampler
        buffer = generate_group(self.velocity_fn, prompts=prompts, group_size=c.group_size, sigmas=sigmas,
                                latent_shape=latent_shape, device=device, dtype=dtype, noise_level=c.noise_level,
                                generator=gen, gradient_steps=self.gradient_steps(),
                                initial_latents=initial_latents, schedule=c.sde_schedule)
        expanded = [p for p in prompts for _ in range(c.group_size)]
        assert buffer.media is not None
        buffer.set_rewards(reward.score(buffer.media, expanded), media=buffer.media)
        return buffer
