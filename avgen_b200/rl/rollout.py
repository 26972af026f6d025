"""Rollouts for diffusion RL: velocity functions, group generation, the rollout
buffer and group-relative advantages (avgen/rl/rollout.py:73-677 API).

Differences from the reference, on purpose:

* :func:`model_velocity_fn` applies classifier-free guidance when given a
  ``guidance`` scale above 1: the conditional and null-text branches run as one
  batched ``[2B]`` forward and are combined in fp32 (the reference's rollouts
  have no CFG, avgen/rl/rollout.py:631-658).
* ODE steps outside the gradient window run the fused guided-Euler kernel on
  CUDA; SDE steps run the fused SDE kernel (:mod:`avgen_b200.rl.sde`).
"""
from __future__ import annotations

from collections.abc import Iterator, Sequence
from dataclasses import dataclass, field
from typing import Any, Protocol

import torch

from avgen_b200.rl.sde import SDEStep, ode_step, to_sde

__all__ = ["RolloutBatch", "RolloutBuffer", "VelocityFn", "distribute_prompts", "gather_rewards", "generate_group",
           "group_advantages", "model_velocity_fn", "rollout_velocity_batch"]


class VelocityFn(Protocol):
    def __call__(self, sample: torch.Tensor, sigma: torch.Tensor, *, prompt_index: torch.Tensor) -> torch.Tensor: ...


def _rows(t: torch.Tensor, batch: int) -> torch.Tensor:
    if t.shape[0] == batch:
        return t
    row = t if t.dim() == 1 else t[0]
    return row.unsqueeze(0).expand(batch, *row.shape)


def model_velocity_fn(model: Any, *, patchifier: Any, positions: torch.Tensor, mask: torch.Tensor,
                      text_features: torch.Tensor, text_mask: torch.Tensor, guidance: float = 1.0,
                      null_features: torch.Tensor | None = None, null_mask: torch.Tensor | None = None,
                      cp_mesh: Any = None) -> VelocityFn:
    """Wrap a model as ``v(sample, sigma, prompt_index)`` in latent-grid space.

    ``text_features`` has one row per distinct prompt; ``prompt_index`` picks
    each sample's row. With ``guidance > 1`` the velocity is
    ``u + w (c - u)`` where ``u`` uses ``null_features`` (zeros with an
    all-false mask by default).
    """
    from avgen_b200.core.model_input import ModelInput
    from avgen_b200.core.patchify import unpatchify_grid
    from avgen_b200.core.tokens import TextContext, TokenStream

    def forward(inputs: ModelInput) -> torch.Tensor:
        if cp_mesh is None or cp_mesh.size() == 1:
            return model(inputs).video
        from avgen_b200.parallel.context import gather_tokens, shard_stream

        out = model(inputs.replace_streams(video=shard_stream(inputs.video, cp_mesh)))
        return gather_tokens(out.video, cp_mesh)

    def velocity(sample: torch.Tensor, sigma: torch.Tensor, *, prompt_index: torch.Tensor) -> torch.Tensor:
        b = sample.shape[0]
        index = prompt_index.to(text_features.device).long()
        if int(index.max()) >= text_features.shape[0]:
            raise ValueError(f"prompt_index reaches {int(index.max())} but text_features has "
                             f"{text_features.shape[0]} rows (one row per distinct prompt is expected)")
        feats = text_features.index_select(0, index)
        tmask = text_mask.index_select(0, index)
        stream = patchifier.to_tokens(sample, positions=_rows(positions, b), mask=_rows(mask, b),
                                      noise_level=sigma.to(torch.float32))
        guided = guidance > 1.0
        if guided:
            nf = torch.zeros_like(feats) if null_features is None else _rows(null_features, b).to(feats.dtype)
            nm = torch.zeros_like(tmask) if null_mask is None else _rows(null_mask, b)
            stream2 = patchifier.to_tokens(torch.cat((sample, sample)), positions=_rows(positions, 2 * b),
                                           mask=_rows(mask, 2 * b), noise_level=torch.cat((sigma, sigma)).float())
            inputs = ModelInput(video=stream2, audio=TokenStream.empty_like(2 * b, stream.width, device=sample.device),
                                text=TextContext(features=torch.cat((feats, nf)), mask=torch.cat((tmask, nm))))
            both = forward(inputs).float()
            cond, uncond = both[:b], both[b:]
            tokens = uncond + guidance * (cond - uncond)
        else:
            inputs = ModelInput(video=stream, audio=TokenStream.empty_like(b, stream.width, device=sample.device),
                                text=TextContext(features=feats, mask=tmask))
            tokens = forward(inputs)
        return unpatchify_grid(tokens, stream.layout)

    return velocity


@dataclass(frozen=True, slots=True)
class RolloutBatch:
    sample_before: torch.Tensor
    sample_after: torch.Tensor
    sigma: torch.Tensor
    sigma_next: torch.Tensor
    log_prob_old: torch.Tensor
    mean_old: torch.Tensor
    std_old: torch.Tensor
    advantage: torch.Tensor
    prompt_index: torch.Tensor
    step_index: torch.Tensor

    @property
    def size(self) -> int:
        return int(self.sample_before.shape[0])


def group_advantages(rewards: torch.Tensor, group_size: int, *, epsilon: float = 1e-4, normalize_by_std: bool = True,
                     clip: float | None = 5.0) -> torch.Tensor:
    """``(r - mean_group) / (std_group + eps)`` per trajectory (population std), optionally clipped."""
    if group_size < 2:
        raise ValueError(f"group_size must be at least 2; got {group_size} (a group of one has no baseline)")
    if rewards.numel() % group_size:
        raise ValueError(f"reward count {rewards.numel()} is not a multiple of group_size={group_size}")
    g = rewards.float().reshape(-1, group_size)
    adv = g - g.mean(1, keepdim=True)
    if normalize_by_std:
        adv = adv / (g.std(1, unbiased=False, keepdim=True) + epsilon)
    if clip is not None:
        adv = adv.clamp(-clip, clip)
    return adv.reshape(-1)


_STEP_KEYS = ("sample_before", "sample_after", "sigma", "sigma_next", "log_prob_old", "mean_old", "std_old",
              "step_index")


@dataclass(slots=True)
class RolloutBuffer:
    """Transitions of a group rollout (only steps inside the gradient window are stored)."""

    group_size: int
    prompts: tuple[str, ...] = ()
    rewards: torch.Tensor | None = None
    advantages: torch.Tensor | None = None
    media: torch.Tensor | None = None
    _steps: list[dict[str, torch.Tensor]] = field(default_factory=list, repr=False)

    def __post_init__(self) -> None:
        if self.group_size < 2:
            raise ValueError(f"group_size must be at least 2; got {self.group_size}")

    def __len__(self) -> int:
        return len(self._steps)

    @property
    def num_samples(self) -> int:
        return int(self._steps[0]["sample_before"].shape[0]) if self._steps else 0

    def add_step(self, *, step_index: int, sample_before: torch.Tensor, step: SDEStep, sigma: torch.Tensor,
                 sigma_next: torch.Tensor) -> None:
        n = sample_before.shape[0]
        self._steps.append({
            "sample_before": sample_before.detach(), "sample_after": step.sample.detach(), "sigma": sigma.detach(),
            "sigma_next": sigma_next.detach(), "log_prob_old": step.log_prob.detach(), "mean_old": step.mean.detach(),
            "std_old": step.std.detach(),
            "step_index": torch.full((n,), step_index, dtype=torch.int64, device=sample_before.device)})

    def set_rewards(self, rewards: torch.Tensor, *, media: torch.Tensor | None) -> None:
        if rewards.numel() != self.num_samples:
            raise ValueError(f"expected {self.num_samples} rewards to match the trajectories; got {rewards.numel()}")
        self.rewards = rewards.detach().float()
        self.media = media

    def compute_advantages(self, *, epsilon: float = 1e-4, normalize_by_std: bool = True,
                           clip: float | None = 5.0) -> torch.Tensor:
        if self.rewards is None:
            raise RuntimeError("call set_rewards() before compute_advantages()")
        self.advantages = group_advantages(self.rewards, self.group_size, epsilon=epsilon,
                                           normalize_by_std=normalize_by_std, clip=clip)
        return self.advantages

    def iter_minibatches(self, batch_size: int, *, generator: torch.Generator | None = None,
                         shuffle: bool = True) -> Iterator[RolloutBatch]:
        if self.advantages is None:
            raise RuntimeError("call compute_advantages() before iterating")
        if batch_size < 1:
            raise ValueError(f"batch_size must be positive; got {batch_size}")
        flat = self._flatten()
        total = int(flat["sample_before"].shape[0])
        order = torch.randperm(total, generator=generator) if shuffle else torch.arange(total)
        order = order.to(flat["sample_before"].device)
        for start in range(0, total, batch_size):
            idx = order[start:start + batch_size]
            yield RolloutBatch(**{k: v[idx] for k, v in flat.items()})

    def _flatten(self) -> dict[str, torch.Tensor]:
        assert self.advantages is not None
        dev = self._steps[0]["sample_before"].device
        flat = {k: torch.cat([s[k] for s in self._steps]) for k in _STEP_KEYS}
        reps = len(self._steps)
        flat["advantage"] = self.advantages.to(dev).repeat(reps)
        flat["prompt_index"] = (torch.arange(self.num_samples, device=dev) // self.group_size).repeat(reps)
        return flat


def distribute_prompts(prompts: Sequence[str], *, data_rank: int, data_world: int,
                       ) -> tuple[tuple[str, ...], tuple[int, ...]]:
    """Strided prompt shard of one data rank: ``range(data_rank, N, data_world)``."""
    if data_world < 1 or not 0 <= data_rank < data_world:
        raise ValueError(f"invalid data coordinates: data_rank={data_rank}, data_world={data_world}")
    idx = tuple(range(data_rank, len(prompts), data_world))
    return tuple(prompts[i] for i in idx), idx


def gather_rewards(rewards: torch.Tensor, mesh: Any | None = None) -> torch.Tensor:
    """All-gather per-rank rewards over ``mesh`` (identity without one)."""
    import torch.distributed as dist

    if mesh is None or not (dist.is_available() and dist.is_initialized()):
        return rewards
    group = mesh.get_group()
    world = dist.get_world_size(group)
    if world == 1:
        return rewards
    parts = [torch.empty_like(rewards) for _ in range(world)]
    dist.all_gather(parts, rewards.contiguous(), group=group)
    return torch.cat(parts)


def generate_group(velocity_fn: VelocityFn, *, prompts: Sequence[str], group_size: int, sigmas: torch.Tensor,
                   latent_shape: tuple[int, ...], device: torch.device | str = "cpu",
                   dtype: torch.dtype = torch.float32, noise_level: float = 0.7,
                   generator: torch.Generator | None = None, gradient_steps: Sequence[int] | None = None,
                   initial_latents: torch.Tensor | None = None, schedule: str = "flow_grpo") -> RolloutBuffer:
    """Sample ``group_size`` trajectories per prompt from shared seed noise.

    Steps in ``gradient_steps`` (all steps if ``None``) take the SDE and are
    stored; the others take a deterministic ODE step and are not.
    """
    if sigmas.ndim != 1 or sigmas.numel() < 2:
        raise ValueError(f"sigmas must be a 1-D schedule with at least two entries; got {tuple(sigmas.shape)}")
    if bool((sigmas[1:] > sigmas[:-1]).any()):
        raise ValueError("sigmas must be non-increasing (1 = noise down to 0 = clean)")
    n_prompts, n_steps = len(prompts), int(sigmas.numel()) - 1
    dev = torch.device(device)
    active = frozenset(range(n_steps)) if gradient_steps is None else frozenset(int(i) for i in gradient_steps)
    if initial_latents is None:
        gen_dev = generator.device if generator is not None else dev
        seed = torch.randn((n_prompts, *latent_shape), device=gen_dev, dtype=dtype, generator=generator).to(dev)
    else:
        if tuple(initial_latents.shape) != (n_prompts, *latent_shape):
            raise ValueError(f"initial_latents must be {(n_prompts, *latent_shape)}; got "
                             f"{tuple(initial_latents.shape)}")
        seed = initial_latents.to(device=dev, dtype=dtype)
    state = seed.repeat_interleave(group_size, 0)
    buffer = RolloutBuffer(group_size=group_size, prompts=tuple(prompts))
    prompt_index = torch.arange(n_prompts, device=dev).repeat_interleave(group_size)
    b = state.shape[0]
    with torch.no_grad():
        for i in range(n_steps):
            sigma = sigmas[i].to(dev, torch.float32).expand(b).contiguous()
            sigma_next = sigmas[i + 1].to(dev, torch.float32).expand(b).contiguous()
            v = velocity_fn(state, sigma, prompt_index=prompt_index)
            if i not in active:
                if state.is_cuda:
                    from avgen_b200.ops import kernels as K

                    state = K.guided_euler(v, None, state, sigma, sigma_next)
                else:
                    state = ode_step(v, state, sigma, sigma_next).to(dtype)
                continue
            step = to_sde(v, state, sigma, sigma_next, noise_level=noise_level, generator=generator,
                          schedule=schedule)
            buffer.add_step(step_index=i, sample_before=state, step=step, sigma=sigma, sigma_next=sigma_next)
            state = step.sample
    buffer.media = state
    return buffer


def rollout_velocity_batch(velocity_fn: VelocityFn, batch: RolloutBatch) -> torch.Tensor:
    return velocity_fn(batch.sample_before, batch.sigma, prompt_index=batch.prompt_index)
