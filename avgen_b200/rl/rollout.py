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


def _need_group(group_size: int) -> None:
    if group_size < 2:
        raise ValueError(f"a GRPO group needs two or more samples to form a baseline (group_size={group_size})")


def group_advantages(rewards: torch.Tensor, group_size: int, *, epsilon: float = 1e-4, normalize_by_std: bool = True,
                     clip: float | None = 5.0) -> torch.Tensor:
    """``(r - mean_group) / (std_group + eps)`` per trajectory (population std), optionally clipped.

    ``rewards`` lists the groups one after another (``group_size`` consecutive
    entries share a prompt)."""
    _need_group(group_size)
    groups, rest = divmod(rewards.numel(), group_size)
    if rest:
        raise ValueError(f"{rewards.numel()} rewards do not split into groups of {group_size}")
    g = rewards.float().reshape(groups, group_size)
    centred = g - g.mean(1, keepdim=True)
    if normalize_by_std:
        centred = centred / (g.std(1, unbiased=False, keepdim=True) + epsilon)
    return (centred if clip is None else centred.clamp(-clip, clip)).reshape(-1)


# per-sample fields of one stored transition, in RolloutBatch order
_FIELDS = ("sample_before", "sample_after", "sigma", "sigma_next", "log_prob_old", "mean_old", "std_old")


@dataclass(slots=True)
class RolloutBuffer:
    """Window transitions of one group rollout, kept in step-major arenas on the rollout's device.

    Every per-sample field is one tensor of shape ``[capacity, N, ...]``,
    allocated when the first step is stored (``capacity`` is the number of
    window steps when the caller knows it, as :func:`generate_group` does;
    otherwise the arenas double when full). Storing a step is an in-place copy
    into row ``len(self)``; a minibatch is one ``index_select`` per field from
    the ``[steps * N]`` flat view. Flat row ``r`` is sample ``r % N`` at stored
    step ``r // N``, so its advantage, prompt and step index come from ``r`` by
    arithmetic: nothing is concatenated or repeated at update time, which would
    otherwise hold a second copy of every latent the rollout kept.
    """

    group_size: int
    prompts: tuple[str, ...] = ()
    rewards: torch.Tensor | None = None
    advantages: torch.Tensor | None = None
    media: torch.Tensor | None = None
    capacity: int = 0
    _arena: dict[str, torch.Tensor] = field(default_factory=dict, repr=False)
    _step_ids: torch.Tensor | None = field(default=None, repr=False)
    _count: int = field(default=0, repr=False)

    def __post_init__(self) -> None:
        _need_group(self.group_size)

    def __len__(self) -> int:
        return self._count

    @property
    def num_samples(self) -> int:
        return int(self._arena["sample_before"].shape[1]) if self._count else 0

    def transitions(self, name: str) -> torch.Tensor:
        """The stored ``[steps, N, ...]`` view of one field (``sample_before``, ``log_prob_old``, ...)."""
        if name not in _FIELDS:
            raise KeyError(f"unknown transition field {name!r}; fields are {', '.join(_FIELDS)}")
        if not self._count:
            raise RuntimeError("the buffer holds no transitions yet")
        return self._arena[name][:self._count]

    def _grow(self, values: dict[str, torch.Tensor]) -> None:
        size = max(self.capacity, 2 * self._count, 1)
        arena = {k: v.new_empty((size, *v.shape)) for k, v in values.items()}
        ids = torch.empty(size, dtype=torch.int64, device=values["sample_before"].device)
        if self._count:
            for k, old in self._arena.items():
                arena[k][:self._count].copy_(old[:self._count])
            ids[:self._count].copy_(self._step_ids[:self._count])
        self._arena, self._step_ids = arena, ids

    def add_step(self, *, step_index: int, sample_before: torch.Tensor, step: SDEStep, sigma: torch.Tensor,
                 sigma_next: torch.Tensor) -> None:
        values = dict(zip(_FIELDS, (sample_before, step.sample, sigma, sigma_next, step.log_prob, step.mean,
                                    step.std)))
        if self._count and values["sample_before"].shape[0] != self.num_samples:
            raise ValueError(f"every stored step must cover the same {self.num_samples} samples; this one has "
                             f"{values['sample_before'].shape[0]}")
        if not self._arena or self._count == self._arena["sample_before"].shape[0]:
            self._grow(values)
        row = self._count
        with torch.no_grad():
            for k, v in values.items():
                self._arena[k][row].copy_(v)
        self._step_ids[row] = int(step_index)
        self._count = row + 1

    def set_rewards(self, rewards: torch.Tensor, *, media: torch.Tensor | None) -> None:
        if rewards.numel() != self.num_samples:
            raise ValueError(f"one reward per trajectory: the buffer holds {self.num_samples} trajectories, "
                             f"{rewards.numel()} rewards were given")
        self.rewards, self.media = rewards.detach().float().reshape(-1), media

    def compute_advantages(self, *, epsilon: float = 1e-4, normalize_by_std: bool = True,
                           clip: float | None = 5.0) -> torch.Tensor:
        if self.rewards is None:
            raise RuntimeError("advantages need rewards: call set_rewards first")
        self.advantages = group_advantages(self.rewards, self.group_size, epsilon=epsilon,
                                           normalize_by_std=normalize_by_std, clip=clip)
        return self.advantages

    def iter_minibatches(self, batch_size: int, *, generator: torch.Generator | None = None,
                         shuffle: bool = True) -> Iterator[RolloutBatch]:
        """Minibatches over every stored (step, sample) transition, shuffled by ``generator``'s draw."""
        if self.advantages is None:
            raise RuntimeError("minibatches need advantages: call compute_advantages first")
        if batch_size < 1:
            raise ValueError(f"batch_size must be at least 1 (got {batch_size})")
        n, steps = self.num_samples, self._count
        dev = self._arena["sample_before"].device
        flat = {k: v[:steps].flatten(0, 1) for k, v in self._arena.items()}
        advantages = self.advantages.to(dev)
        order = torch.randperm(n * steps, generator=generator) if shuffle else torch.arange(n * steps)
        for rows in order.to(dev).split(batch_size):
            sample = rows % n
            yield RolloutBatch(**{k: flat[k].index_select(0, rows) for k in _FIELDS},
                               advantage=advantages.index_select(0, sample),
                               prompt_index=sample // self.group_size,
                               step_index=self._step_ids.index_select(0, rows // n))


def _check_data_coordinates(data_rank: int, data_world: int) -> None:
    if data_world < 1:
        raise ValueError(f"data_world counts ranks and must be at least 1 (got {data_world})")
    if not 0 <= data_rank < data_world:
        raise ValueError(f"data_rank {data_rank} lies outside the {data_world} data ranks")


def distribute_prompts(prompts: Sequence[str], *, data_rank: int, data_world: int,
                       ) -> tuple[tuple[str, ...], tuple[int, ...]]:
    """Strided prompt shard of one data rank: ``range(data_rank, N, data_world)``."""
    _check_data_coordinates(data_rank, data_world)
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
    if sigmas.ndim != 1 or sigmas.numel() < 2 or bool((sigmas[1:] > sigmas[:-1]).any()):
        raise ValueError(f"sigmas must be one non-increasing run of two or more levels from noise (1) towards clean "
                         f"(0); got shape {tuple(sigmas.shape)}")
    n_prompts, n_steps = len(prompts), int(sigmas.numel()) - 1
    dev = torch.device(device)
    active = frozenset(range(n_steps)) if gradient_steps is None else frozenset(int(i) for i in gradient_steps)
    window = sum(1 for i in active if 0 <= i < n_steps)
    if initial_latents is None:
        gen_dev = generator.device if generator is not None else dev
        seed = torch.randn((n_prompts, *latent_shape), device=gen_dev, dtype=dtype, generator=generator).to(dev)
    else:
        if tuple(initial_latents.shape) != (n_prompts, *latent_shape):
            raise ValueError(f"initial_latents must be {(n_prompts, *latent_shape)}; got "
                             f"{tuple(initial_latents.shape)}")
        seed = initial_latents.to(device=dev, dtype=dtype)
    state = seed.repeat_interleave(group_size, 0)
    buffer = RolloutBuffer(group_size=group_size, prompts=tuple(prompts), capacity=window)
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
