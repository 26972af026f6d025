"""``avgen-b200 rl``: GRPO or Diffusion-DPO from a :class:`~avgen_b200.config.RunConfig`
(avgen/rl/entry.py:39-283 API).

GRPO differs from the reference on purpose (its shipped config cannot run,
avgen/rl/entry.py:232 with avgen/rl/grpo.py:491-495):

* ``rl.kl_coefficient > 0`` with no ``rl.reference_checkpoint`` snapshots the
  starting weights as the frozen reference policy;
* rollouts apply classifier-free guidance (``rl.guidance``) as one batched
  cond + null-text forward;
* ``rl.timestep_shift`` applies the sequence-length-dependent shift to the
  rollout sigma schedule;
* with no ``rl.prompts_file`` the synthetic data source's text embeddings
  stand in for encoded prompts (one row per prompt).
"""
from __future__ import annotations

import logging
from pathlib import Path
from typing import Any

import torch

__all__ = ["build_rewards", "rl_from_config", "run_rl"]

_LOG = logging.getLogger("avgen_b200.rl")


def build_rewards(config: Any) -> Any:
    from avgen_b200.rl.rewards import CompositeReward, build_reward

    names = tuple(config.rl.rewards)
    if not names:
        raise ValueError("rl.rewards is empty: with no reward every sample of a group scores the same, every "
                         "group-relative advantage is zero and the run learns nothing")
    weights = tuple(config.rl.reward_weights) or (1.0,) * len(names)
    if len(weights) != len(names):
        raise ValueError(f"rl.reward_weights has {len(weights)} entries for {len(names)} rewards")
    options = {"mlp_scorer": {"channels": config.data.latent_channels}}
    rewards = [build_reward(n, **options.get(n, {})) for n in names]
    return rewards[0] if len(rewards) == 1 else CompositeReward(tuple(zip(rewards, weights, strict=True)))


def _load_prompts(path: str) -> list[str]:
    lines = [ln.strip() for ln in Path(path).read_text(encoding="utf-8").splitlines() if ln.strip()]
    if not lines:
        raise ValueError(f"rl.prompts_file {path!r} contains no prompts")
    return lines


def _reference_model(config: Any, policy: torch.nn.Module) -> torch.nn.Module:
    from avgen_b200.rl.grpo import GRPOTrainer

    ref = GRPOTrainer.snapshot_reference(policy)
    if config.rl.reference_checkpoint:
        from avgen_b200.infer.pipeline import _load_weights

        _load_weights(Path(config.rl.reference_checkpoint), ref)
    return ref


def _context_parallel_reference(reference: torch.nn.Module, stack: Any) -> None:
    """Give the frozen reference the same global attention over the CP group as the policy."""
    cp_mesh = getattr(stack.parallel, "cp_mesh", None)
    if cp_mesh is not None and cp_mesh.size() > 1:
        from avgen_b200.parallel.context import apply_context_parallel

        apply_context_parallel(reference, cp_mesh)


def _close(stack: Any) -> None:
    stack.manager.close()
    close = getattr(stack.logger, "close", None)
    if callable(close):
        close()


def _run_dpo(config: Any) -> Any:
    from avgen_b200.cli._wiring import build_run, run_training
    from avgen_b200.rl.dpo import DPOConfig, DPOObjective

    objective = DPOObjective(DPOConfig(beta=config.rl.dpo_beta), reference_model=None)

    def snapshot(model: torch.nn.Module) -> torch.nn.Module:
        # the reference is frozen from the starting weights (or rl.reference_checkpoint)
        objective.reference_model = _reference_model(config, model)
        return model

    stack = build_run(config, model_hook=snapshot, objective=objective)
    _context_parallel_reference(objective.reference_model, stack)
    run_training(stack)
    return stack


def _run_grpo(config: Any) -> Any:
    from avgen_b200.cli._wiring import build_run
    from avgen_b200.infer.schedule import ScheduleConfig, build_sigma_schedule
    from avgen_b200.rl.grpo import GRPOConfig, GRPOTrainer, WindowSchedule
    from avgen_b200.rl.rollout import model_velocity_fn

    s = config.rl
    reward = build_rewards(config)
    holder: dict[str, Any] = {}

    def snapshot(model: torch.nn.Module) -> torch.nn.Module:
        if s.kl_coefficient > 0.0:
            holder["reference"] = _reference_model(config, model)
        return model

    stack = build_run(config, model_hook=snapshot)
    if "reference" in holder:
        _context_parallel_reference(holder["reference"], stack)
    device = stack.env.device
    batch = next(iter(stack.loader)).to(device)
    prompts = _load_prompts(s.prompts_file) if s.prompts_file else \
        [f"synthetic prompt {i}" for i in range(batch.text.shape[0])]
    n_text = batch.text.shape[0]
    feats = batch.text[torch.arange(len(prompts), device=device) % n_text]
    tmask = batch.text_mask[torch.arange(len(prompts), device=device) % n_text]
    patchifier = stack.trainer.patchifier
    cp_mesh = getattr(stack.parallel, "cp_mesh", None)
    common = dict(patchifier=patchifier, positions=batch.video_positions[:1], mask=batch.video_mask[:1],
                  text_features=feats, text_mask=tmask, guidance=s.guidance, cp_mesh=cp_mesh)
    velocity = model_velocity_fn(stack.parallel.model, **common)
    ref_velocity = model_velocity_fn(holder["reference"], **common) if "reference" in holder else None
    bucket = config.data.buckets[0]
    latent_shape = (config.data.latent_channels, bucket.frames, bucket.height, bucket.width)
    tokens = patchifier.layout_for((1, *latent_shape)).num_tokens
    sched = ScheduleConfig(name="linear", steps=s.sampler_steps, dynamic_shift=bool(s.timestep_shift))
    sigmas = build_sigma_schedule(sched, sequence_length=tokens, device=device).sigmas
    grpo = GRPOConfig(group_size=s.group_size, clip_range=s.clip_range, kl_coefficient=s.kl_coefficient,
                      normalize_advantage_by_std=s.advantage_normalize, noise_level=s.sde_noise_scale,
                      max_grad_norm=config.train.max_grad_norm,
                      window=WindowSchedule(window=s.mixgrpo_window, total_steps=s.sampler_steps)
                      if s.mixgrpo_window else None)
    trainer = GRPOTrainer(stack.state, velocity, grpo, reference_velocity_fn=ref_velocity, cp_mesh=cp_mesh,
                          pp_mesh=getattr(stack.parallel, "pp_mesh", None),
                          data_group=getattr(stack.parallel, "data_group", None))
    per_step = max(1, config.train.global_batch_size // s.group_size)
    _LOG.info("grpo prompts=%d group_size=%d steps=%d kl=%g guidance=%g rewards=%s", len(prompts), s.group_size,
              s.sampler_steps, s.kl_coefficient, s.guidance, ", ".join(s.rewards))
    try:
        for step in range(config.train.steps):
            off = (step * per_step) % len(prompts)
            chosen = [prompts[(off + i) % len(prompts)] for i in range(per_step)]
            buffer = trainer.rollout(chosen, sigmas=sigmas, latent_shape=latent_shape, reward=reward, device=device)
            metrics = trainer.update(buffer)
            if metrics and step % config.telemetry.log_every == 0:
                record = metrics[-1].to_mapping()
                if buffer.rewards is not None:
                    record["grpo/reward_mean"] = float(buffer.rewards.mean())
                stack.logger.log_metrics(record, stack.state.step)
            if config.checkpoint.save_every and stack.state.step % config.checkpoint.save_every == 0:
                stack.manager.save(stack.state.step, stack.state, parallel=stack.parallel, async_save=False)
        stack.manager.save(stack.state.step, stack.state, parallel=stack.parallel, async_save=False)
    finally:
        _close(stack)
    return stack


def rl_from_config(config: Any) -> Any:
    algorithm = config.rl.algorithm
    if algorithm == "dpo":
        return _run_dpo(config)
    if algorithm == "grpo":
        return _run_grpo(config)
    raise ValueError(f"unknown rl.algorithm {algorithm!r}; expected one of: grpo, dpo")


run_rl = rl_from_config
