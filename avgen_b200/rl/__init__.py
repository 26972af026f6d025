"""Reward and preference post-training for flow models (avgen/rl/__init__.py API):
Flow-GRPO with MixGRPO windows and GRPO-Guard regulated ratios, Diffusion-DPO,
the marginal-preserving SDE, rollouts and rewards."""
from avgen_b200.rl.dpo import DPOConfig, DPOObjective, dpo_loss
from avgen_b200.rl.entry import build_rewards, rl_from_config, run_rl
from avgen_b200.rl.grpo import (GRPOConfig, GRPOMetrics, GRPOTrainer, WindowSchedule, clipped_surrogate, kl_penalty,
                                regulated_log_ratio)
from avgen_b200.rl.rewards import (AVSyncProxyReward, CompositeReward, HPSv2Reward, MLPScorerReward,
                                   MotionMagnitudeReward, PickScoreReward, RewardModel, RunningNormalizer,
                                   TemporalConsistencyReward, VideoScoreReward, build_reward, list_rewards,
                                   media_tensors, register_reward)
from avgen_b200.rl.rollout import (RolloutBatch, RolloutBuffer, VelocityFn, distribute_prompts, gather_rewards,
                                   generate_group, group_advantages, model_velocity_fn, rollout_velocity_batch)
from avgen_b200.rl.sde import SDEStep, diffusion_coefficient, gaussian_log_prob, ode_step, to_sde

__all__ = ["AVSyncProxyReward", "CompositeReward", "DPOConfig", "DPOObjective", "GRPOConfig", "GRPOMetrics",
           "GRPOTrainer", "HPSv2Reward", "MLPScorerReward", "MotionMagnitudeReward", "PickScoreReward", "RewardModel",
           "RolloutBatch", "RolloutBuffer", "RunningNormalizer", "SDEStep", "TemporalConsistencyReward", "VelocityFn",
           "VideoScoreReward", "WindowSchedule", "build_reward", "build_rewards", "clipped_surrogate",
           "diffusion_coefficient", "distribute_prompts", "dpo_loss", "gather_rewards", "gaussian_log_prob",
           "generate_group", "group_advantages", "kl_penalty", "list_rewards", "media_tensors", "model_velocity_fn",
           "ode_step", "register_reward", "regulated_log_ratio", "rl_from_config", "rollout_velocity_batch", "run_rl",
           "to_sde"]
