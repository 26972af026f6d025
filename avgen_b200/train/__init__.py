"""Training: flow-matching objective, samplers, conditioning, optimizer, schedules, EMA, trainer."""
from avgen_b200.train.conditioning import ConditioningPlan, ConditioningSampler, MultiTaskConditioning, default_mode_weights
from avgen_b200.train.ema import ShardedEMA
from avgen_b200.train.objective import (FlowMatchingConfig, FlowMatchingObjective, Objective, ObjectiveOutput,
                                        masked_flow_loss)
from avgen_b200.train.optimizer import (DEFAULT_NO_DECAY_PATTERNS, FusedAdamW, build_optimizer, build_param_groups,
                                        list_optimizers)
from avgen_b200.train.schedule import build_schedule, list_schedules, register_schedule
from avgen_b200.train.timestep import (LogitNormalSampler, ModeSampler, ShiftedLogitNormalSampler, TimestepSampler,
                                       UniformSampler, build_timestep_sampler, list_timestep_samplers,
                                       register_timestep_sampler, resolution_shift, shift_timesteps)
from avgen_b200.train.trainer import (Curriculum, CurriculumStage, MetricSink, ResolutionBucket, Trainer,
                                      TrainerTelemetry,
                                      TrainerCallback, TrainerConfig, optimizer_update, train_step)

__all__ = [
    "DEFAULT_NO_DECAY_PATTERNS", "ConditioningPlan", "ConditioningSampler", "Curriculum", "CurriculumStage",
    "FlowMatchingConfig", "FlowMatchingObjective", "FusedAdamW", "LogitNormalSampler", "MetricSink", "ModeSampler",
    "MultiTaskConditioning", "Objective", "ObjectiveOutput", "ResolutionBucket", "ShardedEMA",
    "ShiftedLogitNormalSampler", "TimestepSampler", "Trainer", "TrainerCallback", "TrainerConfig", "TrainerTelemetry", "UniformSampler",
    "build_optimizer", "build_param_groups", "build_schedule", "build_timestep_sampler", "default_mode_weights",
    "list_optimizers", "list_schedules", "list_timestep_samplers", "masked_flow_loss", "register_schedule",
    "optimizer_update", "register_timestep_sampler", "resolution_shift", "shift_timesteps", "train_step",
]
