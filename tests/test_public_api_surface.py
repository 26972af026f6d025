"""The public API surface per package: every name a user of the reference framework
imports from a package (its ``__all__``, avgen/*/__init__.py) resolves here under the
same package path, so code ports by changing the top-level package name."""
from __future__ import annotations

import importlib

import pytest

SURFACE: dict[str, tuple[str, ...]] = {
    "avgen_b200": (
        "ActivationCheckpointConfig", "CheckpointManager", "ConditionMode", "DistributedEnv", "EvalReport",
        "FSDPConfig", "FlowMatchingObjective", "GenerationPipeline", "GridPatchifier", "MediaBatch",
        "MediaBatchSpec", "ModelInput", "ModelOutput", "ModelShape", "ParallelConfig", "ParallelDims",
        "ParallelModel", "PatchLayout", "Patchifier", "PipelineConfig", "PrecisionConfig", "RNGStreams",
        "RunConfig", "SimulationReport", "StepMetrics", "SyntheticSource", "TextContext", "TokenStream",
        "TrainState", "Trainer", "__version__", "build_loader", "build_model", "init_distributed",
        "list_models", "load_config", "parallelize", "run_eval_suite", "shutdown_distributed",
        "simulate_config", "train_step"
    ),
    "avgen_b200.checkpoint": (
        "CHECKPOINT_DIR_PREFIX", "CHECKPOINT_FORMAT_VERSION", "CheckpointEntry", "CheckpointManager",
        "DEFAULT_MAX_SHARD_BYTES", "EMA_KEY", "EXTRAS_KEY", "ExtrasState", "INDEX_FILENAME",
        "MARKER_FILENAME", "MODEL_OPTIMIZER_KEY", "ModelOptimizerState", "PROGRESS_KEY", "ProgressState",
        "RNGState", "RNG_KEY", "SCHEDULE_KEY", "WEIGHTS_FILENAME", "build_stateful", "convert",
        "export_huggingface", "export_safetensors", "import_safetensors", "load", "load_ema", "load_model",
        "save"
    ),
    "avgen_b200.cli": (
        "build_parser", "main"
    ),
    "avgen_b200.codecs": (
        "AudioCodec", "DiffusersVideoCodec", "LatentStatistics", "MelConfig", "MelFrontend",
        "ReferenceAudioCodec", "ReferenceTextEncoder", "ReferenceVideoCodec", "TextEncoder", "TilingConfig",
        "TransformersTextEncoder", "VideoCodec", "Vocoder", "blend_tiles", "codec_fingerprint",
        "denormalize_latents", "hz_to_mel", "mel_filterbank", "mel_to_hz", "normalize_latents",
        "resolve_latent_normalization", "stft_magnitude"
    ),
    "avgen_b200.config": (
        "ActivationSpec", "BucketConfig", "CheckpointConfig", "ConfigError", "DataConfig", "EvalConfig",
        "FSDPSpec", "FinetuneConfig", "InferenceConfig", "ModelConfig", "ParallelConfigSpec",
        "PipelineSpec", "PrecisionSpec", "RLConfig", "RunConfig", "SCHEMA_VERSION", "TelemetryConfig",
        "TrainConfig", "apply_overrides", "build_accelerator", "build_activation_checkpoint",
        "build_fsdp_config", "build_interconnects", "build_model", "build_model_shape",
        "build_parallel_config", "build_parallel_dims", "build_pipeline_config", "build_precision_config",
        "config_diff", "format_diff", "gradient_accumulation", "load_config", "load_mapping",
        "model_kwargs", "parse_override", "save_config", "sequence_length_for", "to_mapping"
    ),
    "avgen_b200.core": (
        "ConditionMode", "DataCursor", "EMA", "GridPatchifier", "LRSchedule", "MediaBatch",
        "MediaBatchSpec", "ModelInput", "ModelOutput", "PatchLayout", "Patchifier", "RNGStreams",
        "Stateful", "StepMetrics", "TensorBundle", "TensorBundleSpec", "TensorDType", "TextContext",
        "TokenStream", "TrainState", "build_spatial_coords", "build_temporal_coords",
        "null_text_conditioning", "patchify_grid", "stack_batches", "unpatchify_grid"
    ),
    "avgen_b200.data": (
        "AlignmentTruth", "Bucket", "BucketBatch", "BucketCurriculum", "BucketPlan", "BucketSampler",
        "ClipProbe", "ClipQA", "ClipReport", "ClipSpec", "ConcatShardReader", "CurriculumPhase",
        "DataSource", "IngestSummary", "LatentSample", "LoaderConfig", "LoaderCursor", "PackPlan",
        "PackedLayout", "QualityGate", "RejectionReason", "SampleDescriptor", "SampleStore",
        "ShardCorruptionError", "ShardManifest", "ShardReader", "ShardRecord", "ShardedLoader",
        "SyntheticConfig", "SyntheticSource", "assign_buckets", "bucket_from_descriptor",
        "build_latent_sample", "build_loader", "collate_samples", "content_fingerprint", "iter_clip_table",
        "largest_remainder", "pack_streams", "plan_clip_spec", "plan_packing", "probe_clip", "split_packed",
        "summarise_reports", "tensor_fingerprint", "validate_shard", "write_shard"
    ),
    "avgen_b200.eval": (
        "AVSyncProxy", "AudioBandwidth", "AudioSilence", "DEFAULT_PROMPTS", "EvalBatch", "EvalPin",
        "EvalReport", "FirstFrameFidelity", "FlickerIndex", "IncomparableReports",
        "InpaintBoundaryConsistency", "LearnedMetricSpec", "Metric", "MetricBundle", "MetricError",
        "MissingBackendError", "MotionMagnitude", "RunningMetric", "SaturationClipping", "SeamContinuity",
        "SharpnessProxy", "StaticFrameRatio", "TemporalConsistency", "available_learned_metrics",
        "build_learned_metric", "build_metric", "build_metrics", "capture_environment", "compare_reports",
        "describe_learned_metrics", "describe_metrics", "format_comparison", "frechet_distance",
        "learned_metric_available", "learned_metric_summary", "list_learned_metrics", "list_metrics",
        "metric_class", "prompt_set_digest", "register_learned_metric", "register_metric",
        "require_backend", "run_eval_suite", "shard_prompts"
    ),
    "avgen_b200.finetune": (
        "AdapterHandles", "ControlAdapter", "ControlAdapterConfig", "DistillationConfig", "FinetuneStage",
        "IPAdapter", "IPAdapterConfig", "LoRAConfig", "LoRALinear", "TimestepPlan", "TrainableSummary",
        "adapter_state_dict", "apply_lora", "apply_stage", "freeze_all", "freeze_except", "freeze_matching",
        "get_stage", "list_stages", "load_adapter", "lora_modules", "lora_parameters",
        "mark_only_lora_trainable", "merge_lora", "register_stage", "resolution_shift", "save_adapter",
        "shift_timesteps", "stage_names_for", "standard_stages", "trainable_summary", "unmerge_lora"
    ),
    "avgen_b200.infer": (
        "DPMSolverPlusPlus2M", "EulerAncestralSampler", "EulerSampler", "GeneratedMedia",
        "GenerationConfig", "GenerationPipeline", "GuidanceConfig", "HeunSampler", "ResMultistepSampler",
        "Sampler", "SamplerConfig", "ScheduleConfig", "SigmaSchedule", "StreamState",
        "adaptive_projected_guidance", "apply_guidance", "apply_modality_guidance", "apply_shift",
        "build_model_input", "build_sampler", "build_sigma_schedule", "classifier_free_guidance",
        "condition_first_frame", "condition_mask", "condition_stream", "condition_temporal_prefix",
        "default_audio_patchifier", "first_frame_mask", "karras_sigmas", "linear_quadratic_sigmas",
        "linear_sigmas", "list_samplers", "list_sigma_schedules", "register_sampler",
        "register_sigma_schedule", "rescale_guidance", "resolution_shift", "temporal_prefix_mask",
        "to_epsilon", "to_x0", "unconditional_branch", "unconditional_input"
    ),
    "avgen_b200.models": (
        "AVDiT", "AVDiTConfig", "AdaLNModulation", "CrossAttention", "CrossModalFusion", "DiTBlock",
        "FUSION_MODES", "MODEL_ENTRY_POINT_GROUP", "MODULATION_CHUNKS", "ROPE_SCALING_MODES", "RoPEScaling",
        "RotaryEmbedding", "RotaryTables", "SelfAttention", "SwiGLU", "TextRefinerBlock",
        "TimestepEmbedding", "VideoDiT", "VideoDiTConfig", "apply_rotary", "attention",
        "attention_backends", "build_model", "build_rotary_tables", "device_arch", "init_linear",
        "init_norm", "key_padding_mask", "list_models", "list_presets", "model_config_class", "modulate",
        "preset", "register_model", "rms_norm", "rope_axis_pairs", "sdpa_context", "sinusoidal_embedding",
        "temporal_neighbour_mask"
    ),
    "avgen_b200.parallel": (
        "ACMode", "ActivationCheckpointConfig", "DistributedEnv", "FSDPConfig", "ParallelConfig",
        "ParallelDims", "ParallelModel", "PipelineConfig", "PrecisionConfig", "TensorParallelPlan",
        "TensorParallelizable", "all_gather_object", "all_reduce_max", "all_reduce_mean", "all_reduce_sum",
        "apply_activation_checkpointing", "apply_fsdp", "apply_tensor_parallel", "balanced_split_points",
        "barrier", "broadcast_object", "build_pipeline_schedule", "clip_grad_norm", "collective_timeout",
        "context_parallel_region", "convert_to_float8", "data_mesh", "float8_available", "gather_object",
        "gather_stream", "gather_tokens", "init_distributed", "is_distributed_launch", "local_rank_device",
        "pad_to_multiple", "parallelize", "shard_stream", "sharded_length", "shutdown_distributed",
        "split_model", "standard_block_plan", "standard_root_plan", "submesh", "summarize_sharding",
        "unwrap_model"
    ),
    "avgen_b200.rl": (
        "AVSyncProxyReward", "CompositeReward", "DPOConfig", "DPOObjective", "GRPOConfig", "GRPOMetrics",
        "GRPOTrainer", "HPSv2Reward", "MotionMagnitudeReward", "PickScoreReward", "RewardModel",
        "RolloutBatch", "RolloutBuffer", "RunningNormalizer", "SDEStep", "TemporalConsistencyReward",
        "VelocityFn", "VideoScoreReward", "WindowSchedule", "build_reward", "clipped_surrogate",
        "diffusion_coefficient", "distribute_prompts", "dpo_loss", "gather_rewards", "gaussian_log_prob",
        "generate_group", "group_advantages", "kl_penalty", "list_rewards", "media_tensors",
        "model_velocity_fn", "ode_step", "register_reward", "regulated_log_ratio", "rollout_velocity_batch",
        "to_sde"
    ),
    "avgen_b200.simulate": (
        "A100_80GB", "Accelerator", "B200", "CollectiveCost", "CommunicationEstimate", "ComputeEstimate",
        "ETHERNET_200G", "FakeWorld", "H100_SXM", "H200_SXM", "INFINIBAND_NDR", "Interconnect",
        "MemoryEstimate", "ModelShape", "NVLINK4", "NVLINK5", "OPTIMIZER_BYTES", "PlanCandidate",
        "SearchSpace", "SimulationReport", "TraceArtifacts", "calibrate_from_busbw", "calibration_error",
        "capture_execution_trace", "capture_with_timing", "count_collectives", "estimate_compute",
        "estimate_memory", "estimate_step_communication", "fake_tensors", "fake_world", "measure_memory",
        "measure_runtime", "meta_init", "render_plan_table", "search_parallel_plan", "simulate_config",
        "simulate_rank", "suggest_activation_policy", "transformer_flops"
    ),
    "avgen_b200.telemetry": (
        "ConsoleLogger", "JSONLLogger", "Logger", "MemoryReport", "MemoryReporter", "MetricAccumulator",
        "MultiLogger", "NoOpLogger", "RankGatedLogger", "TensorBoardLogger", "ThroughputMeter",
        "ThroughputReport", "WandbLogger", "build_logger", "flight_recorder_dump", "memory_snapshot",
        "merge_metrics", "profile_steps", "should_profile_rank"
    ),
    "avgen_b200.train": (
        "ConditioningPlan", "ConditioningSampler", "Curriculum", "CurriculumStage",
        "DEFAULT_NO_DECAY_PATTERNS", "FlowMatchingConfig", "FlowMatchingObjective", "LogitNormalSampler",
        "MetricSink", "ModeSampler", "MultiTaskConditioning", "Objective", "ObjectiveOutput",
        "ResolutionBucket", "ShardedEMA", "ShiftedLogitNormalSampler", "TimestepSampler", "Trainer",
        "TrainerCallback", "TrainerConfig", "UniformSampler", "build_optimizer", "build_param_groups",
        "build_schedule", "build_timestep_sampler", "default_mode_weights", "list_optimizers",
        "list_schedules", "list_timestep_samplers", "register_schedule", "register_timestep_sampler",
        "resolution_shift", "shift_timesteps", "train_step"
    ),
}


@pytest.mark.parametrize("package", sorted(SURFACE))
def test_package_exports_every_public_name(package: str) -> None:
    module = importlib.import_module(package)
    exported = set(getattr(module, "__all__", ()))
    missing = [name for name in SURFACE[package] if not hasattr(module, name)]
    unlisted = [name for name in SURFACE[package] if name not in exported]
    assert not missing, f"{package} lacks {missing}"
    assert not unlisted, f"{package}.__all__ lacks {unlisted}"
