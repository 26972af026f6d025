"""Configuration: frozen schema, YAML loader with composition and overrides, resolution, diff."""
from avgen_b200.config.diff import config_diff, config_to_dict, format_diff, render_diff, save_config, to_mapping
from avgen_b200.config.loader import ConfigError, apply_overrides, load_config, load_mapping, parse_override
from avgen_b200.config.resolve import (build_accelerator, build_activation_checkpoint, build_fsdp_config,
                                       build_interconnects, build_model, build_model_shape, build_parallel_config,
                                       build_parallel_dims, build_pipeline_config, build_precision_config,
                                       gradient_accumulation, model_kwargs, sequence_length_for)
from avgen_b200.config.schema import (ActivationSpec, BucketConfig, CheckpointConfig, DataConfig, EvalConfig,
                                      FinetuneConfig, FSDPSpec, InferenceConfig, ModelConfig, ParallelConfigSpec,
                                      PipelineSpec, PrecisionSpec, RLConfig, RunConfig, SCHEMA_VERSION, TelemetryConfig,
                                      TrainConfig)

__all__ = ["ActivationSpec", "BucketConfig", "CheckpointConfig", "ConfigError", "DataConfig", "EvalConfig",
           "FSDPSpec", "FinetuneConfig", "InferenceConfig", "ModelConfig", "ParallelConfigSpec", "PipelineSpec",
           "PrecisionSpec", "RLConfig", "RunConfig", "SCHEMA_VERSION", "TelemetryConfig", "TrainConfig",
           "apply_overrides", "build_model", "format_diff", "to_mapping",
           "build_accelerator", "build_activation_checkpoint", "build_fsdp_config", "build_interconnects",
           "build_model_shape", "build_parallel_config", "build_parallel_dims", "build_pipeline_config",
           "build_precision_config", "gradient_accumulation", "model_kwargs", "sequence_length_for",
           "config_diff", "config_to_dict", "load_config", "load_mapping", "parse_override", "render_diff",
           "save_config"]
