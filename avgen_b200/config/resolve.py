"""Config -> runtime objects (avgen/config/resolve.py:56-405): parallel dims and
settings, model kwargs and model, simulator shapes and hardware profiles."""
from __future__ import annotations

import contextlib
import os
from typing import TYPE_CHECKING, Any

from avgen_b200.config.schema import BucketConfig, RunConfig

if TYPE_CHECKING:
    from torch import nn

__all__ = ["build_accelerator", "build_activation_checkpoint", "build_fsdp_config", "build_interconnects",
           "build_model", "build_model_shape", "build_parallel_config", "build_parallel_dims", "build_pipeline_config",
           "build_precision_config", "gradient_accumulation", "model_kwargs", "sequence_length_for"]


def build_parallel_dims(config: RunConfig, *, world_size: int | None = None):  # noqa: ANN201
    from avgen_b200.parallel.dims import ParallelDims

    s = config.parallel
    size = world_size if world_size is not None else int(os.environ.get("WORLD_SIZE", "1"))
    return ParallelDims(world_size=size, dp_replicate=s.dp_replicate, dp_shard=s.dp_shard, tensor=s.tensor,
                        context=s.context, pipeline=s.pipeline, enable_loss_parallel=s.enable_loss_parallel)


def build_precision_config(config: RunConfig):  # noqa: ANN201
    from avgen_b200.parallel.precision import PrecisionConfig

    s = config.parallel.precision
    return PrecisionConfig(param_dtype=s.param_dtype, reduce_dtype=s.reduce_dtype, enable_float8=s.enable_float8,
                           float8_min_features=s.float8_min_features, float8_recipe=s.float8_recipe)


def build_activation_checkpoint(config: RunConfig):  # noqa: ANN201
    from avgen_b200.parallel.activation import ActivationCheckpointConfig

    s = config.parallel.activation
    return ActivationCheckpointConfig(mode=s.mode, layer_interval=s.layer_interval,
                                      save_op_frequency=s.save_op_frequency)


def build_fsdp_config(config: RunConfig):  # noqa: ANN201
    from avgen_b200.parallel.fsdp import FSDPConfig

    s = config.parallel.fsdp
    return FSDPConfig(reshard_after_forward=s.reshard_after_forward, cpu_offload=s.cpu_offload,
                      shard_last_block_after_forward=s.shard_last_block_after_forward,
                      ignore_frozen_params=s.ignore_frozen_params)


def build_pipeline_config(config: RunConfig):  # noqa: ANN201
    from avgen_b200.parallel.pipeline import PipelineConfig

    s = config.parallel.pipeline_schedule
    return PipelineConfig(schedule=s.schedule, microbatches=s.microbatches, stages_per_rank=s.stages_per_rank)


def build_parallel_config(config: RunConfig):  # noqa: ANN201
    from avgen_b200.parallel.apply import ParallelConfig

    return ParallelConfig(precision=build_precision_config(config),
                          activation_checkpoint=build_activation_checkpoint(config), fsdp=build_fsdp_config(config),
                          compile_blocks=config.parallel.compile_blocks, compile_mode=config.parallel.compile_mode,
                          sequence_parallel=config.parallel.sequence_parallel)


def gradient_accumulation(config: RunConfig, *, world_size: int | None = None) -> int:
    dims = build_parallel_dims(config, world_size=world_size)
    return dims.gradient_accumulation_for(global_batch_size=config.train.global_batch_size,
                                          local_batch_size=config.micro_batch_size)


def sequence_length_for(config: RunConfig, bucket: BucketConfig | None = None) -> int:
    return (bucket or config.data.largest_bucket()).tokens(config.model)


def build_model_shape(config: RunConfig, *, bucket: BucketConfig | None = None, parameters: int | None = None):  # noqa: ANN201
    from avgen_b200.simulate.memory import ModelShape

    chosen = bucket or config.data.largest_bucket()
    tokens = chosen.tokens(config.model)
    if config.model.has_audio and config.data.audio_frames:
        tokens += config.data.audio_frames // config.model.patch_frames
    micro = config.train.micro_batch_size if config.train.micro_batch_size != -1 else chosen.micro_batch_size
    return ModelShape(parameters=parameters or counted_parameters(config), depth=config.model.depth,
                      width=config.model.width, sequence_length=tokens, micro_batch_size=micro,
                      mlp_ratio=config.model.mlp_ratio, num_heads=config.model.num_heads,
                      text_tokens=config.data.text_tokens if config.model.cross_attention else 0,
                      ffn=config.model.ffn)


_COUNTS: dict[str, int] = {}


def counted_parameters(config: RunConfig) -> int:
    """The parameter count of the model ``config`` builds, counted on the meta device
    (no memory), or the closed-form estimate when the model cannot be built here."""
    if config.model.parameters:
        return config.model.parameters
    key = repr((config.model, config.data.text_width, config.data.text_tokens, config.data.audio_channels))
    if key not in _COUNTS:
        try:
            model = build_model(config, meta=True)
            _COUNTS[key] = int(sum(p.numel() for p in model.parameters()))
        except Exception:  # noqa: BLE001 - a plugin model or an invalid shape: fall back to the formula
            _COUNTS[key] = config.model.estimated_parameters(text_width=config.data.text_width)
    return _COUNTS[key]


def build_accelerator(name: str):  # noqa: ANN201
    from avgen_b200.simulate.compute import ACCELERATORS

    key = name.strip().lower()
    if key not in ACCELERATORS:
        raise ValueError(f"unknown gpu {name!r}; known: {', '.join(sorted(ACCELERATORS))}")
    return ACCELERATORS[key]


def build_interconnects(gpu: str):  # noqa: ANN201
    from avgen_b200.simulate.comms import INFINIBAND_NDR, NVLINK4, NVLINK5

    return (NVLINK5 if gpu.strip().lower() == "b200" else NVLINK4), INFINIBAND_NDR


def model_kwargs(config: RunConfig) -> dict[str, Any]:
    m = config.model
    out: dict[str, Any] = {"depth": m.depth, "width": m.width, "num_heads": m.num_heads, "mlp_ratio": m.mlp_ratio,
                           "patch_frames": m.patch_frames, "patch_height": m.patch_height,
                           "patch_width": m.patch_width, "in_channels": m.in_channels,
                           "out_channels": m.latent_out_channels, "cross_attention": m.cross_attention,
                           "text_width": config.data.text_width, "rope_theta": m.rope_theta, "ffn": m.ffn}
    if m.cross_attention:
        out["text_context_length"] = config.data.text_tokens
    if m.has_audio:
        out["audio_width"] = m.audio_width
        out["audio_in_channels"] = config.data.audio_channels
    out.update(m.extra)
    return out


def build_model(config: RunConfig, *, meta: bool = False) -> nn.Module:
    import torch

    from avgen_b200.models.registry import build_model as _build

    ctx = torch.device("meta") if meta else contextlib.nullcontext()
    with ctx:
        return _build(config.model.name, model_kwargs(config))
