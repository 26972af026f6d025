"""Distributed runtime: topology, process groups, comm, FSDP/HSDP, tensor / context / pipeline
parallelism, activation checkpointing, precision and ``parallelize``."""
from avgen_b200.parallel.activation import ActivationCheckpointConfig, apply_activation_checkpointing
from avgen_b200.parallel.apply import ParallelConfig, ParallelModel, parallelize
from avgen_b200.parallel.comm import (all_gather_object, all_reduce_max, all_reduce_mean, all_reduce_sum,
                                      broadcast_object, clip_grad_norm, data_mesh, gather_object)
from avgen_b200.parallel.context import (ContextParallelAttention, apply_context_parallel, context_parallel_region,
                                         cp_attention, gather_stream, gather_tokens, maybe_context_parallel,
                                         pad_to_multiple, shard_stream, sharded_length)
from avgen_b200.parallel.dims import MESH_DIM_ORDER, ParallelDims, submesh
from avgen_b200.parallel.env import (DistributedEnv, barrier, collective_timeout, init_distributed,
                                     is_distributed_launch, local_rank_device, shutdown_distributed, unwrap_model)
from avgen_b200.parallel.fsdp import FSDPConfig, apply_fsdp, set_prefetch_depth, summarize_sharding
from avgen_b200.parallel.pipeline import (PipelineConfig, balanced_split_points, build_pipeline_schedule, split_model,
                                          stage_for_rank)
from avgen_b200.parallel.precision import PrecisionConfig, convert_to_float8, float8_available, resolve_dtype
from avgen_b200.parallel.tensor import apply_tensor_parallel, standard_block_plan, standard_root_plan

__all__ = [
    "MESH_DIM_ORDER", "ActivationCheckpointConfig", "ContextParallelAttention", "DistributedEnv", "FSDPConfig",
    "ParallelConfig", "ParallelDims", "ParallelModel", "PipelineConfig", "PrecisionConfig", "all_gather_object",
    "all_reduce_max", "all_reduce_mean", "all_reduce_sum", "apply_activation_checkpointing",
    "apply_context_parallel", "apply_fsdp", "apply_tensor_parallel", "balanced_split_points", "barrier",
    "broadcast_object", "build_pipeline_schedule", "clip_grad_norm", "collective_timeout", "context_parallel_region",
    "convert_to_float8", "cp_attention", "data_mesh", "float8_available", "gather_object", "gather_stream",
    "gather_tokens", "init_distributed", "is_distributed_launch", "local_rank_device", "maybe_context_parallel",
    "pad_to_multiple", "parallelize", "resolve_dtype", "set_prefetch_depth", "shard_stream", "sharded_length",
    "shutdown_distributed", "split_model", "stage_for_rank", "standard_block_plan", "standard_root_plan", "submesh",
    "summarize_sharding", "unwrap_model",
]

from avgen_b200.parallel.activation import ACMode  # noqa: E402
from avgen_b200.parallel.tensor import TensorParallelizable, TensorParallelPlan  # noqa: E402

__all__ += ["ACMode", "TensorParallelPlan", "TensorParallelizable"]
