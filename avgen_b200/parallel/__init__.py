"""Distributed runtime: topology, process groups, comm, FSDP/TP/CP/PP, activation checkpointing."""
from avgen_b200.parallel.comm import (all_gather_object, all_reduce_max, all_reduce_mean, all_reduce_sum,
                                      broadcast_object, clip_grad_norm, data_mesh, gather_object)
from avgen_b200.parallel.context import (ContextParallelAttention, apply_context_parallel, context_parallel_region,
                                         cp_attention, gather_stream, gather_tokens, maybe_context_parallel,
                                         pad_to_multiple, shard_stream, sharded_length)
from avgen_b200.parallel.dims import MESH_DIM_ORDER, ParallelDims, submesh
from avgen_b200.parallel.env import (DistributedEnv, barrier, collective_timeout, init_distributed,
                                     is_distributed_launch, local_rank_device, shutdown_distributed, unwrap_model)

__all__ = [
    "MESH_DIM_ORDER", "ContextParallelAttention", "DistributedEnv", "ParallelDims", "all_gather_object",
    "all_reduce_max", "all_reduce_mean", "all_reduce_sum", "apply_context_parallel", "barrier", "broadcast_object",
    "clip_grad_norm", "collective_timeout", "context_parallel_region", "cp_attention", "data_mesh", "gather_object",
    "gather_stream", "gather_tokens", "init_distributed", "is_distributed_launch", "local_rank_device",
    "maybe_context_parallel", "pad_to_multiple", "shard_stream", "sharded_length", "shutdown_distributed", "submesh",
    "unwrap_model",
]
