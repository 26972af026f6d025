"""``parallelize``: apply a parallel plan to a model (avgen/parallel/apply.py:49-259 API).

Order: float8 conversion -> tensor parallel -> ``adapt`` hook (LoRA, control
branches) -> activation checkpointing -> FSDP2/HSDP over the data (and
context) dimensions, or replicated data parallelism.

Parameters are sharded (FSDP2 over ``dp_shard_cp``, or HSDP) whenever
``dp_shard`` or ``cp`` is enabled, as in the reference. Replicated data
parallelism (``dp_replicate`` alone, or ``shard_parameters=False``) is native
by default: the model stays an ordinary module and the fused AdamW
all-reduces its flat fp32 gradient buffer once per step over
``ParallelModel.data_group`` (one collective, no per-bucket hooks). ``ParallelConfig(native_data_parallel=False)``
wraps the model in ``DistributedDataParallel`` instead.
"""
from __future__ import annotations

import warnings
from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Any

from torch import nn

from avgen_b200.parallel.activation import ActivationCheckpointConfig, apply_activation_checkpointing
from avgen_b200.parallel.dims import ParallelDims, submesh
from avgen_b200.parallel.fsdp import FSDPConfig, apply_fsdp
from avgen_b200.parallel.pipeline import PipelineConfig
from avgen_b200.parallel.precision import PrecisionConfig, convert_to_float8
from avgen_b200.parallel.tensor import apply_tensor_parallel

__all__ = ["ParallelConfig", "ParallelModel", "parallelize"]


@dataclass(frozen=True, slots=True)
class ParallelConfig:
    precision: PrecisionConfig = field(default_factory=PrecisionConfig)
    activation_checkpoint: ActivationCheckpointConfig = field(default_factory=ActivationCheckpointConfig)
    fsdp: FSDPConfig = field(default_factory=FSDPConfig)
    compile_blocks: bool = False
    compile_mode: str = "default"
    block_attribute: str = "blocks"
    sequence_parallel: bool = False
    native_data_parallel: bool = True
    shard_parameters: bool = True
    pipeline: PipelineConfig = field(default_factory=PipelineConfig)


@dataclass(frozen=True, slots=True)
class ParallelModel:
    model: nn.Module
    dims: ParallelDims
    mesh: Any
    applied: tuple[str, ...]
    pipeline: Any = None  # PipelineRunner of this rank's stage when pp > 1

    def submesh(self, name: str) -> Any:
        return submesh(self.mesh, name)

    @property
    def cp_mesh(self) -> Any:
        return self.submesh("cp")

    @property
    def pp_mesh(self) -> Any:
        return self.submesh("pp")

    @property
    def data_group(self) -> Any:
        """Process group the optimizer averages gradients over (native data parallelism): the
        replicated data ranks and the context-parallel ranks, which hold identical parameters."""
        if self.mesh is None or not any(a.startswith("native_dp") for a in self.applied):
            return None
        for name in ("dp_cp", "dp_replicate", "cp"):
            m = submesh(self.mesh, name)
            if m is not None:
                return m.get_group()
        return None


def _fsdp_mesh(dims: ParallelDims, mesh: Any) -> Any:
    if dims.dp_replicate_enabled:
        hsdp = submesh(mesh, "hsdp")
        if hsdp is not None:
            return hsdp
    for name in ("dp_shard_cp", "dp_shard", "cp"):
        m = submesh(mesh, name)
        if m is not None:
            return m
    return None


def parallelize(model: nn.Module, dims: ParallelDims, *, mesh: Any = None, config: ParallelConfig | None = None,
                adapt: Callable[[nn.Module], nn.Module] | None = None) -> ParallelModel:
    cfg = config or ParallelConfig()
    applied: list[str] = []
    if mesh is None and dims.world_size > 1:
        mesh = dims.build_mesh()
    runner = None
    if dims.pp_enabled and mesh is not None:
        from avgen_b200.parallel.pipeline import balanced_split_points, split_model, split_model_interleaved

        if cfg.pipeline.schedule == "zero_bubble":
            raise NotImplementedError("the zero-bubble schedule is not implemented; use 1f1b, gpipe or "
                                      "interleaved_1f1b")
        pp = submesh(mesh, "pp")
        stage, stages = pp.get_local_rank(), pp.size()
        depth = len(getattr(model, cfg.block_attribute))
        chunks = stages * cfg.pipeline.stages_per_rank
        points = balanced_split_points(depth, chunks, embedding_weight=cfg.pipeline.embedding_weight,
                                       head_weight=cfg.pipeline.head_weight)
        if cfg.pipeline.is_interleaved:
            model = split_model_interleaved(model, rank=stage, ranks=stages,
                                            chunks_per_rank=cfg.pipeline.stages_per_rank, split_points=points,
                                            block_attribute=cfg.block_attribute)
        else:
            model = split_model(model, stage_index=stage, num_stages=stages, split_points=points,
                                block_attribute=cfg.block_attribute)
        applied.append(f"pipeline(pp={stages}, stage={stage}, {cfg.pipeline.schedule}"
                       + (f", chunks_per_rank={cfg.pipeline.stages_per_rank})" if cfg.pipeline.is_interleaved
                          else ")"))
    n8 = convert_to_float8(model, cfg.precision)
    if n8:
        applied.append(f"float8({n8} linears)")
    if dims.tp_enabled and mesh is not None:
        apply_tensor_parallel(model, mesh["tp"], sequence_parallel=cfg.sequence_parallel,
                              block_attribute=cfg.block_attribute)
        heads = getattr(model, "head_parallel", None)
        applied.append(f"tensor_parallel(tp={dims.tensor}" + (
            f", heads, sequence_parallel={heads.sequence_parallel})" if heads is not None else ", dtensor)"))
    if adapt is not None:
        model = adapt(model)
        applied.append("adapt")
    if cfg.activation_checkpoint.enabled:
        apply_activation_checkpointing(model, cfg.activation_checkpoint, block_attribute=cfg.block_attribute)
        applied.append(f"activation_checkpoint({cfg.activation_checkpoint.mode})")
    if cfg.compile_blocks:
        warnings.warn("compile_blocks is ignored: blocks already run as fused sm_100a kernels", RuntimeWarning,
                      stacklevel=2)
    # Shard whenever there is a data-parallel or context-parallel dimension to
    # shard over (the reference's gate, avgen/parallel/apply.py:226-243): a cp-only
    # job still sums partial gradients, and sharding spreads parameters and
    # optimizer state over the context ranks too (the ``dp_shard_cp`` mesh).
    if mesh is not None and (dims.dp_shard_enabled or dims.cp_enabled) and cfg.shard_parameters:
        target = _fsdp_mesh(dims, mesh)
        if target is not None:
            apply_fsdp(model, target, precision=cfg.precision, config=cfg.fsdp)
            peer = "peer" if getattr(model, "_avgen_peer_collectives", None) else "nccl"
            if dims.dp_replicate_enabled:
                applied.append(f"hsdp(dp_replicate={dims.dp_replicate}, dp_shard={dims.dp_shard})")
            elif dims.dp_shard_enabled:
                applied.append(f"fsdp(dp_shard={dims.dp_shard}" + (f", cp={dims.context}" if dims.cp_enabled
                                                                   else "") + f", collectives={peer})")
            else:
                applied.append(f"fsdp(cp={dims.context}, collectives={peer})")
    elif mesh is not None and (dims.dp_replicate_enabled or dims.cp_enabled):
        if cfg.native_data_parallel:
            applied.append(f"native_dp(dp_replicate={dims.dp_replicate}, cp={dims.context})")
        else:
            from torch.nn.parallel import DistributedDataParallel

            name = "dp_cp" if submesh(mesh, "dp_cp") is not None else (
                "dp_replicate" if dims.dp_replicate_enabled else "cp")
            model = DistributedDataParallel(model, device_mesh=submesh(mesh, name), gradient_as_bucket_view=True)
            applied.append(f"ddp({name})")
    if dims.cp_enabled and mesh is not None:
        from avgen_b200.parallel.context import apply_context_parallel

        apply_context_parallel(model, submesh(mesh, "cp"))
        applied.append(f"context_parallel(cp={dims.context})")
    if dims.pp_enabled and mesh is not None:
        from avgen_b200.parallel.pipeline import InterleavedPipelineRunner, PipelineRunner

        group = submesh(mesh, "pp").get_group()
        if cfg.pipeline.is_interleaved:
            runner = InterleavedPipelineRunner(model, group, chunks_per_rank=cfg.pipeline.stages_per_rank)
        else:
            runner = PipelineRunner(model, group, schedule="gpipe" if cfg.pipeline.schedule == "gpipe" else "1f1b")
    if not applied:
        applied.append("single-device")
    return ParallelModel(model=model, dims=dims, mesh=mesh, applied=tuple(applied), pipeline=runner)
