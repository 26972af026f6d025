"""Tensor parallelism over DTensor plans (avgen/parallel/tensor.py:81-230 API).

Column-parallel q/k/v and gate/up projections, row-parallel output and down
projections (one all-reduce per attention and per FFN). Attention heads split
across the tensor-parallel ranks (layers infer the local head count from the
local projection width). Every parallel style hands plain local tensors to the
rest of the block, so norms, adaLN modulation and the attention kernel see
ordinary tensors.

Uneven head counts (20 heads at tp=8) and sequence parallelism (norms and
residuals on token shards) take the head-parallel path of
:mod:`avgen_b200.parallel.heads` instead of the DTensor plans.
"""
from __future__ import annotations

from typing import Protocol, runtime_checkable

from torch import nn


def _is_block_list(blocks: object) -> bool:
    from avgen_b200.parallel.pipeline import is_block_list

    return is_block_list(blocks)


__all__ = ["TensorParallelPlan", "TensorParallelizable", "apply_tensor_parallel", "standard_block_plan",
           "standard_root_plan"]

TensorParallelPlan = dict  # name -> torch ParallelStyle


@runtime_checkable
class TensorParallelizable(Protocol):
    def tensor_parallel_plan(self, *, sequence_parallel: bool) -> tuple[TensorParallelPlan, TensorParallelPlan]: ...


def _no_sp(sequence_parallel: bool) -> None:
    if sequence_parallel:
        raise NotImplementedError("the DTensor plans have no sequence parallelism; use style='heads' "
                                  "(apply_tensor_parallel picks it automatically)")


def standard_block_plan(*, sequence_parallel: bool = False, attention_prefix: str = "attention",
                        feedforward_prefix: str = "feed_forward",
                        cross_attention_prefix: str | None = "cross_attention",
                        ffn_projections: tuple[str, ...] = ("gate_proj", "up_proj")) -> TensorParallelPlan:
    from torch.distributed.tensor.parallel import ColwiseParallel, RowwiseParallel

    _no_sp(sequence_parallel)
    plan: TensorParallelPlan = {}
    for prefix in (attention_prefix, cross_attention_prefix):
        if prefix is None:
            continue
        for name in ("q_proj", "k_proj", "v_proj"):
            plan[f"{prefix}.{name}"] = ColwiseParallel()
        plan[f"{prefix}.out_proj"] = RowwiseParallel()
    for name in ffn_projections:
        plan[f"{feedforward_prefix}.{name}"] = ColwiseParallel()
    plan[f"{feedforward_prefix}.down_proj"] = RowwiseParallel()
    return plan


def standard_root_plan(*, sequence_parallel: bool = False) -> TensorParallelPlan:
    _no_sp(sequence_parallel)
    return {}


def _heads_divide(model: nn.Module, tp: int, block_attribute: str) -> bool:
    for block in getattr(model, block_attribute, ()):
        for name in ("attention", "cross_attention"):
            att = getattr(block, name, None)
            if att is not None and (att.num_heads % tp or getattr(att, "num_kv_heads", att.num_heads) % tp):
                return False
    return True


def apply_tensor_parallel(model: nn.Module, mesh, *, sequence_parallel: bool = False,  # noqa: ANN001
                          block_attribute: str = "blocks", root_plan: TensorParallelPlan | None = None,
                          block_plan: TensorParallelPlan | None = None, style: str = "auto") -> nn.Module:
    """Shard the blocks over the tensor-parallel ``mesh``.

    ``style="dtensor"``: torch DTensor plans (equal column / row chunks; the head
    counts must divide by the degree; no sequence parallelism). ``style="heads"``:
    whole heads per rank with uneven splits and optional sequence-parallel norms
    (:mod:`avgen_b200.parallel.heads`). ``"auto"`` takes DTensor plans when the
    heads divide and no sequence parallelism is asked for, else heads."""
    from torch.distributed.tensor.parallel import parallelize_module

    if style not in ("auto", "dtensor", "heads"):
        raise ValueError(f"style must be auto, dtensor or heads; got {style!r}")
    if style == "auto":
        style = "dtensor" if (not sequence_parallel and _heads_divide(model, mesh.size(), block_attribute)
                              and block_plan is None) else "heads"
    if style == "heads":
        from avgen_b200.parallel.heads import apply_head_parallel

        if block_plan is not None or root_plan:
            raise ValueError("custom DTensor plans go with style='dtensor'")
        apply_head_parallel(model, mesh, sequence_parallel=sequence_parallel, block_attribute=block_attribute)
        return model
    _no_sp(sequence_parallel)
    if root_plan is None or block_plan is None:
        if isinstance(model, TensorParallelizable):
            derived_root, derived_block = model.tensor_parallel_plan(sequence_parallel=sequence_parallel)
        else:
            derived_root, derived_block = standard_root_plan(), None
        root_plan = root_plan if root_plan is not None else derived_root
        block_plan = block_plan if block_plan is not None else derived_block
    blocks = getattr(model, block_attribute, None)
    if not _is_block_list(blocks):
        raise AttributeError(f"{type(model).__name__} has no nn.ModuleList {block_attribute!r}")
    if root_plan:
        parallelize_module(model, mesh, root_plan)
    tp = mesh.size()
    for block in blocks:
        plan = dict(block_plan) if block_plan is not None else _block_plan_for(block)
        _check_heads(block, tp)
        parallelize_module(block, mesh, plan)
        _sum_head_local_grads(block, mesh.get_group())
        if hasattr(block, "use_fused"):
            block.use_fused = False  # DTensor weights run the module path of every linear
    return model


def _sum_head_local_grads(block: nn.Module, group) -> None:  # noqa: ANN001
    """QK-norm weights are replicated but each rank applies them to its own heads only, so
    each rank holds a partial gradient: sum them over the tensor-parallel group."""
    import torch.distributed as dist

    def hook(grad):  # noqa: ANN001, ANN202
        grad = grad.clone()
        dist.all_reduce(grad, op=dist.ReduceOp.SUM, group=group)
        return grad

    for name in ("attention", "cross_attention"):
        att = getattr(block, name, None)
        for norm_name in ("q_norm", "k_norm"):
            w = getattr(getattr(att, norm_name, None), "weight", None)
            if isinstance(w, nn.Parameter) and w.requires_grad:
                w.register_hook(hook)


def _block_plan_for(block: nn.Module) -> TensorParallelPlan:
    ff = getattr(block, "feed_forward", None)
    projections = ("gate_proj", "up_proj") if hasattr(ff, "gate_proj") else ("up_proj",)
    cross = "cross_attention" if getattr(block, "cross_attention", None) is not None else None
    return standard_block_plan(cross_attention_prefix=cross, ffn_projections=projections)


def _check_heads(block: nn.Module, tp: int) -> None:
    for name in ("attention", "cross_attention"):
        att = getattr(block, name, None)
        if att is None:
            continue
        heads = getattr(att, "num_heads", 0)
        kv = getattr(att, "num_kv_heads", heads)
        if heads % tp or kv % tp:
            raise ValueError(f"{name}: {heads} query / {kv} kv heads do not split over tensor parallel degree {tp}")
