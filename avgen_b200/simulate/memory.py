"""Analytic per-rank memory model (avgen/simulate/memory.py:47-358 API).

``estimate_memory(shape, dims, ...)`` returns parameter / gradient / optimizer /
activation / FSDP-gather / workspace bytes for one rank. Activations follow the
checkpoint policy:

* ``fused`` (this framework's DiT block): the block saves its input and the
  self-attention output plus log-sum-exp; everything else is recomputed, and
  one block's recompute working set is live during backward;
* ``none`` / ``full`` / ``selective_layer`` / ``selective_op``: the eager
  policies of the reference, with the per-block eager activation footprint.

``measure_memory`` runs PyTorch's ``MemTracker`` around a step for calibration.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any

import torch
from torch import nn

__all__ = ["OPTIMIZER_BYTES", "MemoryEstimate", "ModelShape", "calibration_error", "estimate_memory",
           "measure_memory"]

_GIB = 1024.0 ** 3
# fp32 master + moments, in bytes per parameter, on top of the compute copy
OPTIMIZER_BYTES: dict[str, int] = {"sgd": 4, "sgd_momentum": 8, "adamw": 12, "adamw_bf16_state": 8,
                                   "adafactor": 5, "muon": 8, "adamw_8bit": 6}


@dataclass(frozen=True, slots=True)
class ModelShape:
    parameters: int
    depth: int
    width: int
    sequence_length: int
    micro_batch_size: int = 1
    mlp_ratio: int = 4
    num_heads: int = 16
    text_tokens: int = 0
    ffn_hidden: int = 0
    ffn: str = "swiglu"

    @property
    def hidden(self) -> int:
        return self.ffn_hidden or self.mlp_ratio * self.width


@dataclass(frozen=True, slots=True)
class MemoryEstimate:
    parameter_bytes: float
    gradient_bytes: float
    optimizer_bytes: float
    activation_bytes: float
    gather_bytes: float
    workspace_bytes: float

    @property
    def total_bytes(self) -> float:
        return sum(asdict(self).values())

    @property
    def total_gib(self) -> float:
        return self.total_bytes / _GIB

    def fits_in(self, device_gib: float, *, headroom: float = 0.1) -> bool:
        return self.total_gib <= device_gib * (1.0 - headroom)

    def breakdown_gib(self) -> dict[str, float]:
        return dict(sorted(((k, v / _GIB) for k, v in asdict(self).items()), key=lambda kv: kv[1], reverse=True))

    def dominant_term(self) -> str:
        return max(asdict(self).items(), key=lambda kv: kv[1])[0]


def _eager_block_bytes(shape: ModelShape, tokens: float, dtype_bytes: int) -> float:
    """Everything eager autograd keeps for one block (norms, q/k/v, attention, FFN)."""
    h = tokens * shape.width * dtype_bytes
    attn = 7.0 * h
    ffn = tokens * shape.hidden * dtype_bytes * (3.0 if shape.ffn == "swiglu" else 2.0)
    cross = (h + 2.0 * shape.micro_batch_size * shape.text_tokens * shape.width * dtype_bytes
             if shape.text_tokens else 0.0)
    return attn + ffn + cross


def _fused_recompute_bytes(shape: ModelShape, tokens: float, dtype_bytes: int) -> float:
    """Live working set while one fused block runs its backward (recomputed GEMM
    outputs, attention backward buffers, fp32 weight-gradient buffers)."""
    h = tokens * shape.width * dtype_bytes
    inner = 10.0 * h + tokens * shape.hidden * dtype_bytes * 3.0
    wgrad = (4.0 * shape.width * shape.width + 3.0 * shape.width * shape.hidden) * 4.0
    return inner + wgrad


def estimate_memory(shape: ModelShape, dims: Any, *, activation_checkpoint: Any = None, param_dtype_bytes: int = 2,
                    optimizer: str = "adamw", fsdp_prefetch_depth: int = 1, workspace_gib: float = 2.0,
                    policy: str | None = None) -> MemoryEstimate:
    if optimizer not in OPTIMIZER_BYTES:
        raise KeyError(f"unknown optimizer {optimizer!r}; known: {', '.join(sorted(OPTIMIZER_BYTES))}")
    mode = policy or (activation_checkpoint.mode if activation_checkpoint is not None else "fused")
    shards = dims.dp_shard * dims.context * dims.tensor * dims.pipeline
    local = shape.parameters / max(1, shards)
    param = local * param_dtype_bytes
    grad = local * 4.0  # fp32 gradient accumulation
    opt = local * OPTIMIZER_BYTES[optimizer]
    seq = shape.sequence_length / max(1, dims.sequence_shard_size)
    tokens = shape.micro_batch_size * seq
    depth = shape.depth / max(1, dims.pipeline)
    boundary = tokens * shape.width * param_dtype_bytes
    if mode == "fused":
        lse = tokens * shape.num_heads * 4.0
        act = depth * (2.0 * boundary + lse) + _fused_recompute_bytes(shape, tokens, param_dtype_bytes)
    else:
        per_block = _eager_block_bytes(shape, tokens, param_dtype_bytes)
        if mode == "none":
            stored = depth
        elif mode == "full":
            stored = 1.0
        elif mode == "selective_layer":
            interval = getattr(activation_checkpoint, "layer_interval", 2)
            stored = depth - depth / interval + 1.0
        else:
            freq = getattr(activation_checkpoint, "save_op_frequency", 1)
            stored = depth * 0.35 / freq + 1.0
        act = per_block * stored + (boundary * depth if mode != "none" else 0.0)
    gather = 0.0
    if dims.dp_shard_enabled and shape.depth:
        gather = shape.parameters / shape.depth * param_dtype_bytes * (fsdp_prefetch_depth + 1) / max(
            1, dims.tensor * dims.pipeline)
    return MemoryEstimate(param, grad, opt, act, gather, workspace_gib * _GIB)


def measure_memory(model: nn.Module, optimizer: torch.optim.Optimizer, step: Any, *, is_fsdp: bool = False,
                   display: bool = False) -> dict[str, float]:
    """Peak bytes per device of ``step()`` measured with PyTorch's memory tracker."""
    if is_fsdp:
        from torch.distributed._tools.fsdp2_mem_tracker import FSDPMemTracker

        tracker: Any = FSDPMemTracker(model, optimizer)
    else:
        from torch.distributed._tools.mem_tracker import MemTracker

        tracker = MemTracker()
        tracker.track_external(model, optimizer)
    with tracker:
        step()
        if is_fsdp:
            tracker.reset_mod_stats()
            step()
    if display:
        tracker.display_modulewise_snapshots(depth=3, units="GiB")
    snap = tracker.get_tracker_snapshot("peak")
    return {str(dev): float(stats.get("Total", 0.0)) for dev, stats in snap.items()}


def calibration_error(predicted: MemoryEstimate, measured_bytes: float) -> dict[str, float]:
    err = predicted.total_bytes - measured_bytes
    return {"predicted_gib": predicted.total_gib, "measured_gib": measured_bytes / _GIB, "absolute_error_gib": err / _GIB,
            "relative_error": err / measured_bytes if measured_bytes else float("inf"),
            "dominant_term": predicted.dominant_term()}
