"""Accelerator profiles, transformer FLOPs and step-time estimates
(avgen/simulate/compute.py:40-344 API).

The B200 profile is calibrated to this framework's kernels: dense peaks are the
measured cuBLAS bf16 throughput (burst / sustained under the 1 kW cap) when
``MEASURED_PEAKS.json`` is present, and each op class has its own achieved
fraction of that peak (tcgen05 GEMM, flash-attention forward and backward) so a
plan's time reflects where the step actually spends it. Attention backward
counts 2.5x its forward FLOPs (5 GEMM-shaped products against 2); the fused
DiT block recomputes every linear in backward but never the attention forward.
"""
from __future__ import annotations

import json
import os
from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Any, Literal

from avgen_b200.simulate.memory import ModelShape

__all__ = ["A100_80GB", "ACCELERATORS", "Accelerator", "B200", "ComputeEstimate", "H100_SXM", "H200_SXM",
           "KernelEfficiency", "estimate_compute", "measure_runtime", "suggest_activation_policy",
           "transformer_flops"]


@dataclass(frozen=True, slots=True)
class KernelEfficiency:
    """Achieved fraction of the accelerator's dense peak per op class."""

    gemm: float = 0.45
    attention_fwd: float = 0.45
    attention_bwd: float = 0.45


@dataclass(frozen=True, slots=True)
class Accelerator:
    name: str
    bf16_tflops: float
    memory_gib: float
    fp8_tflops: float = 0.0
    memory_bandwidth_tbps: float = 3.35
    sustained_bf16_tflops: float = 0.0
    kernels: KernelEfficiency = field(default_factory=KernelEfficiency)

    def peak_flops(self, *, fp8: bool = False, sustained: bool = False) -> float:
        if fp8 and self.fp8_tflops:
            return self.fp8_tflops * 1e12
        if sustained and self.sustained_bf16_tflops:
            return self.sustained_bf16_tflops * 1e12
        return self.bf16_tflops * 1e12


def _measured_b200() -> tuple[float, float, float]:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json"), encoding="utf-8") as fh:
            m = json.load(fh)
        return float(m["bf16_tflops"]), float(m["bf16_tflops_sustained"]), float(m["hbm_gbs"]) / 1000.0
    except (OSError, KeyError, ValueError):
        return 1590.0, 1400.0, 6.65


A100_80GB = Accelerator("A100 80GB", bf16_tflops=312.0, memory_gib=80.0, memory_bandwidth_tbps=2.0)
H100_SXM = Accelerator("H100 SXM", bf16_tflops=989.0, fp8_tflops=1979.0, memory_gib=80.0, memory_bandwidth_tbps=3.35)
H200_SXM = Accelerator("H200 SXM", bf16_tflops=989.0, fp8_tflops=1979.0, memory_gib=141.0,
                       memory_bandwidth_tbps=4.8)
_burst, _sustained, _hbm = _measured_b200()
B200 = Accelerator("B200", bf16_tflops=2250.0, fp8_tflops=4500.0, memory_gib=178.0, memory_bandwidth_tbps=_hbm,
                   sustained_bf16_tflops=_sustained,
                   # fractions of the nominal 2.25 PFLOP/s dense peak reached by this framework's kernels
                   kernels=KernelEfficiency(gemm=0.53, attention_fwd=0.50, attention_bwd=0.40))
ACCELERATORS = {"a100": A100_80GB, "h100": H100_SXM, "h200": H200_SXM, "b200": B200}


def transformer_flops(shape: ModelShape, *, include_backward: bool = True) -> dict[str, float]:
    """Model FLOPs of one micro-batch by op class (training = 3 x forward)."""
    s, w, d = float(shape.sequence_length), float(shape.width), float(shape.depth)
    hid = float(shape.hidden)
    projections = d * 4.0 * 2.0 * s * w * w
    attention = d * 4.0 * s * s * w
    ffn = d * (3.0 if shape.ffn == "swiglu" else 2.0) * 2.0 * s * w * hid
    cross = 0.0
    if shape.text_tokens:
        t = float(shape.text_tokens)
        cross = d * (2.0 * 2.0 * s * w * w + 2.0 * 2.0 * t * w * w + 4.0 * s * t * w)
    fwd = projections + attention + ffn + cross
    k = 3.0 if include_backward else 1.0
    b = float(shape.micro_batch_size)
    return {"projections": projections * k * b, "attention": attention * k * b, "feed_forward": ffn * k * b,
            "cross_attention": cross * k * b, "total": fwd * k * b,
            "attention_fraction": attention / fwd if fwd else 0.0, "head_dim": w / max(1, shape.num_heads)}


@dataclass(frozen=True, slots=True)
class ComputeEstimate:
    model_flops: float
    hardware_flops: float
    seconds: float
    accelerator: str
    achieved_fraction: float

    @property
    def recompute_overhead(self) -> float:
        return (self.hardware_flops - self.model_flops) / self.model_flops if self.model_flops > 0 else 0.0

    def mfu(self, step_seconds: float, peak_flops: float) -> float:
        return self.model_flops / (step_seconds * peak_flops) if step_seconds > 0 and peak_flops > 0 else 0.0

    def hfu(self, step_seconds: float, peak_flops: float) -> float:
        return self.hardware_flops / (step_seconds * peak_flops) if step_seconds > 0 and peak_flops > 0 else 0.0


def _recompute_fraction(mode: str, activation_checkpoint: Any) -> tuple[float, float]:
    """(extra linear fraction, extra attention-forward fraction) of the forward."""
    if mode == "fused":
        return 1.0, 0.0
    if mode == "full":
        return 1.0, 1.0
    if mode == "selective_layer":
        f = 1.0 / getattr(activation_checkpoint, "layer_interval", 2)
        return f, f
    if mode == "selective_op":
        return 0.25, 1.0  # elementwise recompute, and cuDNN attention is not on the save list
    return 0.0, 0.0


def estimate_compute(shape: ModelShape, dims: Any, *, accelerator: Accelerator = B200, activation_checkpoint: Any = None,
                     achieved_fraction: float | None = None, use_fp8: bool = False,
                     policy: str | None = None) -> ComputeEstimate:
    """Per-rank compute time of one micro-batch, per op class."""
    mode = policy or (activation_checkpoint.mode if activation_checkpoint is not None else "fused")
    f = transformer_flops(shape)
    fwd_lin = (f["projections"] + f["feed_forward"] + f["cross_attention"]) / 3.0
    fwd_attn = f["attention"] / 3.0
    lin_x, attn_x = _recompute_fraction(mode, activation_checkpoint)
    shard = max(1, dims.tensor * dims.context * dims.pipeline)
    lin_total = (3.0 + lin_x) * fwd_lin / shard
    attn_fwd = (1.0 + attn_x) * fwd_attn / shard
    attn_bwd = 2.5 * fwd_attn / shard
    peak = accelerator.peak_flops(fp8=use_fp8)
    k = accelerator.kernels
    if achieved_fraction is not None:
        k = KernelEfficiency(achieved_fraction, achieved_fraction, achieved_fraction)
    seconds = lin_total / (peak * k.gemm) + attn_fwd / (peak * k.attention_fwd) + attn_bwd / (peak * k.attention_bwd)
    hardware = lin_total + attn_fwd + attn_bwd
    model = f["total"] / shard
    eff = model / (seconds * peak) if seconds > 0 else 0.0
    return ComputeEstimate(model_flops=model, hardware_flops=hardware, seconds=seconds, accelerator=accelerator.name,
                           achieved_fraction=eff)


def measure_runtime(step: Callable[[], Any], *,
                    mode: Literal["operator-level-benchmark", "operator-level-cost-model"] = "operator-level-cost-model",
                    ) -> dict[str, float]:
    from torch.distributed._tools.runtime_estimator import RuntimeEstimator

    est = RuntimeEstimator()
    with est(mode):
        step()
    return {"total_ms": float(est.total_runtime),
            **{str(k): float(v) for k, v in getattr(est, "mod_runtimes", {}).items()}}


def suggest_activation_policy(shape: ModelShape, dims: Any, *, accelerator: Accelerator = B200,
                              headroom: float = 0.1) -> str:
    """The cheapest policy whose memory estimate fits (``fused`` first)."""
    from avgen_b200.simulate.memory import estimate_memory

    for mode in ("fused", "none", "selective_layer", "full"):
        if estimate_memory(shape, dims, policy=mode).fits_in(accelerator.memory_gib, headroom=headroom):
            return mode
    return "full"
