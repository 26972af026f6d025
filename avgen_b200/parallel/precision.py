"""Mixed precision and fp8 (avgen/parallel/precision.py:84-284 API).

On this framework's hot path the sm_100a kernels pick their own types: the fused
block reads bf16 copies of fp32 master weights and accumulates in fp32, so a
precision config mostly matters for what FSDP2 stores and reduces. That is one
``MixedPrecisionPolicy`` with ``cast_forward_inputs=False`` (fp32 coordinates
and noise levels are never cast). fp8 training of large linears goes through
torchao's float8 recipes when that package is installed; the field names below
are the reference's configuration keys.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass
from typing import Literal

import torch
from torch import nn

from avgen_b200.core.limits import Limit, enforce

__all__ = ["PrecisionConfig", "convert_to_float8", "float8_available", "resolve_dtype"]

DTypeName = Literal["float32", "bfloat16", "float16"]

# every accepted spelling of each floating type
_ALIASES: dict[torch.dtype, tuple[str, ...]] = {torch.float32: ("float32", "fp32"),
                                                torch.bfloat16: ("bfloat16", "bf16"),
                                                torch.float16: ("float16", "fp16")}
_BY_NAME = {name: dtype for dtype, names in _ALIASES.items() for name in names}

# Linears that stay in bf16 under fp8: the embeddings, the output projection and
# the modulation/time MLPs are small, precision-sensitive or both.
_KEEP_BF16 = ("patch_embed", "proj_in", "proj_out", "final", "time_embed", "text_proj", "modulation")


def resolve_dtype(name: str | torch.dtype) -> torch.dtype:
    if isinstance(name, torch.dtype):
        return name
    dtype = _BY_NAME.get(name.lower())
    if dtype is None:
        raise KeyError(f"unknown dtype {name!r}; supported: {', '.join(sorted(_BY_NAME))}")
    return dtype


@dataclass(frozen=True, slots=True)
class PrecisionConfig:
    param_dtype: DTypeName = "bfloat16"
    reduce_dtype: DTypeName = "float32"
    output_dtype: DTypeName | None = None
    enable_float8: bool = False
    float8_min_features: int = 1024
    float8_exclude: tuple[str, ...] = _KEEP_BF16
    float8_recipe: Literal["tensorwise", "rowwise"] = "tensorwise"

    def __post_init__(self) -> None:
        for name in (self.param_dtype, self.reduce_dtype, self.output_dtype):
            if name is not None:
                resolve_dtype(name)  # raises on an unknown spelling
        enforce(self, {"float8_min_features": Limit(lo=1, integer=True)})
        if self.float8_recipe not in ("tensorwise", "rowwise"):
            raise ValueError(f"float8_recipe must be tensorwise or rowwise; got {self.float8_recipe!r}")
        if resolve_dtype(self.param_dtype) is torch.float16:
            warnings.warn("float16 parameters need loss scaling; bfloat16 is the native B200 training type",
                          RuntimeWarning, stacklevel=2)

    @property
    def param(self) -> torch.dtype:
        return resolve_dtype(self.param_dtype)

    @property
    def reduce(self) -> torch.dtype:
        return resolve_dtype(self.reduce_dtype)

    @property
    def output(self) -> torch.dtype | None:
        return resolve_dtype(self.output_dtype) if self.output_dtype is not None else None

    def fsdp_policy(self):  # noqa: ANN201
        from torch.distributed.fsdp import MixedPrecisionPolicy

        return MixedPrecisionPolicy(param_dtype=self.param, reduce_dtype=self.reduce, output_dtype=self.output,
                                    cast_forward_inputs=False)

    def autocast_dtype(self) -> torch.dtype | None:
        """The autocast type for modules outside the fused kernels (None: full precision)."""
        return self.param if self.param is not torch.float32 else None

    def float8_targets(self, model: nn.Module) -> list[str]:
        """Names of the linears fp8 training would convert: large enough on both sides,
        16-aligned (the fp8 GEMM's tile rule) and not on the keep-in-bf16 list."""
        out = []
        for name, module in model.named_modules():
            if not isinstance(module, nn.Linear) or any(tok in name for tok in self.float8_exclude):
                continue
            dims = (module.in_features, module.out_features)
            if min(dims) >= self.float8_min_features and all(d % 16 == 0 for d in dims):
                out.append(name)
        return out


def float8_available() -> bool:
    """torchao present and a device with fp8 tensor cores (compute capability >= 8.9)."""
    try:
        import torchao  # noqa: F401
    except ImportError:
        return False
    return torch.cuda.is_available() and torch.cuda.get_device_capability() >= (8, 9)


def convert_to_float8(model: nn.Module, config: PrecisionConfig) -> int:
    """Swap the eligible linears to float8 training (torchao); returns how many were converted."""
    if not config.enable_float8:
        return 0
    try:
        from torchao.float8 import Float8LinearConfig, convert_to_float8_training
    except ImportError as exc:
        raise RuntimeError("enable_float8=True needs torchao; install it or set enable_float8=False") from exc
    if not float8_available():
        warnings.warn(f"float8 requested without fp8 tensor cores; continuing in {config.param_dtype}",
                      RuntimeWarning, stacklevel=2)
        return 0
    targets = set(config.float8_targets(model))
    if targets:
        convert_to_float8_training(model, config=Float8LinearConfig.from_recipe_name(config.float8_recipe),
                                   module_filter_fn=lambda _m, n: n in targets)
    return len(targets)
