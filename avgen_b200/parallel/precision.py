"""Mixed precision and fp8 (avgen/parallel/precision.py:84-284 API).

Parameters are computed in bf16 by the sm_100a kernels (the fused block keeps
fp32 master weights and caches bf16 copies); gradients reduce in fp32.
``PrecisionConfig.fsdp_policy()`` gives the FSDP2 policy with
``cast_forward_inputs=False`` so fp32 coordinates and noise levels are never
cast. fp8 training of eligible linears uses torchao's float8 recipes when that
package is installed.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass
from typing import Literal

import torch
from torch import nn

__all__ = ["PrecisionConfig", "convert_to_float8", "float8_available", "resolve_dtype"]

DTypeName = Literal["float32", "bfloat16", "float16"]
_DTYPES: dict[str, torch.dtype] = {"float32": torch.float32, "fp32": torch.float32, "bfloat16": torch.bfloat16,
                                   "bf16": torch.bfloat16, "float16": torch.float16, "fp16": torch.float16}
_EXCLUDE = ("patch_embed", "proj_in", "proj_out", "final", "time_embed", "text_proj", "modulation")


def resolve_dtype(name: str | torch.dtype) -> torch.dtype:
    if isinstance(name, torch.dtype):
        return name
    try:
        return _DTYPES[name.lower()]
    except KeyError as exc:
        raise KeyError(f"unknown dtype {name!r}; supported: {', '.join(sorted(_DTYPES))}") from exc


@dataclass(frozen=True, slots=True)
class PrecisionConfig:
    param_dtype: DTypeName = "bfloat16"
    reduce_dtype: DTypeName = "float32"
    output_dtype: DTypeName | None = None
    enable_float8: bool = False
    float8_min_features: int = 1024
    float8_exclude: tuple[str, ...] = _EXCLUDE
    float8_recipe: Literal["tensorwise", "rowwise"] = "tensorwise"

    def __post_init__(self) -> None:
        resolve_dtype(self.param_dtype)
        resolve_dtype(self.reduce_dtype)
        if self.output_dtype is not None:
            resolve_dtype(self.output_dtype)
        if isinstance(self.float8_min_features, bool) or self.float8_min_features < 1:
            raise ValueError(f"float8_min_features must be >= 1; got {self.float8_min_features!r}")
        if self.float8_recipe not in ("tensorwise", "rowwise"):
            raise ValueError(f"float8_recipe must be tensorwise or rowwise; got {self.float8_recipe!r}")
        if self.param_dtype == "float16":
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
        return None if self.output_dtype is None else resolve_dtype(self.output_dtype)

    def fsdp_policy(self):  # noqa: ANN201
        from torch.distributed.fsdp import MixedPrecisionPolicy

        return MixedPrecisionPolicy(param_dtype=self.param, reduce_dtype=self.reduce, output_dtype=self.output,
                                    cast_forward_inputs=False)

    def autocast_dtype(self) -> torch.dtype | None:
        return None if self.param is torch.float32 else self.param


def float8_available() -> bool:
    """torchao present and a device with fp8 tensor cores (compute capability >= 8.9)."""
    try:
        import torchao  # noqa: F401
    except ImportError:
        return False
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability() >= (8, 9)


def _eligible(name: str, module: nn.Module, config: PrecisionConfig) -> bool:
    if not isinstance(module, nn.Linear) or any(tok in name for tok in config.float8_exclude):
        return False
    if min(module.in_features, module.out_features) < config.float8_min_features:
        return False
    return module.in_features % 16 == 0 and module.out_features % 16 == 0


def convert_to_float8(model: nn.Module, config: PrecisionConfig) -> int:
    """Swap eligible linears to float8 training (torchao); returns how many were converted."""
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
    names = {n for n, m in model.named_modules() if _eligible(n, m, config)}
    if not names:
        return 0
    convert_to_float8_training(model, config=Float8LinearConfig.from_recipe_name(config.float8_recipe),
                               module_filter_fn=lambda _m, n: n in names)
    return len(names)
