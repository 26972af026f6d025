"""Classifier-free guidance and its variants (avgen/infer/guidance.py:76-615 API).

* CFG: ``u + s (c - u)``;
* rescale (Lin et al., 2023): match the per-sample std of the guided prediction
  to the conditional one, blended by ``rescale``;
* APG (adaptive projected guidance, Sadat et al., 2024): split ``c - u`` into
  components parallel and orthogonal to ``c``, keep the orthogonal part and
  ``eta`` of the parallel one, optionally clamp the update norm;
* scale schedules over sampling progress: constant, linear, cosine, power and
  interval (guidance only inside ``[start_fraction, end_fraction]``);
* per-modality scales and chained multi-condition guidance.
"""
from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from dataclasses import asdict, dataclass
from typing import Any

import torch

from avgen_b200.core.limits import Limit, enforce
from avgen_b200.core.model_input import ModelInput

__all__ = ["GuidanceConfig", "adaptive_projected_guidance", "apply_guidance", "apply_modality_guidance",
           "classifier_free_guidance", "rescale_guidance", "unconditional_branch"]

_MODALITIES = ("text", "video", "audio")


# Scale schedules over sampling progress p in [0, 1]: each maps (config, p) to the
# fraction of the way from ``min_scale`` to ``scale`` (1 = full scale). "interval"
# holds full scale inside [start_fraction, end_fraction] and min_scale outside.
_SCHEDULE_WEIGHT = {
    "constant": lambda c, p: 1.0,
    "linear": lambda c, p: 1.0 - p,
    "cosine": lambda c, p: 0.5 * (1.0 + math.cos(math.pi * p)),
    "power": lambda c, p: (1.0 - p) ** c.schedule_power,
    "interval": lambda c, p: 1.0 if c.start_fraction <= p <= c.end_fraction else 0.0,
}
_SCHEDULES = tuple(_SCHEDULE_WEIGHT)
_POSITIVE = Limit(lo=0.0, lo_open=True)
_UNIT = Limit(lo=0.0, hi=1.0)
_GUIDANCE_LIMITS = {"scale": _POSITIVE, "min_scale": _POSITIVE, "schedule_power": _POSITIVE,
                    **{f"{m}_scale": Limit(lo=0.0, lo_open=True, optional=True) for m in _MODALITIES},
                    "rescale": _UNIT, "projection_eta": Limit(), "projection_threshold": Limit(lo=0.0),
                    "start_fraction": _UNIT, "end_fraction": _UNIT}


@dataclass(frozen=True, slots=True)
class GuidanceConfig:
    scale: float = 1.0
    text_scale: float | None = None
    video_scale: float | None = None
    audio_scale: float | None = None
    rescale: float = 0.0
    projection: bool = False
    projection_eta: float = 0.0
    projection_threshold: float = 0.0
    schedule: str = "constant"
    schedule_power: float = 1.0
    min_scale: float = 1.0
    start_fraction: float = 0.0
    end_fraction: float = 1.0

    def __post_init__(self) -> None:
        enforce(self, _GUIDANCE_LIMITS)
        if self.schedule not in _SCHEDULE_WEIGHT:
            raise ValueError(f"unknown guidance schedule {self.schedule!r}; choose from {', '.join(_SCHEDULES)}")
        if self.start_fraction >= self.end_fraction:
            raise ValueError("start_fraction must be below end_fraction")

    @property
    def is_enabled(self) -> bool:
        return self.scale != 1.0 or any(getattr(self, f"{m}_scale") not in (None, 1.0) for m in _MODALITIES)

    def scale_at(self, progress: float) -> float:
        """Guidance scale at sampling progress ``progress`` in [0, 1] (0 = first step)."""
        if not (math.isfinite(progress) and 0.0 <= progress <= 1.0):
            raise ValueError(f"progress must be in [0, 1]; got {progress!r}")
        if self.schedule == "constant":
            return self.scale  # exactly, whatever min_scale says
        weight = _SCHEDULE_WEIGHT[self.schedule](self, progress)
        if weight in (0.0, 1.0):  # the end points exactly
            return self.scale if weight else self.min_scale
        return self.min_scale + (self.scale - self.min_scale) * weight

    def modality_scale(self, modality: str, progress: float = 0.0) -> float:
        if modality not in _MODALITIES:
            raise ValueError(f"unknown guidance modality {modality!r}; choose from {', '.join(_MODALITIES)}")
        factor = getattr(self, f"{modality}_scale")
        return self.scale_at(progress) * (1.0 if factor is None else factor)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: Mapping[str, Any]) -> GuidanceConfig:
        names = set(cls.__dataclass_fields__)  # type: ignore[attr-defined]
        return cls(**{k: v for k, v in values.items() if k in names})


def unconditional_branch(inputs: ModelInput) -> ModelInput:
    return inputs.unconditional()


def _same(a: torch.Tensor, b: torch.Tensor) -> None:
    if tuple(a.shape) != tuple(b.shape) or a.device != b.device:
        raise ValueError(f"guidance branches must match in shape and device; got {tuple(a.shape)} on {a.device} "
                         f"and {tuple(b.shape)} on {b.device}")


def classifier_free_guidance(conditional: torch.Tensor, unconditional: torch.Tensor, scale: float) -> torch.Tensor:
    _same(conditional, unconditional)
    if scale == 1.0:
        return conditional
    return torch.lerp(unconditional, conditional, scale) if conditional.is_floating_point() else \
        unconditional + scale * (conditional - unconditional)


def _sample_dims(t: torch.Tensor) -> tuple[int, ...]:
    return tuple(range(1, t.ndim))


def rescale_guidance(guided: torch.Tensor, conditional: torch.Tensor, factor: float) -> torch.Tensor:
    _same(guided, conditional)
    if not (math.isfinite(factor) and 0.0 <= factor <= 1.0):
        raise ValueError(f"factor must be in [0, 1]; got {factor!r}")
    if factor == 0.0:
        return guided
    dims = _sample_dims(guided)
    ratio = conditional.std(dim=dims, keepdim=True) / guided.std(dim=dims, keepdim=True).clamp_min(1e-8)
    return torch.lerp(guided, guided * ratio, factor)


def adaptive_projected_guidance(conditional: torch.Tensor, unconditional: torch.Tensor, scale: float, *,
                                eta: float = 0.0, norm_threshold: float = 0.0) -> torch.Tensor:
    _same(conditional, unconditional)
    if not (math.isfinite(norm_threshold) and norm_threshold >= 0.0):
        raise ValueError(f"norm_threshold must be non-negative; got {norm_threshold!r}")
    if scale == 1.0:
        return conditional
    dims = _sample_dims(conditional)
    diff = conditional - unconditional
    if norm_threshold > 0.0:
        norm = torch.linalg.vector_norm(diff, dim=dims, keepdim=True)
        diff = diff * (norm_threshold / norm.clamp_min(1e-8)).clamp(max=1.0)
    coef = (diff * conditional).sum(dim=dims, keepdim=True) / (conditional * conditional).sum(
        dim=dims, keepdim=True).clamp_min(1e-8)
    parallel = coef * conditional
    return conditional + (scale - 1.0) * (diff - parallel + eta * parallel)


def apply_guidance(conditional: torch.Tensor, unconditional: torch.Tensor | None = None, *,
                   config: GuidanceConfig | None = None, progress: float = 0.0, modality: str = "text",
                   scale: float | None = None) -> torch.Tensor:
    if config is None or not config.is_enabled:
        return conditional
    s = config.modality_scale(modality, progress) if scale is None else scale
    if s == 1.0:
        return conditional
    if unconditional is None:
        raise ValueError("guidance is enabled but no unconditional prediction was given; evaluate the model on "
                         "ModelInput.unconditional() too, or set the scale to 1")
    if config.projection:
        guided = adaptive_projected_guidance(conditional, unconditional, s, eta=config.projection_eta,
                                             norm_threshold=config.projection_threshold)
    else:
        guided = classifier_free_guidance(conditional, unconditional, s)
    return rescale_guidance(guided, conditional, config.rescale)


def apply_modality_guidance(branches: Sequence[tuple[str, torch.Tensor]], *, config: GuidanceConfig,
                            progress: float = 0.0) -> torch.Tensor:
    """Chained guidance ``base + sum_i s_i (pred_i - pred_{i-1})`` over branches that add one
    condition each (e.g. unconditional -> +text -> +audio)."""
    if len(branches) < 2:
        raise ValueError(f"need a base branch and at least one conditioned branch; got {len(branches)}")
    base = branches[0][1]
    guided, prev = base, base
    for modality, pred in branches[1:]:
        _same(pred, base)
        guided = guided + config.modality_scale(modality, progress) * (pred - prev)
        prev = pred
    return rescale_guidance(guided, branches[-1][1], config.rescale)
