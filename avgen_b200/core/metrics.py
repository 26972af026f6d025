"""Per-step metrics as detached device scalars with a single host sync.

Same contract as avgen/core/metrics.py:21-120: nothing here forces a sync until
:meth:`StepMetrics.to_mapping` (one D2H copy of a stacked vector).
"""
from __future__ import annotations

from dataclasses import dataclass, fields

import torch
from torch.utils import _pytree

__all__ = ["StepMetrics"]


@dataclass(frozen=True, slots=True)
class StepMetrics:
    loss: torch.Tensor
    video_loss: torch.Tensor
    audio_loss: torch.Tensor
    valid_video_tokens: torch.Tensor
    valid_audio_tokens: torch.Tensor
    grad_norm: torch.Tensor
    nonfinite: torch.Tensor
    skipped: torch.Tensor

    def validate(self) -> None:
        for spec in fields(self):
            v = getattr(self, spec.name)
            if v.ndim != 0:
                raise ValueError(f"{spec.name} must be scalar")
            if v.requires_grad:
                raise ValueError(f"{spec.name} must be detached")
            if v.device != self.loss.device:
                raise ValueError(f"{spec.name} must be on the loss device")
        for name in ("loss", "video_loss", "audio_loss", "grad_norm"):
            if getattr(self, name).dtype is not torch.float32:
                raise TypeError(f"{name} must be float32")
        for name in ("valid_video_tokens", "valid_audio_tokens"):
            if getattr(self, name).dtype is not torch.int64:
                raise TypeError(f"{name} must be int64")
        for name in ("nonfinite", "skipped"):
            if getattr(self, name).dtype is not torch.bool:
                raise TypeError(f"{name} must be bool")

    def to_mapping(self) -> dict[str, float]:
        """All fields as Python floats, with exactly one device-to-host copy."""
        names = [f.name for f in fields(self)]
        packed = torch.stack([getattr(self, n).detach().to(torch.float64) for n in names]).cpu()
        return {n: float(v) for n, v in zip(names, packed.tolist())}

    @classmethod
    def zeros(cls, device: torch.device | str = "cpu") -> StepMetrics:
        dev = torch.device(device)

        def z(dtype: torch.dtype) -> torch.Tensor:
            return torch.zeros((), dtype=dtype, device=dev)

        return cls(loss=z(torch.float32), video_loss=z(torch.float32), audio_loss=z(torch.float32),
                   valid_video_tokens=z(torch.int64), valid_audio_tokens=z(torch.int64), grad_norm=z(torch.float32),
                   nonfinite=z(torch.bool), skipped=z(torch.bool))


_pytree.register_dataclass(StepMetrics, serialized_type_name="avgen_b200.StepMetrics")
