"""Model ABI: ``forward(ModelInput) -> ModelOutput`` (avgen/core/model_input.py:33-234).

Outputs stay in token space (``(B, L, patch_dim)`` per stream);
:meth:`ModelInput.unconditional` nulls only the text (the CFG branch).
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

import torch
from torch.utils import _pytree

from avgen_b200.core._validate import require_dtype, require_shape
from avgen_b200.core.batch import ConditionMode
from avgen_b200.core.tokens import TextContext, TokenStream

__all__ = ["ModelInput", "ModelOutput"]


def _empty_i64() -> torch.Tensor:
    return torch.empty(0, dtype=torch.int64)


@dataclass(frozen=True, slots=True)
class ModelInput:
    video: TokenStream
    audio: TokenStream
    text: TextContext
    condition_mode: torch.Tensor = field(default_factory=_empty_i64)

    def __post_init__(self) -> None:
        if self.condition_mode.numel() == 0:
            object.__setattr__(self, "condition_mode", torch.full((self.video.batch_size,), int(ConditionMode.JOINT),
                                                                  dtype=torch.int64, device=self.video.device))

    @property
    def batch_size(self) -> int:
        return self.video.batch_size

    @property
    def device(self) -> torch.device:
        return self.video.device

    @property
    def has_audio(self) -> bool:
        return self.audio.length > 0

    @property
    def has_text(self) -> bool:
        return not self.text.is_empty

    @property
    def total_tokens(self) -> int:
        return self.video.length + self.audio.length

    def replace_streams(self, *, video: TokenStream | None = None, audio: TokenStream | None = None) -> ModelInput:
        return replace(self, video=self.video if video is None else video, audio=self.audio if audio is None else audio)

    def unconditional(self) -> ModelInput:
        return replace(self, text=self.text.nullified())

    def validate(self) -> None:
        self.video.validate()
        self.audio.validate()
        self.text.validate()
        b = self.video.batch_size
        if self.audio.batch_size != b or self.text.features.shape[0] != b:
            raise ValueError("audio and text batch dimensions must match video")
        require_shape("condition_mode", self.condition_mode, (b,))
        require_dtype("condition_mode", self.condition_mode, torch.int64)
        valid = torch.zeros_like(self.condition_mode, dtype=torch.bool)
        for mode in ConditionMode:
            valid |= self.condition_mode == int(mode)
        if not bool(valid.all()):
            raise ValueError("condition_mode contains unsupported values")


@dataclass(frozen=True, slots=True)
class ModelOutput:
    video: torch.Tensor
    audio: torch.Tensor
    auxiliary: tuple[torch.Tensor, ...] = ()

    def validate(self, inputs: ModelInput) -> None:
        ev = (inputs.video.batch_size, inputs.video.length, inputs.video.layout.patch_dim)
        if tuple(self.video.shape) != ev:
            raise ValueError(f"video output shape must be {ev}; got {tuple(self.video.shape)}")
        if inputs.has_audio:
            ea = (inputs.audio.batch_size, inputs.audio.length, inputs.audio.layout.patch_dim)
            if tuple(self.audio.shape) != ea:
                raise ValueError(f"audio output shape must be {ea}; got {tuple(self.audio.shape)}")
        for t in (self.video, self.audio, *self.auxiliary):
            if not t.is_floating_point():
                raise TypeError("model outputs must be floating point")


_pytree.register_dataclass(ModelInput, serialized_type_name="avgen_b200.ModelInput")
_pytree.register_dataclass(ModelOutput, serialized_type_name="avgen_b200.ModelOutput")
