"""Register an architecture of your own and train it with the framework's step.

A model takes a config dataclass as its first constructor argument (so a YAML
mapping builds it), maps a :class:`ModelInput` to a :class:`ModelOutput`, and
keeps its repeated blocks in ``.blocks`` (so activation checkpointing, FSDP2
wrapping and pipeline splitting find them).

    python examples/03_register_a_custom_model.py
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from avgen_b200 import FlowMatchingObjective, ModelInput, ModelOutput, RNGStreams, TrainState, build_model
from avgen_b200 import build_optimizer, list_models, register_model, train_step
from avgen_b200.core.patchify import GridPatchifier
from avgen_b200.data.synthetic_batch import random_batch
from avgen_b200.train import FlowMatchingConfig, MultiTaskConditioning, build_timestep_sampler


@dataclass(frozen=True)
class TokenMLPConfig:
    width: int = 64
    depth: int = 2
    in_channels: int = 4
    text_width: int = 32


class TokenMLPBlock(nn.Module):
    def __init__(self, width: int) -> None:
        super().__init__()
        self.norm = nn.LayerNorm(width)
        self.mlp = nn.Sequential(nn.Linear(width, 4 * width), nn.GELU(), nn.Linear(4 * width, width))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x + self.mlp(self.norm(x))


@register_model("token_mlp")
class TokenMLP(nn.Module):
    """Per-token MLP denoiser conditioned on the noise level and the mean text embedding."""

    def __init__(self, config: TokenMLPConfig) -> None:
        super().__init__()
        self.config = config
        self.patchifier = GridPatchifier(patch_frames=1, patch_height=2, patch_width=2)
        token_width = config.in_channels * 4
        self.embed = nn.Linear(token_width + 1, config.width)
        self.text = nn.Linear(config.text_width, config.width)
        self.blocks = nn.ModuleList(TokenMLPBlock(config.width) for _ in range(config.depth))
        self.head = nn.Linear(config.width, token_width)

    def forward(self, inputs: ModelInput) -> ModelOutput:
        video = inputs.video
        level = video.noise_level.float().reshape(video.tokens.shape[0], -1, 1).expand(*video.tokens.shape[:2], 1)
        x = self.embed(torch.cat((video.tokens.float(), level), dim=-1))
        x = x + self.text(inputs.text.features.float().mean(1, keepdim=True))
        for block in self.blocks:
            x = block(x)
        audio = inputs.audio.tokens.new_zeros(inputs.audio.tokens.shape)  # this model has no audio tower
        return ModelOutput(video=self.head(x).to(video.tokens.dtype), audio=audio)


def main() -> None:
    torch.manual_seed(0)
    assert "token_mlp" in list_models()
    model = build_model("token_mlp", {"width": 64, "depth": 2})  # the mapping a YAML `model:` section gives
    batch = random_batch(batch=2, channels=4, frames=2, height=8, width=8, text_tokens=4, text_width=32,
                         generator=torch.Generator().manual_seed(0))
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"),
                                      MultiTaskConditioning())
    state = TrainState(model=model, optimizer=build_optimizer(model, lr=3e-3), rng=RNGStreams.from_seed(0))
    for _ in range(5):
        state, metrics = train_step(state, batch, objective, patchifier=model.patchifier, max_grad_norm=1.0)
        print(f"step {state.step}  loss {metrics.to_mapping()['loss']:.4f}")


if __name__ == "__main__":
    main()
