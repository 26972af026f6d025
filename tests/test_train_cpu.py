"""End-to-end CPU training slice: model + objective + FusedAdamW/AdamW + train_step."""
from __future__ import annotations

import torch

from avgen_b200.core import RNGStreams, TrainState
from avgen_b200.data.synthetic_batch import random_batch
from avgen_b200.models import build_model
from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                              build_timestep_sampler, train_step)

TINY = {"width": 64, "depth": 2, "num_heads": 4, "ffn_hidden": 128, "in_channels": 4, "text_width": 32,
        "text_context_length": 8, "text_refiner_depth": 1, "cond_width": 64, "time_frequency_dim": 32}


def _state(fused: bool) -> tuple[TrainState, object]:
    torch.manual_seed(0)
    model = build_model("video_dit", TINY)
    model.init_weights()
    torch.nn.init.normal_(model.final_proj.weight, std=0.02)
    opt = build_optimizer(model, lr=1e-3, weight_decay=0.01, fused=fused)
    return TrainState(model=model, optimizer=opt, rng=RNGStreams.from_seed(0)), model


def test_loss_decreases_and_fused_matches_torch_adamw() -> None:
    batch = random_batch(batch=2, channels=4, frames=4, height=16, width=16, text_tokens=8, text_width=32,
                         generator=torch.Generator().manual_seed(0))
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("logit_normal"),
                                      MultiTaskConditioning())
    losses = {}
    for fused in (True, False):
        state, model = _state(fused)
        hist = []
        for _ in range(6):
            _, m = train_step(state, batch, objective, patchifier=model.patchifier, max_grad_norm=1.0)
            hist.append(m.to_mapping()["loss"])
        losses[fused] = hist
        assert state.step == 6
    assert all(torch.isfinite(torch.tensor(losses[True])))
    for a, b in zip(losses[True], losses[False]):
        assert abs(a - b) < 1e-4 * max(1.0, abs(b)), (losses[True], losses[False])
