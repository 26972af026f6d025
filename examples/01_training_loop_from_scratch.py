"""Train a small video DiT for a few steps on a CPU, from procedural data.

The same objects run the 8 x B200 job: a model from the registry, the
flow-matching objective, an optimizer, a :class:`TrainState` and
``train_step``. On a GPU the DiT blocks run the fused sm_100a kernels; here they
run the fp32 PyTorch path.

    python examples/01_training_loop_from_scratch.py
"""
from __future__ import annotations

import torch

from avgen_b200 import FlowMatchingObjective, ParallelDims, RNGStreams, SyntheticSource, TrainState, build_model
from avgen_b200 import build_optimizer, parallelize, train_step
from avgen_b200.data.synthetic import SyntheticConfig
from avgen_b200.train import FlowMatchingConfig, MultiTaskConditioning, build_timestep_sampler


def main() -> None:
    torch.manual_seed(0)
    model = build_model("video_dit", {"width": 64, "depth": 2, "num_heads": 4, "in_channels": 4, "text_width": 32,
                                      "text_context_length": 8, "ffn_hidden": 128, "time_frequency_dim": 32})
    model.init_weights()
    # one process, one device: the plan is the identity, but the call is the one a mesh run makes
    parallel = parallelize(model, ParallelDims(world_size=1))
    source = SyntheticSource(SyntheticConfig(video_channels=4, frames=4, height=16, width=16, text_tokens=8,
                                             text_width=32, audio_frames=0), batch_size=2)
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("logit_normal"),
                                      MultiTaskConditioning())
    state = TrainState(model=parallel.model, optimizer=build_optimizer(parallel.model, lr=1e-3, weight_decay=0.01),
                       rng=RNGStreams.from_seed(0))
    batches = iter(source)
    for _ in range(8):
        state, metrics = train_step(state, next(batches), objective, patchifier=model.patchifier, max_grad_norm=1.0)
        values = metrics.to_mapping()
        print(f"step {state.step:2d}  loss {values['loss']:.4f}  grad_norm {values.get('grad_norm', float('nan')):.3f}")
    print(f"trained {state.step} steps on {state.samples_seen} samples")


if __name__ == "__main__":
    main()
