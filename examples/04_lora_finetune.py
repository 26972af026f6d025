"""Attach LoRA adapters to a DiT, train only them, then merge them into the base.

``apply_lora`` replaces the targeted projections with adapter layers whose B
factor starts at zero, so the adapted model starts out equal to the base; only
the adapters train. ``merge_lora`` folds ``W + (alpha / rank) B A`` back into
plain linears for inference. Under tensor parallelism or FSDP2 the factors are
sharded like their base weight; on a GPU the fused DiT block runs the adapted
weight inside its kernels.

    python examples/04_lora_finetune.py
"""
from __future__ import annotations

import torch

from avgen_b200 import FlowMatchingObjective, RNGStreams, TrainState, apply_lora, build_model, build_optimizer
from avgen_b200 import ModelInput, TextContext, TokenStream, train_step
from avgen_b200.data.synthetic_batch import random_batch
from avgen_b200.finetune.lora import LoRAConfig, mark_only_lora_trainable, merge_lora
from avgen_b200.train import FlowMatchingConfig, MultiTaskConditioning, build_timestep_sampler


def main() -> None:
    torch.manual_seed(0)
    model = build_model("video_dit", {"width": 64, "depth": 2, "num_heads": 4, "in_channels": 4, "text_width": 32,
                                      "text_context_length": 8, "ffn_hidden": 128, "time_frequency_dim": 32})
    model.init_weights()
    torch.nn.init.normal_(model.final_proj.weight, std=0.02)  # a non-zero head, as a pretrained model has
    batch = random_batch(batch=2, channels=4, frames=4, height=16, width=16, text_tokens=8, text_width=32,
                         generator=torch.Generator().manual_seed(1))
    base = {k: v.detach().clone() for k, v in model.state_dict().items()}

    model = apply_lora(model, LoRAConfig(rank=8, alpha=8.0))
    mark_only_lora_trainable(model)  # the base stays frozen
    trainable = sum(p.numel() for p in model.parameters() if p.requires_grad)
    total = sum(p.numel() for p in model.parameters())
    print(f"trainable {trainable:,} of {total:,} parameters ({100.0 * trainable / total:.1f}%)")

    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("logit_normal"),
                                      MultiTaskConditioning())
    params = [p for p in model.parameters() if p.requires_grad]
    state = TrainState(model=model, optimizer=torch.optim.AdamW(params, lr=1e-2), rng=RNGStreams.from_seed(0))
    for _ in range(4):
        state, metrics = train_step(state, batch, objective, patchifier=model.patchifier, max_grad_norm=1.0)
        print(f"step {state.step}  loss {metrics.to_mapping()['loss']:.4f}")

    frozen_same = all(torch.equal(base[k], v) for k, v in model.state_dict().items() if k in base)
    print(f"base weights untouched while training: {frozen_same}")
    model.eval()
    probe = random_batch(batch=1, channels=4, frames=4, height=16, width=16, text_tokens=8, text_width=32,
                         generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        stream = model.patchifier.to_tokens(probe.video, positions=probe.video_positions, mask=probe.video_mask,
                                            noise_level=torch.full((1,), 0.5))
        inputs = ModelInput(video=stream, audio=TokenStream.empty_like(1, stream.width),
                            text=TextContext(features=probe.text, mask=probe.text_mask))
        adapted = model(inputs).video
        merged = merge_lora(model, strip=True)  # plain nn.Linear layers holding W + (alpha / rank) B A
        plain = merged(inputs).video
    left = sum(1 for _, m in merged.named_modules() if "LoRA" in type(m).__name__)
    print(f"adapter layers left after merging: {left}; max output change {float((adapted - plain).abs().max()):.2e}")


if __name__ == "__main__":
    main()
