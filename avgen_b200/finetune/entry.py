"""Fine-tuning from a :class:`~avgen_b200.config.RunConfig` (avgen/finetune/entry.py:39-223 API).

``finetune.mode``: ``lora`` (LoRA or DoRA on ``finetune.lora_targets``),
``full`` (everything but ``finetune.freeze_patterns``), or ``control`` (a
control branch; the base is frozen). The base weights come from
``finetune.base_checkpoint`` (a checkpoint directory or exported safetensors)
before any sharding; the adapter (or the full model) is saved at the end.
"""
from __future__ import annotations

import logging
from pathlib import Path
from typing import Any

from torch import nn

__all__ = ["build_adapter_hook", "finetune_from_config", "run_finetune"]

_LOG = logging.getLogger(__name__)


def build_adapter_hook(config: Any) -> Any:
    """The ``adapt`` callable ``parallelize`` runs after tensor parallelism and before FSDP."""
    from avgen_b200.finetune.freeze import freeze_all, freeze_matching
    from avgen_b200.finetune.lora import LoRAConfig, apply_lora, mark_only_lora_trainable

    ft = config.finetune

    def adapt(model: nn.Module) -> nn.Module:
        if ft.mode == "lora":
            lcfg = LoRAConfig(rank=ft.lora_rank, alpha=ft.lora_alpha, dropout=ft.lora_dropout,
                              target_modules=tuple(ft.lora_targets), use_dora=ft.use_dora)
            apply_lora(model, lcfg)
            extra = ("norm",) if ft.train_norms else ()
            mark_only_lora_trainable(model, extra_trainable=extra)
        elif ft.mode == "control":
            from avgen_b200.finetune.adapters import ControlAdapter, ControlAdapterConfig

            freeze_all(model)
            blocks = ft.control_blocks if ft.control_blocks > 0 else max(1, len(model.blocks) // 4)
            model.control_adapter = ControlAdapter(model, ControlAdapterConfig(control_width=ft.control_channels,
                                                                               num_blocks=blocks,
                                                                               conditioning_scale=ft.control_scale))
        if ft.freeze_patterns:
            freeze_matching(model, ft.freeze_patterns)
        return model

    return adapt


def _load_base(path: str, model: nn.Module) -> None:
    from avgen_b200.infer.pipeline import _load_weights

    _load_weights(Path(path), model)


def finetune_from_config(config: Any) -> Any:
    """Build, train and save; returns the run stack."""
    from avgen_b200.cli._wiring import build_run, run_training
    from avgen_b200.finetune.freeze import trainable_summary
    from avgen_b200.finetune.lora import save_adapter

    ft = config.finetune

    def load_base(model: nn.Module) -> nn.Module:
        if ft.base_checkpoint:
            _load_base(ft.base_checkpoint, model)
        return model

    stack = build_run(config, adapt=build_adapter_hook(config), model_hook=load_base)
    _LOG.info("trainable: %s", trainable_summary(stack.parallel.model).describe())
    run_training(stack)
    if ft.mode == "lora":
        save_adapter(stack.output_dir / "adapter.safetensors", stack.parallel.model,
                     extra_metadata={"base_checkpoint": ft.base_checkpoint})
    return stack


run_finetune = finetune_from_config
