"""Fine-tuning: LoRA / DoRA (tensor-parallel aware), control and image-prompt adapters,
freezing helpers, staged recipes and the config entry point (avgen/finetune)."""
from avgen_b200.finetune.adapters import (AdapterHandles, ControlAdapter, ControlAdapterConfig, IPAdapter,
                                          IPAdapterConfig)
from avgen_b200.finetune.entry import build_adapter_hook, finetune_from_config, run_finetune
from avgen_b200.finetune.freeze import TrainableSummary, freeze_all, freeze_except, freeze_matching, trainable_summary
from avgen_b200.finetune.lora import (DEFAULT_TARGET_MODULES, LoRAConfig, LoRALinear, adapter_state_dict, apply_lora,
                                      load_adapter, lora_modules, lora_parameters, mark_only_lora_trainable,
                                      merge_lora, save_adapter, unmerge_lora)
from avgen_b200.finetune.stages import (DistillationConfig, FinetuneStage, TimestepPlan, apply_stage, get_stage,
                                        list_stages, register_stage, stage_names_for, standard_stages)

__all__ = ["DEFAULT_TARGET_MODULES", "AdapterHandles", "ControlAdapter", "ControlAdapterConfig", "DistillationConfig",
           "FinetuneStage", "IPAdapter", "IPAdapterConfig", "LoRAConfig", "LoRALinear", "TimestepPlan",
           "TrainableSummary", "adapter_state_dict", "apply_lora", "apply_stage", "build_adapter_hook",
           "finetune_from_config", "freeze_all", "freeze_except", "freeze_matching", "get_stage", "list_stages",
           "load_adapter", "lora_modules", "lora_parameters", "mark_only_lora_trainable", "merge_lora",
           "register_stage", "run_finetune", "save_adapter", "stage_names_for", "standard_stages",
           "trainable_summary", "unmerge_lora"]

from avgen_b200.finetune.stages import resolution_shift, shift_timesteps  # noqa: E402

__all__ += ["resolution_shift", "shift_timesteps"]
