"""avgen_b200: a Blackwell-native (sm_100a) video / audio-video diffusion-transformer framework.

Same capabilities, public API and checkpoint format as avgen; every hot op is a
hand-written sm_100a kernel (``avgen_b200._C``) and the communication-bound
ones run over NVLink 5 peer memory. Contracts and the distributed runtime import
eagerly; everything else loads lazily on first attribute access (reference
façade: avgen/__init__.py:62-192).
"""
from __future__ import annotations

import importlib
from typing import Any

from avgen_b200.core import (ConditionMode, GridPatchifier, MediaBatch, MediaBatchSpec, ModelInput, ModelOutput,
                             PatchLayout, Patchifier, RNGStreams, StepMetrics, TextContext, TokenStream, TrainState)

__version__ = "0.1.0"

_LAZY: dict[str, str] = {
    "build_model": "avgen_b200.models",
    "register_model": "avgen_b200.models",
    "list_models": "avgen_b200.models",
    "VideoDiT": "avgen_b200.models",
    "VideoDiTConfig": "avgen_b200.models",
    "AVDiT": "avgen_b200.models",
    "AVDiTConfig": "avgen_b200.models",
    "ParallelDims": "avgen_b200.parallel",
    "init_distributed": "avgen_b200.parallel",
    "shutdown_distributed": "avgen_b200.parallel",
    "DistributedEnv": "avgen_b200.parallel",
    "parallelize": "avgen_b200.parallel",
    "ParallelConfig": "avgen_b200.parallel",
    "ParallelModel": "avgen_b200.parallel",
    "ActivationCheckpointConfig": "avgen_b200.parallel",
    "FSDPConfig": "avgen_b200.parallel",
    "PrecisionConfig": "avgen_b200.parallel",
    "PipelineConfig": "avgen_b200.parallel",
    "load_config": "avgen_b200.config",
    "RunConfig": "avgen_b200.config",
    "FlowMatchingObjective": "avgen_b200.train",
    "Trainer": "avgen_b200.train",
    "train_step": "avgen_b200.train",
    "build_optimizer": "avgen_b200.train",
    "GenerationPipeline": "avgen_b200.infer",
    "build_sampler": "avgen_b200.infer",
    "CheckpointManager": "avgen_b200.checkpoint",
    "simulate_config": "avgen_b200.simulate",
    "SimulationReport": "avgen_b200.simulate",
    "ModelShape": "avgen_b200.simulate",
    "search_parallel_plan": "avgen_b200.simulate",
    "apply_lora": "avgen_b200.finetune",
    "GRPOTrainer": "avgen_b200.rl",
    "SyntheticSource": "avgen_b200.data",
    "build_loader": "avgen_b200.data",
    "run_eval_suite": "avgen_b200.eval",
    "EvalReport": "avgen_b200.eval",
}

__all__ = ["ConditionMode", "GridPatchifier", "MediaBatch", "MediaBatchSpec", "ModelInput", "ModelOutput",
           "PatchLayout", "Patchifier", "RNGStreams", "StepMetrics", "TextContext", "TokenStream", "TrainState", "__version__",
           *sorted(_LAZY)]


def __getattr__(name: str) -> Any:
    module = _LAZY.get(name)
    if module is None:
        raise AttributeError(f"module 'avgen_b200' has no attribute {name!r}")
    value = getattr(importlib.import_module(module), name)
    globals()[name] = value
    return value


def __dir__() -> list[str]:
    return sorted(set(globals()) | set(_LAZY))
