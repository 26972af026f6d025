"""Frozen contracts: token streams, model ABI, dense batches, RNG, state, metrics."""
from avgen_b200.core.batch import ConditionMode, MediaBatch, MediaBatchSpec, null_text_conditioning, stack_batches
from avgen_b200.core.metrics import StepMetrics
from avgen_b200.core.model_input import ModelInput, ModelOutput
from avgen_b200.core.patchify import (GridPatchifier, Patchifier, build_spatial_coords, build_temporal_coords,
                                      patchify_grid, unpatchify_grid)
from avgen_b200.core.rng import RNGStreams, mix_seed
from avgen_b200.core.state import EMA, DataCursor, LRSchedule, Stateful, TrainState
from avgen_b200.core.tensors import TensorBundle, TensorBundleSpec, TensorDType
from avgen_b200.core.tokens import PatchLayout, TextContext, TokenStream

__all__ = [
    "EMA", "ConditionMode", "DataCursor", "GridPatchifier", "LRSchedule", "MediaBatch", "MediaBatchSpec",
    "ModelInput", "ModelOutput", "PatchLayout", "Patchifier", "RNGStreams", "Stateful", "StepMetrics",
    "TensorBundle", "TensorBundleSpec", "TensorDType", "TextContext", "TokenStream", "TrainState",
    "build_spatial_coords", "build_temporal_coords", "mix_seed", "null_text_conditioning", "patchify_grid",
    "stack_batches", "unpatchify_grid",
]
