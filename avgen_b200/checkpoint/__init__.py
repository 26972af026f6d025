"""Checkpointing: DCP manager (async, markers, retention, resharding), stateful keys, export / convert."""
from avgen_b200.checkpoint.export import (DEFAULT_MAX_SHARD_BYTES, INDEX_FILENAME, WEIGHTS_FILENAME, convert,
                                          export_huggingface, export_safetensors, import_safetensors)
from avgen_b200.checkpoint.manager import (CHECKPOINT_DIR_PREFIX, CHECKPOINT_FORMAT_VERSION, MARKER_FILENAME,
                                           CheckpointEntry, CheckpointManager, load, load_ema, load_model, save)
from avgen_b200.checkpoint.stateful import (EMA_KEY, EXTRAS_KEY, MODEL_OPTIMIZER_KEY, PROGRESS_KEY, RNG_KEY,
                                            SCHEDULE_KEY, build_stateful)

__all__ = ["CHECKPOINT_DIR_PREFIX", "CHECKPOINT_FORMAT_VERSION", "DEFAULT_MAX_SHARD_BYTES", "EMA_KEY", "EXTRAS_KEY",
           "INDEX_FILENAME", "MARKER_FILENAME", "MODEL_OPTIMIZER_KEY", "PROGRESS_KEY", "RNG_KEY", "SCHEDULE_KEY",
           "WEIGHTS_FILENAME", "CheckpointEntry", "CheckpointManager", "build_stateful", "convert",
           "export_huggingface", "export_safetensors", "import_safetensors", "load", "load_ema", "load_model", "save"]

from avgen_b200.checkpoint.stateful import ExtrasState, ModelOptimizerState, ProgressState, RNGState  # noqa: E402

__all__ += ["ExtrasState", "ModelOptimizerState", "ProgressState", "RNGState"]
