"""DCP stateful adapters: the checkpoint's top-level keys.

The key set is the checkpoint format shared with avgen
(avgen/checkpoint/stateful.py:58-363): ``model_optimizer`` -> ``{model,
optimizer}`` (DCP ``get_state_dict`` with a flattened optimizer dict, so it
reshards to any rank count), ``rng`` -> ``{data_rank_<i>: ...}``, ``progress``
(step / samples / tokens / epoch), ``schedule``, ``ema`` (``shadow.<fqn>``,
``num_updates``, ``decay``) and ``extras`` (any further stateful components).
"""
from __future__ import annotations

from collections.abc import Mapping
from typing import Any

from torch import nn
from torch.distributed.checkpoint.state_dict import StateDictOptions, get_state_dict, set_state_dict

from avgen_b200.core.rng import RNGStreams
from avgen_b200.core.state import Stateful, TrainState

__all__ = ["EMA_KEY", "EXTRAS_KEY", "MODEL_OPTIMIZER_KEY", "PROGRESS_KEY", "RNG_KEY", "SCHEDULE_KEY", "ExtrasState",
           "ModelOptimizerState", "ProgressState", "RNGState", "StatefulAdapter", "build_stateful"]

MODEL_OPTIMIZER_KEY = "model_optimizer"
RNG_KEY = "rng"
PROGRESS_KEY = "progress"
EXTRAS_KEY = "extras"
SCHEDULE_KEY = "schedule"
EMA_KEY = "ema"


class ModelOptimizerState:
    def __init__(self, model: nn.Module, optimizer: Any, *, strict: bool = True, cpu_offload: bool = False,
                 flatten_optimizer_state_dict: bool = True) -> None:
        self.model = model
        self.optimizer = optimizer
        self._opts = StateDictOptions(strict=strict, cpu_offload=cpu_offload,
                                      flatten_optimizer_state_dict=flatten_optimizer_state_dict)

    def state_dict(self) -> dict[str, Any]:
        m, o = get_state_dict(self.model, self.optimizer, options=self._opts)
        return {"model": m, "optimizer": o}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        for name in ("model", "optimizer"):
            if name not in state:
                raise KeyError(f"checkpoint entry {name!r} missing from {MODEL_OPTIMIZER_KEY!r}")
        set_state_dict(self.model, self.optimizer, model_state_dict=state["model"],
                       optim_state_dict=state["optimizer"], options=self._opts)
        from avgen_b200.models.linear import bump_weight_epoch

        bump_weight_epoch()


class RNGState:
    def __init__(self, rng: RNGStreams, *, data_rank: int = 0) -> None:
        if data_rank < 0:
            raise ValueError("data_rank must be non-negative")
        self.rng = rng
        self.data_rank = data_rank

    @property
    def key(self) -> str:
        return f"data_rank_{self.data_rank}"

    def state_dict(self) -> dict[str, Any]:
        return {self.key: dict(self.rng.state_dict())}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        payload = state.get(self.key)
        if payload is not None:
            self.rng.load_state_dict(payload)


class ProgressState:
    def __init__(self, state: TrainState) -> None:
        self.state = state

    def state_dict(self) -> dict[str, Any]:
        return dict(self.state.progress())

    def load_state_dict(self, values: Mapping[str, Any]) -> None:
        self.state.load_progress({k: int(v) for k, v in values.items()})


class StatefulAdapter:
    """Wraps any object with state_dict / load_state_dict."""

    def __init__(self, target: Stateful) -> None:
        self.target = target

    def state_dict(self) -> dict[str, Any]:
        return dict(self.target.state_dict())

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        self.target.load_state_dict(state)


class ExtrasState:
    def __init__(self, extras: Mapping[str, Stateful]) -> None:
        self.extras = dict(extras)

    def state_dict(self) -> dict[str, Any]:
        return {k: dict(v.state_dict()) for k, v in self.extras.items()}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        for k, v in self.extras.items():
            if k in state:
                v.load_state_dict(state[k])


def build_stateful(state: TrainState, *, data_rank: int = 0, include_rng: bool = True, strict: bool = True,
                   cpu_offload: bool = False) -> dict[str, Any]:
    entries: dict[str, Any] = {
        MODEL_OPTIMIZER_KEY: ModelOptimizerState(state.model, state.optimizer, strict=strict, cpu_offload=cpu_offload),
        PROGRESS_KEY: ProgressState(state),
    }
    if include_rng:
        entries[RNG_KEY] = RNGState(state.rng, data_rank=data_rank)
    if state.schedule is not None:
        entries[SCHEDULE_KEY] = StatefulAdapter(state.schedule)
    if state.ema is not None:
        entries[EMA_KEY] = StatefulAdapter(state.ema)
    if state.extras:
        entries[EXTRAS_KEY] = ExtrasState(state.extras)
    return entries
