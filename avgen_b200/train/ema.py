"""Exponential moving average of the (local shard of the) parameters.

Same contract as avgen/train/ema.py:52-294: bf16 shadow storage, decay ramp
``min(decay, (1 + s) / (10 + s))``, optional warmup and update interval, state
keys ``shadow.<fqn>``, ``num_updates``, ``decay``. When the parameters live in
:class:`~avgen_b200.train.optimizer.FusedAdamW` flat buffers, the shadow is one
flat buffer per group and an update is one sm_100a kernel launch per group.
"""
from __future__ import annotations

from collections.abc import Iterator, Mapping
from contextlib import contextmanager
from typing import Any

import torch
from torch import nn

__all__ = ["ShardedEMA"]

_PREFIX = "shadow."


def _local(t: torch.Tensor) -> torch.Tensor:
    from torch.distributed.tensor import DTensor

    return t.to_local() if isinstance(t, DTensor) else t


class ShardedEMA:
    def __init__(self, model: nn.Module, *, decay: float = 0.9999, storage_dtype: torch.dtype = torch.bfloat16,
                 warmup_steps: int = 0, update_every: int = 1, optimizer: Any = None) -> None:
        if not 0.0 < decay < 1.0:
            raise ValueError(f"decay must be in (0, 1); got {decay!r}")
        if isinstance(warmup_steps, bool) or warmup_steps < 0:
            raise ValueError("warmup_steps must be non-negative")
        if isinstance(update_every, bool) or update_every < 1:
            raise ValueError("update_every must be >= 1")
        self._decay = decay
        self._dtype = storage_dtype
        self._warmup = warmup_steps
        self._every = update_every
        self._num_updates = 0
        self._flat: list[tuple[torch.Tensor, torch.Tensor]] = []  # (flat param, flat shadow)
        self._shadow: dict[str, torch.Tensor] = {}
        flat_owner = {}
        if optimizer is not None and hasattr(optimizer, "flat_buffers"):
            for group, flat in zip(optimizer.param_groups, optimizer.flat_buffers()):
                shadow = flat["param"].detach().to(storage_dtype).clone()
                self._flat.append((flat["param"], shadow))
                for p, off in zip(group["params"], flat["offsets"].tolist()):
                    flat_owner[id(p)] = shadow[off:off + p.numel()].view(p.shape)
        for name, p in model.named_parameters():
            if not p.is_floating_point():
                continue
            view = flat_owner.get(id(p))
            self._shadow[name] = view if view is not None else _local(p.detach()).clone().to(storage_dtype)
        self._only_flat = bool(self._flat) and len(flat_owner) == len(self._shadow)

    @property
    def num_updates(self) -> int:
        return self._num_updates

    @property
    def decay(self) -> float:
        return self._decay

    def effective_decay(self, step: int) -> float:
        if step < self._warmup:
            return 0.0
        return min(self._decay, (1.0 + step) / (10.0 + step)) ** self._every

    @torch.no_grad()
    def update(self, model: nn.Module) -> None:
        step = self._num_updates
        self._num_updates += 1
        if step % self._every:
            return
        decay = self.effective_decay(step)
        if self._only_flat:
            for param, shadow in self._flat:
                if param.device.type == "cuda":
                    from avgen_b200.ops import kernels as K

                    K.ema_(param, shadow, decay)
                else:
                    shadow.lerp_(param.to(shadow.dtype), 1.0 - decay)
            return
        for name, p in model.named_parameters():
            if not p.is_floating_point():
                continue
            shadow = self._shadow.get(name)
            if shadow is None:
                raise KeyError(f"parameter {name!r} is not tracked by this EMA")
            _local(shadow).lerp_(_local(p.detach()).to(shadow.dtype), 1.0 - decay)

    @torch.no_grad()
    def copy_to(self, model: nn.Module) -> None:
        for name, p in model.named_parameters():
            if not p.is_floating_point():
                continue
            shadow = self._shadow.get(name)
            if shadow is None:
                raise KeyError(f"parameter {name!r} is not tracked by this EMA")
            _local(p).copy_(_local(shadow).to(p.dtype))
        from avgen_b200.models.linear import bump_weight_epoch

        bump_weight_epoch()

    @contextmanager
    def apply_to(self, model: nn.Module) -> Iterator[nn.Module]:
        backup = {n: _local(p).detach().clone() for n, p in model.named_parameters() if p.is_floating_point()}
        self.copy_to(model)
        try:
            yield model
        finally:
            with torch.no_grad():
                for n, p in model.named_parameters():
                    if n in backup:
                        _local(p).copy_(backup[n])
            from avgen_b200.models.linear import bump_weight_epoch

            bump_weight_epoch()

    def state_dict(self) -> dict[str, Any]:
        state: dict[str, Any] = {f"{_PREFIX}{n}": t for n, t in self._shadow.items()}
        state["num_updates"] = self._num_updates
        state["decay"] = self._decay
        return state

    @torch.no_grad()
    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        for n, t in self._shadow.items():
            key = f"{_PREFIX}{n}"
            if key not in state:
                raise KeyError(f"EMA state is missing {key!r}")
            _local(t).copy_(_local(state[key]).to(t.dtype))
        self._num_updates = int(state.get("num_updates", self._num_updates))
