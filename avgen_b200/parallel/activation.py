"""Activation checkpointing policies (avgen/parallel/activation.py:25-160 API).

On the B200 path every eligible DiT block is one fused autograd node
(:mod:`avgen_b200.models.fused`) that saves only its input, the self-attention
output and its log-sum-exp, and recomputes the rest inside its own backward.
That is the ``fused`` policy and it needs no wrapper. The reference's eager
policies remain for blocks that run eagerly (CPU, non-eligible shapes):

* ``full`` — recompute the whole block in backward;
* ``selective_layer`` — ``full`` on every ``layer_interval``-th block;
* ``selective_op`` — keep the outputs of matmuls, attention and collectives
  (every ``save_op_frequency``-th call of each), recompute everything else.

Wrapping a block with a policy other than ``fused``/``none`` also switches its
fused path off, so the policy the user asked for is the one that runs.
"""
from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import Any, Literal

import torch
from torch import nn


def _is_block_list(blocks: object) -> bool:
    from avgen_b200.parallel.pipeline import is_block_list

    return is_block_list(blocks)


__all__ = ["ACMode", "ActivationCheckpointConfig", "CheckpointedBlock", "apply_activation_checkpointing",
           "DEFAULT_SAVE_OPS"]

ACMode = Literal["none", "fused", "full", "selective_op", "selective_layer"]
_MODES = ("none", "fused", "full", "selective_op", "selective_layer")

_aten = torch.ops.aten


def _save_ops() -> tuple[Any, ...]:
    ops: list[Any] = [_aten.mm.default, _aten.addmm.default, _aten.bmm.default,
                      _aten._scaled_dot_product_efficient_attention.default,
                      _aten._scaled_dot_product_flash_attention.default]
    for name in ("_scaled_dot_product_cudnn_attention", "_scaled_mm"):
        op = getattr(_aten, name, None)
        if op is not None:
            ops.append(op.default)
    c10d = getattr(torch.ops, "_c10d_functional", None)
    if c10d is not None:
        ops += [c10d.reduce_scatter_tensor.default, c10d.all_gather_into_tensor.default]
    return tuple(ops)


DEFAULT_SAVE_OPS: tuple[Any, ...] = _save_ops()


@dataclass(frozen=True, slots=True)
class ActivationCheckpointConfig:
    mode: ACMode = "fused"
    layer_interval: int = 2
    save_op_frequency: int = 1
    early_stop: bool = True

    def __post_init__(self) -> None:
        for name in ("layer_interval", "save_op_frequency"):
            v = getattr(self, name)
            if isinstance(v, bool) or v < 1:
                raise ValueError(f"{name} must be >= 1; got {v!r}")
        if self.mode not in _MODES:
            raise ValueError(f"unsupported activation checkpoint mode {self.mode!r}; choose from {', '.join(_MODES)}")

    @property
    def enabled(self) -> bool:
        return self.mode not in ("none", "fused")


def _selective_context(config: ActivationCheckpointConfig) -> Callable[[], Any]:
    from torch.utils.checkpoint import CheckpointPolicy, create_selective_checkpoint_contexts

    save = set(DEFAULT_SAVE_OPS)
    every = config.save_op_frequency

    def policy_fn() -> Callable[..., Any]:
        seen: dict[Any, int] = {}

        def policy(_ctx: Any, op: Any, *_a: Any, **_k: Any) -> Any:
            if op not in save:
                return CheckpointPolicy.PREFER_RECOMPUTE
            n = seen.get(op, 0)
            seen[op] = n + 1
            return CheckpointPolicy.MUST_SAVE if n % every == 0 else CheckpointPolicy.PREFER_RECOMPUTE

        return policy

    return lambda: create_selective_checkpoint_contexts(policy_fn())


class CheckpointedBlock(nn.Module):
    """Runs ``block`` under ``torch.utils.checkpoint`` (non-reentrant).

    Parameter names stay those of the wrapped block (``block.`` prefix removed in
    ``state_dict``), so checkpoints do not depend on the policy.
    """

    def __init__(self, block: nn.Module, config: ActivationCheckpointConfig) -> None:
        super().__init__()
        self.block = block
        self.config = config
        if hasattr(block, "use_fused"):
            block.use_fused = False
        self._context_fn = _selective_context(config) if config.mode == "selective_op" else None
        self._register_state_dict_hook(_strip_prefix)
        self.register_load_state_dict_pre_hook(_add_prefix)

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        from torch.utils.checkpoint import checkpoint

        extra: dict[str, Any] = {"use_reentrant": False, "preserve_rng_state": False,
                                 "early_stop": self.config.early_stop}
        if self._context_fn is not None:
            extra["context_fn"] = self._context_fn
        return checkpoint(self.block, *args, **extra, **kwargs)

    def __getattr__(self, name: str) -> Any:
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self._modules["block"], name)


def _strip_prefix(module: nn.Module, state: dict[str, Any], prefix: str, _meta: Any) -> None:
    for key in [k for k in state if k.startswith(prefix + "block.")]:
        state[prefix + key[len(prefix) + 6:]] = state.pop(key)


def _add_prefix(_module: nn.Module, state: dict[str, Any], prefix: str, *_args: Any) -> None:
    for key in [k for k in state if k.startswith(prefix) and not k.startswith(prefix + "block.")]:
        state[prefix + "block." + key[len(prefix):]] = state.pop(key)


def apply_activation_checkpointing(model: nn.Module, config: ActivationCheckpointConfig, *,
                                   block_attribute: str = "blocks") -> nn.Module:
    """Wrap the blocks of ``model.<block_attribute>`` according to ``config``."""
    if not config.enabled:
        return model
    blocks = getattr(model, block_attribute, None)
    if blocks is None:
        raise AttributeError(f"model {type(model).__name__} has no {block_attribute!r}; pass block_attribute=")
    if not _is_block_list(blocks):
        raise TypeError(f"{block_attribute!r} must be an nn.ModuleList; got {type(blocks).__name__}")
    for i, block in enumerate(blocks):
        if isinstance(block, CheckpointedBlock):
            continue
        if config.mode == "selective_layer" and i % config.layer_interval:
            continue
        blocks[i] = CheckpointedBlock(block, config)
    return model
