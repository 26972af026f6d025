"""FSDP2 / HSDP sharding (avgen/parallel/fsdp.py:42-206 API).

``apply_fsdp`` shards every transformer block, then the root, with PyTorch's
``fully_shard`` over the given (possibly 2-D HSDP) mesh. The last block keeps
its gathered parameters after forward by default, since backward starts with
it. ``set_prefetch_depth`` overlaps the next blocks' all-gathers with compute.

On CUDA ranks of one NVSwitch node with a 1-D mesh, the parameter all-gather
and the gradient reduce-scatter run over NVLink peer memory
(:mod:`avgen_b200.parallel.peer_comm`: copy-engine pulls and a pull-reduce
kernel) instead of NCCL; ``FSDPConfig(peer_collectives=False)`` keeps NCCL.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from torch import nn

from avgen_b200.parallel.precision import PrecisionConfig


def _is_block_list(blocks: object) -> bool:
    from avgen_b200.parallel.pipeline import is_block_list

    return is_block_list(blocks)


__all__ = ["FSDPConfig", "apply_fsdp", "set_prefetch_depth", "summarize_sharding"]


@dataclass(frozen=True, slots=True)
class FSDPConfig:
    reshard_after_forward: bool = True
    cpu_offload: bool = False
    block_attribute: str = "blocks"
    shard_last_block_after_forward: bool = False
    ignore_frozen_params: bool = False
    forward_prefetch: int = 1
    backward_prefetch: int = 1
    peer_collectives: bool = True


def apply_fsdp(model: nn.Module, mesh: Any, *, precision: PrecisionConfig | None = None,
               config: FSDPConfig | None = None) -> nn.Module:
    from torch.distributed.fsdp import CPUOffloadPolicy, OffloadPolicy, fully_shard

    cfg = config or FSDPConfig()
    prec = precision or PrecisionConfig()
    blocks = getattr(model, cfg.block_attribute, None)
    if not _is_block_list(blocks):
        raise AttributeError(f"{type(model).__name__} has no nn.ModuleList {cfg.block_attribute!r}; FSDP shards "
                             "per block so communication overlaps compute")
    kwargs: dict[str, Any] = {"mesh": mesh, "mp_policy": prec.fsdp_policy(),
                              "offload_policy": CPUOffloadPolicy(pin_memory=True) if cfg.cpu_offload
                              else OffloadPolicy()}
    if cfg.ignore_frozen_params:
        frozen = {p for p in model.parameters() if not p.requires_grad}
        if frozen:
            kwargs["ignored_params"] = frozen
    last = len(blocks) - 1
    for i, block in enumerate(blocks):
        keep = i == last and not cfg.shard_last_block_after_forward
        fully_shard(block, reshard_after_forward=cfg.reshard_after_forward and not keep, **kwargs)
    fully_shard(model, reshard_after_forward=cfg.reshard_after_forward, **kwargs)
    if cfg.forward_prefetch > 1 or cfg.backward_prefetch > 1:
        set_prefetch_depth(model, forward=cfg.forward_prefetch, backward=cfg.backward_prefetch)
    if cfg.peer_collectives and getattr(mesh, "device_type", "cpu") == "cuda":
        from avgen_b200.parallel.peer_comm import install_peer_collectives

        install_peer_collectives(model, mesh)
    return model


def set_prefetch_depth(model: nn.Module, *, forward: int = 1, backward: int = 1) -> None:
    """Prefetch the next ``forward`` blocks' all-gathers in forward (and ``backward`` in backward)."""
    if forward < 1 or backward < 1:
        raise ValueError(f"prefetch depth must be >= 1; got forward={forward}, backward={backward}")
    sharded = [m for m in model.modules() if hasattr(m, "set_modules_to_forward_prefetch")]
    for i, m in enumerate(sharded):
        ahead = sharded[i + 1:i + 1 + forward]
        behind = sharded[max(0, i - backward):i][::-1]
        if ahead:
            m.set_modules_to_forward_prefetch(ahead)
        if behind and hasattr(m, "set_modules_to_backward_prefetch"):
            m.set_modules_to_backward_prefetch(behind)


def summarize_sharding(model: nn.Module) -> dict[str, int]:
    """Local element count and how many parameters are sharded DTensors."""
    from torch.distributed.tensor import DTensor

    local = sharded = replicated = 0
    for p in model.parameters():
        if isinstance(p, DTensor):
            local += p.to_local().numel()
            sharded += 1
        else:
            local += p.numel()
            replicated += 1
    return {"local_elements": local, "sharded_params": sharded, "replicated_params": replicated}
