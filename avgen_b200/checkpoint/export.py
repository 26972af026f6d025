"""Release export / import and format conversion (avgen/checkpoint/export.py:73-503).

The exported layout is a format shared with avgen: ``model.safetensors`` or
``model-0000i-of-0000n.safetensors`` shards of at most 5 GiB plus
``model.safetensors.index.json`` (``metadata.total_size`` and a ``weight_map``).
Tensors are cloned before writing (parameters here are views of flat optimizer
buffers and share storage). ``convert`` turns a DCP checkpoint's
``model_optimizer/model`` sub-tree into that layout or back.
"""
from __future__ import annotations

import json
import logging
import os
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch import nn
from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict, set_model_state_dict

__all__ = ["DEFAULT_MAX_SHARD_BYTES", "INDEX_FILENAME", "WEIGHTS_FILENAME", "convert", "export_huggingface",
           "export_safetensors", "import_safetensors", "read_safetensors_dir"]

_LOG = logging.getLogger("avgen_b200.checkpoint")
WEIGHTS_FILENAME = "model.safetensors"
INDEX_FILENAME = "model.safetensors.index.json"
DEFAULT_MAX_SHARD_BYTES = 5 * 1024 ** 3


def _main() -> bool:
    return not (dist.is_available() and dist.is_initialized()) or dist.get_rank() == 0


def _shard_name(i: int, n: int) -> str:
    return WEIGHTS_FILENAME if n == 1 else f"model-{i + 1:05d}-of-{n:05d}.safetensors"


def _materialise(tensors: Mapping[str, torch.Tensor], dtype: torch.dtype | None) -> dict[str, torch.Tensor]:
    out = {}
    for name, t in tensors.items():
        v = t.detach().to("cpu")
        if dtype is not None and v.is_floating_point():
            v = v.to(dtype)
        out[name] = v.clone().contiguous()
    return out


def _write(directory: Path, tensors: dict[str, torch.Tensor], header: dict[str, str], max_shard_bytes: int) -> int:
    from safetensors.torch import save_file

    groups: list[list[str]] = [[]]
    size = 0
    for name, t in tensors.items():
        n = t.numel() * t.element_size()
        if groups[-1] and size + n > max_shard_bytes:
            groups.append([])
            size = 0
        groups[-1].append(name)
        size += n
    directory.mkdir(parents=True, exist_ok=True)
    weight_map: dict[str, str] = {}
    total = 0
    for i, names in enumerate(groups):
        fname = _shard_name(i, len(groups))
        save_file({n: tensors[n] for n in names}, str(directory / fname), metadata=header)
        for n in names:
            weight_map[n] = fname
            total += tensors[n].numel() * tensors[n].element_size()
    index = {"metadata": {"total_size": total, **header}, "weight_map": weight_map}
    (directory / INDEX_FILENAME).write_text(json.dumps(index, indent=2, sort_keys=True))
    return total


def export_safetensors(path: str | os.PathLike[str], model: nn.Module, *, dtype: torch.dtype | None = None,
                       metadata: Mapping[str, str] | None = None,
                       max_shard_bytes: int = DEFAULT_MAX_SHARD_BYTES) -> Path:
    """Consolidate the full model state (gathered across ranks) into safetensors shards."""
    if max_shard_bytes <= 0:
        raise ValueError("max_shard_bytes must be positive")
    directory = Path(path)
    state = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True, cpu_offload=True))
    if not _main():
        return directory
    header = {"format": "pt"}
    for k, v in (metadata or {}).items():
        if not isinstance(k, str) or not isinstance(v, str):
            raise TypeError("safetensors metadata must map str -> str")
        header[k] = v
    tensors = _materialise({k: v for k, v in state.items() if isinstance(v, torch.Tensor)}, dtype)
    total = _write(directory, tensors, header, max_shard_bytes)
    _LOG.info("exported %d tensors (%.2f GiB) -> %s", len(tensors), total / 1024 ** 3, directory)
    return directory


def read_safetensors_dir(path: Path) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    if path.is_file():
        return load_file(str(path))
    index = path / INDEX_FILENAME
    files = (sorted(set(json.loads(index.read_text())["weight_map"].values())) if index.is_file()
             else sorted(c.name for c in path.glob("*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no safetensors shards under {path}")
    out: dict[str, torch.Tensor] = {}
    for f in files:
        out.update(load_file(str(path / f)))
    return out


def import_safetensors(path: str | os.PathLike[str], model: nn.Module, *, strict: bool = True) -> nn.Module:
    tensors = read_safetensors_dir(Path(path))
    if strict:  # DCP's full-state load reports unexpected keys but fills missing ones from the model itself
        missing = sorted(set(model.state_dict()) - set(tensors))
        if missing:
            raise RuntimeError(f"{path} lacks {len(missing)} tensor(s) of the model, e.g. {missing[:3]}; pass "
                               "strict=False to load the shared subset")
    set_model_state_dict(model, model_state_dict=tensors,
                         options=StateDictOptions(full_state_dict=True, strict=strict))
    from avgen_b200.models.linear import bump_weight_epoch

    bump_weight_epoch()
    return model


def export_huggingface(path: str | os.PathLike[str], model: nn.Module, *, dtype: torch.dtype | None = None,
                       thread_count: int = 1, save_distributed: bool = False) -> Path:
    """Hugging Face safetensors layout through DCP's HF storage writer."""
    directory = Path(path)
    opts = StateDictOptions(full_state_dict=not save_distributed, cpu_offload=not save_distributed)
    state = get_model_state_dict(model, options=opts)
    state = {k: (v.detach().clone().to(dtype) if dtype is not None and v.is_floating_point() else v.detach().clone())
             for k, v in state.items() if isinstance(v, torch.Tensor)}
    if not save_distributed and not _main():
        return directory
    directory.mkdir(parents=True, exist_ok=True)
    writer = dcp.HuggingFaceStorageWriter(path=str(directory), thread_count=thread_count,
                                          save_distributed=save_distributed, enable_consolidation=save_distributed)
    dcp.save(state, storage_writer=writer, no_dist=not save_distributed)
    return directory


def _read_dcp_flat(source: Path) -> dict[str, Any]:
    from torch.distributed.checkpoint.format_utils import _EmptyStateDictLoadPlanner, _load_state_dict

    state: dict[str, Any] = {}
    _load_state_dict(state, storage_reader=dcp.FileSystemReader(source), planner=_EmptyStateDictLoadPlanner(),
                     no_dist=True)
    return state


def convert(src: str | os.PathLike[str], dst: str | os.PathLike[str], *, to: str = "safetensors",
            dtype: torch.dtype | None = None, max_shard_bytes: int = DEFAULT_MAX_SHARD_BYTES) -> Path:
    """DCP checkpoint <-> consolidated safetensors."""
    from avgen_b200.checkpoint.stateful import MODEL_OPTIMIZER_KEY

    source, dest = Path(src), Path(dst)
    if to == "safetensors":
        node: Any = _read_dcp_flat(source)
        for key in (MODEL_OPTIMIZER_KEY, "model"):
            if not isinstance(node, Mapping) or key not in node:
                raise KeyError(f"checkpoint has no {MODEL_OPTIMIZER_KEY}/model sub-tree")
            node = node[key]
        tensors = _materialise({k: v for k, v in node.items() if isinstance(v, torch.Tensor)}, dtype)
        _write(dest, tensors, {"format": "pt"}, max_shard_bytes)
    elif to == "dcp":
        tensors = _materialise(read_safetensors_dir(source), dtype)
        dest.mkdir(parents=True, exist_ok=True)
        dcp.save({MODEL_OPTIMIZER_KEY: {"model": tensors}}, storage_writer=dcp.FileSystemWriter(dest, overwrite=True),
                 no_dist=True)
    else:
        raise ValueError(f"to must be 'safetensors' or 'dcp'; got {to!r}")
    return dest
