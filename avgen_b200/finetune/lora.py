"""LoRA and DoRA adapters (avgen/finetune/lora.py:136-700 API; adapter file keys kept).

:class:`LoRALinear` subclasses ``nn.Linear``, so the base weight keeps its
state-dict key and the adapter adds ``lora_a`` ``(r, in)``, ``lora_b`` ``(out, r)``
and, for DoRA, ``lora_magnitude`` ``(out,)``:

    W' = W + (alpha / r) B A                       (LoRA)
    W' = m * (W + (alpha / r) B A) / ||row||       (DoRA, row norms detached)

On the B200 path the model's linear layer runs the sm_100a GEMM on the
*effective* weight ``W'``; autograd carries the weight gradient from the GEMM's
fp32 weight-gradient epilogue into ``A`` and ``B`` (two rank-r products), so
adapters need no separate low-rank kernels. Tensor-parallel base weights give
the adapter matching placements: column-parallel (``Shard(0)``) -> ``A``
replicated, ``B`` ``Shard(0)``; row-parallel (``Shard(1)``) -> ``A`` ``Shard(1)``,
``B`` replicated. FSDP-sharded bases are refused: apply adapters before FSDP.
"""
from __future__ import annotations

import json
import math
from collections.abc import Iterator, Mapping, Sequence
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from avgen_b200.finetune._match import matches_any, normalize_patterns

__all__ = ["DEFAULT_TARGET_MODULES", "LoRAConfig", "LoRALinear", "adapter_state_dict", "apply_lora", "load_adapter",
           "lora_modules", "lora_parameters", "mark_only_lora_trainable", "merge_lora", "save_adapter",
           "unmerge_lora"]

DEFAULT_TARGET_MODULES = ("q_proj", "k_proj", "v_proj", "out_proj", "gate_proj", "up_proj", "down_proj")
_TINY = 1e-12


@dataclass(frozen=True, slots=True)
class LoRAConfig:
    rank: int = 16
    alpha: float = 32.0
    dropout: float = 0.0
    target_modules: tuple[str, ...] = DEFAULT_TARGET_MODULES
    exclude_modules: tuple[str, ...] = ()
    use_dora: bool = False
    init_lora_weights: str = "kaiming"
    rank_pattern: tuple[tuple[str, int], ...] = ()
    alpha_pattern: tuple[tuple[str, float], ...] = ()

    def __post_init__(self) -> None:
        if isinstance(self.rank, bool) or self.rank < 1:
            raise ValueError(f"rank must be >= 1; got {self.rank!r}")
        if not (math.isfinite(self.alpha) and self.alpha > 0):
            raise ValueError(f"alpha must be positive; got {self.alpha!r}")
        if not 0.0 <= self.dropout < 1.0:
            raise ValueError(f"dropout must be in [0, 1); got {self.dropout!r}")
        if self.init_lora_weights not in ("kaiming", "gaussian", "zeros"):
            raise ValueError(f"init_lora_weights must be kaiming, gaussian or zeros; got {self.init_lora_weights!r}")
        if not normalize_patterns(self.target_modules):
            raise ValueError("target_modules is empty")
        for pat, r in self.rank_pattern:
            if isinstance(r, bool) or int(r) < 1:
                raise ValueError(f"rank_pattern {pat!r} needs a rank >= 1")

    def rank_for(self, name: str) -> int:
        for pat, r in self.rank_pattern:
            if matches_any(name, (pat,)):
                return int(r)
        return self.rank

    def alpha_for(self, name: str) -> float:
        for pat, a in self.alpha_pattern:
            if matches_any(name, (pat,)):
                return float(a)
        return self.alpha

    def selects(self, name: str) -> bool:
        return matches_any(name, self.target_modules) and not matches_any(name, self.exclude_modules)

    def to_metadata(self) -> dict[str, str]:
        return {"lora_config": json.dumps(asdict(self), sort_keys=True)}


def _placements(t: torch.Tensor) -> tuple[Any, ...] | None:
    from torch.distributed.tensor import DTensor

    return tuple(t.placements) if isinstance(t, DTensor) else None


def _adapter_layout(weight: torch.Tensor) -> tuple[tuple[Any, ...], tuple[Any, ...]] | None:
    """Placements of (A, B) for a DTensor base weight; None for a plain tensor."""
    from torch.distributed.tensor import Replicate, Shard

    pl = _placements(weight)
    if pl is None:
        return None
    sharded = [p.dim for p in pl if isinstance(p, Shard)]
    if len(sharded) != 1 or len(pl) != 1:
        raise ValueError("LoRA supports a base weight sharded on one mesh dimension (tensor parallel); FSDP-"
                         "sharded weights must receive adapters before fully_shard")
    if sharded[0] == 0:
        return (Replicate(),), (Shard(0),)
    return (Shard(1),), (Replicate(),)


def _new_like(ref: torch.Tensor, shape: tuple[int, ...], placements: tuple[Any, ...] | None) -> torch.Tensor:
    from torch.distributed.tensor import DTensor, distribute_tensor

    if placements is None or not isinstance(ref, DTensor):
        return torch.zeros(shape, device=ref.device, dtype=torch.float32 if ref.dtype.is_floating_point else ref.dtype)
    full = torch.zeros(shape, device=ref.to_local().device, dtype=ref.dtype)
    return distribute_tensor(full, ref.device_mesh, list(placements))


def _local(t: torch.Tensor) -> torch.Tensor:
    from torch.distributed.tensor import DTensor

    return t.to_local() if isinstance(t, DTensor) else t


def _row_sq(w: torch.Tensor) -> torch.Tensor:
    """Per-output-row sum of squares (a DTensor reduction when sharded)."""
    return (w.float() * w.float()).sum(dim=1)


class LoRALinear(nn.Linear):
    def __init__(self, in_features: int, out_features: int, *, rank: int, alpha: float, dropout: float = 0.0,
                 use_dora: bool = False, bias: bool = True, device: torch.device | str | None = None,
                 dtype: torch.dtype | None = None) -> None:
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=dtype)
        self.rank = int(rank)
        self.alpha = float(alpha)
        self.scaling = self.alpha / self.rank
        self.use_dora = bool(use_dora)
        self.merged = False
        self._merged_norm: torch.Tensor | None = None
        self.lora_dropout: nn.Module = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.lora_a = nn.Parameter(torch.zeros(self.rank, in_features, device=device, dtype=dtype))
        self.lora_b = nn.Parameter(torch.zeros(out_features, self.rank, device=device, dtype=dtype))
        self.lora_magnitude: nn.Parameter | None = (
            nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) if use_dora else None)

    @classmethod
    def from_linear(cls, linear: nn.Linear, *, rank: int, alpha: float, dropout: float = 0.0, use_dora: bool = False,
                    init: str = "kaiming") -> LoRALinear:
        m = cls(linear.in_features, linear.out_features, rank=rank, alpha=alpha, dropout=dropout, use_dora=use_dora,
                bias=linear.bias is not None, device="meta")
        m.weight = linear.weight
        if linear.bias is not None:
            m.bias = linear.bias
        layout = _adapter_layout(linear.weight)
        a_pl, b_pl = (None, None) if layout is None else layout
        m.lora_a = nn.Parameter(_new_like(linear.weight, (rank, linear.in_features), a_pl))
        m.lora_b = nn.Parameter(_new_like(linear.weight, (linear.out_features, rank), b_pl))
        m.reset_lora_parameters(init)
        if use_dora:
            m.lora_magnitude = nn.Parameter(_new_like(linear.weight, (linear.out_features,), b_pl))
            m.reset_dora_magnitude()
        for name in ("_forward_hooks", "_forward_pre_hooks"):  # keep tensor-parallel hooks of the base layer
            getattr(m, name).update(getattr(linear, name))
        shard = getattr(linear, "_avgen_tp_shard", None)
        if shard is not None:
            _take_head_shard(m, linear, shard)
        return m

    def reset_lora_parameters(self, init: str = "kaiming") -> None:
        a = _local(self.lora_a)
        with torch.no_grad():
            if init == "kaiming":
                bound = 1.0 / math.sqrt(self.in_features)
                a.uniform_(-bound, bound)
            elif init == "gaussian":
                a.normal_(0.0, 1.0 / self.rank)
            elif init == "zeros":
                a.zero_()
            else:
                raise ValueError(f"unknown init {init!r}")
            _local(self.lora_b).zero_()

    def reset_dora_magnitude(self) -> None:
        if self.lora_magnitude is None:
            raise RuntimeError("this adapter has no DoRA magnitude")
        with torch.no_grad():
            self.lora_magnitude.copy_(_row_sq(self.weight).sqrt().to(self.lora_magnitude.dtype))

    def lora_delta(self) -> torch.Tensor:
        return (self.lora_b @ self.lora_a) * self.scaling

    def _dora_scale(self, combined: torch.Tensor) -> torch.Tensor:
        assert self.lora_magnitude is not None
        norm = _row_sq(combined).clamp_min(_TINY).sqrt().detach()
        scale = self.lora_magnitude / norm.to(self.lora_magnitude.dtype)
        return torch.where(self.lora_magnitude.detach() > 0, scale, torch.ones_like(scale))

    def adapted_weight(self) -> torch.Tensor:
        """The effective weight (differentiable in the adapter parameters)."""
        if self.merged:
            return self.weight
        w = self.weight + self.lora_delta().to(self.weight.dtype)
        if self.lora_magnitude is None:
            return w
        return w * self._dora_scale(w).unsqueeze(-1).to(w.dtype)

    def forward(self, input: torch.Tensor) -> torch.Tensor:  # noqa: A002 - nn.Linear signature
        if self.merged or self.lora_magnitude is not None or isinstance(self.lora_dropout, nn.Identity):
            return F.linear(input, self.adapted_weight(), self.bias)
        base = F.linear(input, self.weight, self.bias)
        return base + F.linear(F.linear(self.lora_dropout(input), self.lora_a), self.lora_b) * self.scaling

    def merge(self) -> None:
        if self.merged:
            raise RuntimeError("adapter already merged")
        with torch.no_grad():
            if self.lora_magnitude is not None:
                self._merged_norm = _row_sq(self.weight + self.lora_delta()).clamp_min(_TINY).sqrt().clone()
            self.weight.copy_(self.adapted_weight())
        self.merged = True

    def unmerge(self) -> None:
        if not self.merged:
            raise RuntimeError("adapter is not merged")
        self.merged = False
        with torch.no_grad():
            if self.lora_magnitude is None:
                self.weight.sub_(self.lora_delta().to(self.weight.dtype))
                return
            if self._merged_norm is None:
                raise RuntimeError("a DoRA merge is only reversible in the process that merged it (row norms)")
            mag = self.lora_magnitude.detach()
            factor = torch.where(mag > 0, self._merged_norm / mag.clamp_min(_TINY), torch.ones_like(mag))
            self.weight.copy_(self.weight * factor.unsqueeze(-1).to(self.weight.dtype) - self.lora_delta())
            self._merged_norm = None

    def extra_repr(self) -> str:
        kind = "dora" if self.lora_magnitude is not None else "lora"
        return f"{super().extra_repr()}, {kind}_rank={self.rank}, alpha={self.alpha}, merged={self.merged}"


def _take_head_shard(m: LoRALinear, linear: nn.Linear, shard: tuple[int, list[int], int]) -> None:
    """Adapters on a head-parallel shard (a plain-tensor slice of the full weight, made
    by :mod:`avgen_b200.parallel.heads`), mirroring the DTensor layout above: the factor
    on the sharded side (B and the DoRA magnitude of a column-parallel layer, A of a
    row-parallel one) is this rank's slice and is gathered into the full tensor in
    checkpoints like the base weight; the other factor is replicated, and its gradient,
    each rank's partial sum of the full one, is summed over the tensor-parallel group."""
    from avgen_b200.parallel.heads import gather_slices, local_slice, tp_shard_group

    dim, sizes, full = shard
    if dim == 1 and m.lora_magnitude is not None:
        raise NotImplementedError("DoRA on a row-parallel head shard needs its row norms summed over the group; "
                                  "use LoRA there or DoRA without head-parallel tensor parallelism")
    group = tp_shard_group(linear.weight)
    rank = dist.get_rank(group)
    m._avgen_tp_shard = shard
    sharded = {"lora_b": 0, "lora_magnitude": 0} if dim == 0 else {"lora_a": 1}
    replicated = m.lora_a if dim == 0 else m.lora_b
    for name in sharded:
        t = getattr(m, name, None)
        if isinstance(t, torch.Tensor):
            t._avgen_tp_group = group  # type: ignore[attr-defined]

    def summed(grad: torch.Tensor, _group: Any = group) -> torch.Tensor:
        grad = grad.clone()
        dist.all_reduce(grad, group=_group)
        return grad

    replicated.register_hook(summed)
    for name in ("_state_dict_hooks", "_load_state_dict_pre_hooks"):  # the base weight's full-tensor hooks
        getattr(m, name).update(getattr(linear, name))

    def save_full(module: nn.Module, state: dict, prefix: str, _meta: Any) -> None:
        for name, d in sharded.items():
            t = state.get(prefix + name)
            if t is not None:
                state[prefix + name] = gather_slices(t, d, sizes, group)

    def load_local(state: dict, prefix: str, *_args: Any) -> None:
        for name, d in sharded.items():
            t = state.get(prefix + name)
            if t is not None and t.dim() > d and t.shape[d] == full:
                state[prefix + name] = local_slice(t, d, sizes, rank)

    m._register_state_dict_hook(save_full)
    m._register_load_state_dict_pre_hook(load_local)


def _set_child(root: nn.Module, name: str, module: nn.Module) -> None:
    parent_name, _, child = name.rpartition(".")
    parent = root.get_submodule(parent_name) if parent_name else root
    setattr(parent, child, module)


def apply_lora(model: nn.Module, config: LoRAConfig) -> nn.Module:
    """Replace every selected ``nn.Linear`` by a :class:`LoRALinear` sharing its base weight."""
    targets = [(n, m) for n, m in model.named_modules()
               if isinstance(m, nn.Linear) and not isinstance(m, LoRALinear) and config.selects(n)]
    if not targets:
        raise ValueError(f"no linear layer matches target_modules={config.target_modules}")
    for name, lin in targets:
        _set_child(model, name, LoRALinear.from_linear(lin, rank=config.rank_for(name), alpha=config.alpha_for(name),
                                                       dropout=config.dropout, use_dora=config.use_dora,
                                                       init=config.init_lora_weights))
    return model


def lora_modules(model: nn.Module) -> Iterator[tuple[str, LoRALinear]]:
    for n, m in model.named_modules():
        if isinstance(m, LoRALinear):
            yield n, m


def lora_parameters(model: nn.Module) -> list[nn.Parameter]:
    out: list[nn.Parameter] = []
    for _, m in lora_modules(model):
        out += [m.lora_a, m.lora_b] + ([m.lora_magnitude] if m.lora_magnitude is not None else [])
    return out


def mark_only_lora_trainable(model: nn.Module, *, train_biases: bool = False,
                             extra_trainable: Sequence[str] = ()) -> int:
    """Freeze everything but adapter parameters (and optional biases / extra patterns)."""
    keep = {id(p) for p in lora_parameters(model)}
    extra = normalize_patterns(extra_trainable)
    count = 0
    for name, p in model.named_parameters():
        train = id(p) in keep or (train_biases and name.endswith(".bias")) or (extra and matches_any(name, extra))
        p.requires_grad_(bool(train))
        count += int(bool(train)) * p.numel()
    return count


def merge_lora(model: nn.Module, *, strip: bool = False) -> nn.Module:
    """Fold adapters into the base weights; ``strip`` swaps the modules back to plain linears."""
    for name, m in list(lora_modules(model)):
        m.merge()
        if strip:
            plain = nn.Linear(m.in_features, m.out_features, bias=m.bias is not None, device="meta")
            plain.weight = m.weight
            if m.bias is not None:
                plain.bias = m.bias
            _set_child(model, name, plain)
    return model


def unmerge_lora(model: nn.Module) -> nn.Module:
    for _, m in lora_modules(model):
        m.unmerge()
    return model


def _full(t: torch.Tensor) -> torch.Tensor:
    from torch.distributed.tensor import DTensor

    return (t.full_tensor() if isinstance(t, DTensor) else t).detach().cpu().contiguous()


def adapter_state_dict(model: nn.Module) -> dict[str, torch.Tensor]:
    out: dict[str, torch.Tensor] = {}
    for name, m in lora_modules(model):
        out[f"{name}.lora_a"] = _full(m.lora_a)
        out[f"{name}.lora_b"] = _full(m.lora_b)
        if m.lora_magnitude is not None:
            out[f"{name}.lora_magnitude"] = _full(m.lora_magnitude)
    return out


def save_adapter(path: str | Path, model: nn.Module, *, config: LoRAConfig | None = None,
                 extra_metadata: Mapping[str, str] | None = None) -> Path:
    """Adapter weights as one safetensors file (rank 0 writes)."""
    import torch.distributed as dist
    from safetensors.torch import save_file

    dest = Path(path)
    state = adapter_state_dict(model)
    if not state:
        raise ValueError("the model has no LoRA modules")
    if dist.is_initialized() and dist.get_rank() != 0:
        return dest
    meta = {"format": "avgen_b200.lora"}
    if config is not None:
        meta.update(config.to_metadata())
    meta.update(extra_metadata or {})
    dest.parent.mkdir(parents=True, exist_ok=True)
    save_file(state, str(dest), metadata=meta)
    return dest


def load_adapter(path: str | Path, model: nn.Module, *, strict: bool = True) -> dict[str, Any]:
    """Load adapter weights into an already adapted model; returns the file metadata."""
    from safetensors import safe_open
    from torch.distributed.tensor import DTensor, distribute_tensor

    modules = dict(lora_modules(model))
    seen: set[str] = set()
    with safe_open(str(path), framework="pt") as f:
        meta = dict(f.metadata() or {})
        for key in f.keys():  # noqa: SIM118 - safe_open has no items()
            mod_name, _, attr = key.rpartition(".")
            m = modules.get(mod_name)
            if m is None or getattr(m, attr, None) is None:
                if strict:
                    raise KeyError(f"adapter tensor {key!r} has no target in the model")
                continue
            target = getattr(m, attr)
            value = f.get_tensor(key)
            with torch.no_grad():
                if isinstance(target, DTensor):
                    value = distribute_tensor(value.to(target.dtype), target.device_mesh, list(target.placements))
                    target.to_local().copy_(value.to_local())
                else:
                    target.copy_(value.to(target.dtype))
            seen.add(key)
    if strict:
        missing = set(adapter_state_dict(model)) - seen
        if missing:
            raise KeyError(f"adapter file lacks {sorted(missing)[:5]}")
    if "lora_config" in meta:
        meta["lora_config"] = json.loads(meta["lora_config"])
    return meta
