"""Optimizers: AdamW on flat fp32 buffers (sm_100a kernel), plus the reference set.

``build_optimizer`` keeps the reference contract (avgen/train/optimizer.py:68-222):
decay / no-decay groups (ndim <= 1 or a name containing norm / bias /
scale_shift / embed), names ``adamw`` / ``adamw_8bit`` / ``adafactor``.

On CUDA, ``adamw`` is :class:`FusedAdamW`: each parameter group's parameters and
gradients are re-homed into one contiguous fp32 buffer (parameters become views,
so ``state_dict`` / DCP see ordinary per-parameter tensors), and a step is

1. an optional average of the flat gradients over the data-parallel group
   (one NCCL all-reduce per group),
2. one squared-norm kernel per group, the clip coefficient and the non-finite
   flag computed on the device (no host sync),
3. one fused AdamW kernel per group that also treats a non-finite step's
   gradients as zero (the reference's ``_neutralise_nonfinite`` semantics).
"""
from __future__ import annotations

import math
from collections.abc import Iterable, Sequence
from typing import Any

import torch
import torch.distributed as dist
from torch import nn
from torch.optim import Optimizer

__all__ = ["DEFAULT_NO_DECAY_PATTERNS", "FusedAdamW", "MultiTensorAdamW", "ShardedAdamW", "build_optimizer",
           "build_param_groups", "list_optimizers"]

DEFAULT_NO_DECAY_PATTERNS: tuple[str, ...] = ("norm", "bias", "scale_shift", "embed")
_OPTIMIZERS = ("adafactor", "adamw", "adamw_8bit")
_ALIGN = 4  # fp32 elements: keeps every view 16-byte aligned for the vector kernels


def list_optimizers() -> tuple[str, ...]:
    return _OPTIMIZERS


def build_param_groups(model: nn.Module, *, weight_decay: float,
                       no_decay_patterns: Sequence[str] = DEFAULT_NO_DECAY_PATTERNS) -> list[dict[str, Any]]:
    patterns = tuple(p.lower() for p in no_decay_patterns)
    decayed: list[nn.Parameter] = []
    undecayed: list[nn.Parameter] = []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if p.ndim <= 1 or any(pat in name.lower() for pat in patterns):
            undecayed.append(p)
        else:
            decayed.append(p)
    if not decayed and not undecayed:
        raise ValueError("model has no trainable parameters")
    groups = []
    if decayed:
        groups.append({"params": decayed, "weight_decay": weight_decay})
    if undecayed:
        groups.append({"params": undecayed, "weight_decay": 0.0})
    return groups


# Hyper-parameter keys torch's AdamW keeps in every parameter group. The optimizers
# here carry them too (with the behaviour they implement), so their state dicts and
# DCP checkpoints load into torch's AdamW (the reference's optimizer) and back.
_ADAMW_GROUP_KEYS = {"amsgrad": False, "maximize": False, "foreach": None, "capturable": False,
                     "differentiable": False, "fused": None, "decoupled_weight_decay": True}


class FusedAdamW(Optimizer):
    """AdamW over per-group flat fp32 buffers with the sm_100a fused kernel."""

    def __init__(self, params: Iterable[Any], lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.0, *, dp_group: Any = None) -> None:
        defaults = {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay, **_ADAMW_GROUP_KEYS}
        super().__init__(params, defaults)
        self.dp_group = dp_group
        self.max_grad_norm: float | None = None
        # groups holding other parts of the model (pipeline stages): the squared norm is summed over them
        self.norm_groups: tuple[Any, ...] = ()
        self._flat: list[dict[str, torch.Tensor]] = []
        self._step = 0
        self.last_grad_norm: torch.Tensor | None = None
        self.last_nonfinite: torch.Tensor | None = None
        for group in self.param_groups:
            self._flat.append(self._flatten(group))

    # ------------------------------------------------------------------ layout
    @staticmethod
    def _flatten(group: dict[str, Any]) -> dict[str, torch.Tensor]:
        params: list[torch.Tensor] = group["params"]
        if not params:
            raise ValueError("empty parameter group")
        dev = params[0].device
        offsets = []
        total = 0
        for p in params:
            if p.device != dev:
                raise ValueError("all parameters of a group must share a device")
            offsets.append(total)
            total += -(-p.numel() // _ALIGN) * _ALIGN
        flat_p = torch.zeros(total, device=dev, dtype=torch.float32)
        flat_g = torch.zeros(total, device=dev, dtype=torch.float32)
        with torch.no_grad():
            for p, off in zip(params, offsets):
                n = p.numel()
                flat_p[off:off + n].copy_(p.detach().reshape(-1).float())
                p.data = flat_p[off:off + n].view(p.shape)
                p.grad = flat_g[off:off + n].view(p.shape)
        return {"param": flat_p, "grad": flat_g, "exp_avg": torch.zeros_like(flat_p),
                "exp_avg_sq": torch.zeros_like(flat_p), "offsets": torch.tensor(offsets)}

    def flat_buffers(self) -> list[dict[str, torch.Tensor]]:
        """Per-group flat buffers (``param``, ``grad``, ``exp_avg``, ``exp_avg_sq``)."""
        return self._flat

    @property
    def state(self) -> dict:  # type: ignore[override]
        """Per-parameter views of the flat moments (torch AdamW state layout)."""
        out: dict = {}
        for group, flat in zip(self.param_groups, getattr(self, "_flat", [])):
            for p, off in zip(group["params"], flat["offsets"].tolist()):
                n = p.numel()
                out[p] = {"step": torch.tensor(float(self._step)),
                          "exp_avg": flat["exp_avg"][off:off + n].view(p.shape),
                          "exp_avg_sq": flat["exp_avg_sq"][off:off + n].view(p.shape)}
        return out

    @state.setter
    def state(self, value: dict) -> None:  # torch.optim.Optimizer.__init__ assigns a defaultdict
        if not getattr(self, "_flat", None):
            return
        for group, flat in zip(self.param_groups, self._flat):
            for p, off in zip(group["params"], flat["offsets"].tolist()):
                st = value.get(p)
                if not st:
                    continue
                n = p.numel()
                with torch.no_grad():
                    flat["exp_avg"][off:off + n].copy_(st["exp_avg"].reshape(-1))
                    flat["exp_avg_sq"][off:off + n].copy_(st["exp_avg_sq"].reshape(-1))
                self._step = int(float(st.get("step", self._step)))

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        """Load torch-AdamW-format state into the flat buffers."""
        groups = state_dict["param_groups"]
        if len(groups) != len(self.param_groups):
            raise ValueError("loaded state has a different number of parameter groups")
        index = {}
        for g_saved, g in zip(groups, self.param_groups):
            for pid, p in zip(g_saved["params"], g["params"]):
                index[pid] = p
            for key in ("lr", "betas", "eps", "weight_decay"):
                if key in g_saved:
                    g[key] = g_saved[key]
        mapped = {index[k]: v for k, v in state_dict["state"].items() if k in index}
        self.state = mapped

    # ------------------------------------------------------------------ step
    def zero_grad(self, set_to_none: bool = True) -> None:  # noqa: ARG002 - the flat views must persist
        for flat in self._flat:
            flat["grad"].zero_()
        for group, flat in zip(self.param_groups, self._flat):
            for p, off in zip(group["params"], flat["offsets"].tolist()):
                if p.grad is None or p.grad.data_ptr() != flat["grad"][off:].data_ptr():
                    p.grad = flat["grad"][off:off + p.numel()].view(p.shape)

    def grad_norm(self) -> torch.Tensor:
        """Global L2 norm of all gradients (device scalar, no host sync)."""
        from avgen_b200.ops import kernels as K

        acc = torch.zeros(1, device=self._flat[0]["grad"].device, dtype=torch.float32)
        for flat in self._flat:
            if flat["grad"].device.type == "cuda":
                K.sq_norm_(flat["grad"], acc)
            else:
                acc += flat["grad"].pow(2).sum()
        # head-parallel slices (each rank a different part): their squares sum over the group
        from avgen_b200.parallel.heads import tp_shard_group

        sliced: dict[Any, list[torch.Tensor]] = {}
        for group in self.param_groups:
            for p in group["params"]:
                if tp_shard_group(p) is not None and p.grad is not None:
                    sliced.setdefault(tp_shard_group(p), []).append(p.grad)
        for tp_group, grads in sliced.items():
            part = torch.zeros(1, device=acc.device, dtype=torch.float32)
            for g in grads:
                part += g.float().pow(2).sum()
            local = part.clone()
            dist.all_reduce(part, group=tp_group)
            acc += part - local
        for group in self.norm_groups:
            dist.all_reduce(acc, group=group)
        return acc.sqrt()[0]

    def sync_gradients(self) -> None:
        """Average flat gradients over the data-parallel group (if any)."""
        if self.dp_group is None or not dist.is_initialized() or dist.get_world_size(self.dp_group) == 1:
            return
        world = dist.get_world_size(self.dp_group)
        for flat in self._flat:
            g = flat["grad"]
            if g.device.type == "cuda":
                dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.dp_group)
            else:
                dist.all_reduce(g, group=self.dp_group)
                g.div_(world)

    @torch.no_grad()
    def step(self, closure: Any = None, *, max_grad_norm: float | None = None) -> Any:
        """One AdamW step; clips by ``max_grad_norm`` (argument or attribute) on the device."""
        loss = closure() if closure is not None else None
        from avgen_b200.models.linear import bump_weight_epoch

        self.sync_gradients()
        self._step += 1
        norm = self.grad_norm()
        nonfinite = ~torch.isfinite(norm)
        clip = max_grad_norm if max_grad_norm is not None else self.max_grad_norm
        if clip is not None:
            scale = torch.clamp(clip / (norm + 1e-6), max=1.0)
        else:
            scale = torch.ones_like(norm)
        scale = torch.where(nonfinite, torch.zeros_like(scale), scale).reshape(1)
        skip = nonfinite.to(torch.int32).reshape(1)
        self.last_grad_norm = norm
        self.last_nonfinite = nonfinite
        for group, flat in zip(self.param_groups, self._flat):
            beta1, beta2 = group["betas"]
            if flat["param"].device.type == "cuda":
                from avgen_b200.ops import kernels as K

                K.adamw_step(flat["param"], flat["grad"], flat["exp_avg"], flat["exp_avg_sq"], lr=group["lr"],
                             betas=(beta1, beta2), eps=group["eps"], weight_decay=group["weight_decay"],
                             step=self._step, grad_scale=scale, skip=skip)
            else:
                _adamw_reference(flat, lr=group["lr"], beta1=beta1, beta2=beta2, eps=group["eps"],
                                 weight_decay=group["weight_decay"], step=self._step, scale=scale, nonfinite=nonfinite)
        bump_weight_epoch()
        return loss


class ShardedAdamW(FusedAdamW):
    """AdamW with its moments sharded over a one-node data-parallel group, the
    gradient reduce-scatter and the parameter all-gather done over NVLink peer
    memory inside the optimizer kernels (ZeRO-style; the reference runs an NCCL
    gradient reduction and a replicated AdamW, avgen/train/optimizer.py:198-205).

    Every rank keeps the full fp32 parameters and gradients as flat buffers
    mapped into every peer (CUDA IPC) and owns the contiguous shard
    ``[rank * shard, (rank + 1) * shard)`` of each group's buffer. A step is:

    1. a one-word all-reduce: every rank's gradients are complete;
    2. ``shard_reduce``: this rank sums its shard of every peer's gradients over
       NVLink (averaged) and accumulates the squared norm of the result;
    3. an all-reduce of that scalar: the global gradient norm, and every pull done;
    4. ``shard_adamw_push``: AdamW on the shard (clip coefficient and non-finite
       skip on the device) storing each updated parameter into every rank's
       buffer;
    5. a one-word all-reduce: every push landed before the next forward.

    Adam moments take ``1 / world`` of the memory of the replicated optimizer.
    On CPU (gloo) the same steps run with collectives instead of peer memory.
    """

    def __init__(self, params: Iterable[Any], lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.0, *, group: Any = None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("ShardedAdamW needs an initialised process group")
        self.shard_group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.shard_group)
        self.rank = dist.get_rank(self.shard_group)
        self._full_state: list[tuple[torch.Tensor, torch.Tensor]] | None = None
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, dp_group=None)

    def _flatten(self, group: dict[str, Any]) -> dict[str, Any]:  # type: ignore[override]
        params: list[torch.Tensor] = group["params"]
        if not params:
            raise ValueError("empty parameter group")
        dev = params[0].device
        offsets, total = [], 0
        for p in params:
            if p.device != dev:
                raise ValueError("all parameters of a group must share a device")
            offsets.append(total)
            total += -(-p.numel() // _ALIGN) * _ALIGN
        unit = self.world * _ALIGN
        total = -(-total // unit) * unit
        shard = total // self.world
        out: dict[str, Any] = {"offsets": torch.tensor(offsets), "lo": self.rank * shard, "shard": shard}
        if dev.type == "cuda":
            from avgen_b200.parallel.symmetric import SymmetricBuffer

            out["pbuf"] = SymmetricBuffer(total * 4, self.shard_group, dev)
            out["gbuf"] = SymmetricBuffer(total * 4, self.shard_group, dev)
            flat_p = out["pbuf"].view(self.rank, 0, (total,), torch.float32)
            flat_g = out["gbuf"].view(self.rank, 0, (total,), torch.float32)
        else:
            flat_p = torch.zeros(total, dtype=torch.float32)
            flat_g = torch.zeros(total, dtype=torch.float32)
        with torch.no_grad():
            for p, off in zip(params, offsets):
                n = p.numel()
                flat_p[off:off + n].copy_(p.detach().reshape(-1).float())
                p.data = flat_p[off:off + n].view(p.shape)
                p.grad = flat_g[off:off + n].view(p.shape)
        out.update(param=flat_p, grad=flat_g, exp_avg=torch.zeros(shard, device=dev),
                   exp_avg_sq=torch.zeros(shard, device=dev), reduced=torch.zeros(shard, device=dev))
        return out

    # ------------------------------------------------------------------ state (gathered for checkpoints)
    def _gathered(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        full = []
        for flat in self._flat:
            ms = []
            for key in ("exp_avg", "exp_avg_sq"):
                t = torch.empty(flat["shard"] * self.world, device=flat[key].device)
                dist.all_gather_into_tensor(t, flat[key], group=self.shard_group)
                ms.append(t)
            full.append((ms[0], ms[1]))
        return full

    @property
    def state(self) -> dict:  # type: ignore[override]
        """Per-parameter views of the full moments, gathered over the group
        (collective: every rank of the group reads it, e.g. through state_dict)."""
        if not getattr(self, "_flat", None):
            return {}
        full = self._gathered()
        out: dict = {}
        for group, flat, (m, v) in zip(self.param_groups, self._flat, full):
            for p, off in zip(group["params"], flat["offsets"].tolist()):
                n = p.numel()
                out[p] = {"step": torch.tensor(float(self._step)), "exp_avg": m[off:off + n].view(p.shape),
                          "exp_avg_sq": v[off:off + n].view(p.shape)}
        return out

    @state.setter
    def state(self, value: dict) -> None:
        if not getattr(self, "_flat", None):
            return
        for group, flat in zip(self.param_groups, self._flat):
            lo, hi = flat["lo"], flat["lo"] + flat["shard"]
            for p, off in zip(group["params"], flat["offsets"].tolist()):
                st = value.get(p)
                if not st:
                    continue
                n = p.numel()
                a, b = max(off, lo), min(off + n, hi)
                if a < b:
                    with torch.no_grad():
                        flat["exp_avg"][a - lo:b - lo].copy_(st["exp_avg"].reshape(-1)[a - off:b - off])
                        flat["exp_avg_sq"][a - lo:b - lo].copy_(st["exp_avg_sq"].reshape(-1)[a - off:b - off])
                self._step = int(float(st.get("step", self._step)))

    def sync_gradients(self) -> None:  # the reduction is part of the step
        return

    def _barrier(self, dev: torch.device) -> None:
        token = torch.zeros(1, device=dev)
        dist.all_reduce(token, group=self.shard_group)

    @torch.no_grad()
    def step(self, closure: Any = None, *, max_grad_norm: float | None = None) -> Any:
        loss = closure() if closure is not None else None
        from avgen_b200.models.linear import bump_weight_epoch

        self._step += 1
        dev = self._flat[0]["param"].device
        cuda = dev.type == "cuda"
        acc = torch.zeros(1, device=dev, dtype=torch.float32)
        if cuda:
            from avgen_b200.ops import kernels as K
            from avgen_b200.ops._ext import load

            ext = load()
            self._barrier(dev)  # 1. every rank's gradients are complete
            for flat in self._flat:  # 2. pull-reduce this rank's shard over NVLink
                ext.shard_reduce(flat["gbuf"].ptrs, flat["lo"], flat["reduced"], acc)
                K._count()
        else:
            for flat in self._flat:
                full = flat["grad"].clone()
                dist.all_reduce(full, group=self.shard_group)
                flat["reduced"].copy_(full[flat["lo"]:flat["lo"] + flat["shard"]] / self.world)
                acc += flat["reduced"].pow(2).sum()
        dist.all_reduce(acc, group=self.shard_group)  # 3. global norm; every pull is done
        norm = acc.sqrt()[0]
        nonfinite = ~torch.isfinite(norm)
        clip = max_grad_norm if max_grad_norm is not None else self.max_grad_norm
        scale = torch.clamp(clip / (norm + 1e-6), max=1.0) if clip is not None else torch.ones_like(norm)
        scale = torch.where(nonfinite, torch.zeros_like(scale), scale).reshape(1)
        skip = nonfinite.to(torch.int32).reshape(1)
        self.last_grad_norm = norm
        self.last_nonfinite = nonfinite
        for group, flat in zip(self.param_groups, self._flat):
            b1, b2 = group["betas"]
            if cuda:  # 4. AdamW on the shard, stored into every rank's parameters
                ext.shard_adamw_push(flat["pbuf"].ptrs, self.rank, flat["lo"], flat["reduced"], flat["exp_avg"],
                                     flat["exp_avg_sq"], group["lr"], b1, b2, group["eps"], group["weight_decay"],
                                     self._step, scale, skip)
                K._count()
            else:
                lo, n = flat["lo"], flat["shard"]
                view = {"param": flat["param"][lo:lo + n], "grad": flat["reduced"], "exp_avg": flat["exp_avg"],
                        "exp_avg_sq": flat["exp_avg_sq"]}
                _adamw_reference(view, lr=group["lr"], beta1=b1, beta2=b2, eps=group["eps"],
                                 weight_decay=group["weight_decay"], step=self._step, scale=scale,
                                 nonfinite=nonfinite)
                parts = list(flat["param"].view(self.world, n).unbind(0))
                dist.all_gather(parts, flat["param"][lo:lo + n].clone(), group=self.shard_group)
        if cuda:
            self._barrier(dev)  # 5. every push landed
        bump_weight_epoch()
        return loss


_CHUNK = 65536  # elements per block of the multi-tensor kernels


def _local(t: torch.Tensor) -> torch.Tensor:
    from torch.distributed.tensor import DTensor

    return t._local_tensor if isinstance(t, DTensor) else t


def _shard_groups(p: torch.Tensor) -> tuple[Any, ...]:
    """Process groups over which ``p``'s gradient shards must be summed for the
    global norm: one per mesh dimension that shards it (replicated dimensions hold
    copies and are counted once)."""
    from torch.distributed.tensor import DTensor, Shard

    if not isinstance(p, DTensor):
        return ()
    mesh = p.device_mesh
    return tuple(mesh.get_group(i) for i, pl in enumerate(p.placements) if isinstance(pl, Shard))


class MultiTensorAdamW(Optimizer):
    """AdamW over sharded parameters (FSDP2 / tensor-parallel DTensors) with the
    multi-tensor sm_100a kernels: one squared-norm launch and one AdamW launch
    per parameter group over a table of every parameter's local shard, the
    global-norm clip coefficient and the non-finite skip flag computed on the
    device (the same semantics as :class:`FusedAdamW`, which needs plain
    tensors it can re-home into flat buffers). Moments are DTensors shaped and
    placed like their parameters, so ``state_dict`` and DCP reshard them as
    they do torch's AdamW state. The norm sums each parameter's shard partials
    over the mesh dimensions that shard it. On CPU the same steps run with
    torch operations (``gloo`` tests)."""

    def __init__(self, params: Iterable[Any], lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.0) -> None:
        super().__init__(params, {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay,
                                  **_ADAMW_GROUP_KEYS})
        self.max_grad_norm: float | None = None
        self.last_grad_norm: torch.Tensor | None = None
        self.last_nonfinite: torch.Tensor | None = None
        self.norm_groups: tuple[Any, ...] = ()  # other pipeline stages: the squared norm is summed over them
        self._step = 0
        self._tables: dict[tuple, tuple[torch.Tensor, torch.Tensor]] = {}
        for group in self.param_groups:
            for p in group["params"]:
                if _local(p).dtype != torch.float32:
                    raise TypeError("MultiTensorAdamW keeps fp32 parameters; got " + str(_local(p).dtype))
                st = self.state[p]
                st["step"] = torch.tensor(0.0)
                st["exp_avg"] = torch.zeros_like(p)
                st["exp_avg_sq"] = torch.zeros_like(p)

    def _rows(self, group: dict[str, Any]) -> list[tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]]:
        rows = []
        for p in group["params"]:
            if p.grad is None:
                continue
            st = self.state[p]
            rows.append((_local(p), _local(p.grad), _local(st["exp_avg"]), _local(st["exp_avg_sq"])))
        return rows

    def _table(self, rows: list[tuple[torch.Tensor, ...]], dev: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        """Device tables: addresses [T, 4] (rebuilt every step: gradients move) and chunks [C, 3] (cached)."""
        for t in (x for r in rows for x in r):
            if not t.is_contiguous() or t.dtype != torch.float32:
                raise ValueError("multi-tensor AdamW needs contiguous fp32 shards")
        numels = tuple(r[0].numel() for r in rows)
        addrs = torch.tensor([[t.data_ptr() for t in r] for r in rows], dtype=torch.int64)
        key = (dev, numels)
        chunks = self._tables.get(key)
        if chunks is None:
            spec = [(i, s, min(_CHUNK, n - s)) for i, n in enumerate(numels) for s in range(0, n, _CHUNK)]
            chunks = torch.tensor(spec or [[0, 0, 0]], dtype=torch.int64).to(dev)
            if not spec:
                chunks = chunks[:0]
            self._tables[key] = chunks
        return addrs.pin_memory().to(dev, non_blocking=True), chunks

    def grad_norm(self) -> torch.Tensor:
        """Global L2 norm of all gradients across shards (device scalar, no host sync)."""
        import torch.distributed as dist

        params = [p for g in self.param_groups for p in g["params"] if p.grad is not None]
        if not params:
            total = torch.zeros(1, dtype=torch.float32)
            for group in self.norm_groups:
                dist.all_reduce(total, group=group)
            return total.sqrt()[0]
        dev = _local(params[0]).device
        by_groups: dict[tuple, list[torch.Tensor]] = {}
        for p in params:
            by_groups.setdefault(_shard_groups(p), []).append(p)
        total = torch.zeros(1, dtype=torch.float32, device=dev)
        for groups, ps in by_groups.items():
            acc = torch.zeros(1, dtype=torch.float32, device=dev)
            if dev.type == "cuda":
                from avgen_b200.ops import kernels as K
                from avgen_b200.ops._ext import load

                rows = [(_local(p), _local(p.grad), _local(p.grad), _local(p.grad)) for p in ps]
                addrs, chunks = self._table(rows, dev)
                load().mt_sq_norm(addrs, chunks, acc)
                K._count()
            else:
                for p in ps:
                    acc += _local(p.grad).float().pow(2).sum()
            for g in groups:
                dist.all_reduce(acc, group=g)
            total += acc
        for group in self.norm_groups:
            dist.all_reduce(total, group=group)
        return total.sqrt()[0]

    @torch.no_grad()
    def step(self, closure: Any = None, *, max_grad_norm: float | None = None) -> Any:
        loss = closure() if closure is not None else None
        from avgen_b200.models.linear import bump_weight_epoch

        self._step += 1
        norm = self.grad_norm()
        nonfinite = ~torch.isfinite(norm)
        clip = max_grad_norm if max_grad_norm is not None else self.max_grad_norm
        scale = torch.clamp(clip / (norm + 1e-6), max=1.0) if clip is not None else torch.ones_like(norm)
        scale = torch.where(nonfinite, torch.zeros_like(scale), scale).reshape(1).float()
        skip = nonfinite.to(torch.int32).reshape(1)
        self.last_grad_norm = norm
        self.last_nonfinite = nonfinite
        for group in self.param_groups:
            b1, b2 = group["betas"]
            rows = self._rows(group)
            if not rows:
                continue
            for p in group["params"]:
                if p.grad is not None:
                    self.state[p]["step"] = torch.tensor(float(self._step))
            dev = rows[0][0].device
            if dev.type == "cuda":
                from avgen_b200.ops import kernels as K
                from avgen_b200.ops._ext import load

                addrs, chunks = self._table(rows, dev)
                load().mt_adamw(addrs, chunks, group["lr"], b1, b2, group["eps"], group["weight_decay"], self._step,
                                scale.to(dev), skip.to(dev))
                K._count()
            else:
                for prm, g, m, v in rows:
                    _adamw_reference({"param": prm, "grad": g, "exp_avg": m, "exp_avg_sq": v}, lr=group["lr"],
                                     beta1=b1, beta2=b2, eps=group["eps"], weight_decay=group["weight_decay"],
                                     step=self._step, scale=scale, nonfinite=nonfinite)
        bump_weight_epoch()
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        super().zero_grad(set_to_none=set_to_none)

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        super().load_state_dict(state_dict)
        steps = [float(st["step"]) for st in self.state.values() if "step" in st]
        self._step = int(max(steps)) if steps else 0


def _adamw_reference(flat: dict[str, torch.Tensor], *, lr: float, beta1: float, beta2: float, eps: float,
                     weight_decay: float, step: int, scale: torch.Tensor, nonfinite: torch.Tensor) -> None:
    """CPU fp32 AdamW over a flat buffer (same maths as the kernel)."""
    g = torch.where(nonfinite, torch.zeros_like(flat["grad"]), flat["grad"] * scale)
    flat["exp_avg"].mul_(beta1).add_(g, alpha=1 - beta1)
    flat["exp_avg_sq"].mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = math.sqrt(1 - beta2 ** step)
    denom = flat["exp_avg_sq"].sqrt() / bc2 + eps
    flat["param"].mul_(1 - lr * weight_decay).addcdiv_(flat["exp_avg"], denom, value=-lr / bc1)


def build_optimizer(model: nn.Module, *, name: str = "adamw", lr: float, weight_decay: float = 0.0,
                    betas: tuple[float, float] = (0.9, 0.95), eps: float = 1e-8, fused: bool | None = None,
                    no_decay_patterns: Sequence[str] = DEFAULT_NO_DECAY_PATTERNS, dp_group: Any = None,
                    shard_group: Any = None) -> Optimizer:
    """``shard_group`` (a one-node process group): AdamW with moments sharded over
    it and the gradient reduction / parameter all-gather over NVLink
    (:class:`ShardedAdamW`) instead of ``dp_group``'s all-reduce."""
    if lr <= 0.0:
        raise ValueError(f"lr must be positive; got {lr!r}")
    if weight_decay < 0.0:
        raise ValueError("weight_decay must be non-negative")
    if not all(0.0 <= b < 1.0 for b in betas):
        raise ValueError(f"betas must lie in [0, 1); got {betas!r}")
    if eps <= 0.0:
        raise ValueError("eps must be positive")
    groups = build_param_groups(model, weight_decay=weight_decay, no_decay_patterns=no_decay_patterns)
    if name == "adamw":
        from torch.distributed.tensor import DTensor

        on_cuda = all(p.device.type == "cuda" for g in groups for p in g["params"])
        if any(isinstance(p, DTensor) for g in groups for p in g["params"]):
            # FSDP / tensor-parallel shards: multi-tensor kernels over every local shard
            fp32 = all(p.dtype == torch.float32 for g in groups for p in g["params"])
            if fused is not False and fp32:
                return MultiTensorAdamW(groups, lr=lr, betas=betas, eps=eps)
            return torch.optim.AdamW(groups, lr=lr, betas=betas, eps=eps, fused=on_cuda or None)
        use_fused = on_cuda if fused is None else fused
        if shard_group is not None:
            return ShardedAdamW(groups, lr=lr, betas=betas, eps=eps, group=shard_group)
        if use_fused:
            return FusedAdamW(groups, lr=lr, betas=betas, eps=eps, dp_group=dp_group)
        return torch.optim.AdamW(groups, lr=lr, betas=betas, eps=eps)
    if name == "adamw_8bit":
        try:
            import bitsandbytes
        except ImportError as exc:
            raise RuntimeError("the 'adamw_8bit' optimizer requires bitsandbytes") from exc
        return bitsandbytes.optim.AdamW8bit(list(groups), lr=lr, betas=betas, eps=eps)
    if name == "adafactor":
        return torch.optim.Adafactor(groups, lr=lr, beta2_decay=-0.8, eps=(None, eps), weight_decay=weight_decay)
    raise ValueError(f"unknown optimizer {name!r}; available: {', '.join(_OPTIMIZERS)}")
