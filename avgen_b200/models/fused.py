"""The fused DiT block: one autograd node per block driving the sm_100a kernels.

Forward of one block (reference semantics: avgen/models/blocks.py:173-227):

    n1  = rmsnorm(x) * w_a * (1 + scale_a) + shift_a              rmsnorm_mod kernel
    qkv = n1 @ Wqkv^T                                              tcgen05 GEMM
    q,k,v = rope(qknorm(qkv))  (head-major)                        qkv_rope kernel
    O   = flash_attention(q, k, v)                                 tcgen05 attention
    x1  = x + gate_a * (O @ Wo^T)                                  GEMM, gated-residual epilogue
    x2  = x1 + cross_attention(rmsnorm(x1), text)                  norm + GEMMs + attention + residual epilogue
    x3  = x2 + gate_f * down(silu(gate(n3)) * up(n3)),             GEMM with SwiGLU epilogue, then
          n3 = rmsnorm(x2) * w_f * (1 + scale_f) + shift_f          GEMM with gated-residual epilogue

Only ``x``, the self-attention output ``O`` and its log-sum-exp are saved
(about 2 x B*L*W bf16 per block). Backward recomputes every GEMM and the cheap
cross-attention but never the self-attention forward, then runs the backward
kernels; weight gradients accumulate in fp32 through the GEMM's atomic
epilogue. This is the "selective" activation-checkpoint policy of the
reference (avgen/parallel/activation.py:72-160: keep attention outputs,
recompute the rest) built into the block.

Self-attention can be swapped for a context-parallel implementation through
``BlockSpec.attention`` (see :mod:`avgen_b200.parallel.context`).

Adapter-wrapped linears take part through their effective weights, which the
kernels read packed in bf16: a plain LoRA layer's ``W + s B A`` is formed from
W, A and B when they change, and its gradients come from rank-r products with
no dense weight gradient unless W trains; a DoRA (or merged, or dropout)
adapter's effective weight gets its dense gradient, which autograd carries into
the adapter parameters (``fused_inputs``, ``_weight_grads``). Frozen weights get
no weight-gradient GEMM.

Head-parallel tensor parallelism with sequence parallelism
(:mod:`avgen_b200.parallel.heads`) runs through the same node: the norms,
modulation and gated residuals act on this rank's token chunk; each normalised
input is all-gathered over the tensor-parallel group inside the rank's q/k/v,
cross-attention and MLP GEMMs (copy-engine pulls over NVLink, each tile waiting
on its chunk's arrival flag; its heads and hidden slice over the whole
sequence), and each output projection's partial sums are reduce-scattered back
to the token chunk through peer memory before the gated residual. The backward
mirrors that: the gradient entering each output projection is all-gathered
inside its dX GEMM, the gradient leaving each input projection is
reduce-scattered. ``AVGEN_TP_PEER=0``, several samples per batch or a non-NCCL
group use NCCL collectives between the kernels instead.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Any, Protocol

import torch
from torch import nn

__all__ = ["AttentionImpl", "BlockSpec", "LocalAttention", "close_tp_peer", "fused_block_forward", "packed_weights",
           "tp_peer_guard_violations"]

_BF16 = torch.bfloat16


class AttentionImpl(Protocol):
    """Self-attention implementation used inside the fused block."""

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kmask: torch.Tensor | None,
                scale: float) -> tuple[torch.Tensor, torch.Tensor, Any]: ...

    def backward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, do: torch.Tensor,
                 lse: torch.Tensor, kmask: torch.Tensor | None, scale: float,
                 state: Any) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]: ...


class LocalAttention:
    """Single-device flash attention (tcgen05 kernels)."""

    def forward(self, q, k, v, kmask, scale):  # noqa: ANN001, ANN201
        from avgen_b200.ops import kernels as K

        out, lse = K.attention_fwd(q, k, v, kmask=kmask, scale=scale)
        return out, lse, None

    def backward(self, q, k, v, o, do, lse, kmask, scale, state):  # noqa: ANN001, ANN201
        from avgen_b200.ops import kernels as K

        dq, dk, dv = K.attention_bwd(q, k, v, o, do, lse, kmask=kmask, scale=scale)
        return dq, dk, dv


@dataclass
class BlockSpec:
    """Static description of one fused block call."""

    batch: int
    length: int
    width: int
    heads: int
    kv_heads: int
    head_dim: int
    hidden: int
    ffn: str  # "swiglu" | "gelu"
    eps: float
    qk_norm: bool
    cross: bool
    ctx_heads: int = 0
    ctx_kv_heads: int = 0
    text_length: int = 0
    attention: AttentionImpl | None = None
    mod_rows_per_batch: int = 0   # rows sharing one modulation row (0: ``length``)
    groups: torch.Tensor | None = None  # int32 [B*L] modulation row per token (overrides the above)
    # head-parallel tensor parallelism with sequence parallelism: ``length`` is this rank's
    # token chunk (norms, modulation, residuals), ``full_length`` the sequence the rank's
    # heads attend over; None / 0 without tensor parallelism
    tp: Any = None
    full_length: int = 0

    @property
    def seq(self) -> int:
        """Tokens per sample the attention and its projections see."""
        return self.full_length or self.length

    def mod_rows(self) -> dict[str, Any]:
        """Keyword arguments selecting each token's modulation row in the kernels."""
        return {"rows_per_batch": self.mod_rows_per_batch or self.length, "groups": self.groups}


@dataclass(frozen=True)
class _LoRAWeight:
    """A plain LoRA layer's effective weight ``W + s B A``, formed only when packed."""

    base: torch.Tensor
    a: torch.Tensor
    b: torch.Tensor
    scaling: float

    def parts(self) -> tuple[torch.Tensor, ...]:
        return (self.base, self.a, self.b)

    def value(self) -> torch.Tensor:
        delta = (self.b.detach().float() @ self.a.detach().float()).mul_(self.scaling)
        return self.base.detach() + delta.to(self.base.dtype)


def _packed(module: nn.Module, key: str, params: list[Any], build) -> torch.Tensor:  # noqa: ANN001
    """``build(*params)`` in bf16, cached on ``module`` until one of its source
    parameters changes (a LoRA weight's sources are its base, A and B)."""
    from avgen_b200.models.linear import weight_epoch

    with torch.no_grad():
        fresh = lambda: build(*[p.value() if isinstance(p, _LoRAWeight) else p.detach()  # noqa: E731
                                for p in params]).to(_BF16).contiguous()
        if _fsdp_managed(module):
            return fresh()  # FSDP re-gathers the parameters every forward: never serve a cached copy
        sources = [t for p in params for t in (p.parts() if isinstance(p, _LoRAWeight) else (p,))]
        if not all(isinstance(t, nn.Parameter) for t in sources):
            return fresh()  # a temporary's address and version can repeat after it is freed
        cache = module.__dict__.setdefault("_avgen_packed", {})
        version = (weight_epoch(), *((t._version, t.data_ptr()) for t in sources))
        hit = cache.get(key)
        if hit is not None and hit[0] == version:
            return hit[1]
        value = fresh()
        cache[key] = (version, value)
        return value


def _fsdp_managed(module: nn.Module) -> bool:
    try:
        from torch.distributed.fsdp import FSDPModule
    except ImportError:
        return False
    return isinstance(module, FSDPModule)


def _adapted_layers(block: nn.Module) -> dict[str, nn.Module]:
    """The block's adapter-wrapped linears (LoRA / DoRA), by module name."""
    return {name: m for name, m in block.named_modules()
            if isinstance(m, nn.Linear) and callable(getattr(m, "adapted_weight", None))}


def _plain_lora(layer: nn.Module) -> bool:
    """A LoRA adapter whose effective weight is exactly ``W + s B A`` (no DoRA scale,
    not merged, no adapter dropout)."""
    return (getattr(layer, "lora_magnitude", None) is None and not getattr(layer, "merged", False)
            and isinstance(getattr(layer, "lora_dropout", None), nn.Identity)
            and isinstance(getattr(layer, "lora_a", None), torch.Tensor))


def fused_inputs(block: nn.Module, *, differentiable: bool = True) -> tuple[list[str], list[torch.Tensor]]:
    """The tensors the fused node takes, by block parameter name: every parameter but the
    modulation table. A plain LoRA layer contributes its base weight and ``lora_a`` /
    ``lora_b`` themselves: the node packs ``W + s B A`` for its kernels and forms the
    adapter gradients from low-rank products (``dB = s dY^T (X A^T)``,
    ``dA = s (dY B)^T X``), never the dense weight gradient unless the base weight
    trains. Any other adapter (DoRA, merged, with dropout) contributes its effective
    weight under ``<layer>.weight``; the node returns that weight's dense gradient and
    autograd carries it into the adapter through ``adapted_weight()``."""
    adapted = _adapted_layers(block)
    names: list[str] = []
    tensors: list[torch.Tensor] = []
    for name, p in block.named_parameters():
        if name == "scale_shift_table":
            continue
        owner, _, leaf = name.rpartition(".")
        layer = adapted.get(owner)
        if layer is None or _plain_lora(layer):
            names.append(name)
            tensors.append(p)
        elif leaf == "weight":
            names.append(name)
            if differentiable:
                tensors.append(layer.adapted_weight())
            else:
                with torch.no_grad():
                    tensors.append(layer.adapted_weight())
    return names, tensors


def _packing_weights(block: nn.Module, weights: dict[str, torch.Tensor]) -> dict[str, Any]:
    """``weights`` with each plain LoRA layer's base weight standing for ``W + s B A``
    (formed by the packed-weight cache from its three sources, so no second copy of the
    weight is kept beside the packed one)."""
    out: dict[str, Any] = dict(weights)
    for prefix, layer in _adapted_layers(block).items():
        a, bmat = out.get(f"{prefix}.lora_a"), out.get(f"{prefix}.lora_b")
        if a is not None and bmat is not None and _plain_lora(layer):
            out[f"{prefix}.weight"] = _LoRAWeight(out[f"{prefix}.weight"], a, bmat, float(layer.scaling))
    return out


def packed_weights(block: nn.Module, weights: dict[str, torch.Tensor] | None = None) -> dict[str, torch.Tensor]:
    """bf16 kernel-layout weights of a DiT block, rebuilt only after parameter updates.
    ``weights`` (block parameter name -> tensor) replaces the module's own tensors,
    e.g. with adapters' effective weights."""

    def w(name: str) -> torch.Tensor:
        if weights is not None and name in weights:
            return weights[name]
        return block.get_parameter(name)

    ff = block.feed_forward
    out = {
        "qkv": _packed(block, "qkv", [w("attention.q_proj.weight"), w("attention.k_proj.weight"),
                                      w("attention.v_proj.weight")], lambda q, k, v: torch.cat((q, k, v), 0)),
        "o": _packed(block, "o", [w("attention.out_proj.weight")], lambda t: t),
        "down": _packed(block, "down", [w("feed_forward.down_proj.weight")], lambda t: t),
    }
    if hasattr(ff, "gate_proj"):
        out["gu"] = _packed(block, "gu", [w("feed_forward.gate_proj.weight"), w("feed_forward.up_proj.weight")],
                            lambda g, u: torch.stack((g, u), 1).reshape(2 * g.shape[0], g.shape[1]))
    else:
        out["up"] = _packed(block, "up", [w("feed_forward.up_proj.weight")], lambda t: t)
    if block.cross_attention is not None:
        out["cq"] = _packed(block, "cq", [w("cross_attention.q_proj.weight")], lambda t: t)
        out["ckv"] = _packed(block, "ckv", [w("cross_attention.k_proj.weight"), w("cross_attention.v_proj.weight")],
                             lambda k, v: torch.cat((k, v), 0))
        out["co"] = _packed(block, "co", [w("cross_attention.out_proj.weight")], lambda t: t)
    return out


def _f32(t: torch.Tensor | None) -> torch.Tensor | None:
    return None if t is None else t.detach().float().contiguous()


def _attn_impl(spec: BlockSpec) -> AttentionImpl:
    return spec.attention if spec.attention is not None else LocalAttention()


def _norm_weight(norm: nn.Module) -> torch.Tensor | None:
    w = getattr(norm, "weight", None)
    return _f32(w) if isinstance(w, torch.Tensor) else None


def _tp_gather(spec: BlockSpec, rows: torch.Tensor) -> torch.Tensor:
    """This rank's token rows ``[B*L_local, C]`` -> every rank's, ``[B*L, C]`` in sequence
    order (identity without tensor parallelism)."""
    tp = spec.tp
    if tp is None:
        return rows
    import torch.distributed as dist

    rows = rows.contiguous()
    out = torch.empty((tp.world * rows.shape[0], rows.shape[-1]), dtype=rows.dtype, device=rows.device)
    dist.all_gather_into_tensor(out, rows, group=tp.group)
    if spec.batch == 1:
        return out
    c = rows.shape[-1]
    return out.view(tp.world, spec.batch, spec.length, c).transpose(0, 1).reshape(spec.batch * spec.seq, c)


def _tp_reduce(spec: BlockSpec, rows: torch.Tensor) -> torch.Tensor:
    """Partial sums over the full sequence ``[B*L, C]`` -> this rank's token rows of their
    sum over the tensor-parallel ranks, ``[B*L_local, C]`` (identity without it)."""
    tp = spec.tp
    if tp is None:
        return rows
    import torch.distributed as dist

    c = rows.shape[-1]
    src = rows.contiguous() if spec.batch == 1 else \
        rows.view(spec.batch, tp.world, spec.length, c).transpose(0, 1).reshape(-1, c)
    out = torch.empty((spec.batch * spec.length, c), dtype=rows.dtype, device=rows.device)
    dist.reduce_scatter_tensor(out, src, group=tp.group)
    return out


# Peer-memory collective GEMMs of the tensor-parallel group, one per (kind, group, shape):
# every rank creates them at the same call in the same order, so creation is collective.
_TP_PEER: dict[tuple, Any] = {}


def _tp_peer(spec: BlockSpec) -> bool:
    """Whether this block's tensor-parallel collectives run fused with their GEMMs over
    NVLink peer memory (single-sample rows, an NCCL group; ``AVGEN_TP_PEER=0`` keeps
    the NCCL collectives between the kernels)."""
    tp = spec.tp
    if tp is None or spec.batch != 1 or os.environ.get("AVGEN_TP_PEER", "1") == "0":
        return False
    import torch.distributed as dist

    return dist.get_backend(tp.group) == "nccl"


def _tp_comm(kind: str, spec: BlockSpec, rows: int, cols: int, device: torch.device) -> Any:
    from avgen_b200.parallel.collective_gemm import AllGatherGemm, GemmReduceScatter

    key = (kind, id(spec.tp.group), rows, cols, device.index)
    obj = _TP_PEER.get(key)
    if obj is None:
        obj = (AllGatherGemm(spec.tp.group, rows, cols, device, operand="a") if kind == "ag"
               else GemmReduceScatter(spec.tp.group, rows, cols, device))
        _TP_PEER[key] = obj
    return obj


def tp_peer_guard_violations() -> list[tuple[str, int]]:
    """Changed canary bytes around the tensor-parallel peer buffers of this rank (empty
    when no peer write ran past a buffer). Synchronises with the device."""
    bad: list[tuple[str, int]] = []
    for obj in _TP_PEER.values():
        if obj.buf is not None:
            bad += obj.buf.check_guards()
    return bad


def close_tp_peer() -> None:
    """Free the tensor-parallel peer buffers. Collective over their groups: every rank
    calls it at the same point (the buffers were created in the same order)."""
    for obj in list(_TP_PEER.values()):
        obj.close()
    _TP_PEER.clear()


def _tp_gather_gemm(spec: BlockSpec, rows: torch.Tensor, weight: torch.Tensor, *, keep: bool,
                    **gemm_kwargs: Any) -> tuple[torch.Tensor, torch.Tensor]:
    """``(gemm(all_gather(rows), weight), gathered rows)``. On the peer path the gather
    runs on the copy engines while the GEMM computes, each tile of a peer's rows
    waiting on that chunk's arrival flag; ``keep`` lands the gathered rows in a tensor
    of their own (kept for the weight gradient), else they are a view of the
    double-buffered symmetric buffer, valid until the call after next."""
    from avgen_b200.ops import kernels as K

    if not _tp_peer(spec):
        full = _tp_gather(spec, rows)
        return K.gemm(full, weight, **gemm_kwargs), full
    rows = rows.contiguous()
    ag = _tp_comm("ag", spec, rows.shape[0], rows.shape[1], rows.device)
    out = torch.empty((ag.world * ag.rows, ag.cols), device=rows.device, dtype=_BF16) if keep else None
    return ag(rows, weight, gathered_out=out, **gemm_kwargs)


def _tp_gemm_reduce(spec: BlockSpec, x: torch.Tensor, weight: torch.Tensor, **gemm_kwargs: Any) -> torch.Tensor:
    """``reduce_scatter(gemm(x, weight))`` over the token rows. On the peer path the
    GEMM writes its partial product into symmetric memory and this rank sums its rows
    straight out of every peer's buffer."""
    from avgen_b200.ops import kernels as K

    if not _tp_peer(spec):
        return _tp_reduce(spec, K.gemm(x, weight, **gemm_kwargs))
    n = weight.shape[1] if gemm_kwargs.get("b_mn") else weight.shape[0]
    rs = _tp_comm("rs", spec, x.shape[0], n, x.device)
    return rs(x, weight, **gemm_kwargs)

def _gated_residual(spec: BlockSpec, resid: torch.Tensor, update: torch.Tensor,
                    gate: torch.Tensor | None) -> torch.Tensor:
    """``resid + gate * update`` on local rows (each row's gate picked as the kernels'
    modulation rows do), computed in fp32 and rounded once; the tensor-parallel form of
    the GEMM's gated-residual epilogue, which cannot run before the reduce-scatter."""
    r, u = resid.float(), update.float()
    if gate is None:
        return (r + u).to(_BF16)
    if spec.groups is not None:
        return (r + gate[spec.groups.long()] * u).to(_BF16)
    rpb = spec.mod_rows_per_batch or spec.length
    w = r.shape[-1]
    out = r.view(-1, rpb, w) + gate.view(-1, 1, w) * u.view(-1, rpb, w)
    return out.view(-1, w).to(_BF16)


def _forward_impl(spec, block, pw, xb, modf, ctxb, coords, freq, axis, kmask, cmask, *, save,  # noqa: ANN001, ANN202
                  keep_inter=False):
    """Run the block head; returns (intermediates, O, lse, attn_state). The
    intermediates the backward needs come back when ``save`` is False (the
    backward's recompute) or ``keep_inter`` is True (forward that keeps them)."""
    from avgen_b200.ops import kernels as K

    b, length, w = spec.batch, spec.length, spec.width
    h, hk, d = spec.heads, spec.kv_heads, spec.head_dim
    eps = spec.eps
    shift_a, scale_a, gate_a = modf[:, 0], modf[:, 1], modf[:, 2]
    shift_f, scale_f, gate_f = modf[:, 3], modf[:, 4], modf[:, 5]
    att = block.attention
    n1, rstd1 = K.rmsnorm_mod(xb, _norm_weight(block.attention_norm), scale_a, shift_a, **spec.mod_rows(),
                              eps=block.attention_norm.eps or eps)
    qkv, n1g = _tp_gather_gemm(spec, n1, pw["qkv"], keep=not save or keep_inter)
    qw = _norm_weight(att.q_norm) if spec.qk_norm else None
    kw = _norm_weight(att.k_norm) if spec.qk_norm else None
    impl = _attn_impl(spec)
    kv_out = getattr(impl, "kv_out", None) if save else None  # ring CP: write K/V into the shared buffer
    bufs = kv_out(b, hk, length, d, xb.device) if kv_out is not None else None
    q, k, v = K.qkv_rope(qkv, batch=b, length=spec.seq, heads=h, kv_heads=hk, head_dim=d, q_weight=qw, k_weight=kw,
                         coords=coords, freq=freq, axis=axis, eps=eps, k_out=bufs[0] if bufs else None,
                         v_out=bufs[1] if bufs else None)
    scale = 1.0 / math.sqrt(d)
    if save:
        o, lse, attn_state = impl.forward(q, k, v, kmask, scale)
    else:
        o = lse = attn_state = None
    return_o = o
    inter: dict[str, Any] = {}
    if not save or keep_inter:
        inter.update(n1=n1, n1g=n1g, rstd1=rstd1, qkv=qkv, q=q, k=k, v=v)
    return inter, return_o, lse, attn_state


def _block_tail(spec, block, pw, xb, modf, ctxb, cmask, o, *, keep, want_out=False,  # noqa: ANN001, ANN202
                keep_mlp=True):
    """Everything after the self-attention kernel. Returns x3 (None when only
    the intermediates are wanted: ``keep`` without ``want_out``) and, if keep,
    the intermediates needed for backward (without the MLP activations gu and h
    when ``keep_mlp`` is False)."""
    from avgen_b200.ops import kernels as K

    b, length, w = spec.batch, spec.length, spec.width
    m = b * length
    mf = b * spec.seq
    eps = spec.eps
    gate_a = modf[:, 2]
    shift_f, scale_f, gate_f = modf[:, 3], modf[:, 4], modf[:, 5]
    keep_d: dict[str, Any] = {}
    if spec.tp is None:
        a_o = torch.empty((m, w), device=xb.device, dtype=_BF16) if keep else None
        x1 = K.gemm(o.view(m, -1), pw["o"], epilogue="gate_resid", resid=xb, gate=gate_a, **spec.mod_rows(),
                    aux=a_o)
    else:
        a_o = _tp_gemm_reduce(spec, o.view(mf, -1), pw["o"])
        x1 = _gated_residual(spec, xb, a_o, gate_a)
    x2 = x1
    if spec.cross and ctxb is not None:
        ca = block.cross_attention
        n2, rstd2 = K.rmsnorm_mod(x1, _norm_weight(block.cross_norm), eps=block.cross_norm.eps or eps)
        qc, n2g = _tp_gather_gemm(spec, n2, pw["cq"], keep=keep)
        t = ctxb.shape[1]
        kvc = K.gemm(ctxb.view(b * t, -1), pw["ckv"])
        cqw = _norm_weight(ca.q_norm) if spec.qk_norm else None
        ckw = _norm_weight(ca.k_norm) if spec.qk_norm else None
        qh, _, _ = K.qkv_rope(qc, batch=b, length=spec.seq, heads=spec.ctx_heads, kv_heads=0, head_dim=spec.head_dim,
                              q_weight=cqw, k_weight=None, coords=None, freq=None, axis=None, eps=eps)
        _, kc, vc = K.qkv_rope(kvc, batch=b, length=t, heads=0, kv_heads=spec.ctx_kv_heads, head_dim=spec.head_dim,
                               q_weight=None, k_weight=ckw, coords=None, freq=None, axis=None, eps=eps)
        oc, lsec = K.attention_fwd(qh, kc, vc, kmask=cmask, scale=1.0 / math.sqrt(spec.head_dim))
        if spec.tp is None:
            x2 = K.gemm(oc.view(m, -1), pw["co"], epilogue="gate_resid", resid=x1, gate=None)
        else:
            x2 = _gated_residual(spec, x1, _tp_gemm_reduce(spec, oc.view(mf, -1), pw["co"]), None)
        if keep:
            keep_d.update(x1=x1, n2=n2, n2g=n2g, rstd2=rstd2, qc=qc, kvc=kvc, qh=qh, kc=kc, vc=vc, oc=oc,
                          lsec=lsec)
    elif keep:
        keep_d.update(x1=x1)
    n3, rstd3 = K.rmsnorm_mod(x2, _norm_weight(block.ffn_norm), scale_f, shift_f, **spec.mod_rows(),
                              eps=block.ffn_norm.eps or eps)
    gu, hdn, n3g = _mlp_up(spec, pw, n3, keep=keep and keep_mlp, gather=True, keep_gathered=keep)
    if keep and not want_out:
        f = _tp_gemm_reduce(spec, hdn, pw["down"])
        keep_d.update(a_o=a_o, x2=x2, n3=n3, n3g=n3g, rstd3=rstd3, gu=gu, h=hdn, f=f)
        return None, keep_d
    if spec.tp is None:
        f = torch.empty((m, w), device=xb.device, dtype=_BF16) if keep else None
        x3 = K.gemm(hdn, pw["down"], epilogue="gate_resid", resid=x2, gate=gate_f, **spec.mod_rows(), aux=f)
    else:
        f = _tp_gemm_reduce(spec, hdn, pw["down"])
        x3 = _gated_residual(spec, x2, f, gate_f)
    if keep:
        keep_d.update(a_o=a_o, x2=x2, n3=n3, n3g=n3g, rstd3=rstd3, f=f)
        if keep_mlp:
            keep_d.update(gu=gu, h=hdn)
    return x3, keep_d


def _mlp_up(spec, pw, n3, *, keep, gather=False, keep_gathered=False):  # noqa: ANN001, ANN202
    """MLP up-projection with its activation epilogue: (pre-activation or None, h), and
    the gathered input as a third value when ``gather`` (the tensor-parallel
    all-gather of ``n3``'s token rows runs inside the GEMM)."""
    from avgen_b200.ops import kernels as K

    m = n3.shape[0] * (spec.tp.world if gather and spec.tp is not None else 1)
    swiglu = spec.ffn == "swiglu"
    gu = torch.empty((m, 2 * spec.hidden if swiglu else spec.hidden), device=n3.device, dtype=_BF16) if keep else None
    weight, epilogue = (pw["gu"], "swiglu") if swiglu else (pw["up"], "gelu")
    if not gather:
        return gu, K.gemm(n3, weight, epilogue=epilogue, aux=gu)
    hdn, n3g = _tp_gather_gemm(spec, n3, weight, keep=keep_gathered, epilogue=epilogue, aux=gu)
    return gu, hdn, n3g


def _forward_full(spec, block, pw, xb, modf, ctxb, coords, freq, axis, kmask, cmask):  # noqa: ANN001, ANN202
    _, o, lse, attn_state = _forward_impl(spec, block, pw, xb, modf, ctxb, coords, freq, axis, kmask, cmask,
                                          save=True)
    x3, _ = _block_tail(spec, block, pw, xb, modf, ctxb, cmask, o, keep=False)
    return x3, (o, lse, attn_state)


def _weight_grads(block: nn.Module, members: list[tuple[str, Any]], dy: torch.Tensor, x: torch.Tensor,
                  weights: dict[str, torch.Tensor], need: dict[str, bool], out: dict[str, torch.Tensor | None]) -> None:
    """Gradients of the linears that share input ``x`` and whose output gradients are the
    columns of ``dy``: ``members`` lists ``(layer prefix, columns)`` with ``columns`` a
    ``slice`` of a concatenated output or ``"even"`` / ``"odd"`` for the interleaved
    SwiGLU pair. A dense weight gradient is formed only for weights that train; plain
    LoRA adapters get theirs from rank-r products; frozen weights get nothing."""
    from avgen_b200.ops import kernels as K

    dev = dy.device
    rows = dy.shape[1]
    dense = None
    if any(need.get(f"{p}.weight", False) for p, _ in members):
        dense = torch.zeros((rows, x.shape[1]), device=dev, dtype=torch.float32)
        K.linear_dw(dy, x, dense)
    layers = dict(block.named_modules())
    for prefix, cols in members:
        sel = cols if isinstance(cols, slice) else slice(0 if cols == "even" else 1, None, 2)
        if dense is not None and need.get(f"{prefix}.weight", False):
            out[f"{prefix}.weight"] = dense[sel].contiguous()
        a_name, b_name = f"{prefix}.lora_a", f"{prefix}.lora_b"
        if not (need.get(a_name, False) or need.get(b_name, False)):
            continue
        layer = layers[prefix]
        a = weights[a_name].detach().to(_BF16).contiguous()        # [r, in]
        bm = weights[b_name].detach().to(_BF16).contiguous()       # [out, r]
        r = a.shape[0]
        xa = K.gemm(x, a)                                          # [M, r] = X A^T
        if isinstance(cols, slice):
            dy_m = dy[:, sel]                                      # row-strided view of this layer's columns
            g_b = torch.zeros((bm.shape[0], r), device=dev, dtype=torch.float32)
            K.linear_dw(dy_m, xa, g_b)                             # dY^T (X A^T)
            dyb = K.gemm(dy_m, bm, b_mn=True)                      # [M, r] = dY B
        else:  # interleaved columns: route through a zero-padded B and keep every other row
            full = torch.zeros((rows, r), device=dev, dtype=torch.float32)
            K.linear_dw(dy, xa, full)
            g_b = full[sel].contiguous()
            padded = torch.zeros((rows, r), device=dev, dtype=_BF16)
            padded[sel] = bm
            dyb = K.gemm(dy, padded, b_mn=True)
        g_a = torch.zeros((r, x.shape[1]), device=dev, dtype=torch.float32)
        K.linear_dw(dyb, x, g_a)                                   # (dY B)^T X
        if need.get(a_name, False):
            out[a_name] = g_a.mul_(layer.scaling).to(weights[a_name].dtype)
        if need.get(b_name, False):
            out[b_name] = g_b.mul_(layer.scaling).to(weights[b_name].dtype)


def _backward_impl(spec, block, xb, modf, ctxb, coords, freq, axis, kmask, cmask, o, lse, attn_state, dout,  # noqa: ANN001, ANN202
                   saved=None, names=None, need=None):
    from avgen_b200.ops import kernels as K

    b, length, w = spec.batch, spec.length, spec.width
    m = b * length
    mf = b * spec.seq
    h, hk, d = spec.heads, spec.kv_heads, spec.head_dim
    eps = spec.eps
    dev = xb.device
    if names is None:
        names, tensors = fused_inputs(block, differentiable=False)
    else:
        tensors = fused_inputs(block, differentiable=False)[1]
    weights = dict(zip(names, tensors))
    if need is None:
        need = {n: True for n in names}
    pw = packed_weights(block, _packing_weights(block, weights))
    pgrads: dict[str, torch.Tensor | None] = {}
    att = block.attention
    ff = block.feed_forward
    # ---------------------------------------------------------------- recompute (unless kept in forward)
    if saved is not None:
        inter, keep = saved
        if "gu" not in keep:  # the MLP activations were not kept: rebuild them from n3
            keep = dict(keep)
            keep["gu"], keep["h"] = _mlp_up(spec, pw, keep["n3g"], keep=True)
    else:
        inter, _, _, _ = _forward_impl(spec, block, pw, xb, modf, ctxb, coords, freq, axis, kmask, cmask,
                                       save=False)
        _, keep = _block_tail(spec, block, pw, xb, modf, ctxb, cmask, o, keep=True)
    dmod = torch.zeros_like(modf)  # [modulation rows, 6, W]
    gate_a, gate_f = modf[:, 2], modf[:, 5]
    dx3 = dout.reshape(m, w).to(_BF16).contiguous()

    def zeros_like_param(p: torch.Tensor) -> torch.Tensor:
        return torch.zeros(p.shape, device=dev, dtype=torch.float32)

    # ---------------------------------------------------------------- FFN
    dh, df = _tp_gather_gemm(spec, K.gate_bwd(dx3, keep["f"], gate_f, dmod[:, 5], **spec.mod_rows()), pw["down"],
                             keep=False, b_mn=True)
    _weight_grads(block, [("feed_forward.down_proj", slice(None))], df, keep["h"], weights, need, pgrads)
    if spec.ffn == "swiglu":
        dgu = K.swiglu_bwd(dh, keep["gu"])
        dn3 = _tp_gemm_reduce(spec, dgu, pw["gu"], b_mn=True)
        _weight_grads(block, [("feed_forward.gate_proj", "even"), ("feed_forward.up_proj", "odd")], dgu,
                      keep["n3g"], weights, need, pgrads)
    else:
        dpre = K.gelu_bwd(dh, keep["gu"])
        dn3 = _tp_gemm_reduce(spec, dpre, pw["up"], b_mn=True)
        _weight_grads(block, [("feed_forward.up_proj", slice(None))], dpre, keep["n3g"], weights, need, pgrads)
    g_ffn_norm = zeros_like_param(block.ffn_norm.weight) if block.ffn_norm.weight is not None else None
    dx2 = K.rmsnorm_mod_bwd(keep["x2"], keep["rstd3"], dn3, _norm_weight(block.ffn_norm), modf[:, 4], modf[:, 3],
                            dres=dx3, dweight=g_ffn_norm, dscale=dmod[:, 4], dshift=dmod[:, 3],
                            **spec.mod_rows())
    # ---------------------------------------------------------------- cross attention
    dctx = None
    cross_grads: dict[str, torch.Tensor | None] = {}
    if spec.cross and ctxb is not None:
        ca = block.cross_attention
        t = ctxb.shape[1]
        doc, dco = _tp_gather_gemm(spec, dx2, pw["co"], keep=False, b_mn=True)
        _weight_grads(block, [("cross_attention.out_proj", slice(None))], dco, keep["oc"].view(mf, -1), weights,
                      need, pgrads)
        dqh, dkc, dvc = K.attention_bwd(keep["qh"], keep["kc"], keep["vc"], keep["oc"],
                                        doc.view(b, spec.seq, spec.ctx_heads, d), keep["lsec"], kmask=cmask,
                                        scale=1.0 / math.sqrt(d))
        cqw = _norm_weight(ca.q_norm) if spec.qk_norm else None
        ckw = _norm_weight(ca.k_norm) if spec.qk_norm else None
        g_cqn = zeros_like_param(ca.q_norm.weight) if cqw is not None else None
        g_ckn = zeros_like_param(ca.k_norm.weight) if ckw is not None else None
        dqc = K.qkv_rope_bwd(keep["qc"], dqh.to(_BF16), None, None, batch=b, length=spec.seq, heads=spec.ctx_heads,
                             kv_heads=0, head_dim=d, q_weight=cqw, k_weight=None, coords=None, freq=None, axis=None,
                             dq_weight=g_cqn, eps=eps)
        dkvc = K.qkv_rope_bwd(keep["kvc"], None, dkc, dvc, batch=b, length=t, heads=0, kv_heads=spec.ctx_kv_heads,
                              head_dim=d, q_weight=None, k_weight=ckw, coords=None, freq=None, axis=None,
                              dk_weight=g_ckn, eps=eps)
        dn2 = _tp_gemm_reduce(spec, dqc, pw["cq"], b_mn=True)
        _weight_grads(block, [("cross_attention.q_proj", slice(None))], dqc, keep["n2g"], weights, need, pgrads)
        kv_rows = ca.k_proj.weight.shape[0]
        _weight_grads(block, [("cross_attention.k_proj", slice(0, kv_rows)),
                              ("cross_attention.v_proj", slice(kv_rows, None))], dkvc, ctxb.view(b * t, -1),
                      weights, need, pgrads)
        dctx = K.linear_dx(dkvc, pw["ckv"]).view(b, t, -1)
        g_cross_norm = zeros_like_param(block.cross_norm.weight) if block.cross_norm.weight is not None else None
        dx1 = K.rmsnorm_mod_bwd(keep["x1"], keep["rstd2"], dn2, _norm_weight(block.cross_norm), dres=dx2,
                                dweight=g_cross_norm)
        cross_grads = {"cross_norm.weight": g_cross_norm, "cross_attention.q_norm.weight": g_cqn,
                       "cross_attention.k_norm.weight": g_ckn}
    else:
        dx1 = dx2
    # ---------------------------------------------------------------- self attention
    do, da = _tp_gather_gemm(spec, K.gate_bwd(dx1, keep["a_o"], gate_a, dmod[:, 2], **spec.mod_rows()), pw["o"],
                             keep=False, b_mn=True)
    _weight_grads(block, [("attention.out_proj", slice(None))], da, o.view(mf, -1), weights, need, pgrads)
    impl = _attn_impl(spec)
    dq, dk, dv = impl.backward(inter["q"], inter["k"], inter["v"], o, do.view(b, spec.seq, h, d), lse, kmask,
                               1.0 / math.sqrt(d), attn_state)
    qw = _norm_weight(att.q_norm) if spec.qk_norm else None
    kw = _norm_weight(att.k_norm) if spec.qk_norm else None
    g_qn = zeros_like_param(att.q_norm.weight) if qw is not None else None
    g_kn = zeros_like_param(att.k_norm.weight) if kw is not None else None
    dqkv = K.qkv_rope_bwd(inter["qkv"], dq.to(_BF16), dk, dv, batch=b, length=spec.seq, heads=h, kv_heads=hk,
                          head_dim=d, q_weight=qw, k_weight=kw, coords=coords, freq=freq, axis=axis, dq_weight=g_qn,
                          dk_weight=g_kn, eps=eps)
    dn1 = _tp_gemm_reduce(spec, dqkv, pw["qkv"], b_mn=True)
    qr, kr = h * d, hk * d
    _weight_grads(block, [("attention.q_proj", slice(0, qr)), ("attention.k_proj", slice(qr, qr + kr)),
                          ("attention.v_proj", slice(qr + kr, None))], dqkv, inter["n1g"], weights, need, pgrads)
    g_attn_norm = zeros_like_param(block.attention_norm.weight) if block.attention_norm.weight is not None else None
    dx = K.rmsnorm_mod_bwd(xb, inter["rstd1"], dn1, _norm_weight(block.attention_norm), modf[:, 1], modf[:, 0],
                           dres=dx1, dweight=g_attn_norm, dscale=dmod[:, 1], dshift=dmod[:, 0],
                           **spec.mod_rows())
    pgrads.update({"attention_norm.weight": g_attn_norm, "attention.q_norm.weight": g_qn,
                   "attention.k_norm.weight": g_kn, "ffn_norm.weight": g_ffn_norm, **cross_grads})
    ordered = [pgrads.get(name) if need.get(name, True) else None for name in names]
    return dx, dmod, dctx, ordered


# Bytes per token kept by the forward when it skips the backward's recompute, by
# mode: everything ("all"), everything but the MLP activations ("no_mlp"). Filled
# from the first block that keeps them; the first guess is conservative.
_KEEP_BYTES: dict[str, float] = {}
_KEEP_MARGIN = float(os.environ.get("AVGEN_KEEP_MARGIN_GB", "20")) * 2**30


def _keep_mode(spec: BlockSpec, xb: torch.Tensor) -> str:
    """Whether this block's forward keeps its intermediates for the backward
    (skipping the recompute) given the device memory free right now.

    ``AVGEN_KEEP_ACTIVATIONS``: ``auto`` (default) picks per block the most that
    fits while leaving room for what the rest of the forward must hold (later
    blocks' saved inputs and outputs, ring buffers still to be allocated) plus a
    margin (``AVGEN_KEEP_MARGIN_GB``, 20) for the backward's transients;
    ``all`` / ``no_mlp`` / ``none`` force a mode.
    """
    policy = os.environ.get("AVGEN_KEEP_ACTIVATIONS", "auto")
    if policy in ("all", "no_mlp", "none"):
        return policy
    if not xb.is_cuda:
        return "none"
    free, _ = torch.cuda.mem_get_info(xb.device)
    free += torch.cuda.memory_reserved(xb.device) - torch.cuda.memory_allocated(xb.device)
    tokens = spec.batch * spec.seq
    w, f = spec.width, spec.hidden
    # reserve what the rest of the forward must still hold: every later block's saved
    # input and attention output (up to 40 blocks) and ring buffers not yet allocated
    margin = _KEEP_MARGIN + 40 * tokens * (4 * w + 4 * spec.heads)
    if hasattr(spec.attention, "kv_out"):
        from avgen_b200.parallel.context import ring_buffers_pending

        margin += ring_buffers_pending(spec.batch, spec.kv_heads, spec.length, spec.head_dim)
    guess_no_mlp = tokens * (18 * w * 2 + 64)
    per = {"all": max(_KEEP_BYTES.get("all", 0.0) * tokens, guess_no_mlp + tokens * 3 * f * 2),
           "no_mlp": max(_KEEP_BYTES.get("no_mlp", 0.0) * tokens, guess_no_mlp)}
    for mode in ("all", "no_mlp"):
        if free - per[mode] > margin:
            return mode
    return "none"


class FusedBlockFn(torch.autograd.Function):
    """Autograd node for a whole DiT block."""

    @staticmethod
    def forward(ctx, spec, block, names, coords, freq, axis, kmask, cmask, x, mod, context, *params):  # noqa: ANN001, ANN205
        b, length, w = spec.batch, spec.length, spec.width
        m = b * length
        xb = x.reshape(m, w).to(_BF16).contiguous()
        modf = mod.detach().float().contiguous()
        ctxb = context.detach().to(_BF16).contiguous() if context is not None else None
        pw = packed_weights(block, _packing_weights(block, dict(zip(names, params))))
        mode = _keep_mode(spec, xb) if any(ctx.needs_input_grad) else "none"
        ctx.saved = None
        if mode == "none":
            x3, (o, lse, attn_state) = _forward_full(spec, block, pw, xb, modf, ctxb, coords, freq, axis, kmask,
                                                     cmask)
        else:
            inter, o, lse, attn_state = _forward_impl(spec, block, pw, xb, modf, ctxb, coords, freq, axis, kmask,
                                                      cmask, save=True, keep_inter=True)
            x3, keep = _block_tail(spec, block, pw, xb, modf, ctxb, cmask, o, keep=True, want_out=True,
                                   keep_mlp=mode == "all")
            ctx.saved = (inter, keep)
            if mode not in _KEEP_BYTES:
                seen: set[int] = set()
                total = 0
                for t in (*inter.values(), *keep.values()):
                    if isinstance(t, torch.Tensor) and t.data_ptr() not in seen:
                        seen.add(t.data_ptr())
                        total += t.numel() * t.element_size()
                _KEEP_BYTES[mode] = total * 1.05 / max(1, spec.batch * spec.length)  # bytes per token
        ctx.spec = spec
        ctx.block = block
        ctx.names = names
        ctx.attn_state = attn_state
        ctx.flags = (coords is not None, kmask is not None, cmask is not None, ctxb is not None)
        empty = torch.empty(0)
        ctx.save_for_backward(xb, modf, ctxb if ctxb is not None else empty, o, lse,
                              coords if coords is not None else empty, freq if freq is not None else empty,
                              axis if axis is not None else empty, kmask if kmask is not None else empty,
                              cmask if cmask is not None else empty)
        ctx.x_dtype = x.dtype
        ctx.ctx_dtype = context.dtype if context is not None else None
        return x3.view(b, length, w).to(x.dtype)

    @staticmethod
    def backward(ctx, dout):  # noqa: ANN001, ANN205
        xb, modf, ctxb, o, lse, coords, freq, axis, kmask, cmask = ctx.saved_tensors
        has_coords, has_kmask, has_cmask, has_ctx = ctx.flags
        dx, dmod, dctx, pgrads = _backward_impl(
            ctx.spec, ctx.block, xb, modf, ctxb if has_ctx else None, coords if has_coords else None,
            freq if has_coords else None, axis if has_coords else None, kmask if has_kmask else None,
            cmask if has_cmask else None, o, lse, ctx.attn_state, dout, saved=ctx.saved, names=ctx.names,
            need=dict(zip(ctx.names, ctx.needs_input_grad[11:])))
        ctx.saved = None
        if dctx is not None and ctx.ctx_dtype is not None:
            dctx = dctx.to(ctx.ctx_dtype)
        return (None, None, None, None, None, None, None, None, dx.view_as(dout).to(ctx.x_dtype), dmod, dctx,
                *pgrads)


def fused_block_forward(block: nn.Module, hidden: torch.Tensor, combined_mod: torch.Tensor, *,
                        coords: torch.Tensor | None, freq: torch.Tensor | None, axis: torch.Tensor | None,
                        kmask: torch.Tensor | None, context: torch.Tensor | None, cmask: torch.Tensor | None,
                        attention_impl: AttentionImpl | None = None,
                        mod_index: torch.Tensor | None = None) -> torch.Tensor:
    """Run ``block`` through :class:`FusedBlockFn` (CUDA only).

    ``combined_mod`` is the block's adaLN modulation (shared rows plus its table):
    ``(B, 6, W)`` per sample, ``(B, L, 6, W)`` per token, or ``(R, 6, W)`` rows that
    ``mod_index`` ``(B, L)`` selects for each token. The last form is how per-token
    noise levels with few distinct values (clean conditioning frames vs. noisy ones)
    stay cheap: the kernels read each token's row through the index instead of a
    materialised per-token tensor.
    """
    b, length, w = hidden.shape
    rpb = 0
    groups = None
    if mod_index is not None:
        groups = mod_index.reshape(-1).to(torch.int32).contiguous()
    elif combined_mod.ndim == 4:
        combined_mod = combined_mod.reshape(b * length, *combined_mod.shape[2:])
        rpb = 1
    att = block.attention
    ff = block.feed_forward
    ffn = "swiglu" if hasattr(ff, "gate_proj") else "gelu"
    hidden_dim = ff.down_proj.weight.shape[1]
    ca = block.cross_attention
    spec = BlockSpec(batch=b, length=length, width=w, heads=att.num_heads, kv_heads=att.num_kv_heads,
                     head_dim=att.head_dim, hidden=hidden_dim, ffn=ffn, eps=block.attention_norm.eps or 1e-6,
                     qk_norm=isinstance(att.q_norm, nn.RMSNorm), cross=ca is not None and context is not None,
                     ctx_heads=ca.num_heads if ca is not None else 0,
                     ctx_kv_heads=ca.num_kv_heads if ca is not None else 0,
                     text_length=context.shape[1] if context is not None else 0, attention=attention_impl,
                     mod_rows_per_batch=rpb, groups=groups)
    tp = getattr(block, "tp", None)
    if tp is not None:
        # head-parallel shards: this rank's heads and MLP slice over the whole sequence, the
        # residual stream on its own token chunk; the text context feeds every rank's heads,
        # so its gradient is summed over the group
        if not tp.sequence_parallel or attention_impl is not None:
            raise ValueError("the fused block runs tensor parallelism with sequence parallelism and local "
                             "attention only")
        spec.tp, spec.full_length = tp, length * tp.world
        if context is not None:
            context = tp.shared(context)
    names, params = fused_inputs(block)
    return FusedBlockFn.apply(spec, block, names, coords, freq, axis, kmask, cmask, hidden, combined_mod, context,
                              *params)
