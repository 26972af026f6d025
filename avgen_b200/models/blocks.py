"""DiT blocks: DiTBlock, TextRefinerBlock, CrossModalFusion.

``DiTBlock`` is pre-norm adaLN self-attention -> un-modulated cross-attention ->
adaLN FFN with gated residuals and a per-block ``scale_shift_table`` added to
the shared modulation (adaLN-single; avgen/models/blocks.py:107-249). On CUDA
it runs as one fused autograd node (:mod:`avgen_b200.models.fused`); on the CPU
the eager forward below is the oracle the fused path is tested against.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn

from avgen_b200.models.layers import (MODULATION_CHUNKS, CrossAttention, GeluMLP, SelfAttention, SwiGLU, init_norm,
                                      modulate, rms_norm)
from avgen_b200.models.rope import RotaryEmbedding, RotaryTables

__all__ = ["CrossModalFusion", "DiTBlock", "RopeInputs", "TextRefinerBlock", "temporal_neighbour_mask"]


@dataclass
class RopeInputs:
    """Coordinates plus the rotary module: tables are built only if an eager path needs them."""

    coords: torch.Tensor
    rope: RotaryEmbedding
    _tables: RotaryTables | None = None

    def tables(self) -> RotaryTables:
        if self._tables is None:
            self._tables = self.rope(self.coords)
        return self._tables

    def kernel_args(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        freq, axis = self.rope.kernel_frequencies(self.coords.device)
        return self.coords.contiguous(), freq, axis


def temporal_neighbour_mask(query_seconds: torch.Tensor, key_seconds: torch.Tensor, *, window_seconds: float,
                            key_mask: torch.Tensor | None = None) -> torch.Tensor | None:
    """Cross-modal attention mask keeping keys within ``window_seconds`` of each query.

    Returns ``(B, 1, Lq, Lk)`` bool or ``None``. A query with no neighbour
    attends everywhere allowed (avgen/models/blocks.py:54-104).
    """
    if window_seconds <= 0.0:
        if key_mask is None or bool(key_mask.all()):
            return None
        return key_mask[:, None, None, :]
    delta = (query_seconds[:, :, None] - key_seconds[:, None, :]).abs()
    mask = delta <= window_seconds
    if key_mask is not None:
        mask = mask & key_mask[:, None, :]
    mask = mask | ~mask.any(-1, keepdim=True)
    return mask[:, None]


def _fused_eligible(block: DiTBlock, hidden: torch.Tensor) -> bool:
    if hidden.device.type != "cuda":
        return False
    att = block.attention
    if att.head_dim != 128 or block.width % 8:
        return False
    linears = [att.q_proj, att.k_proj, att.v_proj, att.out_proj, *block.feed_forward.children()]
    if block.cross_attention is not None:
        ca = block.cross_attention
        linears += [ca.q_proj, ca.k_proj, ca.v_proj, ca.out_proj]
        if ca.head_dim != 128:
            return False
    from torch.distributed.tensor import DTensor

    for m in linears:
        if not isinstance(m, nn.Linear):
            continue
        if isinstance(m.weight, DTensor):
            return False  # DTensor shards run the per-layer path
        if hasattr(m, "adapted_weight"):
            # adapters join the fused block through their effective weight, which holds for
            # LoRA / DoRA without adapter dropout (dropout acts on the adapter's input only)
            adapter_params = [getattr(m, n, None) for n in ("lora_a", "lora_b", "lora_magnitude")]
            if any(isinstance(t, DTensor) for t in adapter_params):
                return False
            if not getattr(m, "merged", False) and not isinstance(getattr(m, "lora_dropout", None), nn.Identity):
                return False
    tp = getattr(block, "tp", None)
    if tp is not None and (not tp.sequence_parallel or block.attention_impl is not None):
        return False  # head-parallel shards fuse with sequence parallelism and local attention
    return all(getattr(m, "bias", None) is None for m in linears if isinstance(m, nn.Linear))


class DiTBlock(nn.Module):
    def __init__(self, width: int, num_heads: int, *, hidden: int, head_dim: int | None = None,
                 num_kv_heads: int | None = None, context_width: int | None = None, cross_attention: bool = True,
                 qk_norm: bool = True, eps: float = 1e-6, ffn: str = "swiglu") -> None:
        super().__init__()
        self.width = width
        self.attention_norm = rms_norm(width, eps=eps)
        self.attention = SelfAttention(width, num_heads, head_dim=head_dim, num_kv_heads=num_kv_heads,
                                       qk_norm=qk_norm, eps=eps)
        self.cross_norm: nn.Module | None = None
        self.cross_attention: CrossAttention | None = None
        if cross_attention:
            self.cross_norm = rms_norm(width, eps=eps)
            self.cross_attention = CrossAttention(width, num_heads, context_width=context_width, head_dim=head_dim,
                                                  num_kv_heads=num_kv_heads, qk_norm=qk_norm, eps=eps)
        self.ffn_norm = rms_norm(width, eps=eps)
        if ffn == "swiglu":
            self.feed_forward: nn.Module = SwiGLU(width, hidden)
        elif ffn == "gelu":
            self.feed_forward = GeluMLP(width, hidden)
        else:
            raise ValueError(f"ffn must be 'swiglu' or 'gelu'; got {ffn!r}")
        self.scale_shift_table = nn.Parameter(torch.zeros(MODULATION_CHUNKS, width))
        self.attention_impl = None  # set by context parallelism for the fused path
        self.use_fused = True

    def forward(self, hidden: torch.Tensor, *, modulation: torch.Tensor, rope: RotaryTables | RopeInputs | None = None,
                key_mask: torch.Tensor | None = None, context: torch.Tensor | None = None,
                context_mask: torch.Tensor | None = None,
                modulation_index: torch.Tensor | None = None) -> torch.Tensor:
        """One block. ``modulation`` is ``(B, 6, W)`` per sample, ``(B, L, 6, W)`` per
        token, or ``(R, 6, W)`` shared rows picked per token by ``modulation_index``
        ``(B, L)`` (integer row numbers)."""
        if modulation.ndim not in (3, 4):
            raise ValueError(f"modulation must be (batch, 6, width) or (batch, length, 6, width); got "
                             f"{tuple(modulation.shape)}")
        if modulation_index is not None and modulation.ndim != 3:
            raise ValueError("modulation_index selects rows of a (rows, 6, width) modulation")
        combined = modulation + self.scale_shift_table
        if (self.use_fused and _fused_eligible(self, hidden)
                and (rope is None or isinstance(rope, RopeInputs))):
            return self._fused(hidden, combined, rope, key_mask, context, context_mask, modulation_index)
        if modulation_index is not None:
            combined = combined[modulation_index.long()]
        return self._eager(hidden, combined, rope, key_mask, context, context_mask)

    def _fused(self, hidden, combined, rope, key_mask, context, context_mask, mod_index=None):  # noqa: ANN001, ANN202
        from avgen_b200.models.fused import fused_block_forward
        from avgen_b200.ops.kernels import pack_key_mask

        coords = freq = axis = None
        if rope is not None:
            coords, freq, axis = rope.kernel_args()
        kmask = pack_key_mask(key_mask) if key_mask is not None else None
        cmask = pack_key_mask(context_mask) if (context_mask is not None and context is not None) else None
        if self.cross_attention is None:
            context = None
        return fused_block_forward(self, hidden, combined, coords=coords, freq=freq, axis=axis, kmask=kmask,
                                   context=context, cmask=cmask, attention_impl=self.attention_impl,
                                   mod_index=mod_index)

    def _eager(self, hidden, combined, rope, key_mask, context, context_mask):  # noqa: ANN001, ANN202
        parts = combined.unbind(-2)
        if combined.ndim == 3:
            parts = tuple(p[:, None] for p in parts)
        shift_a, scale_a, gate_a, shift_f, scale_f, gate_f = parts
        tables = rope.tables() if isinstance(rope, RopeInputs) else rope
        normed = modulate(self.attention_norm(hidden), shift_a, scale_a)
        hidden = hidden + gate_a * self.attention(normed, tables, key_mask=key_mask)
        if context is not None and self.cross_norm is not None and self.cross_attention is not None:
            hidden = hidden + self.cross_attention(self.cross_norm(hidden), context, context_mask)
        normed = modulate(self.ffn_norm(hidden), shift_f, scale_f)
        return hidden + gate_f * self.feed_forward(normed)

    def init_weights(self, *, depth: int = 1, std: float = 0.02) -> None:
        out_std = std / math.sqrt(2.0 * max(1, depth))
        init_norm(self.attention_norm)
        init_norm(self.ffn_norm)
        self.attention.init_weights(std=std, out_std=out_std)
        self.feed_forward.init_weights(std=std, out_std=out_std)
        if self.cross_attention is not None and self.cross_norm is not None:
            init_norm(self.cross_norm)
            self.cross_attention.init_weights(std=std)
        nn.init.zeros_(self.scale_shift_table)


class TextRefinerBlock(nn.Module):
    """Un-modulated pre-norm transformer block over the text tokens."""

    def __init__(self, width: int, num_heads: int, *, hidden: int, qk_norm: bool = True, eps: float = 1e-6) -> None:
        super().__init__()
        self.attention_norm = rms_norm(width, eps=eps)
        self.attention = SelfAttention(width, num_heads, qk_norm=qk_norm, eps=eps)
        self.ffn_norm = rms_norm(width, eps=eps)
        self.feed_forward = SwiGLU(width, hidden)

    def forward(self, hidden: torch.Tensor, *, key_mask: torch.Tensor | None = None) -> torch.Tensor:
        hidden = hidden + self.attention(self.attention_norm(hidden), None, key_mask=key_mask)
        return hidden + self.feed_forward(self.ffn_norm(hidden))

    def init_weights(self, *, depth: int = 1, std: float = 0.02) -> None:
        out_std = std / math.sqrt(2.0 * max(1, depth))
        init_norm(self.attention_norm)
        init_norm(self.ffn_norm)
        self.attention.init_weights(std=std, out_std=out_std)
        self.feed_forward.init_weights(std=std, out_std=out_std)


class CrossModalFusion(nn.Module):
    """Bidirectional video<->audio cross-attention with temporal-window masks."""

    def __init__(self, video_width: int, audio_width: int, *, video_heads: int, audio_heads: int,
                 qk_norm: bool = True, eps: float = 1e-6) -> None:
        super().__init__()
        self.video_norm = rms_norm(video_width, eps=eps)
        self.video_from_audio = CrossAttention(video_width, video_heads, context_width=audio_width, qk_norm=qk_norm,
                                               eps=eps)
        self.audio_norm = rms_norm(audio_width, eps=eps)
        self.audio_from_video = CrossAttention(audio_width, audio_heads, context_width=video_width, qk_norm=qk_norm,
                                               eps=eps)

    def forward(self, video: torch.Tensor, audio: torch.Tensor, *, video_to_audio: torch.Tensor | None = None,
                audio_to_video: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        v_upd = _masked_cross(self.video_from_audio, self.video_norm(video), audio, video_to_audio)
        a_upd = _masked_cross(self.audio_from_video, self.audio_norm(audio), video, audio_to_video)
        return video + v_upd, audio + a_upd

    def init_weights(self, *, std: float = 0.02) -> None:
        init_norm(self.video_norm)
        init_norm(self.audio_norm)
        self.video_from_audio.init_weights(std=std)
        self.audio_from_video.init_weights(std=std)


def _masked_cross(module: CrossAttention, hidden: torch.Tensor, context: torch.Tensor,
                  mask: torch.Tensor | None) -> torch.Tensor:
    """Cross-attention with an optional dense ``(B, 1, Lq, Lk)`` mask (fusion windows)."""
    if mask is None or mask.ndim == 2:
        return module(hidden, context, mask)
    from avgen_b200.models.linear import linear

    q = module.q_norm(module._heads(linear(hidden, module.q_proj)))
    k = module.k_norm(module._heads(linear(context, module.k_proj)))
    v = module._heads(linear(context, module.v_proj))
    rep = q.shape[1] // k.shape[1]
    if rep > 1:
        k = k.repeat_interleave(rep, 1)
        v = v.repeat_interleave(rep, 1)
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    s = s.masked_fill(~mask, float("-inf"))
    out = torch.softmax(s, -1) @ v.float()
    return linear(out.to(hidden.dtype).transpose(1, 2).flatten(2), module.out_proj)
