"""Control and image-prompt adapters (avgen/finetune/adapters.py:176-660 API).

* :class:`ControlAdapter` (ControlNet-style): a control latent grid is
  patchified and embedded, passed through trainable copies of the first
  ``num_blocks`` blocks of the frozen base, and each copy's output is added to
  the matching base block's output through a zero-initialised linear (so
  training starts from the base model exactly). Injection is by forward hooks.
* :class:`IPAdapter`: image-embedding tokens get their own key/value
  projections in every targeted cross-attention (decoupled cross-attention);
  the extra attention output, scaled, is added to the block's cross-attention
  output. The new output projections start at zero.
"""
from __future__ import annotations

import copy
import math
from collections.abc import Sequence
from dataclasses import dataclass
from types import TracebackType
from typing import Any

import torch
from torch import nn
from torch.utils.hooks import RemovableHandle


def _is_block_list(blocks: object) -> bool:
    from avgen_b200.parallel.pipeline import is_block_list

    return is_block_list(blocks)


__all__ = ["AdapterHandles", "ControlAdapter", "ControlAdapterConfig", "IPAdapter", "IPAdapterConfig"]


class _Restore:
    """Re-enables a block's fused path when an adapter that needed the module path detaches."""

    def __init__(self, block: nn.Module) -> None:
        self.block = block

    def remove(self) -> None:
        self.block.use_fused = True


class AdapterHandles:
    """Forward hooks of an attached adapter; ``remove()`` (or leaving the ``with``) detaches them."""

    def __init__(self, handles: Sequence[RemovableHandle | _Restore]) -> None:
        self._handles = list(handles)

    def __len__(self) -> int:
        return len(self._handles)

    def remove(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()

    def __enter__(self) -> AdapterHandles:
        return self

    def __exit__(self, exc_type: type[BaseException] | None, exc: BaseException | None,
                 tb: TracebackType | None) -> None:
        self.remove()


def _blocks(model: nn.Module, attribute: str) -> nn.ModuleList:
    blocks = getattr(model, attribute, None)
    if not _is_block_list(blocks) or not len(blocks):
        raise AttributeError(f"{type(model).__name__} has no non-empty nn.ModuleList {attribute!r}")
    return blocks


def _zero_linear(i: int, o: int) -> nn.Linear:
    lin = nn.Linear(i, o)
    nn.init.zeros_(lin.weight)
    nn.init.zeros_(lin.bias)
    return lin


@dataclass(frozen=True, slots=True)
class ControlAdapterConfig:
    control_width: int
    num_blocks: int = 6
    model_width: int | None = None
    block_attribute: str = "blocks"
    conditioning_scale: float = 1.0
    injection_stride: int = 1

    def __post_init__(self) -> None:
        if self.control_width < 1 or self.num_blocks < 1 or self.injection_stride < 1:
            raise ValueError("control_width, num_blocks and injection_stride must be positive")
        if not math.isfinite(self.conditioning_scale):
            raise ValueError("conditioning_scale must be finite")


class ControlAdapter(nn.Module):
    """Trainable copies of the first blocks, fed by an embedded control signal."""

    def __init__(self, base: nn.Module, config: ControlAdapterConfig) -> None:
        super().__init__()
        blocks = _blocks(base, config.block_attribute)
        n = min(config.num_blocks, len(blocks))
        width = config.model_width or getattr(getattr(base, "config", None), "width", None) or \
            blocks[0].attention_norm.normalized_shape[0]
        self.config = config
        self.copies = nn.ModuleList(copy.deepcopy(blocks[i]) for i in range(n))
        for blk in self.copies:
            if hasattr(blk, "use_fused"):
                blk.use_fused = True
            for p in blk.parameters():
                p.requires_grad_(True)
        self.control_in = _zero_linear(config.control_width, width)
        nn.init.normal_(self.control_in.weight, std=0.02)
        self.injections = nn.ModuleList(_zero_linear(width, width) for _ in range(n))

    def forward(self, hidden: torch.Tensor, control: torch.Tensor, *block_args: Any,
                **block_kwargs: Any) -> list[torch.Tensor]:
        """Residuals (one per copied block) for the base blocks 0, stride, 2*stride, ..."""
        h = hidden + self.control_in(control.to(self.control_in.weight.dtype)).to(hidden.dtype)
        outs = []
        for blk, inj in zip(self.copies, self.injections):
            h = blk(h, *block_args, **block_kwargs)
            outs.append(inj(h.to(inj.weight.dtype)).to(hidden.dtype) * self.config.conditioning_scale)
        return outs

    def attach(self, base: nn.Module, control: torch.Tensor) -> AdapterHandles:
        """Hook the base blocks: block 0's input also runs the copies; block ``k * stride`` gets residual k."""
        blocks = _blocks(base, self.config.block_attribute)
        state: dict[str, list[torch.Tensor]] = {}
        handles: list[RemovableHandle] = []

        def pre(_m: nn.Module, args: tuple[Any, ...], kwargs: dict[str, Any]) -> None:
            state["res"] = self(args[0], control, *args[1:], **kwargs)

        handles.append(blocks[0].register_forward_pre_hook(pre, with_kwargs=True))
        for k in range(len(self.copies)):
            idx = k * self.config.injection_stride
            if idx >= len(blocks):
                break

            def post(_m: nn.Module, _a: Any, out: torch.Tensor, k: int = k) -> torch.Tensor:
                return out + state["res"][k]

            handles.append(blocks[idx].register_forward_hook(post))
        return AdapterHandles(handles)


@dataclass(frozen=True, slots=True)
class IPAdapterConfig:
    image_width: int
    num_tokens: int = 4
    scale: float = 1.0
    target_blocks: tuple[str, ...] = ()
    num_heads: int | None = None
    attention_attribute: str = "cross_attention"

    def __post_init__(self) -> None:
        if self.image_width < 1 or self.num_tokens < 1:
            raise ValueError("image_width and num_tokens must be positive")


class IPAdapter(nn.Module):
    """Decoupled cross-attention over image-prompt tokens."""

    def __init__(self, base: nn.Module, config: IPAdapterConfig) -> None:
        super().__init__()
        self.config = config
        targets = self._targets(base)
        if not targets:
            raise ValueError(f"no {config.attention_attribute!r} modules to adapt")
        att0 = targets[0][1]
        width = att0.q_proj.in_features
        self.heads = config.num_heads or att0.num_heads
        self.head_dim = att0.q_proj.out_features // att0.num_heads
        inner = self.heads * self.head_dim
        self.names = [n for n, _ in targets]
        self.image_proj = nn.Linear(config.image_width, config.num_tokens * width)
        self.image_norm = nn.LayerNorm(width)
        self.to_k = nn.ModuleList(nn.Linear(width, inner, bias=False) for _ in targets)
        self.to_v = nn.ModuleList(nn.Linear(width, inner, bias=False) for _ in targets)
        self.to_out = nn.ModuleList(_zero_linear(inner, width) for _ in targets)

    def _targets(self, base: nn.Module) -> list[tuple[str, nn.Module]]:
        out = []
        for name, m in base.named_modules():
            if name.endswith(self.config.attention_attribute) and hasattr(m, "q_proj"):
                if not self.config.target_blocks or any(t in name for t in self.config.target_blocks):
                    out.append((name, m))
        return out

    def image_tokens(self, image_embedding: torch.Tensor) -> torch.Tensor:
        b = image_embedding.shape[0]
        t = self.image_proj(image_embedding.to(self.image_proj.weight.dtype))
        return self.image_norm(t.view(b, self.config.num_tokens, -1))

    def _branch(self, i: int, attention: nn.Module, hidden: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
        b, n, _ = hidden.shape
        q = attention.q_proj(hidden.to(attention.q_proj.weight.dtype)).view(b, n, -1, self.head_dim).transpose(1, 2)
        k = self.to_k[i](tokens).view(b, -1, self.heads, self.head_dim).transpose(1, 2)
        v = self.to_v[i](tokens).view(b, -1, self.heads, self.head_dim).transpose(1, 2)
        if q.shape[1] != self.heads:
            q = q[:, : self.heads]
        o = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
        return self.to_out[i](o.transpose(1, 2).reshape(b, n, -1)) * self.config.scale

    def attach(self, base: nn.Module, image_embedding: torch.Tensor) -> AdapterHandles:
        tokens = self.image_tokens(image_embedding)
        modules = dict(base.named_modules())
        handles: list[Any] = []
        for i, name in enumerate(self.names):
            att = modules[name]
            owner = modules.get(name.rpartition(".")[0])
            if getattr(owner, "use_fused", False):  # the fused block computes cross-attention inline
                owner.use_fused = False
                handles.append(_Restore(owner))

            def post(m: nn.Module, args: tuple[Any, ...], out: torch.Tensor, i: int = i) -> torch.Tensor:
                return out + self._branch(i, m, args[0], tokens.to(out.device)).to(out.dtype)

            handles.append(att.register_forward_hook(post))
        return AdapterHandles(handles)
