"""VideoDiT and AVDiT, the registered flagship models (avgen/models/dit.py:96-1146).

Root modules (names are the checkpoint contract): ``patch_embed``,
``time_embed``, ``text_proj``, ``text_refiner``, ``modulation``, ``blocks``,
``final_norm``, ``final_proj`` (zero-initialised). Conditioning is adaLN-single:
one shared ``modulation`` MLP plus each block's zero-initialised
``scale_shift_table``. ``ffn`` selects SwiGLU (reference default, names
gate/up/down_proj) or a GELU(tanh) MLP (names up/down_proj).

On CUDA every block runs as one fused node over the sm_100a kernels, and the
root linears run the tcgen05 GEMM; on the CPU everything is the fp32 oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, fields, replace
from typing import TYPE_CHECKING, Any

import torch
import torch.nn.functional as F
from torch import nn

from avgen_b200.core.limits import Limit, enforce
from avgen_b200.core.model_input import ModelInput, ModelOutput
from avgen_b200.core.patchify import GridPatchifier, Patchifier
from avgen_b200.core.tokens import TextContext, TokenStream
from avgen_b200.models.attention import key_padding_mask
from avgen_b200.models.blocks import CrossModalFusion, DiTBlock, RopeInputs, TextRefinerBlock, temporal_neighbour_mask
from avgen_b200.models.layers import AdaLNModulation, TimestepEmbedding, init_linear, init_norm, match_dtype, rms_norm
from avgen_b200.models.linear import linear
from avgen_b200.models.registry import register_model
from avgen_b200.models.rope import RoPEScaling, RotaryEmbedding

if TYPE_CHECKING:
    from avgen_b200.simulate.memory import ModelShape

__all__ = ["FUSION_MODES", "AVDiT", "AVDiTConfig", "VideoDiT", "VideoDiTConfig", "list_presets", "preset"]

FUSION_MODES = ("cross_attention", "joint")
FFN_KINDS = ("swiglu", "gelu")


_COUNT = Limit(lo=1, integer=True)
_VIDEO_LIMITS = {**{name: _COUNT for name in ("width", "depth", "num_heads", "ffn_multiple_of", "in_channels",
                                              "patch_frames", "patch_height", "patch_width", "text_width",
                                              "time_frequency_dim")},
                 "num_kv_heads": Limit(lo=1, integer=True, optional=True), "mlp_ratio": Limit(lo=0.0, lo_open=True),
                 "ffn_hidden": Limit(lo=1, integer=True, optional=True), "text_refiner_depth": Limit(lo=0, integer=True)}
_AUDIO_LIMITS = {name: _COUNT for name in ("audio_width", "audio_num_heads", "audio_in_channels", "audio_patch_frames",
                                           "fusion_interval")}


def _check_heads(prefix: str, width: int, heads: int) -> None:
    """Heads split the width evenly into even (rotary pairs) head dims of at least 6
    (two pairs for time, one for each spatial axis at the least)."""
    if width % heads:
        raise ValueError(f"{prefix}width={width} must be divisible by {prefix}num_heads={heads}")
    dim = width // heads
    if dim % 2 or dim < 6:
        raise ValueError(f"{prefix}head_dim={dim} must be even and at least 6")


def _ffn_width(explicit: int | None, ratio: float, width: int, multiple: int) -> int:
    """``explicit``, else ``ratio * width`` rounded up to a multiple of ``multiple``."""
    if explicit is not None:
        return explicit
    return math.ceil(int(ratio * width) / multiple) * multiple


@dataclass(frozen=True, slots=True)
class VideoDiTConfig:
    width: int = 768
    depth: int = 24
    num_heads: int = 12
    num_kv_heads: int | None = None
    mlp_ratio: float = 4.0
    ffn_hidden: int | None = None
    ffn_multiple_of: int = 256
    ffn: str = "swiglu"
    in_channels: int = 16
    out_channels: int | None = None
    patch_frames: int = 1
    patch_height: int = 2
    patch_width: int = 2
    normalize_space: bool = False
    text_width: int = 4096
    text_context_length: int = 0
    text_refiner_depth: int = 0
    cross_attention: bool = True
    rope_theta: float = 10000.0
    rope_time_scale: float = 1.0
    rope_scaling: RoPEScaling = field(default_factory=RoPEScaling)
    cond_width: int | None = None
    time_frequency_dim: int = 256
    qk_norm: bool = True
    norm_eps: float = 1e-6
    assume_dense_mask: bool = False
    init_std: float = 0.02

    def __post_init__(self) -> None:
        if not isinstance(self.rope_scaling, RoPEScaling):
            raise TypeError("rope_scaling must be a RoPEScaling")
        enforce(self, _VIDEO_LIMITS)
        _check_heads("", self.width, self.num_heads)
        if self.num_kv_heads is not None and self.num_heads % self.num_kv_heads:
            raise ValueError(f"num_kv_heads={self.num_kv_heads} must divide num_heads={self.num_heads}")
        if self.ffn not in FFN_KINDS:
            raise ValueError(f"ffn must be one of {FFN_KINDS}; got {self.ffn!r}")
        if self.text_refiner_depth and not self.cross_attention:
            raise ValueError("text_refiner_depth > 0 needs cross_attention")

    @property
    def head_dim(self) -> int:
        return self.width // self.num_heads

    @property
    def ffn_width(self) -> int:
        return _ffn_width(self.ffn_hidden, self.mlp_ratio, self.width, self.ffn_multiple_of)

    @property
    def cond_dim(self) -> int:
        return self.cond_width if self.cond_width is not None else self.width

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.patch_frames * self.patch_height * self.patch_width

    @property
    def out_patch_dim(self) -> int:
        c = self.out_channels if self.out_channels is not None else self.in_channels
        return c * self.patch_frames * self.patch_height * self.patch_width


@register_model("video_dit")
class VideoDiT(nn.Module):
    def __init__(self, config: VideoDiTConfig) -> None:
        super().__init__()
        self.config = config
        self._patchifier = GridPatchifier(patch_frames=config.patch_frames, patch_height=config.patch_height,
                                          patch_width=config.patch_width, normalize_space=config.normalize_space)
        self.rope = RotaryEmbedding(config.head_dim, theta=config.rope_theta, time_scale=config.rope_time_scale,
                                    scaling=config.rope_scaling)
        self.patch_embed = nn.Linear(config.patch_dim, config.width, bias=True)
        self.time_embed = TimestepEmbedding(config.cond_dim, frequency_dim=config.time_frequency_dim)
        self.text_proj = nn.Linear(config.text_width, config.width, bias=True)
        self.text_refiner = nn.ModuleList(
            TextRefinerBlock(config.width, config.num_heads, hidden=config.ffn_width, qk_norm=config.qk_norm,
                             eps=config.norm_eps) for _ in range(config.text_refiner_depth))
        self.modulation = AdaLNModulation(config.cond_dim, config.width)
        self.blocks = nn.ModuleList(
            DiTBlock(config.width, config.num_heads, hidden=config.ffn_width, num_kv_heads=config.num_kv_heads,
                     cross_attention=config.cross_attention, qk_norm=config.qk_norm, eps=config.norm_eps,
                     ffn=config.ffn) for _ in range(config.depth))
        self.final_norm = rms_norm(config.width, eps=config.norm_eps)
        self.final_proj = nn.Linear(config.width, config.out_patch_dim, bias=True)

    @property
    def patchifier(self) -> Patchifier:
        return self._patchifier

    def parameter_count(self) -> int:
        return int(sum(p.numel() for p in self.parameters()))

    def model_shape(self, *, sequence_length: int, micro_batch_size: int = 1) -> ModelShape:
        """Analytic shape for the simulator."""
        from avgen_b200.simulate.memory import ModelShape

        c = self.config
        return ModelShape(parameters=self.parameter_count(), depth=c.depth, width=c.width,
                          sequence_length=sequence_length, micro_batch_size=micro_batch_size,
                          mlp_ratio=max(1, round(c.ffn_width / c.width)), num_heads=c.num_heads,
                          text_tokens=c.text_context_length if c.cross_attention else 0,
                          ffn_hidden=c.ffn_width, ffn=c.ffn)

    def init_weights(self) -> None:
        c = self.config
        init_linear(self.patch_embed, std=c.init_std)
        self.time_embed.init_weights()
        init_linear(self.text_proj, std=c.init_std)
        for refiner in self.text_refiner:
            refiner.init_weights(depth=max(1, c.text_refiner_depth), std=c.init_std)
        self.modulation.init_weights()
        for block in self.blocks:
            block.init_weights(depth=c.depth, std=c.init_std)
        init_norm(self.final_norm)
        init_linear(self.final_proj, zero=True)

    # ------------------------------------------------------------------ pieces
    def _compute_dtype(self, device: torch.device) -> torch.dtype:
        return torch.bfloat16 if device.type == "cuda" else self.patch_embed.weight.dtype

    def encode_text(self, text: TextContext) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        if text.is_empty or not self.config.cross_attention:
            return None, None
        feats = linear(match_dtype(text.features, self.text_proj), self.text_proj)
        mask = key_padding_mask(text.mask, assume_dense=self.config.assume_dense_mask)
        for refiner in self.text_refiner:
            feats = refiner(feats, key_mask=mask)
        return feats, mask

    def _stream_conditioning(self, stream: TokenStream, *, embed: TimestepEmbedding,
                             modulation: AdaLNModulation) -> tuple[torch.Tensor, torch.Tensor | None]:
        """adaLN modulation rows of a stream and the per-token row index.

        Per-sample levels give ``(B, 6, W)`` and no index. Grouped per-token levels
        (``level_values`` / ``level_index``) give one row per distinct level,
        ``(B*G, 6, W)``, and the ``(B, L)`` row of every token; plain per-token
        levels give one row per token. The reference computes the per-token form
        ``(B, L, 6, W)`` (avgen/models/dit.py:330-352); the rows are identical.
        """
        if stream.has_level_groups:
            b, g = stream.level_values.shape
            rows = modulation(embed(stream.level_values.reshape(-1)))
            base = torch.arange(b, device=stream.level_index.device, dtype=torch.int32)[:, None] * g
            return rows, stream.level_index + base
        if stream.per_token_noise:
            b, length = stream.noise_level.shape
            rows = modulation(embed(stream.noise_level.reshape(-1)))
            index = torch.arange(b * length, device=rows.device, dtype=torch.int32).view(b, length)
            return rows, index
        return modulation(embed(stream.noise_level)), None

    def _global_mask(self, mask: torch.Tensor) -> torch.Tensor:
        """Key validity over the whole sequence (gathered across context-parallel shards)."""
        mesh = getattr(self, "cp_mesh", None)
        if mesh is None or mesh.size() == 1:
            return mask
        from avgen_b200.parallel.context import gather_tokens

        return gather_tokens(mask, mesh)

    def _rope_inputs(self, coords: torch.Tensor, rope: RotaryEmbedding | None = None) -> RopeInputs:
        return RopeInputs(coords=coords.float().contiguous(), rope=rope or self.rope)

    def _denoise(self, hidden: torch.Tensor, *, modulation: torch.Tensor, rope: RopeInputs | None,
                 key_mask: torch.Tensor | None, context: torch.Tensor | None,
                 context_mask: torch.Tensor | None, modulation_index: torch.Tensor | None = None,
                 blocks: Any = None) -> torch.Tensor:
        """The block stack (or ``blocks``, a subset of it: an interleaved pipeline's chunk)."""
        tp = getattr(self, "head_parallel", None)
        sequence = tp is not None and tp.sequence_parallel
        if sequence:  # the residual stream between blocks holds this rank's tokens only
            length = hidden.shape[1]
            hidden = tp.local_tokens(hidden)
            modulation = tp.shared(modulation)
            if modulation_index is not None:
                modulation_index = modulation_index[:, tp.token_slice(length)]
            elif modulation.ndim == 4:
                modulation = modulation[:, tp.token_slice(length)]
        for block in (self.blocks if blocks is None else blocks):
            hidden = block(hidden, modulation=modulation, rope=rope, key_mask=key_mask, context=context,
                           context_mask=context_mask, modulation_index=modulation_index)
        return tp.all_tokens(hidden) if sequence else hidden

    def _video_head(self, hidden: torch.Tensor, stream: TokenStream) -> torch.Tensor:
        normed = self.final_norm(hidden)
        predicted = linear(normed, self.final_proj)
        return predicted * stream.mask.unsqueeze(-1).to(predicted.dtype)

    def _null_audio(self, inputs: ModelInput, like: torch.Tensor) -> torch.Tensor:
        a = inputs.audio
        return torch.zeros((a.batch_size, a.length, a.layout.patch_dim), dtype=like.dtype, device=like.device)

    def forward(self, inputs: ModelInput, *, stage: str | None = None, hidden: torch.Tensor | None = None,
                carry: tuple[Any, ...] | None = None, aux: dict[str, Any] | None = None) -> Any:
        """The whole model, or one pipeline part through the module call so that hooks on
        the root module (FSDP2's lazy initialisation and parameter gathering among them)
        run for it: ``stage="embed"`` is ``stage_embed(inputs)``, ``stage="blocks"`` is
        ``stage_blocks(*carry, aux)``, ``stage="head"`` is ``stage_head(hidden, inputs)``."""
        if stage == "embed":
            return self.stage_embed(inputs)
        if stage == "blocks":
            assert carry is not None and aux is not None, "the blocks stage takes the carry and its inputs"
            return self.stage_blocks(*carry, aux)
        if stage == "head":
            assert hidden is not None, "the head stage takes the blocks' output"
            return self.stage_head(hidden, inputs)
        if stage is not None:
            raise ValueError(f"stage must be None, 'embed', 'blocks' or 'head'; got {stage!r}")
        hidden, context, modulation = self.stage_embed(inputs)
        hidden = self.stage_blocks(hidden, context, modulation, self.stage_inputs(inputs))
        return self.stage_head(hidden, inputs)

    # ------------------------------------------------------------------ pipeline stages
    # The forward in three parts so a pipeline stage runs only what it owns: the first
    # stage embeds (patches, text, modulation rows), every stage runs its blocks, the
    # last stage projects to the output. ``stage_inputs`` holds what every stage can
    # rebuild from the model input without parameters (RoPE coordinates, key masks,
    # each token's modulation row).
    def stage_inputs(self, inputs: ModelInput) -> dict[str, Any]:
        video, text = inputs.video, inputs.text
        context_mask = None
        if not text.is_empty and self.config.cross_attention:
            context_mask = key_padding_mask(text.mask, assume_dense=self.config.assume_dense_mask)
        return {"rope": self._rope_inputs(video.coords), "context_mask": context_mask,
                "key_mask": key_padding_mask(self._global_mask(video.mask), assume_dense=self.config.assume_dense_mask),
                "modulation_index": _modulation_index(video)}

    def stage_embed(self, inputs: ModelInput) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor]:
        """(hidden, text context or None, modulation rows): the tensors later stages receive."""
        video = inputs.video
        context, _ = self.encode_text(inputs.text)
        tokens = video.masked()
        if tokens.device.type == "cuda":
            tokens = tokens.to(torch.bfloat16)
        hidden = linear(match_dtype(tokens, self.patch_embed), self.patch_embed)
        modulation, _ = self._stream_conditioning(video, embed=self.time_embed, modulation=self.modulation)
        return hidden, context, modulation

    def stage_blocks(self, hidden: torch.Tensor, context: torch.Tensor | None, modulation: torch.Tensor,
                     aux: dict[str, Any]) -> torch.Tensor:
        return self._denoise(hidden, modulation=modulation, rope=aux["rope"], key_mask=aux["key_mask"],
                             context=context, context_mask=aux["context_mask"],
                             modulation_index=aux["modulation_index"], blocks=aux.get("blocks"))

    def stage_head(self, hidden: torch.Tensor, inputs: ModelInput) -> ModelOutput:
        predicted = self._video_head(hidden, inputs.video)
        return ModelOutput(video=predicted, audio=self._null_audio(inputs, predicted))

    def tensor_parallel_plan(self, *, sequence_parallel: bool) -> tuple[dict[str, Any], dict[str, Any]]:
        from avgen_b200.parallel.tensor import standard_block_plan, standard_root_plan

        block = standard_block_plan(sequence_parallel=sequence_parallel,
                                    cross_attention_prefix="cross_attention" if self.config.cross_attention else None,
                                    ffn_projections=("gate_proj", "up_proj") if self.config.ffn == "swiglu"
                                    else ("up_proj",))
        return standard_root_plan(sequence_parallel=sequence_parallel), block


@dataclass(frozen=True, slots=True)
class AVDiTConfig(VideoDiTConfig):
    audio_width: int = 512
    audio_num_heads: int = 8
    audio_in_channels: int = 8
    audio_out_channels: int | None = None
    audio_patch_frames: int = 1
    audio_ffn_hidden: int | None = None
    audio_rope_time_scale: float | None = None
    fusion: str = "cross_attention"
    fusion_interval: int = 2
    fusion_window_seconds: float = 0.25

    def __post_init__(self) -> None:
        VideoDiTConfig.__post_init__(self)
        enforce(self, _AUDIO_LIMITS)
        if self.fusion not in FUSION_MODES:
            raise ValueError(f"fusion must be one of {FUSION_MODES}; got {self.fusion!r}")
        _check_heads("audio_", self.audio_width, self.audio_num_heads)

    @property
    def audio_head_dim(self) -> int:
        return self.audio_width // self.audio_num_heads

    @property
    def audio_ffn_width(self) -> int:
        # the rounding multiple never exceeds the tower's own width (narrow audio towers)
        return _ffn_width(self.audio_ffn_hidden, self.mlp_ratio, self.audio_width,
                          min(self.ffn_multiple_of, self.audio_width))

    @property
    def audio_patch_dim(self) -> int:
        return self.audio_in_channels * self.audio_patch_frames

    @property
    def audio_out_patch_dim(self) -> int:
        c = self.audio_out_channels if self.audio_out_channels is not None else self.audio_in_channels
        return c * self.audio_patch_frames

    @property
    def audio_cond_dim(self) -> int:
        return self.width if self.fusion == "joint" else self.audio_width

    @property
    def fusion_points(self) -> tuple[int, ...]:
        if self.fusion != "cross_attention":
            return ()
        return tuple(i for i in range(self.depth) if (i + 1) % self.fusion_interval == 0)


@register_model("av_dit")
class AVDiT(VideoDiT):
    """Audio-video DiT: joint sequence or two towers with periodic fusion."""

    def __init__(self, config: AVDiTConfig) -> None:
        super().__init__(config)
        self.config: AVDiTConfig = config
        self._audio_patchifier = GridPatchifier(patch_frames=config.audio_patch_frames, patch_height=1, patch_width=1)
        self.audio_patch_embed = nn.Linear(config.audio_patch_dim, config.audio_width, bias=True)
        self.audio_time_embed = TimestepEmbedding(config.audio_cond_dim, frequency_dim=config.time_frequency_dim)
        self.audio_final_norm = rms_norm(config.audio_width, eps=config.norm_eps)
        self.audio_final_proj = nn.Linear(config.audio_width, config.audio_out_patch_dim, bias=True)
        if config.fusion == "joint":
            self.audio_in_proj: nn.Module = nn.Linear(config.audio_width, config.width, bias=True)
            self.audio_out_proj: nn.Module = nn.Linear(config.width, config.audio_width, bias=True)
            self.audio_modulation = AdaLNModulation(config.audio_cond_dim, config.width)
            self.audio_blocks = nn.ModuleList()
            self.fusion_blocks = nn.ModuleList()
            self.audio_text_proj: nn.Module = nn.Identity()
            self.audio_rope: nn.Module = nn.Identity()
        else:
            self.audio_in_proj = nn.Identity()
            self.audio_out_proj = nn.Identity()
            self.audio_modulation = AdaLNModulation(config.audio_cond_dim, config.audio_width)
            self.audio_blocks = nn.ModuleList(
                DiTBlock(config.audio_width, config.audio_num_heads, hidden=config.audio_ffn_width,
                         num_kv_heads=config.num_kv_heads, cross_attention=config.cross_attention,
                         qk_norm=config.qk_norm, eps=config.norm_eps, ffn=config.ffn) for _ in range(config.depth))
            self.fusion_blocks = nn.ModuleList(
                CrossModalFusion(config.width, config.audio_width, video_heads=config.num_heads,
                                 audio_heads=config.audio_num_heads, qk_norm=config.qk_norm, eps=config.norm_eps)
                for _ in config.fusion_points)
            self.audio_text_proj = nn.Linear(config.text_width, config.audio_width, bias=True)
            self.audio_rope = RotaryEmbedding(
                config.audio_head_dim, theta=config.rope_theta,
                time_scale=config.audio_rope_time_scale if config.audio_rope_time_scale is not None
                else config.rope_time_scale, scaling=config.rope_scaling)

    @property
    def audio_patchifier(self) -> Patchifier:
        return self._audio_patchifier

    def init_weights(self) -> None:
        super().init_weights()
        c = self.config
        init_linear(self.audio_patch_embed, std=c.init_std)
        self.audio_time_embed.init_weights()
        self.audio_modulation.init_weights()
        init_norm(self.audio_final_norm)
        init_linear(self.audio_final_proj, zero=True)
        for block in self.audio_blocks:
            block.init_weights(depth=c.depth, std=c.init_std)
        for fusion in self.fusion_blocks:
            fusion.init_weights(std=c.init_std)
        for mod in (self.audio_in_proj, self.audio_out_proj, self.audio_text_proj):
            if isinstance(mod, nn.Linear):
                init_linear(mod, std=c.init_std)

    def _audio_context(self, text: TextContext) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        if text.is_empty or not self.config.cross_attention or not isinstance(self.audio_text_proj, nn.Linear):
            return None, None
        mask = key_padding_mask(text.mask, assume_dense=self.config.assume_dense_mask)
        return linear(match_dtype(text.features, self.audio_text_proj), self.audio_text_proj), mask

    def _embed(self, stream: TokenStream, layer: nn.Linear) -> torch.Tensor:
        tokens = stream.masked()
        if tokens.device.type == "cuda":
            tokens = tokens.to(torch.bfloat16)
        return linear(match_dtype(tokens, layer), layer)

    def _forward_joint(self, inputs: ModelInput) -> ModelOutput:
        video, audio = inputs.video, inputs.audio
        context, context_mask = self.encode_text(inputs.text)
        hidden = torch.cat((self._embed(video, self.patch_embed),
                            linear(self._embed(audio, self.audio_patch_embed), self.audio_in_proj)), 1)
        vrows, vidx = self._stream_conditioning(video, embed=self.time_embed, modulation=self.modulation)
        arows, aidx = self._stream_conditioning(audio, embed=self.audio_time_embed, modulation=self.audio_modulation)
        vidx = _row_index(vrows, vidx, video.batch_size, video.length)
        aidx = _row_index(arows, aidx, audio.batch_size, audio.length)
        modulation = torch.cat((vrows, arows), 0)
        mod_index = torch.cat((vidx, aidx + vrows.shape[0]), 1)
        rope = self._rope_inputs(torch.cat((video.coords, audio.coords), 1))
        key_mask = key_padding_mask(torch.cat((video.mask, audio.mask), 1), assume_dense=self.config.assume_dense_mask)
        hidden = self._denoise(hidden, modulation=modulation, rope=rope, key_mask=key_mask, context=context,
                               context_mask=context_mask, modulation_index=mod_index)
        vh, ah = hidden.split((video.length, audio.length), 1)
        pa = linear(self.audio_final_norm(linear(ah, self.audio_out_proj)), self.audio_final_proj)
        pa = pa * audio.mask.unsqueeze(-1).to(pa.dtype)
        return ModelOutput(video=self._video_head(vh, video), audio=pa)

    def _forward_two_tower(self, inputs: ModelInput) -> ModelOutput:
        c = self.config
        video, audio = inputs.video, inputs.audio
        context, context_mask = self.encode_text(inputs.text)
        actx, actx_mask = self._audio_context(inputs.text)
        vh = self._embed(video, self.patch_embed)
        ah = self._embed(audio, self.audio_patch_embed)
        vmod, vidx = self._stream_conditioning(video, embed=self.time_embed, modulation=self.modulation)
        amod, aidx = self._stream_conditioning(audio, embed=self.audio_time_embed, modulation=self.audio_modulation)
        vrope = self._rope_inputs(video.coords)
        arope = self._rope_inputs(audio.coords, self.audio_rope)
        vkm = key_padding_mask(video.mask, assume_dense=c.assume_dense_mask)
        akm = key_padding_mask(audio.mask, assume_dense=c.assume_dense_mask)
        v2a = temporal_neighbour_mask(video.coords[..., 0], audio.coords[..., 0], window_seconds=c.fusion_window_seconds,
                                      key_mask=audio.mask)
        a2v = temporal_neighbour_mask(audio.coords[..., 0], video.coords[..., 0], window_seconds=c.fusion_window_seconds,
                                      key_mask=video.mask)
        fusion_at = {p: i for i, p in enumerate(c.fusion_points)}
        for i in range(c.depth):
            vh = self.blocks[i](vh, modulation=vmod, rope=vrope, key_mask=vkm, context=context, context_mask=context_mask,
                                modulation_index=vidx)
            ah = self.audio_blocks[i](ah, modulation=amod, rope=arope, key_mask=akm, context=actx,
                                      context_mask=actx_mask, modulation_index=aidx)
            fi = fusion_at.get(i)
            if fi is not None:
                vh, ah = self.fusion_blocks[fi](vh, ah, video_to_audio=v2a, audio_to_video=a2v)
        pa = linear(self.audio_final_norm(ah), self.audio_final_proj)
        pa = pa * audio.mask.unsqueeze(-1).to(pa.dtype)
        return ModelOutput(video=self._video_head(vh, video), audio=pa)

    def forward(self, inputs: ModelInput) -> ModelOutput:
        if not inputs.has_audio:
            return super().forward(inputs)
        if self.config.fusion == "joint":
            return self._forward_joint(inputs)
        return self._forward_two_tower(inputs)


def _modulation_index(stream: TokenStream) -> torch.Tensor | None:
    """Each token's row in the modulation rows ``_stream_conditioning`` builds (None: one row per sample)."""
    if stream.has_level_groups:
        b, g = stream.level_values.shape
        base = torch.arange(b, device=stream.level_index.device, dtype=torch.int32)[:, None] * g
        return stream.level_index + base
    if stream.per_token_noise:
        b, length = stream.noise_level.shape
        return torch.arange(b * length, device=stream.noise_level.device, dtype=torch.int32).view(b, length)
    return None


def _row_index(rows: torch.Tensor, index: torch.Tensor | None, batch: int, length: int) -> torch.Tensor:
    """Per-token modulation row numbers; per-sample rows become ``b`` for every token of sample ``b``."""
    if index is not None:
        return index
    return torch.arange(batch, device=rows.device, dtype=torch.int32)[:, None].expand(batch, length)


# Identity module in AVDiT joint mode goes through `linear` only for nn.Linear.
def _linear_or_identity(x: torch.Tensor, module: nn.Module) -> torch.Tensor:
    return linear(x, module) if isinstance(module, nn.Linear) else module(x)


_PRESETS: dict[str, VideoDiTConfig] = {
    "tiny": VideoDiTConfig(width=64, depth=2, num_heads=4, ffn_hidden=128, in_channels=4, text_width=32,
                           text_context_length=8, text_refiner_depth=1, cond_width=64, time_frequency_dim=32),
    "tiny_av": AVDiTConfig(width=64, depth=2, num_heads=4, ffn_hidden=128, in_channels=4, text_width=32,
                           text_context_length=8, text_refiner_depth=1, cond_width=64, time_frequency_dim=32,
                           audio_width=32, audio_num_heads=2, audio_in_channels=4, audio_ffn_hidden=64,
                           fusion_interval=1),
    # tiny GPU preset: head_dim 128 so the fused sm_100a path runs
    "tiny_gpu": VideoDiTConfig(width=256, depth=2, num_heads=2, ffn_hidden=512, in_channels=4, text_width=128,
                               text_context_length=16, cond_width=256, time_frequency_dim=64),
    "dit_300m": VideoDiTConfig(width=768, depth=24, num_heads=12, text_context_length=256),
    "dit_2b": VideoDiTConfig(width=2048, depth=24, num_heads=16, text_context_length=512),
    "dit_5b": VideoDiTConfig(width=3072, depth=28, num_heads=24, text_context_length=512),
    "dit_14b": VideoDiTConfig(width=4096, depth=42, num_heads=32, text_context_length=512),
    # the benchmark shapes (depth 32 x width 2560, 20 heads of 128; 40 x 5120 with MLP 13824)
    "bench_2b": VideoDiTConfig(width=2560, depth=32, num_heads=20, text_width=4096, text_context_length=512),
    "bench_14b": VideoDiTConfig(width=5120, depth=40, num_heads=40, ffn_hidden=13824, text_width=4096,
                                text_context_length=512),
}


def preset(name: str) -> VideoDiTConfig:
    try:
        return _PRESETS[name]
    except KeyError:
        raise KeyError(f"unknown preset {name!r}; available: {', '.join(sorted(_PRESETS))}") from None


def list_presets() -> tuple[str, ...]:
    return tuple(sorted(_PRESETS))


def config_overrides(config: VideoDiTConfig, **overrides: Any) -> VideoDiTConfig:
    """``dataclasses.replace`` that rejects unknown fields with a clear message."""
    known = {f.name for f in fields(config)}
    bad = sorted(set(overrides) - known)
    if bad:
        raise ValueError(f"unknown model field(s): {', '.join(bad)}")
    return replace(config, **overrides)


del F
