"""Rectified-flow (flow-matching) objective (avgen/train/objective.py:254-700).

``x_t = x + t (eps - x)`` and the velocity target ``v = eps - x``, with an
independent ``t`` per modality, conditioned tokens at ``t = 0`` and excluded
from the loss, per-token MSE averaged over the patch features, optional
timestep weighting (uniform / sigma_sqrt / cosmap) and SNR clamp, and a
context-parallel-correct reduction: the supervised-token denominator is summed
over the CP group and the local loss is scaled by the CP degree so gradient
averaging over the group reproduces the unsharded loss.

On CUDA the local shard is prepared without ever materialising the full
sequence: clean tokens are sharded first and the noise is drawn by a
counter-based kernel keyed by the *global* token index (so every CP rank gets
exactly its slice of the unsharded draw), and the masked-MSE loss is one
reduction kernel plus one gradient kernel. On the CPU the same maths runs in
PyTorch with ``torch.randn``.
"""
from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field, replace
from typing import Any, Protocol, runtime_checkable

import torch
from torch import nn
from torch.distributed.device_mesh import DeviceMesh

from avgen_b200.core._validate import require_finite
from avgen_b200.core.batch import MediaBatch
from avgen_b200.core.model_input import ModelInput, ModelOutput
from avgen_b200.core.patchify import GridPatchifier, Patchifier
from avgen_b200.core.rng import RNGStreams
from avgen_b200.core.tokens import TextContext, TokenStream
from avgen_b200.parallel.comm import all_reduce_sum
from avgen_b200.parallel.context import shard_bounds, shard_stream
from avgen_b200.train.conditioning import ConditioningPlan, ConditioningSampler
from avgen_b200.train.timestep import TimestepSampler

__all__ = ["FlowMatchingConfig", "FlowMatchingObjective", "FlowTargets", "Objective", "ObjectiveOutput",
           "masked_flow_loss"]

_T_EPS = 1e-5
_WEIGHTINGS = ("uniform", "sigma_sqrt", "cosmap")


def _zero_i64() -> torch.Tensor:
    return torch.empty(0, dtype=torch.int64)


@dataclass(frozen=True, slots=True)
class ObjectiveOutput:
    loss: torch.Tensor
    video_loss: torch.Tensor
    audio_loss: torch.Tensor
    valid_video_tokens: torch.Tensor = field(default_factory=_zero_i64)
    valid_audio_tokens: torch.Tensor = field(default_factory=_zero_i64)

    def __post_init__(self) -> None:
        for name in ("valid_video_tokens", "valid_audio_tokens"):
            if getattr(self, name).numel() == 0:
                object.__setattr__(self, name, torch.zeros((), dtype=torch.int64, device=self.loss.device))

    def validate(self) -> None:
        for name in ("loss", "video_loss", "audio_loss", "valid_video_tokens", "valid_audio_tokens"):
            if getattr(self, name).ndim != 0:
                raise ValueError(f"{name} must be scalar")
        for name in ("video_loss", "audio_loss"):
            if getattr(self, name).requires_grad:
                raise ValueError(f"{name} must be detached")


@runtime_checkable
class Objective(Protocol):
    def __call__(self, model: nn.Module, batch: MediaBatch, rng: RNGStreams, *, patchifier: Patchifier,
                 cp_mesh: DeviceMesh | None = None) -> ObjectiveOutput: ...


@dataclass(frozen=True, slots=True)
class FlowMatchingConfig:
    video_weight: float = 1.0
    audio_weight: float = 1.0
    independent_modality_noise: bool = True
    timestep_weighting: str = "uniform"
    snr_gamma: float | None = None
    validate: bool = False

    def __post_init__(self) -> None:
        for name in ("video_weight", "audio_weight"):
            require_finite(name, getattr(self, name))
            if getattr(self, name) < 0:
                raise ValueError(f"{name} must be non-negative")
        if self.timestep_weighting not in _WEIGHTINGS:
            raise ValueError(f"timestep_weighting must be one of {', '.join(_WEIGHTINGS)}")
        if self.snr_gamma is not None and self.snr_gamma <= 0:
            raise ValueError("snr_gamma must be positive")


class _FlowLoss(torch.autograd.Function):
    """Kernel-backed masked flow loss: returns ``[weighted_num, raw_num, den]``; only
    ``weighted_num`` carries a gradient."""

    @staticmethod
    def forward(ctx, pred, target, loss_mask, weight, rows_per_batch):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        stats = K.flow_loss_stats(pred, target, loss_mask, weight, rows_per_batch=rows_per_batch)
        ctx.save_for_backward(pred, target, loss_mask, weight)
        ctx.rows_per_batch = rows_per_batch
        rest = stats[1:].clone()
        ctx.mark_non_differentiable(rest)
        return stats[0].clone(), rest

    @staticmethod
    def backward(ctx, g_num, g_rest):  # noqa: ANN001, ANN205
        from avgen_b200.ops import kernels as K

        pred, target, loss_mask, weight = ctx.saved_tensors
        scale = g_num.reshape(1).float().contiguous()
        dpred = K.flow_loss_grad(pred, target, loss_mask, weight, scale, rows_per_batch=ctx.rows_per_batch)
        return dpred, None, None, None, None


def masked_flow_loss(prediction: torch.Tensor, target: torch.Tensor, stream: TokenStream,
                     weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(weighted sum, raw sum, supervised count, valid count)`` of per-token MSE."""
    supervised = stream.loss_mask()
    valid = stream.mask.sum().to(torch.float32).detach()
    if prediction.device.type == "cuda" and prediction.numel() > 0:
        rows = prediction.shape[1]
        num, rest = _FlowLoss.apply(prediction.contiguous(), target.contiguous(), supervised.contiguous(),
                                    weight.float().contiguous(), rows)
        return num, rest[0].detach(), rest[1].detach(), valid
    residual = prediction.float() - target.float()
    err = residual.pow(2).mean(-1)
    sup = supervised.to(torch.float32)
    masked = err * sup
    return (masked * weight[:, None]).sum(), masked.sum().detach(), sup.sum().detach(), valid


@dataclass(frozen=True, slots=True)
class FlowTargets:
    """What the loss needs besides the model output: velocity targets and noise levels."""

    video: torch.Tensor
    audio: torch.Tensor
    video_t: torch.Tensor
    audio_t: torch.Tensor
    has_audio: bool
    cp_mesh: Any = None


class FlowMatchingObjective:
    __slots__ = ("audio_patchifier", "conditioning_sampler", "config", "timestep_sampler", "weight_fn")

    def __init__(self, config: FlowMatchingConfig, timestep_sampler: TimestepSampler,
                 conditioning_sampler: ConditioningSampler, *, audio_patchifier: Patchifier | None = None,
                 weight_fn: Callable[[torch.Tensor], torch.Tensor] | None = None) -> None:
        self.config = config
        self.timestep_sampler = timestep_sampler
        self.conditioning_sampler = conditioning_sampler
        self.audio_patchifier = audio_patchifier or GridPatchifier(patch_frames=1, patch_height=1, patch_width=1)
        self.weight_fn = weight_fn

    def __call__(self, model: nn.Module, batch: MediaBatch, rng: RNGStreams, *, patchifier: Patchifier,
                 cp_mesh: DeviceMesh | None = None) -> ObjectiveOutput:
        inputs, targets = self.prepare(batch, rng, patchifier=patchifier, cp_mesh=cp_mesh)
        output: ModelOutput = model(inputs)
        return self.finish(output, inputs, targets)

    def prepare(self, batch: MediaBatch, rng: RNGStreams, *, patchifier: Patchifier,
                cp_mesh: DeviceMesh | None = None) -> tuple[ModelInput, FlowTargets]:
        """The model input (noisy streams, conditioning, text after dropout) and the
        regression targets of one batch. Deterministic in ``rng``: pipeline stages
        that share a data rank draw the same noise and timesteps."""
        plan = self.conditioning_sampler.sample(batch, rng=rng)
        if self.config.validate:
            plan.validate(batch)
        vlayout = patchifier.layout_for(tuple(batch.video.shape))
        agrid = batch.audio[:, :, :, None, None]
        has_audio = batch.spec.has_audio
        seq = vlayout.num_tokens
        if has_audio:
            seq += self.audio_patchifier.layout_for(tuple(agrid.shape)).num_tokens
        dev = batch.device
        vt = self.timestep_sampler.sample(batch.spec.batch_size, device=dev, generator=rng.timestep,
                                          sequence_length=seq)
        at = (self.timestep_sampler.sample(batch.spec.batch_size, device=dev, generator=rng.timestep,
                                           sequence_length=seq)
              if self.config.independent_modality_noise else vt)
        vstream, vtarget = self._prepare(patchifier, grid=batch.video, positions=batch.video_positions,
                                         mask=batch.video_mask, conditioned=plan.video_conditioned, timesteps=vt,
                                         rng=rng, cp_mesh=cp_mesh, purpose="video")
        if has_audio:
            astream, atarget = self._prepare(self.audio_patchifier, grid=agrid, positions=batch.audio_positions,
                                             mask=batch.audio_mask[:, :, None, None],
                                             conditioned=plan.audio_conditioned[:, :, None, None], timesteps=at,
                                             rng=rng, cp_mesh=cp_mesh, purpose="audio")
        else:
            astream = TokenStream.empty_like(batch.spec.batch_size, batch.spec.audio_shape[1], device=dev,
                                             dtype=batch.video.dtype)
            atarget = astream.tokens
        inputs = ModelInput(video=vstream, audio=astream, text=_apply_text_dropout(batch, plan),
                            condition_mode=plan.condition_mode)
        if self.config.validate:
            inputs.validate()
        return inputs, FlowTargets(video=vtarget, audio=atarget, video_t=vt, audio_t=at, has_audio=has_audio,
                                   cp_mesh=cp_mesh)

    def finish(self, output: ModelOutput, inputs: ModelInput, targets: FlowTargets) -> ObjectiveOutput:
        """The loss of ``output`` against ``targets`` (summed across context-parallel shards)."""
        if self.config.validate:
            output.validate(inputs)
        return self._reduce(output=output, vstream=inputs.video, vtarget=targets.video, vt=targets.video_t,
                            astream=inputs.audio, atarget=targets.audio, at=targets.audio_t,
                            has_audio=targets.has_audio, cp_mesh=targets.cp_mesh)

    def _prepare(self, patchifier: Patchifier, *, grid: torch.Tensor, positions: torch.Tensor, mask: torch.Tensor,
                 conditioned: torch.Tensor, timesteps: torch.Tensor, rng: RNGStreams, cp_mesh: DeviceMesh | None,
                 purpose: str) -> tuple[TokenStream, torch.Tensor]:
        clean = patchifier.to_tokens(grid, positions=positions, mask=mask, noise_level=timesteps,
                                     conditioned=conditioned)
        per_token = clean.noise_level[:, None] * (~clean.conditioned).to(torch.float32)
        # two levels per sample: t for noisy tokens, 0 for clean conditioning anchors
        clean = replace(clean, level_values=torch.stack((clean.noise_level, torch.zeros_like(clean.noise_level)), 1),
                        level_index=clean.conditioned.to(torch.int32))
        if clean.tokens.device.type == "cuda":
            from avgen_b200.ops import kernels as K

            total = clean.length
            cp_rank, cp_size = (0, 1) if cp_mesh is None else (cp_mesh.get_local_rank(), cp_mesh.size())
            lo, hi = shard_bounds(total, cp_size, cp_rank)
            local = shard_stream(replace(clean, noise_level=per_token), cp_mesh)
            seed = rng.seed_for(purpose)
            noisy, target, _ = K.noise_interp(local.tokens.contiguous(), local.noise_level.contiguous(), seed=seed,
                                              row_base=lo, rows_per_sample=hi - lo, global_rows_per_sample=total)
            return replace(local, tokens=noisy), target
        noise = torch.randn(clean.tokens.shape, generator=rng.noise, device=rng.noise.device,
                            dtype=torch.float32).to(clean.tokens.device, clean.tokens.dtype)
        level = per_token[..., None]
        noisy = clean.tokens + level * (noise - clean.tokens)
        target = noise - clean.tokens
        stream = replace(clean, tokens=noisy, noise_level=per_token)
        if cp_mesh is None or cp_mesh.size() == 1:
            return stream, target
        width = noisy.shape[-1]
        packed = shard_stream(replace(stream, tokens=torch.cat((noisy, target), -1)), cp_mesh)
        return replace(packed, tokens=packed.tokens[..., :width].contiguous()), packed.tokens[..., width:].contiguous()

    def _timestep_weight(self, t: torch.Tensor) -> torch.Tensor:
        c = t.to(torch.float32).clamp(_T_EPS, 1.0 - _T_EPS)
        if self.config.timestep_weighting == "sigma_sqrt":
            w = c.pow(-2.0)
        elif self.config.timestep_weighting == "cosmap":
            w = 2.0 / (torch.pi * (1.0 - 2.0 * c + 2.0 * c.pow(2)))
        else:
            w = torch.ones_like(c)
        if self.config.snr_gamma is not None:
            snr = ((1.0 - c) / c).pow(2)
            w = w * (snr.clamp(max=self.config.snr_gamma) / (snr + 1.0))
        if self.weight_fn is not None:
            w = w * self.weight_fn(t).to(torch.float32)
        return w

    def _reduce(self, *, output: ModelOutput, vstream: TokenStream, vtarget: torch.Tensor, vt: torch.Tensor,
                astream: TokenStream, atarget: torch.Tensor, at: torch.Tensor, has_audio: bool,
                cp_mesh: DeviceMesh | None) -> ObjectiveOutput:
        vnum, vraw, vden, vvalid = masked_flow_loss(output.video, vtarget, vstream, self._timestep_weight(vt))
        if has_audio:
            anum, araw, aden, avalid = masked_flow_loss(output.audio, atarget, astream, self._timestep_weight(at))
        else:
            z = torch.zeros((), dtype=torch.float32, device=vnum.device)
            anum = araw = aden = avalid = z
        stats = all_reduce_sum(torch.stack((vraw, vden, vvalid, araw, aden, avalid)), cp_mesh)
        vden_g = stats[1].clamp(min=1.0)
        aden_g = stats[4].clamp(min=1.0)
        degree = float(cp_mesh.size()) if cp_mesh is not None else 1.0
        loss = degree * (self.config.video_weight * vnum / vden_g + self.config.audio_weight * anum / aden_g)
        return ObjectiveOutput(loss=loss.to(torch.float32), video_loss=(stats[0] / vden_g).detach(),
                               audio_loss=(stats[3] / aden_g).detach(),
                               valid_video_tokens=stats[2].detach().to(torch.int64),
                               valid_audio_tokens=stats[5].detach().to(torch.int64))


def _apply_text_dropout(batch: MediaBatch, plan: ConditioningPlan) -> TextContext:
    keep = ~plan.drop_text
    feats = batch.text * keep[:, None, None].to(batch.text.dtype)
    return TextContext(features=feats, mask=batch.text_mask & keep[:, None])
