"""Diffusion-DPO for flow models (avgen/rl/dpo.py:67-467 API).

A batch stacks ``pairs`` winners followed by ``pairs`` losers. Both halves are
noised at one shared noise level per pair (and, by default, shared noise), the
policy and a frozen reference predict velocities, and with per-sample
velocity errors ``e`` the margin is

    m = -beta * ((e_pol_w - e_pol_l) - (e_ref_w - e_ref_l))

scored by ``-log sigmoid(m)`` (optionally label-smoothed and centred so a
policy equal to the reference scores 0), a hinge ``relu(1 - m)`` or IPO
``(m - 1/2)^2``. Under context parallelism the error sums and valid-token
counts are all-reduced over the CP group before dividing, so every CP rank
gets the loss of the whole sequence.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F

__all__ = ["DPOConfig", "DPOObjective", "dpo_loss"]


@dataclass(frozen=True, slots=True)
class DPOConfig:
    beta: float = 5000.0
    loss_type: str = "sigmoid"
    label_smoothing: float = 0.0
    share_noise: bool = True
    center_loss: bool = True
    snr_weighting: bool = False
    beta_scales_with_steps: bool = False
    timestep_count: int = 1000

    def __post_init__(self) -> None:
        if self.beta <= 0.0:
            raise ValueError(f"beta must be positive; got {self.beta!r}")
        if self.loss_type not in {"sigmoid", "hinge", "ipo"}:
            raise ValueError(f"loss_type must be 'sigmoid', 'hinge' or 'ipo'; got {self.loss_type!r}")
        if not 0.0 <= self.label_smoothing < 0.5:
            raise ValueError(f"label_smoothing must be in [0, 0.5); got {self.label_smoothing!r}")
        if isinstance(self.timestep_count, bool) or self.timestep_count < 1:
            raise ValueError(f"timestep_count must be a positive integer; got {self.timestep_count!r}")

    @property
    def effective_beta(self) -> float:
        return self.beta * self.timestep_count if self.beta_scales_with_steps else self.beta


def dpo_loss(policy_winner_error: torch.Tensor, policy_loser_error: torch.Tensor,
             reference_winner_error: torch.Tensor, reference_loser_error: torch.Tensor,
             config: DPOConfig) -> tuple[torch.Tensor, torch.Tensor]:
    """Mean per-pair loss and the per-pair margins."""
    margin = -config.effective_beta * ((policy_winner_error - policy_loser_error)
                                       - (reference_winner_error - reference_loser_error))
    if config.loss_type == "hinge":
        per = torch.relu(1.0 - margin)
    elif config.loss_type == "ipo":
        per = (margin - 0.5) ** 2
    else:
        a = config.label_smoothing
        per = -((1.0 - a) * F.logsigmoid(margin) + a * F.logsigmoid(-margin))
        if config.center_loss:
            per = per - math.log(2.0)  # the value at margin 0, whatever the smoothing
    return per.mean(), margin


class DPOObjective:
    """``objective(model, batch, rng, patchifier=..., cp_mesh=...)`` like the flow-matching objective."""

    def __init__(self, config: DPOConfig, reference_model: Any, *, timestep_sampler: Any = None) -> None:
        self.config = config
        self.reference_model = reference_model
        self.timestep_sampler = timestep_sampler
        self.last_margin: torch.Tensor | None = None

    def _levels(self, pairs: int, device: torch.device, generator: torch.Generator | None) -> torch.Tensor:
        gdev = generator.device if generator is not None else device
        if self.timestep_sampler is not None:
            return self.timestep_sampler.sample(pairs, device=gdev, generator=generator).float().to(device)
        return torch.rand(pairs, device=gdev, generator=generator, dtype=torch.float32).to(device)

    def __call__(self, model: Any, batch: Any, rng: Any, *, patchifier: Any, cp_mesh: Any = None) -> Any:
        from avgen_b200.core.model_input import ModelInput
        from avgen_b200.core.tokens import TextContext, TokenStream
        from avgen_b200.train.objective import ObjectiveOutput

        total = int(batch.video.shape[0])
        if total % 2:
            raise ValueError(f"DPO needs an even batch of stacked (winner, loser) pairs; got {total}")
        pairs = total // 2
        dev = batch.video.device
        video = batch.video.float()
        win, lose = video[:pairs], video[pairs:]
        sigma = self._levels(pairs, dev, rng.timestep)
        gdev = rng.noise.device if rng.noise is not None else dev
        eps_w = torch.randn(win.shape, device=gdev, generator=rng.noise).to(dev)
        eps_l = eps_w if self.config.share_noise else torch.randn(lose.shape, device=gdev, generator=rng.noise).to(dev)
        lvl = sigma.reshape(pairs, *((1,) * (win.ndim - 1)))
        noisy = torch.cat(((1 - lvl) * win + lvl * eps_w, (1 - lvl) * lose + lvl * eps_l))
        target = torch.cat((eps_w - win, eps_l - lose))
        sig2 = torch.cat((sigma, sigma))
        stream = patchifier.to_tokens(noisy, positions=batch.video_positions, mask=batch.video_mask, noise_level=sig2)
        target_tokens = patchifier.to_tokens(target, positions=batch.video_positions, mask=batch.video_mask,
                                             noise_level=sig2).tokens
        inputs = ModelInput(video=stream, audio=TokenStream.empty_like(total, stream.width, device=dev),
                            text=TextContext(features=batch.text, mask=batch.text_mask))
        if cp_mesh is not None and cp_mesh.size() > 1:
            from avgen_b200.parallel.context import shard_stream

            inputs = inputs.replace_streams(video=shard_stream(stream, cp_mesh))
            target_tokens = shard_stream(stream.with_tokens(target_tokens), cp_mesh).tokens
        mask = inputs.video.loss_mask().unsqueeze(-1).float()
        policy = model(inputs).video.float()
        with torch.no_grad():
            self.reference_model.eval()
            reference = self.reference_model(inputs).video.float()
        weight = None
        if self.config.snr_weighting:
            weight = ((1.0 - sig2) ** 2).reshape(total, 1, 1)

        def err(pred: torch.Tensor) -> torch.Tensor:
            sq = (pred - target_tokens.float()) ** 2 * mask
            if weight is not None:
                sq = sq * weight
            num = sq.flatten(1).sum(1)
            den = (mask.expand_as(sq)).flatten(1).sum(1)
            if cp_mesh is not None and cp_mesh.size() > 1:
                num = _all_reduce_sum(num, cp_mesh)
                den = _all_reduce_sum(den.detach(), cp_mesh)
            return num / den.clamp_min(1.0)

        pe, re = err(policy), err(reference)
        loss, margin = dpo_loss(pe[:pairs], pe[pairs:], re[:pairs], re[pairs:], self.config)
        self.last_margin = margin.detach().float()
        zero = torch.zeros((), device=dev, dtype=torch.float32)
        return ObjectiveOutput(loss=loss.float(), video_loss=loss.detach().float(), audio_loss=zero)


class _AllReduceSum(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, group: Any) -> torch.Tensor:  # noqa: ANN001
        import torch.distributed as dist

        y = x.clone()
        dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, grad: torch.Tensor):  # noqa: ANN001, ANN205
        # every CP rank computes the same loss from the reduced sums; each owns
        # the gradient of its own shard's contribution
        return grad, None


def _all_reduce_sum(x: torch.Tensor, mesh: Any) -> torch.Tensor:
    return _AllReduceSum.apply(x, mesh.get_group())
