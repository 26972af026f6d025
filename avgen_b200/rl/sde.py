"""Marginal-preserving SDE transitions that turn a flow sampler into a policy
(avgen/rl/sde.py:100-349 behaviour; Flow-GRPO, arXiv:2505.05470).

Convention: noise level ``s`` in [0, 1], 0 = clean, ``x_s = (1 - s) x0 + s eps``
and velocity ``v = eps - x0``. Then ``eps_hat = x + (1 - s) v`` exactly and the
SDE with the same marginals as the probability-flow ODE, discretised by
Euler-Maruyama over ``ds = s_next - s < 0``, is Gaussian::

    mean = x + (v + g^2 / (2 s) * eps_hat) * ds,   std = g * sqrt(|ds|)

with ``g(s) = a * sqrt(s / (1 - s))`` (clamped) or a constant ``a``.

On a CUDA device :func:`to_sde` runs one fused sm_100a kernel (mean, sample and
the per-sample log-density reduction in a single pass over the latents); on the
CPU it runs the same math in PyTorch, which is also the test oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

__all__ = ["DEFAULT_NOISE_LEVEL", "DEFAULT_SIGMA_FLOOR", "SDEStep", "diffusion_coefficient", "gaussian_log_prob",
           "ode_step", "to_sde"]

DEFAULT_NOISE_LEVEL = 0.7
DEFAULT_SIGMA_FLOOR = 1e-3
_HALF_LOG_2PI = 0.5 * math.log(2.0 * math.pi)


def diffusion_coefficient(noise_level_at: torch.Tensor, *, noise_level: float, schedule: str = "flow_grpo",
                          floor: float = DEFAULT_SIGMA_FLOOR) -> torch.Tensor:
    """``g(s)`` per sample: ``a * sqrt(s / (1 - s))`` (``flow_grpo``) or ``a`` (``constant``)."""
    if noise_level < 0.0:
        raise ValueError(f"noise_level must be non-negative; got {noise_level!r}")
    if not 0.0 < floor < 1.0:
        raise ValueError(f"floor must be in (0, 1); got {floor!r}")
    if schedule == "constant":
        return torch.full_like(noise_level_at, noise_level, dtype=torch.float32)
    if schedule != "flow_grpo":
        raise ValueError(f"unknown schedule {schedule!r}; expected 'flow_grpo' or 'constant'")
    s = noise_level_at.float().clamp(min=floor, max=1.0 - floor)
    return noise_level * torch.sqrt(s / (1.0 - s))


@dataclass(frozen=True, slots=True)
class SDEStep:
    """One transition: the state after it, its log-density (summed over every
    non-batch dimension), the Gaussian mean and the per-sample std."""

    sample: torch.Tensor
    log_prob: torch.Tensor
    mean: torch.Tensor
    std: torch.Tensor
    deterministic: bool = False


def _per_sample(value: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return value.reshape(value.shape[0], *((1,) * (like.ndim - 1)))


def gaussian_log_prob(value: torch.Tensor, mean: torch.Tensor, std: torch.Tensor, *,
                      mask: torch.Tensor | None = None) -> torch.Tensor:
    """Normalised isotropic Gaussian log-density, summed per sample (padding excluded by ``mask``)."""
    if value.shape != mean.shape:
        raise ValueError(f"value shape {tuple(value.shape)} must match mean shape {tuple(mean.shape)}")
    sigma = _per_sample(std, value) if std.ndim == 1 else std
    z = (value - mean) / sigma
    per = -0.5 * z * z - torch.log(sigma) - _HALF_LOG_2PI
    if mask is not None:
        per = per * mask.to(per.dtype)
    return per.flatten(1).sum(1)


def ode_step(velocity: torch.Tensor, x_t: torch.Tensor, sigma_t: torch.Tensor, sigma_next: torch.Tensor) -> torch.Tensor:
    """Deterministic Euler step of the probability-flow ODE."""
    return x_t + velocity * _per_sample(sigma_next - sigma_t, x_t)


def _use_kernel(*tensors: torch.Tensor) -> bool:
    return all(t.is_cuda for t in tensors)


def to_sde(velocity: torch.Tensor, x_t: torch.Tensor, sigma_t: torch.Tensor, sigma_next: torch.Tensor, *,
           noise_level: float = DEFAULT_NOISE_LEVEL, generator: torch.Generator | None = None,
           prev_sample: torch.Tensor | None = None, schedule: str = "flow_grpo",
           floor: float = DEFAULT_SIGMA_FLOOR, mask: torch.Tensor | None = None) -> SDEStep:
    """One Euler-Maruyama step of the marginal-preserving SDE.

    ``prev_sample is None``: rollout, a state is drawn and scored (``log pi_old``).
    ``prev_sample`` given: update, the stored state is scored under the current
    velocity (``log pi_theta``); nothing is drawn. ``noise_level == 0`` is the
    exact ODE limit with log-probability 0 by convention.
    """
    if bool((sigma_next > sigma_t + 1e-6).any()):
        raise ValueError("sigma_next must not exceed sigma_t; sampling integrates the noise level down to 0 (clean)")
    if prev_sample is not None and prev_sample.shape != x_t.shape:
        raise ValueError(f"prev_sample shape {tuple(prev_sample.shape)} must match x_t {tuple(x_t.shape)}")
    g = diffusion_coefficient(sigma_t, noise_level=noise_level, schedule=schedule, floor=floor)
    ds = (sigma_next - sigma_t).float()
    if noise_level == 0.0:
        mean = ode_step(velocity, x_t, sigma_t, sigma_next)
        zeros = torch.zeros(x_t.shape[0], device=x_t.device, dtype=torch.float32)
        return SDEStep(sample=mean if prev_sample is None else prev_sample, log_prob=zeros, mean=mean, std=zeros,
                       deterministic=True)
    std = g * torch.sqrt(ds.abs())
    noise = None
    if prev_sample is None:
        gen_dev = generator.device if generator is not None else x_t.device
        noise = torch.randn(x_t.shape, device=gen_dev, dtype=torch.float32, generator=generator).to(x_t.device)
    if _use_kernel(velocity, x_t) and velocity.requires_grad is False:
        from avgen_b200.ops import kernels as K

        sample, mean, log_prob = K.sde_step(velocity, x_t, sigma_t, sigma_next, g, floor=floor, noise=noise,
                                            prev=prev_sample, mask=mask)
        return SDEStep(sample=sample.to(x_t.dtype) if prev_sample is None else prev_sample, log_prob=log_prob,
                       mean=mean, std=std)
    s = _per_sample(sigma_t.float().clamp(min=floor), x_t)
    v = velocity.float()
    x = x_t.float()
    eps_hat = x + (1.0 - s) * v
    mean = x + (v + _per_sample(g * g, x_t) / (2.0 * s) * eps_hat) * _per_sample(ds, x_t)
    if prev_sample is None:
        assert noise is not None
        sample = (mean + _per_sample(std, x_t) * noise).to(x_t.dtype)
    else:
        sample = prev_sample
    log_prob = gaussian_log_prob(sample.float(), mean, std.clamp_min(1e-12), mask=mask)
    return SDEStep(sample=sample, log_prob=log_prob, mean=mean, std=std)
