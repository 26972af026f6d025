"""Integrate the flow ODE with each sampler, and see what the schedule shift does.

A rectified-flow model predicts the velocity ``v = noise - x``. With a model
that knows the clean sample exactly, every sampler recovers it; the interesting
part is how many model evaluations each spends and how the sigma schedule
distributes its steps. Long sequences need more of the steps at high noise, so
the shift grows with the token count.

    python examples/05_sampling_and_schedules.py
"""
from __future__ import annotations

import torch

from avgen_b200.infer.sampler import SamplerConfig, build_sampler, list_samplers
from avgen_b200.infer.schedule import ScheduleConfig, build_sigma_schedule, list_sigma_schedules


def main() -> None:
    generator = torch.Generator().manual_seed(0)
    clean = torch.randn(1, 4, 2, 8, 8, generator=generator)
    noise = torch.randn(clean.shape, generator=generator)

    def velocity(x: torch.Tensor, sigma: float) -> torch.Tensor:
        # the exact velocity field of the straight path from `clean` to `noise`
        return (x - clean) / max(sigma, 1e-6)

    print("schedules:", ", ".join(list_sigma_schedules()))
    for length in (1024, 16384, 65536):
        schedule = build_sigma_schedule(ScheduleConfig(steps=8, dynamic_shift=True, max_length=65536),
                                        sequence_length=length)
        sigmas = ", ".join(f"{s:.2f}" for s in schedule.tolist())
        print(f"  {length:6d} tokens, shift {schedule.shift:.2f}: {sigmas}")

    schedule = build_sigma_schedule(ScheduleConfig(steps=12))
    sigmas = schedule.tolist()
    print("samplers:", ", ".join(list_samplers()))
    for name in list_samplers():
        sampler = build_sampler(SamplerConfig(name=name))
        x = noise.clone()
        for sigma, nxt in zip(sigmas[:-1], sigmas[1:]):
            x = sampler.step(velocity(x, sigma), x, sigma, nxt, denoise=velocity,
                             generator=torch.Generator().manual_seed(1))
        error = float((x - clean).abs().max())
        print(f"  {name:16s} {sampler.evaluations_per_step} evaluation(s) per step, max error {error:.2e}")


if __name__ == "__main__":
    main()
