"""Generator-device-aware random draws (avgen/train/_random.py): draw on the
generator's device, then move, so CPU generators drive CUDA training without
changing the random stream."""
from __future__ import annotations

import torch

__all__ = ["bernoulli", "categorical", "normal", "uniform"]


def _move(value: torch.Tensor, device: torch.device | str) -> torch.Tensor:
    dev = torch.device(device)
    return value if value.device == dev else value.to(dev, non_blocking=True)


def uniform(shape: tuple[int, ...], *, generator: torch.Generator, device: torch.device | str,
            dtype: torch.dtype = torch.float32) -> torch.Tensor:
    return _move(torch.rand(shape, generator=generator, device=generator.device, dtype=dtype), device)


def normal(shape: tuple[int, ...], *, generator: torch.Generator, device: torch.device | str,
           dtype: torch.dtype = torch.float32) -> torch.Tensor:
    return _move(torch.randn(shape, generator=generator, device=generator.device, dtype=dtype), device)


def bernoulli(shape: tuple[int, ...], probability: float, *, generator: torch.Generator,
              device: torch.device | str) -> torch.Tensor:
    return uniform(shape, generator=generator, device=device) < probability


def categorical(weights: torch.Tensor, count: int, *, generator: torch.Generator,
                device: torch.device | str) -> torch.Tensor:
    src = weights.to(generator.device, dtype=torch.float32)
    if float(src.sum()) <= 0.0:
        raise ValueError("categorical weights must contain at least one positive entry")
    drawn = torch.multinomial(src, count, replacement=True, generator=generator)
    return _move(drawn.to(torch.int64), device)
