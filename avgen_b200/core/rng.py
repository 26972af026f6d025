"""Purpose-separated random streams (noise, timestep, conditioning, sampler).

Same contract as avgen/core/rng.py:31-202: four independent generators so
changing how many timesteps are drawn never shifts the noise stream; the
per-rank variant mixes only the *data* rank so context-parallel and
tensor-parallel peers draw identical noise and data. Stream seeds are derived
here with a SplitMix64 finaliser (Steele, Lea, Flood: "Fast splittable
pseudorandom number generators", OOPSLA 2014) over the stream name.
"""
from __future__ import annotations

from collections.abc import Mapping
from typing import Any, ClassVar

import torch

__all__ = ["RNGStreams", "mix_seed"]

_MASK64 = (1 << 64) - 1
_MAX_SEED = (1 << 63) - 1


def _splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & _MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _MASK64
    return x ^ (x >> 31)


def _name_key(name: str) -> int:
    h = 0
    for ch in name.encode():
        h = _splitmix64(h ^ ch)
    return h


def mix_seed(seed: int, *parts: int | str) -> int:
    """Deterministic 63-bit seed derived from ``seed`` and any labels."""
    x = _splitmix64(seed & _MASK64)
    for p in parts:
        x = _splitmix64(x ^ (_name_key(p) if isinstance(p, str) else (p & _MASK64)))
    return x & _MAX_SEED


class RNGStreams:
    """Four named :class:`torch.Generator` streams."""

    __slots__ = ("conditioning", "noise", "sampler", "timestep")
    NAMES: ClassVar[tuple[str, ...]] = ("noise", "timestep", "conditioning", "sampler")

    def __init__(self, noise: torch.Generator, timestep: torch.Generator, conditioning: torch.Generator,
                 sampler: torch.Generator) -> None:
        self.noise = noise
        self.timestep = timestep
        self.conditioning = conditioning
        self.sampler = sampler

    @classmethod
    def from_seed(cls, seed: int, *, device: torch.device | str = "cpu") -> RNGStreams:
        if isinstance(seed, bool) or not isinstance(seed, int) or seed < 0:
            raise ValueError(f"seed must be a non-negative integer; got {seed!r}")
        gens = {}
        for name in cls.NAMES:
            g = torch.Generator(device=device)
            g.manual_seed(mix_seed(seed, name))
            gens[name] = g
        return cls(**gens)

    @classmethod
    def for_rank(cls, seed: int, *, data_rank: int, device: torch.device | str = "cpu") -> RNGStreams:
        """Streams for one data-parallel rank (CP/TP peers share them)."""
        if isinstance(data_rank, bool) or data_rank < 0:
            raise ValueError(f"data_rank must be non-negative; got {data_rank!r}")
        return cls.from_seed(mix_seed(seed, "data_rank", data_rank), device=device)

    def fork(self, purpose: str) -> torch.Generator:
        """A new generator for an ad-hoc purpose, advancing the noise stream once."""
        base = int(torch.randint(0, _MAX_SEED, (1,), generator=self.noise).item())
        g = torch.Generator(device=self.noise.device)
        g.manual_seed(mix_seed(base, purpose))
        return g

    def seed_for(self, purpose: str) -> int:
        """A 63-bit integer seed drawn from the noise stream (for counter-based kernels)."""
        base = int(torch.randint(0, _MAX_SEED, (1,), generator=self.noise).item())
        return mix_seed(base, purpose)

    def state_dict(self) -> dict[str, Any]:
        return {name: getattr(self, name).get_state().clone() for name in self.NAMES}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        if set(state) != set(self.NAMES):
            raise ValueError(f"RNG state keys must be {sorted(self.NAMES)}; got {sorted(state)}")
        for name in self.NAMES:
            value = state[name]
            if not isinstance(value, torch.Tensor) or value.dtype is not torch.uint8 or value.device.type != "cpu":
                raise TypeError(f"RNG state {name!r} must be a CPU uint8 tensor")
            getattr(self, name).set_state(value)

    def validate(self) -> None:
        if len({str(getattr(self, n).device) for n in self.NAMES}) != 1:
            raise ValueError("all RNG streams must target the same device")
