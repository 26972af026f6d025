"""Flow-matching ODE/SDE samplers (avgen/infer/sampler.py:69-839 API).

The model predicts the velocity ``v = noise - x0`` of the rectified-flow path
``x_t = x0 + t (noise - x0)`` (``sigma`` == ``t`` in [0, 1]); a sampler steps
``x_sigma`` to ``x_sigma_next`` with ``sigma_next < sigma``:

* ``euler`` — first order: ``x + (sigma_next - sigma) v``;
* ``heun`` — second order (trapezoid on the velocity, one extra evaluation);
* ``dpmpp_2m`` — DPM-Solver++(2M) in the data-prediction form for flow models
  (log-SNR steps ``h = lambda_next - lambda``, lambda = log((1-sigma)/sigma));
* ``res_multistep`` — second-order exponential multistep with phi-functions;
* ``euler_ancestral`` — Euler to ``sigma_down`` plus fresh noise of std
  ``sigma_up``; exposes the injected noise for policy-gradient RL.

Registered by name; third-party samplers load from the ``avgen.samplers``
entry-point group (the reference's group name, so existing plugins load).
"""
from __future__ import annotations

import math
from collections.abc import Callable, Mapping
from dataclasses import asdict, dataclass
from typing import Any, Protocol, TypeVar, runtime_checkable

import torch

__all__ = ["DPMSolverPlusPlus2M", "EulerAncestralSampler", "EulerSampler", "HeunSampler", "ResMultistepSampler",
           "Sampler", "SamplerConfig", "build_sampler", "list_samplers", "register_sampler", "to_epsilon", "to_x0"]

_FLOOR = 1e-7
SAMPLER_ENTRY_POINT_GROUP = "avgen.samplers"


def to_x0(x_t: torch.Tensor, velocity: torch.Tensor, sigma: float) -> torch.Tensor:
    """Clean-sample estimate ``x0 = x_t - sigma v``."""
    return x_t - sigma * velocity


def to_epsilon(x_t: torch.Tensor, velocity: torch.Tensor, sigma: float) -> torch.Tensor:
    """Noise estimate ``eps = x_t + (1 - sigma) v``."""
    return x_t + (1.0 - sigma) * velocity


Denoiser = Callable[[torch.Tensor, float], torch.Tensor]


@dataclass(frozen=True, slots=True)
class SamplerConfig:
    name: str = "euler"
    eta: float = 0.0
    s_noise: float = 1.0
    lower_order_final: bool = True

    def __post_init__(self) -> None:
        if not self.name or self.name.strip() != self.name:
            raise ValueError(f"name must be a non-empty trimmed string; got {self.name!r}")
        if not (math.isfinite(self.eta) and 0.0 <= self.eta <= 1.0):
            raise ValueError(f"eta must be in [0, 1]; got {self.eta!r}")
        if not (math.isfinite(self.s_noise) and self.s_noise >= 0.0):
            raise ValueError(f"s_noise must be finite and non-negative; got {self.s_noise!r}")

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: Mapping[str, Any]) -> SamplerConfig:
        return cls(**{k: values[k] for k in ("name", "eta", "s_noise", "lower_order_final") if k in values})


@runtime_checkable
class Sampler(Protocol):
    @property
    def evaluations_per_step(self) -> int: ...
    @property
    def is_stochastic(self) -> bool: ...
    def reset(self) -> None: ...
    def step(self, model_output: torch.Tensor, x_t: torch.Tensor, sigma_t: float, sigma_next: float, *,
             denoise: Denoiser | None = None, generator: torch.Generator | None = None) -> torch.Tensor: ...


_REGISTRY: dict[str, Callable[[SamplerConfig], Sampler]] = {}
_F = TypeVar("_F", bound=Callable[..., Any])


def register_sampler(name: str) -> Callable[[_F], _F]:
    if not name or name.strip() != name:
        raise ValueError(f"name must be a non-empty trimmed string; got {name!r}")
    if name in _REGISTRY:
        raise ValueError(f"sampler {name!r} is already registered")

    def deco(factory: _F) -> _F:
        _REGISTRY[name] = factory
        return factory

    return deco


def _accept(name: str, factory: object) -> None:
    if not callable(factory):
        raise TypeError(f"sampler plugin {name!r} must be a callable taking a SamplerConfig")
    _REGISTRY.setdefault(name, factory)  # type: ignore[arg-type]


def _load_plugins() -> None:
    from avgen_b200._plugins import load_entry_points

    load_entry_points(SAMPLER_ENTRY_POINT_GROUP, _accept)


def list_samplers() -> tuple[str, ...]:
    _load_plugins()
    return tuple(sorted(_REGISTRY))


def build_sampler(config: SamplerConfig | str) -> Sampler:
    _load_plugins()
    cfg = SamplerConfig(name=config) if isinstance(config, str) else config
    factory = _REGISTRY.get(cfg.name)
    if factory is None:
        raise KeyError(f"unknown sampler {cfg.name!r}; registered: {', '.join(sorted(_REGISTRY))}")
    return factory(cfg)


def _lambda(sigma: float) -> float:
    """Half log-SNR of the flow path: log(alpha / sigma) with alpha = 1 - sigma."""
    return math.log(max(1.0 - sigma, _FLOOR)) - math.log(max(sigma, _FLOOR))


class _Base:
    __slots__ = ("config",)

    def __init__(self, config: SamplerConfig | None = None) -> None:
        self.config = config or SamplerConfig()

    @property
    def evaluations_per_step(self) -> int:
        return 1

    @property
    def is_stochastic(self) -> bool:
        return False

    def reset(self) -> None:
        pass

    @staticmethod
    def _validate(sigma_t: float, sigma_next: float) -> None:
        if not (math.isfinite(sigma_t) and math.isfinite(sigma_next)):
            raise ValueError(f"sigmas must be finite; got {sigma_t!r} -> {sigma_next!r}")
        if sigma_next >= sigma_t:
            raise ValueError(f"sigma_next={sigma_next} must be below sigma_t={sigma_t}: sampling runs from noise "
                             "to data")


@register_sampler("euler")
class EulerSampler(_Base):
    __slots__ = ()

    def step(self, model_output, x_t, sigma_t, sigma_next, *, denoise=None, generator=None):  # noqa: ANN001, ANN201
        self._validate(sigma_t, sigma_next)
        return x_t + (sigma_next - sigma_t) * model_output


@register_sampler("heun")
class HeunSampler(_Base):
    __slots__ = ()

    @property
    def evaluations_per_step(self) -> int:
        return 2

    def step(self, model_output, x_t, sigma_t, sigma_next, *, denoise=None, generator=None):  # noqa: ANN001, ANN201
        self._validate(sigma_t, sigma_next)
        dt = sigma_next - sigma_t
        euler = x_t + dt * model_output
        if sigma_next == 0.0 and self.config.lower_order_final:
            return euler
        if denoise is None:
            raise ValueError("heun evaluates the model again at the Euler endpoint; pass denoise= (or use euler)")
        return x_t + 0.5 * dt * (model_output + denoise(euler, sigma_next))


class _TwoStep(_Base):
    """Shared state of the second-order multistep samplers: previous x0 and step."""

    __slots__ = ("_prev_h", "_prev_x0")

    def __init__(self, config: SamplerConfig | None = None) -> None:
        super().__init__(config)
        self._prev_x0: torch.Tensor | None = None
        self._prev_h: float | None = None

    def reset(self) -> None:
        self._prev_x0 = None
        self._prev_h = None

    def _first_order(self, x_t: torch.Tensor, x0: torch.Tensor, sigma_t: float, sigma_next: float) -> torch.Tensor:
        # exact solution of the flow ODE with x0 frozen over the step
        ratio = sigma_next / max(sigma_t, _FLOOR)
        return ratio * x_t + ((1.0 - sigma_next) - ratio * (1.0 - sigma_t)) * x0


@register_sampler("dpmpp_2m")
class DPMSolverPlusPlus2M(_TwoStep):
    __slots__ = ()

    def step(self, model_output, x_t, sigma_t, sigma_next, *, denoise=None, generator=None):  # noqa: ANN001, ANN201
        self._validate(sigma_t, sigma_next)
        x0 = to_x0(x_t, model_output, sigma_t)
        h = _lambda(sigma_next) - _lambda(sigma_t)
        last = sigma_next == 0.0 and self.config.lower_order_final
        if self._prev_x0 is None or self._prev_h is None or last:
            d = x0
        else:
            r = self._prev_h / h
            d = x0 + (x0 - self._prev_x0) / (2.0 * r)
        self._prev_x0, self._prev_h = x0, h
        return self._first_order(x_t, d, sigma_t, sigma_next)


@register_sampler("res_multistep")
class ResMultistepSampler(_TwoStep):
    __slots__ = ()

    def step(self, model_output, x_t, sigma_t, sigma_next, *, denoise=None, generator=None):  # noqa: ANN001, ANN201
        self._validate(sigma_t, sigma_next)
        x0 = to_x0(x_t, model_output, sigma_t)
        h = _lambda(sigma_next) - _lambda(sigma_t)
        last = sigma_next == 0.0 and self.config.lower_order_final
        if self._prev_x0 is None or self._prev_h is None or last:
            out = self._first_order(x_t, x0, sigma_t, sigma_next)
        else:
            # exponential integrator: phi_1(h) = (1 - e^-h), phi_2(h) = h - (1 - e^-h) weights on x0 and
            # on its slope in lambda, estimated from the previous step
            e = -math.expm1(-h)
            slope = (x0 - self._prev_x0) / self._prev_h
            ratio = sigma_next / max(sigma_t, _FLOOR)
            out = ratio * x_t + (1.0 - sigma_next) * (e * x0 + (h - e) * slope)
        self._prev_x0, self._prev_h = x0, h
        return out


@register_sampler("euler_ancestral")
class EulerAncestralSampler(_Base):
    __slots__ = ()

    @property
    def is_stochastic(self) -> bool:
        return self.config.eta > 0.0

    def ancestral_split(self, sigma_t: float, sigma_next: float) -> tuple[float, float]:
        """``(sigma_down, sigma_up)`` with ``sigma_down^2 + sigma_up^2 = sigma_next^2``."""
        if self.config.eta <= 0.0 or sigma_next == 0.0 or sigma_t == 0.0:
            return sigma_next, 0.0
        frac = max((sigma_t * sigma_t - sigma_next * sigma_next) / (sigma_t * sigma_t), 0.0)
        up = min(sigma_next, self.config.eta * sigma_next * math.sqrt(frac))
        return math.sqrt(max(sigma_next * sigma_next - up * up, 0.0)), up

    def step_with_noise(self, model_output: torch.Tensor, x_t: torch.Tensor, sigma_t: float, sigma_next: float, *,
                        generator: torch.Generator | None = None,
                        noise: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, float]:
        """The step plus the noise it injected and its scale (for log-probabilities)."""
        self._validate(sigma_t, sigma_next)
        down, up = self.ancestral_split(sigma_t, sigma_next)
        x = x_t + (down - sigma_t) * model_output
        if up == 0.0:
            return x, torch.zeros_like(x_t), 0.0
        if noise is None:
            if generator is None:
                raise ValueError("euler_ancestral with eta > 0 needs a torch.Generator for reproducible noise")
            noise = torch.randn(x_t.shape, generator=generator, device=x_t.device, dtype=x_t.dtype)
        return x + up * self.config.s_noise * noise, noise, up

    def step(self, model_output, x_t, sigma_t, sigma_next, *, denoise=None, generator=None):  # noqa: ANN001, ANN201
        return self.step_with_noise(model_output, x_t, sigma_t, sigma_next, generator=generator)[0]
