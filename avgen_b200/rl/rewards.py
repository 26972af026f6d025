"""Reward models for diffusion RL (avgen/rl/rewards.py:54-691 API).

Built in: ``temporal_consistency`` (mean cosine similarity of consecutive
frames), ``motion_magnitude`` (Gaussian score of the mean absolute frame
difference around a target), ``av_sync_proxy`` (correlation of the visual
motion envelope with the audio energy envelope) and ``mlp_scorer`` (a seeded,
random-init two-layer MLP over mean-pooled latents, the synthetic reward of
the post-training benchmark). ``hps_v2``, ``pick_score`` and ``video_score``
are registered but need external packages and raise with instructions.
Third-party rewards register through the ``avgen.rewards`` entry-point group.
:class:`CompositeReward` mixes rewards with per-component running, batch or no
normalisation.
"""
from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, field
from typing import Any, Protocol, runtime_checkable

import torch

__all__ = ["AVSyncProxyReward", "CompositeReward", "HPSv2Reward", "MLPScorerReward", "MotionMagnitudeReward",
           "PickScoreReward", "REWARD_ENTRY_POINT_GROUP", "RewardModel", "RunningNormalizer",
           "TemporalConsistencyReward", "VideoScoreReward", "build_reward", "list_rewards", "media_tensors",
           "register_reward"]

REWARD_ENTRY_POINT_GROUP = "avgen.rewards"


@runtime_checkable
class RewardModel(Protocol):
    def score(self, media: Any, prompts: Sequence[str]) -> torch.Tensor: ...


def media_tensors(media: Any) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``(video [B, C, T, H, W], audio or None)`` from a tensor, a mapping or an object with ``.video``."""
    if isinstance(media, torch.Tensor):
        video, audio = media, None
    elif isinstance(media, Mapping):
        video, audio = media.get("video"), media.get("audio")
    else:
        video, audio = getattr(media, "video", None), getattr(media, "audio", None)
    if not isinstance(video, torch.Tensor):
        raise TypeError("media must be a video tensor, a mapping with a 'video' key, or an object with a .video "
                        f"attribute; got {type(media).__name__}")
    if video.ndim != 5:
        raise ValueError(f"video must be rank 5 (batch, channels, frames, height, width); got {tuple(video.shape)}")
    return video, audio if isinstance(audio, torch.Tensor) else None


def _check(video: torch.Tensor, prompts: Sequence[str]) -> None:
    if len(prompts) != video.shape[0]:
        raise ValueError(f"expected {video.shape[0]} prompts to match the batch; got {len(prompts)}")


def _frames(video: torch.Tensor) -> torch.Tensor:
    """``[B, T, C*H*W]`` fp32 frame vectors."""
    b, _, t = video.shape[:3]
    return video.transpose(1, 2).reshape(b, t, -1).float()


@dataclass(frozen=True, slots=True)
class TemporalConsistencyReward:
    name: str = "temporal_consistency"

    def score(self, media: Any, prompts: Sequence[str]) -> torch.Tensor:
        video, _ = media_tensors(media)
        _check(video, prompts)
        f = _frames(video)
        if f.shape[1] < 2:
            return torch.ones(f.shape[0], device=video.device)
        return torch.nn.functional.cosine_similarity(f[:, :-1], f[:, 1:], dim=-1).mean(1)


@dataclass(frozen=True, slots=True)
class MotionMagnitudeReward:
    target: float = 0.1
    tolerance: float = 0.08
    name: str = "motion_magnitude"

    def __post_init__(self) -> None:
        if self.tolerance <= 0.0:
            raise ValueError(f"tolerance must be positive; got {self.tolerance!r}")
        if self.target < 0.0:
            raise ValueError(f"target must be non-negative; got {self.target!r}")

    def score(self, media: Any, prompts: Sequence[str]) -> torch.Tensor:
        video, _ = media_tensors(media)
        _check(video, prompts)
        f = _frames(video)
        motion = (f[:, 1:] - f[:, :-1]).abs().mean((1, 2)) if f.shape[1] >= 2 else \
            torch.zeros(f.shape[0], device=video.device)
        z = (motion - self.target) / self.tolerance
        return torch.exp(-0.5 * z * z)


def _resample(x: torch.Tensor, n: int) -> torch.Tensor:
    if x.shape[1] == n:
        return x
    return torch.nn.functional.interpolate(x.unsqueeze(1), size=n, mode="linear", align_corners=False).squeeze(1)


def _pearson(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    a = a - a.mean(1, keepdim=True)
    b = b - b.mean(1, keepdim=True)
    return (a * b).sum(1) / (a.norm(dim=1) * b.norm(dim=1) + 1e-8)


@dataclass(frozen=True, slots=True)
class AVSyncProxyReward:
    name: str = "av_sync_proxy"

    def score(self, media: Any, prompts: Sequence[str]) -> torch.Tensor:
        video, audio = media_tensors(media)
        _check(video, prompts)
        zeros = torch.zeros(video.shape[0], device=video.device)
        if audio is None or audio.ndim != 3 or audio.shape[-1] < 2:
            return zeros
        f = _frames(video)
        if f.shape[1] < 2:
            return zeros
        visual = (f[:, 1:] - f[:, :-1]).abs().mean(-1)
        acoustic = audio.float().abs().mean(1)
        n = min(visual.shape[1], acoustic.shape[1])
        if n < 2:
            return zeros
        return _pearson(_resample(visual, n), _resample(acoustic, n))


class MLPScorerReward(torch.nn.Module):
    """A deterministic random-init 2-layer MLP over per-channel mean-pooled latents
    (``[B, C, T, H, W] -> [B, C] -> hidden -> 1``), seeded so every rank and every
    run scores identically. Scores are tanh-bounded."""

    name = "mlp_scorer"

    def __init__(self, channels: int = 16, hidden: int = 256, seed: int = 0) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.fc1 = torch.nn.Linear(channels, hidden)
        self.fc2 = torch.nn.Linear(hidden, 1)
        with torch.no_grad():
            for lin in (self.fc1, self.fc2):
                bound = 1.0 / lin.in_features ** 0.5
                lin.weight.copy_(torch.empty(lin.weight.shape).uniform_(-bound, bound, generator=g))
                lin.bias.copy_(torch.empty(lin.bias.shape).uniform_(-bound, bound, generator=g))
        self.requires_grad_(False)

    @torch.no_grad()
    def score(self, media: Any, prompts: Sequence[str]) -> torch.Tensor:
        video, _ = media_tensors(media)
        _check(video, prompts)
        pooled = video.float().mean((2, 3, 4))
        if pooled.shape[1] != self.fc1.in_features:
            raise ValueError(f"mlp_scorer expects {self.fc1.in_features} latent channels; got {pooled.shape[1]}")
        if self.fc1.weight.device != pooled.device:
            self.to(pooled.device)
        h = torch.nn.functional.gelu(self.fc1(pooled))
        return torch.tanh(self.fc2(h)).squeeze(-1)


class _Gated:
    package = ""
    name = ""
    reason = ""

    def __init__(self, **_: Any) -> None:
        why = f": {self.reason}" if self.reason else ""
        raise RuntimeError(f"the {self.name!r} reward needs the {self.package!r} package, which avgen_b200 does not "
                           f"depend on{why}; install it and register the reward through the "
                           f"{REWARD_ENTRY_POINT_GROUP!r} entry-point group")

    def score(self, media: Any, prompts: Sequence[str]) -> torch.Tensor:
        raise RuntimeError(f"{self.name} is not available")


class HPSv2Reward(_Gated):
    package, name, reason = "hpsv2", "hps_v2", "it pins an old pytest that modern environments cannot hold"


class PickScoreReward(_Gated):
    package, name = "transformers", "pick_score"


class VideoScoreReward(_Gated):
    package, name = "transformers", "video_score"


_REWARDS: dict[str, Callable[..., RewardModel]] = {}


def register_reward(name: str) -> Callable[[Callable[..., Any]], Callable[..., Any]]:
    def deco(factory: Callable[..., Any]) -> Callable[..., Any]:
        if name in _REWARDS:
            raise KeyError(f"reward {name!r} is already registered")
        _REWARDS[name] = factory
        return factory

    return deco


def _load_plugins() -> None:
    from avgen_b200._plugins import load_entry_points

    def accept(name: str, obj: object) -> None:
        if not callable(obj):
            raise TypeError(f"entry point {name!r} of {REWARD_ENTRY_POINT_GROUP!r} must be a callable returning a "
                            f"RewardModel; got {type(obj).__name__}")
        _REWARDS.setdefault(name, obj)  # type: ignore[arg-type]

    load_entry_points(REWARD_ENTRY_POINT_GROUP, accept)


def build_reward(name: str, **options: Any) -> RewardModel:
    _load_plugins()
    try:
        factory = _REWARDS[name]
    except KeyError:
        raise KeyError(f"unknown reward {name!r}; registered rewards are {list_rewards()}") from None
    return factory(**options)


def list_rewards() -> tuple[str, ...]:
    _load_plugins()
    return tuple(sorted(_REWARDS))


for _name, _factory in (("temporal_consistency", TemporalConsistencyReward), ("motion_magnitude",
                        MotionMagnitudeReward), ("av_sync_proxy", AVSyncProxyReward), ("mlp_scorer", MLPScorerReward),
                        ("hps_v2", HPSv2Reward), ("pick_score", PickScoreReward), ("video_score", VideoScoreReward)):
    register_reward(_name)(_factory)


class RunningNormalizer:
    """Running mean/variance (exact pooled statistics, or an EMA with ``momentum``)."""

    __slots__ = ("_count", "_mean", "_var", "epsilon", "momentum")

    def __init__(self, *, momentum: float | None = None, epsilon: float = 1e-6) -> None:
        if momentum is not None and not 0.0 < momentum < 1.0:
            raise ValueError(f"momentum must be in (0, 1) or None; got {momentum!r}")
        if epsilon <= 0.0:
            raise ValueError(f"epsilon must be positive; got {epsilon!r}")
        self.momentum, self.epsilon = momentum, epsilon
        self._count, self._mean, self._var = 0.0, 0.0, 1.0

    def update(self, values: torch.Tensor) -> None:
        n = values.numel()
        if n == 0:
            return
        m = float(values.float().mean())
        v = float(values.float().var(unbiased=False))
        if self.momentum is not None:
            k = self.momentum
            self._mean = k * self._mean + (1 - k) * m
            self._var = k * self._var + (1 - k) * v
            self._count += n
            return
        tot = self._count + n
        d = m - self._mean
        self._mean += d * n / tot
        self._var = (self._var * self._count + v * n + d * d * self._count * n / tot) / tot
        self._count = tot

    def normalize(self, values: torch.Tensor) -> torch.Tensor:
        if self._count == 0.0:
            return values
        return (values - self._mean) / (max(self._var, 0.0) ** 0.5 + self.epsilon)

    def state_dict(self) -> dict[str, float]:
        return {"count": self._count, "mean": self._mean, "variance": self._var}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        for k in ("count", "mean", "variance"):
            if k not in state:
                raise KeyError(f"missing normalizer statistic {k!r}")
        self._count, self._mean, self._var = float(state["count"]), float(state["mean"]), float(state["variance"])


@dataclass(slots=True)
class CompositeReward:
    components: tuple[tuple[RewardModel, float], ...]
    normalization: str = "running"
    momentum: float | None = None
    _normalizers: list[RunningNormalizer] = field(default_factory=list, repr=False)

    def __post_init__(self) -> None:
        if not self.components:
            raise ValueError("CompositeReward needs at least one component")
        if self.normalization not in {"none", "batch", "running"}:
            raise ValueError(f"normalization must be 'none', 'batch' or 'running'; got {self.normalization!r}")
        self._normalizers = [RunningNormalizer(momentum=self.momentum) for _ in self.components]

    def component_scores(self, media: Any, prompts: Sequence[str]) -> dict[str, torch.Tensor]:
        return {str(getattr(r, "name", None) or f"reward_{i}"): r.score(media, prompts).float()
                for i, (r, _) in enumerate(self.components)}

    def score(self, media: Any, prompts: Sequence[str]) -> torch.Tensor:
        total: torch.Tensor | None = None
        for i, (reward, weight) in enumerate(self.components):
            v = reward.score(media, prompts).float()
            if self.normalization == "batch":
                v = (v - v.mean()) / (v.std(unbiased=False) + 1e-6)
            elif self.normalization == "running":
                n = self._normalizers[i]
                normed = n.normalize(v)
                n.update(v)
                v = normed
            total = v * weight if total is None else total + v * weight
        assert total is not None
        return total

    def state_dict(self) -> dict[str, Any]:
        return {f"component_{i}": n.state_dict() for i, n in enumerate(self._normalizers)}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        for i, n in enumerate(self._normalizers):
            key = f"component_{i}"
            if key not in state:
                raise KeyError(f"missing normalizer state {key!r}")
            n.load_state_dict(state[key])
