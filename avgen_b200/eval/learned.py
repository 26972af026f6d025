"""Learned (feature-network) metrics: declared, gated on their backends, never
substituted (avgen/eval/learned.py:62-507 API).

``fvd``, ``fid``, ``clip_score``, ``video_score`` and ``hps`` are declared with
what they need and what they measure. Building one whose backend or weights are
missing raises :class:`MissingBackendError` instead of computing something else
under the same name. :func:`frechet_distance` is the shared closed form.
"""
from __future__ import annotations

import importlib.util
from collections.abc import Callable, Mapping
from dataclasses import dataclass, field
from typing import Any

import torch

from avgen_b200.eval.protocols import MetricError

__all__ = ["LearnedMetricSpec", "MissingBackendError", "available_learned_metrics", "build_learned_metric",
           "describe_learned_metrics", "frechet_distance", "learned_metric_available", "learned_metric_summary",
           "list_learned_metrics", "merge_feature_banks", "register_learned_metric", "require_backend"]


class MissingBackendError(RuntimeError):
    """A learned metric's package, weights or implementation is not available here."""


@dataclass(frozen=True, slots=True)
class LearnedMetricSpec:
    name: str
    extra: str
    modules: tuple[str, ...]
    weights: str
    measures: str
    caveat: str
    factory: Callable[..., Any] | None = field(default=None, repr=False)

    def install_hint(self) -> str:
        return f"pip install {' '.join(self.modules)}  (and: {self.weights})"

    def missing_modules(self) -> tuple[str, ...]:
        return tuple(m for m in self.modules if importlib.util.find_spec(m.split(".")[0]) is None)


_LEARNED: dict[str, LearnedMetricSpec] = {}


def register_learned_metric(spec: LearnedMetricSpec) -> LearnedMetricSpec:
    if spec.name in _LEARNED:
        raise ValueError(f"learned metric {spec.name!r} is already registered")
    _LEARNED[spec.name] = spec
    return spec


def list_learned_metrics() -> tuple[str, ...]:
    return tuple(sorted(_LEARNED))


def _spec(name: str) -> LearnedMetricSpec:
    if name not in _LEARNED:
        raise MetricError(f"{name!r} is not a declared learned metric; declared: {', '.join(list_learned_metrics())}")
    return _LEARNED[name]


def learned_metric_available(name: str) -> bool:
    return not _spec(name).missing_modules()


def available_learned_metrics() -> dict[str, bool]:
    return {n: learned_metric_available(n) and _spec(n).factory is not None for n in list_learned_metrics()}


def describe_learned_metrics() -> dict[str, dict[str, str]]:
    out: dict[str, dict[str, str]] = {}
    for name in list_learned_metrics():
        spec = _spec(name)
        missing = spec.missing_modules()
        status = (f"backend missing: {', '.join(missing)}" if missing else
                  "declared; no implementation ships (register your own)" if spec.factory is None else "available")
        out[name] = {"measures": spec.measures, "caveat": spec.caveat, "requires": spec.install_hint(),
                     "status": status}
    return out


def require_backend(name: str) -> LearnedMetricSpec:
    spec = _spec(name)
    missing = spec.missing_modules()
    if missing:
        raise MissingBackendError(f"metric {name!r} needs {', '.join(missing)}, which is not installed; install it "
                                  f"with: {spec.install_hint()}\nNo other metric is substituted under this name.")
    return spec


def build_learned_metric(name: str, **kwargs: Any) -> Any:
    spec = require_backend(name)
    if spec.factory is None:
        raise MissingBackendError(f"metric {name!r} is declared but no implementation ships (it measures: "
                                  f"{spec.measures}); register one with register_learned_metric() or record an "
                                  "externally computed value in the report's `external` section")
    return spec.factory(**kwargs)


def _psd_sqrt(m: torch.Tensor) -> torch.Tensor:
    vals, vecs = torch.linalg.eigh(m)
    return (vecs * vals.clamp_min(0.0).sqrt()[None]) @ vecs.T


def frechet_distance(features_a: torch.Tensor, features_b: torch.Tensor, *, epsilon: float = 1e-6) -> float:
    """``|mu_a - mu_b|^2 + tr(C_a) + tr(C_b) - 2 tr((C_a^1/2 C_b C_a^1/2)^1/2)`` in float64,
    with a small ridge on both covariances."""
    if features_a.ndim != 2 or features_b.ndim != 2:
        raise MetricError(f"frechet_distance expects (n, d) matrices; got {tuple(features_a.shape)} and "
                          f"{tuple(features_b.shape)}")
    if features_a.shape[1] != features_b.shape[1]:
        raise MetricError(f"feature dimensions differ: {features_a.shape[1]} vs {features_b.shape[1]}")
    if features_a.shape[0] < 2 or features_b.shape[0] < 2:
        raise MetricError("frechet_distance needs at least two samples per set to estimate a covariance")
    a, b = features_a.detach().double(), features_b.detach().double()
    ridge = epsilon * torch.eye(a.shape[1], dtype=torch.float64, device=a.device)
    ca, cb = a.T.cov() + ridge, b.T.cov() + ridge
    ra = _psd_sqrt(ca)
    cross = _psd_sqrt(ra @ cb @ ra)
    return float((a.mean(0) - b.mean(0)).pow(2).sum() + ca.trace() + cb.trace() - 2.0 * cross.trace())


class _CLIPScore:
    """Prompt/frame cosine similarity in CLIP's joint space (needs ``transformers`` and
    local CLIP weights; nothing is downloaded implicitly)."""

    name = "clip_score"
    required_inputs = ("video", "prompts")
    pixel_space_only = True

    def __init__(self, *, model_id: str = "openai/clip-vit-large-patch14", device: str = "cpu") -> None:
        try:
            from transformers import CLIPModel, CLIPProcessor
            self._model = CLIPModel.from_pretrained(model_id, local_files_only=True).to(device).eval()
            self._proc = CLIPProcessor.from_pretrained(model_id, local_files_only=True)
        except Exception as err:  # weights absent offline
            raise MissingBackendError(f"clip_score could not load {model_id!r} locally: {err}") from err
        self._device = device
        self._sum, self._n = 0.0, 0

    @torch.no_grad()
    def update(self, **inputs: Any) -> None:
        video, prompts = inputs["video"], list(inputs["prompts"])
        frames = ((video.float().clamp(-1, 1) + 1) * 127.5).to(torch.uint8)  # [B, C, T, H, W] in [-1, 1]
        for i, prompt in enumerate(prompts):
            imgs = [frames[i, :, t].permute(1, 2, 0).cpu().numpy() for t in range(frames.shape[2])]
            batch = self._proc(text=[prompt], images=imgs, return_tensors="pt", padding=True).to(self._device)
            out = self._model(**batch)
            img = torch.nn.functional.normalize(out.image_embeds, dim=-1)
            txt = torch.nn.functional.normalize(out.text_embeds, dim=-1)
            self._sum += float((img @ txt.T).mean())
            self._n += 1

    def compute(self) -> dict[str, float]:
        return {"clip_score/cosine": self._sum / self._n} if self._n else {}

    def reset(self) -> None:
        self._sum, self._n = 0.0, 0

    def state(self) -> dict[str, tuple[float, float]]:
        return {"cosine": (self._sum, float(self._n))}

    def merge(self, other: Mapping[str, tuple[float, float]]) -> None:
        s, n = other.get("cosine", (0.0, 0.0))
        self._sum += s
        self._n += int(n)


for _spec_args in (
        ("fvd", "", ("torch",), "an I3D or VideoMAE feature extractor you supply",
         "Frechet distance between video-feature distributions of real and generated clips",
         "not comparable across implementations: feature network, sample and frame counts, resolution and resize "
         "filter each move it more than most reported differences", None),
        ("fid", "", ("torchvision",), "InceptionV3 pool3 weights",
         "Frechet distance between per-frame image-feature distributions",
         "an image metric applied to frames: blind to every temporal property", None),
        ("clip_score", "text", ("transformers",), "a local CLIP checkpoint, e.g. openai/clip-vit-large-patch14",
         "cosine similarity between prompt and per-frame image embeddings",
         "saturated and gameable; cannot separate two videos that both contain the prompted content", _CLIPScore),
        ("video_score", "text", ("transformers",), "a VideoScore reward checkpoint",
         "a learned proxy for human quality judgements of generated video",
         "a reward model of one generation distribution; off-distribution numbers do not track preference", None),
        ("hps", "text", ("transformers",), "a Human Preference Score checkpoint",
         "a learned human-preference score over generated media",
         "trained on image preferences; ignores motion when applied to frames", None)):
    register_learned_metric(LearnedMetricSpec(*_spec_args))


def learned_metric_summary() -> str:
    rows = describe_learned_metrics()
    if not rows:
        return "  (none declared)"
    width = max(len(n) for n in rows)
    lines: list[str] = []
    for name, d in rows.items():
        lines.append(f"  {name.ljust(width)}  {d['status']}")
        lines.append(f"  {' ' * width}  requires: {d['requires']}")
    return "\n".join(lines)


def merge_feature_banks(banks: Mapping[str, torch.Tensor]) -> torch.Tensor:
    """Concatenate per-rank feature banks in key order (deterministic across runs)."""
    if not banks:
        raise MetricError("merge_feature_banks was given no feature banks")
    parts = [banks[k] for k in sorted(banks)]
    dims = {p.shape[-1] for p in parts}
    if len(dims) != 1:
        raise MetricError(f"feature banks disagree in dimension: {sorted(dims)}")
    return torch.cat(parts, 0)
