"""Pinned, comparable evaluation reports (avgen/eval/report.py:57-502 API).

An :class:`EvalReport` carries the full :class:`EvalPin` (sampler, steps,
guidance, seed, prompt-set digest, resolution, latent or pixel space, codec,
precision, metric parameters). :func:`compare_reports` refuses two reports whose
pins differ in anything but the checkpoint unless the caller names the field it
is varying on purpose. The JSON layout (``report_version`` 1) is kept so
reports written by either framework compare.
"""
from __future__ import annotations

import hashlib
import json
import platform
from collections.abc import Iterable, Mapping, Sequence
from dataclasses import asdict, dataclass, field, replace
from datetime import UTC, datetime
from pathlib import Path
from typing import Any, ClassVar

__all__ = ["REPORT_VERSION", "EvalPin", "EvalReport", "IncomparableReports", "capture_environment",
           "compare_reports", "format_comparison", "prompt_set_digest"]

REPORT_VERSION = 1


class IncomparableReports(ValueError):
    def __init__(self, differences: Mapping[str, tuple[Any, Any]]) -> None:
        self.differences = dict(differences)
        detail = "; ".join(f"{k}: {a!r} vs {b!r}" for k, (a, b) in sorted(self.differences.items()))
        super().__init__(f"refusing to compare evaluation reports with different pinned settings: {detail}. Re-run "
                         "one under the other's settings, or pass allow=(...) naming the field varied on purpose")


def prompt_set_digest(prompts: Sequence[str]) -> str:
    """``"<count>:<16 hex chars of sha256 over NUL-terminated prompts>"``."""
    h = hashlib.sha256()
    for p in prompts:
        h.update(p.encode("utf-8") + b"\x00")
    return f"{len(prompts)}:{h.hexdigest()[:16]}"


@dataclass(frozen=True, slots=True)
class EvalPin:
    checkpoint: str = ""
    sampler: str = "euler"
    steps: int = 30
    guidance: float = 5.0
    guidance_rescale: float = 0.0
    negative_prompt: str = ""
    seed: int = 0
    num_samples: int = 0
    prompt_digest: str = ""
    frames: int = 0
    height: int = 0
    width: int = 0
    decoded: bool = False
    codec: str = ""
    precision: str = "bfloat16"
    metrics: dict[str, str] = field(default_factory=dict)

    COMPARABLE_EXEMPT: ClassVar[tuple[str, ...]] = ("checkpoint",)

    def __post_init__(self) -> None:
        if self.steps < 1:
            raise ValueError(f"EvalPin.steps must be >= 1; got {self.steps!r}")
        if self.num_samples < 0:
            raise ValueError(f"EvalPin.num_samples must be >= 0; got {self.num_samples!r}")

    def to_dict(self) -> dict[str, Any]:
        d = asdict(self)
        d["metrics"] = dict(sorted(self.metrics.items()))
        return d

    def differences(self, other: EvalPin, *, allow: Iterable[str] = ()) -> dict[str, tuple[Any, Any]]:
        skip = set(self.COMPARABLE_EXEMPT) | set(allow)
        a, b = self.to_dict(), other.to_dict()
        return {k: (a[k], b[k]) for k in a if k not in skip and a[k] != b[k]}

    def describe(self) -> str:
        space = "pixels" if self.decoded else "latents"
        return (f"{self.sampler} x{self.steps} cfg={self.guidance} seed={self.seed} {self.frames}x{self.height}x"
                f"{self.width} {space} n={self.num_samples} prompts={self.prompt_digest or 'unset'}")


def capture_environment() -> dict[str, str]:
    env = {"python": platform.python_version(), "platform": platform.platform()}
    try:
        import torch

        env["torch"] = torch.__version__
        if torch.cuda.is_available():
            env["cuda"] = torch.version.cuda or "unknown"
            env["device"] = torch.cuda.get_device_name(0)
    except Exception:  # noqa: BLE001
        env["torch"] = "unavailable"
    return env


@dataclass(frozen=True, slots=True)
class EvalReport:
    pin: EvalPin
    metrics: dict[str, float] = field(default_factory=dict)
    skipped: dict[str, str] = field(default_factory=dict)
    run_name: str = ""
    step: int = 0
    external: dict[str, float] = field(default_factory=dict)
    environment: dict[str, str] = field(default_factory=dict)
    created_at: str = ""
    report_version: int = REPORT_VERSION
    notes: str = ""

    def __post_init__(self) -> None:
        if not self.created_at:
            object.__setattr__(self, "created_at", datetime.now(UTC).isoformat(timespec="seconds"))
        if not self.environment:
            object.__setattr__(self, "environment", capture_environment())

    def to_dict(self) -> dict[str, Any]:
        return {"report_version": self.report_version, "run_name": self.run_name, "step": self.step,
                "created_at": self.created_at, "pin": self.pin.to_dict(), "pin_summary": self.pin.describe(),
                "metrics": dict(sorted(self.metrics.items())), "external": dict(sorted(self.external.items())),
                "skipped": dict(sorted(self.skipped.items())), "environment": dict(sorted(self.environment.items())),
                "notes": self.notes}

    @classmethod
    def from_dict(cls, payload: Mapping[str, Any]) -> EvalReport:
        version = int(payload.get("report_version", 0))
        if version > REPORT_VERSION:
            raise ValueError(f"report_version={version} is newer than this reader ({REPORT_VERSION}); an unknown "
                             "pinned field would be ignored and the comparison it guards could not be trusted")
        pin = dict(payload.get("pin", {}))
        pin.pop("COMPARABLE_EXEMPT", None)
        return cls(pin=EvalPin(**pin), metrics=dict(payload.get("metrics", {})),
                   skipped=dict(payload.get("skipped", {})), run_name=str(payload.get("run_name", "")),
                   step=int(payload.get("step", 0)), external=dict(payload.get("external", {})),
                   environment=dict(payload.get("environment", {})), created_at=str(payload.get("created_at", "")),
                   report_version=version or REPORT_VERSION, notes=str(payload.get("notes", "")))

    def save(self, path: str | Path) -> Path:
        dest = Path(path)
        dest.parent.mkdir(parents=True, exist_ok=True)
        tmp = dest.with_suffix(dest.suffix + ".tmp")
        tmp.write_text(json.dumps(self.to_dict(), indent=2, sort_keys=True), encoding="utf-8")
        tmp.replace(dest)
        return dest

    @classmethod
    def load(cls, path: str | Path) -> EvalReport:
        try:
            payload = json.loads(Path(path).read_text(encoding="utf-8"))
        except (OSError, json.JSONDecodeError) as err:
            raise ValueError(f"cannot read evaluation report {path}: {err}") from err
        return cls.from_dict(payload)

    def with_metrics(self, values: Mapping[str, float]) -> EvalReport:
        return replace(self, metrics={**self.metrics, **values})

    def render(self) -> str:
        bar = "=" * 72
        lines = [bar, f"avgen_b200 evaluation - {self.run_name or '(unnamed run)'} step {self.step}", bar,
                 f"  checkpoint  {self.pin.checkpoint or '(unspecified)'}", f"  settings    {self.pin.describe()}", ""]
        if self.metrics:
            w = max(len(k) for k in self.metrics)
            lines.append("METRICS")
            lines += [f"    {k.ljust(w)}  {v: .6f}" for k, v in sorted(self.metrics.items())]
        else:
            lines.append("METRICS  (none computed)")
        if self.external:
            lines += ["", "EXTERNAL (computed elsewhere)"] + [f"    {k}  {v: .6f}" for k, v in
                                                                sorted(self.external.items())]
        if self.skipped:
            lines += ["", "SKIPPED"] + [f"    {k}: {r}" for k, r in sorted(self.skipped.items())]
        lines.append(bar)
        return "\n".join(lines)


def compare_reports(a: EvalReport, b: EvalReport, *, allow: Iterable[str] = ()) -> dict[str, dict[str, float]]:
    diff = a.pin.differences(b.pin, allow=allow)
    if diff:
        raise IncomparableReports(diff)
    out: dict[str, dict[str, float]] = {}
    for key in sorted(set(a.metrics) | set(b.metrics)):
        row: dict[str, float] = {}
        if key in a.metrics:
            row["a"] = a.metrics[key]
        if key in b.metrics:
            row["b"] = b.metrics[key]
        if "a" in row and "b" in row:
            row["delta"] = row["b"] - row["a"]
            row["relative"] = row["delta"] / row["a"] if row["a"] else float("inf")
        out[key] = row
    return out


def format_comparison(comparison: Mapping[str, Mapping[str, float]], *, left: str = "baseline",
                      right: str = "candidate") -> str:
    if not comparison:
        return "no metrics in common"
    w = max(len(k) for k in comparison)
    header = f"{'metric'.ljust(w)}  {left:>14}  {right:>14}  {'delta':>14}  {'relative':>10}"
    lines = [header, "-" * len(header)]
    for key, row in comparison.items():
        cells = [f"{row[c]:14.6f}" if c in row else " " * 14 for c in ("a", "b", "delta")]
        rel = f"{row['relative']:9.2%}" if "relative" in row else " " * 10
        lines.append(f"{key.ljust(w)}  {cells[0]}  {cells[1]}  {cells[2]}  {rel}")
    return "\n".join(lines)
