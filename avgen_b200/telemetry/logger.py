"""Rank-gated experiment loggers (avgen/telemetry/logger.py:68-655).

Only rank 0 writes by default. Backends: console (aligned columns), JSONL (the
format of record: one JSON object per step), TensorBoard and Weights & Biases
(optional packages, imported on construction), a failure-tolerant fan-out and a
no-op. ``build_logger`` maps backend names from the config.
"""
from __future__ import annotations

import json
import logging
import os
import sys
import time
from collections.abc import Mapping, Sequence
from pathlib import Path
from typing import Any, Protocol, runtime_checkable

__all__ = ["ConsoleLogger", "JSONLLogger", "Logger", "MultiLogger", "NoOpLogger", "RankGatedLogger",
           "TensorBoardLogger", "WandbLogger", "build_logger"]

_LOG = logging.getLogger("avgen_b200.telemetry")


@runtime_checkable
class Logger(Protocol):
    def log_metrics(self, metrics: Mapping[str, float], step: int) -> None: ...

    def log_config(self, config: Mapping[str, Any]) -> None: ...

    def log_artifact(self, path: str | os.PathLike[str]) -> None: ...

    def close(self) -> None: ...


def _rank() -> int:
    try:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            return dist.get_rank()
    except ImportError:
        pass
    return int(os.environ.get("RANK", "0"))


class RankGatedLogger:
    """Base: subclasses implement ``_metrics`` / ``_config`` / ``_artifact`` / ``_close``."""

    def __init__(self, *, rank: int | None = None, all_ranks: bool = False) -> None:
        self._rank = _rank() if rank is None else rank
        self._enabled = all_ranks or self._rank == 0
        self._closed = False

    @property
    def enabled(self) -> bool:
        return self._enabled and not self._closed

    def log_metrics(self, metrics: Mapping[str, float], step: int) -> None:
        if self.enabled:
            self._metrics({k: float(v) for k, v in metrics.items()}, int(step))

    def log_config(self, config: Mapping[str, Any]) -> None:
        if self.enabled:
            self._config(dict(config))

    def log_artifact(self, path: str | os.PathLike[str]) -> None:
        if self.enabled:
            self._artifact(Path(path))

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            if self._enabled:
                self._close()

    def _metrics(self, metrics: dict[str, float], step: int) -> None:
        raise NotImplementedError

    def _config(self, config: dict[str, Any]) -> None:
        pass

    def _artifact(self, path: Path) -> None:
        pass

    def _close(self) -> None:
        pass

    def __enter__(self) -> RankGatedLogger:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()


class NoOpLogger(RankGatedLogger):
    def _metrics(self, metrics: dict[str, float], step: int) -> None:
        pass


class ConsoleLogger(RankGatedLogger):
    def __init__(self, *, stream: Any = None, keys: Sequence[str] | None = None, **kw: Any) -> None:
        super().__init__(**kw)
        self._stream = stream or sys.stdout
        self._keys = tuple(keys) if keys else None

    def _metrics(self, metrics: dict[str, float], step: int) -> None:
        keys = self._keys or tuple(sorted(metrics))
        parts = [f"step {step:>7d}"]
        for k in keys:
            if k in metrics:
                v = metrics[k]
                parts.append(f"{k.split('/')[-1]} {v:.4g}" if abs(v) < 1e5 else f"{k.split('/')[-1]} {v:.3e}")
        print(" | ".join(parts), file=self._stream, flush=True)


class JSONLLogger(RankGatedLogger):
    """One JSON object per ``log_metrics`` call: ``{"step", "time", **metrics}``."""

    def __init__(self, path: str | os.PathLike[str], **kw: Any) -> None:
        super().__init__(**kw)
        self._path = Path(path)
        self._fh = None
        if self._enabled:
            self._path.parent.mkdir(parents=True, exist_ok=True)
            self._fh = open(self._path, "a", encoding="utf-8")

    @property
    def path(self) -> Path:
        return self._path

    def _metrics(self, metrics: dict[str, float], step: int) -> None:
        assert self._fh is not None
        self._fh.write(json.dumps({"step": step, "time": time.time(), **metrics}, sort_keys=True) + "\n")
        self._fh.flush()

    def _config(self, config: dict[str, Any]) -> None:
        assert self._fh is not None
        self._fh.write(json.dumps({"config": config}, default=str, sort_keys=True) + "\n")
        self._fh.flush()

    def _close(self) -> None:
        if self._fh is not None:
            self._fh.close()
            self._fh = None


class TensorBoardLogger(RankGatedLogger):
    def __init__(self, log_dir: str | os.PathLike[str], **kw: Any) -> None:
        super().__init__(**kw)
        self._writer = None
        if self._enabled:
            try:
                from torch.utils.tensorboard import SummaryWriter
            except ImportError as exc:
                raise RuntimeError("the tensorboard logger needs the 'tensorboard' package") from exc
            self._writer = SummaryWriter(log_dir=str(log_dir))

    def _metrics(self, metrics: dict[str, float], step: int) -> None:
        for k, v in metrics.items():
            self._writer.add_scalar(k, v, step)

    def _config(self, config: dict[str, Any]) -> None:
        self._writer.add_text("config", json.dumps(config, default=str, indent=2))

    def _close(self) -> None:
        self._writer.close()


class WandbLogger(RankGatedLogger):
    def __init__(self, *, project: str = "avgen", name: str = "", config: Mapping[str, Any] | None = None,
                 **kw: Any) -> None:
        super().__init__(**kw)
        self._run = None
        if self._enabled:
            try:
                import wandb
            except ImportError as exc:
                raise RuntimeError("the wandb logger needs the 'wandb' package") from exc
            self._run = wandb.init(project=project, name=name or None, config=dict(config or {}))

    def _metrics(self, metrics: dict[str, float], step: int) -> None:
        self._run.log(metrics, step=step)

    def _config(self, config: dict[str, Any]) -> None:
        self._run.config.update(config, allow_val_change=True)

    def _artifact(self, path: Path) -> None:
        self._run.save(str(path))

    def _close(self) -> None:
        self._run.finish()


class MultiLogger:
    """Fans out to several loggers; one failing backend never stops the others."""

    def __init__(self, loggers: Sequence[Logger]) -> None:
        self._loggers = tuple(loggers)
        self._failed: set[int] = set()

    @property
    def loggers(self) -> tuple[Logger, ...]:
        return self._loggers

    def _each(self, method: str, *args: Any) -> None:
        for i, lg in enumerate(self._loggers):
            if i in self._failed:
                continue
            try:
                getattr(lg, method)(*args)
            except Exception as exc:  # noqa: BLE001 - a logging failure never kills training
                self._failed.add(i)
                _LOG.warning("logger %s failed in %s (%s); disabled", type(lg).__name__, method, exc)

    def log_metrics(self, metrics: Mapping[str, float], step: int) -> None:
        self._each("log_metrics", metrics, step)

    def log_config(self, config: Mapping[str, Any]) -> None:
        self._each("log_config", config)

    def log_artifact(self, path: str | os.PathLike[str]) -> None:
        self._each("log_artifact", path)

    def close(self) -> None:
        self._each("close")


def build_logger(names: Sequence[str], *, output_dir: str | os.PathLike[str] = "runs/default",
                 jsonl_path: str = "", tensorboard_dir: str = "", project: str = "avgen", run_name: str = "",
                 config: Mapping[str, Any] | None = None) -> MultiLogger:
    out = Path(output_dir)
    loggers: list[Logger] = []
    for name in names:
        if name == "console":
            loggers.append(ConsoleLogger())
        elif name == "jsonl":
            loggers.append(JSONLLogger(jsonl_path or out / "metrics.jsonl"))
        elif name == "tensorboard":
            loggers.append(TensorBoardLogger(tensorboard_dir or out / "tensorboard"))
        elif name == "wandb":
            loggers.append(WandbLogger(project=project, name=run_name, config=config))
        elif name == "noop":
            loggers.append(NoOpLogger())
        else:
            raise ValueError(f"unknown logger {name!r}")
    return MultiLogger(loggers)
