"""Shared CLI helpers: exit codes, error lines, prompt files, JSON output."""
from __future__ import annotations

import json
import sys
from pathlib import Path
from typing import Any

__all__ = ["EXIT_CONFIG", "EXIT_ERROR", "EXIT_INTERRUPT", "EXIT_OK", "EXIT_USAGE", "emit_json", "fail",
           "read_prompts", "version"]

EXIT_OK = 0
EXIT_ERROR = 1
EXIT_USAGE = 2
EXIT_CONFIG = 3
EXIT_INTERRUPT = 130


def fail(message: str, *, code: int = EXIT_ERROR) -> int:
    sys.stderr.write(f"avgen-b200: error: {message}\n")
    return code


def emit_json(payload: Any) -> None:
    sys.stdout.write(json.dumps(payload, indent=2, sort_keys=True, default=str) + "\n")


def read_prompts(prompt: str | None, prompt_file: str | None) -> list[str]:
    """One prompt, or a newline-delimited file (blank lines and ``#`` comments skipped)."""
    if prompt is not None:
        return [prompt]
    if prompt_file:
        lines = Path(prompt_file).read_text(encoding="utf-8").splitlines()
        prompts = [ln.strip() for ln in lines if ln.strip() and not ln.lstrip().startswith("#")]
        if not prompts:
            raise ValueError(f"{prompt_file} holds no prompts")
        return prompts
    raise ValueError("give --prompt or --prompt-file")


def version() -> str:
    from importlib.metadata import PackageNotFoundError
    from importlib.metadata import version as _v

    try:
        return _v("avgen_b200")
    except PackageNotFoundError:
        return "0.1.0 (source tree)"
