"""Run every shipped example as its own program (a fresh interpreter each), so a
drifted public signature fails here rather than on a user's machine."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
EXAMPLES = sorted((REPO / "examples").glob("*.py"))


def test_examples_are_found() -> None:
    assert len(EXAMPLES) >= 5


@pytest.mark.parametrize("script", EXAMPLES, ids=lambda p: p.stem)
def test_example_runs(script: Path) -> None:
    env = {**os.environ, "PYTHONPATH": os.pathsep.join(filter(None, (str(REPO), os.environ.get("PYTHONPATH"))))}
    result = subprocess.run([sys.executable, str(script)], cwd=REPO, env=env, capture_output=True, text=True,
                            timeout=600)
    assert result.returncode == 0, f"{script.name}\n{result.stdout[-2000:]}\n{result.stderr[-2000:]}"
    assert result.stdout.strip()
