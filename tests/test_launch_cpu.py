"""Launch layer and simulator gate on CPU: pinned plans pass their floors with the
mesh built at full world size on the fake process group, the Slurm launcher
parses, and the preflight check reports a missing GPU instead of crashing."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import torch

import avgen_b200.launch as launch
from avgen_b200.simulate.gate import DEFAULT_PLANS, check_plans


def test_pinned_plans_pass_and_a_tight_floor_fails(tmp_path: Path) -> None:
    results, problems = check_plans(DEFAULT_PLANS)
    assert not problems, problems
    assert results["2b_64k_world512"]["memory_gib"] < 170
    spec = json.loads(DEFAULT_PLANS.read_text())
    spec["plans"] = [dict(spec["plans"][0], min_mfu=0.99)]
    path = tmp_path / "plans.json"
    path.write_text(json.dumps(spec))
    _, problems = check_plans(path, build_mesh=False)
    assert problems and "below floor" in problems[0]


def test_slurm_launcher_parses() -> None:
    script = Path(launch.__file__).with_name("train.slurm")
    assert subprocess.run(["bash", "-n", str(script)], check=False).returncode == 0
    text = script.read_text()
    assert "--max-restarts 3" in text and "avgen_b200.cli.main train" in text


def test_preflight_reports_missing_gpu() -> None:
    if torch.cuda.is_available():
        return
    from avgen_b200.launch.preflight import run_checks

    failures = run_checks(world_size=8)
    assert any("no CUDA device" in f for f in failures)


def test_checked_build_flag_compiles_the_tma_checks() -> None:
    """``AVGEN_KCHECK=1`` adds ``-DAVGEN_KCHECK`` to the nvcc flags, and the TMA helpers
    carry the coordinate check only in that build."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = ("import runpy, sys; sys.argv = ['setup.py', '--name']; "
            "g = runpy.run_path('setup.py', run_name='flags'); print('-DAVGEN_KCHECK' in g['NVCC_FLAGS'])")
    for flag, want in (("1", "True"), ("0", "False")):
        out = subprocess.run([sys.executable, "-c", code], cwd=root, env=dict(os.environ, AVGEN_KCHECK=flag),
                             capture_output=True, text=True, timeout=300)
        assert out.stdout.strip().splitlines()[-1] == want, out.stderr[-2000:]
    header = (root / "avgen_b200" / "csrc" / "include" / "sm100.cuh").read_text()
    assert "#ifdef AVGEN_KCHECK" in header and header.count("AVGEN_TMA_X_CHECK(x);") == 4
