"""Pre-launch checks for a B200 node (scripts/preflight.sh role in the reference).

    python -m avgen_b200.launch.preflight [--world-size N] [--tests] [--measure]

1. torch, CUDA, and that every visible device is sm_100 (the only arch the
   in-tree kernels are built for);
2. the in-tree extension loads and the device error word reads zero;
3. peer access between every pair of visible GPUs (the fused NVLink paths need
   it) and the NVLink topology (``nvidia-smi topo -m``, read only);
4. the simulator's plan for this node's GPU count;
5. ``--tests``: the single-device GPU test suite;
6. ``--measure``: peer-copy bandwidth between GPU 0 and 1, to feed
   :func:`avgen_b200.simulate.calibrate_from_busbw`.

Exits non-zero when a check fails. Reads settings only; changes nothing on the GPUs.
"""
from __future__ import annotations

import argparse
import shutil
import subprocess
import sys

__all__ = ["main", "run_checks"]


def _say(title: str) -> None:
    sys.stdout.write(f"\n== {title} ==\n")


def run_checks(*, world_size: int | None = None, tests: bool = False, measure: bool = False) -> list[str]:
    """Run the checks and return the list of failures (empty when all pass)."""
    import torch

    failures: list[str] = []
    _say("1. torch and devices")
    sys.stdout.write(f"   torch {torch.__version__}, CUDA available: {torch.cuda.is_available()}\n")
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for i in range(n):
        cap = torch.cuda.get_device_capability(i)
        free, total = torch.cuda.mem_get_info(i)
        sys.stdout.write(f"   cuda:{i} {torch.cuda.get_device_name(i)} sm_{cap[0]}{cap[1]} "
                         f"{total / 2**30:.0f} GiB ({free / 2**30:.0f} free)\n")
        if cap != (10, 0):
            failures.append(f"cuda:{i} is sm_{cap[0]}{cap[1]}; the kernels are built for sm_100a only")
    if n == 0:
        failures.append("no CUDA device visible")
    _say("2. native extension")
    try:
        from avgen_b200.ops._ext import check_errors, load

        mod = load()
        sys.stdout.write(f"   loaded {mod.__file__}\n")
        for i in range(n):
            code = check_errors(i)
            if code:
                failures.append(f"cuda:{i} error word is {code}")
    except Exception as err:  # noqa: BLE001
        failures.append(f"extension failed to load: {err}")
    _say("3. peer access and topology")
    for i in range(n):
        for j in range(n):
            if i != j and not torch.cuda.can_device_access_peer(i, j):
                failures.append(f"cuda:{i} cannot access cuda:{j} (NVLink peer access is required)")
    if n > 1 and not any("cannot access" in f for f in failures):
        sys.stdout.write(f"   all {n * (n - 1)} ordered GPU pairs have peer access\n")
    if shutil.which("nvidia-smi"):
        topo = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True, text=True, check=False)
        sys.stdout.write("".join("   " + ln + "\n" for ln in topo.stdout.splitlines()[: n + 2]))
    _say("4. plan for this node")
    from avgen_b200.cli.main import main as cli

    ws = world_size or max(1, n)
    if cli(["plan", "--world-size", str(ws), "--gpu", "b200", "--seq-len", "65536", "--params", "2e9",
            "--depth", "32", "--width", "2560", "--top-k", "3"]) != 0:
        failures.append("plan failed")
    if tests:
        _say("5. GPU tests")
        rc = subprocess.run([sys.executable, "-m", "pytest", "-m", "gpu", "-q", "-x"], check=False).returncode
        if rc:
            failures.append(f"GPU tests exited {rc}")
    if measure and n > 1:
        _say("6. peer copy bandwidth")
        src = torch.empty(1 << 30, dtype=torch.uint8, device="cuda:0")
        dst = torch.empty(1 << 30, dtype=torch.uint8, device="cuda:1")
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize(0)
        torch.cuda.synchronize(1)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.device(0):
            ev0.record()
            for _ in range(10):
                dst.copy_(src, non_blocking=True)
            ev1.record()
        ev1.synchronize()
        gbs = 10 * src.numel() / (ev0.elapsed_time(ev1) * 1e-3) / 1e9
        sys.stdout.write(f"   cuda:0 -> cuda:1: {gbs:.0f} GB/s\n")
    return failures


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="python -m avgen_b200.launch.preflight", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--world-size", type=int, default=None)
    p.add_argument("--tests", action="store_true")
    p.add_argument("--measure", action="store_true")
    a = p.parse_args(argv)
    failures = run_checks(world_size=a.world_size, tests=a.tests, measure=a.measure)
    _say("result")
    for f in failures:
        sys.stdout.write(f"   ! {f}\n")
    sys.stdout.write("   ok\n" if not failures else f"   {len(failures)} check(s) failed\n")
    return 1 if failures else 0


if __name__ == "__main__":
    raise SystemExit(main())
