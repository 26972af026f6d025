"""``avgen-b200 info``: versions, devices, kernels and subsystem health (avgen/cli/info.py API)."""
from __future__ import annotations

import argparse
import importlib
import platform
import sys
from typing import Any

from avgen_b200.cli._common import EXIT_OK, version

__all__ = ["add_parser", "run"]


def add_parser(subparsers: Any) -> None:
    p = subparsers.add_parser("info", help="report versions, devices, kernels and optional extras")
    p.add_argument("--metrics", action="store_true", help="also list evaluation metrics")
    p.set_defaults(handler=run)


def _ver(name: str) -> str:
    try:
        mod = importlib.import_module(name)
    except Exception:  # noqa: BLE001 - report absence, never fail
        return "not installed"
    return str(getattr(mod, "__version__", "installed"))


def run(args: argparse.Namespace) -> int:
    import torch

    from avgen_b200.ops import _ext

    lines = [f"avgen-b200   {version()}", f"python       {platform.python_version()}", f"torch        {torch.__version__}",
             f"cuda         {torch.version.cuda}", f"nccl         "
             f"{'.'.join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else 'n/a'}"]
    if torch.cuda.is_available():
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            lines.append(f"device {i}     {p.name} sm_{p.major}{p.minor} {p.multi_processor_count} SMs "
                         f"{p.total_memory / 2**30:.0f} GiB")
    else:
        lines.append("device       none (CPU only: kernels cannot run here)")
    lines.append(f"kernels      {'built (avgen_b200._C)' if _ext.available() else 'NOT BUILT (python setup.py build_ext --inplace)'}")
    for name in ("safetensors", "yaml", "diffusers", "transformers", "torchao", "av", "pyarrow"):
        lines.append(f"{name:12s} {_ver(name)}")
    if args.metrics:
        try:
            from avgen_b200.eval import list_metrics

            for m in list_metrics():
                lines.append(f"metric       {m}")
        except ImportError:
            lines.append("metric       (eval package unavailable)")
    sys.stdout.write("\n".join(lines) + "\n")
    return EXIT_OK
