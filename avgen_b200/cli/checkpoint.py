"""``avgen-b200 checkpoint {inspect,convert,export}`` (avgen/cli/checkpoint.py API)."""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Any

from avgen_b200.cli._common import EXIT_OK, EXIT_USAGE, emit_json

__all__ = ["add_parser", "run"]


def add_parser(subparsers: Any) -> None:
    p = subparsers.add_parser("checkpoint", help="inspect, reshard or export a checkpoint")
    a = p.add_subparsers(dest="action", metavar="ACTION")
    i = a.add_parser("inspect", help="print a checkpoint's metadata without loading weights")
    i.add_argument("path", metavar="PATH")
    i.add_argument("--json", action="store_true")
    c = a.add_parser("convert", help="rewrite a DCP checkpoint for another rank count")
    c.add_argument("path", metavar="SRC")
    c.add_argument("output", metavar="DST")
    c.add_argument("--world-size", type=int, required=True)
    e = a.add_parser("export", help="export inference weights (safetensors or HuggingFace layout)")
    e.add_argument("path", metavar="SRC")
    e.add_argument("output", metavar="DST")
    e.add_argument("--format", default="safetensors", choices=("safetensors", "huggingface"))
    e.add_argument("--dtype", default="", choices=("", "float32", "bfloat16", "float16"))
    e.add_argument("--ema", action="store_true")
    e.add_argument("--config", default="")
    p.set_defaults(handler=run)


def _size(path: Path) -> int:
    return sum(f.stat().st_size for f in path.rglob("*") if f.is_file()) if path.is_dir() else path.stat().st_size


def _describe(path: Path) -> dict[str, Any]:
    from avgen_b200.checkpoint import MARKER_FILENAME

    marker = path / MARKER_FILENAME
    info: dict[str, Any] = {"path": str(path), "bytes": _size(path), "complete": marker.is_file()}
    if marker.is_file():
        info.update(json.loads(marker.read_text()))
    return info


def _config_beside(path: Path, override: str) -> Any:
    from avgen_b200.config import load_config

    if override:
        return load_config(override)
    for cand in (path / "config.yaml", path.parent / "config.yaml", path.parent.parent / "config.yaml"):
        if cand.is_file():
            return load_config(cand)
    raise FileNotFoundError(f"no config.yaml beside {path}; pass --config")


def run(args: argparse.Namespace) -> int:
    action = getattr(args, "action", None)
    if action is None:
        sys.stderr.write("checkpoint: choose inspect, convert or export\n")
        return EXIT_USAGE
    path = Path(args.path)
    if action == "inspect":
        info = _describe(path)
        if args.json:
            emit_json(info)
        else:
            for k in sorted(info):
                sys.stdout.write(f"{k:24s} {info[k]}\n")
        return EXIT_OK
    if action == "convert":
        from avgen_b200.checkpoint import convert

        convert(path, args.output, world_size=args.world_size)
        sys.stdout.write(f"wrote {args.output} for world size {args.world_size}\n")
        return EXIT_OK
    from avgen_b200.checkpoint import export_huggingface, export_safetensors, load_ema, load_model
    from avgen_b200.config.resolve import build_model
    from avgen_b200.parallel.precision import resolve_dtype

    model = build_model(_config_beside(path, args.config))
    (load_ema if args.ema else load_model)(path, model)
    dtype = resolve_dtype(args.dtype) if args.dtype else None
    writer = export_safetensors if args.format == "safetensors" else export_huggingface
    writer(args.output, model, dtype=dtype)
    sys.stdout.write(f"exported {args.format} weights to {args.output}\n")
    return EXIT_OK
