"""``avgen-b200 data {synthesize,shard,inspect,validate}`` (avgen/cli/data.py API)."""
from __future__ import annotations

import argparse
import sys
from pathlib import Path
from typing import Any

from avgen_b200.cli._common import EXIT_ERROR, EXIT_OK, EXIT_USAGE

__all__ = ["add_parser", "run", "shard_directories"]


def add_parser(subparsers: Any) -> None:
    p = subparsers.add_parser("data", help="synthesize, shard, inspect or validate training data")
    a = p.add_subparsers(dest="action", metavar="ACTION")
    s = a.add_parser("synthesize", help="write a deterministic synthetic latent dataset")
    s.add_argument("--output", required=True, metavar="PATH")
    s.add_argument("--samples", type=int, default=64)
    s.add_argument("--seed", type=int, default=0)
    s.add_argument("--samples-per-shard", type=int, default=32)
    sh = a.add_parser("shard", help="pack encoded latents (*.pt LatentSample files) into shards")
    sh.add_argument("input", metavar="SRC")
    sh.add_argument("output", metavar="DST")
    sh.add_argument("--samples-per-shard", type=int, default=1024)
    i = a.add_parser("inspect", help="report a shard directory without reading payloads")
    i.add_argument("path", metavar="PATH")
    v = a.add_parser("validate", help="verify manifest hashes and per-sample shapes")
    v.add_argument("path", metavar="PATH")
    v.add_argument("--config", metavar="PATH", default="")
    v.add_argument("--sample", type=int, default=0)
    p.set_defaults(handler=run)


def shard_directories(root: Path) -> list[Path]:
    """Directories under ``root`` (or root itself) that hold a committed shard."""
    if (root / "COMMIT").is_file():
        return [root]
    return sorted(d for d in root.iterdir() if d.is_dir() and (d / "COMMIT").is_file())


def _chunks(items: list[Any], n: int) -> list[list[Any]]:
    return [items[i:i + n] for i in range(0, len(items), n)]


def run(args: argparse.Namespace) -> int:
    from avgen_b200.data.shard import validate_shard, write_shard

    action = getattr(args, "action", None)
    if action is None:
        sys.stderr.write("data: choose synthesize, shard, inspect or validate\n")
        return EXIT_USAGE
    if action == "synthesize":
        from avgen_b200.data.synthetic import SyntheticConfig, SyntheticSource

        src = SyntheticSource(SyntheticConfig(seed=args.seed, num_samples=args.samples))
        out = Path(args.output)
        samples = [src.sample(i) for i in range(args.samples)]
        for k, chunk in enumerate(_chunks(samples, args.samples_per_shard)):
            write_shard(out / f"shard_{k:05d}", chunk)
        sys.stdout.write(f"wrote {args.samples} samples to {out}\n")
        return EXIT_OK
    if action == "shard":
        import torch

        files = sorted(Path(args.input).glob("*.pt"))
        if not files:
            sys.stderr.write(f"no *.pt samples under {args.input}\n")
            return EXIT_ERROR
        samples = [torch.load(f, weights_only=False) for f in files]
        for k, chunk in enumerate(_chunks(samples, args.samples_per_shard)):
            write_shard(Path(args.output) / f"shard_{k:05d}", chunk)
        sys.stdout.write(f"wrote {len(samples)} samples to {args.output}\n")
        return EXIT_OK
    root = Path(args.path)
    dirs = shard_directories(root)
    if not dirs:
        sys.stderr.write(f"no committed shards under {root}\n")
        return EXIT_ERROR
    total = 0
    bad = 0
    for d in dirs:
        try:
            manifest = validate_shard(d, check_data=action == "validate")
        except Exception as exc:  # noqa: BLE001 - report every broken shard
            bad += 1
            sys.stdout.write(f"{d}: INVALID ({exc})\n")
            continue
        n = len(manifest.records)
        total += n
        sys.stdout.write(f"{d}: {n} samples\n")
    sys.stdout.write(f"{len(dirs)} shards, {total} samples" + (f", {bad} invalid" if bad else "") + "\n")
    return EXIT_ERROR if bad else EXIT_OK
