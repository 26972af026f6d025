"""``avgen-b200 simulate``: price a configured run (avgen/cli/simulate.py API)."""
from __future__ import annotations

import argparse
import sys
from typing import Any

from avgen_b200.cli._common import EXIT_OK, emit_json

__all__ = ["add_parser", "run"]


def add_parser(subparsers: Any) -> None:
    p = subparsers.add_parser("simulate", help="predict memory, time and collectives for a configured run")
    p.add_argument("--config", metavar="PATH", default="")
    p.add_argument("overrides", nargs="*", metavar="KEY=VALUE")
    p.add_argument("--world-size", type=int, default=0, metavar="N")
    p.add_argument("--rank", type=int, default=0, metavar="R")
    p.add_argument("--gpu", default="b200", choices=("a100", "h100", "h200", "b200"))
    p.add_argument("--achieved-fraction", type=float, default=0.0)
    p.add_argument("--topology", action="store_true", help="also build the mesh on a fake process group")
    p.add_argument("--json", action="store_true")
    p.add_argument("--save", metavar="PATH", default="")
    p.set_defaults(handler=run)


def run(args: argparse.Namespace) -> int:
    from avgen_b200.config import load_config
    from avgen_b200.config.resolve import (build_accelerator, build_activation_checkpoint, build_interconnects,
                                           build_model_shape, build_parallel_dims, gradient_accumulation)
    from avgen_b200.simulate import simulate_config

    config = load_config(args.config or None, args.overrides)
    world = args.world_size or None
    dims = build_parallel_dims(config, world_size=world)
    shape = build_model_shape(config)
    accel = build_accelerator(args.gpu)
    intra, inter = build_interconnects(args.gpu)
    report = simulate_config(shape, dims, accelerator=accel, activation_checkpoint=build_activation_checkpoint(config),
                             intra_node=intra, inter_node=inter, achieved_fraction=args.achieved_fraction or None,
                             gradient_accumulation=gradient_accumulation(config, world_size=dims.world_size))
    payload = report.to_dict()
    if args.topology:
        from avgen_b200.simulate import fake_world

        with fake_world(dims, rank=args.rank, device_type="cpu") as w:
            payload["topology"] = w.describe()
    if args.save:
        report.save(args.save)
    if args.json:
        emit_json(payload)
    else:
        sys.stdout.write(report.render() + "\n")
        if "topology" in payload:
            sys.stdout.write(f"topology (rank {args.rank}): {payload['topology']}\n")
    return EXIT_OK
