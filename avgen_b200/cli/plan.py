"""``avgen-b200 plan``: rank parallel plans for a model shape and world size (avgen/cli/plan.py API)."""
from __future__ import annotations

import argparse
import sys
from typing import Any

from avgen_b200.cli._common import EXIT_ERROR, EXIT_OK, emit_json

__all__ = ["add_parser", "run"]


def add_parser(subparsers: Any) -> None:
    p = subparsers.add_parser("plan", help="rank parallelism plans for a model shape and world size")
    s = p.add_argument_group("model shape")
    s.add_argument("--params", type=float, default=2e9, metavar="N")
    s.add_argument("--depth", type=int, default=32)
    s.add_argument("--width", type=int, default=2560)
    s.add_argument("--heads", type=int, default=0, help="0 derives heads at 128 dims per head")
    s.add_argument("--mlp-ratio", type=int, default=4)
    s.add_argument("--seq-len", type=int, default=65536, metavar="L")
    s.add_argument("--text-tokens", type=int, default=226)
    s.add_argument("--micro-batch", type=int, default=1)
    c = p.add_argument_group("cluster")
    c.add_argument("--world-size", type=int, required=True, metavar="N")
    c.add_argument("--gpu", default="b200", choices=("a100", "h100", "h200", "b200"))
    c.add_argument("--gpus-per-node", type=int, default=8)
    c.add_argument("--global-batch", type=int, default=0, metavar="B")
    b = p.add_argument_group("search bounds")
    b.add_argument("--max-tensor", type=int, default=8)
    b.add_argument("--max-context", type=int, default=32)
    b.add_argument("--max-pipeline", type=int, default=1)
    b.add_argument("--min-blocks-per-stage", type=int, default=4)
    b.add_argument("--no-hsdp", action="store_true")
    b.add_argument("--achieved-fraction", type=float, default=0.0,
                   help="uniform fraction of peak; 0 uses the per-kernel efficiencies of the device profile")
    b.add_argument("--headroom", type=float, default=0.1)
    b.add_argument("--top-k", type=int, default=10)
    p.add_argument("--json", action="store_true")
    p.set_defaults(handler=run)


def run(args: argparse.Namespace) -> int:
    from avgen_b200.config.resolve import build_accelerator, build_interconnects
    from avgen_b200.simulate import ModelShape, SearchSpace, render_plan_table, search_parallel_plan

    heads = args.heads or max(1, args.width // 128)
    shape = ModelShape(parameters=int(args.params), depth=args.depth, width=args.width, sequence_length=args.seq_len,
                       micro_batch_size=args.micro_batch, mlp_ratio=args.mlp_ratio, num_heads=heads,
                       text_tokens=args.text_tokens)
    space = SearchSpace(world_size=args.world_size, gpus_per_node=args.gpus_per_node, max_tensor=args.max_tensor,
                        max_context=args.max_context, max_pipeline=args.max_pipeline,
                        allow_hsdp=not args.no_hsdp, global_batch_size=args.global_batch or None,
                        min_blocks_per_stage=args.min_blocks_per_stage)
    accel = build_accelerator(args.gpu)
    intra, inter = build_interconnects(args.gpu)
    found = search_parallel_plan(shape, space, accelerator=accel, intra_node=intra, inter_node=inter,
                                 achieved_fraction=args.achieved_fraction or None, headroom=args.headroom,
                                 top_k=args.top_k)
    if args.json:
        emit_json([c.summary(accel) for c in found])
        return EXIT_OK if found else EXIT_ERROR
    sys.stdout.write(f"{shape.parameters / 1e9:.2f} B params, {args.depth} x {args.width}, {args.seq_len:,} tokens, "
                     f"{args.world_size} x {accel.name}\n\n")
    sys.stdout.write(render_plan_table(found, accel) + "\n")
    if found:
        best = found[0]
        d = best.dims
        sys.stdout.write(f"\nbest: {d.describe()} with {best.activation_checkpoint.mode} activations\n"
                         f"  overrides: parallel.dp_replicate={d.dp_replicate} parallel.dp_shard={d.dp_shard} "
                         f"parallel.context={d.context} parallel.tensor={d.tensor} parallel.pipeline={d.pipeline}\n")
    return EXIT_OK if found else EXIT_ERROR
