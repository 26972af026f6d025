"""``avgen-b200 train`` / ``finetune`` / ``rl`` (avgen/cli/train.py:85-178 API).

Launch under torchrun for more than one GPU::

    torchrun --nproc-per-node 8 -m avgen_b200.cli.main train --config run.yaml train.steps=1000
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path
from typing import Any

from avgen_b200.cli._common import EXIT_OK

__all__ = ["add_parser", "run", "run_finetune", "run_rl"]


def _add_common(p: argparse.ArgumentParser) -> None:
    p.add_argument("--config", metavar="PATH", default="", help="YAML run configuration (defaults apply when empty)")
    p.add_argument("overrides", nargs="*", metavar="KEY=VALUE", help="dotted overrides, e.g. train.lr=3e-4")
    p.add_argument("--dry-run", action="store_true", help="validate the config, resolve the plan, print a summary")
    p.add_argument("--print-config", action="store_true", help="print the resolved configuration as YAML and exit")
    p.add_argument("--output-dir", metavar="PATH", default="", help="override output_dir")


def add_parser(subparsers: Any) -> None:
    train = subparsers.add_parser("train", help="train a model from a YAML configuration",
                                  description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    _add_common(train)
    train.add_argument("--resume", metavar="PATH", default="", help="checkpoint directory or 'latest'")
    train.set_defaults(handler=run)
    ft = subparsers.add_parser("finetune", help="fine-tune a pretrained checkpoint (LoRA, DoRA, full, control)")
    _add_common(ft)
    ft.add_argument("--base", metavar="PATH", default="", help="base checkpoint (overrides finetune.base_checkpoint)")
    ft.set_defaults(handler=run_finetune)
    rl = subparsers.add_parser("rl", help="reward or preference post-training (GRPO, DPO)")
    _add_common(rl)
    rl.set_defaults(handler=run_rl)


def _load(args: argparse.Namespace) -> Any:
    from avgen_b200.config import load_config

    overrides = list(args.overrides)
    if getattr(args, "resume", ""):
        overrides.append(f"checkpoint.resume={args.resume}")
    if args.output_dir:
        overrides.append(f"output_dir={args.output_dir}")
    return load_config(args.config or None, overrides)


def summary(config: Any, *, mode: str) -> str:
    from avgen_b200.config.resolve import build_model_shape, build_parallel_dims, gradient_accumulation
    from avgen_b200.parallel import is_distributed_launch

    world = None if is_distributed_launch() else 1
    dims = build_parallel_dims(config, world_size=world)
    shape = build_model_shape(config)
    lines = [f"avgen-b200 {mode}: {config.resolved_run_name()}",
             f"  model        {config.model.name} depth {config.model.depth} width {config.model.width} "
             f"heads {config.model.num_heads} (~{shape.parameters / 1e9:.2f} B params)",
             f"  tokens       {config.sequence_length} per sample, micro-batch {config.micro_batch_size}, "
             f"accumulation {gradient_accumulation(config, world_size=dims.world_size)}",
             f"  parallel     {dims.describe()}",
             f"  optimizer    {config.train.optimizer} lr {config.train.lr} schedule {config.train.schedule}",
             f"  steps        {config.train.steps}   output {config.output_dir}"]
    return "\n".join(lines)


def _preflight(args: argparse.Namespace, mode: str) -> Any | None:
    from avgen_b200.config import save_config

    config = _load(args)
    if args.print_config:
        import yaml

        from avgen_b200.config.diff import config_to_dict

        sys.stdout.write(yaml.safe_dump(config_to_dict(config), sort_keys=False))
        return None
    sys.stdout.write(summary(config, mode=mode) + "\n")
    if args.dry_run:
        return None
    out = Path(config.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    if config.checkpoint.save_config:
        save_config(config, out / "config.yaml")
    return config


def run(args: argparse.Namespace) -> int:
    from avgen_b200.cli._wiring import build_run, run_training

    config = _preflight(args, "train")
    if config is None:
        return EXIT_OK
    run_training(build_run(config))
    return EXIT_OK


def run_finetune(args: argparse.Namespace) -> int:
    from avgen_b200.finetune.entry import run_finetune as _run

    if args.base:
        args.overrides.append(f"finetune.base_checkpoint={args.base}")
    config = _preflight(args, "finetune")
    if config is None:
        return EXIT_OK
    _run(config)
    return EXIT_OK


def run_rl(args: argparse.Namespace) -> int:
    from avgen_b200.rl.entry import run_rl as _run

    config = _preflight(args, "rl")
    if config is None:
        return EXIT_OK
    _run(config)
    return EXIT_OK
