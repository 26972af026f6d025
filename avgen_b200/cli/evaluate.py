"""``avgen-b200 evaluate``: generate from a checkpoint, measure, and write a pinned
report; or compare two reports (avgen/cli/evaluate.py API).

    avgen-b200 evaluate --checkpoint runs/x/export --output eval.json eval.steps=20
    avgen-b200 evaluate --baseline base.json --report cand.json [--allow seed]
    avgen-b200 evaluate --list-metrics

Under torchrun each data rank generates its share of the prompts and the
metrics' running sums are merged exactly across ranks.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path
from typing import Any

import torch

from avgen_b200.cli._common import EXIT_OK, EXIT_USAGE, emit_json, fail

__all__ = ["add_parser", "run"]


def add_parser(subparsers: Any) -> None:
    p = subparsers.add_parser("evaluate", aliases=["eval"], help="evaluate a checkpoint and write a pinned report",
                              description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", metavar="PATH", default="")
    p.add_argument("--config", metavar="PATH", default="", help="run config (default: config.yaml beside it)")
    p.add_argument("--output", metavar="PATH", default="", help="report path (default: print only)")
    p.add_argument("--step", type=int, default=0, help="training step of the checkpoint, recorded in the report")
    p.add_argument("--json", action="store_true", help="print the report as JSON")
    c = p.add_argument_group("comparison")
    c.add_argument("--baseline", metavar="PATH", default="")
    c.add_argument("--report", metavar="PATH", default="")
    c.add_argument("--allow", action="append", default=[], metavar="FIELD",
                   help="pinned field allowed to differ between the compared reports")
    p.add_argument("--list-metrics", action="store_true")
    p.add_argument("overrides", nargs="*", metavar="KEY=VALUE")
    p.set_defaults(handler=run)


def _list() -> int:
    from avgen_b200.eval import describe_metrics, learned_metric_summary, list_metrics

    desc = describe_metrics()
    sys.stdout.write("built-in metrics:\n")
    for name in list_metrics():
        sys.stdout.write(f"  {name:22s} {desc.get(name, '')}\n")
    sys.stdout.write("learned metrics (gated):\n" + learned_metric_summary() + "\n")
    return EXIT_OK


def _compare(args: argparse.Namespace) -> int:
    from avgen_b200.eval import EvalReport, IncomparableReports, compare_reports, format_comparison

    a, b = EvalReport.load(args.baseline), EvalReport.load(args.report)
    try:
        table = compare_reports(a, b, allow=tuple(args.allow))
    except IncomparableReports as err:
        return fail(str(err))
    if args.json:
        emit_json(table)
    else:
        sys.stdout.write(format_comparison(table) + "\n")
    return EXIT_OK


def _prompts(settings: Any) -> list[str]:
    from avgen_b200.eval import DEFAULT_PROMPTS

    if settings.prompts_file:
        lines = Path(settings.prompts_file).read_text(encoding="utf-8").splitlines()
        prompts = [ln.strip() for ln in lines if ln.strip() and not ln.lstrip().startswith("#")]
    else:
        prompts = list(DEFAULT_PROMPTS)
    return prompts[:settings.num_prompts] if settings.num_prompts else prompts


def _config_path(args: argparse.Namespace) -> str | None:
    if args.config:
        return args.config
    root = Path(args.checkpoint)
    for cand in (root / "config.yaml", root.parent / "config.yaml", root.parent.parent / "config.yaml"):
        if cand.is_file():
            return str(cand)
    return None


def run(args: argparse.Namespace) -> int:
    if args.list_metrics:
        return _list()
    if args.baseline or args.report:
        if not (args.baseline and args.report):
            return fail("--baseline and --report go together", code=EXIT_USAGE)
        return _compare(args)
    if not args.checkpoint:
        return fail("--checkpoint is required to evaluate (or give --baseline/--report to compare)", code=EXIT_USAGE)
    from avgen_b200.cli.generate import _codecs
    from avgen_b200.config import load_config
    from avgen_b200.config.resolve import build_model
    from avgen_b200.eval import EvalBatch, EvalPin, run_eval_suite, shard_prompts, torch_gather
    from avgen_b200.infer import GenerationConfig, GenerationPipeline, GuidanceConfig, SamplerConfig, ScheduleConfig
    from avgen_b200.infer.pipeline import _load_weights

    config = load_config(_config_path(args), list(args.overrides))
    ev = config.eval
    prompts = _prompts(ev)
    import torch.distributed as dist

    rank, world = (dist.get_rank(), dist.get_world_size()) if dist.is_available() and dist.is_initialized() else (0, 1)
    local = shard_prompts(prompts, data_rank=rank, data_world=world)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    model = build_model(config)
    _load_weights(Path(args.checkpoint), model)
    model.to(device).eval()
    codec_args = argparse.Namespace(video_codec="", text_encoder="")
    video_codec, text = _codecs(codec_args, config)
    settings = GenerationConfig(steps=ev.steps, seed=ev.seed, height=ev.height, width=ev.width, num_frames=ev.frames,
                                guidance=GuidanceConfig(scale=ev.guidance), sampler=SamplerConfig(name=ev.sampler),
                                schedule=ScheduleConfig(steps=ev.steps), negative_prompt=ev.negative_prompt,
                                dtype="float32")
    pipe = GenerationPipeline(model, video_codec=video_codec, text_encoder=text, config=settings, device=device)

    def batches():  # noqa: ANN202
        size = max(1, ev.batch_size)
        for start in range(0, len(local), size):
            chunk = tuple(local[start:start + size])
            media = pipe(list(chunk), seed=ev.seed + start, return_latents=not ev.decode)
            vid = media.video if ev.decode else media.latents
            yield EvalBatch(video=vid.float().cpu(), prompts=chunk,
                            audio=None if media.audio is None else media.audio.float().cpu())

    pin = EvalPin(checkpoint=str(args.checkpoint), sampler=ev.sampler, steps=ev.steps, guidance=ev.guidance,
                  negative_prompt=ev.negative_prompt, seed=ev.seed, frames=ev.frames, height=ev.height,
                  width=ev.width, decoded=ev.decode, precision=config.inference.dtype)
    report = run_eval_suite(batches(), metrics=ev.metrics, pin=pin, prompts=prompts, decoded=ev.decode,
                            gather=torch_gather() if world > 1 else None, data_rank=rank,
                            run_name=config.resolved_run_name(), step=args.step)
    if rank == 0:
        if args.output:
            report.save(args.output)
        if args.json:
            emit_json(report.to_dict())
        else:
            sys.stdout.write(report.render() + "\n")
    return EXIT_OK
