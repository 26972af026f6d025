"""``avgen-b200 generate``: sample video from a checkpoint (avgen/cli/generate.py API).

The codecs default to the dependency-free reference codecs sized from the run
configuration, so a checkpoint trained on synthetic latents samples without
any download; pass ``--video-codec diffusers:<path>`` / ``--text-encoder
transformers:<path>`` for pretrained ones.
"""
from __future__ import annotations

import argparse
import json
import random
import sys
from pathlib import Path
from typing import Any

import torch

from avgen_b200.cli._common import EXIT_OK, read_prompts

__all__ = ["add_parser", "run"]


def add_parser(subparsers: Any) -> None:
    p = subparsers.add_parser("generate", help="sample video (and audio) from a checkpoint",
                              description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--checkpoint", required=True, metavar="PATH")
    p.add_argument("--config", metavar="PATH", default="", help="run config (default: config.yaml beside it)")
    g = p.add_mutually_exclusive_group(required=False)
    g.add_argument("--prompt", metavar="TEXT")
    g.add_argument("--prompt-file", metavar="PATH")
    s = p.add_argument_group("sampling")
    s.add_argument("--negative-prompt", metavar="TEXT", default=None)
    s.add_argument("--steps", type=int, default=0)
    s.add_argument("--guidance", type=float, default=None)
    s.add_argument("--guidance-rescale", type=float, default=None)
    s.add_argument("--sampler", default="", choices=("", "euler", "heun", "dpmpp_2m", "res_multistep"))
    s.add_argument("--seed", type=int, default=-1)
    geo = p.add_argument_group("output geometry (latent units)")
    geo.add_argument("--frames", type=int, default=0)
    geo.add_argument("--height", type=int, default=0)
    geo.add_argument("--width", type=int, default=0)
    geo.add_argument("--batch-size", type=int, default=0)
    geo.add_argument("--output", metavar="PATH", default="")
    p.add_argument("--video-codec", default="", help="diffusers:<model id or path>; default: reference codec")
    p.add_argument("--text-encoder", default="", help="transformers:<model id or path>; default: reference encoder")
    p.add_argument("--print-settings", action="store_true")
    p.set_defaults(handler=run)


def _config(args: argparse.Namespace) -> Any:
    from avgen_b200.config import load_config

    if args.config:
        return load_config(args.config)
    root = Path(args.checkpoint)
    for cand in (root / "config.yaml", root.parent / "config.yaml", root.parent.parent / "config.yaml"):
        if cand.is_file():
            return load_config(cand)
    return load_config(None)


def _codecs(args: argparse.Namespace, config: Any) -> tuple[Any, Any]:
    from avgen_b200.codecs import (DiffusersVideoCodec, ReferenceTextEncoder, ReferenceVideoCodec,
                                   TransformersTextEncoder)

    if args.video_codec.startswith("diffusers:"):
        video = DiffusersVideoCodec(args.video_codec.split(":", 1)[1])
    else:
        channels = config.model.in_channels
        video = ReferenceVideoCodec(channels=channels, temporal_compression=1, spatial_compression=1)
    if args.text_encoder.startswith("transformers:"):
        text = TransformersTextEncoder(args.text_encoder.split(":", 1)[1], max_length=config.data.text_tokens)
    else:
        text = ReferenceTextEncoder(width=config.data.text_width, max_length=config.data.text_tokens)
    return video, text


def run(args: argparse.Namespace) -> int:
    from avgen_b200.config.resolve import build_model
    from avgen_b200.infer import GenerationConfig, GenerationPipeline, GuidanceConfig, SamplerConfig, ScheduleConfig
    from avgen_b200.infer.pipeline import _load_weights

    config = _config(args)
    inf = config.inference
    seed = args.seed if args.seed >= 0 else (inf.seed if inf.seed >= 0 else random.randrange(2**31))
    settings = GenerationConfig(steps=args.steps or inf.steps, seed=seed,
                                height=args.height or inf.height, width=args.width or inf.width,
                                num_frames=args.frames or inf.frames, fps=inf.fps,
                                guidance=GuidanceConfig(scale=args.guidance if args.guidance is not None
                                                        else inf.guidance,
                                                        rescale=args.guidance_rescale if args.guidance_rescale
                                                        is not None else inf.guidance_rescale),
                                sampler=SamplerConfig(name=args.sampler or inf.sampler),
                                schedule=ScheduleConfig(steps=args.steps or inf.steps),
                                negative_prompt=args.negative_prompt if args.negative_prompt is not None
                                else inf.negative_prompt, dtype="float32")
    if args.print_settings:
        sys.stdout.write(json.dumps(settings.to_dict(), indent=2, default=str) + "\n")
        return EXIT_OK
    prompts = read_prompts(args.prompt, args.prompt_file)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    model = build_model(config)
    _load_weights(Path(args.checkpoint), model)
    model.to(device).eval()
    video, text = _codecs(args, config)
    pipe = GenerationPipeline(model, video_codec=video, text_encoder=text, config=settings, device=device)
    bsz = args.batch_size or inf.batch_size
    out = Path(args.output or inf.output)
    out.mkdir(parents=True, exist_ok=True)
    for start in range(0, len(prompts), bsz):
        chunk = prompts[start:start + bsz]
        media = pipe(chunk, seed=seed + start)
        for i, prompt in enumerate(chunk):
            path = out / f"sample_{start + i:05d}.pt"
            torch.save({"video": media.video[i].cpu(), "prompt": prompt, "fps": media.fps,
                        "settings": dict(media.config)}, path)
            sys.stdout.write(f"{path}  seed={seed + start}  {prompt!r}\n")
    return EXIT_OK
