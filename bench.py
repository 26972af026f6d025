#!/usr/bin/env python
"""Headline benchmark: training throughput of the 2B video DiT at 65,536 tokens/sample.

Metric: samples/s (+ MFU) of full training steps of the
32 x 2560 (20 heads of 128, SwiGLU MLP 4x, QK-RMSNorm, 3-D RoPE, cross-attention
to 512 x 4096 text tokens) video DiT on 65,536 tokens per sample (latents
16 x 16 x 128 x 128, patch 1 x 2 x 2), flow-matching loss, AdamW, bf16 compute,
synthetic N(0, 1) latents and text, random-init weights.

Weak scaling: every GPU processes 65,536 tokens per step. With N GPUs the job
runs context parallelism cp = min(N, 4) and data parallelism dp = N / cp, and
the global batch is N samples (each data-parallel group accumulates cp
micro-batches of one sample sharded over its cp ranks). N = 8 is the named
config: FSDP-style data parallel dp = 2 x cp = 4, global batch 8.

    python bench.py --gpus N --steps K --warmup W [--impl avgen_b200|reference]

For N > 1 launch with torchrun (one rank per GPU); rank 0 prints one JSON line.
``value`` is device-timed (CUDA events, barrier + synchronize on both sides, max
over ranks); ``e2e`` times the same steps through the public Trainer API with a
pinned host->device copy of every micro-batch and a device->host read of the
loss every step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))

WIDTH, DEPTH, HEADS, TEXT_TOKENS, TEXT_WIDTH, CHANNELS = 2560, 32, 20, 512, 4096, 16
FRAMES, HEIGHT, WIDTH_PX = 16, 128, 128  # 65,536 tokens after 1x2x2 patching
PEAK_NOMINAL = 2.25e15

# The BASELINE.json workloads. "2b_64k" is the headline the driver runs; the others
# are selected with --config. layout: "dp_cp" = cp = min(4, N) ring ranks and dp = N / cp
# data ranks, each GPU a whole sample's tokens per step; "cp_all" = one sample per
# step sharded over all N ranks (ring cp = N, FSDP over the same ranks); "tp_all" =
# tensor parallel over all N ranks by heads with sequence-parallel norms.
WORKLOADS = {
    "2b_64k": {"width": 2560, "depth": 32, "heads": 20, "ffn_hidden": None, "frames": 16, "layout": "dp_cp",
               "samples": None, "label": "2B video DiT @64k tok"},
    "14b_131k": {"width": 5120, "depth": 40, "heads": 40, "ffn_hidden": 13824, "frames": 32, "layout": "cp_all",
                 "samples": 1, "label": "14B video DiT @131k tok, cp ring + FSDP over the same ranks"},
    "2b_32k_tp": {"width": 2560, "depth": 32, "heads": 20, "ffn_hidden": None, "frames": 8, "layout": "tp_all",
                  "samples": 8, "label": "2B video DiT @32k tok, tensor parallel by heads + sequence parallel"},
    "2b_16k_lora": {"width": 2560, "depth": 32, "heads": 20, "ffn_hidden": None, "frames": 4, "layout": "dp_cp",
                    "samples": None, "lora_rank": 64,
                    "label": "2B video DiT @16k tok, LoRA rank 64 on every attention/MLP linear, FSDP2 x cp"},
    "2b_16k_grpo": {"width": 2560, "depth": 32, "heads": 20, "ffn_hidden": None, "frames": 4, "layout": "dp_cp",
                    "samples": None, "lora_rank": 64, "grpo": True,
                    "label": "GRPO on the 2B video DiT @16k tok: LoRA rank 64 under FSDP2 x cp=2, group 8, 20-step "
                             "Euler rollouts with CFG 5.0 and sequence-length shift, MLP-scorer reward"},
}


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--e2e-steps", type=int, default=2)
    p.add_argument("--impl", choices=("avgen_b200", "reference"), default="avgen_b200")
    p.add_argument("--ref-variant", choices=("ring", "shipped"), default="shipped",
                   help="reference CP attention: as shipped (block-local: each rank attends within its own shard, "
                        "the stock training path) or wrapped in its own context_parallel_region (torch ring SDPA; "
                        "fails on this model's text cross-attention with torch 2.11)")
    p.add_argument("--config", choices=tuple(WORKLOADS), default="2b_64k",
                   help="BASELINE workload (default: the headline 2B at 64k tokens)")
    p.add_argument("--depth", type=int, default=None, help="override for quick local checks (not a valid bench)")
    p.add_argument("--frames", type=int, default=None)
    p.add_argument("--profile-step", action="store_true",
                   help="after the timed region, print the device-time breakdown of one step (stderr)")
    args = p.parse_args()
    work = WORKLOADS[args.config]
    args.work = work
    args.full_depth = work["depth"]
    args.full_frames = work["frames"]
    if args.depth is None:
        args.depth = work["depth"]
    if args.frames is None:
        args.frames = work["frames"]
    return args


# --------------------------------------------------------------------------- helpers
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons every 200 ms in the background."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self) -> None:
        self.rows: list[list[str]] = []
        self.proc: subprocess.Popen | None = None
        self.thread: threading.Thread | None = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return

        def pump() -> None:
            assert self.proc is not None and self.proc.stdout is not None
            for line in self.proc.stdout:
                self.rows.append([c.strip() for c in line.split(",")])

        self.thread = threading.Thread(target=pump, daemon=True)
        self.thread.start()

    def stop(self, devices: list[int]) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in self.rows:
            if len(row) < 9:
                continue
            try:
                idx = int(row[0])
            except ValueError:
                continue
            if devices and idx not in devices:
                continue
            try:
                sm.append(float(row[1]))
                mx.append(float(row[2]))
            except ValueError:
                pass
            for name, flag in zip(names, row[5:9]):
                if flag.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def model_flops_per_sample(tokens: int, depth: int, *, attention_shards: int = 1, width: int = WIDTH,
                           hidden: int | None = None) -> float:
    """Training FLOPs of one sample (3 x forward; recompute not counted).

    ``attention_shards`` > 1 counts block-local self-attention over that many
    contiguous shards (each token attends only within its shard): 1/shards of
    the global attention FLOPs."""
    w, f, t = width, hidden or 4 * width, TEXT_TOKENS
    per_block_linear = 2 * tokens * (6 * w * w + 3 * w * f) + 2 * t * 2 * w * w
    per_block_attn = 4 * tokens * tokens * w / attention_shards + 4 * tokens * t * w
    root = 2 * tokens * (64 * w + w * 64) + 2 * t * TEXT_WIDTH * w
    return 3.0 * (depth * (per_block_linear + per_block_attn) + root)


def dist_setup() -> tuple[int, int, int]:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(minutes=10),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier(device_ids=[torch.cuda.current_device()])


def max_over_ranks(value: float) -> float:
    if not dist.is_initialized():
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def layout(world: int) -> tuple[int, int]:
    cp = 1
    for c in (4, 2, 1):
        if world % c == 0 and c <= world:
            cp = c
            break
    return cp, world // cp


# --------------------------------------------------------------------------- our arm
def run_ours(args: argparse.Namespace, rank: int, world: int, local: int) -> dict:
    sys.path.insert(0, HERE)
    from avgen_b200.core.rng import RNGStreams
    from avgen_b200.core.state import TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.models import build_model
    from avgen_b200.ops import kernels as K
    from avgen_b200.parallel import ActivationCheckpointConfig, ParallelConfig, ParallelDims, parallelize
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, Trainer,
                                  TrainerConfig, build_optimizer, build_timestep_sampler, train_step)

    dev = torch.device("cuda", local)
    work = args.work
    tp = 1
    if work["layout"] == "cp_all":
        cp, dp = world, 1
    elif work["layout"] == "tp_all":
        cp, dp, tp = 1, 1, world
    else:
        cp, dp = layout(world)
    # The named config's layout through the public API: parameters (and AdamW
    # state) sharded over dp_shard x cp (FSDP2, collectives over NVLink peer
    # memory), global attention over the cp ranks (NVLink ring); or tensor
    # parallelism by heads with sequence-parallel norms.
    dims = ParallelDims(world_size=world, dp_shard=dp, context=cp, tensor=tp)
    torch.manual_seed(1234)
    spec = {"width": work["width"], "depth": args.depth, "num_heads": work["heads"], "text_width": TEXT_WIDTH,
            "text_context_length": TEXT_TOKENS, "in_channels": CHANNELS}
    if work["ffn_hidden"]:
        spec["ffn_hidden"] = work["ffn_hidden"]
    with torch.device("meta"):
        model = build_model("video_dit", spec)
    model = model.to_empty(device=dev)
    model.init_weights()
    adapt = None
    if work.get("lora_rank"):
        from avgen_b200.finetune.lora import LoRAConfig, apply_lora

        lora = LoRAConfig(rank=work["lora_rank"], alpha=float(work["lora_rank"]),
                          target_modules=("q_proj", "k_proj", "v_proj", "out_proj", "gate_proj", "up_proj",
                                          "down_proj"))
        def adapt(m):  # noqa: ANN001, ANN202 - adapters (only they train) go in before sharding
            from avgen_b200.finetune.lora import mark_only_lora_trainable

            apply_lora(m, lora)
            mark_only_lora_trainable(m)
            return m
    pm = parallelize(model, dims, config=ParallelConfig(activation_checkpoint=ActivationCheckpointConfig(mode="none"),
                                                        sequence_parallel=tp > 1), adapt=adapt)
    model = pm.model
    cp_mesh = pm.cp_mesh
    data_rank = dims.data_coordinates(pm.mesh)[0] if pm.mesh is not None else 0
    optimizer = build_optimizer(model, lr=1e-4, weight_decay=0.0, dp_group=pm.data_group)
    state = TrainState(model=model, optimizer=optimizer, rng=RNGStreams.for_rank(0, data_rank=data_rank))
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("shifted_logit_normal"),
                                      MultiTaskConditioning())
    patchifier = pm.model.patchifier
    micro = work["samples"] or cp
    gen = torch.Generator().manual_seed(1000 + data_rank)
    shape = dict(batch=1, channels=CHANNELS, frames=args.frames, height=HEIGHT, width=WIDTH_PX,
                 text_tokens=TEXT_TOKENS, text_width=TEXT_WIDTH)
    dev_batches = [random_batch(**shape, generator=gen, device=dev) for _ in range(micro)]
    pt, ph, pw = model.config.patch_frames, model.config.patch_height, model.config.patch_width
    tokens = dev_batches[0].spec.video_tokens // (pt * ph * pw)  # transformer tokens (patches)

    def step(batches) -> object:
        metrics = None
        for m, b in enumerate(batches):
            _, metrics = train_step(state, b, objective, patchifier=patchifier, gradient_accumulation_steps=micro,
                                    microbatch_index=m, max_grad_norm=1.0, cp_mesh=cp_mesh, data_world=dp)
        return metrics

    from avgen_b200.telemetry import comm as exposed

    if world > 1:
        exposed.instrument_fsdp(model)
    for _ in range(args.warmup):
        step(dev_batches)
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler()
    if rank == 0:
        clocks.start()
    exposed.enable(world > 1)
    exposed.reset()
    launches0 = K.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    ev0.record()
    for _ in range(args.steps):
        metrics = step(dev_batches)
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    launches = (K.launch_count() - launches0)
    exposed.enable(False)
    clock_info = clocks.stop(list(range(world))) if rank == 0 else {}
    sm_mhz = max_over_ranks(float(clock_info.get("sm_mhz") or 0.0)) if world > 1 else 0.0
    comm_ms = exposed.summary(sm_mhz or None)
    if args.profile_step:
        _profile_one_step(lambda: step(dev_batches), rank)
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    # exposed communication per step: each source's max over ranks (ranks wait for the slowest)
    comm = {k: max_over_ranks(v) / args.steps for k, v in sorted(comm_ms.items())} if world > 1 else {}
    ring_ms = sum(v for k, v in comm.items() if k.startswith("ring"))
    loss_val = float(metrics.loss.item())
    from avgen_b200.ops._ext import check_errors

    err = check_errors(local)

    # ------------------------------------------------------------------ end to end through the Trainer
    trainer = Trainer(state, objective, pm, TrainerConfig(gradient_accumulation_steps=micro, max_grad_norm=1.0,
                                                          data_world=dp))
    host = [random_batch(**shape, generator=gen, pin=True) for _ in range(micro)]
    h2d = sum(b.nbytes() for b in host)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        for m, hb in enumerate(host):
            metrics = trainer.train_step(hb.to(dev, non_blocking=True), microbatch_index=m, accumulation=micro)
        _ = metrics.loss.item()
    torch.cuda.synchronize()
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0) / max(1, args.e2e_steps)

    samples_per_step = dp * micro  # global batch: every data group's micro-batches of one sample
    value = samples_per_step / (ms / 1000.0)
    flops = model_flops_per_sample(tokens, args.depth, width=work["width"], hidden=work["ffn_hidden"])
    if work.get("lora_rank"):
        flops *= 2.0 / 3.0  # frozen base weights: forward and input gradients, no weight gradients
    mfu = flops * value / (world * PEAK_NOMINAL)
    return {
        "value": value, "ms_per_step": ms, "mfu": mfu, "loss": loss_val, "kernel_errors": err,
        "gpu_launches": launches, "gpu_launches_per_step": launches // max(1, args.steps),
        "e2e": {"value": samples_per_step / e2e_s, "unit": "samples/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": 4, "s_per_step": e2e_s},
        "exposed_comm": {"ms_per_step": sum(comm.values()), "share_of_step": sum(comm.values()) / ms,
                         "ring_ms_per_step": ring_ms, "ring_share_of_step": ring_ms / ms,
                         "by_source_ms_per_step": comm} if world > 1 else None,
        "clocks": clock_info, "tokens": tokens, "cp": cp, "dp": dp, "tp": tp, "micro": micro,
        "global_batch": samples_per_step,
        "params": sum(p.numel() for p in model.parameters()), "applied": list(pm.applied),
        "peak_mem_gib": torch.cuda.max_memory_allocated(dev) / 2**30,
    }


def run_grpo(args: argparse.Namespace, rank: int, world: int, local: int) -> dict:
    """One GRPO iteration per timed step through the public API (``GRPOTrainer``):
    a group of 8 trajectories per data rank rolled out with 20-step Euler/SDE
    sampling and CFG 5.0 (conditional and unconditional in one forward), the
    MLP-scorer reward, group advantages, then the clipped-surrogate update of the
    LoRA adapters over a 4-step MixGRPO window in minibatches of 2. Throughput is
    trajectories per second over the whole job."""
    sys.path.insert(0, HERE)
    from avgen_b200.core.rng import RNGStreams
    from avgen_b200.core.state import TrainState
    from avgen_b200.finetune.lora import LoRAConfig, apply_lora, mark_only_lora_trainable
    from avgen_b200.infer.schedule import ScheduleConfig, build_sigma_schedule
    from avgen_b200.models import build_model
    from avgen_b200.ops import kernels as K
    from avgen_b200.parallel import ActivationCheckpointConfig, ParallelConfig, ParallelDims, parallelize
    from avgen_b200.rl.grpo import GRPOConfig, GRPOTrainer, WindowSchedule
    from avgen_b200.rl.rewards import build_reward
    from avgen_b200.rl.rollout import model_velocity_fn
    from avgen_b200.train import build_optimizer

    dev = torch.device("cuda", local)
    work = args.work
    cp = 2 if world % 2 == 0 else 1
    dp = world // cp
    dims = ParallelDims(world_size=world, dp_shard=dp, context=cp)
    torch.manual_seed(1234)
    with torch.device("meta"):
        model = build_model("video_dit", {"width": work["width"], "depth": args.depth, "num_heads": work["heads"],
                                          "text_width": TEXT_WIDTH, "text_context_length": TEXT_TOKENS,
                                          "in_channels": CHANNELS})
    model = model.to_empty(device=dev)
    model.init_weights()
    lora = LoRAConfig(rank=work["lora_rank"], alpha=float(work["lora_rank"]),
                      target_modules=("q_proj", "k_proj", "v_proj", "out_proj", "gate_proj", "up_proj", "down_proj"))

    def adapt(m):  # noqa: ANN001, ANN202
        apply_lora(m, lora)
        mark_only_lora_trainable(m)
        return m

    pm = parallelize(model, dims, config=ParallelConfig(activation_checkpoint=ActivationCheckpointConfig(mode="none")),
                     adapt=adapt)
    data_rank = dims.data_coordinates(pm.mesh)[0] if pm.mesh is not None else 0
    state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-5, dp_group=pm.data_group),
                       rng=RNGStreams.for_rank(0, data_rank=data_rank))
    gen = torch.Generator().manual_seed(77 + data_rank)
    text = torch.randn(1, TEXT_TOKENS, TEXT_WIDTH, generator=gen).to(dev, torch.bfloat16)
    frames = args.frames
    positions = (torch.arange(frames, dtype=torch.float32) / 24.0).to(dev)[None]
    grid_mask = torch.ones(1, frames, HEIGHT, WIDTH_PX, dtype=torch.bool, device=dev)
    velocity = model_velocity_fn(pm.model, patchifier=pm.model.patchifier, positions=positions, mask=grid_mask,
                                 text_features=text, text_mask=torch.ones(1, TEXT_TOKENS, dtype=torch.bool, device=dev),
                                 guidance=5.0, cp_mesh=pm.cp_mesh)
    tokens = frames * (HEIGHT // 2) * (WIDTH_PX // 2)
    sigmas = build_sigma_schedule(ScheduleConfig(steps=20, dynamic_shift=True), sequence_length=tokens).sigmas.to(dev)
    cfg = GRPOConfig(group_size=8, clip_range=2e-4, minibatch_size=2, max_grad_norm=1.0,
                     window=WindowSchedule(window=4, stride=1, interval=25, total_steps=20))
    trainer = GRPOTrainer(state, velocity, cfg, cp_mesh=pm.cp_mesh, data_group=pm.data_group)
    reward = build_reward("mlp_scorer", channels=CHANNELS)
    latent_shape = (CHANNELS, frames, HEIGHT, WIDTH_PX)

    def iteration() -> float:
        buffer = trainer.rollout(["synthetic prompt"], sigmas=sigmas, latent_shape=latent_shape, reward=reward,
                                 device=dev, dtype=torch.bfloat16)
        metrics = trainer.update(buffer)
        return metrics[-1].loss

    for _ in range(args.warmup):
        iteration()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler()
    if rank == 0:
        clocks.start()
    launches0 = K.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        loss = iteration()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    launches = K.launch_count() - launches0
    clock_info = clocks.stop(list(range(world))) if rank == 0 else {}
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    from avgen_b200.ops._ext import check_errors

    err = check_errors(local)
    trajectories = dp * cfg.group_size  # per iteration, over the whole job
    # end to end: the prompt embedding copied in from pinned host memory, the mean reward read back
    host_text = text.cpu().pin_memory()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        text.copy_(host_text.to(dev, non_blocking=True))  # the step's prompt embedding, read by the velocity
        buffer = trainer.rollout(["synthetic prompt"], sigmas=sigmas, latent_shape=latent_shape, reward=reward,
                                 device=dev, dtype=torch.bfloat16)
        trainer.update(buffer)
        _ = float(buffer.rewards.mean().item())
    torch.cuda.synchronize()
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0) / max(1, args.e2e_steps)
    return {
        "value": trajectories / (ms / 1000.0), "unit": "trajectories/s", "ms_per_step": ms, "mfu": None,
        "loss": float(loss), "kernel_errors": err, "gpu_launches": launches,
        "e2e": {"value": trajectories / e2e_s, "unit": "trajectories/s", "h2d_bytes_per_step": host_text.numel() * host_text.element_size(),
                "d2h_bytes_per_step": 4, "s_per_step": e2e_s},
        "exposed_comm": None, "clocks": clock_info, "tokens": tokens, "cp": cp, "dp": dp, "tp": 1, "micro": 1,
        "global_batch": trajectories, "params": sum(p.numel() for p in pm.model.parameters()),
        "applied": list(pm.applied), "peak_mem_gib": torch.cuda.max_memory_allocated(dev) / 2**30,
        "grpo": {"group_size": cfg.group_size, "sampler_steps": 20, "guidance": 5.0, "window": 4,
                 "minibatch_size": cfg.minibatch_size, "reward": "mlp_scorer"},
    }


def _profile_one_step(fn, rank: int) -> None:  # noqa: ANN001
    """Kernel-time shares of one step (torch.profiler CUDA activity); never a bench value."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    if rank != 0:
        return
    rows = [(e.device_time_total, e.count, e.key) for e in prof.key_averages() if e.device_time_total > 0]
    total = sum(r[0] for r in rows)
    print(f"[profile] one step: {total / 1e3:.1f} ms of kernel time", file=sys.stderr)
    for t, n, key in sorted(rows, reverse=True)[:30]:
        print(f"[profile] {t / 1e3:9.2f} ms {100 * t / total:5.1f}%  n={n:5d}  {key[:90]}", file=sys.stderr)


# --------------------------------------------------------------------------- reference arm
def run_reference(args: argparse.Namespace, rank: int, world: int, local: int) -> dict:
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "avgen")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, ref)
    import avgen
    from avgen import RNGStreams, TrainState, build_model, train_step
    from avgen.core.batch import MediaBatch, MediaBatchSpec
    from avgen.core.patchify import GridPatchifier
    from avgen.parallel import ParallelDims, parallelize
    from avgen.parallel.activation import ActivationCheckpointConfig
    from avgen.parallel.apply import ParallelConfig
    from avgen.parallel.context import context_parallel_region
    from avgen.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                             build_timestep_sampler)

    del avgen
    dev = torch.device("cuda", local)
    cp, dp = layout(world)
    micro = cp
    dims = ParallelDims(world_size=world, dp_shard=dp, context=cp)

    def build(mode: str, frequency: int):  # noqa: ANN202
        torch.manual_seed(1234)
        with torch.device("meta"):
            model = build_model("video_dit", {"width": WIDTH, "depth": args.depth, "num_heads": HEADS,
                                              "text_width": TEXT_WIDTH, "text_context_length": TEXT_TOKENS,
                                              "in_channels": CHANNELS})
        model = model.to_empty(device=dev)
        model.init_weights()
        parallel = parallelize(model, dims, config=ParallelConfig(
            activation_checkpoint=ActivationCheckpointConfig(mode=mode, save_op_frequency=frequency)))
        data_rank = dims.data_coordinates(parallel.mesh)[0] if parallel.mesh is not None else 0
        optimizer = build_optimizer(parallel.model, lr=1e-4, weight_decay=0.0)
        state = TrainState(model=parallel.model, optimizer=optimizer,
                           rng=RNGStreams.for_rank(0, data_rank=data_rank))
        return parallel, state, data_rank

    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("shifted_logit_normal"),
                                      MultiTaskConditioning())
    patchifier = GridPatchifier()
    gen = torch.Generator()

    def make(pin: bool) -> MediaBatch:
        spec = MediaBatchSpec(schema_version=1, bucket_id=0, video_shape=(1, CHANNELS, args.frames, HEIGHT, WIDTH_PX),
                              audio_shape=(1, 1, 0), text_shape=(1, TEXT_TOKENS, TEXT_WIDTH), video_timebase_num=24000,
                              video_timebase_den=1000, audio_timebase_num=1, audio_timebase_den=1,
                              video_codec_id="synthetic", audio_codec_id="none")
        t = {
            "video": torch.randn((1, CHANNELS, args.frames, HEIGHT, WIDTH_PX), generator=gen),
            "audio": torch.zeros((1, 1, 0)), "text": torch.randn((1, TEXT_TOKENS, TEXT_WIDTH), generator=gen),
            "video_mask": torch.ones((1, args.frames, HEIGHT, WIDTH_PX), dtype=torch.bool),
            "audio_mask": torch.zeros((1, 0), dtype=torch.bool),
            "video_positions": (torch.arange(args.frames, dtype=torch.float32) / 24.0)[None].contiguous(),
            "audio_positions": torch.zeros((1, 0)),
            "text_mask": torch.ones((1, TEXT_TOKENS), dtype=torch.bool),
        }
        if pin:
            t = {k: v.pin_memory() for k, v in t.items()}
        return MediaBatch(sample_ids=torch.zeros(1, dtype=torch.int64), spec=spec, **t)

    use_ring = cp > 1 and args.ref_variant == "ring"
    cp_buffer = torch.zeros(cp * 128, device=dev)
    if use_ring:
        # torch's ring SDPA enables its head-tail load balancer by default and then
        # refuses non-causal attention; the DiT's attention is bidirectional.
        from torch.distributed.tensor.experimental._context_parallel import _attention as _cp_attention

        _cp_attention._cp_options.enable_load_balance = False

    def step(batches, *, copy: bool) -> object:
        metrics = None
        state = current["state"]
        parallel = current["parallel"]
        for m, b in enumerate(batches):
            if copy:
                b = b.to(dev, non_blocking=True)
            # torch's context_parallel indexes buffers[0], so hand the region one
            # small sequence buffer to shard (and restore); the model's own streams
            # are sharded by the reference's objective as shipped.
            region = context_parallel_region(parallel.cp_mesh, buffers=[cp_buffer], buffer_seq_dims=[0]) \
                if use_ring else _null()
            with region:
                _, metrics = train_step(state, b, objective, patchifier=patchifier, gradient_accumulation_steps=micro,
                                        microbatch_index=m, max_grad_norm=1.0, cp_mesh=parallel.cp_mesh,
                                        autocast_dtype=torch.bfloat16, data_world=dp)
        return metrics

    # Activation checkpointing: the cheapest of the reference's own policies that
    # runs, tried in order of recompute (none, selective_op saving every listed op,
    # then every 2nd, then full), each moved past only after a caught CUDA OOM (or
    # an error of the mode itself) on some rank (every rank takes the same path: the
    # failure flag is max-reduced); the line lists each rejected mode with its reason.
    current: dict = {}
    attempts: list[str] = []
    ac_mode = "full"
    for mode, frequency in (("none", 1), ("selective_op", 1), ("selective_op", 2), ("full", 1)):
        label = mode if mode != "selective_op" else f"selective_op(save_op_frequency={frequency})"
        failed, why = 0.0, ""
        try:
            parallel, state, data_rank = build(mode, frequency)
            current.update(parallel=parallel, state=state)
            gen.manual_seed(1000 + data_rank)
            host = [make(True) for _ in range(micro)]
            dev_batches = [b.to(dev) for b in host]
            if mode != "full":
                step(dev_batches, copy=False)
                torch.cuda.synchronize()
        except torch.OutOfMemoryError:
            failed, why = 1.0, "CUDA out of memory"
        except RuntimeError as exc:  # the mode itself fails on this model (not a memory limit)
            failed, why = 1.0, f"{type(exc).__name__}: {str(exc).splitlines()[0][:160]}"
        if max_over_ranks(failed) == 0.0:
            ac_mode = label
            break
        attempts.append(f"{label}: {why or 'failed on another rank'}")
        current.clear()
        parallel = state = host = dev_batches = None
        import gc

        gc.collect()
        torch.cuda.empty_cache()
        barrier()
    for _ in range(args.warmup):
        step(dev_batches, copy=False)
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler()
    if rank == 0:
        clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        metrics = step(dev_batches, copy=False)
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clock_info = clocks.stop(list(range(world))) if rank == 0 else {}
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    loss_val = float(metrics.loss.item())
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        metrics = step(host, copy=True)
        _ = metrics.loss.item()
    torch.cuda.synchronize()
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0) / max(1, args.e2e_steps)
    h2d = sum(sum(t.numel() * t.element_size() for t in (b.video, b.audio, b.text, b.video_mask, b.audio_mask,
                                                         b.video_positions, b.audio_positions, b.text_mask))
              for b in host)
    tokens = args.frames * HEIGHT * WIDTH_PX // 4
    value = world / (ms / 1000.0)
    return {
        "value": value, "ms_per_step": ms,
        # MFU of the work actually done: as shipped, the reference's CP attention is block-local
        "mfu": model_flops_per_sample(tokens, args.depth, attention_shards=cp if cp > 1 and not use_ring else 1)
        * value / (world * PEAK_NOMINAL),
        "loss": loss_val, "e2e": {"value": world / e2e_s, "unit": "samples/s", "h2d_bytes_per_step": int(h2d),
                                  "d2h_bytes_per_step": 4, "s_per_step": e2e_s},
        "exposed_comm": {"ms_per_step": sum(comm.values()), "share_of_step": sum(comm.values()) / ms,
                         "ring_ms_per_step": ring_ms, "ring_share_of_step": ring_ms / ms,
                         "by_source_ms_per_step": comm} if world > 1 else None,
        "clocks": clock_info, "tokens": tokens, "cp": cp, "dp": dp, "micro": micro, "ac_mode": ac_mode,
        "ac_attempts": attempts,
        "ref_variant": ("ring (context_parallel_region)" if use_ring else
                        f"shipped: block-local attention within each of the {cp} sequence shards "
                        f"(1/{cp} of the global self-attention FLOPs)") if cp > 1 else "n/a (cp=1)",
        "applied": list(current["parallel"].applied),
    }


class _null:
    def __enter__(self) -> None:
        return None

    def __exit__(self, *exc: object) -> None:
        return None


def main() -> None:
    args = parse_args()
    rank, world, local = dist_setup()
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun --nproc-per-node {args.gpus}")
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference" and args.config != "2b_64k":
        out = {"unavailable": f"the reference arm runs the headline workload only (asked for {args.config})"}
    elif args.impl == "reference":
        out = run_reference(args, rank, world, local)
    elif args.work.get("grpo"):
        out = run_grpo(args, rank, world, local)
    else:
        out = run_ours(args, rank, world, local)
    if rank == 0:
        if "unavailable" in out:
            print(json.dumps({"impl": "reference", "unavailable": out["unavailable"]}), flush=True)
        else:
            cp, dp, tp = out["cp"], out["dp"], out.get("tp", 1)
            work = args.work
            metric = ("samples/s + MFU, 2B video DiT @64k tok, 1/2/4/8 B200; ring-attn exposed comm"
                      if args.config == "2b_64k" else f"samples/s + MFU, {work['label']}")
            hidden = f"MLP {work['ffn_hidden']}" if work["ffn_hidden"] else "SwiGLU mlp_ratio 4"
            parallelism = "single" if world == 1 else (f"tp{tp}+sp" if tp > 1 else f"dp{dp}xcp{cp}")
            if work.get("grpo"):
                metric = f"trajectories/s, {work['label']}"
            line = {
                "metric": metric,
                "value": out["value"], "unit": out.get("unit", "samples/s"), "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": out["ms_per_step"], "higher_is_better": True,
                "scaling": "weak" if work["layout"] == "dp_cp" else "strong", "vs_baseline": None, "dtype": "bf16",
                "data": f"synthetic N(0,1) latents [1,16,{args.frames},128,128] and text [1,512,4096]; "
                        "random-init weights",
                "config": {"model": f"video_dit {args.depth}x{work['width']}, {work['heads']} heads x 128, {hidden}, "
                                    f"QK-RMSNorm, 3-D RoPE, cross-attn 512x4096",
                           "global_batch": out.get("global_batch", world), "seq_len": out["tokens"],
                           "parallelism": parallelism,
                           "micro_batches_per_step": out["micro"],
                           "l2": "inputs larger than L2 (each block activation is 335 MB)"},
                "mfu": out["mfu"], "loss": out["loss"], "e2e": out["e2e"], "clocks": out["clocks"],
            }
            if args.impl == "reference":
                line["impl"] = "reference"
                line["config"]["activation_checkpoint"] = out["ac_mode"]
                line["config"]["activation_checkpoint_rejected"] = out["ac_attempts"]
                line["config"]["ref_variant"] = out["ref_variant"]
                line["config"]["applied"] = out["applied"]
            else:
                line["impl"] = "avgen_b200"
                line["gpu_launches"] = out["gpu_launches"]
                line["kernel_errors"] = out["kernel_errors"]
                line["params"] = out["params"]
                line["config"]["applied"] = out["applied"]
                line["peak_mem_gib"] = round(out["peak_mem_gib"], 1)
                if out["exposed_comm"] is not None:
                    line["exposed_comm"] = out["exposed_comm"]
                if out.get("grpo"):
                    line["config"]["grpo"] = out["grpo"]
            if args.depth != args.full_depth or args.frames != args.full_frames:
                line["note"] = "reduced model/config: not a valid benchmark line"
            if args.config != "2b_64k":
                line["config"]["workload"] = args.config
            print(json.dumps(line), flush=True)
    if dist.is_initialized():
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
