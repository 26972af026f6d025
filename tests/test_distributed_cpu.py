"""Multi-process parallelism on CPU (gloo, world size 2): FSDP2, tensor parallel and context
parallel each reproduce single-process forward and gradients; a rank with a non-finite loss
makes every rank skip the same step; data shards are disjoint."""
from __future__ import annotations

import os
import socket
from dataclasses import asdict

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world: int = 2, *args) -> None:  # noqa: ANN001
    mp.spawn(_entry, args=(world, _free_port(), fn, args), nprocs=world, join=True)


def _entry(rank: int, world: int, port: int, fn, args) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


def _model(seed: int = 0):  # noqa: ANN202
    from avgen_b200.models import build_model, preset

    torch.manual_seed(seed)
    cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
    m = build_model("video_dit", cfg)
    m.init_weights()
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.02 * torch.randn_like(p))
    return m


def _inputs(seed: int, model):  # noqa: ANN001, ANN202
    """A ModelInput with per-token levels (a clean first frame) from a synthetic batch."""
    from avgen_b200.codecs import ReferenceTextEncoder  # noqa: F401 (import check)
    from avgen_b200.core.tokens import TextContext
    from avgen_b200.infer.conditioning import StreamState, condition_first_frame

    g = torch.Generator().manual_seed(seed)
    c = model.config
    lat = torch.randn(1, c.in_channels, 4, 8, 8, generator=g)
    text = TextContext(features=torch.randn(1, 6, c.text_width, generator=g), mask=torch.ones(1, 6, dtype=torch.bool))
    return condition_first_frame(StreamState(lat, fps=8.0), lat[:, :, 0], sigma=0.6, text=text,
                                 patchifier=model.patchifier)


def _loss(out) -> torch.Tensor:  # noqa: ANN001
    w = torch.linspace(-1.0, 1.0, out.video.shape[-1])
    return (out.video * w).sum()


def _reference_grads(seeds: list[int]) -> tuple[list[torch.Tensor], dict[str, torch.Tensor]]:
    model = _model()
    outs, grads = [], {}
    for s in seeds:
        model.zero_grad()
        out = model(_inputs(s, model))
        _loss(out).backward()
        outs.append(out.video.detach())
        for n, p in model.named_parameters():
            grads[n] = grads.get(n, 0) + p.grad.detach() / len(seeds)
    return outs, grads


def _fsdp_worker(rank: int, world: int) -> None:
    from torch.distributed.tensor import DTensor

    from avgen_b200.parallel import ParallelDims, parallelize

    ref_outs, ref_grads = _reference_grads([10, 11])
    from avgen_b200.parallel import ParallelConfig, PrecisionConfig

    model = _model()
    dims = ParallelDims(world_size=world, dp_shard=world)
    fp32 = ParallelConfig(precision=PrecisionConfig(param_dtype="float32"))  # exact comparison with fp32 reference
    pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"), config=fp32)
    assert pm.applied[0].startswith("fsdp")
    out = pm.model(_inputs(10 + rank, model))
    torch.testing.assert_close(out.video.detach(), ref_outs[rank], rtol=1e-4, atol=1e-5)
    _loss(out).backward()
    for n, p in pm.model.named_parameters():
        g = p.grad.full_tensor() if isinstance(p.grad, DTensor) else p.grad
        torch.testing.assert_close(g, ref_grads[n], rtol=1e-3, atol=1e-5, msg=n)


def _tp_worker(rank: int, world: int) -> None:
    from torch.distributed.tensor import DTensor

    from avgen_b200.parallel import ParallelDims, parallelize

    ref_outs, ref_grads = _reference_grads([21])
    model = _model()
    dims = ParallelDims(world_size=world, tensor=world)
    pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"))
    assert any(isinstance(p, DTensor) for p in pm.model.parameters())
    out = pm.model(_inputs(21, model))
    torch.testing.assert_close(out.video.detach(), ref_outs[0], rtol=1e-4, atol=1e-5)
    _loss(out).backward()
    for n, p in pm.model.named_parameters():
        g = p.grad.full_tensor() if isinstance(p.grad, DTensor) else p.grad
        torch.testing.assert_close(g, ref_grads[n], rtol=1e-3, atol=1e-5, msg=n)


def _cp_worker(rank: int, world: int, sharded: bool = True) -> None:
    from torch.distributed.tensor import DTensor

    from avgen_b200.parallel import ParallelConfig, ParallelDims, PrecisionConfig, gather_tokens, parallelize, shard_stream

    ref_outs, ref_grads = _reference_grads([31])
    model = _model()
    dims = ParallelDims(world_size=world, context=world)
    cfg = ParallelConfig(precision=PrecisionConfig(param_dtype="float32"), shard_parameters=sharded)
    pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"), config=cfg)
    # cp alone shards parameters over the context ranks, as the reference does
    assert any(a.startswith("fsdp(cp=") for a in pm.applied) == sharded, pm.applied
    inputs = _inputs(31, model)
    local = inputs.replace_streams(video=shard_stream(inputs.video, pm.cp_mesh))
    out = pm.model(local)
    full = gather_tokens(out.video.detach(), pm.cp_mesh)
    torch.testing.assert_close(full, ref_outs[0], rtol=1e-4, atol=1e-5)
    _loss(out).backward()  # per-shard partial loss: the full gradient is the sum over shards
    for n, p in pm.model.named_parameters():
        if isinstance(p.grad, DTensor):  # FSDP averaged the shards' gradients over the cp ranks
            g = p.grad.full_tensor() * world
        else:
            g = p.grad.clone()
            dist.all_reduce(g)
        torch.testing.assert_close(g, ref_grads[n], rtol=1e-3, atol=1e-5, msg=n)


def _cp_replicated_worker(rank: int, world: int) -> None:
    _cp_worker(rank, world, sharded=False)


def _pipeline_worker(rank: int, world: int, schedule: str = "1f1b") -> None:
    """Two pipeline stages (1F1B over gloo point-to-point) take the same two optimizer
    steps, each over 3 micro-batches with gradient clipping, as the unsharded model
    with gradient accumulation: losses and every parameter match."""
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PipelineConfig, PrecisionConfig, parallelize
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)
    from avgen_b200.train.trainer import pipeline_train_step

    ref = _model()
    model = _model()
    dims = ParallelDims(world_size=world, pipeline=world)
    pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"),
                     config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32"),
                                           pipeline=PipelineConfig(schedule=schedule)))
    assert pm.pipeline is not None and any(a.startswith("pipeline(pp=2") for a in pm.applied), pm.applied
    assert len(pm.model.blocks) < len(ref.blocks)
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-2), rng=RNGStreams.for_rank(0, data_rank=0))
    ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-2), rng=RNGStreams.for_rank(0, data_rank=0))
    c = ref.config
    gen = torch.Generator().manual_seed(5)
    for step in range(2):
        micro = [random_batch(batch=1, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                              text_width=c.text_width, generator=gen) for _ in range(3)]
        _, metrics = pipeline_train_step(state, micro, objective, pm.pipeline, patchifier=ref.patchifier,
                                         max_grad_norm=0.05, pp_mesh=pm.pp_mesh)
        losses = []
        for i, b in enumerate(micro):
            _, rm = train_step(ref_state, b, objective, patchifier=ref.patchifier, gradient_accumulation_steps=3,
                               microbatch_index=i, max_grad_norm=0.05)
            losses.append(float(rm.loss))
        assert abs(float(metrics.loss) - sum(losses) / 3) <= 1e-5 * max(1.0, abs(sum(losses))), (step, metrics.loss)
        assert abs(float(metrics.grad_norm) - float(rm.grad_norm)) <= 1e-4 * float(rm.grad_norm)
        mine = dict(pm.model.named_parameters())
        for name, q in ref.named_parameters():
            if name in mine:
                err = (mine[name].detach() - q.detach()).abs().max().item()
                assert err <= 1e-6 + 1e-4 * q.detach().abs().max().item(), f"step {step}: {name}: {err}"
    owned = {n for n, _ in pm.model.named_parameters()}
    every = [None] * world
    dist.all_gather_object(every, sorted(owned))
    assert set().union(*map(set, every)) == {n for n, _ in ref.named_parameters()}


def _pipeline_gpipe_worker(rank: int, world: int) -> None:
    _pipeline_worker(rank, world, schedule="gpipe")


def _pipeline_interleaved_worker(rank: int, world: int) -> None:
    """Interleaved 1F1B: a 4-block model cut into 4 chunks over 2 ranks (rank 0 owns
    chunks 0 and 2, rank 1 chunks 1 and 3, so each micro-batch crosses between the
    ranks three times), 4 micro-batches per step: two clipped optimizer steps equal
    the unsharded model's with gradient accumulation."""
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.models import build_model, preset
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PipelineConfig, PrecisionConfig, parallelize
    from avgen_b200.parallel.pipeline import InterleavedPipelineRunner
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)
    from avgen_b200.train.trainer import pipeline_train_step

    def deep():  # noqa: ANN202
        torch.manual_seed(0)
        cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
        cfg["depth"] = 4
        m = build_model("video_dit", cfg)
        m.init_weights()
        with torch.no_grad():
            for p in m.parameters():
                p.add_(0.02 * torch.randn_like(p))
        return m

    ref = deep()
    dims = ParallelDims(world_size=world, pipeline=world)
    pm = parallelize(deep(), dims, mesh=dims.build_mesh("cpu"),
                     config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32"),
                                           pipeline=PipelineConfig(schedule="interleaved_1f1b", stages_per_rank=2)))
    assert isinstance(pm.pipeline, InterleavedPipelineRunner), pm.applied
    assert [list(c.keys()) for c in pm.model.pipeline_chunks] == ([["0"], ["2"]] if rank == 0 else [["1"], ["3"]])
    assert (pm.model.patch_embed is not None) == (rank == 0) and (pm.model.final_proj is not None) == (rank == 1)
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-2),
                       rng=RNGStreams.for_rank(0, data_rank=0))
    ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-2), rng=RNGStreams.for_rank(0, data_rank=0))
    c = ref.config
    gen = torch.Generator().manual_seed(6)
    for step in range(2):
        micro = [random_batch(batch=1, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                              text_width=c.text_width, generator=gen) for _ in range(4)]
        _, metrics = pipeline_train_step(state, micro, objective, pm.pipeline, patchifier=ref.patchifier,
                                         max_grad_norm=0.05, pp_mesh=pm.pp_mesh)
        losses = []
        for i, b in enumerate(micro):
            _, rm = train_step(ref_state, b, objective, patchifier=ref.patchifier, gradient_accumulation_steps=4,
                               microbatch_index=i, max_grad_norm=0.05)
            losses.append(float(rm.loss))
        assert abs(float(metrics.loss) - sum(losses) / 4) <= 1e-5 * max(1.0, abs(sum(losses))), (step, metrics.loss)
        assert abs(float(metrics.grad_norm) - float(rm.grad_norm)) <= 1e-4 * float(rm.grad_norm)
        mine = dict(pm.model.named_parameters())
        for name, q in ref.named_parameters():
            if name in mine:
                err = (mine[name].detach() - q.detach()).abs().max().item()
                assert err <= 1e-6 + 1e-4 * q.detach().abs().max().item(), f"step {step}: {name}: {err}"
    owned = {n for n, _ in pm.model.named_parameters()}
    every = [None] * world
    dist.all_gather_object(every, sorted(owned))
    assert set().union(*map(set, every)) == {n for n, _ in ref.named_parameters()}


def _lora_tp_worker(rank: int, world: int, use_dora: bool = False) -> None:
    """LoRA / DoRA on tensor-parallel DTensor weights: adapter placements follow the
    base weight's shard dimension (column-parallel Shard(0) -> A replicated, B
    Shard(0); row-parallel Shard(1) -> A Shard(1), B replicated; the DoRA magnitude
    like B), and forward plus every adapter gradient match the unsharded adapted
    model (the DoRA row norms of a row-parallel weight sum squares across ranks)."""
    from torch.distributed.tensor import DTensor, Replicate, Shard, distribute_tensor

    from avgen_b200.finetune.lora import LoRAConfig, apply_lora, lora_modules, mark_only_lora_trainable
    from avgen_b200.parallel import ParallelDims, parallelize

    cfg = LoRAConfig(rank=4, alpha=8.0, use_dora=use_dora, target_modules=("q_proj", "out_proj", "down_proj"))
    ref = apply_lora(_model(), cfg)
    torch.manual_seed(3)
    with torch.no_grad():  # non-zero B: the adapter contributes to the output
        for _, m in lora_modules(ref):
            m.lora_b.normal_(0.0, 0.05)
            if m.lora_magnitude is not None:
                m.lora_magnitude.mul_(1.0 + 0.1 * torch.randn_like(m.lora_magnitude))
    mark_only_lora_trainable(ref)
    dims = ParallelDims(world_size=world, tensor=world)
    pm = parallelize(_model(), dims, mesh=dims.build_mesh("cpu"), adapt=lambda m: apply_lora(m, cfg))
    mark_only_lora_trainable(pm.model)
    ref_mods = dict(lora_modules(ref))
    checked = set()
    for name, mod in lora_modules(pm.model):
        w = mod.weight
        if not isinstance(w, DTensor):  # layers outside the tensor-parallel plan (text refiner) stay plain
            assert not name.startswith("blocks."), name
            with torch.no_grad():
                for attr in ("lora_a", "lora_b", "lora_magnitude"):
                    if getattr(mod, attr) is not None:
                        getattr(mod, attr).copy_(getattr(ref_mods[name], attr))
            continue
        dim = [p.dim for p in w.placements if isinstance(p, Shard)][0]
        want_a, want_b = ((Replicate(),), (Shard(0),)) if dim == 0 else ((Shard(1),), (Replicate(),))
        assert tuple(mod.lora_a.placements) == want_a and tuple(mod.lora_b.placements) == want_b, name
        if mod.lora_magnitude is not None:
            assert tuple(mod.lora_magnitude.placements) == want_b, name
        checked.add(dim)
        r = ref_mods[name]
        with torch.no_grad():  # the same adapter values as the unsharded model
            for attr in ("lora_a", "lora_b", "lora_magnitude"):
                t = getattr(mod, attr)
                if t is not None:
                    t.copy_(distribute_tensor(getattr(r, attr).detach(), t.device_mesh, list(t.placements)))
    assert checked == {0, 1}, "both column- and row-parallel adapters must be covered"
    out = pm.model(_inputs(61, ref))
    want = ref(_inputs(61, ref))
    torch.testing.assert_close(out.video.detach(), want.video.detach(), rtol=1e-4, atol=1e-5)
    _loss(out).backward()
    _loss(want).backward()
    for name, mod in lora_modules(pm.model):
        for attr in ("lora_a", "lora_b", "lora_magnitude"):
            t = getattr(mod, attr)
            if t is None:
                continue
            g = t.grad.full_tensor() if isinstance(t.grad, DTensor) else t.grad
            torch.testing.assert_close(g, getattr(ref_mods[name], attr).grad, rtol=1e-3, atol=1e-5,
                                       msg=f"{name}.{attr}")


def _dora_tp_worker(rank: int, world: int) -> None:
    _lora_tp_worker(rank, world, use_dora=True)


def _head_parallel_worker(rank: int, world: int, sequence_parallel: bool = False) -> None:
    """Tensor parallelism by whole heads over a prime number of ranks (4 heads over 3:
    an uneven [2, 1, 1] split), with and without sequence-parallel norms: output and
    every gradient match the unsharded model; checkpoints hold full tensors."""
    from avgen_b200.core.tokens import TextContext
    from avgen_b200.infer.conditioning import StreamState, condition_first_frame
    from avgen_b200.parallel import ParallelConfig, ParallelDims, parallelize
    from avgen_b200.parallel.heads import head_partition

    assert head_partition(20, 8) == [3, 3, 3, 3, 2, 2, 2, 2]

    def inputs(model):  # noqa: ANN001, ANN202 - 3 frames x 4 x 4 patches = 48 tokens (divisible by 3)
        g = torch.Generator().manual_seed(71)
        c = model.config
        lat = torch.randn(1, c.in_channels, 3, 8, 8, generator=g)
        text = TextContext(features=torch.randn(1, 6, c.text_width, generator=g),
                           mask=torch.ones(1, 6, dtype=torch.bool))
        return condition_first_frame(StreamState(lat, fps=8.0), lat[:, :, 0], sigma=0.6, text=text,
                                     patchifier=model.patchifier)

    ref = _model()
    want = ref(inputs(ref))
    _loss(want).backward()
    ref_grads = {n: p.grad for n, p in ref.named_parameters()}
    full_state = {k: v.clone() for k, v in ref.state_dict().items()}
    dims = ParallelDims(world_size=world, tensor=world)
    pm = parallelize(_model(), dims, mesh=dims.build_mesh("cpu"),
                     config=ParallelConfig(sequence_parallel=sequence_parallel))
    assert any(f"heads, sequence_parallel={sequence_parallel}" in a for a in pm.applied), pm.applied
    assert pm.model.blocks[0].attention.num_heads == [2, 1, 1][rank]
    out = pm.model(inputs(ref))
    torch.testing.assert_close(out.video.detach(), want.video.detach(), rtol=1e-4, atol=1e-5)
    _loss(out).backward()
    modules = dict(pm.model.named_modules())
    for name, p in pm.model.named_parameters():
        g = ref_grads[name]
        owner = modules[name.rsplit(".", 1)[0]]
        shard = getattr(owner, "_avgen_tp_shard", None)
        if shard is not None and (name.endswith("weight") or shard[0] == 0):
            dim, sizes, _ = shard
            g = g.narrow(dim, sum(sizes[:rank]), sizes[rank])
        torch.testing.assert_close(p.grad, g, rtol=1e-3, atol=1e-5, msg=name)
    saved = pm.model.state_dict()  # gathered to full tensors
    for key, value in full_state.items():
        torch.testing.assert_close(saved[key], value, rtol=0, atol=0, msg=key)
    pm.model.load_state_dict(saved)  # sliced back to this rank's heads


def _head_parallel_sp_worker(rank: int, world: int) -> None:
    _head_parallel_worker(rank, world, sequence_parallel=True)


def _head_parallel_train_worker(rank: int, world: int) -> None:
    """Two clipped AdamW steps with head-parallel sequence-parallel sharding over 3 ranks
    equal two steps of the unsharded model: the global gradient norm sums the squares of
    the ranks' slices once and counts replicated parameters once."""
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.parallel import ParallelConfig, ParallelDims, parallelize
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)

    ref = _model()
    dims = ParallelDims(world_size=world, tensor=world)
    pm = parallelize(_model(), dims, mesh=dims.build_mesh("cpu"), config=ParallelConfig(sequence_parallel=True))
    obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-2), rng=RNGStreams.for_rank(0, data_rank=0))
    ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-2), rng=RNGStreams.for_rank(0, data_rank=0))
    c = ref.config
    gen = torch.Generator().manual_seed(9)
    for step in range(2):
        batch = random_batch(batch=1, channels=c.in_channels, frames=3, height=8, width=8, text_tokens=4,
                             text_width=c.text_width, generator=gen)
        _, m = train_step(state, batch, obj, patchifier=ref.patchifier, max_grad_norm=0.05)
        _, rm = train_step(ref_state, batch, obj, patchifier=ref.patchifier, max_grad_norm=0.05)
        assert abs(float(m.grad_norm) - float(rm.grad_norm)) <= 1e-4 * float(rm.grad_norm), (step, m.grad_norm,
                                                                                              rm.grad_norm)
        full = pm.model.state_dict()
        for name, q in ref.state_dict().items():
            err = (full[name].float() - q.float()).abs().max().item()
            assert err <= 1e-6 + 1e-4 * q.float().abs().max().item(), f"step {step}: {name}: {err}"


@pytest.mark.parametrize("worker", [_head_parallel_worker, _head_parallel_sp_worker, _head_parallel_train_worker],
                         ids=["heads_uneven", "heads_uneven_sequence_parallel", "heads_sp_two_clipped_steps"])
def test_three_rank_head_parallel(worker) -> None:  # noqa: ANN001
    _spawn(worker, 3)


def _sharded_adamw_worker(rank: int, world: int) -> None:
    """AdamW over FSDP-sharded parameters (the multi-tensor optimizer) takes the same
    two clipped steps as torch's AdamW on the unsharded model."""
    from torch.distributed.tensor import DTensor

    from avgen_b200.parallel import ParallelConfig, ParallelDims, PrecisionConfig, parallelize
    from avgen_b200.train import build_optimizer
    from avgen_b200.train.optimizer import MultiTensorAdamW

    ref = _model()
    ref_opt = torch.optim.AdamW(ref.parameters(), lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0)
    model = _model()
    dims = ParallelDims(world_size=world, dp_shard=world)
    pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"),
                     config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32")))
    opt = build_optimizer(pm.model, lr=1e-2, weight_decay=0.0)
    assert isinstance(opt, MultiTensorAdamW)
    for step, seeds in enumerate(([10, 11], [12, 13])):
        ref_opt.zero_grad()
        for s in seeds:  # the unsharded model sees both ranks' samples (mean)
            (_loss(ref(_inputs(s, ref))) / len(seeds)).backward()
        torch.nn.utils.clip_grad_norm_(ref.parameters(), 0.05)
        ref_opt.step()
        opt.zero_grad()
        _loss(pm.model(_inputs(seeds[rank], model))).backward()  # FSDP averages over the 2 ranks
        opt.step(max_grad_norm=0.05)
        assert not bool(opt.last_nonfinite)
        for (n, p), (_, q) in zip(pm.model.named_parameters(), ref.named_parameters()):
            full = p.full_tensor() if isinstance(p, DTensor) else p
            err = (full.detach() - q.detach()).abs().max().item()
            assert err <= 1e-6 + 1e-4 * q.detach().abs().max().item(), f"step {step}: {n}: {err} (|ref| {q.abs().max().item()}, grad None: {p.grad is None})"
    # the optimizer state is per-parameter DTensors placed like the parameters (DCP reshards them)
    st = opt.state_dict()["state"]
    assert all(isinstance(v["exp_avg"], DTensor) for v in st.values())


def _nonfinite_worker(rank: int, world: int) -> None:
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.parallel import ParallelDims, parallelize
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)

    model = _model()
    dims = ParallelDims(world_size=world, dp_replicate=world)
    pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"))
    assert pm.data_group is not None
    opt = build_optimizer(pm.model, lr=1e-2)
    state = TrainState(model=pm.model, optimizer=opt, rng=RNGStreams.for_rank(0, data_rank=rank))
    obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    c = model.config
    batch = random_batch(batch=1, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                         text_width=c.text_width, generator=torch.Generator().manual_seed(rank))
    if rank == 1:
        batch.video.view(-1)[0] = float("nan")
    before = {n: p.detach().clone() for n, p in pm.model.named_parameters()}
    _, metrics = train_step(state, batch, obj, patchifier=model.patchifier, max_grad_norm=1.0,
                            data_group=pm.data_group)
    assert bool(metrics.skipped), "every rank must skip the step when one rank's gradients are non-finite"
    for n, p in pm.model.named_parameters():
        assert torch.equal(p.detach(), before[n]), n
    # a clean step moves the parameters identically on both ranks
    batch.video.nan_to_num_(0.0)
    _, metrics = train_step(state, batch, obj, patchifier=model.patchifier, max_grad_norm=1.0,
                            data_group=pm.data_group)
    assert not bool(metrics.skipped)
    flat = torch.cat([p.detach().reshape(-1) for p in pm.model.parameters()])
    other = flat.clone()
    dist.broadcast(other, src=0)
    torch.testing.assert_close(flat, other)


def _shards_worker(rank: int, world: int) -> None:
    from avgen_b200.data.synthetic import SyntheticConfig, SyntheticSource

    src = SyntheticSource(SyntheticConfig(num_samples=37), data_rank=rank, data_world=world)
    it = iter(src)
    ids = [int(i) for _ in range(len(src)) for i in next(it).sample_ids]
    gathered: list = [None] * world
    dist.all_gather_object(gathered, ids)
    allids = [i for part in gathered for i in part]
    assert len(allids) == len(set(allids)) == 37


@pytest.mark.parametrize("worker", [_fsdp_worker, _tp_worker, _cp_worker, _cp_replicated_worker, _nonfinite_worker,
                                    _sharded_adamw_worker, _pipeline_worker, _pipeline_gpipe_worker,
                                    _pipeline_interleaved_worker, _lora_tp_worker, _dora_tp_worker],
                         ids=["fsdp", "tensor_parallel", "context_parallel", "context_parallel_replicated",
                              "nonfinite_skip", "sharded_adamw", "pipeline_1f1b", "pipeline_gpipe",
                              "pipeline_interleaved_1f1b", "lora_tensor_parallel", "dora_tensor_parallel"])
def test_two_rank_parallelism(worker) -> None:  # noqa: ANN001
    _spawn(worker)


def test_data_shards_disjoint() -> None:
    _spawn(_shards_worker)


class _FakePeerMemory:
    """Stands in for the CUDA IPC calls: a 'handle' names the owning rank's allocation."""

    def __init__(self, rank: int) -> None:
        self.rank = rank
        self.opened: list[bytes] = []
        self.closed: list[int] = []
        self.freed: list[int] = []

    def p2p_alloc(self, nbytes: int, device: int) -> int:
        return (self.rank + 1) << 40

    def p2p_export(self, ptr: int) -> bytes:
        return ptr.to_bytes(8, "little") * 8

    def p2p_open(self, handle: bytes, device: int) -> int:
        self.opened.append(handle)
        return int.from_bytes(handle[:8], "little") + (1 << 20)  # a different address for the mapping

    def p2p_close(self, ptr: int) -> None:
        self.closed.append(ptr)

    def p2p_free(self, ptr: int) -> None:
        self.freed.append(ptr)


def _symmetric_worker(rank: int, world: int) -> None:
    from avgen_b200.parallel.symmetric import SymmetricBuffer

    fake = _FakePeerMemory(rank)
    buf = SymmetricBuffer(4096, dist.group.WORLD, torch.device("cpu"), backend=fake)
    assert buf.ptrs[rank] == (rank + 1) << 40
    for r in range(world):
        if r != rank:
            assert buf.ptrs[r] == ((r + 1) << 40) + (1 << 20)
    assert len(fake.opened) == world - 1
    assert buf.address(1 - rank, 8) == buf.ptrs[1 - rank] + 8
    buf.close()
    assert fake.freed == [(rank + 1) << 40] and len(fake.closed) == world - 1
    # sizes that disagree across ranks are refused on every rank
    with pytest.raises(RuntimeError):
        SymmetricBuffer(4096 + 16 * rank, dist.group.WORLD, torch.device("cpu"), backend=_FakePeerMemory(rank))


def test_symmetric_buffer_handle_exchange() -> None:
    _spawn(_symmetric_worker)


def _sharded_optim_worker(rank: int, world: int) -> None:
    from avgen_b200.train.optimizer import FusedAdamW, ShardedAdamW

    torch.manual_seed(0)
    ref = torch.nn.Sequential(torch.nn.Linear(7, 5), torch.nn.Linear(5, 3))
    sharded = torch.nn.Sequential(torch.nn.Linear(7, 5), torch.nn.Linear(5, 3))
    sharded.load_state_dict(ref.state_dict())
    o_ref = FusedAdamW([{"params": list(ref.parameters()), "weight_decay": 0.1}], lr=1e-2,
                       dp_group=dist.group.WORLD)
    o_sh = ShardedAdamW([{"params": list(sharded.parameters()), "weight_decay": 0.1}], lr=1e-2)
    assert o_sh._flat[0]["exp_avg"].numel() * world == o_sh._flat[0]["param"].numel()  # moments are sharded
    g = torch.Generator().manual_seed(100 + rank)  # every rank sees different gradients
    for step in range(3):
        x = torch.randn(4, 7, generator=g)
        for model, opt in ((ref, o_ref), (sharded, o_sh)):
            opt.zero_grad()
            model(x).pow(2).sum().backward()
            opt.step(max_grad_norm=0.5 if step == 1 else None)
    for a, b in zip(ref.parameters(), sharded.parameters()):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(o_ref.last_grad_norm, o_sh.last_grad_norm, rtol=1e-5, atol=1e-6)
    # full moments gather back for checkpoints (collective on every rank)
    st_ref, st_sh = o_ref.state, o_sh.state
    for p_ref, p_sh in zip(ref.parameters(), sharded.parameters()):
        torch.testing.assert_close(st_ref[p_ref]["exp_avg_sq"], st_sh[p_sh]["exp_avg_sq"], rtol=1e-5, atol=1e-9)


def test_sharded_adamw_matches_replicated() -> None:
    _spawn(_sharded_optim_worker)


def _collective_gemm_worker(rank: int, world: int) -> None:
    from avgen_b200.parallel.collective_gemm import AllGatherGemm, GemmReduceScatter

    g = torch.Generator().manual_seed(3)
    rows, cols, m, n = 4, 16, 6, 8
    w_all = torch.randn(world * rows, cols, generator=g)
    x = torch.randn(m, cols, generator=g)
    ag = AllGatherGemm(dist.group.WORLD, rows, cols, "cpu", operand="b")
    y, full = ag(w_all[rank * rows:(rank + 1) * rows], x)
    torch.testing.assert_close(full, w_all)
    torch.testing.assert_close(y, x @ w_all.t())
    w = torch.randn(n, cols, generator=g)
    sp = AllGatherGemm(dist.group.WORLD, rows, cols, "cpu", operand="a")
    y, _ = sp(w_all[rank * rows:(rank + 1) * rows], w)
    torch.testing.assert_close(y, w_all @ w.t())
    kept = torch.empty(world * rows, cols)
    y, gathered = sp(w_all[rank * rows:(rank + 1) * rows], w, gathered_out=kept)  # rows land in the caller's tensor
    assert gathered is kept
    torch.testing.assert_close(kept, w_all)
    # row-parallel: rank r holds columns [r*c, (r+1)*c) of the reduction axis
    xs = torch.randn(world * rows, world * cols, generator=g)
    ws = torch.randn(n, world * cols, generator=g)
    rs = GemmReduceScatter(dist.group.WORLD, world * rows, n, "cpu")
    part = rs(xs[:, rank * cols:(rank + 1) * cols], ws[:, rank * cols:(rank + 1) * cols])
    torch.testing.assert_close(part, (xs @ ws.t())[rank * rows:(rank + 1) * rows], rtol=1e-4, atol=1e-4)


def test_collective_gemms_match_unsharded() -> None:
    _spawn(_collective_gemm_worker)


class _ViewablePeerMemory(_FakePeerMemory):
    """The fake backend with ``tensor_at`` over host bytes, so guard regions exist."""

    def __init__(self, rank: int) -> None:
        super().__init__(rank)
        self.store = torch.zeros(1 << 16, dtype=torch.uint8)

    def tensor_at(self, ptr: int, sizes: list[int], dtype: torch.dtype, device: int) -> torch.Tensor:
        off = ptr - ((self.rank + 1) << 40)
        n = 1
        for s_ in sizes:
            n *= s_
        item = torch.empty((), dtype=dtype).element_size()
        return self.store[off:off + n * item].view(dtype).view(sizes)


def _guard_worker(rank: int, world: int) -> None:
    from avgen_b200.parallel.symmetric import GUARD_PATTERN, SymmetricBuffer

    fake = _ViewablePeerMemory(rank)
    buf = SymmetricBuffer(1024, dist.group.WORLD, torch.device("cpu"), backend=fake, guard=256)
    assert buf.ptrs[rank] == ((rank + 1) << 40) + 256  # the usable region follows the head guard
    assert int(fake.store[0]) == GUARD_PATTERN and int(fake.store[256 + 1024 + 255]) == GUARD_PATTERN
    buf.view(rank, 0, (256,), torch.float32).fill_(1.0)  # a full in-bounds write leaves the guards intact
    assert buf.check_guards() == []
    fake.store[256 + 1024 + 3] = 0  # one byte past the end
    fake.store[255] = 7  # one byte before the start
    assert buf.check_guards() == [("head", 255), ("tail", 3)]
    buf.close()
    peer = 1 - rank
    assert fake.freed == [(rank + 1) << 40]  # the allocation base, guards included
    assert fake.closed == [((peer + 1) << 40) + (1 << 20)]  # the peer's mapping base, not its usable start


def test_symmetric_buffer_guards_catch_out_of_bounds_writes() -> None:
    _spawn(_guard_worker)


def _sequence_parallel_worker(rank: int, world: int) -> None:
    from avgen_b200.parallel.sequence import sp_column_linear, sp_row_linear

    g = torch.Generator().manual_seed(7)
    t, k, f = 8, 16, 12
    x = torch.randn(t, k, generator=g)
    w1, b1 = torch.randn(f, k, generator=g) * 0.3, torch.randn(f, generator=g)
    w2, b2 = torch.randn(k, f, generator=g) * 0.3, torch.randn(k, generator=g)
    up = torch.randn(t, k, generator=g)
    # unsharded reference MLP
    ref = [p.clone().requires_grad_() for p in (x, w1, b1, w2, b2)]
    y_ref = torch.nn.functional.linear(torch.nn.functional.gelu(torch.nn.functional.linear(ref[0], ref[1], ref[2])),
                                       ref[3], ref[4])
    (y_ref * up).sum().backward()
    # sequence parallel: tokens sharded, first weight by rows, second by columns
    tl, fl = t // world, f // world
    rows, cols = slice(rank * tl, (rank + 1) * tl), slice(rank * fl, (rank + 1) * fl)
    xs = x[rows].clone().requires_grad_()
    w1s, b1s = w1[cols].clone().requires_grad_(), b1[cols].clone().requires_grad_()
    w2s, b2s = w2[:, cols].clone().requires_grad_(), b2.clone().requires_grad_()
    h = sp_column_linear(xs, w1s, b1s, dist.group.WORLD)
    assert h.shape == (t, fl)
    y = sp_row_linear(torch.nn.functional.gelu(h), w2s, b2s, dist.group.WORLD)
    assert y.shape == (tl, k)
    (y * up[rows]).sum().backward()
    close = dict(rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(y, y_ref[rows].detach(), **close)
    torch.testing.assert_close(xs.grad, ref[0].grad[rows], **close)
    torch.testing.assert_close(w1s.grad, ref[1].grad[cols], **close)
    torch.testing.assert_close(b1s.grad, ref[2].grad[cols], **close)
    torch.testing.assert_close(w2s.grad, ref[3].grad[:, cols], **close)
    torch.testing.assert_close(b2s.grad, ref[4].grad, **close)


def test_sequence_parallel_mlp_matches_unsharded() -> None:
    _spawn(_sequence_parallel_worker)


def _sp_validation_worker(rank: int, world: int) -> None:
    from avgen_b200.parallel.collective_gemm import AllGatherGemm, GemmReduceScatter
    from avgen_b200.parallel.sequence import sp_column_linear, sp_row_linear

    g = dist.group.WORLD
    with pytest.raises(ValueError):
        sp_column_linear(torch.zeros(1, 4, 8), torch.zeros(8, 8), None, g)  # needs [tokens, features]
    with pytest.raises(ValueError):
        sp_row_linear(torch.zeros(3, 8), torch.zeros(8, 8), None, g)  # 3 tokens do not split over 2 ranks
    with pytest.raises(ValueError):
        AllGatherGemm(g, 4, 12, "cpu")  # feature count must be a multiple of 8
    with pytest.raises(ValueError):
        AllGatherGemm(g, 4, 16, "cpu", operand="c")
    with pytest.raises(ValueError):
        GemmReduceScatter(g, 5, 16, "cpu")  # rows must split evenly
    ag = AllGatherGemm(g, 4, 16, "cpu")
    with pytest.raises(ValueError):
        ag.gather(torch.zeros(3, 16))  # wrong shard shape


def test_sequence_parallel_argument_checks() -> None:
    _spawn(_sp_validation_worker)


def _tp_cp_worker(rank: int, world: int, sequence_parallel: bool) -> None:
    """Tensor parallelism by heads (3 heads over 2 ranks, uneven) inside context
    parallelism (2 sequence shards) on 4 ranks: the gathered output and every gradient
    (summed over the cp shards, this rank's slice of head-sharded weights) match the
    unsharded model."""
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PrecisionConfig, gather_tokens, parallelize, shard_stream

    def model3():  # noqa: ANN202 - 3 heads: an uneven [2, 1] split over tp=2
        from avgen_b200.models import build_model, preset

        torch.manual_seed(0)
        cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
        cfg.update(num_heads=3, width=48)
        m = build_model("video_dit", cfg)
        m.init_weights()
        with torch.no_grad():
            for p in m.parameters():
                p.add_(0.02 * torch.randn_like(p))
        return m

    ref = model3()
    inputs = _inputs(31, ref)
    want = ref(inputs)
    _loss(want).backward()
    ref_grads = {n: p.grad for n, p in ref.named_parameters()}
    dims = ParallelDims(world_size=world, tensor=2, context=2)
    cfg = ParallelConfig(precision=PrecisionConfig(param_dtype="float32"), shard_parameters=False,
                         sequence_parallel=sequence_parallel)
    pm = parallelize(model3(), dims, mesh=dims.build_mesh("cpu"), config=cfg)
    local = inputs.replace_streams(video=shard_stream(inputs.video, pm.cp_mesh))
    out = pm.model(local)
    torch.testing.assert_close(gather_tokens(out.video.detach(), pm.cp_mesh), want.video.detach(), rtol=1e-4,
                               atol=1e-5)
    _loss(out).backward()
    modules = dict(pm.model.named_modules())
    tp_rank = pm.submesh("tp").get_local_rank()
    for name, p in pm.model.named_parameters():
        g = p.grad.clone()
        dist.all_reduce(g, group=pm.cp_mesh.get_group())  # each cp shard holds a partial loss
        want_g = ref_grads[name]
        shard = getattr(modules[name.rsplit(".", 1)[0]], "_avgen_tp_shard", None)
        if shard is not None and (name.endswith("weight") or shard[0] == 0):
            dim, sizes, _ = shard
            want_g = want_g.narrow(dim, sum(sizes[:tp_rank]), sizes[tp_rank])
        torch.testing.assert_close(g, want_g, rtol=1e-3, atol=1e-5, msg=name)


@pytest.mark.parametrize("sequence_parallel", [False, True], ids=["tp_cp", "tp_sp_cp"])
def test_tensor_inside_context_parallel(sequence_parallel: bool) -> None:
    _spawn(_tp_cp_worker, 4, sequence_parallel)


def _pp_cp_worker(rank: int, world: int) -> None:
    """Two pipeline stages, each over two context-parallel ranks (4 ranks): one 1F1B
    optimizer step over 2 micro-batches matches the unsharded model's loss and
    gradient norm with gradient accumulation."""
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PipelineConfig, PrecisionConfig, parallelize
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)
    from avgen_b200.train.trainer import pipeline_train_step

    ref = _model()
    dims = ParallelDims(world_size=world, pipeline=2, context=2)
    pm = parallelize(_model(), dims, mesh=dims.build_mesh("cpu"),
                     config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32"), shard_parameters=False,
                                           pipeline=PipelineConfig(schedule="1f1b")))
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-2),
                       rng=RNGStreams.for_rank(0, data_rank=0))
    ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-2), rng=RNGStreams.for_rank(0, data_rank=0))
    c = ref.config
    gen = torch.Generator().manual_seed(5)
    micro = [random_batch(batch=1, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                          text_width=c.text_width, generator=gen) for _ in range(2)]
    _, metrics = pipeline_train_step(state, micro, objective, pm.pipeline, patchifier=ref.patchifier,
                                     max_grad_norm=None, pp_mesh=pm.pp_mesh, cp_mesh=pm.cp_mesh,
                                     data_group=pm.data_group)  # replicated parameters: gradients summed over cp
    losses = []
    for i, b in enumerate(micro):
        _, rm = train_step(ref_state, b, objective, patchifier=ref.patchifier, gradient_accumulation_steps=2,
                           microbatch_index=i, max_grad_norm=None)
        losses.append(float(rm.loss))
    loss = metrics.loss.detach().reshape(1).clone()
    dist.all_reduce(loss, group=pm.cp_mesh.get_group())  # each cp rank reports its shard's share
    assert abs(float(loss) / 2 - sum(losses) / 2) <= 1e-4 * max(1.0, abs(sum(losses))), (float(loss), losses)
    assert abs(float(metrics.grad_norm) - float(rm.grad_norm)) <= 1e-3 * float(rm.grad_norm), (
        float(metrics.grad_norm), float(rm.grad_norm))


def test_pipeline_over_context_parallel_stages() -> None:
    _spawn(_pp_cp_worker, 4)


def _pp_combo_worker(rank: int, world: int, other: str) -> None:
    """Two pipeline stages, each over two ranks of another layout (head-parallel TP with
    sequence parallelism, or FSDP2 sharding): one clipped 1F1B optimizer step over 2
    micro-batches matches the unsharded model's loss and gradient norm."""
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PipelineConfig, PrecisionConfig, parallelize
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)
    from avgen_b200.train.trainer import pipeline_train_step

    def model3():  # noqa: ANN202 - 3 heads, 2 blocks
        from avgen_b200.models import build_model, preset

        torch.manual_seed(0)
        cfg = {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"}
        cfg.update(num_heads=3, width=48)
        m = build_model("video_dit", cfg)
        m.init_weights()
        with torch.no_grad():
            for p in m.parameters():
                p.add_(0.02 * torch.randn_like(p))
        return m

    ref = model3()
    if other == "tp":
        dims = ParallelDims(world_size=world, pipeline=2, tensor=2)
        extra = {"sequence_parallel": True}
    else:
        dims = ParallelDims(world_size=world, pipeline=2, dp_shard=2)
        extra = {}
    pm = parallelize(model3(), dims, mesh=dims.build_mesh("cpu"),
                     config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32"),
                                           pipeline=PipelineConfig(schedule="1f1b"), **extra))
    objective = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    # micro-batch i draws its noise from the stream of data rank i, here and in the reference
    data_rank = pm.submesh("dp_shard").get_local_rank() if other == "fsdp" else 0
    state = TrainState(model=pm.model, optimizer=build_optimizer(pm.model, lr=1e-2),
                       rng=RNGStreams.for_rank(0, data_rank=data_rank))
    ref_state = TrainState(model=ref, optimizer=build_optimizer(ref, lr=1e-2), rng=RNGStreams.for_rank(0, data_rank=0))
    c = ref.config
    gen = torch.Generator().manual_seed(5)
    micro = [random_batch(batch=1, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                          text_width=c.text_width, generator=gen) for _ in range(2)]
    # the two data ranks of a stage see one sample each; the unsharded step sees both
    mine = [micro[data_rank]] if other == "fsdp" else micro
    _, metrics = pipeline_train_step(state, mine, objective, pm.pipeline, patchifier=ref.patchifier,
                                     max_grad_norm=0.05, pp_mesh=pm.pp_mesh, data_group=pm.data_group)
    losses = []
    for i, b in enumerate(micro):
        if other == "fsdp":
            ref_state.rng = RNGStreams.for_rank(0, data_rank=i)
        _, rm = train_step(ref_state, b, objective, patchifier=ref.patchifier, gradient_accumulation_steps=2,
                           microbatch_index=i, max_grad_norm=0.05)
        losses.append(float(rm.loss))
    loss = metrics.loss.detach().reshape(1).clone()
    if other == "fsdp":
        dist.all_reduce(loss, group=pm.submesh("dp_shard").get_group())
        loss /= 2
    assert abs(float(loss) - sum(losses) / 2) <= 1e-4 * max(1.0, abs(sum(losses))), (float(loss), losses)
    assert abs(float(metrics.grad_norm) - float(rm.grad_norm)) <= 1e-3 * float(rm.grad_norm), (
        float(metrics.grad_norm), float(rm.grad_norm))


@pytest.mark.parametrize("other", ["tp", "fsdp"])
def test_pipeline_with_tensor_or_sharded_data_parallel_stages(other: str) -> None:
    _spawn(_pp_combo_worker, 4, other)
