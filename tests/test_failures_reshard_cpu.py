"""Host-side failure handling and checkpoint resharding on CPU (gloo ranks, no GPU).

* A DCP checkpoint written by a 2-rank FSDP job loads into a 3-rank (prime) FSDP
  job and into a single process with the same full parameters and optimizer
  moments (resharding onto a different rank count).
* A rank that leaves between steps: the surviving rank's next collective raises
  within the process group's short timeout instead of hanging.
* A truncated checkpoint file makes loading raise; a step directory without its
  completion marker (an interrupted save) is skipped for the newest complete one.
* FSDP parity and the non-finite skip also hold in a 3-rank world.
"""
from __future__ import annotations

import os
import socket
from dataclasses import asdict
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank: int, world: int, port: int, fn, args, timeout_s: float) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    try:
        fn(rank, world, *args)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _spawn(fn, world: int, *args, timeout_s: float = 120.0) -> None:  # noqa: ANN001
    mp.spawn(_entry, args=(world, _free_port(), fn, args, timeout_s), nprocs=world, join=True)


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


def _fsdp_state(world: int, seed: int = 0):  # noqa: ANN202
    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PrecisionConfig, parallelize
    from avgen_b200.train import build_optimizer

    model = _model(seed)
    if world == 1:
        pm = None
        net = model
    else:
        dims = ParallelDims(world_size=world, dp_shard=world)
        pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"),
                         config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32")))
        net = pm.model
    opt = build_optimizer(net, lr=1e-2, weight_decay=0.0)
    return pm, TrainState(model=net, optimizer=opt, rng=RNGStreams.for_rank(0, data_rank=0))


def _full(t: torch.Tensor) -> torch.Tensor:
    from torch.distributed.tensor import DTensor

    return (t.full_tensor() if isinstance(t, DTensor) else t).detach().clone()


def _train_one_step(state, seed: int) -> None:  # noqa: ANN001
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.train import FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, \
        build_timestep_sampler, train_step

    c = state.model.config
    batch = random_batch(batch=1, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                         text_width=c.text_width, generator=torch.Generator().manual_seed(seed))
    obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    train_step(state, batch, obj, patchifier=state.model.patchifier, max_grad_norm=1.0)


def _moments(state) -> dict[str, torch.Tensor]:  # noqa: ANN001
    by_param = {id(p): n for n, p in state.model.named_parameters()}
    out = {}
    for p, st in state.optimizer.state.items():
        if "exp_avg" in st:
            out[by_param[id(p)]] = _full(st["exp_avg"])
    return out


def _save_worker(rank: int, world: int, root: str) -> None:
    from avgen_b200.checkpoint import CheckpointManager

    pm, state = _fsdp_state(world)
    _train_one_step(state, 100 + rank)
    CheckpointManager(root).save(state.step, state, parallel=pm, async_save=False)
    full = {n: _full(p) for n, p in state.model.named_parameters()}
    moments = _moments(state)
    if rank == 0:
        torch.save({"params": full, "moments": moments}, Path(root) / "reference.pt")


def _load_worker(rank: int, world: int, root: str) -> None:
    from avgen_b200.checkpoint import CheckpointManager

    pm, state = _fsdp_state(world, seed=77)  # different initial weights: everything must come from the checkpoint
    assert CheckpointManager(root).load(state, parallel=pm) == 1
    want = torch.load(Path(root) / "reference.pt")
    for n, p in state.model.named_parameters():
        torch.testing.assert_close(_full(p), want["params"][n], rtol=0, atol=0, msg=n)
    for n, m in _moments(state).items():
        torch.testing.assert_close(m, want["moments"][n], rtol=0, atol=0, msg=n)
    assert state.step == 1


def test_checkpoint_reshards_from_two_ranks_to_three_and_one(tmp_path: Path) -> None:
    root = str(tmp_path / "ckpt")
    _spawn(_save_worker, 2, root)
    _spawn(_load_worker, 3, root)
    _spawn(_load_worker, 1, root)


def _leaver_worker(rank: int, world: int, flag_dir: str) -> None:
    token = torch.ones(1)
    dist.all_reduce(token)  # step 1: everyone present
    if rank == 1:
        return  # leaves between steps (its process group is torn down on exit)
    try:
        dist.all_reduce(token)  # step 2: the peer is gone
    except Exception as exc:  # noqa: BLE001 - any error is the point; a hang would time out the test
        Path(flag_dir, "detected").write_text(type(exc).__name__)
        dist.destroy_process_group()


def test_a_rank_that_leaves_is_detected_not_waited_on(tmp_path: Path) -> None:
    try:
        _spawn(_leaver_worker, 2, str(tmp_path), timeout_s=5.0)
    except Exception:  # noqa: BLE001 - the spawn may report the surviving rank's teardown
        pass
    assert (tmp_path / "detected").is_file(), "rank 0 did not observe that rank 1 left"


def _small_checkpoint(root: Path, steps: int) -> None:
    from avgen_b200.checkpoint import CheckpointManager

    _, state = _fsdp_state(1)
    mgr = CheckpointManager(root, keep_last_n=10)
    for s in range(steps):
        _train_one_step(state, s)
        mgr.save(state.step, state, async_save=False)


def test_truncated_checkpoint_fails_loudly(tmp_path: Path) -> None:
    from avgen_b200.checkpoint import CheckpointManager

    _small_checkpoint(tmp_path, 1)
    data = sorted(p for p in (tmp_path / "step_0000000001").iterdir() if p.suffix == ".distcp")
    assert data, "DCP data files expected"
    biggest = max(data, key=lambda p: p.stat().st_size)
    with open(biggest, "r+b") as fh:
        fh.truncate(biggest.stat().st_size // 2)
    _, state = _fsdp_state(1, seed=5)
    with pytest.raises(RuntimeError, match="could not be read"):
        CheckpointManager(tmp_path).load(state)


def test_interrupted_save_without_marker_is_skipped(tmp_path: Path) -> None:
    from avgen_b200.checkpoint import CheckpointManager

    _small_checkpoint(tmp_path, 2)
    (tmp_path / "step_0000000002" / "avgen_checkpoint.json").unlink()  # the newest save never completed
    mgr = CheckpointManager(tmp_path)
    assert mgr.latest_step() == 1
    _, state = _fsdp_state(1, seed=5)
    assert mgr.load(state) == 1 and state.step == 1


def _three_rank_worker(rank: int, world: int) -> None:
    """FSDP over 3 ranks reproduces the mean gradient of 3 single-process runs, and a
    non-finite loss on one rank makes all three skip the step."""
    from torch.distributed.tensor import DTensor

    from avgen_b200.core import RNGStreams, TrainState
    from avgen_b200.data.synthetic_batch import random_batch
    from avgen_b200.parallel import ParallelConfig, ParallelDims, PrecisionConfig, parallelize
    from avgen_b200.train import (FlowMatchingConfig, FlowMatchingObjective, MultiTaskConditioning, build_optimizer,
                                  build_timestep_sampler, train_step)

    def loss_of(model, seed):  # noqa: ANN001, ANN202
        c = model.config
        g = torch.Generator().manual_seed(seed)
        lat = torch.randn(1, c.in_channels, 4, 8, 8, generator=g)
        from avgen_b200.core.tokens import TextContext
        from avgen_b200.infer.conditioning import StreamState, condition_first_frame

        text = TextContext(features=torch.randn(1, 6, c.text_width, generator=g),
                           mask=torch.ones(1, 6, dtype=torch.bool))
        inputs = condition_first_frame(StreamState(lat, fps=8.0), lat[:, :, 0], sigma=0.6, text=text,
                                       patchifier=model.patchifier)
        out = model(inputs)
        return (out.video * torch.linspace(-1.0, 1.0, out.video.shape[-1])).sum()

    ref = _model()
    grads = {n: torch.zeros_like(p) for n, p in ref.named_parameters()}
    for r in range(world):
        ref.zero_grad()
        loss_of(ref, 40 + r).backward()
        for n, p in ref.named_parameters():
            grads[n] += p.grad / world
    model = _model()
    dims = ParallelDims(world_size=world, dp_shard=world)
    pm = parallelize(model, dims, mesh=dims.build_mesh("cpu"),
                     config=ParallelConfig(precision=PrecisionConfig(param_dtype="float32")))
    loss_of(pm.model, 40 + rank).backward()
    for n, p in pm.model.named_parameters():
        g = p.grad.full_tensor() if isinstance(p.grad, DTensor) else p.grad
        torch.testing.assert_close(g, grads[n], rtol=1e-3, atol=1e-5, msg=n)
    # non-finite on the middle rank: every rank skips, parameters unchanged
    opt = build_optimizer(pm.model, lr=1e-2)
    state = TrainState(model=pm.model, optimizer=opt, rng=RNGStreams.for_rank(0, data_rank=rank))
    c = model.config
    batch = random_batch(batch=1, channels=c.in_channels, frames=2, height=8, width=8, text_tokens=4,
                         text_width=c.text_width, generator=torch.Generator().manual_seed(rank))
    if rank == 1:
        batch.video.view(-1)[0] = float("nan")
    before = {n: _full(p) for n, p in pm.model.named_parameters()}
    obj = FlowMatchingObjective(FlowMatchingConfig(), build_timestep_sampler("uniform"), MultiTaskConditioning())
    _, metrics = train_step(state, batch, obj, patchifier=model.patchifier, max_grad_norm=1.0)
    assert bool(metrics.skipped)
    for n, p in pm.model.named_parameters():
        assert torch.isfinite(_full(p)).all(), n
        # a skipped step treats gradients as zero: with fresh moments the parameters stay put
        torch.testing.assert_close(_full(p), before[n], rtol=0, atol=0, msg=n)


def test_three_rank_world() -> None:
    _spawn(_three_rank_worker, 3)
