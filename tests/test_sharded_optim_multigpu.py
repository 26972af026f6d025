"""Sharded AdamW over NVLink peer memory on 2 GPUs: the gradient shard pulled
from every peer and reduced in one kernel, the AdamW update pushing each
parameter into every peer's buffer in another; parameters, gradient norm and
gathered moments must match the replicated fused AdamW with an NCCL gradient
all-reduce."""
from __future__ import annotations

import os
import socket

import pytest
import torch
from multigpu_util import leave_on_failure

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from avgen_b200.ops._ext import check_errors
        from avgen_b200.train.optimizer import FusedAdamW, ShardedAdamW

        torch.manual_seed(0)
        ref = torch.nn.Sequential(torch.nn.Linear(300, 257), torch.nn.Linear(257, 64)).to(dev)
        sharded = torch.nn.Sequential(torch.nn.Linear(300, 257), torch.nn.Linear(257, 64)).to(dev)
        sharded.load_state_dict(ref.state_dict())
        o_ref = FusedAdamW([{"params": list(ref.parameters()), "weight_decay": 0.1}], lr=1e-3,
                           dp_group=dist.group.WORLD)
        o_sh = ShardedAdamW([{"params": list(sharded.parameters()), "weight_decay": 0.1}], lr=1e-3)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        for step in range(3):
            x = torch.randn(16, 300, generator=g, device=dev)
            for model, opt in ((ref, o_ref), (sharded, o_sh)):
                opt.zero_grad()
                model(x).pow(2).mean().backward()
                opt.step(max_grad_norm=0.5 if step == 1 else None)
        torch.cuda.synchronize()
        assert check_errors(dev) == 0
        for a, b in zip(ref.parameters(), sharded.parameters()):
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(o_ref.last_grad_norm, o_sh.last_grad_norm, rtol=1e-4, atol=1e-6)
        for flat in o_sh._flat:  # the peer pulls and pushes stayed inside the symmetric buffers
            assert not flat["pbuf"].check_guards() and not flat["gbuf"].check_guards()
        st_ref, st_sh = o_ref.state, o_sh.state
        for p_ref, p_sh in zip(ref.parameters(), sharded.parameters()):
            torch.testing.assert_close(st_ref[p_ref]["exp_avg"], st_sh[p_sh]["exp_avg"], rtol=1e-5, atol=1e-8)
    except BaseException:
        leave_on_failure()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_sharded_adamw_two_gpus() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
