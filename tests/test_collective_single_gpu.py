"""The peer-memory paths on one GPU: a one-rank NCCL group runs the sharded
AdamW kernels (gradient pull with the norm partial, AdamW with the parameter
push), the fused all-gather GEMM and GEMM reduce-scatter, and the trainable
sequence-parallel linears through the same symmetric buffers, flags and
barriers as at several ranks, against the replicated / unsharded results.
What one rank cannot show (peer reads over NVLink, overlap of the transfer) is
covered by the multi-GPU tests."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, port: int) -> None:
    from datetime import timedelta

    import torch.distributed as dist
    import torch.nn.functional as F

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0", WORLD_SIZE="1")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from avgen_b200.ops import kernels as K
        from avgen_b200.ops._ext import check_errors
        from avgen_b200.parallel.collective_gemm import AllGatherGemm, GemmReduceScatter
        from avgen_b200.parallel.sequence import _POOL, sp_column_linear, sp_row_linear
        from avgen_b200.train.optimizer import FusedAdamW, ShardedAdamW

        group = dist.group.WORLD
        # sharded AdamW (one shard) against the replicated optimizer
        torch.manual_seed(0)
        ref = torch.nn.Sequential(torch.nn.Linear(300, 257), torch.nn.Linear(257, 64)).to(dev)
        sh = torch.nn.Sequential(torch.nn.Linear(300, 257), torch.nn.Linear(257, 64)).to(dev)
        sh.load_state_dict(ref.state_dict())
        o_ref = FusedAdamW([{"params": list(ref.parameters()), "weight_decay": 0.1}], lr=1e-3)
        o_sh = ShardedAdamW([{"params": list(sh.parameters()), "weight_decay": 0.1}], lr=1e-3, group=group)
        g = torch.Generator(device=dev).manual_seed(3)
        for step in range(3):
            x = torch.randn(16, 300, generator=g, device=dev)
            for model, opt in ((ref, o_ref), (sh, o_sh)):
                opt.zero_grad()
                model(x).pow(2).mean().backward()
                opt.step(max_grad_norm=0.5 if step == 1 else None)
        torch.cuda.synchronize()
        assert check_errors(dev) == 0
        for a, b in zip(ref.parameters(), sh.parameters()):
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(o_ref.last_grad_norm, o_sh.last_grad_norm, rtol=1e-4, atol=1e-6)
        for flat in o_sh._flat:
            assert not flat["pbuf"].check_guards() and not flat["gbuf"].check_guards()

        # fused all-gather GEMM (both operands) and GEMM reduce-scatter
        x = torch.randn(1024, 512, device=dev).bfloat16()
        w = (torch.randn(768, 512, device=dev) * 0.05).bfloat16()
        ag_b = AllGatherGemm(group, 768, 512, dev, operand="b")
        ag_a = AllGatherGemm(group, 1024, 512, dev, operand="a")
        rs = GemmReduceScatter(group, 1024, 768, dev)
        ref_y = K.gemm(x, w)
        for _ in range(2):
            yb, fb = ag_b(w, x)
            ya, fa = ag_a(x, w)
            yr = rs(x, w)
        torch.cuda.synchronize()
        assert torch.equal(fb, w) and torch.equal(fa, x)
        for y in (yb, ya, yr):
            assert (y.float() - ref_y.float()).abs().max().item() <= 1e-2 * (1 + ref_y.float().abs().max().item())
        for prim in (ag_b, ag_a, rs):
            assert not prim.buf.check_guards()
            prim.close()

        # sequence-parallel MLP (one shard) against the unsharded MLP, forward and gradients
        t, k, f = 512, 256, 512
        xs = torch.randn(t, k, device=dev).requires_grad_()
        w1 = (torch.randn(f, k, device=dev) * 0.05).requires_grad_()
        w2 = (torch.randn(k, f, device=dev) * 0.05).requires_grad_()
        up = torch.randn(t, k, device=dev)
        y = sp_row_linear(F.gelu(sp_column_linear(xs, w1, None, group).float()), w2, None, group)
        (y.float() * up).sum().backward()
        got = (y.detach().float(), xs.grad.clone(), w1.grad.clone(), w2.grad.clone())
        refs = [p.detach().clone().requires_grad_() for p in (xs, w1, w2)]
        y_ref = F.linear(F.gelu(F.linear(refs[0], refs[1])), refs[2])
        (y_ref * up).sum().backward()
        for a, r in zip(got, (y_ref.detach(), refs[0].grad, refs[1].grad, refs[2].grad)):
            err = (a - r).abs().max().item()
            assert err <= 3e-2 * (1 + r.abs().max().item()), f"max err {err}"
        torch.cuda.synchronize()
        assert check_errors(dev) == 0
        for prim in _POOL.values():
            assert not prim.buf.check_guards()
            prim.close()
    finally:
        dist.barrier(device_ids=[0])
        dist.destroy_process_group()


def test_peer_memory_paths_on_one_rank() -> None:
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(_free_port(),), nprocs=1, join=True)
