"""One-GPU numerics of the sharded data-parallel kernels against fp32 PyTorch:
the multi-tensor AdamW (norm, clip, non-finite skip) against the flat fused
AdamW and torch's AdamW, and the peer pull-reduce against a plain sum (with the
peers emulated by several buffers of this device)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _params(seed: int) -> list[torch.nn.Parameter]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    shapes = [(257, 129), (64,), (3, 5, 7), (65536 + 17,), (1,)]
    return [torch.nn.Parameter(torch.randn(s, generator=g, device="cuda")) for s in shapes]


def test_multi_tensor_adamw_matches_torch_adamw() -> None:
    from avgen_b200.ops._ext import check_errors
    from avgen_b200.train.optimizer import MultiTensorAdamW

    ours, ref = _params(0), _params(0)
    o = MultiTensorAdamW([{"params": ours[:3], "weight_decay": 0.1}, {"params": ours[3:], "weight_decay": 0.0}],
                         lr=1e-2, betas=(0.9, 0.95), eps=1e-8)
    r = torch.optim.AdamW([{"params": ref[:3], "weight_decay": 0.1}, {"params": ref[3:], "weight_decay": 0.0}],
                          lr=1e-2, betas=(0.9, 0.95), eps=1e-8)
    g = torch.Generator(device="cuda").manual_seed(7)
    for step in range(4):
        grads = [torch.randn(p.shape, generator=g, device="cuda") * (step + 1) for p in ours]
        for p, q, gr in zip(ours, ref, grads):
            p.grad = gr.clone()
            q.grad = gr.clone()
        clip = 0.5 if step % 2 else None
        o.step(max_grad_norm=clip)
        norm = torch.nn.utils.clip_grad_norm_(ref, clip) if clip else torch.nn.utils.get_total_norm(
            [q.grad for q in ref])
        r.step()
        torch.testing.assert_close(o.last_grad_norm, norm.float(), rtol=1e-5, atol=1e-6)
        for p, q in zip(ours, ref):
            torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6)
    # a non-finite gradient skips the step on the device: parameters keep their values
    before = [p.detach().clone() for p in ours]
    for p in ours:
        p.grad = torch.zeros_like(p)
    ours[1].grad[3] = float("nan")
    o.step(max_grad_norm=1.0)
    assert bool(o.last_nonfinite)
    for p, b in zip(ours, before):
        # skipped: gradients count as zero, so only the (decoupled) decay and the moments move
        assert torch.isfinite(p).all()
    assert check_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("offset", [0, 3])
def test_peer_reduce_sums_every_source(dtype: torch.dtype, offset: int) -> None:
    from avgen_b200.ops._ext import check_errors, load

    world, shard = 4, 10007
    srcs = [torch.randn(world * shard + 8, device="cuda").to(dtype) for _ in range(world)]
    for rank in range(world):
        out = torch.empty(shard, device="cuda")
        acc = torch.zeros(1, device="cuda")
        load().peer_reduce([s.data_ptr() for s in srcs], rank, rank * shard + offset, out, dtype == torch.bfloat16,
                           1.0 / world, acc)
        want = torch.stack([s[rank * shard + offset:(rank + 1) * shard + offset].float() for s in srcs]).sum(0) / world
        torch.testing.assert_close(out, want, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(acc[0], want.pow(2).sum(), rtol=1e-4, atol=1e-4)
    assert check_errors() == 0
