"""Kernel numerics at the shapes the 2B benchmark runs, against fp32 PyTorch.

* Attention at H=20 heads, L=16,384 (the per-rank sequence at cp=4): forward
  output and dQ on a random subset of query rows, dK / dV on a subset of key
  rows (their fp32 values need the whole sequence, computed in query chunks).
* The weight-gradient GEMM at its production reduction length: dW[2560, 2560]
  accumulated over 65,536 rows through the split-K fp32 atomic epilogue.
* A full-width DiT block (2560 wide, 20 heads of 128, SwiGLU 10240) through the
  fused sm_100a path against the eager fp32 block on the same weights.
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    return float((got.float() - ref.float()).norm() / ref.float().norm().clamp_min(1e-12))


def test_attention_20_heads_16k_sampled_rows_match_fp32() -> None:
    from avgen_b200.ops import kernels as K
    from avgen_b200.ops._ext import check_errors

    torch.manual_seed(0)
    b, h, length, d = 1, 20, 16384, 128
    scale = 1.0 / math.sqrt(d)
    q = torch.randn(b, h, length, d, device=DEV).bfloat16()
    k = torch.randn(b, h, length, d, device=DEV).bfloat16()
    v = torch.randn(b, h, length, d, device=DEV).bfloat16()
    out, lse = K.attention_fwd(q, k, v, scale=scale)
    dout = torch.randn(b, length, h, d, device=DEV).bfloat16()
    dq, dk, dv = K.attention_bwd(q, k, v, out, dout, lse, scale=scale)
    torch.cuda.synchronize()
    g = torch.Generator(device="cpu").manual_seed(1)
    for head in (0, 7, 19):
        qf, kf, vf = (t[0, head].float() for t in (q, k, v))
        do = dout[0, :, head].float()
        rows = torch.randperm(length, generator=g)[:96].to(DEV)
        s = (qf[rows] @ kf.T) * scale
        p = torch.softmax(s, -1)
        o = p @ vf
        assert _rel(out[0, rows, head], o) < 1e-2
        # dq for the sampled rows: dS = P * (dP - delta), delta = rowsum(dO * O)
        dp = do[rows] @ vf.T
        delta = (do[rows] * o).sum(-1, keepdim=True)
        dq_ref = (p * (dp - delta)) @ kf * scale
        assert _rel(dq[0, head, rows], dq_ref) < 2e-2
        # dk / dv for sampled key rows need every query: accumulate over query chunks in fp32
        keys = torch.randperm(length, generator=g)[:64].to(DEV)
        dk_ref = torch.zeros(64, d, device=DEV)
        dv_ref = torch.zeros(64, d, device=DEV)
        for lo in range(0, length, 2048):
            qc, doc = qf[lo:lo + 2048], do[lo:lo + 2048]
            sc = (qc @ kf.T) * scale
            pc = torch.softmax(sc, -1)
            oc = pc @ vf
            dpc = doc @ vf[keys].T
            deltac = (doc * oc).sum(-1, keepdim=True)
            pk = pc[:, keys]
            dv_ref += pk.T @ doc
            dk_ref += (pk * (dpc - deltac)).T @ qc * scale
        assert _rel(dv[0, head, keys], dv_ref) < 2e-2
        assert _rel(dk[0, head, keys], dk_ref) < 2e-2
    assert check_errors() == 0


def test_weight_gradient_split_k_at_65536_rows_matches_fp32() -> None:
    from avgen_b200.ops import kernels as K
    from avgen_b200.ops._ext import check_errors

    torch.manual_seed(2)
    rows, n, k = 65536, 2560, 2560
    dy = torch.randn(rows, n, device=DEV).bfloat16()
    x = torch.randn(rows, k, device=DEV).bfloat16()
    grad = torch.zeros(n, k, device=DEV)
    K.linear_dw(dy, x, grad)
    ref = dy.float().T @ x.float()
    assert _rel(grad, ref) < 1e-4  # fp32 accumulation of exact bf16 products
    assert float((grad - ref).abs().max()) < 1e-3 * float(ref.abs().max())
    assert check_errors() == 0


def test_full_width_block_fused_matches_cpu_fp32() -> None:
    import copy

    from avgen_b200.models.blocks import DiTBlock, RopeInputs
    from avgen_b200.models.rope import RotaryEmbedding

    torch.manual_seed(3)
    width, heads, hidden, length = 2560, 20, 10240, 512
    cpu_block = DiTBlock(width, heads, hidden=hidden, context_width=width)
    cpu_block.init_weights(depth=32)
    with torch.no_grad():
        for p in cpu_block.parameters():
            p.add_(0.01 * torch.randn_like(p))
    block = copy.deepcopy(cpu_block).to(DEV)
    x = torch.randn(1, length, width)
    mod = 0.1 * torch.randn(1, 6, width)
    ctx = torch.randn(1, 64, width)
    coords = torch.stack(torch.meshgrid(torch.arange(2.0), torch.arange(16.0), torch.arange(16.0), indexing="ij"),
                         -1).reshape(1, length, 3)
    rotary = RotaryEmbedding(width // heads)
    g = torch.randn(1, length, width)
    # fused sm_100a path (bf16 operands, fp32 accumulation) on the GPU
    xf = x.to(DEV).requires_grad_()
    fused = block(xf, modulation=mod.to(DEV), rope=RopeInputs(coords=coords.to(DEV), rope=copy.deepcopy(rotary).to(DEV)),
                  context=ctx.to(DEV))
    (gf,) = torch.autograd.grad(fused, xf, g.to(DEV))
    # eager fp32 oracle on the CPU
    xe = x.clone().requires_grad_()
    eager = cpu_block(xe, modulation=mod, rope=RopeInputs(coords=coords, rope=rotary), context=ctx)
    (ge,) = torch.autograd.grad(eager, xe, g)
    assert _rel(fused.cpu(), eager) < 2e-2
    assert _rel(gf.cpu(), ge) < 3e-2
