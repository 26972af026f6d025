"""The allocation-free attention-backward C entry point (``avgen_attn_bwd_noalloc``).

Some callers cannot allocate device memory per call (a runtime replaying
captured CUDA graphs, a process that budgets device memory once at start-up);
this entry point keeps its scratch in a static device array instead. The test
calls it through the exported C symbol with ctypes, twice in a row (the second
call reuses the first call's scratch), checks its device error word through
``avgen_attn_bwd_noalloc_device_error``, and compares the gradients with the
Python entry point ``avgen_b200.ops.kernels.attention_bwd`` and with fp32
autograd of plain PyTorch attention.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib() -> ctypes.CDLL:
    from avgen_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.avgen_attn_bwd_noalloc
    vp = ctypes.c_void_p
    fn.argtypes = [vp, vp, vp, vp, vp, vp, ctypes.c_long, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, vp]
    fn.restype = ctypes.c_int
    lib.avgen_attn_bwd_noalloc_last_error.restype = ctypes.c_char_p
    lib.avgen_attn_bwd_noalloc_device_error.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    lib.avgen_attn_bwd_noalloc_device_error.restype = ctypes.c_int
    return lib


def _device_error(lib: ctypes.CDLL, *, clear: bool = False) -> int:
    word = ctypes.c_int(-1)
    status = lib.avgen_attn_bwd_noalloc_device_error(ctypes.byref(word), 1 if clear else 0)
    assert status == 0, lib.avgen_attn_bwd_noalloc_last_error().decode()
    return word.value


def _fp32_grads(q, k, v, dout, valid, scale):  # noqa: ANN001, ANN202
    """dq, dk, dv of plain fp32 attention (GQA by repeating K/V heads)."""
    group = q.shape[1] // k.shape[1]
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    kr, vr = kf.repeat_interleave(group, 1), vf.repeat_interleave(group, 1)
    s = torch.einsum("bhqd,bhkd->bhqk", qf, kr) * scale
    if valid is not None:
        s = s.masked_fill(~valid[:, None, None, :], float("-inf"))
    o = torch.einsum("bhqk,bhkd->bhqd", s.softmax(-1), vr)
    o.backward(dout.float().permute(0, 2, 1, 3))  # dout is [B, Lq, H, D]
    return qf.grad, kf.grad, vf.grad


def _call(lib: ctypes.CDLL, q, k, v, o, dout, lse, kmask, scale):  # noqa: ANN001, ANN202
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    b, h, lq, _ = q.shape
    hk, lk = k.shape[1], k.shape[2]
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    status = lib.avgen_attn_bwd_noalloc(ptr(q), ptr(k), ptr(v), ptr(o), ptr(dout), ptr(lse), lse.stride(1), ptr(dq),
                                        ptr(dk), ptr(dv), ptr(kmask), 0 if kmask is None else kmask.stride(0), b, h,
                                        hk, lq, lk, scale, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == 0, lib.avgen_attn_bwd_noalloc_last_error().decode()
    return dq, dk, dv


@pytest.mark.parametrize("masked", [False, True])
def test_noalloc_matches_entry_point(masked: bool, monkeypatch: pytest.MonkeyPatch) -> None:
    from avgen_b200.ops import kernels as K

    lib = _lib()
    _device_error(lib, clear=True)
    torch.manual_seed(21)
    b, h, hk, lq, lk, d = 2, 4, 2, 390, 301, 128
    q = torch.randn(b, h, lq, d, device="cuda").bfloat16()
    k = torch.randn(b, hk, lk, d, device="cuda").bfloat16()
    v = torch.randn(b, hk, lk, d, device="cuda").bfloat16()
    kmask = valid = None
    if masked:
        valid = torch.rand(b, lk, device="cuda") > 0.3
        valid[:, 0] = True
        kmask = K.pack_key_mask(valid)
    scale = 1.0 / math.sqrt(d)
    o, lse = K.attention_fwd(q, k, v, kmask=kmask, scale=scale)
    dout = torch.randn_like(o)
    first = _call(lib, q, k, v, o, dout, lse, kmask, scale)
    second = _call(lib, q, k, v, o, dout, lse, kmask, scale)
    torch.cuda.synchronize()
    for a, c in zip(first, second):  # scratch reuse between calls changes nothing
        assert torch.equal(a, c)
    monkeypatch.setattr(K, "_ATTN_BWD", "split")
    ref = K.attention_bwd(q, k, v, o, dout, lse, kmask=kmask, scale=scale)
    for got, want in zip(second, ref):
        err = (got.float() - want.float()).abs().max().item()
        assert err <= 1e-2 * (want.float().abs().max().item() + 1e-6), err
    for got, want in zip(second, _fp32_grads(q, k, v, dout, valid, scale)):
        err = (got.float() - want).abs().max().item()
        assert err <= 2e-2 * (want.abs().max().item() + 1e-6), err
    assert _device_error(lib) == 0


def test_noalloc_rejects_oversized_scratch() -> None:
    lib = _lib()
    q = torch.zeros(1, 1, 8, 128, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(1, 1, 8, device="cuda")
    n = ctypes.c_void_p(q.data_ptr())
    status = lib.avgen_attn_bwd_noalloc(n, n, n, n, n, ctypes.c_void_p(lse.data_ptr()), 1 << 21, n, n, n, None, 0, 1,
                                        1, 1, 8, 8, 0.1, None)
    assert status == 2
    assert b"scratch" in lib.avgen_attn_bwd_noalloc_last_error()


def test_noalloc_rejects_a_stream_of_another_device() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lib = _lib()
    q = torch.zeros(1, 1, 8, 128, device="cuda:0", dtype=torch.bfloat16)
    lse = torch.zeros(1, 1, 8, device="cuda:0")
    n = ctypes.c_void_p(q.data_ptr())
    other = torch.cuda.Stream(device=1)
    with torch.cuda.device(0):
        status = lib.avgen_attn_bwd_noalloc(n, n, n, n, n, ctypes.c_void_p(lse.data_ptr()), 8, n, n, n, None, 0, 1, 1,
                                            1, 8, 8, 0.1, ctypes.c_void_p(other.cuda_stream))
    assert status == 1
    assert b"stream" in lib.avgen_attn_bwd_noalloc_last_error()
