"""The allocation-free attention-backward C entry point (``avgen_attn_bwd_noalloc``).

Called through the exported C symbol with ctypes, twice in a row, and checked
against the Python entry point ``avgen_b200.ops.kernels.attention_bwd``.
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
    return lib


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
    from avgen_b200.ops._ext import check_errors

    lib = _lib()
    torch.manual_seed(21)
    b, h, hk, lq, lk, d = 2, 4, 2, 390, 301, 128
    q = torch.randn(b, h, lq, d, device="cuda").bfloat16()
    k = torch.randn(b, hk, lk, d, device="cuda").bfloat16()
    v = torch.randn(b, hk, lk, d, device="cuda").bfloat16()
    kmask = None
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
    assert check_errors() == 0


def test_noalloc_rejects_oversized_scratch() -> None:
    lib = _lib()
    q = torch.zeros(1, 1, 8, 128, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(1, 1, 8, device="cuda")
    n = ctypes.c_void_p(q.data_ptr())
    status = lib.avgen_attn_bwd_noalloc(n, n, n, n, n, ctypes.c_void_p(lse.data_ptr()), 1 << 21, n, n, n, None, 0, 1,
                                        1, 1, 8, 8, 0.1, None)
    assert status == 2
    assert b"scratch" in lib.avgen_attn_bwd_noalloc_last_error()
