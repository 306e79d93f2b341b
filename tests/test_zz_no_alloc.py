"""The no-allocation decode entry point (bd3_decode_attn_noalloc) against the regular one.

Callers such as a serving engine whose allocator owns all device memory cannot hand the
library a workspace from cudaMalloc; this entry point keeps the split-KV partials in a fixed
array inside the library instead. Its output must match bd3_decode_attn's, called through the
C ABI on the same inputs, on two calls in a row (the second reuses the array the first left
behind). This file is named to be collected last.
"""

import ctypes

import pytest
import torch

from gpu_util import O_TOL, LSE_TOL, assert_close, assert_device_ok

pytestmark = pytest.mark.gpu


def _inputs(seed, B, H, q_len, kv_len):
    """Seeded inputs drawn on the GPU (the test compares two entry points, no CPU oracle)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda s: torch.randn(B, H, s, 64, device="cuda", generator=g).bfloat16()  # noqa: E731
    return mk(q_len), mk(kv_len), mk(kv_len)


def _strides(*ts):
    vals = []
    for t in ts:
        vals += [t.stride(0), t.stride(1), t.stride(2)]
    return (ctypes.c_int64 * len(vals))(*vals)


def _regular(lib, q, k, v, bs):
    B, H, q_len, D = q.shape
    kv_len = k.shape[2]
    ns, wb = ctypes.c_int64(0), ctypes.c_size_t(0)
    assert lib.bd3_decode_plan(B, H, q_len, kv_len, bs, -1, 0, ctypes.byref(ns),
                               ctypes.byref(wb)) == 0
    o = torch.empty_like(q)
    lse = torch.empty(B, H, q_len, device="cuda", dtype=torch.float32)
    ws = torch.empty(max(wb.value, 16), dtype=torch.uint8, device="cuda")
    rc = lib.bd3_decode_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                             lse.data_ptr(), B, H, q_len, kv_len, 64, _strides(q, k, v, o), bs,
                             -1, 0, ns.value, 0, 0, ws.data_ptr(), ws.numel(),
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.bd3_last_error()
    return o, lse, ns.value


def _noalloc(lib, q, k, v, bs, o=None, lse=None):
    B, H, q_len, D = q.shape
    kv_len = k.shape[2]
    o = torch.empty_like(q) if o is None else o
    lse = torch.empty(B, H, q_len, device="cuda", dtype=torch.float32) if lse is None else lse
    rc = lib.bd3_decode_attn_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                     lse.data_ptr(), B, H, q_len, kv_len, 64,
                                     _strides(q, k, v, o), bs, -1, 0, 0, 0,
                                     torch.cuda.current_stream().cuda_stream)
    return rc, o, lse


SCRATCH_BYTES = 32 << 20  # the library's fixed no-alloc scratch


@pytest.mark.parametrize("B,H,q_len,kv_len", [(2, 12, 16, 4112), (16, 12, 16, 65552),
                                              (1, 12, 16, 1040), (3, 2, 40, 700)])
def test_noalloc_matches_regular_twice(B, H, q_len, kv_len):
    from bd3attn._lib import LIB
    bs = 16
    q, k, v = _inputs(40 + B, B, H, q_len, kv_len)
    ref_o, ref_lse, n_splits = _regular(LIB, q, k, v, bs)
    assert n_splits > 1 or kv_len <= 1040  # the big shapes exercise the scratch array
    assert B * H * n_splits * q_len * 65 * 4 <= SCRATCH_BYTES  # the case fits the array
    for _ in range(2):  # two calls in a row: the second runs on what the first left behind
        rc, o, lse = _noalloc(LIB, q, k, v, bs)
        assert rc == 0, LIB.bd3_last_error()
        torch.cuda.synchronize()
        assert_device_ok()
        assert_close("O", o, ref_o, O_TOL)
        assert_close("LSE", lse, ref_lse, LSE_TOL)
    # the other inputs in between must not leak into the next call
    q2, k2, v2 = _inputs(77, B, H, q_len, kv_len)
    _noalloc(LIB, q2, k2, v2, bs)
    rc, o, lse = _noalloc(LIB, q, k, v, bs)
    assert rc == 0
    torch.cuda.synchronize()
    assert_close("O after other inputs", o, ref_o, O_TOL)


def test_noalloc_uses_fewer_splits_beyond_its_scratch():
    """A shape whose planned partials need more than the fixed array (64 queries x 384 heads
    over a 64K cache, about 100 MB at the planned split count) runs with fewer splits and
    gives the regular entry point's result."""
    from bd3attn._lib import LIB
    B, H, q_len, kv_len, bs = 32, 12, 64, 65536, 16
    q, k, v = _inputs(5, B, H, q_len, kv_len)
    need = ctypes.c_size_t(0)
    n_splits = ctypes.c_int64(0)
    assert LIB.bd3_decode_plan(B, H, q_len, kv_len, bs, -1, 0, ctypes.byref(n_splits),
                               ctypes.byref(need)) == 0
    assert need.value > 32 << 20  # the case this test is about
    rc, o, lse = _noalloc(LIB, q, k, v, bs)
    assert rc == 0, LIB.bd3_last_error().decode()
    ref_o, ref_lse, _ = _regular(LIB, q, k, v, bs)
    torch.cuda.synchronize()
    assert_close("O", o, ref_o, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)
    assert_device_ok()
