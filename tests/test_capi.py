"""The C-ABI library loads, exports every symbol its header declares, and its tile-range
code (the same __host__ __device__ functions the kernels run) equals the restatement of the
reference formulas. No GPU needed: nothing here launches a kernel."""

import ctypes
import os
import re

import pytest

from conftest import REPO
from oracle import tile_ranges as tr

HEADER = os.path.join(REPO, "include", "bd3_attn.h")


def _declared():
    text = open(HEADER).read()
    return re.findall(r"BD3_API\s+[\w\s\*]+?\b(bd3_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = _declared()
    for must in ("bd3_attn_fwd", "bd3_attn_bwd", "bd3_decode_attn", "bd3_decode_live_blocks",
                 "bd3_lse_merge", "bd3_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from bd3attn._lib import LIB, SIGNATURES
    for name in _declared():
        assert hasattr(LIB, name), name
        assert name in SIGNATURES, f"{name} has no ctypes signature"
    assert LIB.bd3_version() >= 100


def _lib_ranges(kind, start, a, b, nq, kv, bs):
    from bd3attn._lib import LIB
    out = (ctypes.c_int32 * 16)()
    cnt = LIB.bd3_debug_ranges(kind, start, a, b, nq, kv, bs, out)
    assert cnt > 0
    return [tuple(out[4 * i:4 * i + 4]) for i in range(cnt)]


def _tiles():
    from bd3attn._lib import LIB
    out = (ctypes.c_int32 * 8)()
    LIB.bd3_debug_tiles(out)
    return list(out[:6])


@pytest.mark.parametrize("n,bs", [(128, 4), (128, 16), (1024, 16), (1024, 4), (512, 64),
                                  (256, 256), (384, 128), (2048, 1024)])
def test_fwd_and_dq_ranges_bit_exact(n, bs):
    bm, bn, _, _, _, dq_bm = _tiles()
    for q0 in range(0, 2 * n, bm):
        assert _lib_ranges(0, q0, bm, bn, n, 0, bs) == tr.fwd_ranges(q0, bm, bn, n, bs)
    for q0 in range(0, 2 * n, dq_bm):
        assert _lib_ranges(0, q0, dq_bm, bn, n, 0, bs) == tr.dq_ranges(q0, dq_bm, bn, n, bs)


@pytest.mark.parametrize("n,bs", [(128, 4), (128, 16), (1024, 16), (1024, 4), (512, 64),
                                  (256, 256), (384, 128)])
def test_dkdv_ranges_bit_exact(n, bs):
    _, _, bkv, bq, _, _ = _tiles()
    for k0 in range(0, 2 * n, bkv):
        assert _lib_ranges(1, k0, bkv, bq, n, 0, bs) == tr.dkdv_ranges(k0, bkv, bq, n, bs)


@pytest.mark.parametrize("q_len,kv_len,bs", [(3088, 3088, 16), (100, 1000, 64), (65, 65, 16),
                                             (200, 4000, 16)])
def test_prefill_ranges_bit_exact(q_len, kv_len, bs):
    bm, bn = _tiles()[:2]
    for q0 in range(0, q_len, bm):
        assert _lib_ranges(2, q0, bm, bn, q_len, kv_len, bs) == \
            tr.decode_ranges(q0, bm, bn, q_len, kv_len, bs)


def test_library_tile_sizes_cover_masks():
    """The tiling the kernels use is one the coverage tests in test_tile_ranges prove."""
    bm, bn, bkv, bq, dec_bn, dq_bm = _tiles()
    assert (bm, bn) in {(128, 64), (128, 128)}
    assert (bkv, bq) in {(128, 32), (128, 64), (128, 128)}
    assert dec_bn == 64 and dq_bm == 128


def _devlen(**over):
    """bd3_decode_attn_devlen with plausible arguments (fake non-null pointers: each case
    below is rejected before the library touches memory or CUDA)."""
    from bd3attn._lib import LIB, i64_array
    a = dict(B=1, H=2, q_len=16, cap=256, kv_len_dev=0x5000, out_dtype=0)
    a.update(over)
    return LIB.bd3_decode_attn_devlen(0x1000, 0x2000, 0x3000, 0x4000, None, a["B"], a["H"],
                                      a["q_len"], a["cap"], 64, i64_array([0] * 12), 16,
                                      a["kv_len_dev"], 1, 0, a["out_dtype"], None, 0, None)


def test_capi_devlen_decode_argument_checks():
    from bd3attn._lib import BD3_ERR_INVALID, BD3_ERR_UNSUPPORTED, LIB
    assert _devlen(kv_len_dev=None) == BD3_ERR_INVALID
    assert "kv_len_dev" in LIB.bd3_last_error().decode()
    assert _devlen(q_len=65) == BD3_ERR_UNSUPPORTED
    assert _devlen(q_len=0) == BD3_ERR_UNSUPPORTED
    assert _devlen(cap=8) == BD3_ERR_INVALID       # capacity below the query block
    assert _devlen(out_dtype=1) == BD3_ERR_INVALID  # bf16 in, fp16 out


def test_wait_self_check_rejects_bad_limits_on_the_host():
    """bd3_debug_wait_timeout validates its arguments before touching the GPU."""
    from bd3attn._lib import BD3_ERR_INVALID, LIB
    assert LIB.bd3_debug_wait_timeout(10, 0, None, None) == BD3_ERR_INVALID
    assert LIB.bd3_debug_wait_timeout(2 * 10 ** 9, 0, None, None) == BD3_ERR_INVALID
    assert b"limit_ns" in LIB.bd3_last_error()
    assert LIB.bd3_debug_wait_timeout(10 ** 6, 0, None, None) == BD3_ERR_INVALID  # no buffer


def _peer_merge(**over):
    """bd3_peer_merge with the given arguments changed; every pointer is a dummy, so only
    calls that fail its host-side checks (made before any CUDA call) may be made here."""
    import ctypes
    from bd3attn._lib import LIB, i64_array
    a = dict(world=2, rank=0, epoch=1, B=1, H=2, rows=16, out_dtype=0)
    a.update(over)
    bufs = (ctypes.c_uint64 * 8)(*([0x10000] * 8))
    return LIB.bd3_peer_merge(0x1000, 0x2000, bufs, a["world"], a["rank"], a["epoch"], 0x3000,
                              None, a["B"], a["H"], a["rows"], i64_array([0] * 3),
                              a["out_dtype"], None)


def test_peer_merge_buffer_size_and_argument_checks():
    """The exchange buffer of the peer-memory merge holds, per parity and sender, every
    (batch, head, row)'s 64 O values and its LSE (rounded up to 16 bytes), then the per-chunk
    flags; sizes and ranks outside the supported range are refused before the GPU is used."""
    from bd3attn._lib import BD3_ERR_INVALID, LIB
    for world, B, H, rows in ((2, 1, 2, 16), (4, 32, 12, 16), (8, 3, 5, 7)):
        region = (B * H * rows * 65 + 3) // 4 * 4
        assert LIB.bd3_peer_merge_buffer_bytes(world, B, H, rows) == \
            2 * world * region * 4 + 2 * 8 * 256 * 8
    for bad in ((1, 1, 2, 16), (9, 1, 2, 16), (2, 0, 2, 16), (2, 1, 2, 0)):
        assert LIB.bd3_peer_merge_buffer_bytes(*bad) == 0
    assert _peer_merge(world=1) == BD3_ERR_INVALID
    assert b"world" in LIB.bd3_last_error()
    assert _peer_merge(world=9) == BD3_ERR_INVALID
    assert _peer_merge(rank=2) == BD3_ERR_INVALID
    assert _peer_merge(rank=-1) == BD3_ERR_INVALID
    assert _peer_merge(B=0) == BD3_ERR_INVALID
    assert _peer_merge(epoch=0) == BD3_ERR_INVALID
    assert b"epoch" in LIB.bd3_last_error()
    assert _peer_merge(out_dtype=5) == BD3_ERR_INVALID


def test_backward_workspace_sizes():
    """The backward's workspace: per query row Delta and LSE*log2(e) (fp32), then the dQ
    accumulator: 64 fp32 values, or 64 int64 fixed-point values for the deterministic
    variant. Non-positive sizes give 0."""
    from bd3attn._lib import LIB
    for B, H, n in ((1, 1, 128), (8, 12, 1024), (2, 3, 256)):
        rows = B * H * 2 * n
        assert LIB.bd3_attn_bwd_workspace_size(B, H, n, 64) == rows * (2 + 64) * 4
        assert LIB.bd3_attn_bwd_det_workspace_size(B, H, n, 64) == rows * (2 * 4 + 64 * 8)
    for bad in ((0, 1, 128), (1, 0, 128), (1, 1, 0)):
        assert LIB.bd3_attn_bwd_workspace_size(*bad, 64) == 0
        assert LIB.bd3_attn_bwd_det_workspace_size(*bad, 64) == 0
