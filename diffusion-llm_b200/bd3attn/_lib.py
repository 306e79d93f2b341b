"""ctypes binding of libbd3attn.so (the C ABI declared in include/bd3_attn.h).

The shared library is built in-tree (``diffusion-llm_b200/lib/libbd3attn.so``) by
``diffusion-llm_b200/build.py``. There is no fallback: if the library is missing or does
not load, importing this module raises.
"""

from __future__ import annotations

import ctypes
import os

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_ROOT, "lib", "libbd3attn.so")

BD3_OK, BD3_ERR_INVALID, BD3_ERR_UNSUPPORTED, BD3_ERR_CUDA, BD3_ERR_WORKSPACE = range(5)
BD3_BF16, BD3_F16, BD3_F32 = 0, 1, 2

# every symbol include/bd3_attn.h declares, with (restype, argtypes)
_i64, _i32, _vp, _sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
_pi64 = ctypes.POINTER(ctypes.c_int64)
_pi32 = ctypes.POINTER(ctypes.c_int32)
_psz = ctypes.POINTER(ctypes.c_size_t)

SIGNATURES = {
    "bd3_version": (_i32, []),
    "bd3_last_error": (ctypes.c_char_p, []),
    "bd3_device_status": (_i32, [_i32]),
    "bd3_attn_fwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _pi64, _i64, _i32,
                            _vp]),
    "bd3_attn_bwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "bd3_attn_bwd_det_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "bd3_attn_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                            _pi64, _i64, _i32, _vp, _sz, _vp]),
    "bd3_attn_bwd_det": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                            _pi64, _i64, _i32, _vp, _sz, _vp]),
    "bd3_peer_merge_buffer_bytes": (_sz, [_i32, _i64, _i64, _i64]),
    "bd3_peer_merge": (_i32, [_vp, _vp, ctypes.POINTER(ctypes.c_uint64), _i32, _i32,
                              ctypes.c_uint64, _vp, _vp, _i64, _i64, _i64, _pi64, _i32, _vp]),
    "bd3_decode_plan": (_i32, [_i64, _i64, _i64, _i64, _i64, _i64, _i64, _pi64, _psz]),
    "bd3_decode_attn": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _pi64,
                               _i64, _i64, _i64, _i64, _i32, _i32, _vp, _sz, _vp]),
    "bd3_decode_attn_devlen": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                      _pi64, _i64, _vp, _i64, _i32, _i32, _vp, _sz, _vp]),
    "bd3_decode_attn_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                       _pi64, _i64, _i64, _i64, _i32, _i32, _vp]),
    "bd3_decode_live_plan": (_i32, [_i64, _i64, _i64, _i64, _i64, _pi64, _psz]),
    "bd3_decode_live_blocks": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _i64, _i64, _pi64, _i64, _i64, _i32, _i32, _vp,
                                      _sz, _vp]),
    "bd3_lse_merge": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                             _i64, _pi64, _i32, _vp]),
    "bd3_qkv_rope_cache": (_i32, [_vp, _pi64, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64,
                                  _vp, _vp, _vp, _pi64, _i64, _i64, _i32, _vp]),
    "bd3_f32_to_f16_scaled": (_i32, [_vp, _vp, _vp, _pi64, _i64, _i64, _i64, _i64, _i64, _vp,
                                     _vp, _vp, _vp, _vp, _vp]),
    "bd3_subs_sample": (_i32, [_vp, _pi64, _i64, _i64, _i64, _vp, _i64, ctypes.c_double,
                               ctypes.c_double, ctypes.c_uint64, ctypes.c_uint64, _vp, _vp, _i32,
                               _vp]),
    "bd3_subs_sample_dev": (_i32, [_vp, _pi64, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _i32,
                                   _vp]),
    "bd3_profile_enable": (_i32, [_i32]),
    "bd3_profile_collect": (_i32, [ctypes.POINTER(ctypes.c_double), _pi32]),
    "bd3_debug_ranges": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _i64, _pi32]),
    "bd3_debug_tiles": (_i32, [_pi32]),
    "bd3_debug_wait_timeout": (_i32, [_i64, _i32, _vp, _vp]),
    "bd3_debug_wait_site": (_i32, [ctypes.POINTER(ctypes.c_uint32)]),
}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library first "
            "(python diffusion-llm_b200/build.py, or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


class BD3Error(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def check(fn: str, rc: int) -> None:
    if rc != BD3_OK:
        msg = LIB.bd3_last_error().decode(errors="replace")
        raise BD3Error(fn, rc, msg)


def i64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int64 * len(vals))(*vals)
