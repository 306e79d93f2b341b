"""Tensor-level wrappers over the C ABI (one call per entry point of include/bd3_attn.h).

Every function takes CUDA tensors, allocates its outputs (and workspace) with the caching
allocator, and enqueues the kernels on the current CUDA stream of the inputs' device.
They are also registered as ``torch.ops.bd3.*`` custom ops with fake (meta) implementations
so that ``torch.compile`` can trace callers without graph breaks.
"""

from __future__ import annotations

import ctypes

import torch

from bd3attn._lib import (BD3_BF16, BD3_F16, BD3_F32, LIB, check, i64_array)

_DTYPE_CODE = {torch.bfloat16: BD3_BF16, torch.float16: BD3_F16, torch.float32: BD3_F32}


def _code(dtype: torch.dtype) -> int:
    if dtype not in _DTYPE_CODE:
        raise TypeError(f"unsupported dtype {dtype}")
    return _DTYPE_CODE[dtype]


def _rows_contig(x: torch.Tensor) -> torch.Tensor:
    """The kernels read rows with TMA: the last dim must be contiguous and the other
    strides 16-byte multiples; other layouts are copied (as the reference's
    _last_stride_1 / .contiguous() do)."""
    if x.stride(-1) != 1 or any((s * x.element_size()) % 16 for s in x.stride()[:-1]) \
            or x.data_ptr() % 16:
        return x.contiguous()
    return x


def _s3(x: torch.Tensor):
    return (x.stride(0), x.stride(1), x.stride(2))


def _stream(x: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)


def _ptr(x):
    return ctypes.c_void_p(x.data_ptr()) if x is not None else ctypes.c_void_p(0)


def _check_cuda(*xs):
    for x in xs:
        if not x.is_cuda:
            raise AssertionError("inputs must be on CUDA")


# ---------------------------------------------------------------------------------------
def attn_fwd_raw(q, k, v, block_size: int):
    """(O, LSE) of BD3-LM training attention; q, k, v: (B, H, 2n, 64) bf16/f16."""
    _check_cuda(q, k, v)
    q, k, v = _rows_contig(q), _rows_contig(k), _rows_contig(v)
    B, H, S, D = q.shape
    o = torch.empty((B, H, S, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, H, S), dtype=torch.float32, device=q.device)
    strides = i64_array(_s3(q) + _s3(k) + _s3(v) + _s3(o))
    with torch.cuda.device(q.device):
        check("bd3_attn_fwd", LIB.bd3_attn_fwd(
            _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, H, S // 2, D, strides,
            int(block_size), _code(q.dtype), _stream(q)))
    return o, lse


def attn_bwd_raw(q, k, v, o, lse, do, block_size: int, deterministic: bool = False):
    """(dQ, dK, dV) of BD3-LM training attention. deterministic: dQ's partials are added as
    64-bit fixed-point integers (bd3_attn_bwd_det), so dQ is the same on every run; otherwise
    they are added in fp32 in the order the key tiles finish."""
    _check_cuda(q, k, v, o, lse, do)
    q, k, v, o, do = (_rows_contig(t) for t in (q, k, v, o, do))
    B, H, S, D = q.shape
    dq = torch.empty((B, H, S, D), dtype=q.dtype, device=q.device)
    dk = torch.empty_like(dq)
    dv = torch.empty_like(dq)
    size_fn, fn, name = ((LIB.bd3_attn_bwd_det_workspace_size, LIB.bd3_attn_bwd_det,
                          "bd3_attn_bwd_det") if deterministic else
                         (LIB.bd3_attn_bwd_workspace_size, LIB.bd3_attn_bwd, "bd3_attn_bwd"))
    ws_bytes = size_fn(B, H, S // 2, D)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
    lse = lse.contiguous()
    strides = i64_array(_s3(q) + _s3(k) + _s3(v) + _s3(o) + _s3(do) + _s3(dq) + _s3(dk)
                        + _s3(dv))
    with torch.cuda.device(q.device):
        check(name, fn(
            _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), _ptr(do), _ptr(dq), _ptr(dk),
            _ptr(dv), B, H, S // 2, D, strides, int(block_size), _code(q.dtype), _ptr(ws),
            ws.numel(), _stream(q)))
    return dq, dk, dv


def f32_to_f16_scaled_raw(q, k, v):
    """fp32 q, k, v (B, H, rows, 64) as fp16 at tf32's significand (bd3_f32_to_f16_scaled):
    returns (q * 2^-a, k * 2^a, v * 2^-c in fp16, exps) with exps = (a, c, 2^c) fp32 on the
    device. q may have another row count than k and v."""
    _check_cuda(q, k, v)
    q, k, v = (x if x.stride(-1) == 1 and x.data_ptr() % 16 == 0
               and all(st % 4 == 0 for st in x.stride()[:-1]) else x.contiguous()
               for x in (q, k, v))
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    if k.shape != v.shape or k.shape[:2] != q.shape[:2] or k.shape[3] != D:
        raise AssertionError("q, k, v must be (B, H, rows, head_dim) with k, v alike")
    q16 = torch.empty((B, H, Sq, D), dtype=torch.float16, device=q.device)
    k16 = torch.empty((B, H, Skv, D), dtype=torch.float16, device=q.device)
    v16 = torch.empty_like(k16)
    exps = torch.empty(3, dtype=torch.float32, device=q.device)
    ws = torch.empty(4, dtype=torch.int32, device=q.device)
    strides = i64_array(_s3(q) + _s3(k) + _s3(v))
    with torch.cuda.device(q.device):
        check("bd3_f32_to_f16_scaled", LIB.bd3_f32_to_f16_scaled(
            _ptr(q), _ptr(k), _ptr(v), strides, B, H, Sq, Skv, D, _ptr(q16), _ptr(k16),
            _ptr(v16), _ptr(exps), _ptr(ws), _stream(q)))
    return q16, k16, v16, exps


@torch.library.custom_op("bd3::f32_to_f16_scaled", mutates_args=())
def f32_to_f16_scaled_op(q: torch.Tensor, k: torch.Tensor,
                         v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                   torch.Tensor]:
    return f32_to_f16_scaled_raw(q, k, v)


@f32_to_f16_scaled_op.register_fake
def _(q, k, v):
    return (q.new_empty(tuple(q.shape), dtype=torch.float16),
            k.new_empty(tuple(k.shape), dtype=torch.float16),
            v.new_empty(tuple(v.shape), dtype=torch.float16),
            q.new_empty((3,), dtype=torch.float32))


def decode_plan(B, H, q_len, kv_len, block_size, q_pos0=-1, kv_pos0=0):
    ns = ctypes.c_int64(0)
    wb = ctypes.c_size_t(0)
    check("bd3_decode_plan", LIB.bd3_decode_plan(B, H, q_len, kv_len, block_size, q_pos0,
                                                 kv_pos0, ctypes.byref(ns), ctypes.byref(wb)))
    return ns.value, wb.value


def decode_raw(q, k, v, block_size: int, q_pos0: int = -1, kv_pos0: int = 0,
               out_dtype=None, return_lse: bool = False, n_splits: int | None = None,
               kv_len_dev=None):
    """Block-causal decode attention of the q_len queries over kv_len keys.

    kv_len_dev: an int32 device tensor of one element holding the key count; k and v are then
    the whole cache storage (B, H, capacity, 64), the queries sit at the count's end and
    q_pos0 / kv_pos0 / n_splits are ignored. The launch does not depend on the count, so a
    CUDA graph captured around it replays every step of a growing cache.
    """
    _check_cuda(q, k, v)
    q, k, v = _rows_contig(q), _rows_contig(k), _rows_contig(v)
    B, H, q_len, D = q.shape
    kv_len = k.shape[2]
    out_dtype = q.dtype if out_dtype is None else out_dtype
    if kv_len_dev is not None:
        return _decode_devlen(q, k, v, int(block_size), kv_len_dev, out_dtype, return_lse)
    ns, wb = decode_plan(B, H, q_len, kv_len, int(block_size), q_pos0, kv_pos0)
    if n_splits is not None and q_len <= 64:
        ns = int(n_splits)
        wb = B * H * ns * q_len * 65 * 4 if ns > 1 else 0
    o = torch.empty((B, H, q_len, D), dtype=out_dtype, device=q.device)
    lse = torch.empty((B, H, q_len), dtype=torch.float32, device=q.device) if return_lse else None
    ws = torch.empty(max(wb, 16), dtype=torch.uint8, device=q.device)
    strides = i64_array(_s3(q) + _s3(k) + _s3(v) + _s3(o))
    with torch.cuda.device(q.device):
        check("bd3_decode_attn", LIB.bd3_decode_attn(
            _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, H, q_len, kv_len, D, strides,
            int(block_size), int(q_pos0), int(kv_pos0), ns, _code(q.dtype), _code(out_dtype),
            _ptr(ws), wb, _stream(q)))
    return (o, lse) if return_lse else o


def _decode_devlen(q, k, v, block_size, kv_len_dev, out_dtype, return_lse):
    _check_cuda(kv_len_dev)
    if kv_len_dev.dtype != torch.int32 or kv_len_dev.numel() != 1:
        raise AssertionError("kv_len_dev must be a one-element int32 device tensor")
    B, H, q_len, D = q.shape
    capacity = k.shape[2]
    ns, wb = decode_plan(B, H, q_len, capacity, block_size, -1, 0)
    o = torch.empty((B, H, q_len, D), dtype=out_dtype, device=q.device)
    lse = torch.empty((B, H, q_len), dtype=torch.float32, device=q.device) if return_lse else None
    ws = torch.empty(max(wb, 16), dtype=torch.uint8, device=q.device)
    strides = i64_array(_s3(q) + _s3(k) + _s3(v) + _s3(o))
    with torch.cuda.device(q.device):
        check("bd3_decode_attn_devlen", LIB.bd3_decode_attn_devlen(
            _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, H, q_len, capacity, D, strides,
            block_size, _ptr(kv_len_dev), ns, _code(q.dtype), _code(out_dtype), _ptr(ws), wb,
            _stream(q)))
    return (o, lse) if return_lse else o


def live_decode_raw(q, k, v, live_idx, live_cnt, kv_block: int, block_size: int,
                    out_dtype=None, return_lse: bool = False, n_splits: int | None = None):
    """Decode over a per-(batch, head) list of live KV blocks.

    live_idx: (B, H, max_live) int32 ascending block indices (entries past live_cnt ignored);
    live_cnt: (B, H) int32.
    n_splits: None takes the planned split count; k >= 1 splits every (batch, head)'s list
    over k CTAs (k > 1 merges their partials with the combine kernel).
    """
    _check_cuda(q, k, v, live_idx, live_cnt)
    q, k, v = _rows_contig(q), _rows_contig(k), _rows_contig(v)
    B, H, q_len, D = q.shape
    kv_len = k.shape[2]
    out_dtype = q.dtype if out_dtype is None else out_dtype
    live_idx = live_idx.to(torch.int32).contiguous()
    live_cnt = live_cnt.to(torch.int32).contiguous()
    max_live = live_idx.shape[-1]
    ns = ctypes.c_int64(0)
    wb = ctypes.c_size_t(0)
    check("bd3_decode_live_plan", LIB.bd3_decode_live_plan(
        B, H, q_len, max_live, int(kv_block), ctypes.byref(ns), ctypes.byref(wb)))
    if n_splits is not None:
        if n_splits < 1:
            raise ValueError("n_splits must be >= 1")
        ns.value = int(n_splits)
        wb.value = B * H * n_splits * q_len * 65 * 4 if n_splits > 1 else 0
    o = torch.empty((B, H, q_len, D), dtype=out_dtype, device=q.device)
    lse = torch.empty((B, H, q_len), dtype=torch.float32, device=q.device) if return_lse else None
    ws = torch.empty(max(wb.value, 16), dtype=torch.uint8, device=q.device)
    strides = i64_array(_s3(q) + _s3(k) + _s3(v) + _s3(o))
    with torch.cuda.device(q.device):
        check("bd3_decode_live_blocks", LIB.bd3_decode_live_blocks(
            _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), _ptr(live_idx), _ptr(live_cnt),
            max_live, max_live, int(kv_block), B, H, q_len, kv_len, D, strides, int(block_size),
            ns.value, _code(q.dtype), _code(out_dtype), _ptr(ws), wb.value, _stream(q)))
    return (o, lse) if return_lse else o


def lse_merge_raw(parts, lses, out_dtype=torch.bfloat16):
    """Merge G partials: parts (G, B, H, rows, 64) fp32, lses (G, B, H, rows) fp32 ->
    (O (B, H, rows, 64) in out_dtype, LSE (B, H, rows) fp32)."""
    _check_cuda(parts, lses)
    parts = parts.contiguous()
    lses = lses.contiguous()
    G, B, H, rows, D = parts.shape
    o = torch.empty((B, H, rows, D), dtype=out_dtype, device=parts.device)
    lse = torch.empty((B, H, rows), dtype=torch.float32, device=parts.device)
    with torch.cuda.device(parts.device):
        check("bd3_lse_merge", LIB.bd3_lse_merge(
            _ptr(parts), _ptr(lses), _ptr(o), _ptr(lse), B, H, G, rows, D, B * H * rows * D,
            rows * D, B * H * rows, rows, i64_array(_s3(o)), _code(out_dtype), _stream(parts)))
    return o, lse


def debug_wait_timeout(limit_ns: int, arrive: bool = False, device=None) -> tuple[int, int]:
    """Run the bounded-wait self-check (bd3_debug_wait_timeout) on the current stream and
    return (1 if the wait gave up else 0, the wait's duration in ns). Synchronises."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    out = torch.zeros(2, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        check("bd3_debug_wait_timeout", LIB.bd3_debug_wait_timeout(
            int(limit_ns), 1 if arrive else 0, _ptr(out),
            ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
    res = out.cpu()
    return int(res[0]), int(res[1])


def debug_wait_site() -> dict | None:
    """Where the first bounded wait that ran out gave up since the last read (block, thread,
    barrier shared-memory address, awaited parity), or None; reading clears it."""
    out = (ctypes.c_uint32 * 4)()
    check("bd3_debug_wait_site", LIB.bd3_debug_wait_site(out))
    if not out[0]:
        return None
    return {"block": out[1], "thread": out[2], "smem_addr": out[3] & 0x7FFFFFFF,
            "parity": out[3] >> 31}


def device_status(clear: bool = True) -> int:
    """Sticky device-side error bits (1: a bounded wait ran out; 2: a kernel rejected its
    launch; 4: a RoPE position was outside the table). Synchronises."""
    return int(LIB.bd3_device_status(1 if clear else 0))


# ---------------------------------------------------------------------------------------
# torch.library registrations (used under torch.compile; eager callers use the raw calls)
@torch.library.custom_op("bd3::attn_fwd", mutates_args=())
def attn_fwd_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    return attn_fwd_raw(q, k, v, block_size)


@attn_fwd_op.register_fake
def _(q, k, v, block_size):
    B, H, S, D = q.shape
    return q.new_empty((B, H, S, D)), q.new_empty((B, H, S), dtype=torch.float32)


@torch.library.custom_op("bd3::attn_bwd", mutates_args=())
def attn_bwd_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
                lse: torch.Tensor, do: torch.Tensor, block_size: int,
                deterministic: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return attn_bwd_raw(q, k, v, o, lse, do, block_size, deterministic)


@attn_bwd_op.register_fake
def _(q, k, v, o, lse, do, block_size, deterministic):
    shape = tuple(q.shape)
    return q.new_empty(shape), q.new_empty(shape), q.new_empty(shape)


@torch.library.custom_op("bd3::decode", mutates_args=())
def decode_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
              block_size: int) -> torch.Tensor:
    return decode_raw(q, k, v, block_size)


@decode_op.register_fake
def _(q, k, v, block_size):
    return q.new_empty(tuple(q.shape))


def qkv_rope_cache_raw(qkv, n_heads: int, cos_table, sin_table, k_cache, v_cache, row0: int,
                       positions=None, pos0: int = 0, q_out=None):
    """Split a fused QKV projection, rotate q and k (the reference's RoPE), write k and v to
    rows [row0, row0 + seq) of the caches in place and q to q_out; returns q_out.

    qkv: (B, S, 3 * n_heads * D) with its last dim ordered (three, heads, head_dim);
    cos_table, sin_table: (max_pos, D / 2) fp32 (RoPE's buffers); k_cache, v_cache:
    (B, n_heads, rows, D) in qkv's dtype; positions: (S,) int64 absolute positions on the
    device, or None for pos0, pos0 + 1, ...; q_out: (B, n_heads, S, D) or None to allocate.
    row0 < 0 takes the first cache row from the device value positions[0] (positions
    required), so a captured CUDA graph writes each new block at its own rows.
    """
    _check_cuda(qkv, cos_table, sin_table, k_cache, v_cache)
    if qkv.dim() != 3:
        raise AssertionError("qkv must be (batch, seq, 3 * n_heads * head_dim)")
    B, S, F = qkv.shape
    if F % (3 * n_heads):
        raise AssertionError("qkv's last dim must be 3 * n_heads * head_dim")
    D = F // (3 * n_heads)
    if qkv.stride(-1) != 1:
        qkv = qkv.contiguous()
    if q_out is None:
        q_out = torch.empty((B, n_heads, S, D), dtype=qkv.dtype, device=qkv.device)
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache), ("q_out", q_out)):
        if t.dtype != qkv.dtype or t.stride(-1) != 1 or t.shape[0] != B or t.shape[1] != n_heads \
                or t.shape[-1] != D:
            raise AssertionError(f"{name} must be (B, n_heads, rows, head_dim) in qkv's dtype")
    if k_cache.shape[2] != v_cache.shape[2]:
        raise AssertionError("k_cache and v_cache must have the same rows")
    cos_table = cos_table.float().contiguous()
    sin_table = sin_table.float().contiguous()
    if positions is not None:
        positions = positions.to(device=qkv.device, dtype=torch.int64).contiguous()
        if positions.numel() != S:
            raise AssertionError("positions must have one entry per token")
    strides = i64_array(_s3(q_out) + _s3(k_cache) + _s3(v_cache))
    with torch.cuda.device(qkv.device):
        check("bd3_qkv_rope_cache", LIB.bd3_qkv_rope_cache(
            _ptr(qkv), i64_array((qkv.stride(0), qkv.stride(1))), B, S, n_heads, D,
            _ptr(positions), int(pos0), _ptr(cos_table), _ptr(sin_table), cos_table.shape[0],
            _ptr(q_out), _ptr(k_cache), _ptr(v_cache), strides, int(row0), k_cache.shape[2],
            _code(qkv.dtype), _stream(qkv)))
    return q_out


@torch.library.custom_op("bd3::qkv_rope_cache", mutates_args=("k_cache", "v_cache"))
def qkv_rope_cache_op(qkv: torch.Tensor, n_heads: int, cos_table: torch.Tensor,
                      sin_table: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      row0: int, positions: torch.Tensor | None = None) -> torch.Tensor:
    """qkv_rope_cache_raw as a custom op: writes the caches in place, returns q."""
    return qkv_rope_cache_raw(qkv, n_heads, cos_table, sin_table, k_cache, v_cache, row0,
                              positions=positions)


@qkv_rope_cache_op.register_fake
def _(qkv, n_heads, cos_table, sin_table, k_cache, v_cache, row0, positions=None):
    B, S, F = qkv.shape
    return qkv.new_empty((B, n_heads, S, F // (3 * n_heads)))


# ---------------------------------------------------------------------------------------
PROFILE_KERNELS = ("attn_fwd", "attn_prefill", "bwd_prep", "bwd_dq_convert", "bwd_fused",
                   "decode", "decode_combine", "qkv_rope_cache", "subs_sample")


def profile_enable(on: bool = True) -> None:
    """Bracket every library launch with CUDA events on its own stream (see
    bd3_profile_enable)."""
    check("bd3_profile_enable", LIB.bd3_profile_enable(1 if on else 0))


def profile_collect() -> dict:
    """{kernel name: (total ms, launches)} for the launches since the last collect."""
    ms = (ctypes.c_double * 16)()
    cnt = (ctypes.c_int32 * 16)()
    n = LIB.bd3_profile_collect(ms, cnt)
    if n < 0:
        check("bd3_profile_collect", -n)
    return {PROFILE_KERNELS[i]: (ms[i], cnt[i]) for i in range(len(PROFILE_KERNELS)) if cnt[i]}
