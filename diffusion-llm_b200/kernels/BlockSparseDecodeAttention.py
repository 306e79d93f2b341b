"""Block-sparse (block-causal) decode attention for BD3-LM sampling, on B200.

Drop-in for kernels/BlockSparseDecodeAttention.py of the reference:
``block_sparse_decode_attention(q, k, v, block_size)`` (:118-148) — the last q_len
positions attend all kv_len keys under the block-causal rule, keys past the last query's
block skipped — and the helper ``_last_stride_1`` (:113-115). Query blocks of up to 64 rows
run the memory-bound decode kernel of csrc/decode.cuh; longer ones (prefill, the uncached
sampler) run the tcgen05 kernel of csrc/attn_fwd.cuh in its block-causal mode.

Added here (no counterpart in the reference): ``block_sparse_live_decode_attention`` reads
only the KV blocks listed live for each (batch, head).

fp32 inputs run on the fp16 kernels at tf32's operand precision (kernels/_precision.py), and
the output comes back as fp32.
"""

import torch
from torch import Tensor

from bd3attn import ops
from kernels import _precision


def _last_stride_1(x: Tensor) -> Tensor:
    # the kernels read rows with TMA: contiguous rows; other strides are fine
    return x if x.stride(-1) == 1 else x.contiguous()


def _cdt(q: Tensor, k: Tensor, v: Tensor) -> torch.dtype:
    dts = {q.dtype, k.dtype, v.dtype}
    return torch.float16 if dts <= {torch.float16} else torch.bfloat16


def block_sparse_decode_attention(
    q: Tensor,  # (batch, heads, q_len, head_dim): the last q_len positions
    k: Tensor,  # (batch, heads, kv_len, head_dim)
    v: Tensor,
    block_size: int,
) -> Tensor:
    """Block-causal attention of the last q_len positions over all kv_len keys."""
    B, H, q_len, D = q.shape
    kv_len = k.shape[2]
    assert q_len <= kv_len, "queries are the last q_len key positions"
    return _decode(q, k, v, block_size)


def _decode(q: Tensor, k: Tensor, v: Tensor, block_size: int) -> Tensor:
    """The library's block-causal decode (split-KV for q_len <= 64, the tcgen05 prefill
    kernel above), on 16-bit operands; fp32 inputs through the exact power-of-two scaling."""
    out_dtype = q.dtype
    if q.dtype == k.dtype == v.dtype == torch.float32:
        q, k, v, _, c = _precision.qkv_to_f16(q, k, v)
        # decode blocks return fp32 directly; prefill writes the operand dtype
        odt = torch.float32 if q.shape[2] <= 64 else torch.float16
    else:
        cdt = _cdt(q, k, v)
        q, k, v, c, odt = q.to(cdt), k.to(cdt), v.to(cdt), None, None
    # forward only, as the reference's decode kernels: the output carries no autograd
    # history (detached inputs keep torch.compile from asking for a backward formula)
    q, k, v = _last_stride_1(q.detach()), _last_stride_1(k.detach()), _last_stride_1(v.detach())
    if torch.compiler.is_compiling():
        o = torch.ops.bd3.decode(q, k, v, int(block_size))
        if c is not None:
            return _precision.scaled_back(o, c)
    else:
        o = ops.decode_raw(q, k, v, int(block_size), out_dtype=odt)
        if c is not None:
            return _precision.scaled_back(o, c)
    return o if o.dtype == out_dtype else o.to(out_dtype)


def block_sparse_live_decode_attention(
    q: Tensor,         # (batch, heads, q_len <= 64, head_dim)
    k: Tensor,         # (batch, heads, kv_len, head_dim)
    v: Tensor,
    live_idx: Tensor,  # (batch, heads, max_live) int32, ascending block indices
    live_cnt: Tensor,  # (batch, heads) int32, live blocks per (batch, head)
    kv_block: int,     # tokens per KV block (a multiple of 64)
    block_size: int,
) -> Tensor:
    """Decode attention restricted to the live KV blocks of each (batch, head); the
    block-causal rule still applies inside them."""
    out_dtype = q.dtype
    cdt = _cdt(q, k, v)
    o = ops.live_decode_raw(q.to(cdt), k.to(cdt), v.to(cdt), live_idx, live_cnt,
                            int(kv_block), int(block_size))
    return o if o.dtype == out_dtype else o.to(out_dtype)
