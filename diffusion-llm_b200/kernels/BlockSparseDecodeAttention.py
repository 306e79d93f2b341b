"""Block-sparse (block-causal) decode attention for BD3-LM sampling, on B200.

Drop-in for kernels/BlockSparseDecodeAttention.py of the reference:
``block_sparse_decode_attention(q, k, v, block_size)`` (:118-148) — the last q_len
positions attend all kv_len keys under the block-causal rule, keys past the last query's
block skipped — and the helper ``_last_stride_1`` (:113-115). Query blocks of up to 64 rows
run the memory-bound decode kernel of csrc/decode.cuh; longer ones (prefill, the uncached
sampler) run the tcgen05 kernel of csrc/attn_fwd.cuh in its block-causal mode.

Added here (no counterpart in the reference): ``block_sparse_live_decode_attention`` reads
only the KV blocks listed live for each (batch, head).
"""

import torch
from torch import Tensor

from bd3attn import ops


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
    out_dtype = q.dtype
    cdt = _cdt(q, k, v)
    q, k, v = _last_stride_1(q.to(cdt)), _last_stride_1(k.to(cdt)), _last_stride_1(v.to(cdt))
    if torch.compiler.is_compiling():
        o = torch.ops.bd3.decode(q, k, v, int(block_size))
    else:
        o = ops.decode_raw(q, k, v, int(block_size))
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
