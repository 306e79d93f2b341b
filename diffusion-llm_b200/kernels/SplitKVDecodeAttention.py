"""Split-KV (FlashDecoding) attention for BD3-LM cached sampling, on B200.

Drop-in for kernels/SplitKVDecodeAttention.py of the reference:
``split_kv_decode_attention(q, k, v, block_size)`` (:130-171), same result as
block_sparse_decode_attention with the keys split across CTAs so a decode step fills the
GPU, and the reference's prefill hand-off for q_len > 64 (:140-142). The split size is chosen
per shape by the library's planner (bd3_decode_plan) instead of the fixed SPLIT_N; the
constant is kept for callers that read it.
"""

from torch import Tensor

from kernels.BlockSparseDecodeAttention import (  # noqa: F401
    _cdt, _decode, _last_stride_1, block_sparse_decode_attention,
)

# keys per split of the reference (kernels/SplitKVDecodeAttention.py:13); informational here
SPLIT_N = 256


def split_kv_decode_attention(
    q: Tensor,  # (batch, heads, q_len, head_dim): the last q_len positions
    k: Tensor,  # (batch, heads, kv_len, head_dim)
    v: Tensor,
    block_size: int,
) -> Tensor:
    """Same result as block_sparse_decode_attention, with the keys split across CTAs."""
    B, H, q_len, D = q.shape
    if q_len > 64:
        # prefill: many query tiles already fill the GPU
        return block_sparse_decode_attention(q, k, v, block_size)
    return _decode(q, k, v, block_size)
