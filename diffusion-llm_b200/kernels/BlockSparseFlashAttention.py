"""Block-sparse FlashAttention under the BD3-LM training mask, on B200 tensor cores.

Drop-in for kernels/BlockSparseFlashAttention.py of the reference: the autograd function
``BlockSparseFlashAttention.apply(q, k, v, block_size)`` with the same arguments, the same
assertions (:474-476, :487, :522) and the same saved tensors (q, k, v, O, L), where L is the
per-row natural-log LSE of shape (B, H, 2n) in fp32 (:482, :169). The forward is the
tcgen05 kernel of csrc/attn_fwd.cuh, the backward the three kernels of csrc/attn_bwd.cuh.

Inputs are 16-bit (bf16 or f16), which is what autocast hands the model's attention, or fp32.
The reference's Triton path computes fp32 inputs with tf32 dots (11-bit significands, fp32
accumulation); here they run on the fp16 kernels, whose operands have the same 11-bit
significand, after an exact power-of-two scaling into fp16's range (kernels/_precision.py),
and O, dQ, dK, dV come back as fp32. Mixed input dtypes run in bf16.
"""

from typing import Any

import torch
from torch import Tensor

from bd3attn import ops
from kernels import _precision


# query-tile height of the sm_100a training kernels; n must be a multiple of it (a module
# constant: torch.compile cannot read attributes of the autograd.Function class while tracing)
_FWD_TILE_M = 128


def _compute_dtype(*xs: Tensor) -> torch.dtype:
    dts = {x.dtype for x in xs}
    if dts <= {torch.float16}:
        return torch.float16
    return torch.bfloat16


class BlockSparseFlashAttention(torch.autograd.Function):
    """Attention under the BD3-LM block diffusion mask."""

    # tile shape of the sm_100a kernels (the reference's Triton tiles were 128x64 forward,
    # 128x64 dQ and 128x32 dK/dV); the same range formulas select the visited tiles
    FWD_BLOCK_M, FWD_BLOCK_N = _FWD_TILE_M, 128
    BWD_DQ_BLOCK_M, BWD_DQ_BLOCK_N = 128, 128
    BWD_DKDV_BLOCK_KV, BWD_DKDV_BLOCK_Q = 128, 128

    @staticmethod
    def forward(ctx: Any, q: Tensor, k: Tensor, v: Tensor, block_size: int) -> Tensor:
        B, H, seq_len, D = q.shape
        assert q.is_cuda, "inputs must be on CUDA"
        assert q.shape == k.shape == v.shape, "q, k, v must match"
        assert seq_len % 2 == 0, "BD3-LM input is cat(x_t, x_0): length 2n"
        n = seq_len // 2
        assert n % _FWD_TILE_M == 0, "n must be a multiple of the 128-row query tile"
        out_dtype = q.dtype
        scaled = q.dtype == k.dtype == v.dtype == torch.float32
        if scaled:
            qc, kc, vc, a, c = _precision.qkv_to_f16(q, k, v)
        else:
            cdt = _compute_dtype(q, k, v)
            qc, kc, vc = q.to(cdt), k.to(cdt), v.to(cdt)
        if torch.compiler.is_compiling():
            o, lse = torch.ops.bd3.attn_fwd(qc, kc, vc, int(block_size))
        else:
            o, lse = ops.attn_fwd_raw(qc, kc, vc, int(block_size))
        ctx.scaled = scaled
        ctx.save_for_backward(qc, kc, vc, o, lse, *((a, c) if scaled else ()))
        ctx.block_size = block_size
        ctx.out_dtypes = (q.dtype, k.dtype, v.dtype)
        if scaled:
            return _precision.scaled_back(o, c)
        return o if out_dtype == o.dtype else o.to(out_dtype)

    @staticmethod
    def backward(ctx: Any, dO: Tensor):  # type: ignore[override]
        q, k, v, O, L = ctx.saved_tensors[:5]
        block_size = ctx.block_size
        n = q.shape[2] // 2
        assert n % block_size == 0
        if ctx.scaled:
            a, c = ctx.saved_tensors[5:]
            dO, e = _precision.grad_to_f16(dO)
        else:
            dO = dO.to(q.dtype)
        # torch.use_deterministic_algorithms(True) selects the backward whose dQ is the same
        # on every run (fixed-point accumulation), as the reference's dQ kernel's is
        det = torch.are_deterministic_algorithms_enabled()
        if torch.compiler.is_compiling():
            dq, dk, dv = torch.ops.bd3.attn_bwd(q, k, v, O, L, dO, int(block_size), det)
        else:
            dq, dk, dv = ops.attn_bwd_raw(q, k, v, O, L, dO, int(block_size), det)
        if ctx.scaled:
            # the kernel got 2^-e dO = 2^-(c+e) * (2^c dO), and 2^c dO is the cotangent of
            # O' = 2^-c O, so its gradients are 2^-(c+e) times those of q', k', v'
            d = c + e
            return (_precision.scaled_back(dq, d - a), _precision.scaled_back(dk, d + a),
                    _precision.scaled_back(dv, e), None)
        tq, tk, tv = ctx.out_dtypes
        return dq.to(tq), dk.to(tk), dv.to(tv), None
