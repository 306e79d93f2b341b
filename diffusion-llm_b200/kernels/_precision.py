"""fp32 inputs on the 16-bit tensor-core kernels, at tf32's precision.

The reference computes fp32 inputs with Triton's ``tl.dot``, which on tensor cores is tf32
(kernels/BlockSparseFlashAttention.py:45-70): operands rounded to an 11-bit significand (10
stored bits) and products accumulated in fp32. fp16 has the same 11-bit significand but a
narrower exponent range (normal numbers from 2^-14 to 65504), so fp32 tensors are first scaled
by powers of two, which is exact, into fp16's range and then rounded:

* q by 2^-a and k by 2^a, a = floor((e_q - e_k) / 2) with e_x = floor(log2(max |x|)): every
  score q . k is unchanged, and the two operands get balanced magnitudes;
* v by 2^-c, c = e_v - 4, so that max |v| lies in [16, 32); the output is scaled back by 2^c;
* in the backward, dO by 2^-e_dO (max in [1, 2)); the gradients are scaled back by the
  matching powers of two (chain rule through the three scalings).

The exponents are computed on the device, so nothing waits on the host: torch.compile and
CUDA graph capture see one custom op (two kernels, bd3_f32_to_f16_scaled) for the operands.
Where the two differ:

* values far below a tensor's maximum become fp16 subnormals or zero (absolute error below
  2^-25 of fp16's unit at the scaled maximum), which tf32 keeps normal;
* when max|q| * max|k| >= 2^30 the balanced operands cannot both fit in fp16 (the scores
  then exceed 2^26, a one-hot softmax); they saturate at +-65504 instead of overflowing.
"""

from __future__ import annotations

import torch
from torch import Tensor

from bd3attn import ops


def exponent(t: Tensor) -> Tensor:
    """floor(log2(max |t|)) as a 0-d fp32 tensor on t's device, exactly (from the binary
    exponent), and at least -100."""
    m = t.detach().abs().amax().float()
    return (torch.frexp(m).exponent.float() - 1.0).clamp_min(-100.0)


def qkv_to_f16(q: Tensor, k: Tensor, v: Tensor):
    """(q16, k16, v16, a, c): q * 2^-a, k * 2^a, v * 2^-c rounded to fp16 (q and k
    saturated), and the exponents a, c as 0-d fp32 device tensors; one library call."""
    if torch.compiler.is_compiling():
        q16, k16, v16, exps = torch.ops.bd3.f32_to_f16_scaled(q, k, v)
    else:
        q16, k16, v16, exps = ops.f32_to_f16_scaled_raw(q, k, v)
    return q16, k16, v16, exps[0], exps[1]


def grad_to_f16(do: Tensor):
    """(dO * 2^-e rounded to fp16, e) with e = floor(log2(max |dO|))."""
    e = exponent(do)
    return (do.float() * torch.exp2(-e)).to(torch.float16), e


def scaled_back(x: Tensor, e: Tensor) -> Tensor:
    """x (16-bit) as fp32 times 2^e."""
    return x.float() * torch.exp2(e)
