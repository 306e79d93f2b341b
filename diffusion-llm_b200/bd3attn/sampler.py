"""The BD3-LM block sampler's denoising step as one kernel (bd3_subs_sample).

``subs_sample_step(logits, block, mask_index, t, s)`` returns the block after one ancestral
step of ``sample/sampler.py:100-122``: SUBS log-probabilities of the backbone's logits
(``model/subs.py:11-43``), the weights ``exp(log_probs) * (1 - s/t)`` with ``s/t`` on
[MASK], the float64 Gumbel-max draw of ``sample_categorical`` (``sample/sampler.py:11-34``)
and the ``where`` that keeps unmasked tokens. In the reference loop it replaces

    log_probs = model.cached_block_logprobs(block, cache)      # backbone + SUBS
    q = torch.exp(log_probs).double() * (1 - s / t)
    q[..., mask_index] = s / t
    block = torch.where(block != mask_index, block, sample_categorical(q))

with the backbone call and one ``subs_sample_step``. The draw comes from Philox4x32-10 in
the kernel, seeded from ``generator`` (torch's default CPU generator when None), so no
(batch, block, vocab) float64 tensor of uniforms is written; ``uniforms=`` replays a given
draw instead.
"""

from __future__ import annotations

import torch

from bd3attn._lib import LIB, check, i64_array
from bd3attn.ops import _check_cuda, _code, _ptr, _stream


def subs_sample_step(logits: torch.Tensor, block: torch.Tensor, mask_index: int, t: float,
                     s: float, generator: torch.Generator | None = None,
                     uniforms: torch.Tensor | None = None, out: torch.Tensor | None = None,
                     offset: int = 0) -> torch.Tensor:
    """Next (batch, block_size) int64 tokens from logits (batch, block_size, vocab)."""
    _check_cuda(logits, block)
    if logits.dim() != 3 or block.shape != logits.shape[:2]:
        raise AssertionError("logits must be (batch, seq, vocab) and block (batch, seq)")
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    block = block.to(torch.int64).contiguous()
    B, S, V = logits.shape
    if out is None:
        out = torch.empty_like(block)
    if uniforms is not None:
        if uniforms.shape != logits.shape:
            raise AssertionError("uniforms must have the logits' shape")
        uniforms = uniforms.to(device=logits.device, dtype=torch.float64).contiguous()
        seed = 0
    else:
        seed = int(torch.randint(0, 2 ** 63 - 1, (1,), generator=generator).item())
    with torch.cuda.device(logits.device):
        check("bd3_subs_sample", LIB.bd3_subs_sample(
            _ptr(logits), i64_array((logits.stride(0), logits.stride(1))), B, S, V, _ptr(block),
            int(mask_index), float(t), float(s), seed, int(offset), _ptr(uniforms), _ptr(out),
            _code(logits.dtype), _stream(logits)))
    return out


def subs_sample_step_dev(logits: torch.Tensor, block: torch.Tensor, mask_index: int,
                         ts: torch.Tensor, seed_offset: torch.Tensor,
                         out: torch.Tensor | None = None) -> torch.Tensor:
    """subs_sample_step's Philox draw with the step's values on the device, for a sampling
    loop captured in a CUDA graph: ts is a float64 device tensor (t, s) and seed_offset an
    int64 device tensor (seed, offset) read as unsigned 64-bit words. Advance them between
    replays (for example ``seed_offset[1] += 1``); nothing here reads them on the host."""
    _check_cuda(logits, block, ts, seed_offset)
    if logits.dim() != 3 or block.shape != logits.shape[:2]:
        raise AssertionError("logits must be (batch, seq, vocab) and block (batch, seq)")
    if ts.dtype != torch.float64 or ts.numel() != 2 or not ts.is_contiguous():
        raise AssertionError("ts must be a contiguous float64 device tensor (t, s)")
    if seed_offset.dtype != torch.int64 or seed_offset.numel() != 2 \
            or not seed_offset.is_contiguous():
        raise AssertionError("seed_offset must be a contiguous int64 device tensor (seed, offset)")
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    if block.dtype != torch.int64 or not block.is_contiguous():
        raise AssertionError("block must be a contiguous int64 tensor")
    B, S, V = logits.shape
    if out is None:
        out = torch.empty_like(block)
    with torch.cuda.device(logits.device):
        check("bd3_subs_sample_dev", LIB.bd3_subs_sample_dev(
            _ptr(logits), i64_array((logits.stride(0), logits.stride(1))), B, S, V, _ptr(block),
            int(mask_index), _ptr(ts), _ptr(seed_offset), _ptr(out), _code(logits.dtype),
            _stream(logits)))
    return out
