"""Masked attention, its gradients, masks and the split-KV merge, on the CPU in float64.

TEST INFRASTRUCTURE ONLY (see the package docstring): the checker for the CUDA path.

Reference files restated here (paths inside tusharsonthalia/diffusion-llm):
  model/bd3lm.py:10-52                      block_diff_mask
  model/modules.py:728-771                  softmax, scaled_dot_product_attention
  kernels/BlockSparseFlashAttention.py:169  LSE = m + ln(l), natural log
  kernels/BlockSparseDecodeAttention.py:84-94 and model/bd3lm.py:168
                                            block-causal rule of the decode kernels
  kernels/SplitKVDecodeAttention.py:109-119 LSE-weighted merge of partials
"""

from __future__ import annotations

import numpy as np
import torch


def block_diff_mask(n: int, block_size: int) -> np.ndarray:
    """The (2n, 2n) BD3-LM training mask over cat(x_t, x_0) (model/bd3lm.py:10-52).

    Rows are queries, columns keys; [0, n) is the noisy copy, [n, 2n) the clean one.
    noisy q in block b sees noisy keys of block b and clean keys of blocks < b;
    clean q in block b sees clean keys of blocks <= b; clean q never sees noisy keys.
    """
    idx = np.arange(2 * n, dtype=np.int64)
    q = idx[:, None]
    k = idx[None, :]
    q_clean = q >= n
    k_clean = k >= n
    q_block = (q % n) // block_size
    k_block = (k % n) // block_size
    diag = ~q_clean & ~k_clean & (q_block == k_block)
    offset_causal = ~q_clean & k_clean & (k_block < q_block)
    causal = q_clean & k_clean & (k_block <= q_block)
    return diag | offset_causal | causal


def block_causal_mask(q_len: int, kv_len: int, block_size: int) -> np.ndarray:
    """(q_len, kv_len) mask of the decode kernels: the queries are the LAST q_len of the
    kv_len positions and see every key whose block is <= their own block.

    This is the rule of kernels/BlockSparseDecodeAttention.py:84-94 (mask at :25-26), and it
    equals rows [kv_len - q_len, kv_len) of the prefill mask attn_mask[n:n+L, n:n+L] that
    model/bd3lm.py:168 and sample/sampler.py:85 pass to the reference attention.
    """
    q_pos = np.arange(kv_len - q_len, kv_len, dtype=np.int64)[:, None]
    kv = np.arange(kv_len, dtype=np.int64)[None, :]
    return (q_pos // block_size) >= (kv // block_size)


def live_block_mask(live: list[list[list[int]]], q_len: int, kv_len: int,
                    kv_block: int, block_size: int) -> np.ndarray:
    """(B, H, q_len, kv_len) mask for block-sparse decode with a per-(batch, head) list of
    live KV blocks of ``kv_block`` tokens, intersected with the block-causal rule.

    The reference has no kernel for a per-head KV block mask; its oracle for one is the
    reference attention given this expanded boolean mask, which model/modules.py:750
    broadcasts over (batch, heads, q, kv).
    """
    B, H = len(live), len(live[0])
    base = block_causal_mask(q_len, kv_len, block_size)
    out = np.zeros((B, H, q_len, kv_len), dtype=bool)
    for b in range(B):
        for h in range(H):
            cols = np.zeros(kv_len, dtype=bool)
            for blk in live[b][h]:
                cols[blk * kv_block:min((blk + 1) * kv_block, kv_len)] = True
            out[b, h] = base & cols[None, :]
    return out


def _as64(x, dtype=torch.float64) -> torch.Tensor:
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(x)
    if x.requires_grad and x.dtype == dtype and x.device.type == "cpu":
        return x  # keep the autograd graph of attention_grads
    return x.detach().to(device="cpu", dtype=dtype)


def attention(q, k, v, mask=None, dtype=torch.float64, with_lse=True):
    """(O, LSE) of softmax(q k^T / sqrt(d) masked) v, computed in ``dtype`` (float64 for the
    parity checks; float32 is the reference's own CPU arithmetic, used for timing).

    O restates model/modules.py:738-771 (logits upcast before the product, masked scores
    set to -inf, a max-subtracted softmax, then P V). LSE is the per-row natural-log
    log-sum-exp of the scaled, masked scores, the quantity the reference training kernel
    writes as m + ln(l) (kernels/BlockSparseFlashAttention.py:169).

    q: (..., Sq, D), k and v: (..., Sk, D); mask: bool broadcastable to (..., Sq, Sk).
    """
    q, k, v = _as64(q, dtype), _as64(k, dtype), _as64(v, dtype)
    scale = 1.0 / (q.shape[-1] ** 0.5)
    scores = torch.einsum("...qd,...kd->...qk", q, k) * scale
    if mask is not None:
        m = torch.as_tensor(np.asarray(mask)) if not torch.is_tensor(mask) else mask.cpu()
        scores = torch.where(m, scores, torch.tensor(-torch.inf, dtype=dtype))
    z = scores - scores.amax(dim=-1, keepdim=True)
    e = torch.exp(z)
    p = e / e.sum(dim=-1, keepdim=True)
    out = torch.einsum("...qk,...kd->...qd", p, v)
    lse = torch.logsumexp(scores, dim=-1) if with_lse else None
    return out, lse


def attention_grads(q, k, v, do, mask=None, dtype=torch.float64):
    """(dQ, dK, dV) of attention(q, k, v, mask)[0] against the cotangent ``do``, by
    autograd through the float64 restatement (the oracle named for the training kernels'
    backward, kernels/BlockSparseFlashAttention.py:509-562)."""
    q = _as64(q, dtype).requires_grad_(True)
    k = _as64(k, dtype).requires_grad_(True)
    v = _as64(v, dtype).requires_grad_(True)
    out, _ = attention(q, k, v, mask, dtype=dtype, with_lse=False)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), _as64(do, dtype))
    return dq, dk, dv


def lse_merge(o_parts, lse_parts):
    """Merge partial attention results over disjoint key sets.

    o_parts: (G, ..., Sq, D) outputs each normalised over its own keys; lse_parts:
    (G, ..., Sq) their log-sum-exps. Restates kernels/SplitKVDecodeAttention.py:109-119:
    weights exp(LSE_g - max_g LSE_g), normalised by their sum. Returns (O, LSE).
    A partial that saw no key (LSE = -inf, O undefined) gets weight 0 and contributes
    nothing, as a split of only masked keys does in the reference (its -1e6 masking leaves
    such a split a finite LSE whose weight underflows to 0).
    """
    o = _as64(o_parts)
    lse = _as64(lse_parts)
    m = lse.amax(dim=0, keepdim=True)
    w = torch.exp(lse - m)
    den = w.sum(dim=0)
    contrib = torch.where(w[..., None] > 0, w[..., None] * o, torch.zeros_like(o))
    out = contrib.sum(dim=0) / den[..., None]
    return out, m[0] + torch.log(den)
