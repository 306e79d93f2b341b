"""A stand-in BD3-LM training backbone for measuring attention backends inside a real loss.

The reference trains its DiT (model/modules.py) on the 2n input cat(x_t, x_0) with the block
diffusion mask and positions arange(n) repeated twice (model/bd3lm.py:112-140), calling
``modules.scaled_dot_product_attention(q, k, v, mask)`` in every layer; train/train.py:230
picks the backend with install_attention. This module keeps exactly that attention call
site and the reference's sizes (d_model 768, 12 heads of 64, d_ff 3072, 12 layers) around
a plain pre-norm transformer: fused QKV projection, rotate-half RoPE, attention through
``ATTENTION.scaled_dot_product_attention``, output projection, GELU MLP, and an LM head.
The DiT's adaLN conditioning is left out (the reference runs with sigma = 0); it changes no
attention shape. The loss is the cross-entropy of the x_t half's logits against x_0 at the
masked positions.

``use_attention(name, block_size)`` routes the layers. (The reference's own registry,
bench/attention.py, patches its model.modules instead; bound to this repository's
``kernels`` package it drives the reference's DiT the same way.)
"""

from __future__ import annotations

import types

import torch
import torch.nn.functional as F
from torch import nn

# the call site the layers look the attention function up on (set by use_attention)
ATTENTION = types.SimpleNamespace(scaled_dot_product_attention=None)

# implementations use_attention can route to; the first three are this library's kernels
# (through the drop-in kernels package) and take the block size, "sdpa" is PyTorch's
# attention with the boolean mask as attn_mask, for comparison
ROUTES = ("bsfa", "bsdfa", "split_kv", "sdpa")


def use_attention(name: str, block_size: int | None = None) -> None:
    """Point every layer's attention call (q, k, v, mask) at one implementation.

    "bsfa": BlockSparseFlashAttention on the 2n training input (the mask argument is
    implied by block_size); "bsdfa": block-causal attention of the last q_len positions
    (prefill; with block_size equal to the length, plain bidirectional attention);
    "split_kv": the same with the keys split for short query blocks; "sdpa": PyTorch's
    attention given the mask. ValueError for an unknown name or a missing block size.
    """
    if name not in ROUTES:
        raise ValueError(f"unknown attention route {name!r}; expected one of {ROUTES}")
    if name == "sdpa":
        ATTENTION.scaled_dot_product_attention = (
            lambda q, k, v, mask: F.scaled_dot_product_attention(q, k, v, attn_mask=mask))
        return
    if block_size is None or block_size <= 0:
        raise ValueError(f"route {name!r} needs a positive block_size")
    if name == "bsfa":
        from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
        fn = BlockSparseFlashAttention.apply
    elif name == "bsdfa":
        from kernels.BlockSparseDecodeAttention import block_sparse_decode_attention as fn
    else:
        from kernels.SplitKVDecodeAttention import split_kv_decode_attention as fn
    bs = int(block_size)
    ATTENTION.scaled_dot_product_attention = lambda q, k, v, mask: fn(q, k, v, bs)


def block_diff_mask(n: int, block_size: int, device=None) -> torch.Tensor:
    """The (2n, 2n) BD3-LM training mask (model/bd3lm.py:10-52): noisy tokens see their own
    noisy block and the clean blocks before it, clean tokens the clean blocks up to their
    own, and no clean token sees a noisy one."""
    idx = torch.arange(2 * n, device=device)
    clean = idx >= n
    blk = (idx % n) // block_size
    qc, kc = clean[:, None], clean[None, :]
    qb, kb = blk[:, None], blk[None, :]
    noisy_noisy = ~qc & ~kc & (qb == kb)
    noisy_clean = ~qc & kc & (kb < qb)
    clean_clean = qc & kc & (kb <= qb)
    return noisy_noisy | noisy_clean | clean_clean


def rope_tables(head_dim: int, max_pos: int, device=None):
    """(cos, sin) of shape (max_pos, head_dim / 2), base 10000."""
    inv = 10000.0 ** (-torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float().to(device), torch.sin(ang).float().to(device)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    c, s = cos.to(x.dtype), sin.to(x.dtype)
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


class Layer(nn.Module):
    def __init__(self, d_model: int, n_heads: int, d_ff: int):
        super().__init__()
        self.n_heads = n_heads
        self.norm1 = nn.LayerNorm(d_model)
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=False)
        self.out = nn.Linear(d_model, d_model, bias=False)
        self.norm2 = nn.LayerNorm(d_model)
        self.up = nn.Linear(d_model, d_ff)
        self.down = nn.Linear(d_ff, d_model)

    def forward(self, x, mask, cos, sin):
        B, L, d = x.shape
        q, k, v = self.qkv(self.norm1(x)).view(B, L, 3, self.n_heads, -1).permute(2, 0, 3, 1, 4)
        q, k = rope(q, cos, sin), rope(k, cos, sin)
        o = ATTENTION.scaled_dot_product_attention(q, k, v, mask)
        x = x + self.out(o.transpose(1, 2).reshape(B, L, d))
        return x + self.down(F.gelu(self.up(self.norm2(x)), approximate="tanh"))


class Backbone(nn.Module):
    """Embedding, ``n_layers`` layers on the 2n input, final norm and LM head."""

    def __init__(self, vocab_size: int, n: int, block_size: int, d_model: int = 768,
                 n_heads: int = 12, n_layers: int = 12, d_ff: int = 3072):
        super().__init__()
        self.n, self.mask_index, self.block_size = n, vocab_size - 1, block_size
        self.n_heads = n_heads
        self.embed = nn.Embedding(vocab_size, d_model)
        self.layers = nn.ModuleList(Layer(d_model, n_heads, d_ff) for _ in range(n_layers))
        self.norm = nn.LayerNorm(d_model)
        self.head = nn.Linear(d_model, vocab_size, bias=False)
        cos, sin = rope_tables(d_model // n_heads, n)
        pos = torch.arange(n).repeat(2)
        self.register_buffer("cos", cos[pos], persistent=False)
        self.register_buffer("sin", sin[pos], persistent=False)
        self.register_buffer("attn_mask", block_diff_mask(n, block_size), persistent=False)

    def encode(self, tokens: torch.Tensor, mask, cos: torch.Tensor,
               sin: torch.Tensor) -> torch.Tensor:
        """Logits of every position of ``tokens`` (batch, L) under ``mask`` (L, L) or None,
        with the RoPE rows ``cos``, ``sin`` (L, head_dim / 2) of their positions."""
        x = self.embed(tokens)
        for layer in self.layers:
            x = layer(x, mask, cos, sin)
        return self.head(self.norm(x))

    def forward(self, xt: torch.Tensor, x0: torch.Tensor) -> torch.Tensor:
        return self.encode(torch.cat([xt, x0], dim=-1), self.attn_mask, self.cos,
                           self.sin)[:, :self.n]

    def loss(self, xt: torch.Tensor, x0: torch.Tensor) -> torch.Tensor:
        """Mean cross-entropy over the masked positions (no host synchronisation)."""
        logits = self(xt, x0).float()
        ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), x0.reshape(-1),
                             reduction="none")
        masked = (xt == self.mask_index).reshape(-1).float()
        return (ce * masked).sum() / masked.sum().clamp_min(1.0)


def noisy_batch(gen: torch.Generator, batch: int, n: int, block_size: int, vocab_size: int,
                repeat_blocks: bool = False, n_tokens: int | None = None):
    """Seeded synthetic (x_t, x_0): tokens uniform over the first n_tokens ids (all but
    [MASK] by default; with repeat_blocks every block is a copy of the first, so a masked
    token is predictable from the clean block before it), each block masked at its own rate
    in [0.1, 0.9] (the reference draws a per-block noise level)."""
    hi = vocab_size - 1 if n_tokens is None else n_tokens
    if repeat_blocks:
        first = torch.randint(0, hi, (batch, block_size), generator=gen)
        x0 = first.repeat(1, n // block_size)
    else:
        x0 = torch.randint(0, hi, (batch, n), generator=gen)
    rate = 0.1 + 0.8 * torch.rand(batch, n // block_size, 1, generator=gen)
    rate = rate.expand(-1, -1, block_size).reshape(batch, n)
    xt = torch.where(torch.rand(batch, n, generator=gen) < rate,
                     torch.full_like(x0, vocab_size - 1), x0)
    return xt, x0


def train_step(model: Backbone, optimizer: torch.optim.Optimizer, xt: torch.Tensor,
               x0: torch.Tensor, grad_clip: float = 1.0) -> torch.Tensor:
    """One step as the reference's baseline step (train/train.py:110-133): forward and loss
    under bf16 autocast, backward, gradient-norm clipping, AdamW step, zero_grad. Returns
    the loss (a device scalar; nothing here synchronises)."""
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        loss = model.loss(xt, x0)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), grad_clip)
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return loss.detach()
