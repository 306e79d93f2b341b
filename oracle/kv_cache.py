"""RoPE, the QKV split and the reference's concatenating KV cache, on the CPU in numpy.

TEST INFRASTRUCTURE ONLY (see the package docstring): the checker for bd3_qkv_rope_cache and
bd3attn.kv_cache.

Reference files restated here (paths inside tusharsonthalia/diffusion-llm):
  model/modules.py:164-240   RoPE: tables (float64 angles -> fp32 sin/cos), rotate-half
                             forward with the tables cast to the activation dtype and one
                             rounding per elementwise op
  model/modules.py:395-417   fused projection split (three, heads, head_dim), RoPE on q and
                             k, cached K/V concatenated in front of the new ones, append
  model/kv_cache.py:9-55     KVCache: empty, length, get, append (torch.cat along seq)
"""

from __future__ import annotations

import numpy as np


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to `dtype` ("bf16", "f16" or "f32") and back to float32
    (round to nearest even, as torch's casts do)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype != "bf16":
        raise ValueError(dtype)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(nan, x, out).astype(np.float32)


def rope_tables(head_dim: int, max_seq_len: int, theta: float = 10000.0):
    """(sin, cos), each (max_seq_len, head_dim/2) float32 (model/modules.py:196-207):
    angles = position * theta^(-2k/d) in float64, then sin/cos rounded to float32."""
    pos = np.arange(max_seq_len, dtype=np.float64)
    pair = np.arange(0, head_dim, 2, dtype=np.float64)
    inv = theta ** (-pair / head_dim)
    ang = pos[:, None] * inv[None, :]
    return np.sin(ang).astype(np.float32), np.cos(ang).astype(np.float32)


def rope(x: np.ndarray, positions: np.ndarray, sin_table: np.ndarray, cos_table: np.ndarray,
         dtype: str) -> np.ndarray:
    """RoPE.forward (model/modules.py:209-240) on (..., seq, d) values already in `dtype`:
    sin/cos rows cast to the dtype, out_1 = x_1*cos - x_2*sin, out_2 = x_1*sin + x_2*cos,
    each product, difference and sum rounded to the dtype (float32 arithmetic in between)."""
    x = np.asarray(x, dtype=np.float32)
    sin = round_to(sin_table[positions], dtype)
    cos = round_to(cos_table[positions], dtype)
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    r = lambda a: round_to(a, dtype)  # noqa: E731
    o1 = r(r(x1 * cos) - r(x2 * sin))
    o2 = r(r(x1 * sin) + r(x2 * cos))
    return np.concatenate([o1, o2], axis=-1)


def split_qkv(qkv: np.ndarray, n_heads: int):
    """rearrange(qkv, "b s (three h d) -> three b h s d") (model/modules.py:398-402)."""
    B, S, F = qkv.shape
    D = F // (3 * n_heads)
    t = qkv.reshape(B, S, 3, n_heads, D).transpose(2, 0, 3, 1, 4)
    return t[0], t[1], t[2]


class ConcatKVCache:
    """The reference's KVCache semantics (model/kv_cache.py:9-55): per-layer (B, H, L, D)
    arrays, None until the first append, each append a concatenation along seq."""

    def __init__(self, n_layers: int):
        self.k = [None] * n_layers
        self.v = [None] * n_layers

    @property
    def length(self) -> int:
        return 0 if self.k[0] is None else self.k[0].shape[-2]

    def get(self, layer_idx: int):
        return self.k[layer_idx], self.v[layer_idx]

    def append(self, layer_idx: int, k: np.ndarray, v: np.ndarray) -> None:
        if self.k[layer_idx] is None:
            self.k[layer_idx], self.v[layer_idx] = k, v
        else:
            self.k[layer_idx] = np.concatenate([self.k[layer_idx], k], axis=-2)
            self.v[layer_idx] = np.concatenate([self.v[layer_idx], v], axis=-2)


def cached_qkv(cache: ConcatKVCache, layer_idx: int, qkv: np.ndarray, n_heads: int,
               positions: np.ndarray, sin_table, cos_table, dtype: str, store: bool):
    """The K/V side of the cached attention forward (model/modules.py:395-417): returns
    (q, k_all, v_all) and appends the new k, v when `store`."""
    q, k, v = split_qkv(qkv, n_heads)
    q = rope(q, positions, sin_table, cos_table, dtype)
    k = rope(k, positions, sin_table, cos_table, dtype)
    kc, vc = cache.get(layer_idx)
    k_all = k if kc is None else np.concatenate([kc, k], axis=-2)
    v_all = v if vc is None else np.concatenate([vc, v], axis=-2)
    if store:
        cache.append(layer_idx, k, v)
    return q, k_all, v_all
