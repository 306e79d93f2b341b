"""In-place KV cache for cached BD3-LM sampling, and the fused QKV + RoPE + cache write.

``KVCache`` is a drop-in for the reference's ``model/kv_cache.py:KVCache`` (:9-55): the same
``KVCache.empty(n_layers)``, ``length``, ``get(layer_idx)`` and ``append(layer_idx, k, v)``,
and ``k`` / ``v`` lists that read like the reference's fields. Each layer's keys and values
live in one preallocated ``(batch, heads, capacity, head_dim)`` tensor: ``get`` returns views
of its first ``length`` rows and ``append`` writes the new rows in place, where the reference
concatenates the whole cache on every commit (:54-55).

``KVCache.rope_qkv`` is the cached path of ``BidirectionalMultiHeadAttention.forward``
(``model/modules.py:393-417``) in one kernel (``bd3_qkv_rope_cache``): it splits the fused QKV
projection, applies the layer's RoPE to q and k with the reference's roundings, writes the
new K/V into the rows right after the committed ones and returns q with views of the cached
plus new K/V, so the per-step ``torch.cat`` of the cache (:410-414) is gone as well. Without
``store`` the new rows sit past ``length`` (the next call overwrites them); with ``store`` the
layer's length advances, as ``append`` does in the reference (:416-417).

``install(modules)`` points the reference's attention forward at ``rope_qkv`` whenever it is
handed this cache; with any other cache (or none) the original forward runs.
"""

from __future__ import annotations

import torch

from bd3attn import ops


class KVCache:
    """Per-layer post-RoPE keys/values of committed blocks, stored in place.

    Args:
        n_layers: number of attention layers (one slot each).
        capacity: rows per layer to allocate on a layer's first write (e.g. the model's
            max_seq_len). None grows the storage geometrically when it fills.
    """

    def __init__(self, n_layers: int, capacity: int | None = None):
        if n_layers < 1:
            raise ValueError("n_layers must be >= 1")
        if capacity is not None and capacity < 1:
            raise ValueError("capacity must be >= 1")
        self.n_layers = n_layers
        self.capacity = capacity
        self._k: list[torch.Tensor | None] = [None] * n_layers
        self._v: list[torch.Tensor | None] = [None] * n_layers
        self._len = [0] * n_layers

    @classmethod
    def empty(cls, n_layers: int, capacity: int | None = None) -> "KVCache":
        """A cache with no committed tokens, one slot per layer (model/kv_cache.py:27-30)."""
        return cls(n_layers, capacity)

    @property
    def length(self) -> int:
        """Number of committed tokens (layer 0's, as in model/kv_cache.py:32-36)."""
        return self._len[0]

    @property
    def k(self) -> list[torch.Tensor | None]:
        return [self.get(i)[0] for i in range(self.n_layers)]

    @property
    def v(self) -> list[torch.Tensor | None]:
        return [self.get(i)[1] for i in range(self.n_layers)]

    def get(self, layer_idx: int):
        """Views (batch, heads, length, head_dim) of one layer's cached k, v, or (None, None)."""
        n = self._len[layer_idx]
        if n == 0:
            return None, None
        return self._k[layer_idx][:, :, :n], self._v[layer_idx][:, :, :n]

    def _reserve(self, layer_idx: int, B: int, H: int, D: int, dtype, device, rows: int):
        """Storage for at least `rows` rows of this layer, allocated or grown in place of the
        old one (its committed rows copied over)."""
        k = self._k[layer_idx]
        if k is not None and (k.shape[0] != B or k.shape[1] != H or k.shape[3] != D
                              or k.dtype != dtype or k.device != torch.device(device)):
            raise RuntimeError(
                f"layer {layer_idx}: new keys ({B}, {H}, *, {D}) {dtype} do not match the "
                f"cache ({k.shape[0]}, {k.shape[1]}, *, {k.shape[3]}) {k.dtype}")
        have = 0 if k is None else k.shape[2]
        if rows <= have:
            return
        if self.capacity is not None:
            if rows > self.capacity:
                raise RuntimeError(f"KV cache capacity {self.capacity} exceeded ({rows} rows)")
            cap = self.capacity
        else:
            cap = max(rows, 2 * have, 256)
        n = self._len[layer_idx]
        nk = torch.empty((B, H, cap, D), dtype=dtype, device=device)
        nv = torch.empty_like(nk)
        if n:
            nk[:, :, :n].copy_(self._k[layer_idx][:, :, :n])
            nv[:, :, :n].copy_(self._v[layer_idx][:, :, :n])
        self._k[layer_idx], self._v[layer_idx] = nk, nv

    def append(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append one layer's post-RoPE keys/values (batch, heads, new, head_dim) in place."""
        if k.shape != v.shape or k.dim() != 4:
            raise RuntimeError("k and v must both be (batch, heads, new, head_dim)")
        B, H, s, D = k.shape
        n = self._len[layer_idx]
        self._reserve(layer_idx, B, H, D, k.dtype, k.device, n + s)
        self._k[layer_idx][:, :, n:n + s].copy_(k)
        self._v[layer_idx][:, :, n:n + s].copy_(v)
        self._len[layer_idx] = n + s

    def rope_qkv(self, layer_idx: int, qkv: torch.Tensor, n_heads: int, cos_table: torch.Tensor,
                 sin_table: torch.Tensor, positions: torch.Tensor | None = None,
                 store: bool = False):
        """(q, k_all, v_all) of one layer from its fused QKV projection (batch, seq, 3*d).

        q: (batch, heads, seq, head_dim) rotated queries; k_all, v_all: views of the cached
        rows followed by this call's rotated keys / values (what the reference builds with
        torch.cat). positions: (seq,) absolute positions (None: 0 .. seq-1, as RoPE.forward).
        """
        if qkv.dim() != 3:
            raise AssertionError("qkv must be (batch, seq, 3 * d_model)")
        B, S, F = qkv.shape
        D = F // (3 * n_heads)
        n = self._len[layer_idx]
        self._reserve(layer_idx, B, n_heads, D, qkv.dtype, qkv.device, n + S)
        kc, vc = self._k[layer_idx], self._v[layer_idx]
        q = ops.qkv_rope_cache_op(qkv, n_heads, cos_table, sin_table, kc, vc, n, positions)
        if store:
            self._len[layer_idx] = n + S
        return q, kc[:, :, :n + S], vc[:, :, :n + S]


def install(modules) -> None:
    """Route ``modules.BidirectionalMultiHeadAttention.forward`` (model/modules.py:368-422)
    through ``KVCache.rope_qkv`` when it is given a ``bd3attn.kv_cache.KVCache`` on a CUDA
    input; every other call runs the original forward. Idempotent."""
    cls = modules.BidirectionalMultiHeadAttention
    orig = cls.forward
    if getattr(orig, "_bd3_fused", False):
        return

    def forward(self, x, mask=None, positions=None, kv_cache=None, layer_idx=0, store=False):
        if not isinstance(kv_cache, KVCache) or not x.is_cuda or x.dim() != 3:
            return orig(self, x, mask, positions, kv_cache, layer_idx, store)
        qkv = self.qkv(x)
        q, k_all, v_all = kv_cache.rope_qkv(layer_idx, qkv, self.n_heads, self.rope.cos_table,
                                            self.rope.sin_table, positions, store)
        o = modules.scaled_dot_product_attention(q, k_all, v_all, mask)
        B, H, S, D = o.shape
        return self.out(o.transpose(1, 2).reshape(B, S, H * D))

    forward._bd3_fused = True
    forward.__doc__ = orig.__doc__
    cls.forward = forward
