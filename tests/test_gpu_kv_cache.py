"""bd3_qkv_rope_cache and the in-place KVCache on the GPU against the CPU oracle (bit-exact):
the fused QKV split + RoPE + cache write, a cached sampling sequence (commit, steps, commit)
through KVCache.rope_qkv, and the reference attention forward routed through it by install().
"""

import types

import numpy as np
import pytest
import torch

from gpu_util import assert_device_ok
from oracle import kv_cache as okv

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _qkv(gen, B, S, H, D, dt, pad=0):
    """(B, S, 3*H*D) activations in dtype `dt` on the CPU and on the GPU; with pad > 0 the GPU
    copy is a strided slice (batch stride (S + pad) * 3*H*D) of a wider device tensor."""
    big = (2 * torch.randn((B, S + pad, 3 * H * D), generator=gen)).to(DT[dt])
    return big[:, pad:], big.cuda()[:, pad:]


def _tables(D, max_pos):
    sin, cos = okv.rope_tables(D, max_pos)
    return torch.from_numpy(sin), torch.from_numpy(cos)


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("B,S,H,D,row0,use_pos", [(2, 16, 3, 64, 5, True), (1, 1, 12, 64, 0, False),
                                                  (3, 37, 2, 64, 100, True), (1, 8, 2, 128, 3, False)])
def test_kernel_bit_exact(dt, B, S, H, D, row0, use_pos):
    from bd3attn import ops
    gen = torch.Generator().manual_seed(S * 31 + H)
    max_pos = 256
    sin, cos = _tables(D, max_pos)
    qkv, qkv_d = _qkv(gen, B, S, H, D, dt, pad=3)
    assert B == 1 or not qkv_d.is_contiguous()  # (a size-1 batch is contiguous anyway)
    if use_pos:
        pos = torch.randint(0, max_pos, (S,), generator=gen)
        pos0 = 0
    else:
        pos, pos0 = None, 200
    rows = row0 + S + 9
    sentinel = torch.full((B, H, rows, D), 7.0).to(DT[dt])
    kc, vc = sentinel.clone().cuda(), sentinel.clone().cuda()
    q = ops.qkv_rope_cache_raw(qkv_d, H, cos.cuda(), sin.cuda(), kc, vc, row0,
                               positions=None if pos is None else pos.cuda(), pos0=pos0)
    assert_device_ok()
    p = pos.numpy() if pos is not None else np.arange(pos0, pos0 + S)
    qo, ko, vo = okv.split_qkv(qkv.float().numpy(), H)
    q_ref = okv.rope(qo, p, sin.numpy(), cos.numpy(), dt)
    k_ref = okv.rope(ko, p, sin.numpy(), cos.numpy(), dt)
    np.testing.assert_array_equal(q.float().cpu().numpy(), q_ref)
    np.testing.assert_array_equal(kc[:, :, row0:row0 + S].float().cpu().numpy(), k_ref)
    np.testing.assert_array_equal(vc[:, :, row0:row0 + S].float().cpu().numpy(), vo)
    # rows outside [row0, row0 + S) untouched
    for c in (kc, vc):
        assert torch.all(c[:, :, :row0].float() == 7.0) and torch.all(c[:, :, row0 + S:].float() == 7.0)


def test_kernel_strided_q_out_and_cache_views():
    """q_out and the caches as strided views (the head axis outermost in memory)."""
    from bd3attn import ops
    gen = torch.Generator().manual_seed(3)
    B, S, H, D = 2, 16, 4, 64
    sin, cos = _tables(D, 64)
    _, qkv = _qkv(gen, B, S, H, D, "bf16")
    q_out = torch.empty(H, B, S, D, dtype=torch.bfloat16, device="cuda").transpose(0, 1)
    kc = torch.zeros(H, B, 40, D, dtype=torch.bfloat16, device="cuda").transpose(0, 1)
    vc = torch.zeros(H, B, 40, D, dtype=torch.bfloat16, device="cuda").transpose(0, 1)
    ops.qkv_rope_cache_raw(qkv, H, cos.cuda(), sin.cuda(), kc, vc, 20, pos0=30, q_out=q_out)
    assert_device_ok()
    qo, ko, vo = okv.split_qkv(qkv.float().cpu().numpy(), H)
    p = np.arange(30, 30 + S)
    np.testing.assert_array_equal(q_out.float().cpu().numpy(), okv.rope(qo, p, sin.numpy(), cos.numpy(), "bf16"))
    np.testing.assert_array_equal(kc[:, :, 20:36].float().cpu().numpy(), okv.rope(ko, p, sin.numpy(), cos.numpy(), "bf16"))
    np.testing.assert_array_equal(vc[:, :, 20:36].float().cpu().numpy(), vo)


def test_device_position_outside_table_sets_status():
    """A position past the table (the reference raises IndexError) writes nothing for that
    token and raises device status bit 4; the other tokens are written."""
    from bd3attn import ops
    gen = torch.Generator().manual_seed(4)
    B, S, H, D = 1, 4, 2, 64
    sin, cos = _tables(D, 16)
    _, qkv = _qkv(gen, B, S, H, D, "bf16")
    kc = torch.full((B, H, 8, D), 7.0, dtype=torch.bfloat16, device="cuda")
    vc = kc.clone()
    pos = torch.tensor([0, 1, 16, 3], device="cuda")
    ops.qkv_rope_cache_raw(qkv, H, cos.cuda(), sin.cuda(), kc, vc, 0, positions=pos)
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 4
    assert torch.all(kc[:, :, 2].float() == 7.0) and torch.all(vc[:, :, 2].float() == 7.0)
    _, ko, _ = okv.split_qkv(qkv.float().cpu().numpy(), H)
    k_ref = okv.rope(ko[:, :, [0, 1, 3]], np.array([0, 1, 3]), sin.numpy(), cos.numpy(), "bf16")
    np.testing.assert_array_equal(kc[:, :, [0, 1, 3]].float().cpu().numpy(), k_ref)


@pytest.mark.parametrize("capacity", [None, 96])
def test_cached_sampling_sequence_matches_reference(capacity):
    """Prefill 32 tokens (store), two denoising steps of a 16-token block (no store), then
    commit the block (store), in two layers: q, k_all, v_all equal the reference's
    rope + torch.cat + append flow at every call."""
    from bd3attn.kv_cache import KVCache
    gen = torch.Generator().manual_seed(5)
    B, H, D, L = 2, 3, 64, 2
    sin, cos = _tables(D, 128)
    ours, ref = KVCache.empty(L, capacity=capacity), okv.ConcatKVCache(L)
    plan = [(0, 32, True), (32, 16, False), (32, 16, False), (32, 16, True), (48, 16, False)]
    for start, S, store in plan:
        pos = torch.arange(start, start + S)
        for layer in range(L):
            qkv, qkv_d = _qkv(gen, B, S, H, D, "bf16")
            q, k_all, v_all = ours.rope_qkv(layer, qkv_d, H, cos.cuda(), sin.cuda(),
                                            pos.cuda(), store)
            rq, rk, rv = okv.cached_qkv(ref, layer, qkv.float().numpy(), H, pos.numpy(),
                                        sin.numpy(), cos.numpy(), "bf16", store)
            np.testing.assert_array_equal(q.float().cpu().numpy(), rq)
            np.testing.assert_array_equal(k_all.float().cpu().numpy(), rk)
            np.testing.assert_array_equal(v_all.float().cpu().numpy(), rv)
        assert ours.length == ref.length
    assert_device_ok()


def _reference_like_modules():
    """A stand-in for the reference's model.modules with the attention forward of
    model/modules.py:368-422 (fused QKV Linear, RoPE, cache concatenation, attention,
    output projection), for checking that install() leaves its results unchanged."""
    ns = types.SimpleNamespace()

    def sdpa(q, k, v, mask=None):
        s = (q.float() @ k.float().transpose(-1, -2)) / q.shape[-1] ** 0.5
        if mask is not None:
            s = s.masked_fill(~mask, float("-inf"))
        return (torch.softmax(s, dim=-1) @ v.float()).to(q.dtype)

    class Rope:
        def __init__(self, D, max_pos):
            sin, cos = _tables(D, max_pos)
            self.sin_table, self.cos_table = sin.cuda(), cos.cuda()

        def __call__(self, x, positions):
            sin = self.sin_table[positions].to(x.dtype)
            cos = self.cos_table[positions].to(x.dtype)
            x1, x2 = x.chunk(2, dim=-1)
            return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)

    class ConcatCache:
        def __init__(self, n):
            self.k, self.v = [None] * n, [None] * n

        def get(self, i):
            return self.k[i], self.v[i]

        def append(self, i, k, v):
            if self.k[i] is None:
                self.k[i], self.v[i] = k, v
            else:
                self.k[i] = torch.cat([self.k[i], k], dim=-2)
                self.v[i] = torch.cat([self.v[i], v], dim=-2)

    class Attention(torch.nn.Module):
        def __init__(self, d_model, n_heads, rope):
            super().__init__()
            self.n_heads, self.rope = n_heads, rope
            self.qkv = torch.nn.Linear(d_model, 3 * d_model, bias=False)
            self.out = torch.nn.Linear(d_model, d_model, bias=False)

        def forward(self, x, mask=None, positions=None, kv_cache=None, layer_idx=0, store=False):
            B, S, _ = x.shape
            q, k, v = self.qkv(x).view(B, S, 3, self.n_heads, -1).permute(2, 0, 3, 1, 4)
            q, k = self.rope(q, positions), self.rope(k, positions)
            k_all, v_all = k, v
            if kv_cache is not None:
                kc, vc = kv_cache.get(layer_idx)
                if kc is not None:
                    k_all, v_all = torch.cat([kc, k], dim=-2), torch.cat([vc, v], dim=-2)
            if store and kv_cache is not None:
                kv_cache.append(layer_idx, k, v)
            o = ns.scaled_dot_product_attention(q, k_all, v_all, mask)
            return self.out(o.transpose(1, 2).reshape(B, S, -1))

    ns.scaled_dot_product_attention = sdpa
    ns.BidirectionalMultiHeadAttention = Attention
    ns.ConcatCache = ConcatCache
    ns.Rope = Rope
    return ns


def test_install_routes_cached_attention_bit_exact():
    from bd3attn.kv_cache import KVCache, install
    ns = _reference_like_modules()
    torch.manual_seed(6)
    attn = ns.BidirectionalMultiHeadAttention(192, 3, ns.Rope(64, 64)).cuda().bfloat16()
    gen = torch.Generator().manual_seed(7)
    xs = [(torch.randn(2, 16, 192, generator=gen).bfloat16().cuda(), s) for s in (0, 16, 16, 32)]
    stores = [True, False, True, False]
    ref_cache = ns.ConcatCache(1)
    ref_out = [attn(x, positions=torch.arange(s, s + 16, device="cuda"), kv_cache=ref_cache,
                    store=st) for (x, s), st in zip(xs, stores)]
    install(ns)
    install(ns)  # idempotent
    ours = KVCache.empty(1)
    our_out = [attn(x, positions=torch.arange(s, s + 16, device="cuda"), kv_cache=ours, store=st)
               for (x, s), st in zip(xs, stores)]
    assert_device_ok()
    # the cached K/V are bit-identical; the outputs go through the same attention and output
    # projection (matmuls on differently laid out q: equal up to accumulation order)
    assert ours.length == 32
    for got, want in zip(ours.get(0), ref_cache.get(0)):
        assert torch.equal(got, want)
    for a, b in zip(ref_out, our_out):
        assert (a.float() - b.float()).abs().max().item() <= 2e-2
    # any other cache still runs the original forward
    other = ns.ConcatCache(1)
    again = [attn(x, positions=torch.arange(s, s + 16, device="cuda"), kv_cache=other, store=st)
             for (x, s), st in zip(xs, stores)]
    for a, b in zip(ref_out, again):
        assert torch.equal(a, b)
