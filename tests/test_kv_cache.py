"""The RoPE / KV-cache oracle against the reference's own outputs (tests/golden/golden_kv.npz),
the in-place KVCache's host logic against the reference's concatenating one, and the
argument checks of bd3_qkv_rope_cache (they return before any CUDA call). No GPU needed."""

import os

import numpy as np
import pytest
import torch

from conftest import REPO
from oracle import kv_cache as okv

GOLDEN_KV = os.path.join(REPO, "tests", "golden", "golden_kv.npz")


@pytest.fixture(scope="module")
def gkv():
    with np.load(GOLDEN_KV) as z:
        return {k: z[k] for k in z.files}


def test_rope_tables_match_reference(gkv):
    sin, cos = okv.rope_tables(64, 64)
    ulp = np.spacing(np.abs(gkv["rope_sin"]).astype(np.float32))
    assert np.all(np.abs(sin - gkv["rope_sin"]) <= ulp)
    assert np.all(np.abs(cos - gkv["rope_cos"]) <= np.spacing(np.abs(gkv["rope_cos"])))


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_rope_oracle_bit_exact_vs_reference(gkv, dt):
    y = okv.rope(gkv[f"rope_{dt}_x"], gkv[f"rope_{dt}_pos"], gkv["rope_sin"], gkv["rope_cos"], dt)
    np.testing.assert_array_equal(y, gkv[f"rope_{dt}_y"])


def test_round_to_bf16_ties_to_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0], dtype=np.float32)
    np.testing.assert_array_equal(okv.round_to(x, "bf16"),
                                  torch.from_numpy(x).bfloat16().float().numpy())


def _append_sequence(gkv, cache):
    for i in range(3):
        for layer in range(2):
            cache.append(layer, gkv[f"kv_append{i}_l{layer}_k"], gkv[f"kv_append{i}_l{layer}_v"])


def test_concat_cache_oracle_matches_reference(gkv):
    c = okv.ConcatKVCache(2)
    assert c.length == 0 and c.get(0) == (None, None)
    _append_sequence(gkv, c)
    assert c.length == int(gkv["kv_length"])
    for layer in range(2):
        np.testing.assert_array_equal(c.get(layer)[0], gkv[f"kv_final_l{layer}_k"])
        np.testing.assert_array_equal(c.get(layer)[1], gkv[f"kv_final_l{layer}_v"])


@pytest.mark.parametrize("capacity", [None, 6, 4096])
def test_inplace_cache_matches_reference(gkv, capacity):
    from bd3attn.kv_cache import KVCache
    c = KVCache.empty(2, capacity=capacity)
    assert c.length == 0 and c.get(1) == (None, None) and c.k == [None, None]
    for i in range(3):
        for layer in range(2):
            c.append(layer, torch.from_numpy(gkv[f"kv_append{i}_l{layer}_k"]),
                     torch.from_numpy(gkv[f"kv_append{i}_l{layer}_v"]))
    assert c.length == int(gkv["kv_length"])
    for layer in range(2):
        k, v = c.get(layer)
        np.testing.assert_array_equal(k.numpy(), gkv[f"kv_final_l{layer}_k"])
        np.testing.assert_array_equal(v.numpy(), gkv[f"kv_final_l{layer}_v"])
        assert c.k[layer].shape == k.shape
    # views of one storage: no copy per get
    assert c.get(0)[0].data_ptr() == c.get(0)[0].data_ptr()


def test_inplace_cache_growth_keeps_rows():
    from bd3attn.kv_cache import KVCache
    g = torch.Generator().manual_seed(0)
    c = KVCache.empty(1)
    ref = okv.ConcatKVCache(1)
    for s in (200, 100, 300, 7):  # crosses the first 256-row allocation and a doubling
        k, v = torch.randn(1, 2, s, 8, generator=g), torch.randn(1, 2, s, 8, generator=g)
        c.append(0, k, v)
        ref.append(0, k.numpy(), v.numpy())
        np.testing.assert_array_equal(c.get(0)[0].numpy(), ref.get(0)[0])
        np.testing.assert_array_equal(c.get(0)[1].numpy(), ref.get(0)[1])


def test_inplace_cache_errors():
    from bd3attn.kv_cache import KVCache
    c = KVCache.empty(1, capacity=4)
    c.append(0, torch.zeros(1, 2, 3, 8), torch.zeros(1, 2, 3, 8))
    with pytest.raises(RuntimeError):  # capacity
        c.append(0, torch.zeros(1, 2, 2, 8), torch.zeros(1, 2, 2, 8))
    with pytest.raises(RuntimeError):  # shape mismatch (torch.cat would refuse it too)
        c.append(0, torch.zeros(1, 3, 1, 8), torch.zeros(1, 3, 1, 8))
    with pytest.raises(ValueError):
        KVCache.empty(0)


def _call(**over):
    """bd3_qkv_rope_cache with plausible arguments (fake non-null pointers: every case below
    is rejected before the library touches memory or CUDA)."""
    from bd3attn._lib import LIB, i64_array
    a = dict(qkv=0x1000, B=1, S=4, H=2, D=64, positions=None, pos0=0, cos=0x2000, sin=0x3000,
             max_pos=64, q=0x4000, k=0x5000, v=0x6000, row0=0, rows=16, dtype=0)
    a.update(over)
    return LIB.bd3_qkv_rope_cache(
        a["qkv"], i64_array((a["S"] * 3 * a["H"] * a["D"], 3 * a["H"] * a["D"])), a["B"], a["S"],
        a["H"], a["D"], a["positions"], a["pos0"], a["cos"], a["sin"], a["max_pos"], a["q"],
        a["k"], a["v"], i64_array([0] * 9), a["row0"], a["rows"], a["dtype"], None)


def test_capi_rope_cache_argument_checks():
    from bd3attn._lib import BD3_ERR_INVALID, BD3_ERR_UNSUPPORTED, LIB
    assert _call(D=60) == BD3_ERR_UNSUPPORTED
    assert _call(dtype=7) == BD3_ERR_INVALID
    assert _call(S=0) == BD3_ERR_INVALID
    assert _call(cos=None) == BD3_ERR_INVALID
    assert _call(k=None) == BD3_ERR_INVALID
    assert _call(pos0=61) == BD3_ERR_INVALID        # 61 + 4 > 64: outside the RoPE table
    assert _call(pos0=-1) == BD3_ERR_INVALID
    assert _call(row0=13) == BD3_ERR_INVALID        # rows [13, 17) outside 16
    assert "cache rows" in LIB.bd3_last_error().decode()
    assert _call(row0=-1) == BD3_ERR_INVALID        # rows from positions[0], but no positions
    assert "positions is required" in LIB.bd3_last_error().decode()
    assert _call(row0=-1, positions=0x7000, S=17) == BD3_ERR_INVALID  # S > cache rows
