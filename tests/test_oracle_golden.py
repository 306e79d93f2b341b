"""Pin the CPU oracle against golden vectors produced by the reference itself."""

import numpy as np
import pytest
import torch

import oracle
from conftest import bf16_from_bits


def _cases(golden, prefix):
    return sorted({k.rsplit("_", 1)[0] for k in golden if k.startswith(prefix)})


def test_block_diff_mask_matches_reference(golden):
    keys = [k for k in golden if k.startswith("mask_")]
    assert keys
    for key in keys:
        _, n, bs = key.split("_")
        n, bs = int(n[1:]), int(bs[2:])
        ref = np.unpackbits(golden[key], axis=-1)[:, : 2 * n].astype(bool)
        mine = oracle.block_diff_mask(n, bs)
        assert np.array_equal(mine, ref), key
        # nnz = n^2 + n*bs when bs divides n
        if n % bs == 0:
            assert int(mine.sum()) == n * n + n * bs


@pytest.mark.parametrize("bs", [4, 16, 128])
def test_training_attention_matches_reference(golden, bs):
    tag = f"train_n128_bs{bs}"
    q, k, v, do = (bf16_from_bits(golden[f"{tag}_{x}"]).float() for x in ("q", "k", "v", "do"))
    mask = oracle.block_diff_mask(128, bs)
    o, lse = oracle.attention(q, k, v, mask)
    np.testing.assert_allclose(o.numpy(), golden[f"{tag}_o"], atol=2e-5, rtol=1e-4)
    dq, dk, dv = oracle.attention_grads(q, k, v, do, mask)
    for name, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(t.numpy(), golden[f"{tag}_{name}"], atol=5e-5, rtol=1e-4)
    # LSE is finite everywhere: every query sees at least its own block
    assert torch.isfinite(lse).all()


def test_decode_attention_matches_reference(golden):
    tags = _cases(golden, "decode_")
    assert len(tags) >= 5
    for tag in tags:
        _, ql, kvl, bs = tag.split("_")
        q_len, kv_len, bs = int(ql[1:]), int(kvl[2:]), int(bs[2:])
        q, k, v = (bf16_from_bits(golden[f"{tag}_{x}"]).float() for x in ("q", "k", "v"))
        mask = oracle.block_causal_mask(q_len, kv_len, bs)
        o, _ = oracle.attention(q, k, v, mask)
        np.testing.assert_allclose(o.numpy(), golden[f"{tag}_o"], atol=2e-5, rtol=1e-4,
                                   err_msg=tag)


def test_live_block_decode_matches_reference(golden):
    q, k, v = (bf16_from_bits(golden[f"live_{x}"]).float() for x in ("q", "k", "v"))
    live = golden["live_blocks"].tolist()
    B, H, q_len, _ = q.shape
    kv_len = k.shape[2]
    mask = oracle.live_block_mask(live, q_len, kv_len, 64, 16)
    o, _ = oracle.attention(q, k, v, mask)
    np.testing.assert_allclose(o.numpy(), golden["live_o"], atol=2e-5, rtol=1e-4)


def test_lse_merge_equals_full_attention():
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 3, 16, 64, generator=g)
    k = torch.randn(2, 3, 300, 64, generator=g)
    v = torch.randn(2, 3, 300, 64, generator=g)
    full, full_lse = oracle.attention(q, k, v)
    parts, lses = [], []
    for lo in range(0, 300, 64):
        o, l = oracle.attention(q, k[:, :, lo:lo + 64], v[:, :, lo:lo + 64])
        parts.append(o)
        lses.append(l)
    merged, merged_lse = oracle.lse_merge(torch.stack(parts), torch.stack(lses))
    torch.testing.assert_close(merged, full, atol=1e-12, rtol=1e-12)
    torch.testing.assert_close(merged_lse, full_lse, atol=1e-12, rtol=1e-12)
