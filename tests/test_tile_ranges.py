"""Tile-skip coverage: the restated reference ranges, at the reference tiling and at the
tiling of the CUDA kernels, visit every nonzero of the mask and nothing is masked wrongly."""

import numpy as np
import pytest

import oracle
from oracle import tile_ranges as tr


def _fwd_cover(n, bs, bm, bn):
    mask = oracle.block_diff_mask(n, bs)
    seen = np.zeros_like(mask)
    for q0 in range(0, 2 * n, bm):
        q_idx = np.arange(q0, q0 + bm)[:, None]
        for s, rule, shift in tr.tiles(tr.fwd_ranges(q0, bm, bn, n, bs), bn):
            kv_idx = np.arange(s, s + bn)[None, :]
            m = tr.rule_mask(rule, shift, q_idx, kv_idx, n, bs)
            # an applied rule never admits a key the mask forbids
            assert not (m & ~mask[q0:q0 + bm, s:s + bn]).any(), (q0, s, rule)
            seen[q0:q0 + bm, s:s + bn] |= m
    return mask, seen


@pytest.mark.parametrize("n,bs", [(128, 4), (128, 16), (256, 16), (512, 64), (256, 256),
                                  (1024, 16), (1024, 4), (384, 128), (512, 32)])
@pytest.mark.parametrize("bm,bn", [(128, 64), (128, 128)])
def test_fwd_ranges_cover_mask(n, bs, bm, bn):
    mask, seen = _fwd_cover(n, bs, bm, bn)
    assert np.array_equal(seen, mask)


@pytest.mark.parametrize("n,bs", [(128, 4), (128, 16), (256, 16), (512, 64), (256, 256),
                                  (1024, 16), (384, 128), (512, 32)])
@pytest.mark.parametrize("bkv,bq", [(128, 32), (128, 64), (128, 128)])
def test_dkdv_ranges_cover_mask(n, bs, bkv, bq):
    mask = oracle.block_diff_mask(n, bs)
    seen = np.zeros_like(mask)
    for k0 in range(0, 2 * n, bkv):
        kv_idx = np.arange(k0, k0 + bkv)[None, :]
        for s, rule, shift in tr.tiles(tr.dkdv_ranges(k0, bkv, bq, n, bs), bq):
            q_idx = np.arange(s, s + bq)[:, None]
            m = tr.rule_mask(rule, shift, q_idx, kv_idx, n, bs)
            assert not (m & ~mask[s:s + bq, k0:k0 + bkv]).any(), (k0, s, rule)
            # each (query, key) pair is visited once: no double counting in dK/dV
            assert not (seen[s:s + bq, k0:k0 + bkv] & m).any(), (k0, s)
            seen[s:s + bq, k0:k0 + bkv] |= m
    assert np.array_equal(seen, mask)


@pytest.mark.parametrize("q_len,kv_len,bs", [(16, 16, 16), (16, 1040, 16), (40, 200, 16),
                                             (3088, 3088, 16), (64, 300, 16), (100, 1000, 64),
                                             (17, 129, 4)])
@pytest.mark.parametrize("bm,bn", [(16, 64), (64, 64), (128, 128)])
def test_decode_ranges_cover_mask(q_len, kv_len, bs, bm, bn):
    mask = oracle.block_causal_mask(q_len, kv_len, bs)
    seen = np.zeros_like(mask)
    for q0 in range(0, q_len, bm):
        q_idx = np.arange(q0, min(q0 + bm, q_len))[:, None]
        for s, rule, shift in tr.tiles(tr.decode_ranges(q0, bm, bn, q_len, kv_len, bs), bn):
            kv_idx = np.arange(s, min(s + bn, kv_len))[None, :]
            m = tr.rule_mask(rule, shift, q_idx, kv_idx, 0, bs, kv_len, q_len)
            assert not (m & ~mask[q_idx[:, 0]][:, kv_idx[0]]).any()
            seen[q0:q0 + q_idx.shape[0], s:s + kv_idx.shape[1]] |= m
    assert np.array_equal(seen, mask)


@pytest.mark.parametrize("q_len,kv_len,bs", [(16, 16, 16), (16, 1040, 16), (40, 200, 16),
                                             (64, 300, 16), (17, 129, 4)])
@pytest.mark.parametrize("split_n", [256, 1024])
def test_split_ranges_cover_mask(q_len, kv_len, bs, split_n):
    mask = oracle.block_causal_mask(q_len, kv_len, bs)
    seen = np.zeros_like(mask)
    q_idx = np.arange(q_len)[:, None]
    for sp in range(-(-kv_len // split_n)):
        for s, rule, shift in tr.tiles(tr.split_ranges(sp, split_n, 64, q_len, kv_len, bs), 64):
            kv_idx = np.arange(s, min(s + 64, kv_len))[None, :]
            m = tr.rule_mask(rule, shift, q_idx, kv_idx, 0, bs, kv_len, q_len)
            assert not (m & ~mask[:, kv_idx[0]]).any()
            seen[:, s:s + kv_idx.shape[1]] |= m
    assert np.array_equal(seen, mask)


def test_visited_fraction_n1024():
    """The reference tiling visits 31.25% of the (2n)^2 tiles at n=1024, bs=16, against a
    mask density of 25.39%; the 128x128 tiling here visits the same fraction."""
    n, bs = 1024, 16
    for bm, bn in ((128, 64), (128, 128)):
        visited = sum(len(tr.tiles(tr.fwd_ranges(q0, bm, bn, n, bs), bn)) * bm * bn
                      for q0 in range(0, 2 * n, bm))
        assert visited / (2 * n) ** 2 == pytest.approx(0.3125)
    assert oracle.block_diff_mask(n, bs).mean() == pytest.approx(0.25390625)
