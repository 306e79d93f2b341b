"""The sampler-step oracle against the reference's own outputs (tests/golden/golden_sampler.npz),
Philox4x32-10 against its published known-answer vectors, and the argument checks of
bd3_subs_sample (rejected before any CUDA call). No GPU needed."""

import os

import numpy as np
import pytest

from conftest import REPO
from oracle import sampler as osm

GOLDEN_S = os.path.join(REPO, "tests", "golden", "golden_sampler.npz")
CASES = [("f32", "f32"), ("bf16", "bf16"), ("f32_last", "f32")]


@pytest.fixture(scope="module")
def gs():
    with np.load(GOLDEN_S) as z:
        return {k: z[k] for k in z.files}


def test_philox_known_answers():
    """Random123's known-answer vectors for philox4x32-10."""
    kat = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
           ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF),
            (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
           ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
            (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in kat:
        got = osm.philox4x32_10(np.array(ctr, dtype=np.uint32), key)
        assert tuple(int(x) for x in got) == want


def test_row_uniforms_in_range_and_distinct():
    r = osm.row_uniforms(seed=123, offset=5, rows=4000)
    assert r.min() >= 0 and r.max() < 1 and len(np.unique(r)) == r.size
    assert abs(r.mean() - 0.5) < 0.02


def test_inverse_cdf_scan_and_walk():
    """The kernel's slice arithmetic: every target falls in the element whose cumulative
    range (in the kernel's order: thread t, its 8-entry chunks t, t + 512, ...) holds it,
    including zero-weight elements."""
    rng = np.random.default_rng(0)
    q = rng.random(5003)
    q[rng.random(5003) < 0.3] = 0.0
    order = [j for t in range(512) for j in osm.thread_order(5003, t)]
    assert sorted(order) == list(range(5003))
    assert order[:10] == [0, 1, 2, 3, 4, 5, 6, 7, 4096, 4097]
    cum = np.cumsum(q[order])
    for r in (0.0, 1e-9, 0.25, 0.5, 0.999999, 1 - 2 ** -53):
        j, margin = osm.inverse_cdf(q, r)
        k = int(np.searchsorted(cum, r * cum[-1], side="right"))
        k = min(k, len(order) - 1)
        while q[order[k]] == 0:  # a target at the very end lands on the last nonzero one
            k -= 1
        assert q[j] > 0
        if margin > 1e-12:
            assert j == order[k]


@pytest.mark.parametrize("tag,dt", CASES)
def test_subs_weights_match_reference(gs, tag, dt):
    mask = int(gs["mask_index"])
    t, s = gs[f"{tag}_ts"]
    masked = gs[f"{tag}_xt"] == mask
    q = osm.subs_weights(gs[f"{tag}_logits"], mask, t, s, dt)
    ref = gs[f"{tag}_q"]
    # the rows the step uses (masked tokens); the sum's order is the only difference
    np.testing.assert_allclose(q[masked], ref[masked], rtol=1e-5 if dt == "f32" else 1e-2,
                               atol=1e-30)
    if dt == "bf16":
        assert np.mean(q[masked] == ref[masked]) > 0.99


@pytest.mark.parametrize("tag,dt", CASES)
def test_subs_sample_oracle_matches_reference(gs, tag, dt):
    mask = int(gs["mask_index"])
    t, s = gs[f"{tag}_ts"]
    tokens, margin = osm.subs_sample(gs[f"{tag}_logits"], gs[f"{tag}_xt"], mask, t, s,
                                     gs[f"{tag}_u"], dt)
    decided = margin > 1e-5
    assert decided.mean() > 0.9
    np.testing.assert_array_equal(tokens[decided], gs[f"{tag}_next"][decided])


def _call(**over):
    """bd3_subs_sample with plausible arguments (fake non-null pointers: each case below is
    rejected before the library touches memory or CUDA)."""
    from bd3attn._lib import LIB, i64_array
    a = dict(logits=0x1000, B=2, S=4, V=100, xt=0x2000, mask=99, t=0.5, s=0.25, u=None,
             out=0x3000, dtype=2)
    a.update(over)
    return LIB.bd3_subs_sample(a["logits"], i64_array((a["S"] * a["V"], a["V"])), a["B"], a["S"],
                               a["V"], a["xt"], a["mask"], a["t"], a["s"], 1, 0, a["u"], a["out"],
                               a["dtype"], None)


def test_capi_sampler_argument_checks():
    from bd3attn._lib import BD3_ERR_INVALID, LIB
    assert _call(dtype=1) == BD3_ERR_INVALID          # fp16: the reference's SUBS raises
    assert "bf16 or fp32" in LIB.bd3_last_error().decode()
    assert _call(mask=100) == BD3_ERR_INVALID
    assert _call(mask=-1) == BD3_ERR_INVALID
    assert _call(t=0.0) == BD3_ERR_INVALID
    assert _call(V=1, mask=0) == BD3_ERR_INVALID
    assert _call(xt=None) == BD3_ERR_INVALID


def test_capi_sampler_device_args_checks():
    """bd3_subs_sample_dev: the same argument checks, and both device value pointers
    required (rejected before any CUDA call)."""
    from bd3attn._lib import BD3_ERR_INVALID, LIB, i64_array

    def call(ts=0x5000, rng=0x6000, dtype=2, mask=99):
        return LIB.bd3_subs_sample_dev(0x1000, i64_array((400, 100)), 2, 4, 100, 0x2000, mask,
                                       ts, rng, 0x3000, dtype, None)
    assert call(ts=None) == BD3_ERR_INVALID
    assert "ts (t, s)" in LIB.bd3_last_error().decode()
    assert call(rng=None) == BD3_ERR_INVALID
    assert call(dtype=1) == BD3_ERR_INVALID
    assert call(mask=100) == BD3_ERR_INVALID


@pytest.mark.parametrize("V", [1, 7, 8, 9, 4096, 4097, 50258])
def test_thread_order_partitions_the_row(V):
    """The kernel's element order visits every entry exactly once, in 8-entry chunks."""
    order = [j for t in range(512) for j in osm.thread_order(V, t)]
    assert sorted(order) == list(range(V))
    for t in (0, 1, 511):
        mine = osm.thread_order(V, t)
        assert all(j // 8 % 512 == t for j in mine)


def test_inverse_cdf_single_nonzero_weight():
    """A row with one nonzero weight draws it for every uniform, including the extremes."""
    q = np.zeros(1000)
    q[637] = 0.25
    for r in (0.0, 0.5, 1 - 2 ** -53):
        j, _ = osm.inverse_cdf(q, r)
        assert j == 637


def test_subs_weights_step_structure():
    """q at [MASK] is s/t; the others are exp(log-softmax) * (1 - s/t), summing to it."""
    rng = np.random.default_rng(2)
    logits = rng.standard_normal((3, 50)).astype(np.float32)
    t, s = 0.8, 0.3
    q = osm.subs_weights(logits, 49, t, s, "f32")
    assert np.allclose(q[:, 49], s / t)
    assert np.allclose(q[:, :49].sum(-1), 1 - s / t, rtol=1e-5)
