"""bd3_subs_sample on the GPU: with the reference's own uniforms it reproduces the reference's
sampled tokens (tests/golden/golden_sampler.npz); its production draw (inverse CDF with one
Philox uniform per row) equals the oracle's replay of the same arithmetic; over many rows its
draws follow q / sum(q)."""

import os

import numpy as np
import pytest
import torch

from conftest import REPO
from gpu_util import assert_device_ok
from oracle import sampler as osm

pytestmark = pytest.mark.gpu

GOLDEN_S = os.path.join(REPO, "tests", "golden", "golden_sampler.npz")
DT = {"f32": torch.float32, "bf16": torch.bfloat16}


@pytest.fixture(scope="module")
def gs():
    with np.load(GOLDEN_S) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("tag,dt", [("f32", "f32"), ("bf16", "bf16"), ("f32_last", "f32")])
def test_replayed_uniforms_reproduce_reference_tokens(gs, tag, dt):
    from bd3attn.sampler import subs_sample_step
    mask = int(gs["mask_index"])
    t, s = gs[f"{tag}_ts"]
    logits = torch.from_numpy(gs[f"{tag}_logits"]).to(DT[dt]).cuda()
    xt = torch.from_numpy(gs[f"{tag}_xt"]).cuda()
    got = subs_sample_step(logits, xt, mask, t, s,
                           uniforms=torch.from_numpy(gs[f"{tag}_u"]).cuda())
    assert_device_ok()
    _, margin = osm.subs_sample(gs[f"{tag}_logits"], gs[f"{tag}_xt"], mask, t, s,
                                gs[f"{tag}_u"], dt)
    decided = margin > 1e-5
    assert decided.mean() > 0.9
    np.testing.assert_array_equal(got.cpu().numpy()[decided], gs[f"{tag}_next"][decided])
    # unmasked tokens are carried over
    keep = gs[f"{tag}_xt"] != mask
    np.testing.assert_array_equal(got.cpu().numpy()[keep], gs[f"{tag}_xt"][keep])


@pytest.mark.parametrize("dt,V,B,S", [("bf16", 50258, 2, 16), ("f32", 50258, 1, 16),
                                      ("f32", 1001, 3, 5),
                                      ("bf16", 1001, 3, 5),   # rows at every 2-byte offset
                                      ("bf16", 9, 2, 4)])     # two chunks, one entry in the last
def test_philox_draw_equals_oracle(dt, V, B, S):
    """The production draw (inverse CDF, one Philox uniform per row) equals the oracle's
    replay of the same arithmetic wherever rounding cannot decide it."""
    from bd3attn.sampler import subs_sample_step
    g = torch.Generator().manual_seed(V + B)
    mask = V - 1
    logits = (2 * torch.randn(B, S, V, generator=g)).to(DT[dt])
    xt = torch.randint(0, V - 1, (B, S), generator=g)
    xt[torch.rand(B, S, generator=g) < 0.7] = mask
    seed = int(torch.randint(0, 2 ** 63 - 1, (1,), generator=torch.Generator().manual_seed(99)).item())
    t, s = 0.625, 0.5
    got = subs_sample_step(logits.cuda(), xt.cuda(), mask, t, s,
                           generator=torch.Generator().manual_seed(99), offset=3)
    assert_device_ok()
    want, margin = osm.subs_sample_philox(logits.float().numpy(), xt.numpy(), mask, t, s, seed, 3, dt)
    decided = margin > 1e-6
    assert decided.mean() > 0.9
    np.testing.assert_array_equal(got.cpu().numpy()[decided], want[decided])


def test_draws_follow_the_step_distribution():
    """4096 masked rows of one fixed 8-token distribution: the sampled frequencies match
    q / sum(q) (chi-square, 7 degrees of freedom)."""
    from bd3attn.sampler import subs_sample_step
    V, rows = 8, 4096
    mask = V - 1
    logits_row = torch.tensor([0.0, 1.0, -1.0, 2.0, 0.5, -0.5, 1.5, 3.0])
    logits = logits_row.expand(1, rows, V).contiguous().cuda()
    xt = torch.full((1, rows), mask, dtype=torch.int64, device="cuda")
    t, s = 0.5, 0.25
    got = subs_sample_step(logits, xt, mask, t, s, generator=torch.Generator().manual_seed(5))
    assert_device_ok()
    q = osm.subs_weights(logits_row.numpy()[None], mask, t, s, "f32")[0]
    p = q / q.sum()
    counts = np.bincount(got.cpu().numpy().ravel(), minlength=V)
    chi2 = float(((counts - rows * p) ** 2 / (rows * p)).sum())
    assert chi2 < 30.0, (chi2, counts, rows * p)  # P(chi2_7 > 30) < 1e-4


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_strided_logits_and_in_place_update(dt):
    """Logits as a slice of the backbone's (batch, seq, vocab) output, and out aliasing xt."""
    from bd3attn.sampler import subs_sample_step
    g = torch.Generator().manual_seed(8)
    V, mask = 777, 776
    full = torch.randn(2, 20, V, generator=g).to(dt).cuda()
    logits = full[:, -16:]  # model/bd3lm.py:164 takes the block's last positions
    xt = torch.randint(0, V - 1, (2, 16), generator=g)
    xt[:, ::2] = mask
    xt_d = xt.cuda()
    u = torch.rand(2, 16, V, dtype=torch.float64, generator=g)
    want = subs_sample_step(logits.contiguous(), xt_d.clone(), mask, 0.5, 0.25, uniforms=u.cuda())
    got = subs_sample_step(logits, xt_d, mask, 0.5, 0.25, uniforms=u.cuda(), out=xt_d)
    assert_device_ok()
    assert got.data_ptr() == xt_d.data_ptr()
    assert torch.equal(got, want)
    assert torch.equal(got[:, 1::2].cpu(), xt[:, 1::2])
