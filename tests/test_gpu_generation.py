"""BD3-LM generation on the library (workloads/generation.py) with a small stand-in backbone:
one CUDA graph replay per block gives the same tokens as the same loop run eagerly; every
generated token is a real token; and the cached forward over the committed blocks gives the
logits of a full re-encode of the sequence under the block-causal mask (the reference's
uncached block_logprobs, model/bd3lm.py:142-172), block after block."""

import pytest
import torch

from gpu_util import assert_device_ok

pytestmark = pytest.mark.gpu

V, BS, B, N_BLOCKS, STEPS = 1000, 16, 4, 4, 4
CFG = dict(d_model=128, n_heads=2, n_layers=2, d_ff=256)


@pytest.fixture(scope="module")
def model():
    from workloads.backbone import Backbone
    torch.manual_seed(0)
    return Backbone(V, BS * N_BLOCKS, BS, **CFG).cuda().bfloat16().eval()


def test_graph_replay_equals_eager_and_tokens_are_real(model):
    from workloads.generation import CachedGeneration
    got = CachedGeneration(model, B, N_BLOCKS, STEPS, seed=7).run().clone()
    again = CachedGeneration(model, B, N_BLOCKS, STEPS, seed=7, use_graph=False).run()
    assert_device_ok()
    assert torch.equal(got, again)
    assert got.shape == (B, BS * N_BLOCKS)
    assert bool(((got >= 0) & (got < V - 1)).all())  # no [MASK] left, nothing out of range
    other = CachedGeneration(model, B, N_BLOCKS, STEPS, seed=8).run()
    assert not torch.equal(got, other)  # the seed reaches the draw


def test_cached_forward_matches_full_reencode(model):
    from workloads import backbone as bb
    from workloads.generation import CachedGeneration
    bb.use_attention("sdpa")
    gen = CachedGeneration(model, B, N_BLOCKS, STEPS, seed=3, use_graph=False)
    tokens = gen.run().clone()
    gen._reset()  # teacher-forced pass over the generated tokens
    with torch.no_grad():
        for b in range(N_BLOCKS):
            gen.block.copy_(tokens[:, b * BS:(b + 1) * BS])
            cached = gen.forward_block().float()
            gen.pos += BS
            gen.kv_len += BS
            n = (b + 1) * BS
            idx = torch.arange(n, device="cuda")
            mask = (idx[None, :] // BS) <= (idx[:, None] // BS)  # block-causal
            full = model.encode(tokens[:, :n], mask, gen.cos[:n], gen.sin[:n])[:, -BS:].float()
            err = (cached - full).abs().max().item()
            assert err <= 0.03 * max(1.0, full.abs().max().item()), (b, err)
    assert_device_ok()


def test_reference_flow_runs(model):
    from workloads.generation import ReferenceGeneration
    out = ReferenceGeneration(model, B, 2, STEPS, generator=torch.Generator(device="cuda").manual_seed(1)).run()
    assert out.shape == (B, 2 * BS) and bool(((out >= 0) & (out < V - 1)).all())


def test_mdlm_variant(model):
    """The MDLM loop (whole-sequence block, no cache): with the library's prefill attention
    the per-step logits equal PyTorch attention's within bf16 tolerance, and every token is
    unmasked at the end."""
    from workloads import backbone as bb
    from workloads.generation import MDLMGeneration
    L = 128
    out = MDLMGeneration(model, 2, L, steps=8, seed=5).run()
    assert_device_ok()
    assert out.shape == (2, L) and bool(((out >= 0) & (out < V - 1)).all())
    x = out.clone()
    x[:, ::3] = V - 1  # a partly masked sequence
    gen = MDLMGeneration(model, 2, L, steps=1)
    with torch.no_grad():
        bb.use_attention("bsdfa", block_size=L)
        ours = model.encode(x, None, gen.cos, gen.sin).float()
        bb.use_attention("sdpa")
        ref = model.encode(x, None, gen.cos, gen.sin).float()
    err = (ours - ref).abs().max().item()
    assert err <= 0.03 * max(1.0, ref.abs().max().item()), err
    ref_out = MDLMGeneration(model, 2, L, steps=8, use_library=False, seed=5).run()
    assert bool(((ref_out >= 0) & (ref_out < V - 1)).all())
