"""The stand-in training backbone and its generation loops, on the CPU: the attention
router's names and errors, that every layer calls the routed function with the (2n, 2n)
mask, that the backbone's mask is the reference's block_diff_mask, and that the
reference-flow generators (the comparison arms of the generation benchmark) run."""

import numpy as np
import pytest
import torch

import oracle


def test_router_names_and_errors():
    from workloads import backbone as bb
    assert bb.ROUTES == ("bsfa", "bsdfa", "split_kv", "sdpa")
    with pytest.raises(ValueError):
        bb.use_attention("nope")
    for name in ("bsfa", "bsdfa", "split_kv"):
        with pytest.raises(ValueError):
            bb.use_attention(name)  # needs a block size
    bb.use_attention("bsfa", block_size=16)
    assert callable(bb.ATTENTION.scaled_dot_product_attention)


@pytest.mark.parametrize("n,bs", [(64, 4), (128, 16), (256, 256), (96, 32)])
def test_backbone_mask_is_block_diff_mask(n, bs):
    from workloads.backbone import block_diff_mask
    np.testing.assert_array_equal(block_diff_mask(n, bs).numpy(),
                                  np.asarray(oracle.block_diff_mask(n, bs)))


def test_backbone_routes_attention_and_trains_on_cpu(monkeypatch):
    """With PyTorch's attention routed in, the stand-in backbone runs forward and backward
    on the CPU; a counting wrapper shows every layer calls the routed function with the
    (2n, 2n) mask."""
    from workloads import backbone as bb
    bb.use_attention("sdpa")
    sdpa = bb.ATTENTION.scaled_dot_product_attention
    calls = []

    def counting(q, k, v, mask):
        calls.append(tuple(mask.shape))
        return sdpa(q, k, v, mask)

    monkeypatch.setattr(bb.ATTENTION, "scaled_dot_product_attention", counting)
    torch.manual_seed(0)
    model = bb.Backbone(64, 32, 8, d_model=64, n_heads=1, n_layers=2, d_ff=128)
    xt, x0 = bb.noisy_batch(torch.Generator().manual_seed(1), 2, 32, 8, 64)
    loss = model.loss(xt, x0)
    loss.backward()
    assert calls == [(64, 64), (64, 64)]
    assert torch.isfinite(loss) and model.layers[0].qkv.weight.grad is not None


def test_reference_generation_flows_run_on_cpu():
    """The reference-flow generators run on the CPU with a tiny backbone: every generated
    token is a real token."""
    from workloads.backbone import Backbone
    from workloads.generation import MDLMGeneration, ReferenceGeneration, subs_log_probs
    torch.manual_seed(0)
    model = Backbone(100, 32, 8, d_model=64, n_heads=1, n_layers=1, d_ff=128).eval()
    ref = ReferenceGeneration(model, 2, 3, 4, generator=torch.Generator().manual_seed(1))
    out = ref.run()
    assert out.shape == (2, 24) and bool(((out >= 0) & (out < 99)).all())
    out = MDLMGeneration(model, 2, 32, steps=4, use_library=False).run()
    assert out.shape == (2, 32) and bool(((out >= 0) & (out < 99)).all())
    # SUBS: [MASK] gets no mass; unmasked rows are one-hot at their token
    logits = torch.randn(1, 2, 100)
    lp = subs_log_probs(logits, torch.tensor([[99, 5]]), 99)
    assert lp[0, 0, 99] < -1e5 and torch.allclose(lp[0, 0].exp().sum(), torch.tensor(1.0))
    assert lp[0, 1, 5] == 0 and bool((lp[0, 1, torch.arange(100) != 5] == -1e6).all())
