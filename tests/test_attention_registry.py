"""The attention backend registry (drop-in for the reference's bench/attention.py) and the
stand-in training backbone, on the CPU: the registry's names and errors, that
install_attention routes a layer's attention call, that the package merges with another
``bench`` directory on the path, and that the backbone's mask is the reference's."""

import os
import sys
import types

import numpy as np
import pytest
import torch

import oracle


def test_registry_names_and_errors():
    from bench import attention as ba
    assert {"sdpa", "flex", "bsfa", "bsdfa", "split_kv"} <= set(ba.BACKENDS)
    assert ba.BLOCK_SIZE_BACKENDS == ("bsfa", "bsdfa", "split_kv")
    ns = types.SimpleNamespace(scaled_dot_product_attention=None)
    with pytest.raises(KeyError):
        ba.install_attention("nope", modules=ns)
    with pytest.raises(AssertionError):
        ba.install_attention("bsfa", modules=ns)  # needs block_size
    ba.install_attention("bsfa", block_size=16, modules=ns)
    fn = ns.scaled_dot_product_attention
    assert fn.func is ba.bsfa and fn.keywords == {"block_size": 16}
    ba.install_attention("sdpa", nvtx=True, modules=ns)
    assert ns.scaled_dot_product_attention is not ba.torch_sdpa  # wrapped in NVTX ranges


def test_bench_package_merges_with_other_bench_dirs(tmp_path):
    other = tmp_path / "bench"
    other.mkdir()
    (other / "extra_tool.py").write_text("VALUE = 7\n")
    sys.path.append(str(tmp_path))
    try:
        import importlib
        import bench
        importlib.reload(bench)  # re-extend __path__ with the new directory
        from bench import extra_tool
        assert extra_tool.VALUE == 7
        from bench import attention
        assert os.path.dirname(attention.__file__).endswith(os.path.join("diffusion-llm_b200", "bench"))
    finally:
        sys.path.remove(str(tmp_path))
        sys.modules.pop("bench.extra_tool", None)


@pytest.mark.parametrize("n,bs", [(64, 4), (128, 16), (256, 256), (96, 32)])
def test_backbone_mask_is_block_diff_mask(n, bs):
    from bench.backbone import block_diff_mask
    np.testing.assert_array_equal(block_diff_mask(n, bs).numpy(),
                                  np.asarray(oracle.block_diff_mask(n, bs)))


def test_backbone_routes_attention_and_trains_on_cpu():
    """With the registry's "sdpa" backend the stand-in backbone runs forward and backward on
    the CPU; a counting wrapper shows every layer calls the installed function with the
    (2n, 2n) mask."""
    from bench import attention as ba
    from bench import backbone as bb
    calls = []

    def counting(q, k, v, mask=None):
        calls.append(tuple(mask.shape))
        return ba.torch_sdpa(q, k, v, mask)

    ba.BACKENDS["counting"] = counting
    try:
        ba.install_attention("counting", modules=bb.ATTENTION)
        torch.manual_seed(0)
        model = bb.Backbone(64, 32, 8, d_model=64, n_heads=1, n_layers=2, d_ff=128)
        xt, x0 = bb.noisy_batch(torch.Generator().manual_seed(1), 2, 32, 8, 64)
        loss = model.loss(xt, x0)
        loss.backward()
    finally:
        del ba.BACKENDS["counting"]
    assert calls == [(64, 64), (64, 64)]
    assert torch.isfinite(loss) and model.layers[0].qkv.weight.grad is not None


def test_reference_generation_flows_run_on_cpu():
    """The reference-flow generators (the comparison arms of the generation benchmark) run
    on the CPU with a tiny backbone: every generated token is a real token."""
    from bench.backbone import Backbone
    from bench.generation import MDLMGeneration, ReferenceGeneration, subs_log_probs
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
