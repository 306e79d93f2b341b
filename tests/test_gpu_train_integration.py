"""The training backward inside a real loss: the stand-in BD3-LM backbone (the reference's
attention call site, 2n input, block diffusion mask) trained with the "bsfa" backend (the
sm_100a kernels) and, from the same initial weights and batches, with the "sdpa" backend
(PyTorch's attention given the boolean mask). The first step's parameter gradients agree,
and so do the loss curves over 30 AdamW steps."""

import copy

import pytest
import torch

from gpu_util import assert_device_ok

pytestmark = pytest.mark.gpu

V, N, BS, BATCH = 1024, 256, 16, 4
CFG = dict(d_model=128, n_heads=2, n_layers=2, d_ff=512)


def _models():
    from workloads.backbone import Backbone
    torch.manual_seed(0)
    a = Backbone(V, N, BS, **CFG).cuda()
    return a, copy.deepcopy(a)


def _use(name):
    from workloads import backbone as bb
    bb.use_attention(name, block_size=BS)


def test_first_step_gradients_agree():
    from workloads.backbone import noisy_batch
    ours, ref = _models()
    xt, x0 = (t.cuda() for t in noisy_batch(torch.Generator().manual_seed(1), BATCH, N, BS, V,
                                              repeat_blocks=True, n_tokens=64))
    grads = []
    for name, model in (("bsfa", ours), ("sdpa", ref)):
        _use(name)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            loss = model.loss(xt, x0)
        loss.backward()
        grads.append({k: p.grad.float() for k, p in model.named_parameters()})
    assert_device_ok()
    for k, g_ref in grads[1].items():
        g = grads[0][k]
        rel = ((g - g_ref).norm() / g_ref.norm().clamp_min(1e-12)).item()
        assert rel < 3e-2, f"{k}: relative gradient difference {rel:.3e}"


def test_loss_curves_agree_over_training():
    from workloads.backbone import noisy_batch, train_step
    ours, ref = _models()
    gen = torch.Generator().manual_seed(2)
    batches = [tuple(t.cuda() for t in noisy_batch(gen, BATCH, N, BS, V, repeat_blocks=True,
                                                   n_tokens=64))
               for _ in range(30)]
    curves = []
    for name, model in (("bsfa", ours), ("sdpa", ref)):
        _use(name)
        opt = torch.optim.AdamW(model.parameters(), lr=2e-3, betas=(0.9, 0.999),
                                weight_decay=0.0)
        curves.append(torch.stack([train_step(model, opt, xt, x0) for xt, x0 in batches]).cpu())
    assert_device_ok()
    a, b = curves
    assert torch.isfinite(a).all() and torch.isfinite(b).all()
    assert (a[:5] - b[:5]).abs().max().item() < 0.02, (a, b)
    assert (a - b).abs().max().item() < 0.05 * b[0].item(), (a, b)
    assert a[-5:].mean() < a[:5].mean() - 1.0  # training makes progress (7.3 -> ~4 on CPU)
