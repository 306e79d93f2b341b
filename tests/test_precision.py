"""The exact power-of-two scaling that puts fp32 inputs on the fp16 kernels
(bd3_f32_to_f16_scaled, kernels/_precision.py).

On the CPU, a restatement of the scaling (``qkv_to_f16_reference`` below) is checked for
what the design relies on: the scaled operands round-trip to the inputs within fp16's
half-ulp (tf32's), every score q . k survives the rebalancing, out-of-range products saturate.
On the GPU, the library's two kernels must equal the restatement bit for bit, strided inputs
included.
"""

import pytest
import torch

F16_MAX = 65504.0


def _exponent(t):
    """floor(log2(max |t|)) from the binary exponent, at least -100."""
    m = t.abs().amax().float()
    return (torch.frexp(m).exponent.float() - 1.0).clamp_min(-100.0)


def qkv_to_f16_reference(q, k, v):
    """q * 2^-a, k * 2^a (saturated at 65504), v * 2^-c in fp16, a = floor((e_q - e_k) / 2),
    c = e_v - 4."""
    a = torch.floor((_exponent(q) - _exponent(k)) * 0.5)
    c = _exponent(v) - 4.0
    q16 = (q.float() * torch.exp2(-a)).clamp(-F16_MAX, F16_MAX).to(torch.float16)
    k16 = (k.float() * torch.exp2(a)).clamp(-F16_MAX, F16_MAX).to(torch.float16)
    v16 = (v.float() * torch.exp2(-c)).to(torch.float16)
    return q16, k16, v16, a, c


@pytest.mark.parametrize("sq,sk,sv", [(1.0, 1.0, 1.0), (2.0 ** 20, 2.0 ** -18, 2.0 ** 30),
                                      (2.0 ** -8, 2.0 ** -5, 2.0 ** -40), (3e4, 1e-3, 7e4)])
def test_scaling_is_exact_and_in_range(sq, sk, sv):
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(2, 3, 256, 64, generator=g) * s for s in (sq, sk, sv))
    q16, k16, v16, a, c = qkv_to_f16_reference(q, k, v)
    assert q16.dtype == k16.dtype == v16.dtype == torch.float16
    for t in (q16, k16, v16):
        assert torch.isfinite(t).all()
    # fp16 rounding of a normal number: relative error at most 2^-11 (tf32's unit roundoff)
    back_q = q16.float() * torch.exp2(a)
    back_k = k16.float() * torch.exp2(-a)
    back_v = v16.float() * torch.exp2(c)
    for got, want, t16 in ((back_q, q, q16), (back_k, k, k16), (back_v, v, v16)):
        normal = t16.float().abs() >= 2.0 ** -14  # fp16 normal numbers
        assert normal.float().mean().item() > 0.99
        rel = ((got - want).abs() / want.abs())[normal]
        assert rel.max().item() <= 2.0 ** -11
    assert 16 <= v16.float().abs().amax().item() < 32
    # the scores are q . k: rebalancing by 2^-a, 2^a leaves them unchanged up to rounding
    s_ref = q.double() @ k.double().transpose(-1, -2)
    s16 = q16.double() @ k16.double().transpose(-1, -2)
    scale = (q.double().abs().amax(-1, keepdim=True) * k.double().abs().amax(-1)[..., None, :])
    assert ((s16 - s_ref).abs() / (64 * scale)).max().item() < 2.0 ** -10


def test_gradient_scaling():
    from kernels import _precision
    do = torch.randn(1, 2, 128, 64, generator=torch.Generator().manual_seed(2)) * 2.0 ** 13
    do16, e = _precision.grad_to_f16(do)
    assert e.item() == 13 + torch.floor(torch.log2(do.abs().amax() / 2 ** 13)).item()
    assert 1 <= do16.float().abs().amax().item() < 2
    assert torch.equal(_precision.scaled_back(do16, e), do16.float() * 2.0 ** e.item())


def test_tiny_scores_stay_accurate_in_softmax_units():
    """When max|q| * max|k| is below fp16's normal range, the balanced operands are fp16
    subnormals: their relative precision drops, but the scores (s / 8 in the softmax) are then
    within 1e-9 of 0 and of their exact values, so the attention weights are uniform to that
    accuracy either way."""
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 2, 128, 64, generator=g) * 2.0 ** -30
    k = torch.randn(1, 2, 128, 64, generator=g) * 2.0 ** -5
    v = torch.randn(1, 2, 128, 64, generator=g)
    q16, k16, _, _, _ = qkv_to_f16_reference(q, k, v)
    s_ref = (q.double() @ k.double().transpose(-1, -2)) / 8
    s16 = (q16.double() @ k16.double().transpose(-1, -2)) / 8
    assert (s16 - s_ref).abs().max().item() < 1e-9


def test_out_of_range_product_saturates():
    """max|q| * max|k| >= 2^30 cannot be balanced into fp16: the operands saturate (finite)."""
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(1, 1, 64, 64, generator=g) * 3e5 for _ in range(3))
    q16, k16, v16, _, _ = qkv_to_f16_reference(q, k, v)
    assert all(torch.isfinite(t).all() for t in (q16, k16, v16))


@pytest.mark.gpu
@pytest.mark.parametrize("sq,sk,sv", [(1.0, 1.0, 1.0), (2.0 ** 20, 2.0 ** -18, 2.0 ** 30),
                                      (2.0 ** -8, 2.0 ** -5, 2.0 ** -40), (3e4, 1e-3, 7e4),
                                      (3e5, 3e5, 3e5), (0.7, 1.3, 2.0 ** -130)])
def test_library_scaling_equals_restatement(sq, sk, sv):
    """bd3_f32_to_f16_scaled equals the restatement bit for bit, with strided inputs and a
    query count different from the key count, and reports exps = (a, c, 2^c)."""
    from bd3attn import ops
    g = torch.Generator().manual_seed(5)
    base = torch.randn(2, 3, 3, 200, 64, generator=g)
    q = (base[:, :, 0, :96] * sq).cuda()         # strided view: rows of a wider tensor
    k = (torch.randn(2, 3, 200, 64, generator=g) * sk).cuda()
    v = (torch.randn(2, 3, 200, 64, generator=g) * sv).cuda()
    q = torch.empty(2, 3, 3, 200, 64, device="cuda")[:, :, 1, :96].copy_(q)
    q16, k16, v16, exps = ops.f32_to_f16_scaled_raw(q, k, v)
    torch.cuda.synchronize()
    rq, rk, rv, a, c = qkv_to_f16_reference(q.cpu(), k.cpu(), v.cpu())
    assert torch.equal(q16.cpu().view(torch.int16), rq.view(torch.int16))
    assert torch.equal(k16.cpu().view(torch.int16), rk.view(torch.int16))
    assert torch.equal(v16.cpu().view(torch.int16), rv.view(torch.int16))
    e = exps.cpu()
    assert e[0].item() == a.item() and e[1].item() == c.item() and e[2].item() == 2.0 ** c.item()
