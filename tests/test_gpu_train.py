"""Training attention (BD3-LM mask) forward and backward on the GPU against the CPU oracle."""

import numpy as np
import pytest
import torch

import oracle
from conftest import bf16_from_bits
from gpu_util import GRAD_TOL, LSE_TOL, O_TOL, assert_close, assert_device_ok, qkv, randn

pytestmark = pytest.mark.gpu

CASES = [  # (B, H, n, block_size)
    (1, 1, 128, 16), (1, 2, 128, 4), (2, 1, 256, 16), (1, 2, 256, 128), (1, 1, 512, 64),
    (1, 1, 256, 256), (1, 2, 1024, 16), (1, 1, 1024, 4), (1, 1, 384, 32), (1, 1, 512, 1024 // 2),
    (1, 1, 128, 1),      # one-token blocks: the densest rule pattern
    (1, 1, 2048, 64), (1, 1, 4096, 128),  # long sequences (2n = 4096, 8192)
    (16, 12, 256, 16),   # 384 items on 148 persistent CTAs: several items per CTA
]


def _run(B, H, n, bs, seed=0, dtype=torch.bfloat16):
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    q, k, v = qkv(seed, B, H, 2 * n, 2 * n, dtype)
    do = randn(torch.Generator().manual_seed(seed + 99), (B, H, 2 * n, 64), dtype)
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = BlockSparseFlashAttention.apply(qd, kd, vd, bs)
    dq, dk, dv = torch.autograd.grad(o, (qd, kd, vd), do.cuda())
    assert_device_ok()
    return (q, k, v, do), (o, dq, dk, dv)


@pytest.mark.parametrize("B,H,n,bs", CASES)
def test_forward_matches_oracle(B, H, n, bs):
    from bd3attn import ops
    q, k, v = qkv(1, B, H, 2 * n, 2 * n)
    o, lse = ops.attn_fwd_raw(q.cuda(), k.cuda(), v.cuda(), bs)
    assert_device_ok()
    ref_o, ref_lse = oracle.attention(q, k, v, oracle.block_diff_mask(n, bs))
    assert o.dtype == torch.bfloat16 and o.shape == q.shape
    assert_close("O", o, ref_o, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)


@pytest.mark.parametrize("B,H,n,bs", [c for c in CASES if c[2] <= 512] + [(1, 1, 1024, 16),
                                                                          (1, 1, 2048, 64)])
def test_backward_matches_oracle(B, H, n, bs):
    (q, k, v, do), (o, dq, dk, dv) = _run(B, H, n, bs, seed=2)
    mask = oracle.block_diff_mask(n, bs)
    ref_o, _ = oracle.attention(q, k, v, mask)
    rdq, rdk, rdv = oracle.attention_grads(q, k, v, do, mask)
    assert_close("O", o, ref_o, O_TOL)
    assert_close("dQ", dq, rdq, GRAD_TOL)
    assert_close("dK", dk, rdk, GRAD_TOL)
    assert_close("dV", dv, rdv, GRAD_TOL)


def test_dkdv_deterministic():
    """dK and dV are bitwise reproducible (one CTA owns each key tile and writes it once);
    by default dQ is an fp32 atomic sum, equal up to summation order."""
    _, (_, dq1, dk1, dv1) = _run(2, 2, 256, 16, seed=5)
    _, (_, dq2, dk2, dv2) = _run(2, 2, 256, 16, seed=5)
    assert torch.equal(dk1, dk2) and torch.equal(dv1, dv2)
    assert (dq1.float() - dq2.float()).abs().max().item() <= 1e-2


@pytest.mark.parametrize("B,H,n,bs", [(2, 2, 256, 16), (1, 1, 128, 1), (1, 2, 1024, 4),
                                      (16, 12, 256, 16), (8, 12, 1024, 16)])
def test_deterministic_backward(B, H, n, bs):
    """Under torch.use_deterministic_algorithms(True) the backward adds dQ's partials as
    64-bit fixed-point integers: dQ, dK and dV are bitwise equal from run to run (the
    reference's dQ kernel is deterministic too), and equal the fp32-accumulating backward's
    within bf16 rounding and the oracle's within the stated tolerance."""
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        (q, k, v, do), (o, dq1, dk1, dv1) = _run(B, H, n, bs, seed=5)
        for _ in range(2):
            _, (_, dq2, dk2, dv2) = _run(B, H, n, bs, seed=5)
            assert torch.equal(dq1, dq2) and torch.equal(dk1, dk2) and torch.equal(dv1, dv2)
    finally:
        torch.use_deterministic_algorithms(prev)
    _, (_, dqf, dkf, dvf) = _run(B, H, n, bs, seed=5)
    assert torch.equal(dk1, dkf) and torch.equal(dv1, dvf)  # the same kernel for dK, dV
    # the two round the same sums (in different orders, or not) to bf16: one ulp apart at most
    rel = ((dq1.float() - dqf.float()).abs() / dqf.float().abs().clamp_min(1.0)).max().item()
    assert rel <= 1e-2, f"dQ det vs fp32 accumulation: relative {rel:.3e}"
    if B * H * n <= 4096:
        rdq, _, _ = oracle.attention_grads(q, k, v, do, oracle.block_diff_mask(n, bs))
        assert_close("dQ det vs oracle", dq1, rdq, GRAD_TOL)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_deterministic_backward_other_dtypes(dtype):
    """The deterministic backward with fp16 inputs and with fp32 inputs (config 1's, run on
    fp16 operands scaled by powers of two): bitwise equal from run to run, and within the
    stated tolerance of the oracle."""
    B, H, n, bs = 2, 3, 256, 16
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        (q, k, v, do), (_, dq1, dk1, dv1) = _run(B, H, n, bs, seed=7, dtype=dtype)
        _, (_, dq2, dk2, dv2) = _run(B, H, n, bs, seed=7, dtype=dtype)
    finally:
        torch.use_deterministic_algorithms(prev)
    assert dq1.dtype == dtype
    assert torch.equal(dq1, dq2) and torch.equal(dk1, dk2) and torch.equal(dv1, dv2)
    rdq, rdk, rdv = oracle.attention_grads(q, k, v, do, oracle.block_diff_mask(n, bs))
    assert_close("dQ", dq1, rdq, GRAD_TOL)
    assert_close("dK", dk1, rdk, GRAD_TOL)
    assert_close("dV", dv1, rdv, GRAD_TOL)


@pytest.mark.parametrize("bs", [4, 16, 128])
def test_against_reference_golden(golden, bs):
    """Kernel vs the outputs the reference itself produced (fp32, on bf16-valued inputs)."""
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    tag = f"train_n128_bs{bs}"
    q, k, v, do = (bf16_from_bits(golden[f"{tag}_{x}"]) for x in ("q", "k", "v", "do"))
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = BlockSparseFlashAttention.apply(qd, kd, vd, bs)
    dq, dk, dv = torch.autograd.grad(o, (qd, kd, vd), do.cuda())
    assert_device_ok()
    for name, got in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert_close(name, got, torch.from_numpy(golden[f"{tag}_{name}"]), O_TOL)


def test_strided_inputs_like_the_model():
    """q/k/v as views of a fused qkv projection: (B, S, 3*H*64) -> (B, H, S, 64) per tensor,
    the layout model/modules.py:399-403 hands the attention (no copy is made)."""
    from bd3attn import ops
    B, H, n, bs = 2, 3, 256, 16
    g = torch.Generator().manual_seed(4)
    qkv_proj = randn(g, (B, 2 * n, 3 * H * 64))
    t = qkv_proj.view(B, 2 * n, 3, H, 64).permute(2, 0, 3, 1, 4)
    q, k, v = t[0], t[1], t[2]
    dev = qkv_proj.cuda().view(B, 2 * n, 3, H, 64).permute(2, 0, 3, 1, 4)
    o, lse = ops.attn_fwd_raw(dev[0], dev[1], dev[2], bs)
    assert_device_ok()
    ref_o, ref_lse = oracle.attention(q, k, v, oracle.block_diff_mask(n, bs))
    assert_close("O", o, ref_o, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)


def test_fp16_inputs():
    from bd3attn import ops
    q, k, v = qkv(8, 1, 2, 512, 512, torch.float16)
    o, lse = ops.attn_fwd_raw(q.cuda(), k.cuda(), v.cuda(), 16)
    assert_device_ok()
    ref_o, ref_lse = oracle.attention(q, k, v, oracle.block_diff_mask(256, 16))
    assert o.dtype == torch.float16
    assert_close("O", o, ref_o, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)


# fp32 inputs run at tf32's operand precision (11-bit significands, fp32 accumulation), the
# precision of the reference's Triton tl.dot on fp32. Rounding this config's operands to an
# 11-bit significand (and P before P V, as tl.dot does) gives max-abs errors of 0.93e-3 in O
# and 0.55e-3 in LSE against float64 (a CPU emulation of tf32 over these seeded inputs); the
# fp16 output adds at most half an ulp of |O| (2^-12 relative). The tolerances below leave 2x
# on O and LSE; the bf16 path of 16-bit callers sits at 9.3e-3 / 5.9e-3 on the same inputs.
F32_O_TOL, F32_LSE_TOL, F32_GRAD_TOL = 2e-3, 1e-3, 4e-3


def test_fp32_inputs_config1():
    """Benchmark config 1 (B=2, H=12, n=1024, bs=16, fp32 N(0,1)): every head's O and LSE
    against the float64 oracle at tf32-level tolerances."""
    from bd3attn import ops
    from kernels import _precision
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    q, k, v = qkv(9, 2, 12, 2048, 2048, torch.float32)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o = BlockSparseFlashAttention.apply(qd, kd, vd, 16)
    q16, k16, v16, a, c = _precision.qkv_to_f16(qd, kd, vd)
    _, lse = ops.attn_fwd_raw(q16, k16, v16, 16)
    assert_device_ok()
    assert o.dtype == torch.float32
    mask = oracle.block_diff_mask(1024, 16)
    for b in range(2):
        ref_o, ref_lse = oracle.attention(q[b], k[b], v[b], mask)
        assert_close(f"O[{b}]", o[b], ref_o, F32_O_TOL)
        assert_close(f"LSE[{b}]", lse[b], ref_lse, F32_LSE_TOL)


def test_fp32_inputs_wide_range_and_backward():
    """fp32 inputs far outside fp16's range (q x 2^20, k x 2^-20, v x 2^30) give the same
    results as unscaled ones up to the power-of-two factors: the scaling into fp16 is exact.
    The backward's dQ, dK, dV come back in fp32 at tf32-level error."""
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    n, bs = 256, 16
    q, k, v = qkv(12, 1, 3, 2 * n, 2 * n, torch.float32)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(13))
    mask = oracle.block_diff_mask(n, bs)
    ref_o, _ = oracle.attention(q, k, v, mask)
    rdq, rdk, rdv = oracle.attention_grads(q, k, v, do, mask)
    xs = [t.cuda().requires_grad_(True) for t in (q, k, v)]
    o = BlockSparseFlashAttention.apply(*xs, bs)
    dq, dk, dv = torch.autograd.grad(o, xs, do.cuda())
    assert_device_ok()
    assert all(t.dtype == torch.float32 for t in (o, dq, dk, dv))
    assert_close("O", o, ref_o, F32_O_TOL)
    for name, got, ref in (("dQ", dq, rdq), ("dK", dk, rdk), ("dV", dv, rdv)):
        assert_close(name, got, ref, F32_GRAD_TOL)
    sq, sk, sv = 2.0 ** 20, 2.0 ** -20, 2.0 ** 30
    ys = [(t.detach() * s).requires_grad_(True) for t, s in zip(xs, (sq, sk, sv))]
    o2 = BlockSparseFlashAttention.apply(*ys, bs)
    dq2, dk2, dv2 = torch.autograd.grad(o2, ys, do.cuda() * 2.0 ** -7)
    assert_device_ok()
    # the scores q . k are unchanged: O2 = 2^30 O, and with dO2 = 2^-7 dO the gradients are
    # dQ2 = 2^30 2^-20 2^-7 dQ, dK2 = 2^30 2^20 2^-7 dK, dV2 = 2^-7 dV
    assert_close("O (wide range) / 2^30", o2 / sv, ref_o, F32_O_TOL)
    assert_close("dQ (wide range)", dq2 * 2.0 ** -3, rdq, F32_GRAD_TOL)
    assert_close("dK (wide range)", dk2 * 2.0 ** -43, rdk, F32_GRAD_TOL)
    assert_close("dV (wide range)", dv2 * 2.0 ** 7, rdv, F32_GRAD_TOL)


def test_reference_assertions():
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    q = torch.zeros(1, 1, 200, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        BlockSparseFlashAttention.apply(q, q, q, 16)  # n = 100 is not a multiple of 128
    q = torch.zeros(1, 1, 256, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 1, 512, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        BlockSparseFlashAttention.apply(q, k, k, 16)


@pytest.mark.parametrize("bs", [4, 16])
def test_forward_with_row_divergent_rescales(bs):
    """Keys grow tile by tile, so the running maximum jumps by more than 2^8 for some rows of
    a warp and not for others: the lazy-rescale path must stay warp-collective and exact."""
    from bd3attn import ops
    B, H, n = 1, 4, 1024
    q, k, v = qkv(21, B, H, 2 * n, 2 * n)
    ramp = torch.ones(2 * n)
    ramp[n:] = torch.linspace(0.5, 3.0, n)       # clean keys: later blocks score higher
    ramp[:n] = torch.linspace(0.5, 3.0, n)
    k = (k.float() * ramp[None, None, :, None]).bfloat16()
    o, lse = ops.attn_fwd_raw(q.cuda(), k.cuda(), v.cuda(), bs)
    assert_device_ok()
    ref_o, ref_lse = oracle.attention(q, k, v, oracle.block_diff_mask(n, bs))
    assert_close("O", o, ref_o, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)


@pytest.mark.parametrize("bs", [4, 16])
def test_full_config2_size_runs_clean(bs):
    """Benchmark config 2 at full size (B=8, H=12, n=1024): repeated fwd+bwd launches finish
    with no bounded wait running out; two heads checked against the oracle."""
    from bd3attn import ops
    B, H, n = 8, 12, 1024
    q, k, v = qkv(30 + bs, B, H, 2 * n, 2 * n)
    do = randn(torch.Generator().manual_seed(31), (B, H, 2 * n, 64))
    qd, kd, vd, dod = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    for _ in range(3):
        o, lse = ops.attn_fwd_raw(qd, kd, vd, bs)
        dq, dk, dv = ops.attn_bwd_raw(qd, kd, vd, o, lse, dod, bs)
    assert_device_ok()
    mask = oracle.block_diff_mask(n, bs)
    sl = (slice(7, 8), slice(10, 12))
    ref_o, ref_lse = oracle.attention(q[sl], k[sl], v[sl], mask)
    assert_close("O", o[sl], ref_o, O_TOL)
    assert_close("LSE", lse[sl], ref_lse, LSE_TOL)
    rdq, rdk, rdv = oracle.attention_grads(q[sl], k[sl], v[sl], do[sl], mask)
    assert_close("dQ", dq[sl], rdq, GRAD_TOL)
    assert_close("dK", dk[sl], rdk, GRAD_TOL)
    assert_close("dV", dv[sl], rdv, GRAD_TOL)
