"""The drop-in modules under torch.compile: inference/generate.py compiles the reference's
backbone with dynamic=True, so the ``torch.ops.bd3.*`` custom ops must trace through their
fake implementations (shapes and dtypes of the real outputs) without a graph break. A
function calling the three kernels' entry points (training forward and backward, block-causal
prefill, split-KV decode) is compiled with fullgraph=True, which raises on any graph break,
and its outputs and gradients equal the eager calls' at two sequence lengths."""

import pytest
import torch

from gpu_util import assert_device_ok, qkv

pytestmark = pytest.mark.gpu


def _attention_calls(q, k, v, qd, kd, vd, block_size: int):
    from kernels.BlockSparseDecodeAttention import block_sparse_decode_attention
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    o = BlockSparseFlashAttention.apply(q, k, v, block_size)
    prefill = block_sparse_decode_attention(q, k, v, block_size)
    dec = split_kv_decode_attention(qd, kd, vd, block_size)
    return o, prefill, dec


@pytest.mark.parametrize("dynamic", [True, False])
def test_compiled_matches_eager(dynamic):
    torch._dynamo.reset()
    compiled = torch.compile(_attention_calls, fullgraph=True, dynamic=dynamic)
    for i, (n, kv) in enumerate(((256, 1040), (384, 2064))):
        q, k, v = (t.cuda().requires_grad_(True) for t in qkv(20 + i, 2, 12, 2 * n, 2 * n))
        qd, kd, vd = (t.cuda() for t in qkv(30 + i, 2, 12, 16, kv))
        do = torch.randn(q.shape, generator=torch.Generator().manual_seed(40 + i)).bfloat16().cuda()
        outs_c = compiled(q, k, v, qd, kd, vd, 16)
        grads_c = torch.autograd.grad(outs_c[0], (q, k, v), do)
        outs_e = _attention_calls(q, k, v, qd, kd, vd, 16)
        grads_e = torch.autograd.grad(outs_e[0], (q, k, v), do)
        assert_device_ok()
        for a, b in zip(outs_c, outs_e):
            assert a.shape == b.shape and a.dtype == b.dtype
            assert torch.equal(a.detach(), b.detach())
        for a, b in zip(grads_c, grads_e):
            assert a.shape == b.shape and a.dtype == b.dtype
            # dK, dV are deterministic; dQ's reduce-adds in L2 are not ordered
            assert (a.float() - b.float()).abs().max().item() <= 1e-2
