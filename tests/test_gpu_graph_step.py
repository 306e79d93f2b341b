"""One decode step of a BD3-LM sampling loop captured once in a CUDA graph and replayed for
block after block: per layer the fused QKV/RoPE cache write (cache rows taken from the device
positions) and the split-KV decode (key count read from the device), then the sampler step
with its (t, s) and (seed, offset) in device memory. Every replay must leave the caches
bit-equal to the eager calls with host-side rows and lengths, give the same attention output
and tokens, and agree with the CPU oracle."""

import pytest
import torch

import oracle
from gpu_util import O_TOL, assert_close, assert_device_ok
from oracle import kv_cache as okv

pytestmark = pytest.mark.gpu

B, H, D, S, BS, LAYERS, CAP, MAX_POS = 2, 4, 64, 16, 16, 2, 256, 512


def _tables():
    sin, cos = okv.rope_tables(D, MAX_POS)
    return torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()


def _caches():
    return [(torch.zeros(B, H, CAP, D, dtype=torch.bfloat16, device="cuda"),
             torch.zeros(B, H, CAP, D, dtype=torch.bfloat16, device="cuda"))
            for _ in range(LAYERS)]


def _prefill(caches, cos, sin, gen, n):
    """The prompt's k, v written eagerly at rows [0, n) (identical in every cache set)."""
    from bd3attn import ops
    xs = [(2 * torch.randn(B, n, 3 * H * D, generator=gen)).bfloat16().cuda() for _ in range(LAYERS)]
    for sets in caches:
        for (kc, vc), x in zip(sets, xs):
            ops.qkv_rope_cache_raw(x, H, cos, sin, kc, vc, 0, pos0=0)


def test_captured_step_replays_every_block():
    from bd3attn import ops
    gen = torch.Generator().manual_seed(11)
    cos, sin = _tables()
    ours, ref = _caches(), _caches()
    prompt = 32
    _prefill([ours, ref], cos, sin, gen, prompt)

    # static inputs of the captured step
    x_in = [torch.zeros(B, S, 3 * H * D, dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]
    q_buf = [torch.empty(B, H, S, D, dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]
    pos = torch.arange(prompt, prompt + S, device="cuda")
    kv_len = torch.tensor([prompt + S], dtype=torch.int32, device="cuda")

    def step():
        outs = []
        for layer, (kc, vc) in enumerate(ours):
            q = ops.qkv_rope_cache_raw(x_in[layer], H, cos, sin, kc, vc, -1, positions=pos,
                                       q_out=q_buf[layer])
            outs.append(ops.decode_raw(q, kc, vc, BS, out_dtype=torch.float32,
                                       kv_len_dev=kv_len))
        return outs

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):  # warm-up outside the capture (first-call set-up happens here)
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = step()
    assert_device_ok()

    for blk in range(6):
        start = prompt + blk * S
        xs = [(2 * torch.randn(B, S, 3 * H * D, generator=gen)).bfloat16().cuda()
              for _ in range(LAYERS)]
        for layer in range(LAYERS):
            x_in[layer].copy_(xs[layer])
        pos.copy_(torch.arange(start, start + S, device="cuda"))
        kv_len.fill_(start + S)
        graph.replay()
        assert_device_ok()
        for layer in range(LAYERS):
            kr, vr = ref[layer]
            q_ref = ops.qkv_rope_cache_raw(xs[layer], H, cos, sin, kr, vr, start, pos0=start)
            o_ref = ops.decode_raw(q_ref, kr[:, :, :start + S], vr[:, :, :start + S], BS,
                                   out_dtype=torch.float32)
            kc, vc = ours[layer]
            assert torch.equal(kc, kr) and torch.equal(vc, vr)  # untouched rows included
            assert torch.equal(q_buf[layer], q_ref)
            # the same kernel over the same keys; only the split partition differs
            assert_close(f"block {blk} layer {layer} O", static_out[layer], o_ref, 1e-5)
        if blk == 5:
            n = start + S
            want, _ = oracle.attention(q_ref.cpu(), kr[:, :, :n].cpu(), vr[:, :, :n].cpu(),
                                       oracle.block_causal_mask(S, n, BS))
            assert_close("O vs oracle", static_out[-1], want, O_TOL)
    del graph


def test_device_count_past_capacity_is_clamped_and_flagged():
    from bd3attn import ops
    gen = torch.Generator().manual_seed(12)
    q = torch.randn(B, H, S, D, generator=gen).bfloat16().cuda()
    k = torch.randn(B, H, CAP, D, generator=gen).bfloat16().cuda()
    v = torch.randn(B, H, CAP, D, generator=gen).bfloat16().cuda()
    o = ops.decode_raw(q, k, v, BS, kv_len_dev=torch.tensor([4096], dtype=torch.int32,
                                                           device="cuda"))
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 2
    assert_close("clamped O", o, ops.decode_raw(q, k, v, BS), 1e-2)
    assert_device_ok()


def test_device_cache_row_outside_cache_writes_nothing():
    from bd3attn import ops
    gen = torch.Generator().manual_seed(13)
    cos, sin = _tables()
    x = torch.randn(B, S, 3 * H * D, generator=gen).bfloat16().cuda()
    kc = torch.full((B, H, CAP, D), 7.0, dtype=torch.bfloat16, device="cuda")
    vc = kc.clone()
    pos = torch.arange(CAP - 8, CAP - 8 + S, device="cuda")  # rows [248, 264) of 256
    ops.qkv_rope_cache_raw(x, H, cos, sin, kc, vc, -1, positions=pos)
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 4
    assert torch.all(kc.float() == 7.0) and torch.all(vc.float() == 7.0)
    assert_device_ok()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_sampler_device_args_equal_host_args(dt):
    """bd3_subs_sample_dev with (t, s) and (seed, offset) in device memory draws the same
    tokens as bd3_subs_sample given them as host arguments; a device t <= 0 keeps every
    token and raises status bit 2."""
    from bd3attn.sampler import subs_sample_step, subs_sample_step_dev
    gen = torch.Generator().manual_seed(21)
    V, mask = 50258, 50257
    logits = (2 * torch.randn(2, 16, V, generator=gen)).to(dt).cuda()
    xt = torch.randint(0, V - 1, (2, 16), generator=gen)
    xt[torch.rand(2, 16, generator=gen) < 0.7] = mask
    xt = xt.cuda()
    seed = int(torch.randint(0, 2 ** 63 - 1, (1,), generator=torch.Generator().manual_seed(4)).item())
    for t, s, off in ((0.75, 0.5, 0), (0.5, 0.25, 7), (1.0, 0.0, 2 ** 40 + 3)):
        want = subs_sample_step(logits, xt, mask, t, s,
                                generator=torch.Generator().manual_seed(4), offset=off)
        got = subs_sample_step_dev(logits, xt, mask,
                                   torch.tensor([t, s], dtype=torch.float64, device="cuda"),
                                   torch.tensor([seed, off], dtype=torch.int64, device="cuda"))
        assert_device_ok()
        assert torch.equal(got, want)
    bad = subs_sample_step_dev(logits, xt, mask,
                               torch.tensor([0.0, 0.0], dtype=torch.float64, device="cuda"),
                               torch.tensor([seed, 0], dtype=torch.int64, device="cuda"))
    torch.cuda.synchronize()
    from bd3attn import ops
    assert ops.device_status(clear=True) == 2
    assert torch.equal(bad, xt)


def test_captured_denoising_step_with_sampler():
    """A whole denoising step in one graph: two layers' cache write + decode, a stand-in
    output projection (a torch GEMM from the last layer's attention output to logits) and
    the sampler with device (t, s) and (seed, offset), updating the block in place. Replays
    over two blocks of three steps each equal the same step run eagerly."""
    from bd3attn import ops
    from bd3attn.sampler import subs_sample_step_dev
    gen = torch.Generator().manual_seed(31)
    cos, sin = _tables()
    V, mask, prompt, steps = 4099, 4098, 32, 3
    ours, ref = _caches(), _caches()
    _prefill([ours, ref], cos, sin, gen, prompt)
    w_out = (torch.randn(H * D, V, generator=gen) / 8).bfloat16().cuda()
    x_in = [torch.zeros(B, S, 3 * H * D, dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]
    q_buf = [torch.empty(B, H, S, D, dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]
    pos = torch.arange(prompt, prompt + S, device="cuda")
    kv_len = torch.tensor([prompt + S], dtype=torch.int32, device="cuda")
    ts = torch.tensor([1.0, 0.5], dtype=torch.float64, device="cuda")
    rng = torch.tensor([123456789, 0], dtype=torch.int64, device="cuda")

    def step(caches, block):
        o = None
        for layer, (kc, vc) in enumerate(caches):
            q = ops.qkv_rope_cache_raw(x_in[layer], H, cos, sin, kc, vc, -1, positions=pos,
                                       q_out=q_buf[layer])
            o = ops.decode_raw(q, kc, vc, BS, kv_len_dev=kv_len)
        logits = o.transpose(1, 2).reshape(B, S, H * D) @ w_out
        return subs_sample_step_dev(logits, block, mask, ts, rng, out=block)

    block_g = torch.full((B, S), mask, dtype=torch.int64, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step(ours, block_g.clone())
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(ours, block_g)

    for blk in range(2):
        start = prompt + blk * S
        pos.copy_(torch.arange(start, start + S, device="cuda"))
        kv_len.fill_(start + S)
        block_g.fill_(mask)
        block_e = block_g.clone()
        for st in range(steps):
            t, s = 1.0 - st / steps, 1.0 - (st + 1) / steps
            for layer in range(LAYERS):
                x_in[layer].copy_((2 * torch.randn(B, S, 3 * H * D, generator=gen)).bfloat16())
            ts.copy_(torch.tensor([t, s], dtype=torch.float64))
            rng[1] = blk * steps + st
            graph.replay()
            step(ref, block_e)  # eager, same inputs, the reference caches
            assert_device_ok()
            assert torch.equal(block_g, block_e), (blk, st)
            for (kc, vc), (kr, vr) in zip(ours, ref):
                assert torch.equal(kc, kr) and torch.equal(vc, vr)
        assert bool((block_g != mask).all())  # the last step (s = 0) unmasks every token
    del graph
