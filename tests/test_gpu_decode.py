"""Decode attention (split-KV, block-causal prefill, live blocks, LSE merge) on the GPU
against the CPU oracle."""

import numpy as np
import pytest
import torch

import oracle
from conftest import bf16_from_bits
from gpu_util import LSE_TOL, O_TOL, assert_close, assert_device_ok, qkv

pytestmark = pytest.mark.gpu

SPLIT_CASES = [  # (B, H, q_len, kv_len, bs)
    (1, 12, 16, 16, 16), (1, 12, 16, 1040, 16), (2, 3, 16, 4112, 16), (1, 2, 16, 300, 16),
    (1, 2, 40, 200, 16), (1, 2, 64, 1000, 16), (2, 2, 7, 129, 4), (1, 1, 1, 1, 1),
    (1, 2, 33, 64, 32), (3, 2, 16, 16400, 16),
    (1, 4, 1, 70000, 16),  # one query row over a long cache (15 of the tile's rows padding)
    (2, 2, 64, 64, 64),    # the largest decode tile, no cache before the block
]


@pytest.mark.parametrize("B,H,q_len,kv_len,bs", SPLIT_CASES)
def test_split_kv_matches_oracle(B, H, q_len, kv_len, bs):
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    q, k, v = qkv(3, B, H, q_len, kv_len)
    o = split_kv_decode_attention(q.cuda(), k.cuda(), v.cuda(), bs)
    assert_device_ok()
    ref, _ = oracle.attention(q, k, v, oracle.block_causal_mask(q_len, kv_len, bs))
    assert o.shape == q.shape and o.dtype == q.dtype
    assert_close("O", o, ref, O_TOL)


@pytest.mark.parametrize("n_splits", [1, 2, 3, 7, 8, 9, 16, 17, 24])
def test_split_counts_and_lse(n_splits):
    """2 to 16 splits are merged inside the kernel through a thread-block cluster, more by
    the combine kernel: every count gives the oracle's O and LSE."""
    from bd3attn import ops
    q, k, v = qkv(4, 2, 3, 16, 1040)
    o, lse = ops.decode_raw(q.cuda(), k.cuda(), v.cuda(), 16, return_lse=True, n_splits=n_splits)
    assert_device_ok()
    ref, ref_lse = oracle.attention(q, k, v, oracle.block_causal_mask(16, 1040, 16))
    assert_close("O", o, ref, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)


@pytest.mark.parametrize("q_len,n_splits", [(32, 5), (32, 16), (40, 12), (1, 16), (64, 3)])
def test_cluster_merge_row_groups(q_len, n_splits):
    """The cluster merge with two 16-row groups per CTA, several row groups per (batch,
    head), a single query row and fp32 output; equal to the combine kernel's merge up to
    fp32 rounding, and to the oracle within the stated tolerances."""
    from bd3attn import ops
    q, k, v = qkv(12, 2, 3, q_len, 2000)
    args = (q.cuda(), k.cuda(), v.cuda(), 16)
    o, lse = ops.decode_raw(*args, return_lse=True, n_splits=n_splits, out_dtype=torch.float32)
    assert_device_ok()
    oc, lc = ops.decode_raw(*args, return_lse=True, n_splits=n_splits + 17,
                            out_dtype=torch.float32)  # past a cluster: the combine kernel
    assert_device_ok()
    ref, ref_lse = oracle.attention(q, k, v, oracle.block_causal_mask(q_len, 2000, 16))
    assert_close("O", o, ref, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)
    assert_close("O cluster vs combine", o, oc, 2e-3)
    assert_close("LSE cluster vs combine", lse, lc, 1e-4)


@pytest.mark.parametrize("B,H,q_len,kv_len,bs", [(1, 2, 65, 65, 16), (1, 2, 200, 1000, 16),
                                                 (1, 3, 3088, 3088, 16), (2, 2, 300, 300, 64),
                                                 (1, 1, 129, 4000, 16)])
def test_prefill_matches_oracle(B, H, q_len, kv_len, bs):
    from kernels.BlockSparseDecodeAttention import block_sparse_decode_attention
    q, k, v = qkv(5, B, H, q_len, kv_len)
    o = block_sparse_decode_attention(q.cuda(), k.cuda(), v.cuda(), bs)
    assert_device_ok()
    ref, _ = oracle.attention(q, k, v, oracle.block_causal_mask(q_len, kv_len, bs))
    assert_close("O", o, ref, O_TOL)


def test_decode_against_reference_golden(golden):
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    tags = sorted({k.rsplit("_", 1)[0] for k in golden if k.startswith("decode_")})
    for tag in tags:
        bs = int(tag.split("_")[3][2:])
        q, k, v = (bf16_from_bits(golden[f"{tag}_{x}"]) for x in ("q", "k", "v"))
        o = split_kv_decode_attention(q.cuda(), k.cuda(), v.cuda(), bs)
        assert_device_ok()
        assert_close(tag, o, torch.from_numpy(golden[f"{tag}_o"]), O_TOL)


def test_live_blocks_against_reference_golden(golden):
    from kernels.BlockSparseDecodeAttention import block_sparse_live_decode_attention
    q, k, v = (bf16_from_bits(golden[f"live_{x}"]) for x in ("q", "k", "v"))
    live = torch.from_numpy(golden["live_blocks"]).int()
    cnt = torch.full(live.shape[:2], live.shape[2], dtype=torch.int32)
    o = block_sparse_live_decode_attention(q.cuda(), k.cuda(), v.cuda(), live.cuda(), cnt.cuda(),
                                           64, 16)
    assert_device_ok()
    assert_close("O", o, torch.from_numpy(golden["live_o"]), O_TOL)


@pytest.mark.parametrize("B,H,kv_len,n_blocks_live,kv_block", [(16, 12, 8192, 32, 64),
                                                                (2, 3, 1000, 4, 128),
                                                                (1, 2, 4096, 64, 64)])
def test_live_blocks_matches_oracle(B, H, kv_len, n_blocks_live, kv_block):
    from kernels.BlockSparseDecodeAttention import block_sparse_live_decode_attention
    q_len, bs = 16, 16
    q, k, v = qkv(6, B, H, q_len, kv_len)
    rng = np.random.default_rng(0)
    nb = -(-kv_len // kv_block)
    live = np.zeros((B, H, n_blocks_live), dtype=np.int32)
    cnt = np.zeros((B, H), dtype=np.int32)
    for b in range(B):
        for h in range(H):
            c = int(rng.integers(1, n_blocks_live + 1))  # ragged counts per (b, h)
            pick = rng.choice(nb - 1, size=c - 1, replace=False) if c > 1 else []
            blocks = sorted(list(pick) + [nb - 1])  # the query block is always live
            live[b, h, :c] = blocks
            cnt[b, h] = c
    o = block_sparse_live_decode_attention(q.cuda(), k.cuda(), v.cuda(),
                                           torch.from_numpy(live).cuda(),
                                           torch.from_numpy(cnt).cuda(), kv_block, bs)
    assert_device_ok()
    lists = [[live[b, h, :cnt[b, h]].tolist() for h in range(H)] for b in range(B)]
    sub_b = min(B, 2)
    mask = oracle.live_block_mask(lists[:sub_b], q_len, kv_len, kv_block, bs)
    ref, _ = oracle.attention(q[:sub_b], k[:sub_b], v[:sub_b], mask)
    assert_close("O", o[:sub_b], ref, O_TOL)


def _ragged_lists(B, H, nb, max_live, seed, empty_every=0):
    """Ascending live block lists with ragged counts (some empty when empty_every > 0); the
    query block nb - 1 is live in every non-empty list."""
    rng = np.random.default_rng(seed)
    live = np.zeros((B, H, max_live), dtype=np.int32)
    cnt = np.zeros((B, H), dtype=np.int32)
    for b in range(B):
        for h in range(H):
            if empty_every and (b * H + h) % empty_every == 1:
                continue
            c = int(rng.integers(1, max_live + 1))
            pick = rng.choice(nb - 1, size=c - 1, replace=False) if c > 1 else []
            live[b, h, :c] = sorted(list(pick) + [nb - 1])
            cnt[b, h] = c
    return live, cnt


@pytest.mark.parametrize("B,H,q_len,kv_len,max_live,kv_block,empty_every", [
    (16, 12, 16, 8192, 32, 64, 0),     # benchmark config 4 shape, ragged counts
    (16, 12, 16, 8192, 32, 64, 5),     # some (batch, head) lists empty
    (2, 3, 32, 1000, 4, 128, 0),       # two 16-row groups, 128-token blocks
    (1, 2, 7, 4096, 64, 64, 0),        # few (batch, head) pairs: the plan splits the lists
])
def test_live_split_counts_agree(B, H, q_len, kv_len, max_live, kv_block, empty_every):
    """Live-block decode with one CTA per (batch, head) list, with the list split over 2 and 3
    CTAs (partials merged by the combine kernel) and with the planned split count agree with
    each other and with the oracle within the stated tolerances; an empty list gives NaN and
    LSE -inf. Splits round P to bf16 against different running maxima, so they agree to about
    1e-3, not bit for bit."""
    from bd3attn import ops
    q, k, v = qkv(11, B, H, q_len, kv_len)
    nb = -(-kv_len // kv_block)
    live, cnt = _ragged_lists(B, H, nb, max_live, 3, empty_every)
    args = (q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(live).cuda(),
            torch.from_numpy(cnt).cuda(), kv_block, 16)
    has = torch.from_numpy(cnt > 0)
    o1, l1 = ops.live_decode_raw(*args, out_dtype=torch.float32, return_lse=True, n_splits=1)
    assert_device_ok()
    for ns in (None, 2, 3):
        o, lse = ops.live_decode_raw(*args, out_dtype=torch.float32, return_lse=True, n_splits=ns)
        assert_device_ok()
        assert torch.isnan(o.cpu()[~has]).all() and (lse.cpu()[~has] == float("-inf")).all()
        assert_close(f"O {ns} splits vs 1", o.cpu()[has], o1.cpu()[has], 2e-3)
        assert_close(f"LSE {ns} splits vs 1", lse.cpu()[has], l1.cpu()[has], 1e-4)
    sub = [(b, h) for b in range(min(B, 2)) for h in range(H) if cnt[b, h] > 0]
    lists = [[live[b, h, :cnt[b, h]].tolist() for h in range(H)] for b in range(min(B, 2))]
    mask = oracle.live_block_mask(lists, q_len, kv_len, kv_block, 16)
    ref, ref_lse = oracle.attention(q[:2], k[:2], v[:2], mask)
    for b, h in sub:
        assert_close("O vs oracle", o1[b, h], ref[b, h], O_TOL)
        assert_close("LSE vs oracle", l1[b, h], ref_lse[b, h], LSE_TOL)


def test_lse_merge_of_shards_equals_full():
    """Sequence-sharded decode: per-shard partial (O fp32, LSE) then the merge kernel."""
    from bd3attn import ops
    B, H, q_len, kv_len, G, bs = 2, 3, 16, 4112, 4, 16
    q, k, v = qkv(7, B, H, q_len, kv_len)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    edges = np.linspace(0, kv_len, G + 1).astype(int)
    parts, lses = [], []
    for g in range(G):
        lo, hi = int(edges[g]), int(edges[g + 1])
        o, l = ops.decode_raw(qd, kd[:, :, lo:hi], vd[:, :, lo:hi], bs, q_pos0=kv_len - q_len,
                              kv_pos0=lo, out_dtype=torch.float32, return_lse=True)
        parts.append(o)
        lses.append(l)
    o, lse = ops.lse_merge_raw(torch.stack(parts), torch.stack(lses), torch.bfloat16)
    assert_device_ok()
    ref, ref_lse = oracle.attention(q, k, v, oracle.block_causal_mask(q_len, kv_len, bs))
    assert_close("O", o, ref, O_TOL)
    assert_close("LSE", lse, ref_lse, LSE_TOL)


def test_fp32_output_and_inputs():
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    q, k, v = qkv(8, 1, 2, 16, 500, torch.float32)
    o = split_kv_decode_attention(q.cuda(), k.cuda(), v.cuda(), 16)
    assert_device_ok()
    assert o.dtype == torch.float32
    ref, _ = oracle.attention(q, k, v, oracle.block_causal_mask(16, 500, 16))
    assert_close("O", o, ref, O_TOL)


def test_non_contiguous_cache_views():
    """k/v as views into a larger preallocated cache (length-sliced), q a strided view."""
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    q, k, v = qkv(9, 2, 3, 16, 2048)
    kd = torch.zeros(2, 3, 4096, 64, dtype=torch.bfloat16, device="cuda")
    vd = torch.zeros_like(kd)
    kd[:, :, :2048] = k.cuda()
    vd[:, :, :2048] = v.cuda()
    qbig = torch.zeros(2, 16, 3, 64, dtype=torch.bfloat16, device="cuda")
    qbig.copy_(q.cuda().transpose(1, 2))
    o = split_kv_decode_attention(qbig.transpose(1, 2), kd[:, :, :2048], vd[:, :, :2048], 16)
    assert_device_ok()
    ref, _ = oracle.attention(q, k, v, oracle.block_causal_mask(16, 2048, 16))
    assert_close("O", o, ref, O_TOL)


def test_live_blocks_long_list_single_split():
    """One split over a 300-entry live list, through the C ABI: the kernel stages the first
    256 entries of a split in shared memory and reads the rest from global memory."""
    import ctypes
    from bd3attn._lib import LIB
    B, H, q_len, kv_len, kv_block, bs, n_live = 1, 2, 16, 64 * 400, 64, 16, 300
    q, k, v = qkv(12, B, H, q_len, kv_len)
    rng = np.random.default_rng(3)
    nb = kv_len // kv_block
    live = np.stack([np.sort(np.concatenate([rng.choice(nb - 1, n_live - 1, replace=False),
                                             [nb - 1]])) for _ in range(B * H)])
    live = live.reshape(B, H, n_live).astype(np.int32)
    cnt = np.full((B, H), n_live, dtype=np.int32)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    ld, cd = torch.from_numpy(live).cuda(), torch.from_numpy(cnt).cuda()
    o = torch.empty_like(qd)
    st = []
    for t in (qd, kd, vd, o):
        st += [t.stride(0), t.stride(1), t.stride(2)]
    rc = LIB.bd3_decode_live_blocks(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(),
                                    None, ld.data_ptr(), cd.data_ptr(), n_live, n_live, kv_block,
                                    B, H, q_len, kv_len, 64, (ctypes.c_int64 * 12)(*st), bs, 1,
                                    0, 0, None, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, LIB.bd3_last_error()
    torch.cuda.synchronize()
    assert_device_ok()
    lists = [[live[0, h].tolist() for h in range(H)]]
    mask = oracle.live_block_mask(lists, q_len, kv_len, kv_block, bs)
    ref, _ = oracle.attention(q, k, v, mask)
    assert_close("O", o, ref, O_TOL)


def test_full_config3_size():
    """Benchmark config 3 at its largest single-GPU size (B=32, H=12, q_len 16, a 64K cache
    plus the block itself): the planned split-KV decode equals the oracle on two (b, h)
    slices, and equals the LSE merge of two sequence-shard decodes of the same cache (a
    size-independent consistency check over all 384 (b, h) pairs)."""
    from bd3attn import ops
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    B, H, q_len, kv_len, bs = 32, 12, 16, 65536 + 16, 16
    g = torch.Generator(device="cuda").manual_seed(17)
    q = torch.randn(B, H, q_len, 64, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, H, kv_len, 64, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, H, kv_len, 64, device="cuda", generator=g).bfloat16()
    o = split_kv_decode_attention(q, k, v, bs)
    full, full_lse = ops.decode_raw(q, k, v, bs, out_dtype=torch.float32, return_lse=True)
    torch.cuda.synchronize()
    assert_device_ok()
    sl = (slice(31, 32), slice(0, 2))
    mask = oracle.block_causal_mask(q_len, kv_len, bs)
    ref, ref_lse = oracle.attention(q[sl].cpu(), k[sl].cpu(), v[sl].cpu(), mask)
    assert_close("O", o[sl], ref, O_TOL)
    assert_close("LSE", full_lse[sl], ref_lse, LSE_TOL)
    half = 32768  # shard edge, a multiple of the 64-key tile
    parts, lses = [], []
    for lo, hi in ((0, half), (half, kv_len)):
        po, pl = ops.decode_raw(q, k[:, :, lo:hi], v[:, :, lo:hi], bs, q_pos0=kv_len - q_len,
                                kv_pos0=lo, out_dtype=torch.float32, return_lse=True)
        parts.append(po)
        lses.append(pl)
    merged, merged_lse = ops.lse_merge_raw(torch.stack(parts), torch.stack(lses), torch.float32)
    torch.cuda.synchronize()
    assert_device_ok()
    assert_close("O merged vs planned", merged, full, 1e-3)
    assert_close("LSE merged vs planned", merged_lse, full_lse, 1e-4)


@pytest.mark.parametrize("q_len,kv_len", [(16, 1040), (16, 4112), (128, 640)])
def test_fp32_decode_at_tf32_precision(q_len, kv_len):
    """fp32 decode inputs (split-KV for a 16-token block, the tcgen05 prefill kernel for 128
    queries) run on the fp16 kernels after the exact power-of-two scaling and return fp32 at
    tf32-level error (11-bit operand significands)."""
    from kernels.BlockSparseDecodeAttention import block_sparse_decode_attention
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    q, k, v = qkv(70 + q_len, 2, 12, q_len, kv_len, torch.float32)
    ref, _ = oracle.attention(q, k, v, oracle.block_causal_mask(q_len, kv_len, 16))
    for fn in (split_kv_decode_attention, block_sparse_decode_attention):
        o = fn(q.cuda(), k.cuda(), v.cuda(), 16)
        assert_device_ok()
        assert o.dtype == torch.float32
        assert_close(fn.__name__, o, ref, 2e-3)
