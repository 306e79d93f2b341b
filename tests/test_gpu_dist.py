"""The multi-GPU partitions on real GPUs over NCCL (needs 2 GPUs; skipped otherwise).

- Sequence-sharded decode: each rank decodes its slice of the KV cache with the CUDA kernels;
  one NCCL all-gather moves the [O | LSE] partials and bd3_lse_merge combines them, or one
  kernel exchanges them over NVLink peer memory and merges them (bd3_peer_merge). The result
  must equal a single-GPU decode over the whole cache.
- Batch x head sharding of training attention: each rank runs the forward and backward on its
  (batch, head) shard; the shards must equal the same slices of a single-GPU run.

Ranks are spawned processes (one per GPU) with a short process-group timeout; NVLS is off.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gpu_util import O_TOL, LSE_TOL, GRAD_TOL, assert_close

pytestmark = pytest.mark.gpu

WORLD = 2


def _need_gpus():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs, found {torch.cuda.device_count()}")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


def _decode_inputs(B, H, q_len, kv_len):
    g = torch.Generator().manual_seed(11)
    mk = lambda s: torch.randn(B, H, s, 64, generator=g).bfloat16()  # noqa: E731
    return mk(q_len), mk(kv_len), mk(kv_len)


def _decode_worker(rank, port, B, H, q_len, kv_len, bs, path, exchange="nccl"):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "diffusion-llm_b200"))
    from bd3attn.dist import PeerMerge, seq_shard, sharded_decode
    _init(rank, port)
    try:
        q, k, v = (t.cuda() for t in _decode_inputs(B, H, q_len, kv_len))
        a, b = seq_shard(kv_len, WORLD, rank)
        kl, vl = k[:, :, a:b].contiguous(), v[:, :, a:b].contiguous()
        peer = PeerMerge(B, H, q_len) if exchange == "p2p" else None
        results = []
        # several calls in a row: the exchange alternates buffer parities by epoch
        for _ in range(3 if peer is not None else 1):
            o, lse = sharded_decode(q, kl, vl, bs, a, kv_len, out_dtype=torch.float32,
                                    peer=peer)
            results.append((o.clone(), lse.clone()))
        torch.cuda.synchronize()
        from bd3attn import ops
        assert ops.device_status(clear=True) == 0
        for o2, l2 in results[1:]:  # every call gives the first one's result, bit for bit
            assert torch.equal(o2, results[0][0]) and torch.equal(l2, results[0][1])
        if rank == 0:
            torch.save((results[0][0].cpu(), results[0][1].cpu()), path)
        dist.barrier()
        del peer
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
@pytest.mark.parametrize("B,H,q_len,kv_len,bs", [(2, 12, 16, 4160, 16), (1, 4, 40, 1000, 8)])
def test_sharded_decode_equals_single_gpu(tmp_path, B, H, q_len, kv_len, bs, exchange):
    """The partials meet through an NCCL all-gather and bd3_lse_merge, or through NVLink peer
    memory in one kernel (bd3_peer_merge, three calls in a row, equal to each other bit for
    bit); either way the merged result equals a single-GPU decode of the whole cache."""
    _need_gpus()
    from bd3attn import ops
    path = str(tmp_path / "out.pt")
    mp.spawn(_decode_worker, args=(_free_port(), B, H, q_len, kv_len, bs, path, exchange),
             nprocs=WORLD, join=True)
    o, lse = torch.load(path)
    q, k, v = (t.cuda() for t in _decode_inputs(B, H, q_len, kv_len))
    ref_o, ref_lse = ops.decode_raw(q, k, v, bs, out_dtype=torch.float32, return_lse=True)
    assert_close("O", o.cuda(), ref_o, O_TOL)
    assert_close("LSE", lse.cuda(), ref_lse, LSE_TOL)


def _train_inputs(B, H, n):
    g = torch.Generator().manual_seed(5)
    mk = lambda: torch.randn(B, H, 2 * n, 64, generator=g).bfloat16()  # noqa: E731
    return mk(), mk(), mk(), mk()


def _train_worker(rank, port, B, H, n, bs, path):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "diffusion-llm_b200"))
    from bd3attn.dist import bh_shard
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    _init(rank, port)
    try:
        q, k, v, do = _train_inputs(B, H, n)
        b0, b1 = bh_shard(B, H, WORLD, rank)
        flat = lambda t: t.reshape(B * H, 2 * n, 64)[b0:b1].unsqueeze(0).cuda()  # noqa: E731
        qs, ks, vs, dos = (flat(t).requires_grad_(t is not do) for t in (q, k, v, do))
        o = BlockSparseFlashAttention.apply(qs, ks, vs, bs)
        dq, dk, dv = torch.autograd.grad(o, (qs, ks, vs), dos)
        torch.cuda.synchronize()
        out = torch.stack([o, dq, dk, dv]).squeeze(1).contiguous()  # (4, shard, 2n, 64)
        sizes = [torch.zeros(1, dtype=torch.long, device="cuda") for _ in range(WORLD)]
        dist.all_gather(sizes, torch.tensor([out.shape[1]], device="cuda"))
        cap = max(int(s.item()) for s in sizes)
        padded = torch.zeros(4, cap, 2 * n, 64, dtype=out.dtype, device="cuda")
        padded[:, : out.shape[1]] = out
        gathered = [torch.empty_like(padded) for _ in range(WORLD)]
        dist.all_gather(gathered, padded)
        if rank == 0:
            full = torch.cat([g_[:, : int(s.item())] for g_, s in zip(gathered, sizes)], dim=1)
            torch.save(full.cpu(), path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_bh_sharded_training_nccl_equals_single_gpu(tmp_path):
    _need_gpus()
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    B, H, n, bs = 2, 3, 256, 16
    path = str(tmp_path / "train.pt")
    mp.spawn(_train_worker, args=(_free_port(), B, H, n, bs, path), nprocs=WORLD, join=True)
    got = torch.load(path).cuda()  # (4, B*H, 2n, 64): O, dQ, dK, dV over all shards
    q, k, v, do = (t.cuda() for t in _train_inputs(B, H, n))
    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)
    o = BlockSparseFlashAttention.apply(q, k, v, bs)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), do)
    ref = torch.stack([t.reshape(B * H, 2 * n, 64) for t in (o, dq, dk, dv)])
    assert_close("O", got[0], ref[0], O_TOL)
    for name, idx in (("dQ", 1), ("dK", 2), ("dV", 3)):
        assert_close(name, got[idx], ref[idx], GRAD_TOL)
