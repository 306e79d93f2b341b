"""Host-side logic of the multi-GPU partitions on world_size-2 gloo ranks (no GPU):
the batch x head and sequence shard arithmetic, and the sequence-sharded decode's gather and
merge, with the CPU oracle standing in for the device kernels."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bd3attn.dist import bh_shard, seq_shard, sharded_decode


@pytest.mark.parametrize("B,H,world", [(8, 12, 2), (8, 12, 8), (1, 12, 8), (3, 5, 4), (1, 1, 2)])
def test_bh_shard_tiles_exactly(B, H, world):
    seen = []
    for r in range(world):
        a, b = bh_shard(B, H, world, r)
        seen.extend(range(a, b))
    assert seen == list(range(B * H))


@pytest.mark.parametrize("kv_len,world", [(65552, 8), (1000, 2), (64, 4), (130, 3)])
def test_seq_shard_tiles_exactly(kv_len, world):
    pos = []
    for r in range(world):
        a, b = seq_shard(kv_len, world, r)
        assert a % 64 == 0
        pos.extend(range(a, b))
    assert pos == list(range(kv_len))


def _oracle_partial(q, k, v, block_size, q_pos0, kv_pos0):
    import oracle
    q_len, kv_len = q.shape[2], k.shape[2]
    qp = np.arange(q_pos0, q_pos0 + q_len)[:, None]
    kp = np.arange(kv_pos0, kv_pos0 + kv_len)[None, :]
    mask = (qp // block_size) >= (kp // block_size)
    o, lse = oracle.attention(q, k, v, mask)
    return o.float(), lse.float()


def _oracle_merge(parts, lses, out_dtype):
    import oracle
    o, lse = oracle.lse_merge(parts, lses)
    return o.to(out_dtype), lse.float()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, kv_len, q_len, bs, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 3, q_len, 64, generator=g)
    k = torch.randn(2, 3, kv_len, 64, generator=g)
    v = torch.randn(2, 3, kv_len, 64, generator=g)
    a, b = seq_shard(kv_len, world, rank)
    o, lse = sharded_decode(q, k[:, :, a:b], v[:, :, a:b], bs, a, kv_len,
                            out_dtype=torch.float64, partial_fn=_oracle_partial,
                            merge_fn=_oracle_merge)
    if rank == 0:
        torch.save((o, lse), result_path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,kv_len,q_len,bs", [(2, 1040, 16, 16), (2, 300, 40, 16),
                                                   (3, 130, 16, 16)])
def test_sharded_decode_equals_full_attention(tmp_path, world, kv_len, q_len, bs):
    import oracle
    path = str(tmp_path / "out.pt")
    mp.spawn(_worker, args=(world, _free_port(), kv_len, q_len, bs, path), nprocs=world,
             join=True)
    o, lse = torch.load(path)
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 3, q_len, 64, generator=g)
    k = torch.randn(2, 3, kv_len, 64, generator=g)
    v = torch.randn(2, 3, kv_len, 64, generator=g)
    ref, ref_lse = oracle.attention(q, k, v, oracle.block_causal_mask(q_len, kv_len, bs))
    torch.testing.assert_close(o, ref, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(lse.double(), ref_lse, atol=1e-5, rtol=1e-5)


def _dropout_worker(rank, world, port, leave_rank, leave_after, mode, out_dir):
    """Steps of sequence-sharded decode on gloo ranks; ``leave_rank`` returns after finishing
    step ``leave_after`` (between steps: none of its collectives in flight). mode "watch":
    the survivors check their peers in the store before each step; mode "collective": they
    do not, and the process group's short timeout ends the next collective with an error."""
    import datetime
    import json

    from bd3attn.dist import PeerWatch, RankDropped
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    # joining may take a while (each spawned rank imports the package first); only the
    # data path's group carries the short timeout
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    dist.barrier()
    group = dist.new_group(list(range(world)), timeout=datetime.timedelta(seconds=3))
    watch = PeerWatch(store, rank, world, timeout_s=2.0)
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 2, 16, 64, generator=g)
    k = torch.randn(1, 2, 320, 64, generator=g)
    v = torch.randn(1, 2, 320, 64, generator=g)
    a, b = seq_shard(320, world, rank)
    record = {"rank": rank, "steps_done": [], "error": None}
    try:
        for step in range(4):
            if mode == "watch":
                watch.enter(step)
            o, _ = sharded_decode(q, k[:, :, a:b], v[:, :, a:b], 16, a, 320, group=group,
                                  out_dtype=torch.float64, partial_fn=_oracle_partial,
                                  merge_fn=_oracle_merge)
            record["steps_done"].append(step)
            record["o_sum"] = float(o.sum())
            if rank == leave_rank and step == leave_after:
                record["left"] = True
                break
    except RankDropped as e:
        record["error"] = {"kind": "RankDropped", "step": e.step, "missing": e.missing}
    except RuntimeError as e:  # the collective's timeout
        record["error"] = {"kind": "collective", "message": str(e)[:200]}
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(record, f)
    if rank == 0:
        # the store's server lives in rank 0: keep it up until the peers have read it
        import time
        time.sleep(1.0)
    # leave at once, as a rank that drops out does: the process group is not torn down, and
    # letting the interpreter destroy it under its running threads can abort the process
    os._exit(0)


@pytest.mark.parametrize("mode", ["watch", "collective"])
def test_rank_dropout_between_steps(tmp_path, mode):
    """world_size 3: rank 2 leaves after step 1. The survivors finish steps 0 and 1 with the
    right result and then end with an error instead of waiting: with the store watch they
    name rank 2 as missing at step 2 before launching anything of that step; without it the
    process group's 3 s timeout ends their step-2 all-gather."""
    import json
    world = 3
    mp.spawn(_dropout_worker, args=(world, _free_port(), 2, 1, mode, str(tmp_path)),
             nprocs=world, join=True)
    recs = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]
    assert recs[2].get("left") and recs[2]["steps_done"] == [0, 1] and recs[2]["error"] is None
    sums = {r["o_sum"] for r in recs}
    assert len(sums) == 1  # every rank merged the same result before the dropout
    for r in recs[:2]:
        assert r["steps_done"] == [0, 1], r
        if mode == "watch":
            assert r["error"] == {"kind": "RankDropped", "step": 2, "missing": [2]}, r
        else:
            assert r["error"]["kind"] == "collective", r
