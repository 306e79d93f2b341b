"""Multi-GPU partitioning of the attention path (one process per GPU, torch.distributed).

The reference is single-GPU; these are the two partitions the B200 build adds:

* Batch x head sharding (training attention, decode, block-sparse decode, generation):
  (batch, head) pairs are independent, so each rank takes a contiguous slice of them and
  no collective touches the data path. ``bh_shard`` gives a rank's slice.

* Sequence-sharded long-context decode: each rank holds a contiguous slice of the KV cache,
  computes a partial attention (O in fp32, natural-log LSE) of the same query block over
  its slice with the library's decode kernel, and one all-gather of the partials (NCCL over
  NVLink on GPUs) feeds the LSE-weighted merge (bd3_lse_merge, the math of
  kernels/SplitKVDecodeAttention.py:109-119). Peer memory is never read directly.

``sharded_decode`` takes the local-partial and merge functions as arguments so the same
partition logic runs on CPU ranks (gloo) in the tests with a checker in their place; on the
GPU the defaults are the library's kernels and there is no fallback.

Failure detection between steps (``PeerWatch``): before a step's first launch, every rank
posts that it reached the step in the process group's key-value store and waits, with a short
limit, for every peer's post. A rank that left between steps is named on the survivors
(``RankDropped``) before any of them launches a kernel or a collective of that step, so no
GPU is left waiting inside a collective for a peer that will never arrive.
"""

from __future__ import annotations

import datetime
from typing import Callable

import torch
import torch.distributed as dist


def bh_shard(B: int, H: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the flattened (batch * head) index range owned by ``rank``; the
    ranges tile [0, B*H) in rank order and differ in length by at most one."""
    total = B * H
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def seq_shard(kv_len: int, world: int, rank: int, align: int = 64) -> tuple[int, int]:
    """[start, stop) of the KV positions held by ``rank``: contiguous slices in rank order,
    boundaries on multiples of ``align`` (the decode kernel's key tile) except the end."""
    tiles = -(-kv_len // align)
    base, rem = divmod(tiles, world)
    t0 = rank * base + min(rank, rem)
    t1 = t0 + base + (1 if rank < rem else 0)
    return min(t0 * align, kv_len), min(t1 * align, kv_len)


def _gpu_partial(q, k, v, block_size, q_pos0, kv_pos0):
    from bd3attn import ops
    return ops.decode_raw(q, k, v, block_size, q_pos0=q_pos0, kv_pos0=kv_pos0,
                          out_dtype=torch.float32, return_lse=True)


def _gpu_merge(parts, lses, out_dtype):
    from bd3attn import ops
    return ops.lse_merge_raw(parts, lses, out_dtype)


class PeerMerge:
    """The exchange buffers of sharded_decode's merge over NVLink peer memory
    (bd3_peer_merge: every rank stores its partial straight into each peer's buffer and merges
    what the peers stored into its own, in one kernel, instead of an NCCL all-gather and a
    merge launch). One symmetric buffer per rank, mapped into every rank's process by torch's
    symmetric memory and zeroed once. One instance serves one (group, B, H, rows); its epoch
    advances by one per call, identically on every rank, since every rank calls it once per
    step. Collective to create."""

    def __init__(self, B: int, H: int, rows: int, group=None, device=None):
        import ctypes

        import torch.distributed._symmetric_memory as symm_mem

        from bd3attn._lib import LIB
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        nbytes = LIB.bd3_peer_merge_buffer_bytes(self.world, B, H, rows)
        if nbytes == 0:
            raise ValueError("peer merge: 2 <= world <= 8 and sizes >= 1")
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.buf = symm_mem.empty(nbytes // 4, dtype=torch.float32, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        self.ptrs = (ctypes.c_uint64 * self.world)(*self.handle.buffer_ptrs)
        self.shape = (B, H, rows)
        self.epoch = 0
        dist.barrier(group=self.group)  # every buffer is zeroed before a peer stores into it

    def merge(self, part_o: torch.Tensor, part_lse: torch.Tensor, out_dtype):
        """(O (B, H, rows, 64) in out_dtype, LSE (B, H, rows) fp32) of every rank's partial;
        part_o (B, H, rows, 64) fp32 and part_lse (B, H, rows) fp32 are this rank's."""
        from bd3attn import ops
        from bd3attn._lib import LIB, check, i64_array
        B, H, rows = self.shape
        part_o, part_lse = part_o.float().contiguous(), part_lse.float().contiguous()
        assert tuple(part_o.shape) == (B, H, rows, 64) and tuple(part_lse.shape) == (B, H, rows)
        self.epoch += 1
        o = torch.empty((B, H, rows, 64), dtype=out_dtype, device=part_o.device)
        lse = torch.empty((B, H, rows), dtype=torch.float32, device=part_o.device)
        with torch.cuda.device(part_o.device):
            check("bd3_peer_merge", LIB.bd3_peer_merge(
                ops._ptr(part_o), ops._ptr(part_lse), self.ptrs, self.world, self.rank,
                self.epoch, ops._ptr(o), ops._ptr(lse), B, H, rows,
                i64_array(ops._s3(o)), ops._code(out_dtype), ops._stream(part_o)))
        return o, lse


def sharded_decode(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                   block_size: int, kv_start: int, kv_len_total: int,
                   group=None, out_dtype=None,
                   partial_fn: Callable = _gpu_partial,
                   merge_fn: Callable = _gpu_merge,
                   peer: "PeerMerge | None" = None):
    """Decode attention of ``q`` (B, H, q_len, 64) over a KV cache sharded by sequence.

    k_local/v_local: (B, H, L_r, 64), this rank's keys at global positions
    [kv_start, kv_start + L_r). The queries sit at the last q_len of kv_len_total positions
    (the reference's placement). Returns (O (B, H, q_len, 64) in out_dtype, LSE), identical
    on every rank. A rank whose slice no query can see contributes LSE = -inf. With ``peer``
    (a PeerMerge of this shape) the partials meet over NVLink peer memory in one kernel;
    otherwise one all-gather of the process group moves them and ``merge_fn`` combines them.
    """
    world = dist.get_world_size(group)
    B, H, q_len, D = q.shape
    out_dtype = q.dtype if out_dtype is None else out_dtype
    q_pos0 = kv_len_total - q_len
    if k_local.shape[2] > 0:
        o, lse = partial_fn(q, k_local, v_local, block_size, q_pos0, kv_start)
        o = o.float()
        lse = lse.float()
    else:
        o = torch.zeros(B, H, q_len, D, dtype=torch.float32, device=q.device)
        lse = torch.full((B, H, q_len), float("-inf"), dtype=torch.float32, device=q.device)
    if peer is not None:
        return peer.merge(o, lse, out_dtype)
    # one all-gather of [O | LSE] per rank, packed so a single collective moves both
    packed = torch.cat([o.reshape(B, H, q_len * D), lse.reshape(B, H, q_len)], dim=-1)
    # ranks' blocks concatenated along dim 0 (the layout both NCCL and gloo produce)
    gathered = torch.empty((world * B,) + tuple(packed.shape[1:]), dtype=packed.dtype,
                           device=q.device)
    dist.all_gather_into_tensor(gathered, packed.contiguous(), group=group)
    gathered = gathered.view((world,) + tuple(packed.shape))
    parts = gathered[..., : q_len * D].reshape(world, B, H, q_len, D)
    lses = gathered[..., q_len * D:].reshape(world, B, H, q_len)
    return merge_fn(parts.contiguous(), lses.contiguous(), out_dtype)


class RankDropped(RuntimeError):
    """Peers did not reach a step within the watch's limit; ``missing`` lists their ranks."""

    def __init__(self, step: int, missing: list[int]):
        super().__init__(f"ranks {missing} did not reach step {step}")
        self.step = step
        self.missing = missing


class PeerWatch:
    """Host-side liveness check of the ranks of one job, run between steps.

    ``enter(step)`` sets the key ``<prefix>/<step>/<rank>`` in ``store`` (any
    torch.distributed Store: the TCPStore or FileStore of the process group) and waits up to
    ``timeout_s`` seconds for the same key of every rank. It raises RankDropped naming the
    ranks whose key is missing. Keys of finished steps are not deleted (a step index is never
    reused within a prefix).
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 2.0,
                 prefix: str = "bd3/step"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.prefix = prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def enter(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), "1")
        keys = [self._key(step, r) for r in range(self.world)]
        try:
            self.store.wait(keys, self.timeout)
        except Exception:  # the store's own timeout error; name who is missing
            missing = [r for r in range(self.world) if not self.store.check([keys[r]])]
            raise RankDropped(step, missing) from None
