"""Tile-skipping key/query ranges of the reference kernels, restated in Python.

TEST INFRASTRUCTURE ONLY (see the package docstring).

Every function returns the list of ranges one program of the reference kernel visits, as
tuples (lo, hi, rule, shift): the program steps over tiles starting at lo, lo+TILE, ... < hi
and applies ``rule`` to each (0: no mask; 1: same block, the noisy diagonal; 2: clean
keys of earlier blocks, ``q_block >= kv_block + shift``; 3: the decode block-causal rule
with the kv_len bound). The formulas are parameterised by the tile sizes so that the same
restatement checks the reference tiling (128x64 forward, 128x32 dK/dV) and the tiling of
the CUDA kernels here, whose range code must produce exactly these tuples.

  fwd_ranges / dq_ranges  kernels/BlockSparseFlashAttention.py:133-153 and :420-440
  dkdv_ranges             kernels/BlockSparseFlashAttention.py:274-325
  decode_ranges           kernels/BlockSparseDecodeAttention.py:84-94
  split_ranges            kernels/SplitKVDecodeAttention.py:57-66
"""

from __future__ import annotations


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def fwd_ranges(q_start: int, block_m: int, block_n: int, n: int, bs: int):
    """Key ranges of one forward (or dQ) program over query rows [q_start, +block_m)."""
    r0, r1 = q_start, q_start + block_m - 1
    out = []
    if q_start < n:
        shift = 1
        lo_a = ((r0 // bs) * bs // block_n) * block_n
        hi_a = min((r1 // bs + 1) * bs, n)
        out.append((lo_a, hi_a, 1, shift))
        full = n + ((r0 // bs) * bs // block_n) * block_n
        hi = n + (r1 // bs) * bs
    else:
        shift = 0
        full = n + ((((r0 - n) // bs + 1) * bs) // block_n) * block_n
        hi = min(n + ((r1 - n) // bs + 1) * bs, 2 * n)
    out.append((n, full, 0, shift))
    out.append((full, hi, 2, shift))
    return out


dq_ranges = fwd_ranges


def dkdv_ranges(k_start: int, block_kv: int, block_q: int, n: int, bs: int):
    """Query ranges of one dK/dV program over keys [k_start, +block_kv)."""
    c0, c1 = k_start, k_start + block_kv - 1
    if k_start < n:
        lo = ((c0 // bs) * bs // block_q) * block_q
        hi = min((c1 // bs + 1) * bs, n)
        return [(lo, hi, 1, 0)]
    kb_first = (c0 - n) // bs
    kb_last = (c1 - n) // bs
    out = []
    lo = min(((kb_first + 1) * bs // block_q) * block_q, n)
    full = min(_cdiv((kb_last + 1) * bs, block_q) * block_q, n)
    out.append((lo, full, 2, 1))
    out.append((full, n, 0, 1))
    lo = n + (kb_first * bs // block_q) * block_q
    full = n + min(_cdiv(kb_last * bs, block_q) * block_q, n)
    out.append((lo, full, 2, 0))
    out.append((full, 2 * n, 0, 0))
    return out


def decode_ranges(q_start: int, block_m: int, block_n: int, q_len: int, kv_len: int,
                  bs: int):
    """Key ranges of one block-causal decode program over query rows [q_start, +block_m)."""
    q_offset = kv_len - q_len
    first_block = (q_offset + q_start) // bs
    last_row = min(q_start + block_m, q_len) - 1
    last_block = (q_offset + last_row) // bs
    full = min((first_block + 1) * bs, kv_len)
    full = (full // block_n) * block_n
    hi = min((last_block + 1) * bs, kv_len)
    return [(0, full, 0, 0), (full, hi, 3, 0)]


def split_ranges(split: int, split_n: int, block_n: int, q_len: int, kv_len: int, bs: int):
    """Key ranges of one split-KV program (all queries in one tile) over split ``split``."""
    q_offset = kv_len - q_len
    full = min((q_offset // bs + 1) * bs, kv_len)
    full = (full // block_n) * block_n
    lo = split * split_n
    hi = min(lo + split_n, kv_len)
    mid = min(max(full, lo), hi)
    return [(lo, mid, 0, 0), (mid, hi, 3, 0)]


def tiles(ranges, tile: int):
    """Expand ranges into (start, rule, shift) tiles, in visiting order."""
    out = []
    for lo, hi, rule, shift in ranges:
        for s in range(lo, hi, tile):
            out.append((s, rule, shift))
    return out


def rule_mask(rule: int, shift: int, q_idx, kv_idx, n: int, bs: int, kv_len: int = 0,
              q_len: int = 0):
    """Element mask one rule applies inside a tile (numpy broadcasting of q_idx x kv_idx).

    Rules 1/2 follow kernels/BlockSparseFlashAttention.py:54-61 (forward, dQ) and :197-203
    (dK/dV, identical predicates); rule 3 follows kernels/BlockSparseDecodeAttention.py:23-27.
    """
    import numpy as np

    if rule == 0:
        return np.ones(np.broadcast(q_idx, kv_idx).shape, dtype=bool)
    if rule == 3:
        q_block = (kv_len - q_len + q_idx) // bs
        return (q_block >= kv_idx // bs) & (kv_idx < kv_len)
    q_block = (q_idx % n) // bs
    kv_block = (kv_idx % n) // bs
    if rule == 1:
        return q_block == kv_block
    return q_block >= kv_block + shift
