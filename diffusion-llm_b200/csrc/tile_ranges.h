// Tile-skipping ranges and per-row visible intervals of the BD3-LM masks.
//
// One __host__ __device__ implementation serves the kernels and the C-ABI export
// bd3_debug_ranges(), through which the CPU tests compare it with the restatement of the
// reference formulas. The formulas are the reference's, evaluated at this library's tile
// sizes:
//   forward / dQ key ranges   kernels/BlockSparseFlashAttention.py:133-153 (:420-440)
//   dK/dV query ranges        kernels/BlockSparseFlashAttention.py:274-325
//   decode key ranges         kernels/BlockSparseDecodeAttention.py:84-94
// Rules: 0 no mask; 1 same block (noisy diagonal); 2 clean keys, q_block >= kv_block + shift;
// 3 decode block-causal with the kv_len bound.
#pragma once

#ifdef __CUDACC__
#define BD3_HD __host__ __device__ __forceinline__
#else
#define BD3_HD inline
#endif

namespace bd3 {

struct Range {
  int lo, hi, rule, shift;
};

BD3_HD int imin(int a, int b) { return a < b ? a : b; }
BD3_HD int imax(int a, int b) { return a > b ? a : b; }
BD3_HD int cdiv(int a, int b) { return (a + b - 1) / b; }

// Key ranges of the program over query rows [q_start, q_start + bm) of the 2n training
// sequence, for a noisy program (q_start < n): rule 1 over its own noisy blocks, then rule 0
// and rule 2 (shift 1) over the clean keys.
BD3_HD void fwd_ranges_noisy(int q_start, int bm, int bn, int n, int bs, Range& a, Range& b,
                             Range& c) {
  const int r0 = q_start, r1 = q_start + bm - 1;
  const int lo_a = ((r0 / bs) * bs / bn) * bn;
  const int hi_a = imin((r1 / bs + 1) * bs, n);
  a = Range{lo_a, hi_a, 1, 1};
  const int full = n + ((r0 / bs) * bs / bn) * bn;
  const int hi = n + (r1 / bs) * bs;
  b = Range{n, full, 0, 1};
  c = Range{full, hi, 2, 1};
}

// The same for a clean program (q_start >= n): rule 0, then rule 2 (shift 0).
BD3_HD void fwd_ranges_clean(int q_start, int bm, int bn, int n, int bs, Range& b, Range& c) {
  const int r0 = q_start, r1 = q_start + bm - 1;
  const int full = n + ((((r0 - n) / bs + 1) * bs) / bn) * bn;
  const int hi = imin(n + ((r1 - n) / bs + 1) * bs, 2 * n);
  b = Range{n, full, 0, 0};
  c = Range{full, hi, 2, 0};
}

// Both, as the reference's program computes them: returns the number of ranges written to
// out (3 for noisy tiles, 2 for clean).
BD3_HD int fwd_ranges(int q_start, int bm, int bn, int n, int bs, Range* out) {
  if (q_start < n) {
    fwd_ranges_noisy(q_start, bm, bn, n, bs, out[0], out[1], out[2]);
    return 3;
  }
  fwd_ranges_clean(q_start, bm, bn, n, bs, out[0], out[1]);
  return 2;
}

// Query ranges of the program over keys [k_start, k_start + bkv). Returns 1 or 4.
BD3_HD int dkdv_ranges(int k_start, int bkv, int bq, int n, int bs, Range* out) {
  const int c0 = k_start, c1 = k_start + bkv - 1;
  if (k_start < n) {
    const int lo = ((c0 / bs) * bs / bq) * bq;
    const int hi = imin((c1 / bs + 1) * bs, n);
    out[0] = Range{lo, hi, 1, 0};
    return 1;
  }
  const int kb_first = (c0 - n) / bs, kb_last = (c1 - n) / bs;
  int lo = imin(((kb_first + 1) * bs / bq) * bq, n);
  int full = imin(cdiv((kb_last + 1) * bs, bq) * bq, n);
  out[0] = Range{lo, full, 2, 1};
  out[1] = Range{full, n, 0, 1};
  lo = n + (kb_first * bs / bq) * bq;
  full = n + imin(cdiv(kb_last * bs, bq) * bq, n);
  out[2] = Range{lo, full, 2, 0};
  out[3] = Range{full, 2 * n, 0, 0};
  return 4;
}

// Key ranges of the decode program over query rows [q_start, q_start + bm); the queries are
// the last q_len of kv_len positions. Returns 2.
BD3_HD int decode_ranges(int q_start, int bm, int bn, int q_len, int kv_len, int bs,
                         Range* out) {
  const int q_offset = kv_len - q_len;
  const int first_block = (q_offset + q_start) / bs;
  const int last_row = imin(q_start + bm, q_len) - 1;
  const int last_block = (q_offset + last_row) / bs;
  int full = imin((first_block + 1) * bs, kv_len);
  full = (full / bn) * bn;
  const int hi = imin((last_block + 1) * bs, kv_len);
  out[0] = Range{0, full, 0, 0};
  out[1] = Range{full, hi, 3, 0};
  return 2;
}

// Visible key interval [lo, hi) of query `q` (training sequence index) under a rule, in
// absolute key indices. The rules' predicates are intervals per row:
//   rule 1: (kv % n)/bs == (q % n)/bs       -> kv in [blk*bs, (blk+1)*bs)
//   rule 2: (q % n)/bs >= (kv - n)/bs + s   -> kv in [n, n + (q_block - s + 1)*bs)
// (rule 1 is only used on keys < n and rule 2 only on keys >= n.)
BD3_HD void train_row_interval(int rule, int shift, int q, int n, int bs, int* lo, int* hi) {
  const int qb = (q % n) / bs;
  if (rule == 1) {
    *lo = qb * bs;
    *hi = (qb + 1) * bs;
  } else if (rule == 2) {
    *lo = n;
    *hi = n + (qb - shift + 1) * bs;  // empty when qb - shift + 1 <= 0
  } else {
    *lo = -2147483647;
    *hi = 2147483647;
  }
}

// Same for the dK/dV direction: visible QUERY interval of key `kv` under a rule.
//   rule 1: q in [kb*bs, (kb+1)*bs) (noisy queries of the key's block)
//   rule 2: (q % n)/bs >= kb + s    -> q in [base + (kb + s)*bs, base + n) with base = n
//           for clean queries (q >= n) and 0 for noisy ones
BD3_HD void dkdv_col_interval(int rule, int shift, int kv, int q_base, int n, int bs, int* lo,
                              int* hi) {
  const int kb = (kv % n) / bs;
  if (rule == 1) {
    *lo = kb * bs;
    *hi = (kb + 1) * bs;
  } else if (rule == 2) {
    *lo = q_base + (kb + shift) * bs;
    *hi = q_base + n;
  } else {
    *lo = -2147483647;
    *hi = 2147483647;
  }
}

// Decode rule 3: visible keys of query row r are [0, min((blk + 1)*bs, kv_len)) with
// blk = (q_pos0 + r)/bs, minus keys before kv_pos0 (the shard's first global position).
BD3_HD int decode_row_hi(int q_pos, int bs, int kv_end) {
  return imin((q_pos / bs + 1) * bs, kv_end);
}

}  // namespace bd3
