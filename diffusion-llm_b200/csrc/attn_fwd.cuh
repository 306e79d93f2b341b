// Block-sparse attention forward on tcgen05 tensor cores (sm_100a), one query tile per item.
//
// Replaces block_sparse_decode_kern (kernels/BlockSparseDecodeAttention.py:41-110) for
// prefill-sized decode calls (q_len > 64): the library instantiates it in kDecode mode. The
// training layout (block_sparse_attention_fwd_kern, kernels/BlockSparseFlashAttention.py:
// 76-172) runs on attn_fwd_pair_kernel (attn_fwd_pair.cuh), which serves both query tiles
// that share a K/V stream at once; the kTrain branches below are that path's earlier form and
// are not instantiated. This header also holds the constants and TMA helpers both share.
//
// Persistent: one CTA per SM steps through (batch*head, 128-row query tile) work items,
// heaviest tiles first, with TMEM, barriers and the K/V ring kept across items and the Q tile
// double-buffered, so one item's prologue and epilogue overlap its neighbours' work. Key
// tiles are 128 wide. S = Q K_j^T is double-buffered in TMEM, so the tensor cores compute
// tile j+1 while the softmax works on tile j. The softmax is split by key columns between
// two warpgroups: each owns 64 of every tile's 128 keys for all 128 rows and keeps its own running max, row sum
// and O accumulator (an in-CTA split of the keys), and the two halves are merged once at the
// end with the split-KV weighting. No per-tile exchange between the warpgroups is needed.
// Roles (320 threads):
//   warps 0-3  softmax, key columns [0,64) of every tile: thread t owns query row t (TMEM lane
//              t); at each item's end they merge the halves and write O with a TMA store
//   warps 4-7  softmax, key columns [64,128)
//   warp 8     TMA producer: each item's Q tile, then its K and V tiles into the ring
//   warp 9     TMEM owner and UMMA issuer (one thread):
//              S[j&1] = Q K_j^T (SS, M=128 N=128 K=64), then for each half g
//              O_g += P_g V_j[64g, 64g+64) (TS: P_g from TMEM, V an MN-major smem operand)
// TMEM columns: S0 [0,128), S1 [128,256), O_0 [256,320), O_1 [320,384). Warpgroup g writes
// P_g (packed 16-bit pairs) over the S columns it has read, [64g, 64g+32) of the buffer.
// Each softmax runs in the log2 domain with lazy rescaling: O_g is rescaled only when its
// running max grows by more than 2^8, the decision voted per warp because the TMEM
// load/store is warp-collective.
#pragma once

#include "common.cuh"
#include "tile_ranges.h"

namespace bd3 {

constexpr int kD = 64;
constexpr int kFwdBM = 128;
constexpr int kFwdBN = 128;
constexpr int kFwdStages = 4;
// Column pairs (of a thread's 32 per tile) whose exponentials run on the FMA pipe
// (exp2_fma2) instead of MUFU: MUFU alone needs 1024 cycles per 128 x 128 tile.
constexpr int kFwdPolyPairs = 10;
constexpr int kFwdThreads = 320;
constexpr uint32_t kTile16 = 128u * 128u;  // a 128-row x 64-element 16-bit tile: 16 KB
constexpr float kRescaleLog2 = 8.0f;        // lazy-rescale threshold (log2 units)

enum FwdMode : int { kTrain = 0, kDecode = 1 };

struct FwdParams {
  void* o;
  float* lse;            // may be null (decode)
  long long o_sb, o_sh, o_ss;
  long long lse_sb, lse_sh;
  int H;
  int n;                 // training: half length; sequence length is 2n
  int q_len, kv_len;     // decode: rows and keys per (batch, head)
  int bs;                // block size
  int num_q_tiles;       // query tiles per (batch, head)
  int num_bh;            // batch * heads
  float scale_log2;      // softmax scale * log2(e)
};

struct FwdSmem {
  static constexpr uint32_t kQ = 0;                          // [item parity]
  static constexpr uint32_t kK = kQ + 2 * kTile16;
  static constexpr uint32_t kV = kK + kFwdStages * kTile16;
  static constexpr uint32_t kOut = kV + kFwdStages * kTile16;  // O staging for the TMA store
  static constexpr uint32_t kBar = kOut + kTile16;
  // q_full[2], q_empty[2], k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2],
  // o_done[2], o_free
  static constexpr uint32_t kNumBars = 4 + 3 * kFwdStages + 7;
  static constexpr uint32_t kMerge = kBar + kNumBars * 8;    // [item parity] warpgroup 1's m, l
  static constexpr uint32_t kTmemSlot = kMerge + 2 * 2 * 128 * 4;
  static constexpr uint32_t kBytes = kTmemSlot + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;  // room to align the base to 1 KB
};

// Query tile processed by linear CTA index `t` (within one batch*head column of the grid):
// heaviest tiles first so the long programs start in the first wave.
__device__ __forceinline__ int fwd_tile_order(int t, int num_q_tiles, int mode) {
  if (mode == kTrain) {
    const int half = num_q_tiles / 2;     // tiles per copy; noisy i costs i+2, clean i costs i+1
    const int i = half - 1 - (t >> 1);
    return (t & 1) ? half + i : i;
  }
  return num_q_tiles - 1 - t;
}

template <int kMode>
__device__ __forceinline__ int fwd_make_ranges(const FwdParams& p, int q_start, Range* r) {
  if (kMode == kTrain) return fwd_ranges(q_start, kFwdBM, kFwdBN, p.n, p.bs, r);
  return decode_ranges(q_start, kFwdBM, kFwdBN, p.q_len, p.kv_len, p.bs, r);
}

// TMA store of a 128-row x 64-element 16-bit box from shared memory (128-byte swizzle).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::
          "l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group_fwd() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group_read0_fwd() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group0_fwd() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Decode work item w of the persistent loop: its (batch*head) and query tile.
__device__ __forceinline__ void fwd_item(int w, const FwdParams& p, int mode, int* bh,
                                         int* q_tile) {
  *bh = w % p.num_bh;
  *q_tile = fwd_tile_order(w / p.num_bh, p.num_q_tiles, mode);
}

__device__ __forceinline__ int fwd_count_tiles(const Range* r, int nr) {
  int c = 0;
  for (int i = 0; i < nr; ++i)
    if (r[i].hi > r[i].lo) c += cdiv(r[i].hi - r[i].lo, kFwdBN);
  return c;
}

template <int kMode, bool kBF16>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FwdSmem::kBar);
  uint64_t* q_full = bars;                        // [item parity]
  uint64_t* q_empty = bars + 2;                   // [item parity]
  uint64_t* k_full = bars + 4;
  uint64_t* v_full = bars + 4 + kFwdStages;
  uint64_t* kv_empty = bars + 4 + 2 * kFwdStages;
  uint64_t* s_full = bars + 4 + 3 * kFwdStages;  // [buffer]
  uint64_t* p_full = s_full + 2;                  // [warpgroup]
  uint64_t* o_done = s_full + 4;                  // [warpgroup]
  uint64_t* o_free = s_full + 6;                  // the epilogue has read O_0 and O_1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + FwdSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int num_items = p.num_bh * p.num_q_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 128);
      mbar_init(&o_done[g], 1);
    }
    mbar_init(o_free, 128);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane_id() == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      bool ok = true;
      int J = 0;  // key tiles loaded so far by this CTA
      for (int it = 0, w = persistent_item(0); w < num_items && ok; w = persistent_item(++it)) {
        int bh, q_tile;
        fwd_item(w, p, kMode, &bh, &q_tile);
        const int bb = bh / p.H, hh = bh % p.H;
        Range rg[3];
        const int nr = fwd_make_ranges<kMode>(p, q_tile * kFwdBM, rg);
        const int qb = it & 1;
        if (it >= 2) ok = mbar_wait(&q_empty[qb], ((it >> 1) - 1) & 1);
        if (!ok) break;
        mbar_expect_tx(&q_full[qb], kTile16);
        tma_load_4d(&tm_q, &q_full[qb], smem + FwdSmem::kQ + qb * kTile16, 0, q_tile * kFwdBM, hh, bb);
        for (int ri = 0; ri < nr && ok; ++ri) {
          for (int s = rg[ri].lo; s < rg[ri].hi && ok; s += kFwdBN, ++J) {
            const int st = J % kFwdStages;
            if (J >= kFwdStages) ok = mbar_wait(&kv_empty[st], ((J / kFwdStages) - 1) & 1);
            if (!ok) break;
            mbar_expect_tx(&k_full[st], kTile16);
            tma_load_4d(&tm_k, &k_full[st], smem + FwdSmem::kK + st * kTile16, 0, s, hh, bb);
            mbar_expect_tx(&v_full[st], kTile16);
            tma_load_4d(&tm_v, &v_full[st], smem + FwdSmem::kV + st * kTile16, 0, s, hh, bb);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------- UMMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_f16(128, 128, false, false, kBF16);
      constexpr uint32_t idesc_pv = idesc_f16(128, 64, false, true, kBF16);
      const uint32_t sbase = smem_u32(smem);
      bool ok = true;
      // O_g += P_g V_J[64g, 64g+64) for both halves, then release the K/V stage; the first PV
      // of an item overwrites O, after the previous item's epilogue has read it
      auto issue_pv = [&](int Jg, bool first, int it) {
        const int st = Jg % kFwdStages;
        ok = ok && mbar_wait(&v_full[st], (Jg / kFwdStages) & 1);
        if (ok && first && it > 0) ok = mbar_wait(o_free, (it - 1) & 1);
        const uint32_t sbuf = tmem + (Jg & 1) * 128;
        for (int g = 0; g < 2 && ok; ++g) {
          ok = mbar_wait(&p_full[g], Jg & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t vdesc = sw128_desc(
              sbase + FwdSmem::kV + st * kTile16 + g * (kTile16 / 2), kTile16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts(tmem + 256 + g * 64, sbuf + g * 64 + kk * 8, vdesc + ((kk * 2048) >> 4),
                    idesc_pv, (!first || kk > 0) ? 1u : 0u);
          umma_commit(&o_done[g]);
        }
        if (ok) umma_commit(&kv_empty[st]);
      };
      // One flat loop over this CTA's key tiles across its items: S(J) is issued before
      // O += P V of tile J-1, also across item boundaries, so the S buffers never drain.
      int J = 0;                 // key tiles issued so far by this CTA
      int it = -1, w = 0, nt = 0, j = 0;
      uint64_t qdesc = 0;
      int prev_J = -1, prev_it = 0;
      bool prev_first = false;
      while (ok) {
        if (j == nt) {  // next item (an item always has at least one key tile)
          w = persistent_item(++it);
          if (w >= num_items) break;
          int bh, q_tile;
          fwd_item(w, p, kMode, &bh, &q_tile);
          Range rg[3];
          const int nr = fwd_make_ranges<kMode>(p, q_tile * kFwdBM, rg);
          nt = fwd_count_tiles(rg, nr);
          j = 0;
          const int qb = it & 1;
          ok = mbar_wait(&q_full[qb], (it >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          qdesc = sw128_desc(sbase + FwdSmem::kQ + qb * kTile16, 16, 1024);
        }
        const int st = J % kFwdStages;
        ok = mbar_wait(&k_full[st], (J / kFwdStages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint64_t kdesc = sw128_desc(sbase + FwdSmem::kK + st * kTile16, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_ss(tmem + (J & 1) * 128, qdesc + ((kk * 32) >> 4), kdesc + ((kk * 32) >> 4),
                  idesc_qk, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[J & 1]);
        if (j == nt - 1) umma_commit(&q_empty[it & 1]);  // this item's Q is no longer read
        if (prev_J >= 0) issue_pv(prev_J, prev_first, prev_it);
        prev_J = J;
        prev_first = (j == 0);
        prev_it = it;
        ++J;
        ++j;
      }
      if (ok && prev_J >= 0) issue_pv(prev_J, prev_first, prev_it);
    }
    __syncwarp();
  } else {
    // ---------------- softmax: warpgroup g owns key columns [64g, 64g+64) ----------------
    const int g = warp >> 2;
    const int row = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + lane_base + 256 + g * 64;
    bool ok = true;
    int J = 0;  // key tiles consumed so far by this CTA
    for (int it = 0, w = persistent_item(0); w < num_items; w = persistent_item(++it)) {
      int bh, q_tile;
      fwd_item(w, p, kMode, &bh, &q_tile);
      const int bb = bh / p.H, hh = bh % p.H;
      const int q_start = q_tile * kFwdBM;
      const int qi = q_start + row;
      Range rg[3];
      const int nr = fwd_make_ranges<kMode>(p, q_start, rg);
      float m_run = -INFINITY, l_run = 0.f;
      int j = 0;
      for (int ri = 0; ri < nr && ok; ++ri) {
        const int rule = rg[ri].rule, shift = rg[ri].shift;
        // visible key interval of this row under the range's rule (absolute key indices)
        int vlo = -2147483647, vhi = 2147483647;
        if (kMode == kTrain) {
          if (rule != 0) train_row_interval(rule, shift, qi, p.n, p.bs, &vlo, &vhi);
        } else if (rule == 3) {
          vlo = 0;
          vhi = decode_row_hi(p.kv_len - p.q_len + qi, p.bs, p.kv_len);
        }
        for (int s = rg[ri].lo; s < rg[ri].hi; s += kFwdBN, ++j) {
          const int Jg = J + j;
          const int b = Jg & 1;
          ok = mbar_wait_warp(&s_full[b], (Jg >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t tS = tmem + lane_base + b * 128 + g * 64;
          // this row's visible columns within this warpgroup's 64 (rule != 0 tiles only); a
          // warp whose 32 rows see none of them writes P = 0 and skips the exponentials
          const int lo = vlo - s - g * 64, hi = vhi - s - g * 64;
          const bool skip = rule != 0 && __all_sync(0xffffffffu, hi <= 0 || lo >= 64 || hi <= lo);
          float alpha = 1.f, sum = 0.f;
          bool rescale = false;
          if (skip) {
            uint32_t zero[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) zero[i] = 0u;
            tmem_st32(tS, zero);
          } else {
            float x[64];
            {
              uint32_t r[2][32];
              tmem_ld32_async(tS, r[0]);
              tmem_ld32_async(tS + 32, r[1]);
              tmem_ld_wait();
#pragma unroll
              for (int c2 = 0; c2 < 2; ++c2) {
                reg_fence(r[c2]);
#pragma unroll
                for (int i = 0; i < 32; ++i) x[c2 * 32 + i] = __uint_as_float(r[c2][i]);
              }
            }
            if (rule != 0) {
#pragma unroll
              for (int c = 0; c < 64; ++c)
                if (c < lo || c >= hi) x[c] = -INFINITY;
            }
            const float mx = max64(x) * p.scale_log2;
            const float m_new = fmaxf(m_run, mx);
            if (m_new - m_run > kRescaleLog2) {  // false for NaN (-inf - -inf)
              alpha = ex2(m_run - m_new);        // 0 when m_run = -inf
              rescale = (j > 0);
              m_run = m_new;
            }
            const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
            // P = 2^(x * scale - m): kFwdPolyPairs of the 32 column pairs on the FMA pipe, the
            // rest on MUFU, so that the two units share the exponentials
            const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
            const float2 nm2 = make_float2(-m_use, -m_use);
            float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float2 t = __ffma2_rn(make_float2(x[2 * i], x[2 * i + 1]), sc2, nm2);
              float2 e;
              if ((i * kFwdPolyPairs) / 32 != ((i + 1) * kFwdPolyPairs) / 32)
                e = exp2_fma2(t);
              else
                e = make_float2(ex2(t.x), ex2(t.y));
              acc[i & 3] = __fadd2_rn(acc[i & 3], e);
              pk[i] = pack2<kBF16>(e.x, e.y);
            }
            const float2 a01 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
            sum = a01.x + a01.y;
            tmem_st32(tS, pk);  // P_g over this warpgroup's own (already read) S columns
          }
          l_run = l_run * alpha + sum;
          tmem_st_wait();
          if (j > 0) {
            ok = mbar_wait_warp(&o_done[g], (Jg - 1) & 1);  // O_g += P_g V has landed
            if (!ok) break;
            tc_fence_after();
          }
          // the rescale's TMEM load/store is warp-collective: vote, and let the rows that do
          // not need it multiply by alpha = 1
          if (__any_sync(0xffffffffu, rescale)) {
            uint32_t r[2][32];
            tmem_ld32_async(tO, r[0]);
            tmem_ld32_async(tO + 32, r[1]);
            tmem_ld_wait();
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
              reg_fence(r[c2]);
#pragma unroll
              for (int i = 0; i < 32; ++i)
                r[c2][i] = __float_as_uint(__uint_as_float(r[c2][i]) * alpha);
              tmem_st32(tO + c2 * 32, r[c2]);
            }
            tmem_st_wait();
          }
          tc_fence_before();
          mbar_arrive(&p_full[g]);
        }
      }
      // ---- epilogue: both halves' last O_g += P_g V have landed; warpgroup 1 hands its
      // (max, sum) to warpgroup 0, which merges O_0 and O_1, stores O and the LSE, and frees
      // the accumulators for the next item ----
      if (ok && j > 0) ok = mbar_wait_warp(&o_done[g], (J + j - 1) & 1);
      ok = __all_sync(0xffffffffu, ok);
      float* merge_m = reinterpret_cast<float*>(smem + FwdSmem::kMerge) + (it & 1) * 256;
      float* merge_l = merge_m + 128;
      if (g == 1) {
        merge_m[row] = m_run;
        merge_l[row] = l_run;
      }
      tc_fence_before();
      {  // both warpgroups meet here once per item and agree on whether to go on
        uint32_t all;
        asm volatile(
            "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 256, p;\n"
            " selp.u32 %0, 1, 0, q;\n}\n"
            : "=r"(all)
            : "r"(static_cast<uint32_t>(ok))
            : "memory");
        ok = all != 0;
      }
      tc_fence_after();
      if (g == 0 && ok && j > 0) {
        const float m1 = merge_m[row], l1 = merge_l[row];
        const float M = fmaxf(m_run, m1);
        const float Mu = (M == -INFINITY) ? 0.f : M;
        const float w0 = ex2(m_run - Mu), w1 = ex2(m1 - Mu);  // 0 for a half that saw no key
        const float L = l_run * w0 + l1 * w1;
        const float a0 = w0 / L, a1 = w1 / L;
        const int rows_valid = (kMode == kTrain) ? 2 * p.n : p.q_len;
        uint32_t r0[2][32], r1[2][32];
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          tmem_ld32_async(tmem + lane_base + 256 + c2 * 32, r0[c2]);
          tmem_ld32_async(tmem + lane_base + 320 + c2 * 32, r1[c2]);
        }
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(o_free);  // O_0 and O_1 are in registers: the next item may overwrite them
        // O goes out through a swizzled shared-memory tile and one TMA store (rows past the
        // end of a ragged prefill tile are clipped by the tensor map)
        const bool leader = (threadIdx.x == 0);
        uint8_t* stage = smem + FwdSmem::kOut;
        if (leader) bulk_wait_group_read0_fwd();  // the previous item's store has read it
        asm volatile("bar.sync 2, 128;" ::: "memory");
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          reg_fence(r0[c2]);
          reg_fence(r1[c2]);
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            packed[i] = pack2<kBF16>(
                __uint_as_float(r0[c2][2 * i]) * a0 + __uint_as_float(r1[c2][2 * i]) * a1,
                __uint_as_float(r0[c2][2 * i + 1]) * a0 + __uint_as_float(r1[c2][2 * i + 1]) * a1);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<uint4*>(stage + sw128_offset(row, c2 * 4 + i)) =
                make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
        }
        fence_proxy_async_smem();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (leader) {
          tma_store_4d(&tm_o, stage, 0, q_start, hh, bb);
          bulk_commit_group_fwd();
        }
        if (qi < rows_valid && p.lse != nullptr)
          p.lse[bb * p.lse_sb + hh * p.lse_sh + qi] = (Mu + __log2f(L)) * 0.69314718055994530942f;
      } else if (g == 0) {
        mbar_arrive(o_free);  // keep the phase count in step with the issuer
      }
      J += j;
      if (!ok) break;
    }
  }
  if (threadIdx.x == 0) bulk_wait_group0_fwd();  // the last O store has landed
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bd3
