// Block-sparse attention forward on tcgen05 tensor cores (sm_100a).
//
// Replaces block_sparse_attention_fwd_kern (kernels/BlockSparseFlashAttention.py:76-172) for
// the training layout, and block_sparse_decode_kern (kernels/BlockSparseDecodeAttention.py:
// 41-110) for prefill-sized decode calls (q_len > 64).
//
// One CTA per (batch*head, 128-row query tile); key tiles of 128, visited heaviest tile first.
// S = Q K_j^T is double-buffered in TMEM, so the tensor cores compute tile j+1 while the
// softmax works on tile j. The softmax is split by key columns between two warpgroups: each
// owns 64 of every tile's 128 keys for all 128 rows and keeps its own running max, row sum
// and O accumulator (an in-CTA split of the keys), and the two halves are merged once at the
// end with the split-KV weighting. No per-tile exchange between the warpgroups is needed.
// Roles (320 threads):
//   warps 0-3  softmax, key columns [0,64) of every tile: thread t owns query row t (TMEM lane t)
//   warps 4-7  softmax, key columns [64,128)
//   warp 8     TMA producer: Q once, then K and V tiles into a kFwdStages-deep ring
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
  float scale_log2;      // softmax scale * log2(e)
};

struct FwdSmem {
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK = kQ + kTile16;
  static constexpr uint32_t kV = kK + kFwdStages * kTile16;
  static constexpr uint32_t kBar = kV + kFwdStages * kTile16;
  // q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2], o_done[2]
  static constexpr uint32_t kNumBars = 1 + 3 * kFwdStages + 6;
  static constexpr uint32_t kMerge = kBar + kNumBars * 8;    // warpgroup 1's (m, l) per row
  static constexpr uint32_t kTmemSlot = kMerge + 2 * 128 * 4;
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

template <int kMode, bool kBF16>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FwdSmem::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 1 + kFwdStages;
  uint64_t* kv_empty = bars + 1 + 2 * kFwdStages;
  uint64_t* s_full = bars + 1 + 3 * kFwdStages;  // [buffer]
  uint64_t* p_full = s_full + 2;                  // [warpgroup]
  uint64_t* o_done = s_full + 4;                  // [warpgroup]
  float* merge_m = reinterpret_cast<float*>(smem + FwdSmem::kMerge);
  float* merge_l = merge_m + 128;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + FwdSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int BH = gridDim.x / p.num_q_tiles;
  const int bh = blockIdx.x % BH;
  const int q_tile = fwd_tile_order(blockIdx.x / BH, p.num_q_tiles, kMode);
  const int q_start = q_tile * kFwdBM;
  const int bb = bh / p.H, hh = bh % p.H;

  Range rg[3];
  const int nr = fwd_make_ranges<kMode>(p, q_start, rg);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
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
      mbar_expect_tx(q_full, kTile16);
      tma_load_4d(&tm_q, q_full, smem + FwdSmem::kQ, 0, q_start, hh, bb);
      int j = 0;
      for (int ri = 0; ri < nr && ok; ++ri) {
        for (int s = rg[ri].lo; s < rg[ri].hi && ok; s += kFwdBN, ++j) {
          const int st = j % kFwdStages;
          if (j >= kFwdStages) ok = mbar_wait(&kv_empty[st], ((j / kFwdStages) - 1) & 1);
          if (!ok) break;
          mbar_expect_tx(&k_full[st], kTile16);
          tma_load_4d(&tm_k, &k_full[st], smem + FwdSmem::kK + st * kTile16, 0, s, hh, bb);
          mbar_expect_tx(&v_full[st], kTile16);
          tma_load_4d(&tm_v, &v_full[st], smem + FwdSmem::kV + st * kTile16, 0, s, hh, bb);
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
      const uint64_t qdesc = sw128_desc(sbase + FwdSmem::kQ, 16, 1024);
      bool ok = mbar_wait(q_full, 0);
      tc_fence_after();
      // O_g += P_g V_jj[64g, 64g+64) for both halves, then release the K/V stage
      auto issue_pv = [&](int jj) {
        const int st = jj % kFwdStages;
        ok = ok && mbar_wait(&v_full[st], (jj / kFwdStages) & 1);
        const uint32_t sbuf = tmem + (jj & 1) * 128;
        for (int g = 0; g < 2 && ok; ++g) {
          ok = mbar_wait(&p_full[g], jj & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t vdesc = sw128_desc(
              sbase + FwdSmem::kV + st * kTile16 + g * (kTile16 / 2), kTile16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts(tmem + 256 + g * 64, sbuf + g * 64 + kk * 8, vdesc + ((kk * 2048) >> 4),
                    idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&o_done[g]);
        }
        if (ok) umma_commit(&kv_empty[st]);
      };
      int j = 0;
      for (int ri = 0; ri < nr && ok; ++ri) {
        for (int s = rg[ri].lo; s < rg[ri].hi && ok; s += kFwdBN, ++j) {
          const int st = j % kFwdStages;
          ok = mbar_wait(&k_full[st], (j / kFwdStages) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t kdesc = sw128_desc(sbase + FwdSmem::kK + st * kTile16, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ss(tmem + (j & 1) * 128, qdesc + ((kk * 32) >> 4), kdesc + ((kk * 32) >> 4),
                    idesc_qk, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[j & 1]);
          if (j > 0) issue_pv(j - 1);
        }
      }
      if (ok && j > 0) issue_pv(j - 1);
    }
    __syncwarp();
  } else {
    // ---------------- softmax: warpgroup g owns key columns [64g, 64g+64) ----------------
    const int g = warp >> 2;
    const int row = threadIdx.x & 127;
    const int qi = q_start + row;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + lane_base + 256 + g * 64;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
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
        const int b = j & 1;
        ok = mbar_wait_warp(&s_full[b], (j >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t tS = tmem + lane_base + b * 128 + g * 64;
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
          const int lo = vlo - s - g * 64, hi = vhi - s - g * 64;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c < lo || c >= hi) x[c] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) mx = fmaxf(mx, x[c]);
        mx *= p.scale_log2;
        const float m_new = fmaxf(m_run, mx);
        float alpha = 1.f;
        bool rescale = false;
        if (m_new - m_run > kRescaleLog2) {  // false for NaN (-inf - -inf)
          alpha = ex2(m_run - m_new);        // 0 when m_run = -inf
          rescale = (j > 0);
          m_run = m_new;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        float sum = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p0 = ex2(fmaf(x[2 * i], p.scale_log2, -m_use));
          const float p1 = ex2(fmaf(x[2 * i + 1], p.scale_log2, -m_use));
          sum += p0 + p1;
          pk[i] = pack2<kBF16>(p0, p1);
        }
        tmem_st32(tS, pk);  // P_g over this warpgroup's own (already read) S columns
        l_run = l_run * alpha + sum;
        tmem_st_wait();
        if (j > 0) {
          ok = mbar_wait_warp(&o_done[g], (j - 1) & 1);  // O_g += P_g V has landed
          if (!ok) break;
          tc_fence_after();
        }
        // the rescale's TMEM load/store is warp-collective: vote, and let the rows that do not
        // need it multiply by alpha = 1
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
    // (max, sum) to warpgroup 0, which merges O_0 and O_1 and stores O and the LSE ----
    if (ok && j > 0) ok = mbar_wait_warp(&o_done[g], (j - 1) & 1);
    ok = __all_sync(0xffffffffu, ok) && j > 0;
    if (g == 1) {
      merge_m[row] = m_run;
      merge_l[row] = l_run;
    }
    tc_fence_before();
    asm volatile("bar.sync 1, 256;" ::: "memory");
    tc_fence_after();
    if (g == 0 && ok) {
      const float m1 = merge_m[row], l1 = merge_l[row];
      const float M = fmaxf(m_run, m1);
      const float Mu = (M == -INFINITY) ? 0.f : M;
      const float w0 = ex2(m_run - Mu), w1 = ex2(m1 - Mu);  // 0 for a half that saw no key
      const float L = l_run * w0 + l1 * w1;
      const float a0 = w0 / L, a1 = w1 / L;
      const int rows_valid = (kMode == kTrain) ? 2 * p.n : p.q_len;
      const bool store = qi < rows_valid;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                      2 * (bb * p.o_sb + hh * p.o_sh + static_cast<long long>(qi) * p.o_ss);
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t r0[32], r1[32];
        tmem_ld32_async(tmem + lane_base + 256 + c2 * 32, r0);
        tmem_ld32_async(tmem + lane_base + 320 + c2 * 32, r1);
        tmem_ld_wait();
        reg_fence(r0);
        reg_fence(r1);
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = pack2<kBF16>(
              __uint_as_float(r0[2 * i]) * a0 + __uint_as_float(r1[2 * i]) * a1,
              __uint_as_float(r0[2 * i + 1]) * a0 + __uint_as_float(r1[2 * i + 1]) * a1);
        uint4* dst = reinterpret_cast<uint4*>(orow + c2 * 64);
        if (store) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                                packed[4 * i + 3]);
        }
      }
      if (store && p.lse != nullptr)
        p.lse[bb * p.lse_sb + hh * p.lse_sh + qi] = (Mu + __log2f(L)) * 0.69314718055994530942f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bd3
