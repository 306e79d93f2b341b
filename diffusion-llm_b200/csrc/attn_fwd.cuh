// Block-sparse attention forward on tcgen05 tensor cores (sm_100a).
//
// Replaces block_sparse_attention_fwd_kern (kernels/BlockSparseFlashAttention.py:76-172) for
// the training layout, and block_sparse_decode_kern (kernels/BlockSparseDecodeAttention.py:
// 41-110) for prefill-sized decode calls (q_len > 64).
//
// One CTA per (batch*head, 128-row query tile); key tiles of 128. Roles:
//   warps 0-3  softmax: thread t owns query row t (= TMEM lane t). Reads S from TMEM, masks
//              the partial tiles by exact per-row intervals, online softmax in the log2
//              domain with lazy rescaling (O is only rescaled when the running max grows by
//              more than 2^8), writes P back into TMEM as packed 16-bit pairs.
//   warp 4     TMA producer: Q once, then K and V tiles into a kFwdStages-deep ring.
//   warp 5     TMEM owner and UMMA issuer (one elected thread):
//              S[j&1] = Q K_j^T (SS form, M=128 N=128 K=64), then O += P_{j-1} V_{j-1}
//              (TS form: P from TMEM, V from shared memory, M=128 N=64 K=128).
// TMEM columns: S0 [0,128), S1 [128,256), O [256,320); P_j overwrites S[j&1] columns [0,64).
// All tiles use the 128-byte swizzle: Q and K are K-major operands, V is an MN-major operand.
#pragma once

#include "common.cuh"
#include "tile_ranges.h"

namespace bd3 {

constexpr int kD = 64;
constexpr int kFwdBM = 128;
constexpr int kFwdBN = 128;
constexpr int kFwdStages = 4;
constexpr int kFwdThreads = 192;
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
  // barriers: q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full, o_done
  static constexpr uint32_t kNumBars = 1 + 3 * kFwdStages + 2 + 2;
  static constexpr uint32_t kTmemSlot = kBar + kNumBars * 8;
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
  uint64_t* s_full = bars + 1 + 3 * kFwdStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = s_full + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + FwdSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int bh = blockIdx.x % (gridDim.x / p.num_q_tiles);
  const int BH = gridDim.x / p.num_q_tiles;
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
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 4 && lane_id() == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
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
  } else if (warp == 5) {
    // ---------------- UMMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_f16(128, 128, false, false, kBF16);
      constexpr uint32_t idesc_pv = idesc_f16(128, 64, false, true, kBF16);
      const uint32_t sbase = smem_u32(smem);
      const uint64_t qdesc = sw128_desc(sbase + FwdSmem::kQ, 16, 1024);
      bool ok = mbar_wait(q_full, 0);
      tc_fence_after();
      auto issue_pv = [&](int jj) {
        const int st = jj % kFwdStages;
        ok = ok && mbar_wait(p_full, jj & 1);
        ok = ok && mbar_wait(&v_full[st], (jj / kFwdStages) & 1);
        if (!ok) return;
        tc_fence_after();
        const uint64_t vdesc = sw128_desc(sbase + FwdSmem::kV + st * kTile16, kTile16, 1024);
        const uint32_t p_tmem = tmem + (jj & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + 256, p_tmem + kk * 8, vdesc + ((kk * 2048) >> 4), idesc_pv,
                  (jj > 0 || kk > 0) ? 1u : 0u);
        umma_commit(o_done);
        umma_commit(&kv_empty[st]);
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
    // ---------------- softmax: thread = query row ----------------
    const int row = threadIdx.x;
    const int qi = q_start + row;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
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
        float x[128];
        {
          uint32_t r[4][32];
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) tmem_ld32_async(tmem + lane_base + b * 128 + c4 * 32, r[c4]);
          tmem_ld_wait();
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            reg_fence(r[c4]);
#pragma unroll
            for (int i = 0; i < 32; ++i) x[c4 * 32 + i] = __uint_as_float(r[c4][i]);
          }
        }
        if (rule != 0) {
          const int lo = vlo - s, hi = vhi - s;
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c < lo || c >= hi) x[c] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 128; ++c) mx = fmaxf(mx, x[c]);
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
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int c = h2 * 64 + 2 * i;
            const float p0 = ex2(fmaf(x[c], p.scale_log2, -m_use));
            const float p1 = ex2(fmaf(x[c + 1], p.scale_log2, -m_use));
            sum += p0 + p1;
            pk[i] = pack2<kBF16>(p0, p1);
          }
          tmem_st32(tmem + lane_base + b * 128 + h2 * 32, pk);
        }
        l_run = l_run * alpha + sum;
        tmem_st_wait();
        if (j > 0) {
          ok = mbar_wait_warp(o_done, (j - 1) & 1);  // O += P_{j-1} V_{j-1} has landed
          if (!ok) break;
          tc_fence_after();
        }
        // the rescale's TMEM load/store is warp-collective: vote, and let the rows that do not
        // need it multiply by alpha = 1
        if (__any_sync(0xffffffffu, rescale)) {
          uint32_t r[2][32];
          tmem_ld32_async(tmem + lane_base + 256, r[0]);
          tmem_ld32_async(tmem + lane_base + 256 + 32, r[1]);
          tmem_ld_wait();
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            reg_fence(r[c2]);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              r[c2][i] = __float_as_uint(__uint_as_float(r[c2][i]) * alpha);
            tmem_st32(tmem + lane_base + 256 + c2 * 32, r[c2]);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(p_full);
      }
    }
    // epilogue: wait for the last O += P V, normalise, store O and LSE
    if (ok && j > 0) ok = mbar_wait_warp(o_done, (j - 1) & 1);
    // every lane of the warp takes part in the TMEM loads (.sync.aligned); only the stores
    // of rows past the end (a ragged last prefill tile) are skipped
    ok = __all_sync(0xffffffffu, ok);
    const int rows_valid = (kMode == kTrain) ? 2 * p.n : p.q_len;
    const bool store = qi < rows_valid;
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                      2 * (bb * p.o_sb + hh * p.o_sh + static_cast<long long>(qi) * p.o_ss);
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + 256 + c2 * 32, r);
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          packed[i] = pack2<kBF16>(__uint_as_float(r[2 * i]) * inv_l,
                                   __uint_as_float(r[2 * i + 1]) * inv_l);
        uint4* dst = reinterpret_cast<uint4*>(orow + c2 * 64);
        if (store) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                                packed[4 * i + 3]);
        }
      }
      if (store && p.lse != nullptr)
        p.lse[bb * p.lse_sb + hh * p.lse_sh + qi] = (m_use + __log2f(l_run)) * 0.69314718055994530942f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bd3
