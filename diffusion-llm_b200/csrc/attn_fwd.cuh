// Block-sparse attention forward on tcgen05 tensor cores (sm_100a).
//
// Replaces block_sparse_attention_fwd_kern (kernels/BlockSparseFlashAttention.py:76-172) for
// the training layout, and block_sparse_decode_kern (kernels/BlockSparseDecodeAttention.py:
// 41-110) for prefill-sized decode calls (q_len > 64).
//
// One CTA runs two 128-row query tiles of one (batch, head) as two independent streams,
// so the softmax of one stream overlaps the tensor-core work of the other:
//   training: stream A = noisy tile i, stream B = clean tile i (they share most key tiles and
//             together cost (i+2) + (i+1) key tiles; pairs are launched heaviest first);
//   prefill:  streams A, B = tiles 2p and 2p+1 (B may be empty for an odd tile count).
// Each stream has its own Q tile, its own K/V ring (kFwdStages deep, so the streams never
// wait on each other's loads), its own softmax warpgroup and its own TMEM: S (128 columns,
// with P written back over its first 64 as packed 16-bit pairs) and O (64 columns).
// Roles (320 threads):
//   warps 0-3  softmax of stream A: thread t owns query row t (TMEM lane t)
//   warps 4-7  softmax of stream B
//   warp 8     TMA: lane 0 feeds stream A, lane 1 stream B
//   warp 9     TMEM owner and UMMA issuer (one thread), alternating between the streams:
//              S_X = Q_X K^T (SS, M=128 N=128 K=64); O_X += P_X V (TS: P from TMEM, V an
//              MN-major smem operand, M=128 N=64 K=128).
// The softmax masks partial tiles by exact per-row intervals and runs an online softmax in
// the log2 domain with lazy rescaling (O is rescaled only when the running max grows by more
// than 2^8; the decision is voted per warp because the TMEM load/store is warp-collective).
#pragma once

#include "common.cuh"
#include "tile_ranges.h"

namespace bd3 {

constexpr int kD = 64;
constexpr int kFwdBM = 128;
constexpr int kFwdBN = 128;
constexpr int kFwdStages = 2;    // K/V ring depth per stream
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
  int num_pairs;         // CTAs per (batch, head)
  float scale_log2;      // softmax scale * log2(e)
};

struct FwdSmem {
  static constexpr uint32_t kQ = 0;                                  // [stream]
  static constexpr uint32_t kK = kQ + 2 * kTile16;                   // [stream][stage]
  static constexpr uint32_t kV = kK + 2 * kFwdStages * kTile16;      // [stream][stage]
  static constexpr uint32_t kBar = kV + 2 * kFwdStages * kTile16;
  // per stream: q_full, k_full[S], v_full[S], kv_empty[S], s_full, p_full, o_done
  static constexpr uint32_t kBarsPerStream = 1 + 3 * kFwdStages + 3;
  static constexpr uint32_t kTmemSlot = kBar + 2 * kBarsPerStream * 8;
  static constexpr uint32_t kBytes = kTmemSlot + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;  // room to align the base to 1 KB
};

struct StreamBars {
  uint64_t* q_full;
  uint64_t* k_full;
  uint64_t* v_full;
  uint64_t* kv_empty;
  uint64_t* s_full;
  uint64_t* p_full;
  uint64_t* o_done;
};

__device__ __forceinline__ StreamBars stream_bars(uint64_t* bars, int x) {
  uint64_t* b = bars + x * FwdSmem::kBarsPerStream;
  return StreamBars{b, b + 1, b + 1 + kFwdStages, b + 1 + 2 * kFwdStages,
                    b + 1 + 3 * kFwdStages, b + 2 + 3 * kFwdStages, b + 3 + 3 * kFwdStages};
}

// Query tiles (A, B) of linear pair index t within one (batch, head); B = -1 if none.
// Heaviest pairs first so the long programs start in the first wave.
__device__ __forceinline__ void fwd_pair(int t, const FwdParams& p, int mode, int* a, int* b) {
  if (mode == kTrain) {
    const int i = p.num_pairs - 1 - t;    // noisy tile i costs i+2 key tiles, clean tile i i+1
    *a = i;
    *b = p.num_pairs + i;
  } else {
    const int pp = p.num_pairs - 1 - t;
    *a = 2 * pp;
    *b = (2 * pp + 1 < p.num_q_tiles) ? 2 * pp + 1 : -1;
  }
}

template <int kMode>
__device__ __forceinline__ int fwd_make_ranges(const FwdParams& p, int q_start, Range* r) {
  if (kMode == kTrain) return fwd_ranges(q_start, kFwdBM, kFwdBN, p.n, p.bs, r);
  return decode_ranges(q_start, kFwdBM, kFwdBN, p.q_len, p.kv_len, p.bs, r);
}

__device__ __forceinline__ int count_tiles(const Range* r, int nr) {
  int c = 0;
  for (int i = 0; i < nr; ++i)
    if (r[i].hi > r[i].lo) c += cdiv(r[i].hi - r[i].lo, kFwdBN);
  return c;
}

// Start key of tile k of a range list (k counts tiles over all ranges, in order).
__device__ __forceinline__ int tile_start(const Range* r, int nr, int k) {
  for (int i = 0; i < nr; ++i) {
    if (r[i].hi <= r[i].lo) continue;
    const int c = cdiv(r[i].hi - r[i].lo, kFwdBN);
    if (k < c) return r[i].lo + k * kFwdBN;
    k -= c;
  }
  return -1;
}

// Softmax warpgroup of one stream: thread = query row qi of the tile starting at q_start.
template <int kMode, bool kBF16>
__device__ __forceinline__ void fwd_softmax(const FwdParams& p, const StreamBars& sb,
                                            const Range* rg, int nr, int q_start, int bb,
                                            int hh, uint32_t tS, uint32_t tO, int warp4) {
  const int row = threadIdx.x & 127;
  const int qi = q_start + row;
  const uint32_t lane_base = static_cast<uint32_t>(warp4 * 32) << 16;
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
      ok = mbar_wait_warp(sb.s_full, j & 1);
      if (!ok) break;
      tc_fence_after();
      float x[128];
      {
        uint32_t r[4][32];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) tmem_ld32_async(tS + lane_base + c4 * 32, r[c4]);
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
        tmem_st32(tS + lane_base + h2 * 32, pk);
      }
      l_run = l_run * alpha + sum;
      tmem_st_wait();
      if (j > 0) {
        ok = mbar_wait_warp(sb.o_done, (j - 1) & 1);  // O += P_{j-1} V_{j-1} has landed
        if (!ok) break;
        tc_fence_after();
      }
      // the rescale's TMEM load/store is warp-collective: vote, and let the rows that do not
      // need it multiply by alpha = 1
      if (__any_sync(0xffffffffu, rescale)) {
        uint32_t r[2][32];
        tmem_ld32_async(tO + lane_base, r[0]);
        tmem_ld32_async(tO + lane_base + 32, r[1]);
        tmem_ld_wait();
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          reg_fence(r[c2]);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            r[c2][i] = __float_as_uint(__uint_as_float(r[c2][i]) * alpha);
          tmem_st32(tO + lane_base + c2 * 32, r[c2]);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(sb.p_full);
    }
  }
  // epilogue: wait for the last O += P V, normalise, store O and LSE
  if (ok && j > 0) ok = mbar_wait_warp(sb.o_done, (j - 1) & 1);
  // every lane of the warp takes part in the TMEM loads (.sync.aligned); only the stores
  // of rows past the end (a ragged last prefill tile) are skipped
  ok = __all_sync(0xffffffffu, ok) && j > 0;
  const int rows_valid = (kMode == kTrain) ? 2 * p.n : p.q_len;
  const bool store = qi < rows_valid;
  if (ok) {
    tc_fence_after();
    const float inv_l = 1.f / l_run;
    const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
    uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                    2 * (bb * p.o_sb + hh * p.o_sh + static_cast<long long>(qi) * p.o_ss);
    uint32_t r[2][32];
    tmem_ld32_async(tO + lane_base, r[0]);
    tmem_ld32_async(tO + lane_base + 32, r[1]);
    tmem_ld_wait();
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      reg_fence(r[c2]);
      uint32_t packed[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        packed[i] = pack2<kBF16>(__uint_as_float(r[c2][2 * i]) * inv_l,
                                 __uint_as_float(r[c2][2 * i + 1]) * inv_l);
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

template <int kMode, bool kBF16>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FwdSmem::kBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + FwdSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int BH = gridDim.x / p.num_pairs;
  const int bh = blockIdx.x % BH;
  int tile[2];
  fwd_pair(blockIdx.x / BH, p, kMode, &tile[0], &tile[1]);
  const int bb = bh / p.H, hh = bh % p.H;

  Range rg[2][3];
  int nr[2] = {0, 0}, nt[2] = {0, 0};
#pragma unroll
  for (int x = 0; x < 2; ++x)
    if (tile[x] >= 0) {
      nr[x] = fwd_make_ranges<kMode>(p, tile[x] * kFwdBM, rg[x]);
      nt[x] = count_tiles(rg[x], nr[x]);
    }

  if (threadIdx.x == 0) {
    for (int x = 0; x < 2; ++x) {
      const StreamBars sb = stream_bars(bars, x);
      mbar_init(sb.q_full, 1);
      for (int s = 0; s < kFwdStages; ++s) {
        mbar_init(&sb.k_full[s], 1);
        mbar_init(&sb.v_full[s], 1);
        mbar_init(&sb.kv_empty[s], 1);
      }
      mbar_init(sb.s_full, 1);
      mbar_init(sb.p_full, 128);
      mbar_init(sb.o_done, 1);
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
  // TMEM columns: S_A [0,128), S_B [128,256), O_A [256,320), O_B [320,384)

  if (warp == 8) {
    // ---------------- TMA: lane x feeds stream x ----------------
    const int x = static_cast<int>(lane_id());
    if (x < 2 && nt[x] > 0) {
      const StreamBars sb = stream_bars(bars, x);
      uint8_t* sk = smem + FwdSmem::kK + x * kFwdStages * kTile16;
      uint8_t* sv = smem + FwdSmem::kV + x * kFwdStages * kTile16;
      bool ok = true;
      mbar_expect_tx(sb.q_full, kTile16);
      tma_load_4d(&tm_q, sb.q_full, smem + FwdSmem::kQ + x * kTile16, 0, tile[x] * kFwdBM, hh, bb);
      for (int k = 0; k < nt[x] && ok; ++k) {
        const int st = k % kFwdStages;
        if (k >= kFwdStages) ok = mbar_wait(&sb.kv_empty[st], ((k / kFwdStages) - 1) & 1);
        if (!ok) break;
        const int s = tile_start(rg[x], nr[x], k);
        mbar_expect_tx(&sb.k_full[st], kTile16);
        tma_load_4d(&tm_k, &sb.k_full[st], sk + st * kTile16, 0, s, hh, bb);
        mbar_expect_tx(&sb.v_full[st], kTile16);
        tma_load_4d(&tm_v, &sb.v_full[st], sv + st * kTile16, 0, s, hh, bb);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------- UMMA issuer, alternating between the streams ----------------
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_f16(128, 128, false, false, kBF16);
      constexpr uint32_t idesc_pv = idesc_f16(128, 64, false, true, kBF16);
      const uint32_t sbase = smem_u32(smem);
      bool ok = true;
      auto issue_s = [&](int x, int k) {
        const StreamBars sb = stream_bars(bars, x);
        const int st = k % kFwdStages;
        ok = ok && mbar_wait(&sb.k_full[st], (k / kFwdStages) & 1);
        if (!ok) return;
        tc_fence_after();
        const uint64_t qdesc = sw128_desc(sbase + FwdSmem::kQ + x * kTile16, 16, 1024);
        const uint64_t kdesc =
            sw128_desc(sbase + FwdSmem::kK + (x * kFwdStages + st) * kTile16, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_ss(tmem + x * 128, qdesc + kk * 2, kdesc + kk * 2, idesc_qk, kk > 0 ? 1u : 0u);
        umma_commit(sb.s_full);
      };
      auto issue_pv = [&](int x, int k) {
        const StreamBars sb = stream_bars(bars, x);
        const int st = k % kFwdStages;
        ok = ok && mbar_wait(sb.p_full, k & 1);
        ok = ok && mbar_wait(&sb.v_full[st], (k / kFwdStages) & 1);
        if (!ok) return;
        tc_fence_after();
        const uint64_t vdesc =
            sw128_desc(sbase + FwdSmem::kV + (x * kFwdStages + st) * kTile16, kTile16, 1024);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + 256 + x * 64, tmem + x * 128 + kk * 8, vdesc + ((kk * 2048) >> 4),
                  idesc_pv, (k > 0 || kk > 0) ? 1u : 0u);
        umma_commit(sb.o_done);
        umma_commit(&sb.kv_empty[st]);
      };
      bool q_ok[2] = {true, true};
      for (int x = 0; x < 2; ++x)
        if (nt[x] > 0) q_ok[x] = mbar_wait(stream_bars(bars, x).q_full, 0);
      ok = q_ok[0] && q_ok[1];
      for (int x = 0; x < 2; ++x)
        if (nt[x] > 0) issue_s(x, 0);
      const int kmax = nt[0] > nt[1] ? nt[0] : nt[1];
      for (int k = 0; k < kmax && ok; ++k) {
        for (int x = 0; x < 2; ++x) {
          if (k < nt[x]) {
            issue_pv(x, k);
            if (k + 1 < nt[x]) issue_s(x, k + 1);
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax: warpgroup x = stream x ----------------
    const int x = warp >> 2;
    if (tile[x] >= 0)
      fwd_softmax<kMode, kBF16>(p, stream_bars(bars, x), rg[x], nr[x], tile[x] * kFwdBM, bb, hh,
                                tmem + x * 128, tmem + 256 + x * 64, warp & 3);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bd3
