// Block-sparse attention backward on tcgen05 tensor cores (sm_100a).
//
// Replaces BlockSparseFlashAttention.backward (kernels/BlockSparseFlashAttention.py:509-562):
//   bwd_delta_kernel   Delta = rowsum(dO * O) in fp32 (the host op at :525)
//   bwd_dq_kernel      dQ = scale * sum_j dS_j K_j over the forward's key ranges
//                      (block_sparse_attention_bwd_dq_kern, :369-452)
//   bwd_dkdv_kernel    dV = sum_i P_i^T dO_i, dK = scale * sum_i dS_i^T Q_i over the query
//                      ranges of one key tile (block_sparse_attention_dk_dv_bwd_kern, :213-328);
//                      one CTA owns each key tile, so dK and dV are deterministic.
// with P = exp(scale * Q K^T - LSE) masked to 0 and dS = P * (dO V^T - Delta).
//
// Both tile kernels compute S = Q K^T and dP = dO V^T with the query rows on the TMEM lanes
// (M = 128 queries, N = 128 keys), so every softmax thread owns one query row and keeps that
// row's LSE and Delta in registers.
//   dQ kernel:   dS is written back into the S columns of TMEM as packed 16-bit pairs and
//                consumed by a TS-form MMA: dQ[q, :] += dS[q, keys] K[keys, :].
//   dK/dV kernel: P and dS are written to shared memory as [query][key] 128-byte-swizzled
//                tiles; the same bytes are the MN-major A operand of dV += P^T dO and
//                dK += dS^T Q (M = 128 keys, N = 64, K = 128 queries).
#pragma once

#include "attn_fwd.cuh"
#include "common.cuh"
#include "tile_ranges.h"

namespace bd3 {

constexpr int kBwdBKV = 128;   // dK/dV: keys per CTA
constexpr int kBwdBQ = 128;    // dK/dV: queries per step
constexpr int kBwdDqBM = 128;  // dQ: queries per CTA
constexpr int kBwdDqBN = 128;  // dQ: keys per step
constexpr int kBwdStages = 2;
constexpr int kBwdThreads = 192;

struct BwdParams {
  const void* o;
  const void* dout;
  const float* lse;      // (B, H, 2n)
  float* delta;          // (B, H, 2n), written by bwd_delta_kernel
  void* dq;
  void* dk;
  void* dv;
  long long o_sb, o_sh, o_ss, do_sb, do_sh, do_ss;
  long long dq_sb, dq_sh, dq_ss, dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  int H, n, bs;
  int num_tiles;         // query tiles (dQ) or key tiles (dK/dV) per (batch, head)
  float scale, scale_log2;
};

// Delta[bh, r] = sum_d dO[r, d] * O[r, d]; 8 threads per row, 16 bytes each.
template <bool kBF16>
__global__ void __launch_bounds__(256) bwd_delta_kernel(const BwdParams p, int rows_total) {
  const int gid = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = gid >> 3, part = gid & 7;
  float acc = 0.f;
  if (row < rows_total) {
    const int S = 2 * p.n;
    const int bh = row / S, r = row % S;
    const int bb = bh / p.H, hh = bh % p.H;
    const uint4 a = *reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint16_t*>(p.dout) + bb * p.do_sb + hh * p.do_sh + r * p.do_ss + part * 8);
    const uint4 b = *reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint16_t*>(p.o) + bb * p.o_sb + hh * p.o_sh + r * p.o_ss + part * 8);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = unpack2<kBF16>(av[i]), y = unpack2<kBF16>(bv[i]);
      acc = fmaf(x.x, y.x, acc);
      acc = fmaf(x.y, y.y, acc);
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (row < rows_total && part == 0) p.delta[row] = acc;
}

// Store 64 fp32 accumulator columns of one row (read from TMEM) as 16-bit values * mul.
template <bool kBF16>
__device__ __forceinline__ void store_row64(uint32_t taddr, void* dst, float mul) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c2 = 0; c2 < 2; ++c2) {
    uint32_t r[32];
    tmem_ld32(taddr + c2 * 32, r);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      d4[c2 * 4 + i] = make_uint4(
          pack2<kBF16>(__uint_as_float(r[8 * i + 0]) * mul, __uint_as_float(r[8 * i + 1]) * mul),
          pack2<kBF16>(__uint_as_float(r[8 * i + 2]) * mul, __uint_as_float(r[8 * i + 3]) * mul),
          pack2<kBF16>(__uint_as_float(r[8 * i + 4]) * mul, __uint_as_float(r[8 * i + 5]) * mul),
          pack2<kBF16>(__uint_as_float(r[8 * i + 6]) * mul, __uint_as_float(r[8 * i + 7]) * mul));
  }
}

// ---------------------------------------------------------------------------------------
// dQ: one CTA per (batch*head, 128-query tile), stepping over the forward's key ranges.
struct DqSmem {
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kDO = kQ + kTile16;
  static constexpr uint32_t kK = kDO + kTile16;
  static constexpr uint32_t kV = kK + kBwdStages * kTile16;
  static constexpr uint32_t kBar = kV + kBwdStages * kTile16;
  // qo_full, kv_full[S], kv_empty[S], s_full, ds_full, dq_done
  static constexpr uint32_t kNumBars = 1 + 2 * kBwdStages + 3;
  static constexpr uint32_t kTmemSlot = kBar + kNumBars * 8;
  static constexpr uint32_t kAlloc = kTmemSlot + 16 + 1024;
};

template <bool kBF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DqSmem::kBar);
  uint64_t* qo_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 1 + kBwdStages;
  uint64_t* s_full = bars + 1 + 2 * kBwdStages;
  uint64_t* ds_full = s_full + 1;
  uint64_t* dq_done = s_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + DqSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int BH = gridDim.x / p.num_tiles;
  const int bh = blockIdx.x % BH;
  const int q_tile = fwd_tile_order(blockIdx.x / BH, p.num_tiles, kTrain);
  const int q_start = q_tile * kBwdDqBM;
  const int bb = bh / p.H, hh = bh % p.H;
  Range rg[3];
  const int nr = fwd_ranges(q_start, kBwdDqBM, kBwdDqBN, p.n, p.bs, rg);

  if (threadIdx.x == 0) {
    mbar_init(qo_full, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(ds_full, 128);
    mbar_init(dq_done, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (elect_one()) {
      bool ok = true;
      mbar_expect_tx(qo_full, 2 * kTile16);
      tma_load_4d(&tm_q, qo_full, smem + DqSmem::kQ, 0, q_start, hh, bb);
      tma_load_4d(&tm_do, qo_full, smem + DqSmem::kDO, 0, q_start, hh, bb);
      int j = 0;
      for (int ri = 0; ri < nr && ok; ++ri)
        for (int s = rg[ri].lo; s < rg[ri].hi && ok; s += kBwdDqBN, ++j) {
          const int st = j % kBwdStages;
          if (j >= kBwdStages) ok = mbar_wait(&kv_empty[st], ((j / kBwdStages) - 1) & 1);
          if (!ok) break;
          mbar_expect_tx(&kv_full[st], 2 * kTile16);
          tma_load_4d(&tm_k, &kv_full[st], smem + DqSmem::kK + st * kTile16, 0, s, hh, bb);
          tma_load_4d(&tm_v, &kv_full[st], smem + DqSmem::kV + st * kTile16, 0, s, hh, bb);
        }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = idesc_f16(128, 128, false, false, kBF16);
      constexpr uint32_t idesc_dq = idesc_f16(128, 64, false, true, kBF16);
      const uint32_t sbase = smem_u32(smem);
      const uint64_t qdesc = sw128_desc(sbase + DqSmem::kQ, 16, 1024);
      const uint64_t dodesc = sw128_desc(sbase + DqSmem::kDO, 16, 1024);
      bool ok = mbar_wait(qo_full, 0);
      int j = 0;
      for (int ri = 0; ri < nr && ok; ++ri)
        for (int s = rg[ri].lo; s < rg[ri].hi && ok; s += kBwdDqBN, ++j) {
          const int st = j % kBwdStages;
          ok = mbar_wait(&kv_full[st], (j / kBwdStages) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t kdesc = sw128_desc(sbase + DqSmem::kK + st * kTile16, 16, 1024);
          const uint64_t vdesc = sw128_desc(sbase + DqSmem::kV + st * kTile16, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ss(tmem, qdesc + kk * 2, kdesc + kk * 2, idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ss(tmem + 128, dodesc + kk * 2, vdesc + kk * 2, idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(s_full);
          ok = mbar_wait(ds_full, j & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t kmn = sw128_desc(sbase + DqSmem::kK + st * kTile16, kTile16, 1024);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ts(tmem + 256, tmem + kk * 8, kmn + ((kk * 2048) >> 4), idesc_dq,
                    (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&kv_empty[st]);
        }
      umma_commit(dq_done);
    }
    __syncwarp();
  } else {
    const int row = threadIdx.x;
    const int qi = q_start + row;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const long long lrow = static_cast<long long>(bh) * 2 * p.n + qi;
    const float L2 = p.lse[lrow] * 1.4426950408889634f;
    const float Dl = p.delta[lrow];
    bool ok = true;
    int j = 0;
    for (int ri = 0; ri < nr && ok; ++ri) {
      const int rule = rg[ri].rule, shift = rg[ri].shift;
      int vlo = -2147483647, vhi = 2147483647;
      if (rule != 0) train_row_interval(rule, shift, qi, p.n, p.bs, &vlo, &vhi);
      for (int s = rg[ri].lo; s < rg[ri].hi; s += kBwdDqBN, ++j) {
        ok = mbar_wait_warp(s_full, j & 1);
        if (!ok) break;
        tc_fence_after();
        const int lo = vlo - s, hi = vhi - s;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t sr[32], dr[32];
          tmem_ld32(tmem + lane_base + c * 32, sr);
          tmem_ld32(tmem + lane_base + 128 + c * 32, dr);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float ds2[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int col = c * 32 + 2 * i + h;
              float pv = ex2(fmaf(__uint_as_float(sr[2 * i + h]), p.scale_log2, -L2));
              if (rule != 0 && (col < lo || col >= hi)) pv = 0.f;
              ds2[h] = pv * (__uint_as_float(dr[2 * i + h]) - Dl);
            }
            pk[i] = pack2<kBF16>(ds2[0], ds2[1]);
          }
          tmem_st16(tmem + lane_base + c * 16, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(ds_full);
      }
    }
    if (ok) ok = mbar_wait_warp(dq_done, 0);
    ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
    if (ok) {
      tc_fence_after();
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.dq) +
                     2 * (bb * p.dq_sb + hh * p.dq_sh + static_cast<long long>(qi) * p.dq_ss);
      store_row64<kBF16>(tmem + lane_base + 256, dst, p.scale);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------
// dK/dV: one CTA per (batch*head, 128-key tile), stepping over the query ranges that see it.
struct DkdvSmem {
  static constexpr uint32_t kK = 0;
  static constexpr uint32_t kV = kK + kTile16;
  static constexpr uint32_t kQ = kV + kTile16;
  static constexpr uint32_t kDO = kQ + kBwdStages * kTile16;
  static constexpr uint32_t kP = kDO + kBwdStages * kTile16;   // [2 key halves][128 q][128 B]
  static constexpr uint32_t kDS = kP + 2 * kTile16;
  static constexpr uint32_t kBar = kDS + 2 * kTile16;
  // kv_full, qd_full[S], qd_empty[S], s_full, p_full, mma_done
  static constexpr uint32_t kNumBars = 1 + 2 * kBwdStages + 3;
  static constexpr uint32_t kTmemSlot = kBar + kNumBars * 8;
  static constexpr uint32_t kAlloc = kTmemSlot + 16 + 1024;
};

// Key tile processed by linear CTA index t: the clean key tiles near the start of the clean
// copy are seen by the most query tiles, so they go first.
__device__ __forceinline__ int dkdv_tile_order(int t, int num_tiles) {
  const int half = num_tiles / 2;
  if (t < half) return half + t;  // clean tiles, heaviest (lowest index) first
  return t - half;                // noisy tiles: one query tile each
}

template <bool kBF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DkdvSmem::kBar);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;
  uint64_t* qd_empty = bars + 1 + kBwdStages;
  uint64_t* s_full = bars + 1 + 2 * kBwdStages;
  uint64_t* p_full = s_full + 1;
  uint64_t* mma_done = s_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + DkdvSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int BH = gridDim.x / p.num_tiles;
  const int bh = blockIdx.x % BH;
  const int k_tile = dkdv_tile_order(blockIdx.x / BH, p.num_tiles);
  const int k_start = k_tile * kBwdBKV;
  const int bb = bh / p.H, hh = bh % p.H;
  Range rg[4];
  const int nr = dkdv_ranges(k_start, kBwdBKV, kBwdBQ, p.n, p.bs, rg);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S [0,128), dP [128,256), dV [256,320), dK [320,384)

  if (warp == 4) {
    if (elect_one()) {
      bool ok = true;
      mbar_expect_tx(kv_full, 2 * kTile16);
      tma_load_4d(&tm_k, kv_full, smem + DkdvSmem::kK, 0, k_start, hh, bb);
      tma_load_4d(&tm_v, kv_full, smem + DkdvSmem::kV, 0, k_start, hh, bb);
      int i = 0;
      for (int ri = 0; ri < nr && ok; ++ri)
        for (int s = rg[ri].lo; s < rg[ri].hi && ok; s += kBwdBQ, ++i) {
          const int st = i % kBwdStages;
          if (i >= kBwdStages) ok = mbar_wait(&qd_empty[st], ((i / kBwdStages) - 1) & 1);
          if (!ok) break;
          mbar_expect_tx(&qd_full[st], 2 * kTile16);
          tma_load_4d(&tm_q, &qd_full[st], smem + DkdvSmem::kQ + st * kTile16, 0, s, hh, bb);
          tma_load_4d(&tm_do, &qd_full[st], smem + DkdvSmem::kDO + st * kTile16, 0, s, hh, bb);
        }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = idesc_f16(128, 128, false, false, kBF16);
      constexpr uint32_t idesc_acc = idesc_f16(128, 64, true, true, kBF16);
      const uint32_t sbase = smem_u32(smem);
      const uint64_t kdesc = sw128_desc(sbase + DkdvSmem::kK, 16, 1024);
      const uint64_t vdesc = sw128_desc(sbase + DkdvSmem::kV, 16, 1024);
      const uint64_t pdesc = sw128_desc(sbase + DkdvSmem::kP, kTile16, 1024);
      const uint64_t dsdesc = sw128_desc(sbase + DkdvSmem::kDS, kTile16, 1024);
      bool ok = mbar_wait(kv_full, 0);
      int i = 0;
      for (int ri = 0; ri < nr && ok; ++ri)
        for (int s = rg[ri].lo; s < rg[ri].hi && ok; s += kBwdBQ, ++i) {
          const int st = i % kBwdStages;
          ok = mbar_wait(&qd_full[st], (i / kBwdStages) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t qa = sbase + DkdvSmem::kQ + st * kTile16;
          const uint32_t da = sbase + DkdvSmem::kDO + st * kTile16;
          const uint64_t qdesc = sw128_desc(qa, 16, 1024);
          const uint64_t dodesc = sw128_desc(da, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ss(tmem, qdesc + kk * 2, kdesc + kk * 2, idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ss(tmem + 128, dodesc + kk * 2, vdesc + kk * 2, idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(s_full);
          ok = mbar_wait(p_full, i & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t domn = sw128_desc(da, kTile16, 1024);
          const uint64_t qmn = sw128_desc(qa, kTile16, 1024);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ss(tmem + 256, pdesc + ((kk * 2048) >> 4), domn + ((kk * 2048) >> 4), idesc_acc,
                    (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ss(tmem + 320, dsdesc + ((kk * 2048) >> 4), qmn + ((kk * 2048) >> 4), idesc_acc,
                    (i > 0 || kk > 0) ? 1u : 0u);
          umma_commit(mma_done);
          umma_commit(&qd_empty[st]);
        }
    }
    __syncwarp();
  } else {
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const int row = threadIdx.x;  // query row within the step's tile
    uint8_t* sP = smem + DkdvSmem::kP;
    uint8_t* sDS = smem + DkdvSmem::kDS;
    bool ok = true;
    int i = 0;
    for (int ri = 0; ri < nr && ok; ++ri) {
      const int rule = rg[ri].rule, shift = rg[ri].shift;
      for (int s = rg[ri].lo; s < rg[ri].hi; s += kBwdBQ, ++i) {
        const int qi = s + row;
        const long long lrow = static_cast<long long>(bh) * 2 * p.n + qi;
        const float L2 = p.lse[lrow] * 1.4426950408889634f;
        const float Dl = p.delta[lrow];
        int lo = -2147483647, hi = 2147483647;
        if (rule != 0) {
          train_row_interval(rule, shift, qi, p.n, p.bs, &lo, &hi);
          lo -= k_start;
          hi -= k_start;
        }
        ok = mbar_wait_warp(s_full, i & 1);
        if (ok && i > 0) ok = mbar_wait_warp(mma_done, (i - 1) & 1);  // P/dS tiles are free
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t sr[32], dr[32];
          tmem_ld32(tmem + lane_base + c * 32, sr);
          tmem_ld32(tmem + lane_base + 128 + c * 32, dr);
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float pv2[2], ds2[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int col = c * 32 + 2 * e + h;
              float pv = ex2(fmaf(__uint_as_float(sr[2 * e + h]), p.scale_log2, -L2));
              if (rule != 0 && (col < lo || col >= hi)) pv = 0.f;
              pv2[h] = pv;
              ds2[h] = pv * (__uint_as_float(dr[2 * e + h]) - Dl);
            }
            pk[e] = pack2<kBF16>(pv2[0], pv2[1]);
            dk[e] = pack2<kBF16>(ds2[0], ds2[1]);
          }
          // columns [32c, 32c+32) are 4 16-byte chunks of key half c/2
          const uint32_t half_off = (c >> 1) * kTile16;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const uint32_t off = half_off + sw128_offset(row, (c & 1) * 4 + ch);
            *reinterpret_cast<uint4*>(sP + off) =
                make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
            *reinterpret_cast<uint4*>(sDS + off) =
                make_uint4(dk[4 * ch], dk[4 * ch + 1], dk[4 * ch + 2], dk[4 * ch + 3]);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(p_full);
      }
    }
    if (ok && i > 0) ok = mbar_wait_warp(mma_done, (i - 1) & 1);
    ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
    if (ok) {
      tc_fence_after();
      const int key = k_start + row;  // accumulator lanes are keys
      uint8_t* dvp = reinterpret_cast<uint8_t*>(p.dv) +
                     2 * (bb * p.dv_sb + hh * p.dv_sh + static_cast<long long>(key) * p.dv_ss);
      uint8_t* dkp = reinterpret_cast<uint8_t*>(p.dk) +
                     2 * (bb * p.dk_sb + hh * p.dk_sh + static_cast<long long>(key) * p.dk_ss);
      if (i > 0) {
        store_row64<kBF16>(tmem + lane_base + 256, dvp, 1.f);
        store_row64<kBF16>(tmem + lane_base + 320, dkp, p.scale);
      } else {  // a key tile no query sees (cannot happen under the BD3-LM mask)
        uint4* a = reinterpret_cast<uint4*>(dvp);
        uint4* b = reinterpret_cast<uint4*>(dkp);
        for (int t = 0; t < 8; ++t) a[t] = b[t] = make_uint4(0, 0, 0, 0);
      }
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
