// Block-sparse attention backward on tcgen05 tensor cores (sm_100a).
//
// Replaces BlockSparseFlashAttention.backward (kernels/BlockSparseFlashAttention.py:509-562),
// i.e. the host Delta = rowsum(dO * O) (:525) and the kernels block_sparse_attention_bwd_dq_kern
// (:369-452) and block_sparse_attention_dk_dv_bwd_kern (:213-328), with three launches:
//
//   bwd_prep_kernel     Delta = rowsum(dO * O) and LSE * log2(e) per query row (fp32), and
//                       zeroes the fp32 dQ accumulator.
//   bwd_fused_kernel    persistent: one CTA per SM loops over (batch*head, 128-key tile) items,
//                       heaviest first, stepping over the query ranges that see each tile (the
//                       reference's dK/dV ranges, :274-325):
//                         S^T  = K Q_i^T,  dP^T = V dO_i^T          (SS MMAs, keys on TMEM lanes)
//                         P^T  = exp2(S^T * scale*log2e - L2[q]) masked to 0,
//                         dS^T = P^T * (dP^T - Delta[q])            (element-wise, thread = key)
//                         dV  += P^T dO_i,  dK += dS^T Q_i          (TS MMAs: P^T, dS^T in TMEM)
//                         dQ_i = dS_i K                              (SS MMA from a smem dS tile)
//                       dV and dK accumulate in TMEM and are written once, so they are
//                       deterministic; each dQ_i is added to the fp32 accumulator by a reducer
//                       warpgroup through TMA reduce-adds (cp.reduce.async.bulk.tensor).
//   bwd_dq_convert_kernel  dQ = scale * accumulator, in the input dtype.
//
// Deterministic variant (kDet, bd3_attn_bwd_det): the fp32 reduce-adds make dQ's last bits
// depend on the order in which key tiles finish. With kDet each dQ_i partial is rounded to a
// 64-bit integer in units of 2^-32 and added with integer bulk reductions
// (cp.reduce.async.bulk .add.u64), which are associative, so dQ is the same on every run, as
// the reference's dQ kernel (:369-452), which loops over key tiles in order, is. A partial of
// magnitude 2^20 or more (or NaN) sets device status bit 8 instead of wrapping silently;
// 2^20 * 2^32 summed over up to 2^10 key tiles stays inside the 63-bit range.
//
// Each 128-query step runs as two 64-query halves whose S^T/dP^T live in two TMEM buffers, so
// the MMAs of one half overlap the element-wise pass over the other. K/V are double-buffered
// across items (the next item's tiles load during the current one), the step and half-step
// counters behind every barrier phase run on across items, and an item's dV/dK epilogue
// overlaps the next item's first S^T/dP^T.
// Roles in the fused kernel (704 threads):
//   warps 0-15  element-wise: four warpgroups; thread t of each owns key row t (TMEM lane t),
//               warpgroup g takes queries [16g, 16g+16) of every half-step (four warps per
//               SM sub-partition keep the exponential and FMA pipes busy)
//   warps 16-19 dQ reducer and dV/dK writer: thread t owns row t (TMEM lane t); stages dQ_i
//               in shared memory and adds it to the fp32 accumulator with TMA reduce-adds, and
//               writes each item's dV and dK tiles with TMA stores
//   warp 20     TMA producer: K, V once; Q_i, dO_i (and their LSE/Delta rows) per step
//   warp 21     TMEM owner and UMMA issuer
// TMEM columns: half-step buffers [0,128) and [128,256) (S^T then dP^T, 64 columns each),
// dV [256,320), dK [320,384), dQ_i [384,448). P^T and dS^T (packed 16-bit) overwrite the
// columns each thread has already read. dS for the dQ MMA lives in shared memory (two
// buffers) as [query half][key row][64 queries] with the 128-byte swizzle: the MN-major A
// operand of dQ_i = dS_i K (M = 128 queries, K = 128 keys).
#pragma once

#include "attn_fwd.cuh"
#include "common.cuh"
#include "tile_ranges.h"

namespace bd3 {

constexpr int kBwdBKV = 128;  // keys per CTA
constexpr int kBwdBQ = 128;   // queries per step
constexpr int kBwdStages = 2;
constexpr int kBwdThreads = 704;

struct BwdParams {
  const void* o;
  const void* dout;
  const float* lse;      // (B, H, 2n), natural log
  float* delta;          // (B, H, 2n), written by bwd_prep_kernel
  float* lse2;           // (B, H, 2n), LSE * log2(e), written by bwd_prep_kernel
  float* dq_acc;         // (B, H, 2n, 64) fp32, zeroed by bwd_prep_kernel
  // kDet: per 128-query tile T, four 16 KB blocks (columns [16b, 16b+16)) of 128 rows x 16
  // int64 (2^-32 units), each row's 16-byte chunks swizzled as sw128_offset; zeroed likewise
  unsigned long long* dq_fix;
  void* dq;
  void* dk;
  void* dv;
  long long o_sb, o_sh, o_ss, do_sb, do_sh, do_ss;
  long long dq_sb, dq_sh, dq_ss, dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  int H, n, bs;
  int num_tiles;         // key tiles per (batch, head)
  int num_bh;            // batch * heads
  float scale, scale_log2;
};

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// Tiled TMA reduce-add of a shared-memory box into global memory (fp32 add in L2), tracked by
// the issuing thread's bulk async-group.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0,
                                                  int c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::
          "l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every committed bulk group has finished reading its shared-memory source.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk group has completed.
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// 1-D bulk reduce-add of `bytes` of int64 (two's complement, added as u64) from shared
// memory into global memory, tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_reduce_add_u64(unsigned long long* dst, const void* src,
                                                    uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.u64 [%0], [%1], %2;" ::"l"(
                   dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> shared completing on an mbarrier (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Delta, LSE*log2(e) and the dQ accumulator's zeroing; 8 threads per query row.
template <bool kBF16, bool kDet>
__global__ void __launch_bounds__(256) bwd_prep_kernel(const BwdParams p, int rows_total) {
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
    if constexpr (kDet) {  // 64 bytes of the int64 accumulator per thread (any layout)
      float4* z = reinterpret_cast<float4*>(p.dq_fix + static_cast<long long>(gid) * 8);
#pragma unroll
      for (int k = 0; k < 4; ++k) z[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      float4* z = reinterpret_cast<float4*>(p.dq_acc + static_cast<long long>(row) * 64 + part * 8);
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (row < rows_total && part == 0) {
    p.delta[row] = acc;
    p.lse2[row] = p.lse[row] * 1.4426950408889634f;
  }
}

// dQ = scale * accumulator in the output dtype; 8 threads per query row.
template <bool kBF16, bool kDet>
__global__ void __launch_bounds__(256) bwd_dq_convert_kernel(const BwdParams p, int rows_total) {
  const int gid = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = gid >> 3, part = gid & 7;
  if (row >= rows_total) return;
  const int S = 2 * p.n;
  const int bh = row / S, r = row % S;
  const int bb = bh / p.H, hh = bh % p.H;
  float4 x, y;
  if constexpr (kDet) {
    // columns [8 part, 8 part + 8): block part / 2, 16-byte chunks 4 (part % 2) .. + 3 of the
    // row, each at its swizzled position
    const int rt = row & 127;
    const unsigned long long* blk =
        p.dq_fix + static_cast<long long>(row >> 7) * 8192 + (part >> 1) * 2048 + rt * 16;
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = 4 * (part & 1) + k;
      const longlong2 w = *reinterpret_cast<const longlong2*>(blk + 2 * (c ^ (rt & 7)));
      v[2 * k] = __ll2float_rn(w.x) * 2.3283064365386963e-10f;  // 2^-32
      v[2 * k + 1] = __ll2float_rn(w.y) * 2.3283064365386963e-10f;
    }
    x = make_float4(v[0], v[1], v[2], v[3]);
    y = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    const float4* src =
        reinterpret_cast<const float4*>(p.dq_acc + static_cast<long long>(row) * 64 + part * 8);
    x = src[0];
    y = src[1];
  }
  const float s = p.scale;
  *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.dq) + bb * p.dq_sb + hh * p.dq_sh +
                            r * p.dq_ss + part * 8) =
      make_uint4(pack2<kBF16>(x.x * s, x.y * s), pack2<kBF16>(x.z * s, x.w * s),
                 pack2<kBF16>(y.x * s, y.y * s), pack2<kBF16>(y.z * s, y.w * s));
}

struct BwdSmem {
  static constexpr uint32_t kK = 0;                             // [item parity]
  static constexpr uint32_t kV = kK + 2 * kTile16;              // [item parity]
  static constexpr uint32_t kQ = kV + 2 * kTile16;              // [stage]
  static constexpr uint32_t kDO = kQ + kBwdStages * kTile16;    // [stage]
  static constexpr uint32_t kDS = kDO + kBwdStages * kTile16;   // [buffer][q half][key][128 B]
  static constexpr uint32_t kVec = kDS + 2 * 2 * kTile16;       // [stage][L2 128 | Delta 128]
  static constexpr uint32_t kRed = kVec + kBwdStages * 1024;    // dQ_i staging: one [128][128 B] box
  static constexpr uint32_t kBar = kRed + kTile16;
  // kv_full[2], kv_empty[2], qd_full[S], qd_empty[S], s_full[2], p_full[2], ds_free[2],
  // dq_full, dq_empty, acc_done, acc_free
  static constexpr uint32_t kNumBars = 4 + 2 * kBwdStages + 6 + 4;
  static constexpr uint32_t kTmemSlot = kBar + kNumBars * 8;
  static constexpr uint32_t kAlloc = kTmemSlot + 16 + 1024;
};

// Key tile of the t-th group of work items: the clean key tiles near the start of the clean
// copy are seen by the most query tiles, so they go first; noisy tiles (one step) last.
__device__ __forceinline__ int bwd_tile_order(int t, int num_tiles) {
  const int half = num_tiles / 2;
  if (t < half) return half + t;
  return t - half;
}

// Column of the packed 16-bit P^T / dS^T operand for k-step kk (16 queries) of a half-step:
// element-wise warpgroup g writes queries [16g, 16g+16) of the half, packed, into the first 8
// of its own 16 read columns, so k-step kk sits at columns [16kk, 16kk+8).
__device__ __forceinline__ uint32_t half_ts_col(int kk) { return static_cast<uint32_t>(kk) * 16; }

// Work item w of the persistent loop: one key tile of one (batch, head). Items are numbered
// heaviest first (bwd_tile_order), and CTAs take them in alternating rounds (persistent_item).
struct BwdItem {
  int bb, hh, k_start, nr, nsteps;
  long long row0;  // first row of this (batch, head) in the flattened (B*H*2n) row space
  Range rg[4];
};
__device__ __forceinline__ void bwd_item(int w, const BwdParams& p, BwdItem* t) {
  const int bh = w % p.num_bh;
  t->k_start = bwd_tile_order(w / p.num_bh, p.num_tiles) * kBwdBKV;
  t->bb = bh / p.H;
  t->hh = bh % p.H;
  t->row0 = static_cast<long long>(bh) * 2 * p.n;
  t->nr = dkdv_ranges(t->k_start, kBwdBKV, kBwdBQ, p.n, p.bs, t->rg);
  int ns = 0;
  for (int r = 0; r < t->nr; ++r)
    if (t->rg[r].hi > t->rg[r].lo) ns += cdiv(t->rg[r].hi - t->rg[r].lo, kBwdBQ);
  t->nsteps = ns;
}

template <bool kBF16, bool kDet>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_fused_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dqacc,
                     const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                     const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BwdSmem::kBar);
  uint64_t* kv_full = bars;                       // [item parity]
  uint64_t* kv_empty = bars + 2;                  // [item parity]
  uint64_t* qd_full = bars + 4;                   // [stage]
  uint64_t* qd_empty = bars + 4 + kBwdStages;     // [stage]
  uint64_t* s_full = bars + 4 + 2 * kBwdStages;   // [half]
  uint64_t* p_full = s_full + 2;                  // [half]
  uint64_t* ds_free = s_full + 4;                 // [dS buffer]
  uint64_t* dq_full = s_full + 6;
  uint64_t* dq_empty = s_full + 7;
  uint64_t* acc_done = s_full + 8;                // an item's dV/dK accumulators are final
  uint64_t* acc_free = s_full + 9;                // ... and have been read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + BwdSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int num_items = p.num_bh * p.num_tiles;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&kv_full[b], 1);
      mbar_init(&kv_empty[b], 1);
    }
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&s_full[h], 1);
      mbar_init(&p_full[h], 512);
      mbar_init(&ds_free[h], 1);
    }
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
    mbar_init(acc_done, 1);
    mbar_init(acc_free, 128);
    fence_mbar_init();
  }
  if (warp == 21) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: half-step buffer h at [128h, 128h+128) = S^T [0,64) then dP^T [64,128);
  // dV [256,320), dK [320,384), dQ [384,448)
  constexpr uint32_t tDV = 256, tDK = 320, tDQ = 384;

  if (warp == 20) {
    // ---------------- TMA producer: per item K, V; per step Q_i, dO_i, L2_i, Delta_i --------
    if (elect_one()) {
      const uint64_t keep = l2_policy_evict_last();
      bool ok = true;
      int it = 0, i = 0;
      for (int k = 0, w = persistent_item(0); w < num_items && ok; w = persistent_item(++k)) {
        BwdItem t;
        bwd_item(w, p, &t);
        if (t.nsteps == 0) continue;
        const int kb = it & 1;
        if (it >= 2) ok = mbar_wait(&kv_empty[kb], ((it >> 1) - 1) & 1);
        if (!ok) break;
        mbar_expect_tx(&kv_full[kb], 2 * kTile16);
        tma_load_4d(&tm_k, &kv_full[kb], smem + BwdSmem::kK + kb * kTile16, 0, t.k_start, t.hh, t.bb);
        tma_load_4d(&tm_v, &kv_full[kb], smem + BwdSmem::kV + kb * kTile16, 0, t.k_start, t.hh, t.bb);
        for (int ri = 0; ri < t.nr && ok; ++ri)
          for (int s = t.rg[ri].lo; s < t.rg[ri].hi && ok; s += kBwdBQ, ++i) {
            const int st = i % kBwdStages;
            if (i >= kBwdStages) ok = mbar_wait(&qd_empty[st], ((i / kBwdStages) - 1) & 1);
            if (!ok) break;
            mbar_expect_tx(&qd_full[st], 2 * kTile16 + 1024);
            // Q and dO tiles are read again by every key tile of this (batch, head) that
            // sees them: keep them in L2 ahead of the fp32 dQ accumulator's lines
            tma_load_4d_hint(&tm_q, &qd_full[st], smem + BwdSmem::kQ + st * kTile16, 0, s, t.hh,
                             t.bb, keep);
            tma_load_4d_hint(&tm_do, &qd_full[st], smem + BwdSmem::kDO + st * kTile16, 0, s,
                             t.hh, t.bb, keep);
            uint8_t* vec = smem + BwdSmem::kVec + st * 1024;
            bulk_load(vec, p.lse2 + t.row0 + s, 512, &qd_full[st]);
            bulk_load(vec + 512, p.delta + t.row0 + s, 512, &qd_full[st]);
          }
        ++it;
      }
    }
    __syncwarp();
  } else if (warp == 21) {
    // ---------------- UMMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc_s = idesc_f16(128, 64, false, false, kBF16);
      constexpr uint32_t idesc_ts = idesc_f16(128, 64, false, true, kBF16);
      constexpr uint32_t idesc_dq = idesc_f16(128, 64, true, true, kBF16);
      const uint32_t sbase = smem_u32(smem);
      bool ok = true;
      // A half-step whose dV/dK MMAs are still to be issued: global half index j, its Q/dO
      // stage, its item (counted over this CTA's items), and whether it is the item's first or
      // last half.
      struct Half {
        int j, st, it;
        bool first, last;
      };
      Half prev{-1, 0, 0, false, false};
      int pend_i = -1, pend_kb = 0;  // step whose dQ MMA is still to be issued, its K buffer
      bool pend_last = false;        // ... and whether it is its item's last step
      // dV += P^T dO_i, dK += dS^T Q_i of one half-step; a step's last half frees its Q/dO
      // stage and queues its dQ; an item's last half publishes dV/dK.
      auto finish = [&](const Half& hf) {
        const int hp = hf.j & 1, ip = hf.j >> 1;
        ok = ok && mbar_wait(&p_full[hp], ip & 1);
        if (!ok) return;
        if (hf.first && hf.it > 0) {  // the previous item's dV/dK have been read out
          ok = mbar_wait(acc_free, (hf.it - 1) & 1);
          if (!ok) return;
        }
        tc_fence_after();
        const uint32_t qa = sbase + BwdSmem::kQ + hf.st * kTile16 + hp * (kTile16 / 2);
        const uint32_t da = sbase + BwdSmem::kDO + hf.st * kTile16 + hp * (kTile16 / 2);
        const uint64_t domn = sw128_desc(da, kTile16, 1024);
        const uint64_t qmn = sw128_desc(qa, kTile16, 1024);
        const uint32_t tbuf = tmem + hp * 128;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_ts(tmem + tDV, tbuf + half_ts_col(kk), domn + ((kk * 2048) >> 4), idesc_ts,
                  (hf.first && kk == 0) ? 0u : 1u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_ts(tmem + tDK, tbuf + 64 + half_ts_col(kk), qmn + ((kk * 2048) >> 4), idesc_ts,
                  (hf.first && kk == 0) ? 0u : 1u);
        if (hp == 1) {
          umma_commit(&qd_empty[hf.st]);
          pend_i = ip;
          pend_kb = hf.it & 1;
          pend_last = hf.last;
        }
        if (hf.last) umma_commit(acc_done);
      };
      // dQ_i = dS_i K. Issued after the next half-step's S^T/dP^T, which the element-wise
      // warps wait for, while dQ only feeds the reducer. An item's last dQ is the last reader
      // of its K/V buffer.
      auto issue_dq = [&]() {
        if (pend_i > 0) {
          ok = mbar_wait(dq_empty, (pend_i - 1) & 1);  // the reducer has read dQ_{i-1}
          if (!ok) return;
          tc_fence_after();
        }
        const uint64_t kmn = sw128_desc(sbase + BwdSmem::kK + pend_kb * kTile16, kTile16, 1024);
        const uint64_t dsdesc =
            sw128_desc(sbase + BwdSmem::kDS + (pend_i & 1) * 2 * kTile16, kTile16, 1024);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss(tmem + tDQ, dsdesc + ((kk * 2048) >> 4), kmn + ((kk * 2048) >> 4), idesc_dq,
                  kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(&ds_free[pend_i & 1]);
        if (pend_last) umma_commit(&kv_empty[pend_kb]);
        pend_i = -1;
      };
      int it = 0, i = 0, j = 0;
      for (int k = 0, w = persistent_item(0); w < num_items && ok; w = persistent_item(++k)) {
        BwdItem t;
        bwd_item(w, p, &t);
        if (t.nsteps == 0) continue;
        const int kb = it & 1;
        ok = mbar_wait(&kv_full[kb], (it >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint64_t kdesc = sw128_desc(sbase + BwdSmem::kK + kb * kTile16, 16, 1024);
        const uint64_t vdesc = sw128_desc(sbase + BwdSmem::kV + kb * kTile16, 16, 1024);
        int step = 0;
        for (int ri = 0; ri < t.nr && ok; ++ri)
          for (int s = t.rg[ri].lo; s < t.rg[ri].hi && ok; s += kBwdBQ, ++i, ++step) {
            const int st = i % kBwdStages;
            ok = mbar_wait(&qd_full[st], (i / kBwdStages) & 1);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; ++h, ++j) {
              const uint32_t qa = sbase + BwdSmem::kQ + st * kTile16 + h * (kTile16 / 2);
              const uint32_t da = sbase + BwdSmem::kDO + st * kTile16 + h * (kTile16 / 2);
              const uint64_t qdesc = sw128_desc(qa, 16, 1024);
              const uint64_t dodesc = sw128_desc(da, 16, 1024);
              const uint32_t tbuf = tmem + h * 128;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_ss(tbuf, kdesc + kk * 2, qdesc + kk * 2, idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_ss(tbuf + 64, vdesc + kk * 2, dodesc + kk * 2, idesc_s, kk > 0 ? 1u : 0u);
              umma_commit(&s_full[h]);
              if (pend_i >= 0) issue_dq();
              if (ok && prev.j >= 0) finish(prev);
              prev = Half{j, st, it, step == 0 && h == 0, step == t.nsteps - 1 && h == 1};
              if (!ok) break;
            }
          }
        ++it;
      }
      if (ok && prev.j >= 0) finish(prev);
      if (ok && pend_i >= 0) issue_dq();
    }
    __syncwarp();
  } else if (warp >= 16) {
    // ---------------- dQ reducer and dV/dK writer: thread = row of a 128-row tile ----------
    // dQ_i goes from TMEM to a swizzled shared-memory box (32 fp32 columns at a time) and from
    // there into the fp32 accumulator by TMA reduce-adds, so the additions run in L2 without
    // occupying this SM's load/store path. Before an item's last dQ, the same box carries its
    // dV and then its dK tile (64 16-bit columns) out with TMA stores, so the element-wise
    // warps go straight on to the next item.
    const int row = threadIdx.x - 512;
    const bool leader = (threadIdx.x == 512);
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint8_t* stage = smem + BwdSmem::kRed;
    // all four reducer warps agree on `ok` (they share named barrier 2 below)
    auto agree = [](bool v) {
      uint32_t all;
      asm volatile(
          "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 2, 128, p;\n"
          " selp.u32 %0, 1, 0, q;\n}\n"
          : "=r"(all)
          : "r"(static_cast<uint32_t>(v))
          : "memory");
      return all != 0;
    };
    bool ok = true;
    int it = 0, i = 0;
    for (int k = 0, w = persistent_item(0); w < num_items && ok; w = persistent_item(++k)) {
      BwdItem t;
      bwd_item(w, p, &t);
      if (t.nsteps == 0) {  // a key tile no query sees (cannot happen under the BD3-LM mask)
        const long long key = t.k_start + row;
        uint4* a = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.dv) + t.bb * p.dv_sb +
                                            t.hh * p.dv_sh + key * p.dv_ss);
        uint4* b = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.dk) + t.bb * p.dk_sb +
                                            t.hh * p.dk_sh + key * p.dk_ss);
        for (int q8 = 0; q8 < 8; ++q8) a[q8] = b[q8] = make_uint4(0, 0, 0, 0);
        continue;
      }
      int step = 0;
      for (int ri = 0; ri < t.nr && ok; ++ri)
        for (int s = t.rg[ri].lo; s < t.rg[ri].hi; s += kBwdBQ, ++i, ++step) {
          if (step == t.nsteps - 1) {
            // ---- this item's dV, then dK (scaled), as 16-bit tiles. Read out as soon as the
            // item's last dV/dK MMAs are done, before its last dQ (which queues behind the
            // next item's first S^T/dP^T), so the next item's first dV/dK MMAs need not wait.
            ok = agree(mbar_wait_warp(acc_done, it & 1));
            if (!ok) break;
            tc_fence_after();
#pragma unroll 1
            for (int m = 0; m < 2; ++m) {
              if (leader) bulk_wait_group_read0();  // the previous bulk op has read the box
              asm volatile("bar.sync 2, 128;" ::: "memory");
              const float mul = m == 0 ? 1.f : p.scale;
#pragma unroll
              for (int c2 = 0; c2 < 2; ++c2) {
                uint32_t r[32];
                tmem_ld32_async(tmem + lane_base + (m == 0 ? tDV : tDK) + 32 * c2, r);
                tmem_ld_wait();
                reg_fence(r);
                if (m == 1 && c2 == 1) {  // both accumulators have been read
                  tc_fence_before();
                  mbar_arrive(acc_free);
                }
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  *reinterpret_cast<uint4*>(stage + sw128_offset(row, 4 * c2 + c)) = make_uint4(
                      pack2<kBF16>(__uint_as_float(r[8 * c + 0]) * mul, __uint_as_float(r[8 * c + 1]) * mul),
                      pack2<kBF16>(__uint_as_float(r[8 * c + 2]) * mul, __uint_as_float(r[8 * c + 3]) * mul),
                      pack2<kBF16>(__uint_as_float(r[8 * c + 4]) * mul, __uint_as_float(r[8 * c + 5]) * mul),
                      pack2<kBF16>(__uint_as_float(r[8 * c + 6]) * mul, __uint_as_float(r[8 * c + 7]) * mul));
              }
              fence_proxy_async_smem();
              asm volatile("bar.sync 2, 128;" ::: "memory");
              if (leader) {
                tma_store_4d(m == 0 ? &tm_dv : &tm_dk, stage, 0, t.k_start, t.hh, t.bb);
                bulk_commit_group();
              }
            }
          }
          ok = agree(mbar_wait_warp(dq_full, i & 1));
          const uint32_t tdq = tmem + lane_base + tDQ;
          if (!ok) break;
          tc_fence_after();
          if constexpr (kDet) {
            // dQ_i in 64-bit fixed point: four 16-column rounds through the box, each one
            // bulk integer reduce-add of its 16 KB block (the box's bytes as they are)
            unsigned long long* blk = p.dq_fix + ((t.row0 + s) >> 7) * 8192;
#pragma unroll 1
            for (int b = 0; b < 4; ++b) {
              if (leader) bulk_wait_group_read0();  // the previous bulk op has read the box
              asm volatile("bar.sync 2, 128;" ::: "memory");
              uint32_t r[16];
              tmem_ld16_async(tdq + 16 * b, r);
              tmem_ld_wait();
              reg_fence(r);
              if (b == 3) {
                tc_fence_before();
                mbar_arrive(dq_empty);
              }
              bool bad = false;
              long long qv[16];
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const float v = __uint_as_float(r[k]);
                bad |= !(fabsf(v) < 1048576.f);  // 2^20; NaN too
                qv[k] = __float2ll_rn(v * 4294967296.f);
              }
              if (bad) atomicOr(&g_bd3_status, kStatusFixedRange);
#pragma unroll
              for (int c = 0; c < 8; ++c)
                *reinterpret_cast<longlong2*>(stage + sw128_offset(row, c)) =
                    make_longlong2(qv[2 * c], qv[2 * c + 1]);
              fence_proxy_async_smem();
              asm volatile("bar.sync 2, 128;" ::: "memory");
              if (leader) {
                bulk_reduce_add_u64(blk + b * 2048, stage, kTile16);
                bulk_commit_group();
              }
            }
            continue;
          }
          // the two 32-column halves of dQ_i go through the box in turn
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            if (leader) bulk_wait_group_read0();  // the previous bulk op has read the box
            asm volatile("bar.sync 2, 128;" ::: "memory");
            uint32_t r[32];
            tmem_ld32_async(tdq + 32 * b, r);
            tmem_ld_wait();
            reg_fence(r);
            if (b == 1) {
              tc_fence_before();
              mbar_arrive(dq_empty);
            }
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(stage + sw128_offset(row, c)) =
                  make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
            fence_proxy_async_smem();
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (leader) {
              tma_reduce_add_2d(&tm_dqacc, stage, 32 * b, static_cast<int>(t.row0 + s));
              bulk_commit_group();
            }
          }
        }
      ++it;
    }
    if (leader) bulk_wait_group0();  // every reduce and store has landed before the CTA exits
  } else {
    // ------- element-wise: thread = key row; warpgroup g takes queries [16g, 16g+16) of
    // each 64-query half-step -------
    const int g = warp >> 2;
    const int row = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    int i = 0;
    for (int k = 0, w = persistent_item(0); w < num_items && ok; w = persistent_item(++k)) {
      BwdItem t;
      bwd_item(w, p, &t);
      const int key = t.k_start + row;
      for (int ri = 0; ri < t.nr && ok; ++ri) {
        const int rule = t.rg[ri].rule, shift = t.rg[ri].shift;
        int qlo = -2147483647, qhi = 2147483647;  // visible query interval of this key
        if (rule != 0)
          dkdv_col_interval(rule, shift, key, t.rg[ri].lo < p.n ? 0 : p.n, p.n, p.bs, &qlo, &qhi);
        for (int s = t.rg[ri].lo; s < t.rg[ri].hi; s += kBwdBQ, ++i) {
          const int st = i % kBwdStages;
          ok = mbar_wait_warp(&qd_full[st], (i / kBwdStages) & 1);  // L2 / Delta rows landed
          if (ok && i >= 2) ok = mbar_wait_warp(&ds_free[i & 1], ((i >> 1) - 1) & 1);
          if (!ok) break;
          const float* vL = reinterpret_cast<const float*>(smem + BwdSmem::kVec + st * 1024);
          const float* vD = vL + 128;
          uint8_t* sDS = smem + BwdSmem::kDS + (i & 1) * 2 * kTile16;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            ok = mbar_wait_warp(&s_full[h], i & 1);
            if (!ok) break;
            tc_fence_after();
            const uint32_t tbuf = tmem + lane_base + h * 128 + g * 16;
            const int c0 = h * 64 + g * 16;  // first query of this thread's columns, in the step
            const int lo = qlo - s - c0, hi = qhi - s - c0;
            // a warp whose 32 keys see none of its 16 queries writes P^T = dS^T = 0 and skips
            // the exponentials (rule != 0 steps only)
            const bool skip = rule != 0 && __all_sync(0xffffffffu, hi <= 0 || lo >= 16 || hi <= lo);
            uint32_t pk[8], dk[8];
            if (skip) {
#pragma unroll
              for (int e = 0; e < 8; ++e) pk[e] = dk[e] = 0u;
            } else {
              uint32_t sr[16], dr[16];
              tmem_ld16_async(tbuf, sr);
              tmem_ld16_async(tbuf + 64, dr);
              tmem_ld_wait();
              reg_fence(sr);
              reg_fence(dr);
#pragma unroll
              for (int e4 = 0; e4 < 4; ++e4) {
                const float4 l4 = *reinterpret_cast<const float4*>(vL + c0 + 4 * e4);
                const float4 d4 = *reinterpret_cast<const float4*>(vD + c0 + 4 * e4);
                const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
                float pv[4], dsv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int col = 4 * e4 + e;
                  float pe = ex2(fmaf(__uint_as_float(sr[col]), p.scale_log2, -lv[e]));
                  if (rule != 0 && (col < lo || col >= hi)) pe = 0.f;
                  pv[e] = pe;
                  dsv[e] = pe * (__uint_as_float(dr[col]) - dv4[e]);
                }
                pk[2 * e4] = pack2<kBF16>(pv[0], pv[1]);
                pk[2 * e4 + 1] = pack2<kBF16>(pv[2], pv[3]);
                dk[2 * e4] = pack2<kBF16>(dsv[0], dsv[1]);
                dk[2 * e4 + 1] = pack2<kBF16>(dsv[2], dsv[3]);
              }
            }
            tmem_st8(tbuf, pk);        // P^T over this thread's own (already read) S^T columns
            tmem_st8(tbuf + 64, dk);   // dS^T likewise over dP^T
            // dS row for the dQ MMA: queries [16g, 16g+16) of half h are 16-byte chunks 2g, 2g+1
#pragma unroll
            for (int ch = 0; ch < 2; ++ch)
              *reinterpret_cast<uint4*>(sDS + h * kTile16 + sw128_offset(row, 2 * g + ch)) =
                  make_uint4(dk[4 * ch], dk[4 * ch + 1], dk[4 * ch + 2], dk[4 * ch + 3]);
            tmem_st_wait();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&p_full[h]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 21) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bd3
