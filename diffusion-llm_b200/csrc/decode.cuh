// Split-KV decode and block-sparse (live-block) decode, plus the LSE combine (sm_100a).
//
// Replaces split_kv_kern + split_kv_reduce_kern (kernels/SplitKVDecodeAttention.py:17-127)
// and block_sparse_decode_kern for q_len <= 64 (kernels/BlockSparseDecodeAttention.py:41-110),
// and adds a per-(batch, head) live-KV-block variant the reference does not have.
//
// The path is HBM-bound (about 16 FLOP per byte of K/V), so the design is about bytes in
// flight: one producer warp streams 64-key K and V tiles with TMA (128-byte swizzle) into a
// kDecStages-deep ring; four consumer warps each take 16 keys of every tile and run
// mma.sync m16n8k16 for Q K^T and P V with an online softmax in registers (q_len <= 64 is
// below the 64-row minimum of tcgen05 and the tensor cores are nowhere near the bound).
// The warps' partial softmax states merge through shared memory at the end of the split.
// With one split per (batch, head) the CTA writes O directly; otherwise it writes an fp32
// partial (normalised O, natural-log LSE) and decode_combine_kernel merges the splits.
#pragma once

#include "common.cuh"
#include "tile_ranges.h"

namespace bd3 {

constexpr int kDecBN = 64;         // keys per tile
constexpr int kDecStages = 4;
constexpr int kDecThreads = 160;   // 4 consumer warps + 1 producer warp
constexpr uint32_t kDecTile = 64u * 128u;  // 64 keys x 128 B = 8 KB

struct DecParams {
  void* o;               // (B, H, q_len, 64) in the output dtype; used when n_splits == 1
  float* lse;            // optional (B*H, q_len) natural-log LSE; used when n_splits == 1
  float* ws_o;           // (B*H, n_splits, q_len, 64) fp32 partials; when n_splits > 1
  float* ws_lse;         // (B*H, n_splits, q_len)
  const int* live_idx;   // live mode: (B*H, live_stride) block indices, ascending
  const int* live_cnt;   // live mode: (B*H)
  const int* kv_len_dev; // optional device key count (contiguous mode; see decode_kernel)
  long long o_sb, o_sh, o_ss;
  int H;
  int q_len, kv_len;
  int bs;
  int q_pos0, kv_pos0;   // global positions of query row 0 and key 0 (block-causal rule)
  int n_splits;
  int tiles_per_split;   // contiguous mode: key tiles per split; live mode: entries per split
  int live_stride, kv_block;
  int out_f32;           // 1: o is fp32
  float scale_log2;
};

// Exclusive end of the keys visible to query row r (local key indices).
__device__ __forceinline__ int dec_row_hi(const DecParams& p, int r) {
  const long long hi = (static_cast<long long>((p.q_pos0 + r) / p.bs) + 1) * p.bs - p.kv_pos0;
  return hi < p.kv_len ? static_cast<int>(hi) : p.kv_len;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                        uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
template <bool kBF16>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (kBF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7},"
        " {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7},"
        " {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

constexpr int kDecLiveCache = 256;  // live entries of a split cached in shared memory

// Key tile `t` of this CTA's list: its first key, or -1 past the end. Live mode reads the
// split's block indices from `live` (the first kDecLiveCache entries, staged in shared memory
// by the producer warp; `n_live` = entries of this split) and any beyond from global memory.
template <bool kLive>
__device__ __forceinline__ int dec_tile_key(const DecParams& p, int bh, int split, int t,
                                            int n_tiles, const int* live, int n_live) {
  if constexpr (!kLive) {
    const int g = split * p.tiles_per_split + t;
    return (t < p.tiles_per_split && g < n_tiles) ? g * kDecBN : -1;
  } else {
    const int per_block = p.kv_block / kDecBN;
    const int e = t / per_block;
    if (e >= n_live) return -1;
    const int blk = e < kDecLiveCache
                        ? live[e]
                        : p.live_idx[static_cast<long long>(bh) * p.live_stride +
                                     split * p.tiles_per_split + e];
    return blk * p.kv_block + (t % per_block) * kDecBN;
  }
}

// Live entries of this split: min(tiles_per_split, live_cnt - first entry), at least 0.
__device__ __forceinline__ int dec_split_entries(const DecParams& p, int bh, int split) {
  const int left = p.live_cnt[bh] - split * p.tiles_per_split;
  return left < 0 ? 0 : (left < p.tiles_per_split ? left : p.tiles_per_split);
}

// One 64-key K/V tile for the calling consumer warp (`warp` 0-3 takes keys [16 warp,
// 16 warp + 16)): Q K^T and P V with mma.sync m16n8k16 and the online softmax of its rows
// in registers. sk / sv: the tile's swizzled K and V in shared memory; the warp arrives on
// `empty_bar` once its fragments are in registers. Keys at or past full_all are masked per
// row against row_hi (the block-causal rule).
template <int kMB, bool kBF16>
__device__ __forceinline__ void dec_tile_step(uint32_t sk, uint32_t sv, uint64_t* empty_bar,
                                              int warp, int lane, int key, int full_all,
                                              const int (&row_hi)[kMB][2],
                                              const uint32_t (&qa)[kMB][4][4],
                                              float (&acc)[kMB][8][4], float (&m_run)[kMB][2],
                                              float (&l_run)[kMB][2], float scale_log2) {
  const int tq = lane & 3;
  // K fragments for this warp's 16 keys: 2 n-tiles x 4 k-steps
  uint32_t kb[4][4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int mi = lane >> 3;
    const int krow = warp * 16 + (mi >> 1) * 8 + (lane & 7);
    const int chunk = ks * 2 + (mi & 1);
    ldsm_x4(sk + sw128_offset(krow, chunk), kb[ks][0], kb[ks][1], kb[ks][2], kb[ks][3]);
  }
  // V fragments (transposed): 8 D-tiles for one 16-key k-step
  uint32_t vb[8][2];
#pragma unroll
  for (int dp = 0; dp < 4; ++dp) {
    const int mi = lane >> 3;
    const int vrow = warp * 16 + (mi & 1) * 8 + (lane & 7);
    const int chunk = dp * 2 + (mi >> 1);
    ldsm_x4_t(sv + sw128_offset(vrow, chunk), vb[2 * dp][0], vb[2 * dp][1],
              vb[2 * dp + 1][0], vb[2 * dp + 1][1]);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);

  const int key0 = key + warp * 16;  // first key of this warp's slice
  const bool partial = key0 + 16 > full_all;
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb) {
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[nt][i] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      mma16816<kBF16>(s[0], qa[mb][ks], kb[ks][0], kb[ks][1]);
      mma16816<kBF16>(s[1], qa[mb][ks], kb[ks][2], kb[ks][3]);
    }
    if (partial) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = key0 + nt * 8 + 2 * tq + (i & 1);
          if (c >= row_hi[mb][i >> 1]) s[nt][i] = -INFINITY;
        }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = fmaxf(fmaxf(s[0][2 * hr], s[0][2 * hr + 1]), fmaxf(s[1][2 * hr], s[1][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[mb][hr], mx * scale_log2);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2(m_run[mb][hr] - m_use);
      m_run[mb][hr] = m_new;
      float rs = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float e = ex2(fmaf(s[nt][2 * hr + i], scale_log2, -m_use));
          s[nt][2 * hr + i] = e;
          rs += e;
        }
      l_run[mb][hr] = l_run[mb][hr] * alpha + rs;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        acc[mb][nt][2 * hr] *= alpha;
        acc[mb][nt][2 * hr + 1] *= alpha;
      }
    }
    uint32_t pa[4];
    pa[0] = pack2<kBF16>(s[0][0], s[0][1]);
    pa[1] = pack2<kBF16>(s[0][2], s[0][3]);
    pa[2] = pack2<kBF16>(s[1][0], s[1][1]);
    pa[3] = pack2<kBF16>(s[1][2], s[1][3]);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) mma16816<kBF16>(acc[mb][nt], pa, vb[nt][0], vb[nt][1]);
  }
}

// ---- thread-block clusters (the split merge of a small decode) ----
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The address of this CTA's shared-memory word `addr` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 dsmem_ld4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ float dsmem_ld(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

struct DecSmem {
  static constexpr uint32_t kQ = 0;                            // up to 32 rows x 128 B
  static constexpr uint32_t kStage = 8192;                     // K then V, per stage
  static constexpr uint32_t kBar = kStage + kDecStages * 2 * kDecTile;
  static constexpr uint32_t kNumBars = 1 + 2 * kDecStages;     // q_full, full[S], empty[S]
  static constexpr uint32_t kLive = kBar + kNumBars * 8;       // [kDecLiveCache] block indices
  static constexpr uint32_t kBytes = kLive + kDecLiveCache * 4;
  static constexpr uint32_t kAlloc = kBytes + 1024;
};

// kCluster: the n_splits CTAs of a (batch*head, row group) form one thread-block cluster
// (2 <= n_splits <= 16). Each writes its partial (O normalised over its keys, natural-log LSE)
// into its own shared memory; after a cluster barrier the cluster's CTA 0 merges the partials
// through distributed shared memory in split order (the merge of decode_combine_kernel) and
// writes O, so no combine launch and no workspace are needed.
template <int kMB, bool kBF16, bool kLive, bool kCluster = false>
__global__ void __launch_bounds__(kDecThreads)
    decode_kernel(const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const DecParams p_in) {
  // With kv_len_dev the key count is read on the device (kv_len is then the cache capacity
  // the tensor maps and the split count were built for): the queries are the last q_len of
  // those keys, key 0 at position 0, and the key tiles are spread over all n_splits again.
  // A count outside [q_len, capacity] is clamped and raises status bit 2. A CUDA graph
  // captured once thus serves a cache that grows between replays.
  // Launched after the QKV/RoPE cache write with programmatic serialization: wait for it
  // (q and the block's K/V rows) before any global read, and let the combine launch early.
  griddep_wait();
  griddep_launch_dependents();
  DecParams p = p_in;
  if (!kLive && p.kv_len_dev != nullptr) {
    int kl = *p.kv_len_dev;
    if (kl < p.q_len || kl > p.kv_len) {
      if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
        atomicOr(&g_bd3_status, kStatusBadLaunch);
      kl = kl < p.q_len ? p.q_len : p.kv_len;
    }
    p.kv_len = kl;
    p.q_pos0 = kl - p.q_len;
    p.kv_pos0 = 0;
    const int tiles = cdiv(kl, kDecBN);
    p.tiles_per_split = tiles > p.n_splits ? cdiv(tiles, p.n_splits) : 1;
  }
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DecSmem::kBar);
  uint64_t* q_full = bars;
  uint64_t* full = bars + 1;
  uint64_t* empty = bars + 1 + kDecStages;

  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int row0 = blockIdx.z * kMB * 16;  // first query row of this CTA's row group
  const int bb = bh / p.H, hh = bh % p.H;
  const int warp = static_cast<int>(warp_id());
  const int lane = static_cast<int>(lane_id());
  // key tiles of the contiguous mode: up to the last key any query row can see
  const int n_tiles = kLive ? 0 : cdiv(dec_row_hi(p, p.q_len - 1), kDecBN);
  static_assert(kMB == 1 || kMB == 2, "a CTA holds at most 32 query rows");

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();

  int* live = reinterpret_cast<int*>(smem + DecSmem::kLive);
  const int n_live = kLive ? dec_split_entries(p, bh, split) : 0;
  if (warp == 4) {
    // ---------------- producer ----------------
    if constexpr (kLive) {
      // stage this split's block indices in shared memory with coalesced loads, so no tile
      // waits on a dependent global read (the consumers see them after q_full completes)
      const int* src = p.live_idx + static_cast<long long>(bh) * p.live_stride +
                       split * p.tiles_per_split;
      const int n_cache = n_live < kDecLiveCache ? n_live : kDecLiveCache;
      for (int e = lane; e < n_cache; e += 32) live[e] = src[e];
      __threadfence_block();
      __syncwarp();
    }
    if (elect_one()) {
      mbar_expect_tx(q_full, kMB * 16 * 128);
      tma_load_4d(&tm_q, q_full, smem + DecSmem::kQ, 0, row0, hh, bb);
      bool ok = true;
      for (int t = 0;; ++t) {
        const int key = dec_tile_key<kLive>(p, bh, split, t, n_tiles, live, n_live);
        if (key < 0) break;
        const int st = t % kDecStages;
        if (t >= kDecStages) ok = mbar_wait(&empty[st], ((t / kDecStages) - 1) & 1);
        if (!ok) break;
        uint8_t* sk = smem + DecSmem::kStage + st * 2 * kDecTile;
        mbar_expect_tx(&full[st], 2 * kDecTile);
        tma_load_4d(&tm_k, &full[st], sk, 0, key, hh, bb);
        tma_load_4d(&tm_v, &full[st], sk + kDecTile, 0, key, hh, bb);
      }
    }
    if constexpr (kCluster) {  // the cluster's barriers count every thread of every CTA
      __syncwarp();
      cluster_sync_all();
      cluster_sync_all();
    }
    return;  // the producer takes no part in the merge below
  }

  // ---------------- consumers: warp w takes keys [16w, 16w+16) of every tile ----------------
  const int g = lane >> 2, tq = lane & 3;
  bool ok = mbar_wait_warp(q_full, 0);
  uint32_t qa[kMB][4][4];  // A fragments: m-block, k-step (16 of D), regs
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int mi = lane >> 3;
      const int row = mb * 16 + (mi & 1) * 8 + (lane & 7);
      const int chunk = ks * 2 + (mi >> 1);
      ldsm_x4(sbase + DecSmem::kQ + sw128_offset(row, chunk), qa[mb][ks][0], qa[mb][ks][1],
              qa[mb][ks][2], qa[mb][ks][3]);
    }

  float acc[kMB][8][4];
  float m_run[kMB][2], l_run[kMB][2];
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mb][nt][i] = 0.f;
    m_run[mb][0] = m_run[mb][1] = -INFINITY;
    l_run[mb][0] = l_run[mb][1] = 0.f;
  }
  int row_hi[kMB][2];
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb) {
    row_hi[mb][0] = dec_row_hi(p, row0 + mb * 16 + g);
    row_hi[mb][1] = dec_row_hi(p, row0 + mb * 16 + g + 8);
  }
  const int full_all = dec_row_hi(p, row0);  // keys below this are seen by every row here

  for (int t = 0; ok; ++t) {
    const int key = dec_tile_key<kLive>(p, bh, split, t, n_tiles, live, n_live);
    if (key < 0) break;
    const int st = t % kDecStages;
    ok = mbar_wait_warp(&full[st], (t / kDecStages) & 1);
    if (!ok) break;
    const uint32_t sk = sbase + DecSmem::kStage + st * 2 * kDecTile;
    dec_tile_step<kMB, kBF16>(sk, sk + kDecTile, &empty[st], warp, lane, key, full_all, row_hi,
                              qa, acc, m_run, l_run, p.scale_log2);
  }

  // ---------------- merge the four warps' states ----------------
  // the row sums are still per-thread partials over the quad: reduce them first
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float l = l_run[mb][hr];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      l_run[mb][hr] = l;
    }
  asm volatile("bar.sync 1, 128;" ::: "memory");  // all consumers are done with the ring
  constexpr int kRows = kMB * 16;
  float* s_o = reinterpret_cast<float*>(smem + DecSmem::kStage);   // [4][kRows][64]
  float* s_m = reinterpret_cast<float*>(smem + DecSmem::kQ);         // [4][kRows], Q is dead
  float* s_l = s_m + 4 * kRows;                                       // [4][kRows]
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mb * 16 + g + hr * 8;
      if (tq == 0) {
        s_m[warp * kRows + r] = m_run[mb][hr];
        s_l[warp * kRows + r] = l_run[mb][hr];
      }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        float2 v = make_float2(acc[mb][nt][2 * hr], acc[mb][nt][2 * hr + 1]);
        *reinterpret_cast<float2*>(&s_o[(warp * kRows + r) * 64 + nt * 8 + 2 * tq]) = v;
      }
    }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (!kCluster && !ok) return;

  // kCluster: this split's partial, after the warps' states in the ring area
  float* s_po = s_o + 4 * kRows * 64;   // [kRows][64] O normalised over this split's keys
  float* s_pl = s_po + kRows * 64;      // [kRows] natural-log LSE (-inf: no key)
  const bool direct = (p.n_splits == 1);
  for (int idx = threadIdx.x; idx < kRows * 8; idx += 128) {
    const int rl = idx >> 3, c8 = (idx & 7) * 8;
    const int r = row0 + rl;
    if (r >= p.q_len) continue;
    float mw[4], M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      mw[w] = s_m[w * kRows + rl];
      M = fmaxf(M, mw[w]);
    }
    const float M_use = (M == -INFINITY) ? 0.f : M;
    float L = 0.f, o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float sc = ex2(mw[w] - M_use);  // 0 for a warp that saw no key of this row
      L += sc * s_l[w * kRows + rl];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += sc * s_o[(w * kRows + rl) * 64 + c8 + i];
    }
    const float inv = 1.f / L;
    const float lse = (M_use + __log2f(L)) * 0.69314718055994530942f;
    if constexpr (kCluster) {
      *reinterpret_cast<float4*>(&s_po[rl * 64 + c8]) =
          make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
      *reinterpret_cast<float4*>(&s_po[rl * 64 + c8 + 4]) =
          make_float4(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv);
      if (c8 == 0) s_pl[rl] = (L > 0.f) ? lse : -INFINITY;
      continue;
    }
    if (direct) {
      if (p.out_f32) {
        float* dst = reinterpret_cast<float*>(p.o) + bb * p.o_sb + hh * p.o_sh + r * p.o_ss + c8;
        *reinterpret_cast<float4*>(dst) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv);
      } else {
        uint16_t* dst = reinterpret_cast<uint16_t*>(p.o) + bb * p.o_sb + hh * p.o_sh + r * p.o_ss + c8;
        *reinterpret_cast<uint4*>(dst) =
            make_uint4(pack2<kBF16>(o[0] * inv, o[1] * inv), pack2<kBF16>(o[2] * inv, o[3] * inv),
                       pack2<kBF16>(o[4] * inv, o[5] * inv), pack2<kBF16>(o[6] * inv, o[7] * inv));
      }
      if (p.lse != nullptr && c8 == 0) p.lse[static_cast<long long>(bh) * p.q_len + r] = lse;
    } else {
      const long long slot = (static_cast<long long>(bh) * p.n_splits + split) * p.q_len + r;
      float* dst = p.ws_o + slot * 64 + c8;
      *reinterpret_cast<float4*>(dst) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv);
      if (c8 == 0) p.ws_lse[slot] = (L > 0.f) ? lse : -INFINITY;
    }
  }
  if constexpr (kCluster) {
    __syncwarp();
    cluster_sync_all();  // every split's partial is in its CTA's shared memory
    if (split == 0 && ok) {
      // merge the splits in order: weights exp(LSE_s - max LSE); an empty split (LSE = -inf)
      // weighs 0 and is not read; a row with no key at all gets NaN, as the combine gives
      const uint32_t po = smem_u32(s_po), pl = smem_u32(s_pl);
      for (int idx = threadIdx.x; idx < kRows * 8; idx += 128) {
        const int rl = idx >> 3, c8 = (idx & 7) * 8;
        const int r = row0 + rl;
        if (r >= p.q_len) continue;
        float M = -INFINITY;
        for (int sp = 0; sp < p.n_splits; ++sp)
          M = fmaxf(M, dsmem_ld(dsmem_addr(pl + rl * 4, sp)));
        const float M_use = (M == -INFINITY) ? 0.f : M;
        float W = 0.f, o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
        for (int sp = 0; sp < p.n_splits; ++sp) {
          const float w = __expf(dsmem_ld(dsmem_addr(pl + rl * 4, sp)) - M_use);
          if (w == 0.f) continue;
          W += w;
          const uint32_t a = dsmem_addr(po + (rl * 64 + c8) * 4, sp);
          const float4 x = dsmem_ld4(a), y = dsmem_ld4(a + 16);
          o[0] += w * x.x; o[1] += w * x.y; o[2] += w * x.z; o[3] += w * x.w;
          o[4] += w * y.x; o[5] += w * y.y; o[6] += w * y.z; o[7] += w * y.w;
        }
        const float inv = 1.f / W;
        if (p.out_f32) {
          float* dst = reinterpret_cast<float*>(p.o) + bb * p.o_sb + hh * p.o_sh + r * p.o_ss + c8;
          *reinterpret_cast<float4*>(dst) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
          *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv);
        } else {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.o) + bb * p.o_sb + hh * p.o_sh + r * p.o_ss + c8;
          *reinterpret_cast<uint4*>(dst) =
              make_uint4(pack2<kBF16>(o[0] * inv, o[1] * inv), pack2<kBF16>(o[2] * inv, o[3] * inv),
                         pack2<kBF16>(o[4] * inv, o[5] * inv), pack2<kBF16>(o[6] * inv, o[7] * inv));
        }
        if (p.lse != nullptr && c8 == 0)
          p.lse[static_cast<long long>(bh) * p.q_len + r] = M_use + __logf(W);
      }
    }
    __syncwarp();
    cluster_sync_all();  // CTA 0 has read every partial: the others may exit
  }
}

// LSE-weighted merge of fp32 partials (kernels/SplitKVDecodeAttention.py:91-127).
// Partial g of (batch*head) bh, row r, column d sits at parts[g*part_g + bh*part_bh + r*64 + d]
// (normalised over its own keys) with its natural-log LSE at lses[g*lse_g + bh*lse_bh + r].
// One thread per (bh, row, 8 columns). A row whose partials are all empty (LSE = -inf)
// gets NaN, as the reference softmax does for a fully masked row.
struct CombineParams {
  const float* parts;
  const float* lses;
  void* o;
  float* lse_out;        // optional, (B*H, rows)
  long long part_g, part_bh, lse_g, lse_bh;
  long long o_sb, o_sh, o_ss;
  int H, G, rows, n_bh;
  int out_dtype;         // 0 bf16, 1 f16, 2 f32
};

__global__ void __launch_bounds__(256) decode_combine_kernel(const CombineParams p) {
  griddep_wait();  // the partials of the decode launched just before (see decode_kernel)
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int per_bh = p.rows * 8;
  if (idx >= p.n_bh * per_bh) return;
  const int bh = idx / per_bh;
  const int r = (idx % per_bh) >> 3;
  const int c8 = (idx & 7) * 8;
  const float* lse = p.lses + bh * p.lse_bh + r;
  float M = -INFINITY;
  for (int gi = 0; gi < p.G; ++gi) M = fmaxf(M, lse[gi * p.lse_g]);
  const float M_use = (M == -INFINITY) ? 0.f : M;
  float W = 0.f, o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  for (int gi = 0; gi < p.G; ++gi) {
    const float w = __expf(lse[gi * p.lse_g] - M_use);
    if (w == 0.f) continue;  // an empty partial may hold garbage
    W += w;
    const float* src = p.parts + gi * p.part_g + bh * p.part_bh + r * 64 + c8;
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 b = *reinterpret_cast<const float4*>(src + 4);
    o[0] += w * a.x; o[1] += w * a.y; o[2] += w * a.z; o[3] += w * a.w;
    o[4] += w * b.x; o[5] += w * b.y; o[6] += w * b.z; o[7] += w * b.w;
  }
  const float inv = 1.f / W;
  const int bb = bh / p.H, hh = bh % p.H;
  const long long off = bb * p.o_sb + hh * p.o_sh + static_cast<long long>(r) * p.o_ss + c8;
  if (p.out_dtype == 2) {
    float* dst = reinterpret_cast<float*>(p.o) + off;
    *reinterpret_cast<float4*>(dst) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv);
  } else {
    uint16_t* dst = reinterpret_cast<uint16_t*>(p.o) + off;
    uint4 v;
    if (p.out_dtype == 0)
      v = make_uint4(pack2<true>(o[0] * inv, o[1] * inv), pack2<true>(o[2] * inv, o[3] * inv),
                     pack2<true>(o[4] * inv, o[5] * inv), pack2<true>(o[6] * inv, o[7] * inv));
    else
      v = make_uint4(pack2<false>(o[0] * inv, o[1] * inv), pack2<false>(o[2] * inv, o[3] * inv),
                     pack2<false>(o[4] * inv, o[5] * inv), pack2<false>(o[6] * inv, o[7] * inv));
    *reinterpret_cast<uint4*>(dst) = v;
  }
  if (p.lse_out != nullptr && c8 == 0)
    p.lse_out[static_cast<long long>(bh) * p.rows + r] = M_use + __logf(W);
}

}  // namespace bd3
