// The exchange and merge step of sequence-sharded decode in one kernel over NVLink peer memory
// (sm_100a; every rank runs it on its own GPU).
//
// Sequence-sharded decode (bd3attn.dist.sharded_decode) gives each rank a partial (O
// normalised over its keys, fp32; natural-log LSE) of the same query block; the partials are
// then merged with the LSE weighting of kernels/SplitKVDecodeAttention.py:109-119. With NCCL
// that is an all-gather of every partial followed by bd3_lse_merge. Here each rank's kernel
// stores its partial straight into every peer's exchange buffer with plain stores over
// NVLink, raises a per-chunk flag in each peer's buffer, waits (bounded) for the peers' flags
// on its own buffer and merges, all in one launch. No loads from peer memory, no TMA and no
// multicast: only stores to peers and loads of the local buffer.
//
// Exchange buffer of one rank (allocated symmetric on every rank; float offsets):
//   region (parity p, sender s): [B*H*rows*64 O | B*H*rows LSE] at (p*world + s) * kUnitRegion
//   flags (parity p, sender s, chunk c): uint64 after the regions
// The parity is that of the call's epoch (a counter every rank advances by one per call), so
// a rank may start the next call while a slower peer still reads this call's parity; it can
// not get two calls ahead, because the next call's merge waits for that peer's push.
//
// Work is chunked by (batch*head, row) units identically on every rank: CTA c pushes units
// [c*U, (c+1)*U) and merges the same units, so it waits only for the peers' CTA c. The grid
// is at most one CTA per SM, so every CTA is resident and every push happens.
#pragma once

#include "common.cuh"

namespace bd3 {

constexpr int kPeerMaxWorld = 8;
constexpr int kPeerMaxCtas = 256;
constexpr int kPeerThreads = 256;
constexpr unsigned long long kPeerWaitNs = 1000000000ull;  // 1 s: a peer that never arrives

enum : unsigned { kStatusPeerTimeout = 16u };  // a peer's partial did not arrive in time

struct PeerMergeParams {
  float* bufs[kPeerMaxWorld];   // every rank's exchange buffer, mapped in this process
  const float* part_o;          // this rank's partial O, (B*H*rows, 64) fp32
  const float* part_lse;        // (B*H*rows) natural-log LSE
  void* o;                      // (B, H, rows, 64) in out_dtype
  float* lse_out;               // optional (B*H, rows)
  long long o_sb, o_sh, o_ss;
  unsigned long long epoch;
  long long region;             // floats per (parity, sender) region: units * 65
  int world, rank, H, units, rows, out_dtype;
};

__device__ __forceinline__ unsigned long long* peer_flags(const PeerMergeParams& p, float* buf) {
  return reinterpret_cast<unsigned long long*>(buf + 2LL * p.world * p.region);
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* a, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

__global__ void __launch_bounds__(kPeerThreads) peer_merge_kernel(const PeerMergeParams p) {
  griddep_wait();  // the partial comes from the decode launched just before
  const int c = blockIdx.x, C = gridDim.x;
  const int u0 = static_cast<int>(static_cast<long long>(p.units) * c / C);
  const int u1 = static_cast<int>(static_cast<long long>(p.units) * (c + 1) / C);
  const int parity = static_cast<int>(p.epoch & 1ull);

  // ---- push this rank's units of the partial into every peer's region (parity, rank) ----
  const int n4 = (u1 - u0) * 16;  // float4s of O in this chunk
  for (int s = 1; s < p.world; ++s) {
    const int peer = (p.rank + s) % p.world;
    float* dst = p.bufs[peer] + (static_cast<long long>(parity) * p.world + p.rank) * p.region;
    const float4* src4 = reinterpret_cast<const float4*>(p.part_o + static_cast<long long>(u0) * 64);
    float4* dst4 = reinterpret_cast<float4*>(dst + static_cast<long long>(u0) * 64);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) dst4[i] = __ldcg(src4 + i);
    float* dl = dst + static_cast<long long>(p.units) * 64;
    for (int u = u0 + threadIdx.x; u < u1; u += blockDim.x) dl[u] = __ldcg(p.part_lse + u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the chunk's stores are visible before any flag
    for (int s = 1; s < p.world; ++s) {
      const int peer = (p.rank + s) % p.world;
      unsigned long long* f = peer_flags(p, p.bufs[peer]);
      st_release_sys_u64(f + (static_cast<long long>(parity) * kPeerMaxWorld + p.rank) * kPeerMaxCtas + c,
                         p.epoch);
    }
    // ---- wait for every peer's CTA c to have pushed into this rank's buffer ----
    unsigned long long* mine = peer_flags(p, p.bufs[p.rank]);
    for (int s = 1; s < p.world; ++s) {
      const int peer = (p.rank + s) % p.world;
      const unsigned long long* f =
          mine + (static_cast<long long>(parity) * kPeerMaxWorld + peer) * kPeerMaxCtas + c;
      if (ld_acquire_sys_u64(f) == p.epoch) continue;
      const unsigned long long t0 = globaltimer_ns();
      for (uint32_t it = 1;; ++it) {
        if (ld_acquire_sys_u64(f) == p.epoch) break;
        if ((it & 255u) == 0 && globaltimer_ns() - t0 > kPeerWaitNs) {
          atomicOr(&g_bd3_status, kStatusPeerTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();

  // ---- merge: one thread per (unit, 8 columns), senders in rank order ----
  const float* my = p.bufs[p.rank] + static_cast<long long>(parity) * p.world * p.region;
  for (int idx = u0 * 8 + threadIdx.x; idx < u1 * 8; idx += blockDim.x) {
    const int u = idx >> 3, c8 = (idx & 7) * 8;
    float lse_s[kPeerMaxWorld];
    float M = -INFINITY;
    for (int s = 0; s < p.world; ++s) {
      lse_s[s] = s == p.rank ? __ldcg(p.part_lse + u)
                             : __ldcg(my + s * p.region + static_cast<long long>(p.units) * 64 + u);
      M = fmaxf(M, lse_s[s]);
    }
    const float M_use = (M == -INFINITY) ? 0.f : M;
    float W = 0.f, o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.f;
    for (int s = 0; s < p.world; ++s) {
      const float w = __expf(lse_s[s] - M_use);
      if (w == 0.f) continue;  // a shard no query sees
      W += w;
      const float* src = s == p.rank ? p.part_o + static_cast<long long>(u) * 64 + c8
                                     : my + s * p.region + static_cast<long long>(u) * 64 + c8;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(src) + 1);
      o[0] += w * a.x; o[1] += w * a.y; o[2] += w * a.z; o[3] += w * a.w;
      o[4] += w * b.x; o[5] += w * b.y; o[6] += w * b.z; o[7] += w * b.w;
    }
    const float inv = 1.f / W;
    const int bh = u / p.rows, r = u % p.rows;
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
    if (p.lse_out != nullptr && c8 == 0) p.lse_out[u] = M_use + __logf(W);
  }
}

}  // namespace bd3
