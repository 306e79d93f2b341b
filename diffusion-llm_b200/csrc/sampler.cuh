// One ancestral denoising step of the BD3-LM sampler for a block of tokens (sm_100a).
//
// Replaces, per step, the reference's
//   log_probs = subs_parameterization(logits, block, mask_index)      model/subs.py:11-43
//   q = torch.exp(log_probs).double() * (1 - s / t); q[..., mask] = s / t
//   new = sample_categorical(q)                                       sample/sampler.py:11-34
//   block = torch.where(block != mask_index, block, new)              sample/sampler.py:114-122
// with one kernel that reads each masked row's logits and writes one token. Rows whose token
// is already unmasked keep it (the reference computes them and discards the result). For a
// masked row (one CTA, V logits):
//   lp_j   = log_softmax(logits + bias)_j, bias = -1e6 at mask_index: shifted = x - max,
//            sum of exp(shifted), shifted - log(sum) (model/modules.py:791-799), each op
//            rounded to the logits' dtype as the reference's tensors of that dtype are (the
//            sum accumulates in fp32 and is rounded once, as torch.sum does)
//   q_j    = (double) exp(lp_j) * (1 - s/t) for j != mask_index;  q_mask = s/t
// The draw is either a replay of the reference's own: u_j read from a caller's float64
// tensor (the reference's torch.rand_like), g_j = EPS - log(u_j + EPS), token = argmax_j
// q_j / g_j (the first index among equal maxima, as torch.argmax); or, in production, an
// exact draw from the same distribution q / sum(q) by inverse CDF with one uniform per row:
// the elements are ordered (thread t, then its chunks c = t, t + T, t + 2T, ..., each the 8
// entries [8c, 8c + 8) in order), each thread sums its q_j in float64 in that order, a block
// scan (Hillis-Steele within warps, then over the warp totals) gives every thread its slice
// [excl, incl) of [0, total), and
// r * total with r = (x << 21 | y >> 11) * 2^-53 from words x, y of Philox4x32-10 (Salmon,
// Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) at counter
// (row, offset lo, offset hi, 0x5A3) under key = seed falls in one slice, whose thread walks
// it (the smallest claimed index wins where rounding makes slices overlap; a walk that
// rounds past its slice takes its last nonzero element). float64 sums keep tokens with
// probability down to ~1e-16 of the row's mass, as the reference's float64 noise does.
#pragma once

#include "common.cuh"

namespace bd3 {

constexpr int kSampleThreads = 512;

struct SampleParams {
  const void* logits;        // (B, S, V), vocab contiguous
  long long l_sb, l_ss;
  const long long* xt;       // (B, S) current tokens
  long long* out;            // (B, S) next tokens (may alias xt)
  const double* u;           // (B, S, V) contiguous uniforms, or null for Philox
  unsigned long long seed, offset;
  double keep;               // 1 - s/t, the weight of the unmasking tokens
  double stay;               // s/t, the weight of staying masked
  long long mask_index;
  const double* ts_dev;                  // optional device (t, s): overrides keep and stay
  const unsigned long long* rng_dev;     // optional device (seed, offset): overrides both
  int B, S, V;
};

// ---- Philox4x32-10 (the published round function and Weyl key schedule) ----------------
struct U4 {
  uint32_t x, y, z, w;
};
__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kM0, c.x), lo0 = kM0 * c.x;
    const uint32_t hi1 = __umulhi(kM1, c.z), lo1 = kM1 * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += kW0;
    k1 += kW1;
  }
  return c;
}
__device__ __forceinline__ double u53(uint32_t hi, uint32_t lo) {
  const unsigned long long m = (static_cast<unsigned long long>(hi) << 21) | (lo >> 11);
  return static_cast<double>(m) * 0x1.0p-53;
}

template <int kDtype>
__device__ __forceinline__ float logit_at(const void* row, int j) {
  if constexpr (kDtype == 0) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[j]);
  else if constexpr (kDtype == 1) return __half2float(reinterpret_cast<const __half*>(row)[j]);
  else return reinterpret_cast<const float*>(row)[j];
}

// Block-wide reductions over kSampleThreads threads through shared memory.
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < kSampleThreads / 32 ? red[l] : -INFINITY;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return __shfl_sync(0xffffffffu, v, 0);  // lanes 0-15 hold the result; give it to all
}
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < kSampleThreads / 32 ? red[l] : 0.f;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return __shfl_sync(0xffffffffu, v, 0);
}

constexpr int kChunk = 8;               // entries of a 16-byte chunk of a bf16 row
constexpr int kWalkChunks = 32;         // chunks per thread the parallel walk holds (V <= 131072)
constexpr uint16_t kBf16NegInf = 0xFF80u;

__device__ __forceinline__ __nv_bfloat162 as_bf162(uint32_t u) {
  return *reinterpret_cast<const __nv_bfloat162*>(&u);
}

// Round a pair to the dtype with one packed conversion (bf16 and fp16; fp32 is left as is).
template <int kDtype>
__device__ __forceinline__ void rnd2(float& a, float& b) {
  if constexpr (kDtype == 0) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    a = __low2float(v), b = __high2float(v);
  } else if constexpr (kDtype == 1) {
    const __half2 v = __floats2half2_rn(a, b);
    a = __low2float(v), b = __high2float(v);
  }
}

// Bytes [a, a + 16) of the 32 bytes lo:hi (a even, q = a / 4 words and r = 8 * (a % 4) bits).
template <int kQ>
__device__ __forceinline__ uint4 realign_q(const uint32_t (&w)[8], int r) {
  return make_uint4(__funnelshift_r(w[kQ], w[kQ + 1], r), __funnelshift_r(w[kQ + 1], w[kQ + 2], r),
                    __funnelshift_r(w[kQ + 2], w[kQ + 3], r),
                    __funnelshift_r(w[kQ + 3], w[kQ + 4], r));
}
__device__ __forceinline__ uint4 realign(uint4 lo, uint4 hi, int a) {
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  const int r = (a & 3) * 8;
  switch (a >> 2) {  // uniform over the CTA (one row)
    case 0: return realign_q<0>(w, r);
    case 1: return realign_q<1>(w, r);
    case 2: return realign_q<2>(w, r);
    default: return realign_q<3>(w, r);
  }
}

// Copy a 16-bit row of V entries into shared memory so that entry j sits at dst16[j] with
// dst 16-byte aligned, whatever the row's own alignment: 16-byte loads of the aligned words
// that hold the row's bytes (lane m of a warp loads word c and takes word c + 1 from lane
// m + 1), realigned in registers. Chunk c of dst (entries [8c, 8c + 8)) is written for
// c < n_chunks; entries past V are left for the caller to overwrite. Only words that hold at
// least one byte of the row are read.
__device__ __forceinline__ void stage_row(const uint16_t* g16, int V, int n_chunks, uint4* dst) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(g16);
  const int a = static_cast<int>(addr & 15u);
  const uint4* src = reinterpret_cast<const uint4*>(addr - static_cast<uintptr_t>(a));
  const int n_words = (a + 2 * V + 15) >> 4;
  const int lane = threadIdx.x & 31;
  constexpr int kDepth = 4;  // chunks in flight per thread
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int c0 = static_cast<int>(threadIdx.x & ~31u); c0 < n_chunks;
       c0 += kDepth * kSampleThreads) {
    uint4 lo[kDepth], edge[kDepth];
#pragma unroll
    for (int d = 0; d < kDepth; ++d) {
      const int c = c0 + d * kSampleThreads + lane;
      lo[d] = c < n_words ? src[c] : zero;
      edge[d] = (lane == 31 && c + 1 < n_words) ? src[c + 1] : zero;
    }
#pragma unroll
    for (int d = 0; d < kDepth; ++d) {
      const int c = c0 + d * kSampleThreads + lane;
      uint4 hi;
      hi.x = __shfl_down_sync(0xffffffffu, lo[d].x, 1);
      hi.y = __shfl_down_sync(0xffffffffu, lo[d].y, 1);
      hi.z = __shfl_down_sync(0xffffffffu, lo[d].z, 1);
      hi.w = __shfl_down_sync(0xffffffffu, lo[d].w, 1);
      if (lane == 31) hi = edge[d];
      if (c < n_chunks) dst[c] = realign(lo[d], hi, a);
    }
  }
}

// exp of a non-positive bf16 value, rounded to bf16, by table: rnd(expf(a)) for every a with
// |a| in [2^-9, 128), indexed by a's magnitude bits minus 0x3B00 (2^-9) plus one, with entry 0
// = 1.0 (every |a| below 2^-9: expf rounds to 1.0 there) and entry kExpTab - 1 = 0.0 (|a| of
// 128 or more, -inf included: expf underflows bf16 from |a| = 93 on). Built per CTA with the
// same expf the per-entry path calls, so the values are those of that path, bit for bit.
constexpr int kExpTab = 2048 + 2;
__device__ __forceinline__ void build_exp_tab(uint16_t* tab) {
  for (int i = threadIdx.x; i < kExpTab; i += blockDim.x) {
    float e;
    if (i == 0) e = 1.f;
    else if (i == kExpTab - 1) e = 0.f;
    else e = expf(__uint_as_float((0x8000u | (0x3B00u + static_cast<uint32_t>(i - 1))) << 16));
    tab[i] = static_cast<uint16_t>(__float_as_uint(rnd<0>(e)) >> 16);
  }
}
// rnd(expf(a)) for the bf16 a in the low 16 bits of `bits` (a <= 0)
__device__ __forceinline__ float exp_tab_lookup(const uint16_t* tab, uint32_t bits) {
  int i = static_cast<int>(bits & 0x7FFFu) - 0x3B00 + 1;
  i = i < 0 ? 0 : (i > kExpTab - 1 ? kExpTab - 1 : i);
  return __uint_as_float(static_cast<uint32_t>(tab[i]) << 16);
}

// (score, index) with the larger score, the smaller index on a tie (torch.argmax's first max).
__device__ __forceinline__ void best_of(double& s, int& i, double s2, int i2) {
  if (s2 > s || (s2 == s && i2 < i)) s = s2, i = i2;
}

// The row is processed in chunks of 8 consecutive entries, thread t taking chunks t, t + T,
// t + 2T, ... (T = 512) in every pass. kStage (bf16 rows): the row is first copied into
// shared memory, realigned so that each chunk is one 16-byte word, with the [MASK] entry
// biased and the last chunk padded with -inf, so the passes read a chunk with one 16-byte
// load and need no bounds or [MASK] test; the max is taken on packed bf16 pairs. Without
// staging (fp32 rows, or bf16 rows too long for shared memory) each chunk's entries are
// read from global memory. The element order, and so the draw, is the same either way.
//
// kDevArgs: the step's (t, s) and (seed, offset) are read from ts_dev and rng_dev on the
// device, so the launch arguments stay fixed from step to step and a CUDA graph captured
// once draws each step afresh. The weights are computed as on the host (1 - s/t and s/t in
// float64, IEEE division), so they equal the host-argument launch's bit for bit. A device
// t <= 0 (or NaN) raises status bit 2 and leaves every token as it was.
template <int kDtype, bool kStage, bool kDevArgs>
__global__ void __launch_bounds__(kSampleThreads) subs_sample_kernel(const SampleParams p) {
  extern __shared__ __align__(16) uint16_t srow_raw[];
  __shared__ float red[kSampleThreads / 32];
  __shared__ double rs[kSampleThreads / 32];
  __shared__ double wscan[kSampleThreads / 32];
  __shared__ double last_incl[kSampleThreads / 32];
  __shared__ int ri[kSampleThreads / 32];
  __shared__ double walk_q[kWalkChunks * kChunk];  // the claimed slice's weights
  __shared__ int walk_owner;
  __shared__ uint16_t exp_tab[kStage ? kExpTab : 1];
  const int row = blockIdx.x;
  const int b = row / p.S, i = row % p.S;
  const long long tok = p.xt[static_cast<long long>(b) * p.S + i];
  bool bad_ts = false;
  if constexpr (kDevArgs) bad_ts = !(p.ts_dev[0] > 0.0);
  if (tok != p.mask_index || bad_ts) {  // carry-over: the reference's where() keeps the token
    if (threadIdx.x == 0) {
      p.out[static_cast<long long>(b) * p.S + i] = tok;
      if (bad_ts && row == 0) atomicOr(&g_bd3_status, kStatusBadLaunch);
    }
    return;
  }
  const void* lrow = reinterpret_cast<const uint8_t*>(p.logits) +
                     (b * p.l_sb + i * p.l_ss) * (kDtype == 2 ? 4 : 2);
  const int mask = static_cast<int>(p.mask_index);
  const float bias = rnd<kDtype>(-1e6f);  // model/subs.py:8
  const int n_chunks = (p.V + kChunk - 1) / kChunk;
  // staged rows: element j at srow[j] (16-byte aligned whatever the row's alignment), the
  // [MASK] entry already biased, and the last chunk padded with -inf
  uint4* const schunk = reinterpret_cast<uint4*>(srow_raw);
  if constexpr (kStage) {
    static_assert(kDtype == 0, "staging holds bf16 rows");
    build_exp_tab(exp_tab);
    stage_row(reinterpret_cast<const uint16_t*>(lrow), p.V, n_chunks, schunk);
    __syncthreads();
    if (threadIdx.x == 0) {
      const float x = __uint_as_float(static_cast<uint32_t>(srow_raw[mask]) << 16);
      srow_raw[mask] = static_cast<uint16_t>(__float_as_uint(rnd<kDtype>(x + bias)) >> 16);
    }
    if (threadIdx.x < kChunk * n_chunks - p.V) srow_raw[p.V + threadIdx.x] = kBf16NegInf;
    __syncthreads();
  }
  // the 8 (biased) logits of chunk c, -inf past the vocabulary
  auto chunk = [&](int c, float (&x)[kChunk]) {
    if constexpr (kStage) {
      const uint4 v = schunk[c];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        x[2 * k] = __uint_as_float(w[k] << 16);
        x[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
      }
    } else {
#pragma unroll
      for (int k = 0; k < kChunk; ++k) {
        const int j = c * kChunk + k;
        const float v = j < p.V ? logit_at<kDtype>(lrow, j) : -INFINITY;
        x[k] = j == mask ? rnd<kDtype>(v + bias) : v;
      }
    }
  };
  // pass 1: the row max
  float mx = -INFINITY;
  if constexpr (kStage) {  // bf16 max is exact: compare packed pairs
    __nv_bfloat162 m2 = __floats2bfloat162_rn(-INFINITY, -INFINITY);
    for (int c = threadIdx.x; c < n_chunks; c += kSampleThreads) {
      const uint4 v = schunk[c];
      m2 = __hmax2(m2, __hmax2(__hmax2(as_bf162(v.x), as_bf162(v.y)),
                               __hmax2(as_bf162(v.z), as_bf162(v.w))));
    }
    mx = fmaxf(__low2float(m2), __high2float(m2));
  } else {
    for (int c = threadIdx.x; c < n_chunks; c += kSampleThreads) {
      float x[kChunk];
      chunk(c, x);
#pragma unroll
      for (int k = 0; k < kChunk; ++k) mx = fmaxf(mx, x[k]);
    }
  }
  mx = block_max(mx, red);
  // pass 2: sum of exp(x - max), each op rounded to the dtype. Staged rows: the rounded
  // x - max replaces x in shared memory (pass 3 and the walk start from it) and the
  // exponential comes from the table
  float sum = 0.f;
  for (int c = threadIdx.x; c < n_chunks; c += kSampleThreads) {
    if constexpr (kStage) {
      const uint4 v = schunk[c];
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __nv_bfloat162 a2 = __floats2bfloat162_rn(__uint_as_float(w[k] << 16) - mx,
                                                        __uint_as_float(w[k] & 0xffff0000u) - mx);
        w[k] = *reinterpret_cast<const uint32_t*>(&a2);
        sum += exp_tab_lookup(exp_tab, w[k]);
        sum += exp_tab_lookup(exp_tab, w[k] >> 16);
      }
      schunk[c] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      float x[kChunk];
      chunk(c, x);
#pragma unroll
      for (int k = 0; k < kChunk; k += 2) {
        float a = x[k] - mx, bb = x[k + 1] - mx;
        rnd2<kDtype>(a, bb);
        a = expf(a), bb = expf(bb);
        rnd2<kDtype>(a, bb);
        sum += a;
        sum += bb;
      }
    }
  }
  sum = rnd<kDtype>(block_sum(sum, red));
  const float lse = rnd<kDtype>(logf(sum));
  // pass 3: q_j in float64 (the reference's exp(log_probs).double() * (1 - s/t), s/t at
  // mask_index), then one draw.
  double keep = p.keep, stay = p.stay;
  if constexpr (kDevArgs) {
    const double t = p.ts_dev[0], s = p.ts_dev[1];
    keep = 1.0 - s / t;
    stay = s / t;
  }
  // q of the 8 entries of chunk c (0 past the vocabulary)
  auto chunk_q = [&](int c, double (&q)[kChunk]) {
    if constexpr (kStage) {  // the staged row holds rnd(x - max) after pass 2
      const uint4 v = schunk[c];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __nv_bfloat162 l2 = __floats2bfloat162_rn(__uint_as_float(w[k] << 16) - lse,
                                                        __uint_as_float(w[k] & 0xffff0000u) - lse);
        const uint32_t lw = *reinterpret_cast<const uint32_t*>(&l2);
        q[2 * k] = static_cast<double>(exp_tab_lookup(exp_tab, lw)) * keep;
        q[2 * k + 1] = static_cast<double>(exp_tab_lookup(exp_tab, lw >> 16)) * keep;
      }
    } else {
      float x[kChunk];
      chunk(c, x);
#pragma unroll
      for (int k = 0; k < kChunk; k += 2) {
        float a = x[k] - mx, bb = x[k + 1] - mx;
        rnd2<kDtype>(a, bb);
        a -= lse, bb -= lse;
        rnd2<kDtype>(a, bb);
        a = expf(a), bb = expf(bb);
        rnd2<kDtype>(a, bb);
        q[k] = static_cast<double>(a) * keep;
        q[k + 1] = static_cast<double>(bb) * keep;
      }
    }
    if (c == mask / kChunk) {
#pragma unroll
      for (int k = 0; k < kChunk; ++k)
        if (c * kChunk + k == mask) q[k] = stay;
    }
  };
  auto q64 = [&](int j) -> double {
    if (j == mask) return stay;
    if constexpr (kStage) {  // the staged row holds rnd(x - max) after pass 2
      const float a = __uint_as_float(static_cast<uint32_t>(srow_raw[j]) << 16);
      const float lp = rnd<kDtype>(a - lse);
      return static_cast<double>(
                 exp_tab_lookup(exp_tab, __float_as_uint(lp) >> 16)) * keep;
    } else {
      const float x = logit_at<kDtype>(lrow, j);
      const float lp = rnd<kDtype>(rnd<kDtype>(x - mx) - lse);
      return static_cast<double>(rnd<kDtype>(expf(lp))) * keep;
    }
  };
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  long long pick;
  if (p.u != nullptr) {
    // replay of the reference's own draw: argmax_j q_j / (EPS - log(u_j + EPS)) in float64
    const double* urow = p.u + static_cast<long long>(row) * p.V;
    double best = -1.0;
    int best_i = 0x7fffffff;
    for (int j = threadIdx.x; j < p.V; j += kSampleThreads)
      best_of(best, best_i, q64(j) / (1e-10 - log(urow[j] + 1e-10)), j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const double s2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, best_i, o);
      best_of(best, best_i, s2, i2);
    }
    if (l == 0) rs[w] = best, ri[w] = best_i;
    __syncthreads();
    best = l < kSampleThreads / 32 ? rs[l] : -1.0;
    best_i = l < kSampleThreads / 32 ? ri[l] : 0x7fffffff;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      const double s2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, best_i, o);
      best_of(best, best_i, s2, i2);
    }
    pick = best_i;
  } else {
    // inverse CDF over the element order (thread t, its chunks c = t, t + T, t + 2T, ...,
    // the 8 entries of each chunk in order): each thread sums its q_j in that order, a
    // block scan gives each thread its slice [excl_t, incl_t) of [0, total), and one Philox
    // uniform r per row selects r * total.
    double part = 0.0;
    for (int c = threadIdx.x; c < n_chunks; c += kSampleThreads) {
      double q[kChunk];
      chunk_q(c, q);
#pragma unroll
      for (int k = 0; k < kChunk; ++k) part += q[k];
    }
    // inclusive scan: within warps (Hillis-Steele), then of the warp totals in warp 0
    double x = part;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, x, o);
      if (l >= o) x += y;
    }
    if (l == 31) rs[w] = x;
    __syncthreads();
    if (w == 0) {
      double v = l < kSampleThreads / 32 ? rs[l] : 0.0;
#pragma unroll
      for (int o = 1; o < kSampleThreads / 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, v, o);
        if (l >= o) v += y;
      }
      if (l < kSampleThreads / 32) wscan[l] = v;
    }
    __syncthreads();
    const double incl = (w > 0 ? wscan[w - 1] : 0.0) + x;
    if (l == 31) last_incl[w] = incl;
    __syncthreads();
    double excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (l == 0) excl = w > 0 ? last_incl[w - 1] : 0.0;
    const double total = last_incl[kSampleThreads / 32 - 1];
    unsigned long long seed = p.seed, offset = p.offset;
    if constexpr (kDevArgs) seed = p.rng_dev[0], offset = p.rng_dev[1];
    const U4 r = philox4x32_10(U4{static_cast<uint32_t>(row), static_cast<uint32_t>(offset),
                                  static_cast<uint32_t>(offset >> 32), 0x5A3u},
                               static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    double target = u53(r.x, r.y) * total;
    if (target >= total) target = nextafter(total, 0.0);
    int mine = 0x7fffffff;
    const bool claim = excl <= target && target < incl;
    // The slices tile [0, total) exactly (each excl is the previous thread's incl), so one
    // thread claims the target. Its chunks' weights are then computed by one thread each
    // into shared memory, and the claimant adds them up in its own order (the additions
    // and so the token are those of a walk by the claimant alone, which is the fallback).
    const int per_thread = (n_chunks + kSampleThreads - 1) / kSampleThreads;
    if (__syncthreads_count(claim) == 1 && per_thread <= kWalkChunks) {
      if (claim) walk_owner = static_cast<int>(threadIdx.x);
      __syncthreads();
      const int owner = walk_owner;
      if (static_cast<int>(threadIdx.x) < per_thread) {
        const int c = owner + static_cast<int>(threadIdx.x) * kSampleThreads;
        if (c < n_chunks) {
          double q[kChunk];
          chunk_q(c, q);
#pragma unroll
          for (int k = 0; k < kChunk; ++k) walk_q[threadIdx.x * kChunk + k] = q[k];
        }
      }
      __syncthreads();
      if (claim) {
        const double local = target - excl;
        double acc = 0.0;
        int last_nz = 0x7fffffff;
        for (int i = 0, c = owner; c < n_chunks && mine == 0x7fffffff; ++i, c += kSampleThreads) {
#pragma unroll
          for (int k = 0; k < kChunk; ++k) {
            if (mine != 0x7fffffff) continue;
            const double q = walk_q[i * kChunk + k];
            acc += q;
            if (q > 0.0) last_nz = c * kChunk + k;
            if (local < acc) mine = c * kChunk + k;
          }
        }
        if (mine == 0x7fffffff) mine = last_nz;  // the local offset rounded past the slice
      }
    } else if (claim) {  // this thread's slice: walk it chunk by chunk,
      const double local = target - excl;  // adding in the same order as part
      double acc = 0.0;
      int last_nz = 0x7fffffff;
      for (int c = threadIdx.x; c < n_chunks && mine == 0x7fffffff; c += kSampleThreads) {
        double q[kChunk];
        chunk_q(c, q);
#pragma unroll
        for (int k = 0; k < kChunk; ++k) {
          if (mine != 0x7fffffff) continue;
          acc += q[k];
          if (q[k] > 0.0) last_nz = c * kChunk + k;
          if (local < acc) mine = c * kChunk + k;
        }
      }
      if (mine == 0x7fffffff) mine = last_nz;  // the local offset rounded past the slice
    }
    // the smallest claimed index (slices only overlap through rounding)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mine = min(mine, __shfl_xor_sync(0xffffffffu, mine, o));
    if (l == 0) ri[w] = mine;
    __syncthreads();
    mine = l < kSampleThreads / 32 ? ri[l] : 0x7fffffff;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mine = min(mine, __shfl_xor_sync(0xffffffffu, mine, o));
    pick = mine;
  }
  if (threadIdx.x == 0) p.out[static_cast<long long>(b) * p.S + i] = pick;
}

}  // namespace bd3
