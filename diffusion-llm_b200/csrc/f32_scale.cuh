// fp32 attention operands onto the fp16 kernels at tf32's significand (sm_100a).
//
// The reference computes fp32 inputs with Triton's tl.dot (kernels/BlockSparseFlashAttention.py:
// 45-70), i.e. tf32 operands: an 11-bit significand and fp32 accumulation. fp16 has the same
// significand and a narrower exponent range, so each tensor is scaled by a power of two (exact)
// into fp16's range and rounded to nearest: q by 2^-a and k by 2^a, which leaves every score
// q . k unchanged (a = floor((e_q - e_k) / 2) balances their magnitudes), and v by 2^-c with
// c = e_v - 4 (max |v| in [16, 32)); e_x = floor(log2(max |x|)), at least -100. q and k
// saturate at +-65504 (only when max|q| max|k| >= 2^30, a one-hot softmax).
//   f32_absmax_kernel        max |x| of q, k, v as float bits, atomicMax into ws[0..2]
//                            (non-negative floats order like their bit patterns)
//   f32_to_f16_scaled_kernel the exponents from ws, then the scaled fp16 copies; block 0
//                            writes exps = {a, c, 2^c}
// Two launches and no host round trip, where the same arithmetic in PyTorch ops takes about
// thirty launches.
#pragma once

#include "common.cuh"

namespace bd3 {

struct F32ScaleParams {
  const float* src[3];        // q, k, v: (B, H, rows, 64), last dim contiguous
  long long sb[3], sh[3], ss[3];
  int rows[3];                // rows per (batch, head) of each tensor
  uint16_t* dst[3];           // contiguous (B, H, rows, 64) fp16
  unsigned int* ws;           // [3] max |x| bits, zeroed before the first kernel
  float* exps;                // {a, c, 2^c}
  int H, bh;                  // heads, batch * heads
};

// float4 j (of 16 per row) of row r of tensor t
__device__ __forceinline__ const float4* f32s_src(const F32ScaleParams& p, int t, long long idx) {
  const long long row = idx >> 4;
  const int part = static_cast<int>(idx & 15);
  const long long bh = row / p.rows[t];
  const long long r = row % p.rows[t];
  const long long b = bh / p.H, h = bh % p.H;
  return reinterpret_cast<const float4*>(p.src[t] + b * p.sb[t] + h * p.sh[t] + r * p.ss[t]) +
         part;
}

__global__ void __launch_bounds__(256) f32_absmax_kernel(const F32ScaleParams p) {
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const long long n4 = static_cast<long long>(p.bh) * p.rows[t] * 16;
    unsigned int m = 0;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n4; i += 256ll * gridDim.x) {
      const float4 x = *f32s_src(p, t, i);
      const unsigned int a = __float_as_uint(fabsf(x.x)), b = __float_as_uint(fabsf(x.y)),
                         c = __float_as_uint(fabsf(x.z)), d = __float_as_uint(fabsf(x.w));
      m = max(m, max(max(a, b), max(c, d)));
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0 && m != 0) atomicMax(&p.ws[t], m);
  }
}

// floor(log2(x)) of a non-negative float given as bits, at least -100 (zero, subnormals and
// anything below 2^-100 give -100)
__device__ __forceinline__ int f32s_exponent(unsigned int bits) {
  const int e = static_cast<int>((bits >> 23) & 0xffu) - 127;
  return e < -100 ? -100 : e;
}
// 2^e as a float, for -126 <= e <= 127
__device__ __forceinline__ float f32s_pow2(int e) { return __int_as_float((e + 127) << 23); }
// x limited to [-lim, lim]; NaN stays NaN (as torch.clamp leaves it)
__device__ __forceinline__ float f32s_sat(float x, float lim) {
  return fabsf(x) > lim ? copysignf(lim, x) : x;
}

__global__ void __launch_bounds__(256) f32_to_f16_scaled_kernel(const F32ScaleParams p) {
  const int eq = f32s_exponent(p.ws[0]), ek = f32s_exponent(p.ws[1]), ev = f32s_exponent(p.ws[2]);
  const int d = eq - ek;
  const int a = d >= 0 ? d / 2 : -((1 - d) / 2);  // floor(d / 2)
  const int c = ev - 4;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    p.exps[0] = static_cast<float>(a);
    p.exps[1] = static_cast<float>(c);
    p.exps[2] = f32s_pow2(c);
  }
  const float scale[3] = {f32s_pow2(-a), f32s_pow2(a), f32s_pow2(-c)};
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const long long n4 = static_cast<long long>(p.bh) * p.rows[t] * 16;
    const float s = scale[t];
    const float lim = t < 2 ? 65504.f : INFINITY;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n4; i += 256ll * gridDim.x) {
      const float4 x = *f32s_src(p, t, i);
      const __half2 lo = __floats2half2_rn(f32s_sat(x.x * s, lim), f32s_sat(x.y * s, lim));
      const __half2 hi = __floats2half2_rn(f32s_sat(x.z * s, lim), f32s_sat(x.w * s, lim));
      uint2 out;
      out.x = *reinterpret_cast<const uint32_t*>(&lo);
      out.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(p.dst[t] + i * 4) = out;
    }
  }
}

}  // namespace bd3
