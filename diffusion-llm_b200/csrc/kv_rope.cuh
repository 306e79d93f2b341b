// Fused QKV split + rotary embedding + in-place KV-cache write (sm_100a).
//
// Replaces, for one attention layer, the reference's
//   q, k, v = rearrange(qkv_proj, "... seq (three n_heads d_k) -> three ... n_heads seq d_k")
//   q = self.rope(q, positions); k = self.rope(k, positions)            model/modules.py:395-405
//   k_all = torch.cat([k_cache, k], dim=-2) (and v)                     model/modules.py:410-414
//   kv_cache.append(layer_idx, k, v)   -> torch.cat of the whole cache  model/kv_cache.py:42-55
// with one pass over the projection: q goes to its own (batch, heads, seq, head_dim) tensor,
// k and v straight into rows [row0, row0 + seq) of preallocated cache tensors, so neither the
// per-step concatenation nor the per-commit one copies the cache.
//
// RoPE is the reference's rotate-half form (model/modules.py:164-240): pair k couples
// coordinates k and k + D/2 and rotates them by the angle of the token's position,
//   out_1 = x_1 * cos - x_2 * sin,   out_2 = x_1 * sin + x_2 * cos,
// with the reference's sin/cos tables (fp32, (max_pos, D/2)) passed in. The reference casts
// the tables to the activation dtype and evaluates each product, difference and sum as a
// separate elementwise op (computed in fp32, rounded to the dtype); the kernel does the same
// operations in the same order with the same roundings (no FMA contraction), so its output
// is bit-identical for bf16, fp16 and fp32 activations.
#pragma once

#include "common.cuh"

namespace bd3 {

enum : unsigned {
  kStatusBadPosition = 4u,  // a RoPE position outside [0, max_pos): nothing written for it
};

struct RopeCacheParams {
  const void* qkv;                 // (B, S, 3, H, D) with (3, H, D) contiguous
  long long qkv_sb, qkv_ss;
  const long long* positions;      // (S,) absolute positions, or null for pos0 + s
  long long pos0;
  const float* cos_table;          // (max_pos, D/2) fp32, row-major
  const float* sin_table;
  long long max_pos;
  void* q_out;                     // (B, H, S, D); may be null
  long long q_sb, q_sh, q_ss;
  void* k_cache;                   // (B, H, rows, D)
  long long k_sb, k_sh, k_ss;
  void* v_cache;
  long long v_sb, v_sh, v_ss;
  long long row0;                  // cache row of token s = 0; < 0: positions[0] (device)
  long long cache_rows;            // rows of each cache (bounds the row read from positions)
  int B, S, H, D;
};

// kN consecutive elements moved as 16-byte pieces (8 two-byte values or 4 floats per piece;
// the host checks that every tensor's base and strides are 16-byte aligned, and element
// offsets here are multiples of 8).
template <int kDtype>
__device__ __forceinline__ void load8(const void* base, long long i, float (&x)[8]) {
  if constexpr (kDtype == 2) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    const float4 a = p[0], b = p[1];
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack2<kDtype == 0>(w[j]);
      x[2 * j] = f.x, x[2 * j + 1] = f.y;
    }
  }
}
template <int kDtype>
__device__ __forceinline__ void store8(void* base, long long i, const float (&x)[8]) {
  if constexpr (kDtype == 2) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i);
    p[0] = make_float4(x[0], x[1], x[2], x[3]);
    p[1] = make_float4(x[4], x[5], x[6], x[7]);
  } else {
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base) + i) =
        make_uint4(pack2<kDtype == 0>(x[0], x[1]), pack2<kDtype == 0>(x[2], x[3]),
                   pack2<kDtype == 0>(x[4], x[5]), pack2<kDtype == 0>(x[6], x[7]));
  }
}

// One thread per (batch, token, head, group of 8 rotation pairs): it rotates pairs
// [8t, 8t + 8) of q and of k and copies the same coordinates of v (elements [8t, 8t + 8)
// and [8t + D/2, 8t + D/2 + 8)), every access a 16-byte piece (two for fp32).
template <int kDtype>
__global__ void __launch_bounds__(256) qkv_rope_cache_kernel(const RopeCacheParams p) {
  griddep_launch_dependents();  // the decode after it may launch now and wait for it there
  const int groups = p.D / 16;  // threads per (batch, token, head)
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long units = static_cast<long long>(p.B) * p.S * p.H * groups;
  if (gid >= units) return;
  const int t = static_cast<int>(gid % groups);
  long long u = gid / groups;
  const int h = static_cast<int>(u % p.H);
  u /= p.H;
  const int s = static_cast<int>(u % p.S);
  const int b = static_cast<int>(u / p.S);

  // A negative row0 places the tokens at cache rows positions[0] + s: the cache row then
  // follows a position tensor that stays on the device, so one captured launch serves every
  // block of a sampling loop. A row range outside the cache writes nothing (status bit 4).
  const long long row0 = p.row0 >= 0 ? p.row0 : p.positions[0];
  if (row0 < 0 || row0 + p.S > p.cache_rows) {
    if (t == 0) atomicOr(&g_bd3_status, kStatusBadPosition);
    return;
  }
  const long long pos = p.positions != nullptr ? p.positions[s] : p.pos0 + s;
  if (pos < 0 || pos >= p.max_pos) {
    if (t == 0) atomicOr(&g_bd3_status, kStatusBadPosition);
    return;
  }
  const int half = p.D / 2;
  const long long src = b * p.qkv_sb + s * p.qkv_ss;  // this token's (3, H, D) block
  const long long hq = static_cast<long long>(h) * p.D;
  const long long hk = hq + static_cast<long long>(p.H) * p.D;
  const long long hv = hk + static_cast<long long>(p.H) * p.D;
  const float* ct = p.cos_table + pos * half + 8 * t;
  const float* st = p.sin_table + pos * half + 8 * t;
  const long long qo = b * p.q_sb + h * p.q_sh + s * p.q_ss;
  const long long ko = b * p.k_sb + h * p.k_sh + (row0 + s) * p.k_ss;
  const long long vo = b * p.v_sb + h * p.v_sh + (row0 + s) * p.v_ss;
  const int k = 8 * t;
  float c[8], sn[8];
  {
    const float4 c0 = reinterpret_cast<const float4*>(ct)[0], c1 = reinterpret_cast<const float4*>(ct)[1];
    const float4 s0 = reinterpret_cast<const float4*>(st)[0], s1 = reinterpret_cast<const float4*>(st)[1];
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) c[e] = rnd<kDtype>(cv[e]), sn[e] = rnd<kDtype>(sv[e]);
  }
#pragma unroll
  for (int w = 0; w < 2; ++w) {  // q, then k
    const long long base = src + (w == 0 ? hq : hk);
    float x1[8], x2[8], o1[8], o2[8];
    load8<kDtype>(p.qkv, base + k, x1);
    load8<kDtype>(p.qkv, base + k + half, x2);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o1[e] = rnd<kDtype>(__fsub_rn(rnd<kDtype>(__fmul_rn(x1[e], c[e])),
                                    rnd<kDtype>(__fmul_rn(x2[e], sn[e]))));
      o2[e] = rnd<kDtype>(__fadd_rn(rnd<kDtype>(__fmul_rn(x1[e], sn[e])),
                                    rnd<kDtype>(__fmul_rn(x2[e], c[e]))));
    }
    if (w == 0) {
      if (p.q_out != nullptr) {
        store8<kDtype>(p.q_out, qo + k, o1);
        store8<kDtype>(p.q_out, qo + k + half, o2);
      }
    } else {
      store8<kDtype>(p.k_cache, ko + k, o1);
      store8<kDtype>(p.k_cache, ko + k + half, o2);
    }
  }
  float v1[8], v2[8];
  load8<kDtype>(p.qkv, src + hv + k, v1);
  load8<kDtype>(p.qkv, src + hv + k + half, v2);
  store8<kDtype>(p.v_cache, vo + k, v1);
  store8<kDtype>(p.v_cache, vo + k + half, v2);
}

}  // namespace bd3
