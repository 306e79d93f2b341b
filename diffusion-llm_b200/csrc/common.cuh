// Device helpers shared by the BD3-LM attention kernels (sm_100a only).
//
// mbarrier / TMA (cp.async.bulk.tensor) / tcgen05 (UMMA into TMEM) wrappers written from
// the PTX ISA. The shared-memory and instruction descriptor bit layouts follow the public
// CUTLASS header cute/arch/mma_sm100_desc.hpp (UMMA::SmemDescriptor, UMMA::InstrDescriptor).
//
// Every wait is bounded: a barrier that does not complete within kWaitNs nanoseconds sets
// a sticky bit in g_bd3_status (read by the host through bd3_device_status) and the wait
// returns false, so a kernel can unwind, free its TMEM and exit instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library targets sm_100a only"
#endif

namespace bd3 {

// ---- sticky device status ------------------------------------------------------------
enum : unsigned {
  kStatusWaitTimeout = 1u,   // an mbarrier wait ran out of time
  kStatusBadLaunch = 2u,     // a kernel saw launch parameters it cannot handle
  kStatusFixedRange = 8u,    // a dQ partial outside the deterministic backward's fixed-point range
};
__device__ unsigned int g_bd3_status;
// Where the first bounded wait that ran out gave up: [0] set flag, [1] block, [2] thread,
// [3] the barrier's shared-memory address | parity << 31 (read by bd3_debug_wait_site).
__device__ unsigned int g_bd3_wait_site[4];

constexpr unsigned long long kWaitNs = 500000000ull;  // 0.5 s: far above any legitimate wait

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Work item of this CTA's k-th turn in a persistent loop: turns are rounds of gridDim.x
// consecutive items taken in alternating directions, so a list ordered heaviest first gives
// each CTA one early (heavy) and one late (light) item of every pair of rounds. Increasing
// in k for every CTA, so the first item index past the end ends the loop.
__device__ __forceinline__ int persistent_item(int k) {
  const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
  return k * G + ((k & 1) ? G - 1 - c : c);
}
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }
__device__ __forceinline__ uint32_t warp_id() {
  return __shfl_sync(0xffffffffu, threadIdx.x >> 5, 0);
}
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// ---- mbarrier ------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of the given parity to complete. Bounded: returns false when limit_ns
// nanoseconds pass first (kWaitNs in the kernels; the self-check below passes a short one).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      atomicOr(&g_bd3_status, kStatusWaitTimeout);
      if (atomicCAS(&g_bd3_wait_site[0], 0u, 1u) == 0u) {
        g_bd3_wait_site[1] = blockIdx.x;
        g_bd3_wait_site[2] = threadIdx.x;
        g_bd3_wait_site[3] = smem_u32(bar) | (parity << 31);
      }
      return false;
    }
  }
}

// Self-check of the bounded wait (bd3_debug_wait_timeout): thread 0 initialises an mbarrier
// expecting one arrival, arrives on it only when `arrive` is set, and waits for its first
// phase with the given limit. With no arrival nothing can complete the phase, so the wait
// must give up after limit_ns, set kStatusWaitTimeout and return; the kernel then exits
// normally. out[0] = 1 when the wait gave up, 0 when the phase completed; out[1] = the
// nanoseconds the wait took.
__global__ void wait_probe_kernel(unsigned long long limit_ns, int arrive,
                                  unsigned long long* out) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  if (arrive) mbar_arrive(&bar);
  const unsigned long long t0 = globaltimer_ns();
  const bool ok = mbar_wait(&bar, 0, limit_ns);
  out[1] = globaltimer_ns() - t0;
  out[0] = ok ? 0ull : 1ull;
}

// Warp-uniform wait for warps that go on to issue warp-collective (.sync.aligned)
// instructions: either every lane proceeds or none does, so a timeout cannot split a warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// ---- TMA -----------------------------------------------------------------------------
// 4-D tiled load of box {c0 (elements, innermost), c1, c2, c3} into shared memory,
// completing on `bar` (transaction bytes). Never multicast.
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}
// L2 eviction-priority policy for the cache-hinted copy below (createpolicy, whole fraction):
// evict_last keeps the lines in L2 ahead of lines loaded with the normal policy.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// tma_load_4d with an L2 cache policy.
__device__ __forceinline__ void tma_load_4d_hint(const CUtensorMap* map, uint64_t* bar, void* dst,
                                                 int c0, int c1, int c2, int c3, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Make generic-proxy shared-memory writes visible to the async proxy (TMA / tensor cores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 -------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16/f16 in, fp32 accumulate).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16; A is M lanes x 16 elements (8 columns).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor for a 128-byte-swizzled operand (sm100 version bits).
//   K-major:  8-row x 128 B atoms, atoms stacked along M/N every `sbo` bytes; lbo unused (16).
//   MN-major: 64-element x 8-row atoms; `sbo` = stride between 8-row K groups, `lbo` =
//             stride between 64-element M/N groups.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16 with fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn_major,
                                                 bool b_mn_major, bool bf16) {
  return (1u << 4)                                          // D format: F32
         | (static_cast<uint32_t>(bf16) << 7)               // A format: BF16=1, F16=0
         | (static_cast<uint32_t>(bf16) << 10)              // B format
         | (static_cast<uint32_t>(a_mn_major) << 15)        // A major
         | (static_cast<uint32_t>(b_mn_major) << 16)        // B major
         | (static_cast<uint32_t>(N >> 3) << 17)            // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);           // M / 16
}

// TMEM load: 32 lanes x 32 bits, N consecutive columns per thread, with the wait folded in
// so no register is read before the data has arrived.
#define BD3_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                  "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : BD3_R8(0), BD3_R8(8), BD3_R8(16), BD3_R8(24)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : BD3_R8(0), BD3_R8(8)
      : "r"(taddr)
      : "memory");
}
// The same loads without the wait, so several can be in flight: call tmem_ld_wait() and then
// reg_fence() on the destination registers before reading them (the fence makes every later
// use of the registers depend on an instruction that follows the wait).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n"
      : BD3_R8(0), BD3_R8(8)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : BD3_R8(0), BD3_R8(8), BD3_R8(16), BD3_R8(24)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}
#undef BD3_R8
#define BD3_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), \
                  "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(
                   taddr),
               BD3_W8(0)
               : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};\n" ::"r"(taddr),
      BD3_W8(0), BD3_W8(8)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(
          taddr),
      BD3_W8(0), BD3_W8(8), BD3_W8(16), BD3_W8(24)
      : "memory");
}
#undef BD3_W8
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- small numeric helpers -----------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// max of three floats in one instruction (sm_100)
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Max over 64 registers as a tree of three-input maxes (depth 4, 32 instructions).
__device__ __forceinline__ float max64(const float (&x)[64]) {
  float m[22], n[8];
#pragma unroll
  for (int i = 0; i < 21; ++i) m[i] = max3(x[3 * i], x[3 * i + 1], x[3 * i + 2]);
  m[21] = x[63];
#pragma unroll
  for (int i = 0; i < 7; ++i) n[i] = max3(m[3 * i], m[3 * i + 1], m[3 * i + 2]);
  n[7] = m[21];
  return max3(max3(n[0], n[1], n[2]), max3(n[3], n[4], n[5]), fmaxf(n[6], n[7]));
}

// 2^t for two arguments on the FMA pipe instead of the MUFU unit (which the softmax saturates).
// Range reduction after Cody and Waite: t = j + f with j = floor(t) and f in [0, 1), so
// 2^t = 2^j * 2^f; 2^j is added to the exponent field and 2^f is a cubic
// p(f) = 1 + f (c1 + f (c2 + f c3)). The coefficients minimise the maximum relative error on
// [0, 1): a weighted least-squares fit of (2^f - 1) / 2^f by f (c1 + f (c2 + f c3)) / 2^f on
// 20000 points of (0, 1], its weights updated by Lawson's iteration (each weight times its
// point's absolute residual, renormalised) until the residual equioscillates, the result
// rounded to fp32. Maximum relative error of the fp32 evaluation:
// 8.6e-5, under half an ulp of bf16 and fp16 (the P operand's types). The floor comes from
// adding 1.5 * 2^23 with rounding toward -inf, which leaves floor(t) in the low mantissa bits.
// t is clamped to -127 first: there j = -127 and p(0) = 1, so the result's bits are exactly 0
// (+0.0, matching ex2.approx.ftz for -inf). The callers keep t <= 8.
__device__ __forceinline__ float2 exp2_fma2(float2 t) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC1 = 0.6951168179512024f, kC2 = 0.22764484584331512f,
                  kC3 = 0.07706718146800995f;
  t.x = fmaxf(t.x, -127.f);
  t.y = fmaxf(t.y, -127.f);
  const float2 y = __fadd2_rd(t, make_float2(kMagic, kMagic));
  const float2 jf = __fadd2_rn(y, make_float2(-kMagic, -kMagic));
  const float2 f = __ffma2_rn(jf, make_float2(-1.f, -1.f), t);
  float2 p = __ffma2_rn(f, make_float2(kC3, kC3), make_float2(kC2, kC2));
  p = __ffma2_rn(f, p, make_float2(kC1, kC1));
  p = __ffma2_rn(f, p, make_float2(1.f, 1.f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(y.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(y.y) << 23)));
}

// Round a float through dtype kDtype (0 bf16, 1 fp16, 2 fp32: identity) and back, as a
// PyTorch elementwise op on tensors of that dtype rounds its fp32 result.
// Programmatic dependent launch. A kernel launched with the programmatic-serialization
// attribute may start while the kernel before it on the stream is still running, once every
// CTA of that kernel has called griddep_launch_dependents (or exited); griddep_wait then
// blocks until that kernel has completed and its memory is visible. Without the attribute
// (or after a kernel that never triggers) both are no-ops in effect.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <int kDtype>
__device__ __forceinline__ float rnd(float x) {
  if constexpr (kDtype == 0) return __bfloat162float(__float2bfloat16_rn(x));
  else if constexpr (kDtype == 1) return __half2float(__float2half_rn(x));
  else return x;
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}
template <bool kBF16>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(v);
  } else {
    __half2 v = *reinterpret_cast<__half2*>(&u);
    return __half22float2(v);
  }
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a 128B-swizzled tile whose
// rows are 128 bytes: the swizzle XORs the chunk index with the row index modulo 8.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace bd3
