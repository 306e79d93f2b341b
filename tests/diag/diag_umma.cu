// Diagnostic library (libbd3diag.so, tests only): one CTA exercises, in isolation, each
// tcgen05 operand layout the attention kernels rely on, so a layout error shows up as a
// precise mismatch instead of a wrong attention output.
//   S = A Bk^T       SS form, both operands K-major, 128-byte swizzle (forward Q K^T)
//   O = P V          TS form: P = bf16(S / 16) written to TMEM by the threads, V an MN-major
//                    operand (forward P V, dQ += dS K)
//   C = X^T Y        SS form: X written by threads as a [k][m] swizzled tile = MN-major A,
//                    Y an MN-major B (dK/dV: dV += P^T dO)
// Inputs are contiguous bf16: A, Bk, V, Y are 128 x 64; X is 128 (k) x 128 (m).
// Outputs are fp32: S 128 x 128, O 128 x 64, C 128 x 64.
#include <cstdint>

#include "../../diffusion-llm_b200/csrc/common.cuh"

namespace {

using namespace bd3;

struct DiagSmem {
  static constexpr uint32_t kA = 0, kB = 16384, kV = 32768, kY = 49152, kX = 65536;  // X: 32 KB
  static constexpr uint32_t kBar = 98304;  // load, s_full, p_full, done
  static constexpr uint32_t kSlot = kBar + 64;
  static constexpr uint32_t kAlloc = kSlot + 16 + 1024;
};

__global__ void __launch_bounds__(192, 1)
    diag_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_y,
                const uint16_t* __restrict__ X, float* S, float* O, float* C) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DiagSmem::kBar);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + DiagSmem::kSlot);
  const int warp = static_cast<int>(warp_id());
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 128);
    mbar_init(&bars[3], 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  // X into the [m half][k row][128 B] swizzled layout, by plain stores
  for (int idx = threadIdx.x; idx < 128 * 16; idx += blockDim.x) {
    const int krow = idx >> 4, chunk = idx & 15;  // 16 chunks of 8 m-values per k row
    const uint4 val = *reinterpret_cast<const uint4*>(X + krow * 128 + chunk * 8);
    *reinterpret_cast<uint4*>(smem + DiagSmem::kX + (chunk >> 3) * 16384 +
                              sw128_offset(krow, chunk & 7)) = val;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 4) {
    if (elect_one()) {
      mbar_expect_tx(&bars[0], 4 * 16384);
      tma_load_4d(&tm_a, &bars[0], smem + DiagSmem::kA, 0, 0, 0, 0);
      tma_load_4d(&tm_b, &bars[0], smem + DiagSmem::kB, 0, 0, 0, 0);
      tma_load_4d(&tm_v, &bars[0], smem + DiagSmem::kV, 0, 0, 0, 0);
      tma_load_4d(&tm_y, &bars[0], smem + DiagSmem::kY, 0, 0, 0, 0);
    }
    __syncwarp();
  } else if (warp == 5) {
    if (elect_one()) {
      bool ok = mbar_wait(&bars[0], 0);
      tc_fence_after();
      const uint64_t ad = sw128_desc(sbase + DiagSmem::kA, 16, 1024);
      const uint64_t bd = sw128_desc(sbase + DiagSmem::kB, 16, 1024);
      if (ok) {
        for (int kk = 0; kk < 4; ++kk)
          umma_ss(tmem, ad + kk * 2, bd + kk * 2, idesc_f16(128, 128, false, false, true), kk > 0);
        umma_commit(&bars[1]);
        ok = mbar_wait(&bars[2], 0);
      }
      if (ok) {
        tc_fence_after();
        const uint64_t vd = sw128_desc(sbase + DiagSmem::kV, 16384, 1024);
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + 256, tmem + 128 + kk * 8, vd + ((kk * 2048) >> 4),
                  idesc_f16(128, 64, false, true, true), kk > 0);
        const uint64_t xd = sw128_desc(sbase + DiagSmem::kX, 16384, 1024);
        const uint64_t yd = sw128_desc(sbase + DiagSmem::kY, 16384, 1024);
        for (int kk = 0; kk < 8; ++kk)
          umma_ss(tmem + 320, xd + ((kk * 2048) >> 4), yd + ((kk * 2048) >> 4),
                  idesc_f16(128, 64, true, true, true), kk > 0);
        umma_commit(&bars[3]);
      }
    }
    __syncwarp();
  } else {
    const int row = threadIdx.x;
    const uint32_t lb = static_cast<uint32_t>(warp * 32) << 16;
    bool ok = mbar_wait(&bars[1], 0);
    if (ok) {
      tc_fence_after();
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lb + c * 32, r);
        uint32_t pk[16];
        for (int i = 0; i < 32; ++i) S[row * 128 + c * 32 + i] = __uint_as_float(r[i]);
        for (int i = 0; i < 16; ++i)
          pk[i] = pack2<true>(__uint_as_float(r[2 * i]) * 0.0625f,
                              __uint_as_float(r[2 * i + 1]) * 0.0625f);
        tmem_st16(tmem + lb + 128 + c * 16, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars[2]);
      ok = mbar_wait(&bars[3], 0);
    }
    if (ok) {
      tc_fence_after();
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lb + 256 + c * 32, r);
        for (int i = 0; i < 32; ++i) O[row * 64 + c * 32 + i] = __uint_as_float(r[i]);
        tmem_ld32(tmem + lb + 320 + c * 32, r);
        for (int i = 0; i < 32; ++i) C[row * 64 + c * 32 + i] = __uint_as_float(r[i]);
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

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int map128x64(CUtensorMap* m, const void* p) {
  void* fp = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fp, cudaEnableDefault, &q) != cudaSuccess)
    return 3;
  cuuint64_t dims[4] = {64, 128, 1, 1};
  cuuint64_t str[3] = {128, 128 * 128, 128 * 128};
  cuuint32_t box[4] = {64, 128, 1, 1}, es[4] = {1, 1, 1, 1};
  return reinterpret_cast<EncodeTiledFn>(fp)(
             m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(p), dims, str, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : 3;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int bd3diag_umma_selftest(const void* A, const void* Bk, const void* V,
                                     const void* X, const void* Y, float* S, float* O, float* C,
                                     void* stream) {
  CUtensorMap ta, tb, tv, ty;
  if (map128x64(&ta, A) || map128x64(&tb, Bk) || map128x64(&tv, V) || map128x64(&ty, Y)) return 3;
  if (cudaFuncSetAttribute(diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DiagSmem::kAlloc) != cudaSuccess)
    return 3;
  diag_kernel<<<1, 192, DiagSmem::kAlloc, static_cast<cudaStream_t>(stream)>>>(
      ta, tb, tv, ty, static_cast<const uint16_t*>(X), S, O, C);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// exp2_fma2 (the FMA-pipe exponential of the forward softmax) and ex2.approx on the same
// arguments, for the error-bound test.
__global__ void diag_exp2_kernel(const float* t, float* poly, float* mufu, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i + 1 >= n) return;
  const float2 e = bd3::exp2_fma2(make_float2(t[i], t[i + 1]));
  poly[i] = e.x;
  poly[i + 1] = e.y;
  mufu[i] = bd3::ex2(t[i]);
  mufu[i + 1] = bd3::ex2(t[i + 1]);
}

extern "C" __attribute__((visibility("default"))) int bd3diag_exp2(const float* t, float* poly,
                                                                  float* mufu, int n,
                                                                  void* stream) {
  if (n <= 0 || n % 2) return 1;
  const int threads = 256, blocks = (n / 2 + threads - 1) / threads;
  diag_exp2_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(t, poly, mufu, n);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}
