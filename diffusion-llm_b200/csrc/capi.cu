// C-ABI entry points of libbd3attn.so (declared in include/bd3_attn.h).
//
// Host side only: argument validation (mirroring the reference's assertions), TMA tensor
// map construction, launch planning and kernel launches. No allocation happens here: the
// caller passes every output and workspace buffer.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/bd3_attn.h"
#include "attn_bwd.cuh"
#include "attn_fwd.cuh"
#include "attn_fwd_pair.cuh"
#include "decode.cuh"
#include "f32_scale.cuh"
#include "kv_rope.cuh"
#include "peer_merge.cuh"
#include "sampler.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(BD3_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ---- cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda) ----
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

size_t elem_bytes(int dtype) { return dtype == BD3_F32 ? 4 : 2; }

// 4-D map over (head_dim=64, seq, heads, batch) with a {64, box_rows, 1, 1} box, 128-byte
// swizzle, zero fill out of bounds.
int make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t seq, int64_t H, int64_t B,
             const int64_t* strides /* b, h, s */, int box_rows, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(BD3_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const size_t es = elem_bytes(dtype);
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
    return fail(BD3_ERR_INVALID, "%s: pointer must be 16-byte aligned", name);
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(seq), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(B)};
  int64_t sb = strides[0], sh = strides[1], ss = strides[2];
  // a size-1 dimension is never stepped over: give it a legal stride
  if (seq == 1) ss = 64;
  if (H == 1) sh = ss * seq;
  if (B == 1) sb = sh * H;
  const int64_t st[3] = {ss, sh, sb};
  cuuint64_t gstr[3];
  for (int i = 0; i < 3; ++i) {
    const int64_t bytes = st[i] * static_cast<int64_t>(es);
    if (st[i] <= 0 || bytes % 16 != 0 || bytes >= (int64_t(1) << 40))
      return fail(BD3_ERR_INVALID,
                  "%s: strides must be positive multiples of 16 bytes (got %lld elements)", name,
                  static_cast<long long>(st[i]));
    gstr[i] = static_cast<cuuint64_t>(bytes);
  }
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == BD3_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dtype == BD3_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUresult r = fn(map, dt, 4, const_cast<void*>(ptr), dims, gstr, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BD3_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, int(r));
  return BD3_OK;
}

int current_device_sms(int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  static int cache[64] = {0};
  if (dev < 64 && cache[dev] > 0) {
    *sms = cache[dev];
    return BD3_OK;
  }
  e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if (dev < 64) cache[dev] = *sms;
  return BD3_OK;
}

// Opt a kernel into its dynamic shared memory once per device.
template <typename K>
int set_smem(K kernel, uint32_t bytes, int slot) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  static bool done[64][32] = {};
  if (dev < 64 && slot < 32 && done[dev][slot]) return BD3_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  if (dev < 64 && slot < 32) done[dev][slot] = true;
  return BD3_OK;
}


// ---- optional per-kernel timing (bd3_profile_*): CUDA event pairs around each launch ----
enum ProfId {
  kPfFwd = 0, kPfPrefill, kPfDelta, kPfDq, kPfDkdv, kPfDecode, kPfCombine, kPfRope, kPfSample,
  kPfNum
};
constexpr int kProfCap = 8192;
struct Prof {
  bool on = false;
  int n = 0;
  int id[kProfCap];
  cudaEvent_t ev[kProfCap][2];
  bool created = false;
};
Prof& prof() {
  static Prof p;
  return p;
}
struct ProfScope {
  int slot = -1;
  cudaStream_t st;
  ProfScope(int kernel, cudaStream_t s) : st(s) {
    Prof& p = prof();
    if (!p.on || p.n >= kProfCap) return;
    slot = p.n++;
    p.id[slot] = kernel;
    cudaEventRecord(p.ev[slot][0], st);
  }
  ~ProfScope() {
    if (slot >= 0) cudaEventRecord(prof().ev[slot][1], st);
  }
};

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BD3_OK : cuda_fail(e, what);
}

// Launch with programmatic stream serialization: the kernel may begin while the previous
// kernel on the stream finishes, and orders itself after it with griddep_wait (the decode
// and combine kernels do so before reading anything the previous kernel writes).
template <typename... Params, typename... Args>
int launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
               cudaStream_t stream, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e == cudaSuccess ? check_launch(what) : cuda_fail(e, what);
}

// Launch with programmatic stream serialization and a (cluster_x, 1, 1) cluster.
template <typename... Params, typename... Args>
int launch_pdl_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       unsigned cluster_x, cudaStream_t stream, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e == cudaSuccess ? check_launch(what) : cuda_fail(e, what);
}

// Bind the current device's primary context to this host thread. A thread that has only
// used another CUDA runtime (torch's autograd workers, for one) may have no current driver
// context, and cuTensorMapEncodeTiled is a driver call.
int ensure_context() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return BD3_OK;
}

int check_dims(int64_t B, int64_t H, int64_t D, int dtype) {
  const int rc = ensure_context();
  if (rc != BD3_OK) return rc;
  if (B < 1 || H < 1) return fail(BD3_ERR_INVALID, "batch and heads must be >= 1");
  if (D != 64) return fail(BD3_ERR_UNSUPPORTED, "head_dim must be 64 (got %lld)", (long long)D);
  if (dtype != BD3_BF16 && dtype != BD3_F16)
    return fail(BD3_ERR_UNSUPPORTED, "inputs must be bf16 or f16 (dtype code %d)", dtype);
  if (B * H > 65535 * 1024LL) return fail(BD3_ERR_UNSUPPORTED, "batch * heads too large");
  return BD3_OK;
}

// ---------------------------------------------------------------------------------------
int launch_fwd(int mode, const void* q, const void* k, const void* v, void* o, float* lse,
               int64_t B, int64_t H, int64_t n, int64_t q_len, int64_t kv_len,
               const int64_t* strides, int64_t bs, int dtype, cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  const int64_t q_rows = mode == bd3::kTrain ? 2 * n : q_len;
  const int64_t kv_rows = mode == bd3::kTrain ? 2 * n : kv_len;
  int rc;
  if ((rc = make_map(&tq, q, dtype, q_rows, H, B, strides + 0, bd3::kFwdBM, "q")) != BD3_OK) return rc;
  if ((rc = make_map(&tk, k, dtype, kv_rows, H, B, strides + 3, bd3::kFwdBN, "k")) != BD3_OK) return rc;
  if ((rc = make_map(&tv, v, dtype, kv_rows, H, B, strides + 6, bd3::kFwdBN, "v")) != BD3_OK) return rc;
  const int64_t* so = strides + 9;
  if (reinterpret_cast<uintptr_t>(o) % 16 || so[0] % 8 || so[1] % 8 || so[2] % 8)
    return fail(BD3_ERR_INVALID, "o: pointer and strides must be 16-byte aligned");
  CUtensorMap to;
  if ((rc = make_map(&to, o, dtype, q_rows, H, B, so, bd3::kFwdBM, "o")) != BD3_OK) return rc;
  bd3::FwdParams p{};
  p.o = o;
  p.lse = lse;
  p.o_sb = so[0];
  p.o_sh = so[1];
  p.o_ss = so[2];
  p.lse_sh = q_rows;
  p.lse_sb = H * q_rows;
  p.H = static_cast<int>(H);
  p.n = static_cast<int>(n);
  p.q_len = static_cast<int>(q_len);
  p.kv_len = static_cast<int>(kv_len);
  p.bs = static_cast<int>(bs);
  p.num_q_tiles = static_cast<int>(bd3::cdiv(static_cast<int>(q_rows), bd3::kFwdBM));
  p.num_bh = static_cast<int>(B * H);
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  const int64_t items = B * H * p.num_q_tiles;
  if (items > 2147483647LL) return fail(BD3_ERR_UNSUPPORTED, "too many query tiles");
  int sms = 148;
  if ((rc = current_device_sms(&sms)) != BD3_OK) return rc;
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
               const bd3::FwdParams);
  int slot;
  if (mode == bd3::kTrain) {
    // items are (batch*head, tile pair): the noisy and clean query tiles i share K/V
    const int64_t pairs = B * H * (n / bd3::kFwdBM);
    const int64_t grid = pairs < sms ? pairs : sms;  // persistent: one CTA per SM
    kern = dtype == BD3_BF16 ? bd3::attn_fwd_pair_kernel<true> : bd3::attn_fwd_pair_kernel<false>;
    slot = dtype == BD3_BF16 ? 0 : 1;
    if ((rc = set_smem(kern, bd3::PairSmem::kAlloc, slot)) != BD3_OK) return rc;
    ProfScope ps(kPfFwd, stream);
    kern<<<static_cast<unsigned>(grid), bd3::kPairThreads, bd3::PairSmem::kAlloc, stream>>>(
        tq, tk, tv, to, p);
    return check_launch("attn_fwd_pair_kernel launch");
  }
  const int64_t grid = items < sms ? items : sms;  // persistent: one CTA per SM
  {
    kern = dtype == BD3_BF16 ? bd3::attn_fwd_kernel<bd3::kDecode, true>
                             : bd3::attn_fwd_kernel<bd3::kDecode, false>;
    slot = dtype == BD3_BF16 ? 2 : 3;
  }
  if ((rc = set_smem(kern, bd3::FwdSmem::kAlloc, slot)) != BD3_OK) return rc;
  ProfScope ps(kPfPrefill, stream);
  kern<<<static_cast<unsigned>(grid), bd3::kFwdThreads, bd3::FwdSmem::kAlloc, stream>>>(tq, tk, tv, to, p);
  return check_launch("attn_fwd_kernel launch");
}

// Visible-key bound of the last query row: tiles at or past it are never read.
int64_t decode_hi(int64_t q_len, int64_t kv_len, int64_t bs, int64_t q_pos0, int64_t kv_pos0) {
  const int64_t hi = ((q_pos0 + q_len - 1) / bs + 1) * bs - kv_pos0;
  return hi < kv_len ? hi : kv_len;
}

// Splits of a (batch*head, row group) merged inside the decode kernel through a thread-block
// cluster (decode_kernel<..., kCluster>; no workspace, no combine launch): 2 to 16 of them,
// and only when the whole grid is resident at once (two decode CTAs per SM). In a grid of
// several waves a cluster's finished CTAs would hold their SMs at the cluster barrier until
// the slowest sibling is done (measured: B=8 x 16K keys, 9 splits, 89 us against 75 with the
// combine kernel), while a single-wave grid saves the combine launch (B=1 x 1K: 12.3 against
// 15.4 us).
constexpr int64_t kMaxClusterSplits = 16;
bool cluster_splits(int64_t n_splits, int64_t groups_total, int sms) {
  return n_splits >= 2 && n_splits <= kMaxClusterSplits && groups_total * n_splits <= 2 * sms;
}

// Pick units (key tiles or live entries) per split with a small cost model: whole waves of
// resident CTAs times (units per CTA + a fixed per-CTA overhead of 1.5 units).
int64_t pick_units_per_split(int64_t ctas_per_split_unit_group, int64_t units, int sms) {
  const int64_t slots = static_cast<int64_t>(sms) * 3;  // 3 resident decode CTAs per SM
  int64_t best_u = 1;
  double best = 1e300;
  for (int64_t u = 1; u <= 64 && u <= units; ++u) {
    const int64_t ctas = ctas_per_split_unit_group * ((units + u - 1) / u);
    const double est = static_cast<double>((ctas + slots - 1) / slots) * (u + 1.5);
    if (est <= best) {
      best = est;
      best_u = u;
    }
  }
  return best_u;
}

}  // namespace

extern "C" {

int bd3_version(void) { return 100; }

const char* bd3_last_error(void) { return g_last_error.c_str(); }

int bd3_device_status(int clear) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, bd3::g_bd3_status, sizeof(v));
  if (e != cudaSuccess) {
    cuda_fail(e, "reading the device status");
    return -1;
  }
  if (clear && v) {
    unsigned z = 0;
    e = cudaMemcpyToSymbol(bd3::g_bd3_status, &z, sizeof(z));
    if (e != cudaSuccess) {
      cuda_fail(e, "clearing the device status");
      return -1;
    }
  }
  return static_cast<int>(v);
}

int bd3_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                 int64_t H, int64_t n, int64_t D, const int64_t* strides, int64_t block_size,
                 int dtype, void* stream) {
  int rc = check_dims(B, H, D, dtype);
  if (rc != BD3_OK) return rc;
  if (n < 1 || n % bd3::kFwdBM != 0)
    return fail(BD3_ERR_INVALID, "n must be a positive multiple of 128 (got %lld)", (long long)n);
  if (n > (1 << 29)) return fail(BD3_ERR_UNSUPPORTED, "sequence too long");
  if (block_size < 1) return fail(BD3_ERR_INVALID, "block_size must be >= 1");
  if (lse == nullptr || reinterpret_cast<uintptr_t>(lse) % 4)
    return fail(BD3_ERR_INVALID, "lse must be a valid fp32 buffer");
  return launch_fwd(bd3::kTrain, q, k, v, o, lse, B, H, n, 2 * n, 2 * n, strides, block_size,
                    dtype, static_cast<cudaStream_t>(stream));
}

size_t bd3_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t n, int64_t D) {
  (void)D;
  if (B < 1 || H < 1 || n < 1) return 0;
  // Delta and LSE*log2(e) per query row, then the fp32 dQ accumulator (64 per row)
  return static_cast<size_t>(B * H * 2 * n) * (1 + 1 + 64) * sizeof(float);
}

size_t bd3_attn_bwd_det_workspace_size(int64_t B, int64_t H, int64_t n, int64_t D) {
  (void)D;
  if (B < 1 || H < 1 || n < 1) return 0;
  // Delta and LSE*log2(e) per query row, then the int64 fixed-point dQ accumulator
  return static_cast<size_t>(B * H * 2 * n) * (2 * sizeof(float) + 64 * sizeof(int64_t));
}

}  // extern "C"

namespace {
int launch_bwd(bool det, const void* q, const void* k, const void* v, const void* o,
               const float* lse, const void* dout, void* dq, void* dk, void* dv, int64_t B,
               int64_t H, int64_t n, int64_t D, const int64_t* strides, int64_t block_size,
               int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_dims(B, H, D, dtype);
  if (rc != BD3_OK) return rc;
  if (n < 1 || n % bd3::kBwdBKV != 0)
    return fail(BD3_ERR_INVALID, "n must be a positive multiple of 128 (got %lld)", (long long)n);
  if (n > (1 << 29)) return fail(BD3_ERR_UNSUPPORTED, "sequence too long");
  if (block_size < 1 || n % block_size != 0)
    return fail(BD3_ERR_INVALID, "n must be a multiple of block_size (n=%lld, block_size=%lld)",
                (long long)n, (long long)block_size);
  const size_t need = det ? bd3_attn_bwd_det_workspace_size(B, H, n, D)
                          : bd3_attn_bwd_workspace_size(B, H, n, D);
  if (workspace == nullptr || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 16)
    return fail(BD3_ERR_WORKSPACE, "backward workspace too small: need %zu bytes, got %zu", need,
                workspace_bytes);
  if (lse == nullptr || reinterpret_cast<uintptr_t>(lse) % 16)
    return fail(BD3_ERR_INVALID, "lse must be a 16-byte aligned fp32 buffer");
  const int64_t S = 2 * n;
  CUtensorMap tq, tk, tv, tdo;
  if ((rc = make_map(&tq, q, dtype, S, H, B, strides + 0, 128, "q")) != BD3_OK) return rc;
  if ((rc = make_map(&tk, k, dtype, S, H, B, strides + 3, 128, "k")) != BD3_OK) return rc;
  if ((rc = make_map(&tv, v, dtype, S, H, B, strides + 6, 128, "v")) != BD3_OK) return rc;
  if ((rc = make_map(&tdo, dout, dtype, S, H, B, strides + 12, 128, "dout")) != BD3_OK) return rc;
  CUtensorMap tdk, tdv;
  if ((rc = make_map(&tdk, dk, dtype, S, H, B, strides + 18, 128, "dk")) != BD3_OK) return rc;
  if ((rc = make_map(&tdv, dv, dtype, S, H, B, strides + 21, 128, "dv")) != BD3_OK) return rc;
  const void* ptrs[5] = {o, dout, dq, dk, dv};
  const int idx[5] = {9, 12, 15, 18, 21};
  const char* names[5] = {"o", "dout", "dq", "dk", "dv"};
  for (int t = 0; t < 5; ++t) {
    const int64_t* s3 = strides + idx[t];
    if (reinterpret_cast<uintptr_t>(ptrs[t]) % 16 || s3[0] % 8 || s3[1] % 8 || s3[2] % 8)
      return fail(BD3_ERR_INVALID, "%s: pointer and strides must be 16-byte aligned", names[t]);
  }
  const int64_t rows = B * H * S;
  // the fp32 dQ accumulator as a (rows, 64) matrix for the TMA reduce-adds: 32-column boxes
  // of 128 rows with the 128-byte swizzle
  CUtensorMap tdqa;
  {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return fail(BD3_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    float* acc = static_cast<float*>(workspace) + 2 * rows;
    cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(rows)};
    cuuint64_t gstr[1] = {64 * sizeof(float)};
    cuuint32_t box[2] = {32, 128}, estr[2] = {1, 1};
    const CUresult r = fn(&tdqa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, acc, dims, gstr, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(BD3_ERR_CUDA, "dQ accumulator tensor map failed (%d)", int(r));
  }
  bd3::BwdParams p{};
  p.o = o;
  p.dout = dout;
  p.lse = lse;
  p.delta = static_cast<float*>(workspace);
  p.lse2 = p.delta + rows;
  p.dq_acc = p.lse2 + rows;
  p.dq_fix = reinterpret_cast<unsigned long long*>(p.lse2 + rows);  // kDet: the int64 accumulator
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.o_sb = strides[9]; p.o_sh = strides[10]; p.o_ss = strides[11];
  p.do_sb = strides[12]; p.do_sh = strides[13]; p.do_ss = strides[14];
  p.dq_sb = strides[15]; p.dq_sh = strides[16]; p.dq_ss = strides[17];
  p.dk_sb = strides[18]; p.dk_sh = strides[19]; p.dk_ss = strides[20];
  p.dv_sb = strides[21]; p.dv_sh = strides[22]; p.dv_ss = strides[23];
  p.H = static_cast<int>(H);
  p.n = static_cast<int>(n);
  p.bs = static_cast<int>(block_size);
  p.num_tiles = static_cast<int>(S / bd3::kBwdBKV);
  p.num_bh = static_cast<int>(B * H);
  p.scale = 0.125f;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == BD3_BF16;
  const unsigned eblocks = static_cast<unsigned>((rows * 8 + 255) / 256);
  {
    ProfScope ps(kPfDelta, st);
    auto prep = bf ? (det ? bd3::bwd_prep_kernel<true, true> : bd3::bwd_prep_kernel<true, false>)
                   : (det ? bd3::bwd_prep_kernel<false, true> : bd3::bwd_prep_kernel<false, false>);
    prep<<<eblocks, 256, 0, st>>>(p, static_cast<int>(rows));
  }
  if ((rc = check_launch("bwd_prep_kernel launch")) != BD3_OK) return rc;
  const int64_t items = B * H * p.num_tiles;
  if (items > 2147483647LL) return fail(BD3_ERR_UNSUPPORTED, "too many key tiles");
  int sms = 148;
  if ((rc = current_device_sms(&sms)) != BD3_OK) return rc;
  const unsigned grid = static_cast<unsigned>(items < sms ? items : sms);  // persistent
  auto fused = bf ? (det ? bd3::bwd_fused_kernel<true, true> : bd3::bwd_fused_kernel<true, false>)
                  : (det ? bd3::bwd_fused_kernel<false, true> : bd3::bwd_fused_kernel<false, false>);
  if ((rc = set_smem(fused, bd3::BwdSmem::kAlloc, (det ? 18 : 6) + (bf ? 0 : 1))) != BD3_OK)
    return rc;
  {
    ProfScope ps(kPfDkdv, st);
    fused<<<grid, bd3::kBwdThreads, bd3::BwdSmem::kAlloc, st>>>(tq, tk, tv, tdo, tdqa, tdk, tdv, p);
  }
  if ((rc = check_launch("bwd_fused_kernel launch")) != BD3_OK) return rc;
  {
    ProfScope ps(kPfDq, st);
    auto conv = bf ? (det ? bd3::bwd_dq_convert_kernel<true, true>
                          : bd3::bwd_dq_convert_kernel<true, false>)
                   : (det ? bd3::bwd_dq_convert_kernel<false, true>
                          : bd3::bwd_dq_convert_kernel<false, false>);
    conv<<<eblocks, 256, 0, st>>>(p, static_cast<int>(rows));
  }
  return check_launch("bwd_dq_convert_kernel launch");
}
}  // namespace

extern "C" {

int bd3_attn_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
                 const void* dout, void* dq, void* dk, void* dv, int64_t B, int64_t H,
                 int64_t n, int64_t D, const int64_t* strides, int64_t block_size, int dtype,
                 void* workspace, size_t workspace_bytes, void* stream) {
  return launch_bwd(false, q, k, v, o, lse, dout, dq, dk, dv, B, H, n, D, strides, block_size,
                    dtype, workspace, workspace_bytes, stream);
}

int bd3_attn_bwd_det(const void* q, const void* k, const void* v, const void* o,
                     const float* lse, const void* dout, void* dq, void* dk, void* dv, int64_t B,
                     int64_t H, int64_t n, int64_t D, const int64_t* strides,
                     int64_t block_size, int dtype, void* workspace, size_t workspace_bytes,
                     void* stream) {
  return launch_bwd(true, q, k, v, o, lse, dout, dq, dk, dv, B, H, n, D, strides, block_size,
                    dtype, workspace, workspace_bytes, stream);
}

int bd3_decode_plan(int64_t B, int64_t H, int64_t q_len, int64_t kv_len, int64_t block_size,
                    int64_t q_pos0, int64_t kv_pos0, int64_t* n_splits, size_t* workspace_bytes) {
  if (B < 1 || H < 1 || q_len < 1 || kv_len < 1 || block_size < 1)
    return fail(BD3_ERR_INVALID, "decode sizes must be >= 1");
  if (q_pos0 < 0) q_pos0 = kv_len - q_len;
  if (q_len > 64) {  // prefill: the tcgen05 kernel, no splits
    *n_splits = 1;
    *workspace_bytes = 0;
    return BD3_OK;
  }
  int sms = 148;
  int rc = current_device_sms(&sms);
  if (rc != BD3_OK) return rc;
  const int64_t hi = decode_hi(q_len, kv_len, block_size, q_pos0, kv_pos0);
  const int64_t tiles = hi > 0 ? (hi + bd3::kDecBN - 1) / bd3::kDecBN : 1;
  const int64_t groups = (q_len + 31) / 32;
  int64_t u = pick_units_per_split(B * H * groups, tiles, sms);
  int64_t s = (tiles + u - 1) / u;
  // more than a cluster's 16 splits: take 16 or fewer, larger splits merged inside the
  // kernel instead, when that grid is one wave and a split keeps at most 32 tiles (small,
  // launch-bound decodes, where the combine launch costs more than the longer splits)
  if (s > kMaxClusterSplits) {
    const int64_t u2 = (tiles + kMaxClusterSplits - 1) / kMaxClusterSplits;
    const int64_t s2 = (tiles + u2 - 1) / u2;
    if (u2 <= 32 && cluster_splits(s2, B * H * groups, sms)) u = u2, s = s2;
  }
  *n_splits = s;
  *workspace_bytes = s > 1 && !cluster_splits(s, B * H * groups, sms)
                         ? static_cast<size_t>(B * H * s * q_len) * (64 + 1) * 4 : 0;
  return BD3_OK;
}

namespace {
int launch_decode(bool live, const void* q, const void* k, const void* v, void* o,
                  float* lse_out, const int32_t* live_idx, const int32_t* live_cnt,
                  int64_t live_stride, int64_t max_live, int64_t kv_block, int64_t B, int64_t H,
                  int64_t q_len, int64_t kv_len, const int64_t* strides, int64_t bs,
                  int64_t q_pos0, int64_t kv_pos0, int64_t n_splits, int dtype, int out_dtype,
                  void* workspace, size_t workspace_bytes, cudaStream_t stream,
                  const int32_t* kv_len_dev = nullptr) {
  const int kmb = q_len <= 16 ? 1 : 2;
  const int64_t groups = q_len <= 32 ? 1 : (q_len + 31) / 32;
  int rc;
  CUtensorMap tq, tk, tv;
  if ((rc = make_map(&tq, q, dtype, q_len, H, B, strides + 0, kmb * 16, "q")) != BD3_OK) return rc;
  if ((rc = make_map(&tk, k, dtype, kv_len, H, B, strides + 3, bd3::kDecBN, "k")) != BD3_OK) return rc;
  if ((rc = make_map(&tv, v, dtype, kv_len, H, B, strides + 6, bd3::kDecBN, "v")) != BD3_OK) return rc;
  const int64_t* so = strides + 9;
  const int64_t oal = out_dtype == BD3_F32 ? 4 : 8;
  if (reinterpret_cast<uintptr_t>(o) % 16 || so[0] % oal || so[1] % oal || so[2] % oal)
    return fail(BD3_ERR_INVALID, "o: pointer and strides must be 16-byte aligned");
  if (n_splits < 1 || n_splits > 65535) return fail(BD3_ERR_INVALID, "n_splits out of range");
  int sms = 148;
  if ((rc = current_device_sms(&sms)) != BD3_OK) return rc;
  const bool cluster = cluster_splits(n_splits, B * H * groups, sms);
  const size_t need = n_splits > 1 && !cluster
                          ? static_cast<size_t>(B * H * n_splits * q_len) * 65 * 4 : 0;
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(BD3_ERR_WORKSPACE, "decode workspace too small: need %zu bytes, got %zu", need,
                workspace_bytes);
  bd3::DecParams p{};
  p.o = o;
  p.lse = lse_out;
  p.ws_o = static_cast<float*>(workspace);
  p.ws_lse = need > 0 ? p.ws_o + B * H * n_splits * q_len * 64 : nullptr;
  p.live_idx = live_idx;
  p.live_cnt = live_cnt;
  p.kv_len_dev = kv_len_dev;
  p.o_sb = so[0];
  p.o_sh = so[1];
  p.o_ss = so[2];
  p.H = static_cast<int>(H);
  p.q_len = static_cast<int>(q_len);
  p.kv_len = static_cast<int>(kv_len);
  p.bs = static_cast<int>(bs);
  p.q_pos0 = static_cast<int>(q_pos0);
  p.kv_pos0 = static_cast<int>(kv_pos0);
  p.n_splits = static_cast<int>(n_splits);
  if (live) {
    p.tiles_per_split = static_cast<int>((max_live + n_splits - 1) / n_splits);
  } else {
    const int64_t hi = decode_hi(q_len, kv_len, bs, q_pos0, kv_pos0);
    const int64_t tiles = hi > 0 ? (hi + bd3::kDecBN - 1) / bd3::kDecBN : 0;
    p.tiles_per_split = static_cast<int>((tiles + n_splits - 1) / n_splits);
    if (p.tiles_per_split < 1) p.tiles_per_split = 1;
  }
  p.live_stride = static_cast<int>(live_stride);
  p.kv_block = static_cast<int>(kv_block);
  p.out_f32 = out_dtype == BD3_F32 ? 1 : 0;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  const dim3 grid(static_cast<unsigned>(n_splits), static_cast<unsigned>(B * H),
                  static_cast<unsigned>(groups));
  using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const bd3::DecParams);
  const bool bf = dtype == BD3_BF16;
  if (cluster) {
    Kern kern;
    if (live) {
      kern = kmb == 1 ? (bf ? bd3::decode_kernel<1, true, true, true> : bd3::decode_kernel<1, false, true, true>)
                      : (bf ? bd3::decode_kernel<2, true, true, true> : bd3::decode_kernel<2, false, true, true>);
    } else {
      kern = kmb == 1 ? (bf ? bd3::decode_kernel<1, true, false, true> : bd3::decode_kernel<1, false, false, true>)
                      : (bf ? bd3::decode_kernel<2, true, false, true> : bd3::decode_kernel<2, false, false, true>);
    }
    const int slot = 24 + (live ? 4 : 0) + (kmb == 1 ? 0 : 2) + (bf ? 0 : 1);
    if ((rc = set_smem(kern, bd3::DecSmem::kAlloc, slot)) != BD3_OK) return rc;
    if (n_splits > 8) {  // 9 to 16 CTAs per cluster: the non-portable sizes B200 allows
      int dev = 0;
      cudaError_t e = cudaGetDevice(&dev);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
      static bool done[64][8] = {};
      const int k = slot - 24;
      if (dev >= 64 || !done[dev][k]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute (cluster size)");
        if (dev < 64) done[dev][k] = true;
      }
    }
    ProfScope ps(kPfDecode, stream);
    return launch_pdl_cluster(kern, grid, dim3(bd3::kDecThreads), bd3::DecSmem::kAlloc,
                              static_cast<unsigned>(n_splits), stream,
                              "decode_kernel (cluster) launch", tq, tk, tv, p);
  }
  Kern kern;
  if (live) {
    kern = kmb == 1 ? (bf ? bd3::decode_kernel<1, true, true> : bd3::decode_kernel<1, false, true>)
                    : (bf ? bd3::decode_kernel<2, true, true> : bd3::decode_kernel<2, false, true>);
  } else {
    kern = kmb == 1 ? (bf ? bd3::decode_kernel<1, true, false> : bd3::decode_kernel<1, false, false>)
                    : (bf ? bd3::decode_kernel<2, true, false> : bd3::decode_kernel<2, false, false>);
  }
  const int slot = 8 + (live ? 4 : 0) + (kmb == 1 ? 0 : 2) + (bf ? 0 : 1);
  if ((rc = set_smem(kern, bd3::DecSmem::kAlloc, slot)) != BD3_OK) return rc;
  {
    ProfScope ps(kPfDecode, stream);
    if ((rc = launch_pdl(kern, grid, dim3(bd3::kDecThreads), bd3::DecSmem::kAlloc, stream,
                         "decode_kernel launch", tq, tk, tv, p)) != BD3_OK)
      return rc;
  }
  if (n_splits > 1) {
    bd3::CombineParams c{};
    c.parts = p.ws_o;
    c.lses = p.ws_lse;
    c.o = o;
    c.lse_out = lse_out;
    c.part_bh = n_splits * q_len * 64;
    c.part_g = q_len * 64;
    c.lse_bh = n_splits * q_len;
    c.lse_g = q_len;
    c.o_sb = so[0];
    c.o_sh = so[1];
    c.o_ss = so[2];
    c.H = static_cast<int>(H);
    c.G = static_cast<int>(n_splits);
    c.rows = static_cast<int>(q_len);
    c.n_bh = static_cast<int>(B * H);
    c.out_dtype = out_dtype;
    const int64_t threads = B * H * q_len * 8;
    ProfScope ps(kPfCombine, stream);
    if ((rc = launch_pdl(bd3::decode_combine_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)),
                         dim3(256), 0, stream, "decode_combine_kernel launch", c)) != BD3_OK)
      return rc;
  }
  return BD3_OK;
}
}  // namespace

int bd3_decode_attn(const void* q, const void* k, const void* v, void* o, float* lse_out,
                    int64_t B, int64_t H, int64_t q_len, int64_t kv_len, int64_t D,
                    const int64_t* strides, int64_t block_size, int64_t q_pos0, int64_t kv_pos0,
                    int64_t n_splits, int dtype, int out_dtype, void* workspace,
                    size_t workspace_bytes, void* stream) {
  int rc = check_dims(B, H, D, dtype);
  if (rc != BD3_OK) return rc;
  if (q_len < 1 || kv_len < 1) return fail(BD3_ERR_INVALID, "q_len and kv_len must be >= 1");
  if (q_len > kv_len && q_pos0 < 0)
    return fail(BD3_ERR_INVALID, "queries are the last q_len key positions: q_len <= kv_len");
  if (block_size < 1) return fail(BD3_ERR_INVALID, "block_size must be >= 1");
  if (kv_len > (1LL << 30) || q_len > (1LL << 30)) return fail(BD3_ERR_UNSUPPORTED, "too long");
  if (out_dtype != dtype && out_dtype != BD3_F32)
    return fail(BD3_ERR_INVALID, "out_dtype must equal dtype or be fp32");
  if (q_pos0 < 0) q_pos0 = kv_len - q_len;
  if (kv_pos0 < 0) return fail(BD3_ERR_INVALID, "kv_pos0 must be >= 0");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (q_len > 64) {
    if (n_splits != 1 || q_pos0 != kv_len - q_len || kv_pos0 != 0 || out_dtype != dtype)
      return fail(BD3_ERR_UNSUPPORTED,
                  "prefill (q_len > 64) supports the reference placement and dtype only");
    if (lse_out != nullptr) return fail(BD3_ERR_UNSUPPORTED, "prefill does not return LSE");
    return launch_fwd(bd3::kDecode, q, k, v, o, nullptr, B, H, 0, q_len, kv_len, strides,
                      block_size, dtype, st);
  }
  return launch_decode(false, q, k, v, o, lse_out, nullptr, nullptr, 0, 0, 64, B, H, q_len,
                       kv_len, strides, block_size, q_pos0, kv_pos0, n_splits, dtype,
                       out_dtype, workspace, workspace_bytes, st);
}

// Decode over a cache whose key count lives on the device. The host plans the split count
// and builds the tensor maps for the capacity; the kernel reads the count, places the
// queries at its end and spreads the key tiles over the splits (decode_kernel), so the
// launch arguments stay the same while the cache grows and one captured CUDA graph replays
// every step of a sampling loop.
int bd3_decode_attn_devlen(const void* q, const void* k, const void* v, void* o,
                           float* lse_out, int64_t B, int64_t H, int64_t q_len,
                           int64_t kv_capacity, int64_t D, const int64_t* strides,
                           int64_t block_size, const int32_t* kv_len_dev, int64_t n_splits,
                           int dtype, int out_dtype, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (kv_len_dev == nullptr) return fail(BD3_ERR_INVALID, "kv_len_dev is required");
  if (q_len < 1 || q_len > 64)
    return fail(BD3_ERR_UNSUPPORTED, "device-length decode handles 1 <= q_len <= 64 (got %lld)",
                (long long)q_len);
  if (kv_capacity < q_len || kv_capacity > (1LL << 30))
    return fail(BD3_ERR_INVALID, "kv_capacity must be in [q_len, 2^30]");
  if (block_size < 1) return fail(BD3_ERR_INVALID, "block_size must be >= 1");
  if (out_dtype != dtype && out_dtype != BD3_F32)
    return fail(BD3_ERR_INVALID, "out_dtype must equal dtype or be fp32");
  const int rc = check_dims(B, H, D, dtype);
  if (rc != BD3_OK) return rc;
  return launch_decode(false, q, k, v, o, lse_out, nullptr, nullptr, 0, 0, 64, B, H, q_len,
                       kv_capacity, strides, block_size, kv_capacity - q_len, 0, n_splits,
                       dtype, out_dtype, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream), kv_len_dev);
}

// ---------------------------------------------------------------------------------------
// Decode without allocation.
//
// Some callers cannot call cudaMalloc: a serving engine that has reserved all of the
// device's memory for its own allocator, or a decode loop that must not take the
// synchronisation a cudaMalloc/cudaFree can imply. For them, bd3_decode_attn_noalloc runs the
// same split-KV decode as bd3_decode_attn, but keeps its split partials in the fixed array
// below instead of a caller-provided workspace. The caller still passes q, k, v and the
// output buffers.
//
// The array is a file-scope __device__ variable: every GPU that loads this library holds its
// kNoAllocScratchBytes until the process exits. In host code its name is only a host-side
// stand-in, not a device address, so the device address is looked up with
// cudaGetSymbolAddress on the first call on each device (with that device current) and kept.
// That first call on a device therefore does a little set-up work; make it before any stream
// capture. All calls share the one array and it keeps the last call's contents: nothing in it
// needs to start at zero (every partial the combine step reads is written earlier in the same
// call), but calls that overlap on the GPU (two streams, two host threads) race on it.
// When the planner's split count needs more than the array, fewer splits are used (each
// covering more key tiles), down to one split, which needs no scratch.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {};

int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(BD3_ERR_UNSUPPORTED, "device index %d too large", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return BD3_OK;
}
}  // namespace

int bd3_decode_attn_noalloc(const void* q, const void* k, const void* v, void* o,
                            float* lse_out, int64_t B, int64_t H, int64_t q_len,
                            int64_t kv_len, int64_t D, const int64_t* strides,
                            int64_t block_size, int64_t q_pos0, int64_t kv_pos0, int dtype,
                            int out_dtype, void* stream) {
  int rc = check_dims(B, H, D, dtype);
  if (rc != BD3_OK) return rc;
  if (q_len < 1 || q_len > 64)
    return fail(BD3_ERR_UNSUPPORTED, "no-alloc decode handles 1 <= q_len <= 64 (got %lld)",
                (long long)q_len);
  int64_t n_splits = 1;
  size_t need = 0;
  if ((rc = bd3_decode_plan(B, H, q_len, kv_len, block_size, q_pos0, kv_pos0, &n_splits,
                            &need)) != BD3_OK)
    return rc;
  if (need > kNoAllocScratchBytes) {
    // fewer splits need less scratch (one split needs none): take as many as the array holds
    const size_t per_split = static_cast<size_t>(B * H * q_len) * (64 + 1) * 4;
    n_splits = static_cast<int64_t>(kNoAllocScratchBytes / per_split);
    if (n_splits < 1) n_splits = 1;
  }
  float* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch)) != BD3_OK) return rc;
  return bd3_decode_attn(q, k, v, o, lse_out, B, H, q_len, kv_len, D, strides, block_size,
                         q_pos0, kv_pos0, n_splits, dtype, out_dtype, scratch,
                         kNoAllocScratchBytes, stream);
}

int bd3_decode_live_plan(int64_t B, int64_t H, int64_t q_len, int64_t max_live,
                         int64_t kv_block, int64_t* n_splits, size_t* workspace_bytes) {
  if (B < 1 || H < 1 || q_len < 1 || q_len > 64 || max_live < 1)
    return fail(BD3_ERR_INVALID, "live decode: sizes must be >= 1 and q_len <= 64");
  if (kv_block < 64 || kv_block % 64) return fail(BD3_ERR_UNSUPPORTED, "kv_block must be a multiple of 64");
  int sms = 148;
  int rc = current_device_sms(&sms);
  if (rc != BD3_OK) return rc;
  const int64_t groups = (q_len + 31) / 32;
  const int64_t per = kv_block / 64;
  // units are live entries; each entry is `per` tiles. Once (batch, head) x row groups give
  // every SM a CTA, one split per (batch, head) is fastest: the lists are short, so extra
  // splits only add CTAs contending for the same scattered blocks plus the combine pass
  // (measured on B=16, H=12, 32 live 64-key blocks: 26.6 us with 1 split, 29.7 with 2).
  int64_t u = B * H * groups >= sms ? max_live
                                    : (pick_units_per_split(B * H * groups, max_live * per, sms) +
                                       per - 1) / per;
  const int64_t s = (max_live + u - 1) / u;
  *n_splits = s;
  *workspace_bytes = s > 1 && !cluster_splits(s, B * H * groups, sms)
                         ? static_cast<size_t>(B * H * s * q_len) * 65 * 4 : 0;
  return BD3_OK;
}

int bd3_decode_live_blocks(const void* q, const void* k, const void* v, void* o,
                           float* lse_out, const int32_t* live_idx, const int32_t* live_cnt,
                           int64_t live_stride, int64_t max_live, int64_t kv_block, int64_t B,
                           int64_t H, int64_t q_len, int64_t kv_len, int64_t D,
                           const int64_t* strides, int64_t block_size, int64_t n_splits,
                           int dtype, int out_dtype, void* workspace, size_t workspace_bytes,
                           void* stream) {
  int rc = check_dims(B, H, D, dtype);
  if (rc != BD3_OK) return rc;
  if (q_len < 1 || q_len > 64 || q_len > kv_len)
    return fail(BD3_ERR_INVALID, "live decode needs 1 <= q_len <= min(64, kv_len)");
  if (kv_block < 64 || kv_block % 64) return fail(BD3_ERR_UNSUPPORTED, "kv_block must be a multiple of 64");
  if (live_idx == nullptr || live_cnt == nullptr || max_live < 1 || live_stride < max_live)
    return fail(BD3_ERR_INVALID, "live block list missing or malformed");
  if (block_size < 1) return fail(BD3_ERR_INVALID, "block_size must be >= 1");
  if (out_dtype != dtype && out_dtype != BD3_F32)
    return fail(BD3_ERR_INVALID, "out_dtype must equal dtype or be fp32");
  return launch_decode(true, q, k, v, o, lse_out, live_idx, live_cnt, live_stride, max_live,
                       kv_block, B, H, q_len, kv_len, strides, block_size, kv_len - q_len, 0,
                       n_splits, dtype, out_dtype, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

size_t bd3_peer_merge_buffer_bytes(int world, int64_t B, int64_t H, int64_t rows) {
  if (world < 2 || world > bd3::kPeerMaxWorld || B < 1 || H < 1 || rows < 1) return 0;
  const int64_t region = (B * H * rows * 65 + 3) / 4 * 4;  // floats, 16-byte multiples
  return static_cast<size_t>(2 * world * region) * 4 +
         static_cast<size_t>(2 * bd3::kPeerMaxWorld * bd3::kPeerMaxCtas) * 8;
}

int bd3_peer_merge(const float* part_o, const float* part_lse, const uint64_t* peer_bufs,
                   int world, int rank, uint64_t epoch, void* o, float* lse_out, int64_t B,
                   int64_t H, int64_t rows, const int64_t* o_strides, int out_dtype,
                   void* stream) {
  if (world < 2 || world > bd3::kPeerMaxWorld || rank < 0 || rank >= world)
    return fail(BD3_ERR_INVALID, "peer merge: 2 <= world <= %d and 0 <= rank < world",
                bd3::kPeerMaxWorld);
  if (B < 1 || H < 1 || rows < 1 || B * H * rows > (int64_t(1) << 30))
    return fail(BD3_ERR_INVALID, "peer merge: sizes must be >= 1");
  if (epoch == 0) return fail(BD3_ERR_INVALID, "peer merge: epochs start at 1");
  if (out_dtype < BD3_BF16 || out_dtype > BD3_F32) return fail(BD3_ERR_INVALID, "bad out_dtype");
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  if (reinterpret_cast<uintptr_t>(part_o) % 16 || reinterpret_cast<uintptr_t>(part_lse) % 4)
    return fail(BD3_ERR_INVALID, "peer merge: the partial O must be 16-byte aligned");
  const int64_t oal = out_dtype == BD3_F32 ? 4 : 8;
  if (reinterpret_cast<uintptr_t>(o) % 16 || o_strides[0] % oal || o_strides[1] % oal ||
      o_strides[2] % oal)
    return fail(BD3_ERR_INVALID, "o: pointer and strides must be 16-byte aligned");
  bd3::PeerMergeParams p{};
  for (int r = 0; r < world; ++r) {
    if (peer_bufs[r] == 0 || peer_bufs[r] % 16)
      return fail(BD3_ERR_INVALID, "peer merge: exchange buffer %d missing or misaligned", r);
    p.bufs[r] = reinterpret_cast<float*>(peer_bufs[r]);
  }
  int sms = 148;
  int rc = current_device_sms(&sms);
  if (rc != BD3_OK) return rc;
  const int64_t units = B * H * rows;
  int64_t ctas = units < sms ? units : sms;  // one CTA per SM at most: every CTA is resident
  if (ctas > bd3::kPeerMaxCtas) ctas = bd3::kPeerMaxCtas;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.o = o;
  p.lse_out = lse_out;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.epoch = epoch;
  p.region = (units * 65 + 3) / 4 * 4;
  p.world = world;
  p.rank = rank;
  p.H = static_cast<int>(H);
  p.units = static_cast<int>(units);
  p.rows = static_cast<int>(rows);
  p.out_dtype = out_dtype;
  ProfScope ps(kPfCombine, static_cast<cudaStream_t>(stream));
  return launch_pdl(bd3::peer_merge_kernel, dim3(static_cast<unsigned>(ctas)),
                    dim3(bd3::kPeerThreads), 0, static_cast<cudaStream_t>(stream),
                    "peer_merge_kernel launch", p);
}

int bd3_lse_merge(const float* parts, const float* lses, void* o, float* lse_out, int64_t B,
                  int64_t H, int64_t G, int64_t rows, int64_t D, const int64_t part_g,
                  int64_t part_bh, int64_t lse_g, int64_t lse_bh, const int64_t* o_strides,
                  int out_dtype, void* stream) {
  if (B < 1 || H < 1 || G < 1 || rows < 1) return fail(BD3_ERR_INVALID, "merge sizes must be >= 1");
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  if (D != 64) return fail(BD3_ERR_UNSUPPORTED, "head_dim must be 64");
  if (out_dtype < BD3_BF16 || out_dtype > BD3_F32) return fail(BD3_ERR_INVALID, "bad out_dtype");
  if (reinterpret_cast<uintptr_t>(parts) % 16 || part_g % 4 || part_bh % 4)
    return fail(BD3_ERR_INVALID, "parts must be 16-byte aligned");
  const int64_t oal = out_dtype == BD3_F32 ? 4 : 8;
  if (reinterpret_cast<uintptr_t>(o) % 16 || o_strides[0] % oal || o_strides[1] % oal ||
      o_strides[2] % oal)
    return fail(BD3_ERR_INVALID, "o: pointer and strides must be 16-byte aligned");
  bd3::CombineParams c{};
  c.parts = parts;
  c.lses = lses;
  c.o = o;
  c.lse_out = lse_out;
  c.part_g = part_g;
  c.part_bh = part_bh;
  c.lse_g = lse_g;
  c.lse_bh = lse_bh;
  c.o_sb = o_strides[0];
  c.o_sh = o_strides[1];
  c.o_ss = o_strides[2];
  c.H = static_cast<int>(H);
  c.G = static_cast<int>(G);
  c.rows = static_cast<int>(rows);
  c.n_bh = static_cast<int>(B * H);
  c.out_dtype = out_dtype;
  const int64_t threads = B * H * rows * 8;
  bd3::decode_combine_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0,
                               static_cast<cudaStream_t>(stream)>>>(c);
  return check_launch("decode_combine_kernel launch");
}

int bd3_f32_to_f16_scaled(const float* q, const float* k, const float* v, const int64_t* strides,
                          int64_t B, int64_t H, int64_t q_rows, int64_t kv_rows, int64_t D,
                          void* q16, void* k16, void* v16, float* exps, uint32_t* workspace,
                          void* stream) {
  if (B < 1 || H < 1 || q_rows < 1 || kv_rows < 1)
    return fail(BD3_ERR_INVALID, "sizes must be >= 1");
  if (D != 64) return fail(BD3_ERR_UNSUPPORTED, "head_dim must be 64 (got %lld)", (long long)D);
  if (q_rows > (1LL << 30) || kv_rows > (1LL << 30) || B * H > (1LL << 24))
    return fail(BD3_ERR_UNSUPPORTED, "too large");
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  const float* src[3] = {q, k, v};
  void* dst[3] = {q16, k16, v16};
  bd3::F32ScaleParams p{};
  for (int t = 0; t < 3; ++t) {
    const int64_t* s3 = strides + 3 * t;
    if (src[t] == nullptr || reinterpret_cast<uintptr_t>(src[t]) % 16 || s3[0] % 4 ||
        s3[1] % 4 || s3[2] % 4)
      return fail(BD3_ERR_INVALID, "fp32 inputs: pointer and strides must be 16-byte aligned");
    if (dst[t] == nullptr || reinterpret_cast<uintptr_t>(dst[t]) % 8)
      return fail(BD3_ERR_INVALID, "fp16 outputs must be 8-byte aligned");
    p.src[t] = src[t];
    p.dst[t] = static_cast<uint16_t*>(dst[t]);
    p.sb[t] = s3[0];
    p.sh[t] = s3[1];
    p.ss[t] = s3[2];
    p.rows[t] = static_cast<int>(t == 0 ? q_rows : kv_rows);
  }
  if (exps == nullptr || workspace == nullptr || reinterpret_cast<uintptr_t>(workspace) % 4)
    return fail(BD3_ERR_WORKSPACE, "exps (3 floats) and workspace (3 uint32) are required");
  p.ws = workspace;
  p.exps = exps;
  p.H = static_cast<int>(H);
  p.bh = static_cast<int>(B * H);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(workspace, 0, 3 * sizeof(uint32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "zeroing the maxima");
  int sms = 148;
  if (const int rc = current_device_sms(&sms); rc != BD3_OK) return rc;
  const int64_t n4 = B * H * (q_rows > kv_rows ? q_rows : kv_rows) * 16;
  int64_t blocks = (n4 + 255) / 256;
  if (blocks > 4LL * sms) blocks = 4LL * sms;
  bd3::f32_absmax_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  if (const int rc = check_launch("f32_absmax_kernel launch"); rc != BD3_OK) return rc;
  bd3::f32_to_f16_scaled_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  return check_launch("f32_to_f16_scaled_kernel launch");
}

int bd3_qkv_rope_cache(const void* qkv, const int64_t* qkv_strides, int64_t B, int64_t S,
                       int64_t H, int64_t D, const int64_t* positions, int64_t pos0,
                       const float* cos_table, const float* sin_table, int64_t max_pos,
                       void* q_out, void* k_cache, void* v_cache, const int64_t* strides,
                       int64_t cache_row0, int64_t cache_rows, int dtype, void* stream) {
  if (dtype < BD3_BF16 || dtype > BD3_F32) return fail(BD3_ERR_INVALID, "bad dtype %d", dtype);
  if (B < 1 || S < 1 || H < 1 || D < 1) return fail(BD3_ERR_INVALID, "sizes must be >= 1");
  if (D % 16 != 0 || D > 1024)
    return fail(BD3_ERR_UNSUPPORTED, "head_dim must be a multiple of 16 up to 1024 (got %lld)",
                (long long)D);
  if (qkv == nullptr || cos_table == nullptr || sin_table == nullptr || k_cache == nullptr ||
      v_cache == nullptr)
    return fail(BD3_ERR_INVALID, "qkv, the RoPE tables and both caches are required");
  if (max_pos < 1) return fail(BD3_ERR_INVALID, "max_pos must be >= 1");
  if (positions == nullptr && (pos0 < 0 || pos0 + S > max_pos))
    return fail(BD3_ERR_INVALID, "positions [%lld, %lld) outside the RoPE table of %lld rows",
                (long long)pos0, (long long)(pos0 + S), (long long)max_pos);
  if (cache_row0 < 0 && positions == nullptr)
    return fail(BD3_ERR_INVALID, "cache_row0 < 0 takes the cache row from positions[0]: "
                "positions is required");
  if (S > cache_rows || (cache_row0 >= 0 && cache_row0 + S > cache_rows))
    return fail(BD3_ERR_INVALID, "cache rows [%lld, %lld) outside a cache of %lld rows",
                (long long)cache_row0, (long long)(cache_row0 + S), (long long)cache_rows);
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  const int64_t eb = static_cast<int64_t>(elem_bytes(dtype));
  auto aligned = [&](const void* ptr, const int64_t* st, int n) {
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return false;
    for (int i = 0; i < n; ++i)
      if ((st[i] * eb) % 16) return false;
    return true;
  };
  if (!aligned(qkv, qkv_strides, 2)) return fail(BD3_ERR_INVALID, "qkv: pointer and strides must be 16-byte aligned");
  if (q_out != nullptr && !aligned(q_out, strides, 3))
    return fail(BD3_ERR_INVALID, "q_out: pointer and strides must be 16-byte aligned");
  if (!aligned(k_cache, strides + 3, 3) || !aligned(v_cache, strides + 6, 3))
    return fail(BD3_ERR_INVALID, "k_cache/v_cache: pointer and strides must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(cos_table) % 16 || reinterpret_cast<uintptr_t>(sin_table) % 16)
    return fail(BD3_ERR_INVALID, "RoPE tables must be 16-byte aligned");
  const int64_t threads = B * S * H * (D / 16);
  if ((threads + 255) / 256 > 2147483647LL) return fail(BD3_ERR_UNSUPPORTED, "too many tokens");
  bd3::RopeCacheParams p{};
  p.qkv = qkv;
  p.qkv_sb = qkv_strides[0];
  p.qkv_ss = qkv_strides[1];
  p.positions = reinterpret_cast<const long long*>(positions);
  p.pos0 = pos0;
  p.cos_table = cos_table;
  p.sin_table = sin_table;
  p.max_pos = max_pos;
  p.q_out = q_out;
  if (q_out != nullptr) {
    p.q_sb = strides[0]; p.q_sh = strides[1]; p.q_ss = strides[2];
  }
  p.k_cache = k_cache;
  p.k_sb = strides[3]; p.k_sh = strides[4]; p.k_ss = strides[5];
  p.v_cache = v_cache;
  p.v_sb = strides[6]; p.v_sh = strides[7]; p.v_ss = strides[8];
  p.row0 = cache_row0;
  p.cache_rows = cache_rows;
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.H = static_cast<int>(H);
  p.D = static_cast<int>(D);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  {
    ProfScope ps(kPfRope, st);
    if (dtype == BD3_BF16) bd3::qkv_rope_cache_kernel<0><<<blocks, 256, 0, st>>>(p);
    else if (dtype == BD3_F16) bd3::qkv_rope_cache_kernel<1><<<blocks, 256, 0, st>>>(p);
    else bd3::qkv_rope_cache_kernel<2><<<blocks, 256, 0, st>>>(p);
  }
  return check_launch("qkv_rope_cache_kernel launch");
}

extern "C++" {  // the launcher is a template
namespace {
int check_sample_args(const void* logits, int64_t B, int64_t S, int64_t V, const int64_t* xt,
                      int64_t mask_index, const int64_t* out, int dtype) {
  if (dtype != BD3_BF16 && dtype != BD3_F32)  // the reference's SUBS cannot hold -1e6 in fp16
    return fail(BD3_ERR_INVALID, "logits must be bf16 or fp32 (got dtype %d)", dtype);
  if (B < 1 || S < 1 || V < 2) return fail(BD3_ERR_INVALID, "need B, S >= 1 and V >= 2");
  if (V > 2147483647LL / 2 || B * S > 2147483647LL)
    return fail(BD3_ERR_UNSUPPORTED, "vocabulary or batch too large");
  if (mask_index < 0 || mask_index >= V)
    return fail(BD3_ERR_INVALID, "mask_index %lld outside the vocabulary of %lld",
                (long long)mask_index, (long long)V);
  if (logits == nullptr || xt == nullptr || out == nullptr)
    return fail(BD3_ERR_INVALID, "logits, xt and out are required");
  return BD3_OK;
}

template <bool kDevArgs>
int launch_sample(const bd3::SampleParams& p, int dtype, cudaStream_t st) {
  const unsigned blocks = static_cast<unsigned>(static_cast<int64_t>(p.B) * p.S);
  {
    ProfScope ps(kPfSample, st);
    // bf16 rows up to 100,000 entries are staged in shared memory (two CTAs per SM)
    constexpr size_t kMaxStage = 200016;
    const size_t stage = static_cast<size_t>(p.V) * 2 + 16;
    if (dtype == BD3_BF16 && stage <= kMaxStage) {
      auto kern = bd3::subs_sample_kernel<0, true, kDevArgs>;
      if (const int rc = set_smem(kern, static_cast<uint32_t>(kMaxStage), kDevArgs ? 17 : 16);
          rc != BD3_OK)
        return rc;
      kern<<<blocks, bd3::kSampleThreads, stage, st>>>(p);
    } else if (dtype == BD3_BF16) {
      bd3::subs_sample_kernel<0, false, kDevArgs><<<blocks, bd3::kSampleThreads, 0, st>>>(p);
    } else {
      bd3::subs_sample_kernel<2, false, kDevArgs><<<blocks, bd3::kSampleThreads, 0, st>>>(p);
    }
  }
  return check_launch("subs_sample_kernel launch");
}
}  // namespace
}  // extern "C++"

int bd3_subs_sample(const void* logits, const int64_t* logit_strides, int64_t B, int64_t S,
                    int64_t V, const int64_t* xt, int64_t mask_index, double t, double s,
                    uint64_t seed, uint64_t offset, const double* uniforms, int64_t* out,
                    int dtype, void* stream) {
  if (const int rc = check_sample_args(logits, B, S, V, xt, mask_index, out, dtype);
      rc != BD3_OK)
    return rc;
  if (!(t > 0.0)) return fail(BD3_ERR_INVALID, "t must be > 0 (the step divides by it)");
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  bd3::SampleParams p{};
  p.logits = logits;
  p.l_sb = logit_strides[0];
  p.l_ss = logit_strides[1];
  p.xt = reinterpret_cast<const long long*>(xt);
  p.out = reinterpret_cast<long long*>(out);
  p.u = uniforms;
  p.seed = seed;
  p.offset = offset;
  p.keep = 1.0 - s / t;  // the reference's Python floats: (1 - s / t) and s / t
  p.stay = s / t;
  p.mask_index = mask_index;
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.V = static_cast<int>(V);
  return launch_sample<false>(p, dtype, static_cast<cudaStream_t>(stream));
}

// The same step with (t, s) and (seed, offset) in device memory (the Philox draw only), so
// that a sampling loop captured in a CUDA graph advances them on the device between replays.
int bd3_subs_sample_dev(const void* logits, const int64_t* logit_strides, int64_t B,
                        int64_t S, int64_t V, const int64_t* xt, int64_t mask_index,
                        const double* ts, const uint64_t* seed_offset, int64_t* out, int dtype,
                        void* stream) {
  if (const int rc = check_sample_args(logits, B, S, V, xt, mask_index, out, dtype);
      rc != BD3_OK)
    return rc;
  if (ts == nullptr || seed_offset == nullptr)
    return fail(BD3_ERR_INVALID, "ts (t, s) and seed_offset (seed, offset) are required");
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  bd3::SampleParams p{};
  p.logits = logits;
  p.l_sb = logit_strides[0];
  p.l_ss = logit_strides[1];
  p.xt = reinterpret_cast<const long long*>(xt);
  p.out = reinterpret_cast<long long*>(out);
  p.ts_dev = ts;
  p.rng_dev = reinterpret_cast<const unsigned long long*>(seed_offset);
  p.mask_index = mask_index;
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.V = static_cast<int>(V);
  return launch_sample<true>(p, dtype, static_cast<cudaStream_t>(stream));
}

int bd3_profile_enable(int on) {
  Prof& p = prof();
  if (on && !p.created) {
    for (int i = 0; i < kProfCap; ++i)
      for (int j = 0; j < 2; ++j) {
        const cudaError_t e = cudaEventCreate(&p.ev[i][j]);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
      }
    p.created = true;
  }
  p.on = on != 0;
  p.n = 0;
  return BD3_OK;
}

int bd3_profile_collect(double* total_ms, int32_t* counts) {
  Prof& p = prof();
  for (int k = 0; k < kPfNum; ++k) {
    total_ms[k] = 0.0;
    counts[k] = 0;
  }
  for (int i = 0; i < p.n; ++i) {
    cudaError_t e = cudaEventSynchronize(p.ev[i][1]);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize");
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, p.ev[i][0], p.ev[i][1]);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime");
    total_ms[p.id[i]] += ms;
    counts[p.id[i]] += 1;
  }
  p.n = 0;
  return kPfNum;
}

int bd3_debug_ranges(int kind, int64_t start, int64_t tile_a, int64_t tile_b, int64_t n_or_qlen,
                     int64_t kv_len, int64_t block_size, int32_t* out) {
  bd3::Range r[4];
  int cnt = 0;
  const int s = static_cast<int>(start), a = static_cast<int>(tile_a),
            b = static_cast<int>(tile_b), nq = static_cast<int>(n_or_qlen),
            kv = static_cast<int>(kv_len), bs = static_cast<int>(block_size);
  if (kind == 0) cnt = bd3::fwd_ranges(s, a, b, nq, bs, r);
  else if (kind == 1) cnt = bd3::dkdv_ranges(s, a, b, nq, bs, r);
  else if (kind == 2) cnt = bd3::decode_ranges(s, a, b, nq, kv, bs, r);
  else return fail(BD3_ERR_INVALID, "unknown range kind %d", kind);
  for (int i = 0; i < cnt; ++i) {
    out[4 * i + 0] = r[i].lo;
    out[4 * i + 1] = r[i].hi;
    out[4 * i + 2] = r[i].rule;
    out[4 * i + 3] = r[i].shift;
  }
  return cnt;
}

int bd3_debug_wait_timeout(int64_t limit_ns, int arrive, uint64_t* out, void* stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000)
    return fail(BD3_ERR_INVALID, "limit_ns must be in [1e3, 1e9] (got %lld)", (long long)limit_ns);
  if (out == nullptr || reinterpret_cast<uintptr_t>(out) % 8)
    return fail(BD3_ERR_INVALID, "out must be an 8-byte aligned device buffer of 2 uint64");
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  bd3::wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(limit_ns), arrive, reinterpret_cast<unsigned long long*>(out));
  return check_launch("wait_probe_kernel launch");
}

int bd3_debug_wait_site(uint32_t* out) {
  if (out == nullptr) return fail(BD3_ERR_INVALID, "out must hold 4 uint32");
  if (const int rc = ensure_context(); rc != BD3_OK) return rc;
  cudaError_t e = cudaMemcpyFromSymbol(out, bd3::g_bd3_wait_site, 4 * sizeof(uint32_t));
  if (e != cudaSuccess) return cuda_fail(e, "reading the wait site");
  const uint32_t zero[4] = {0, 0, 0, 0};
  e = cudaMemcpyToSymbol(bd3::g_bd3_wait_site, zero, sizeof(zero));
  return e == cudaSuccess ? BD3_OK : cuda_fail(e, "clearing the wait site");
}

int bd3_debug_tiles(int32_t* out) {
  out[0] = bd3::kFwdBM;
  out[1] = bd3::kFwdBN;
  out[2] = bd3::kBwdBKV;
  out[3] = bd3::kBwdBQ;
  out[4] = bd3::kDecBN;
  out[5] = bd3::kBwdBQ;
  return 6;
}

}  // extern "C"
