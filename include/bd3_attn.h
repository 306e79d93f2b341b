/* C ABI of the B200 BD3-LM attention library (libbd3attn.so).
 *
 * Plain pointers, sizes and strides; no framework types. Every entry point returns an int
 * status (BD3_OK or one of the BD3_ERR_* codes) and leaves a message for bd3_last_error().
 * Kernels are enqueued on `stream` (a cudaStream_t; NULL is the legacy default stream) and
 * nothing synchronises: outputs are ready when the stream reaches that point.
 *
 * Tensors are 4-D (batch, heads, seq, head_dim) with head_dim contiguous. Each tensor
 * argument is described by a pointer plus three element strides (batch, head, seq), passed
 * in the `strides` array in argument order. Pointers and strides must be 16-byte aligned
 * (the kernels read rows with TMA). head_dim must be 64.
 *
 * dtype codes: BD3_BF16, BD3_F16 (inputs); BD3_F32 is accepted as an output dtype of the
 * decode entry points and of bd3_lse_merge.
 */
#ifndef BD3_ATTN_H_
#define BD3_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BD3_API __attribute__((visibility("default")))
#else
#define BD3_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  BD3_OK = 0,
  BD3_ERR_INVALID = 1,     /* the reference would raise AssertionError on these arguments */
  BD3_ERR_UNSUPPORTED = 2, /* valid for the reference, not supported here (e.g. head_dim) */
  BD3_ERR_CUDA = 3,        /* a CUDA runtime or driver call failed */
  BD3_ERR_WORKSPACE = 4    /* workspace missing or smaller than the plan asks for */
};
enum { BD3_BF16 = 0, BD3_F16 = 1, BD3_F32 = 2 };

/* Library version (major * 10000 + minor * 100 + patch). */
BD3_API int bd3_version(void);
/* Message of the last failed call on this host thread ("" if none). */
BD3_API const char* bd3_last_error(void);
/* Sticky device-side status bits of the current device (1: a bounded wait inside a kernel
 * ran out; 2: a kernel rejected its launch parameters; 4: a RoPE position was outside the
 * table; 8: a dQ partial left the deterministic backward's fixed-point range). Synchronises
 * the device. Clears the
 * bits when `clear` is non-zero. Returns a negative value if the CUDA call itself failed. */
BD3_API int bd3_device_status(int clear);

/* ---------------------------------------------------------------------------------------
 * Training attention forward under the BD3-LM block-diffusion mask.
 * Replaces BlockSparseFlashAttention.forward (kernels/BlockSparseFlashAttention.py:466-506)
 * and its kernel block_sparse_attention_fwd_kern (:76-172).
 *   q, k, v, o: (B, H, 2n, 64); strides[12] = q, k, v, o (batch, head, seq) in elements.
 *   lse:        (B, H, 2n) fp32, contiguous; per-row natural-log log-sum-exp (m + ln l).
 * Requires n % 128 == 0 (the reference asserts n % BLOCK_M == 0 with BLOCK_M = 128).
 */
BD3_API int bd3_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                 int64_t H, int64_t n, int64_t D, const int64_t* strides, int64_t block_size,
                 int dtype, void* stream);

/* Training attention backward: dQ, dK, dV from q, k, v, o, lse and dO.
 * Replaces BlockSparseFlashAttention.backward (kernels/BlockSparseFlashAttention.py:509-562),
 * i.e. the host Delta = rowsum(dO * O) (:525) and the kernels
 * block_sparse_attention_bwd_dq_kern (:369-452) and block_sparse_attention_dk_dv_bwd_kern
 * (:213-328), fused into one kernel per key tile. dK and dV are deterministic (one CTA owns
 * each key tile and writes it once); dQ is summed in fp32 with atomic adds, so its last bits
 * may vary from run to run.
 *   strides[24] = q, k, v, o, do, dq, dk, dv (batch, head, seq) in elements.
 *   lse: 16-byte aligned. workspace: bd3_attn_bwd_workspace_size() bytes of device memory
 *   (Delta, LSE*log2(e) and the fp32 dQ accumulator: 264 bytes per query row).
 * Requires n % 128 == 0 and n % block_size == 0 (the reference asserts both, :522, :548).
 */
BD3_API size_t bd3_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t n, int64_t D);
BD3_API int bd3_attn_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
                 const void* dout, void* dq, void* dk, void* dv, int64_t B, int64_t H,
                 int64_t n, int64_t D, const int64_t* strides, int64_t block_size, int dtype,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Deterministic training attention backward: bd3_attn_bwd with dQ the same on every run, as
 * the reference's dQ kernel (kernels/BlockSparseFlashAttention.py:369-452, a loop over key
 * tiles in order) gives it. Each key tile's dQ partial is rounded to an int64 in units of
 * 2^-32 and the partials are added as integers, so their order does not matter. A partial of
 * magnitude 2^20 or more (or NaN) sets device status bit 8 (its sum would leave the 63-bit
 * range). Arguments as bd3_attn_bwd; workspace: bd3_attn_bwd_det_workspace_size() bytes
 * (520 per query row). The Python binding takes this path when
 * torch.are_deterministic_algorithms_enabled(). */
BD3_API size_t bd3_attn_bwd_det_workspace_size(int64_t B, int64_t H, int64_t n, int64_t D);
BD3_API int bd3_attn_bwd_det(const void* q, const void* k, const void* v, const void* o,
                             const float* lse, const void* dout, void* dq, void* dk, void* dv,
                             int64_t B, int64_t H, int64_t n, int64_t D, const int64_t* strides,
                             int64_t block_size, int dtype, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Decode attention: the q_len queries attend kv_len keys under the block-causal rule
 * (query row r sits at global position q_pos0 + r, key c at kv_pos0 + c; the row sees the key
 * iff (q_pos0 + r) / bs >= (kv_pos0 + c) / bs). Pass q_pos0 = -1 for the reference's
 * placement (the queries are the last q_len of the kv_len positions) and kv_pos0 = 0.
 * Replaces split_kv_decode_attention (kernels/SplitKVDecodeAttention.py:130-171) and
 * block_sparse_decode_attention (kernels/BlockSparseDecodeAttention.py:118-148):
 * q_len <= 64 runs the split-KV kernel plus (when n_splits > 1) the LSE combine; longer
 * query blocks (prefill) run the tcgen05 block-causal kernel and need n_splits == 1. When 2 to
 * 16 splits of a grid that fits on the GPU at once are asked for, the splits of each
 * (batch*head, row group) run as one thread-block cluster and merge through distributed
 * shared memory inside the kernel (no combine launch, no workspace: the plan then reports 0
 * bytes).
 *   q: (B, H, q_len, 64); k, v: (B, H, kv_len, 64); o: (B, H, q_len, 64) in out_dtype.
 *   strides[12] = q, k, v, o (batch, head, seq) in elements.
 *   lse_out: optional (B*H, q_len) fp32 natural-log LSE of each row (NULL to skip).
 * bd3_decode_plan() picks n_splits (pass the result back) and the workspace size.
 * The split-KV kernel and the combine are launched with programmatic stream serialization:
 * they may start while the previous kernel on the stream finishes but wait for it before
 * reading or writing any memory, so stream order is as for any launch.
 */
BD3_API int bd3_decode_plan(int64_t B, int64_t H, int64_t q_len, int64_t kv_len, int64_t block_size,
                    int64_t q_pos0, int64_t kv_pos0, int64_t* n_splits, size_t* workspace_bytes);
BD3_API int bd3_decode_attn(const void* q, const void* k, const void* v, void* o, float* lse_out,
                    int64_t B, int64_t H, int64_t q_len, int64_t kv_len, int64_t D,
                    const int64_t* strides, int64_t block_size, int64_t q_pos0, int64_t kv_pos0,
                    int64_t n_splits, int dtype, int out_dtype, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Decode over a KV cache whose key count is a device int32 (*kv_len_dev), so the launch
 * arguments do not change as the cache grows and one captured CUDA graph replays every
 * denoising step. The same attention as bd3_decode_attn with the reference's placement (the
 * queries are the last q_len of the *kv_len_dev keys, kv_pos0 = 0); the reference's
 * kernels/SplitKVDecodeAttention.py:130-171 reads the count from k.shape instead.
 *   k, v: (B, H, kv_capacity, 64) cache storage (rows past the count are never read).
 *   n_splits, workspace: from bd3_decode_plan(B, H, q_len, kv_capacity, block_size, -1, 0).
 * A count outside [q_len, kv_capacity] is clamped into it and sets device status bit 2.
 * q_len <= 64; the other arguments are those of bd3_decode_attn. */
BD3_API int bd3_decode_attn_devlen(const void* q, const void* k, const void* v, void* o,
                                   float* lse_out, int64_t B, int64_t H, int64_t q_len,
                                   int64_t kv_capacity, int64_t D, const int64_t* strides,
                                   int64_t block_size, const int32_t* kv_len_dev,
                                   int64_t n_splits, int dtype, int out_dtype, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Decode without allocation: the same result as bd3_decode_attn (split count from
 * bd3_decode_plan) for callers that cannot call cudaMalloc, such as a serving engine whose
 * allocator owns all device memory, or a decode loop that must not take the synchronisation
 * an allocation can imply. No counterpart in the reference. The split partials live in a
 * fixed 32 MiB array inside the library (held on every GPU that loads it until exit) instead
 * of a workspace; where the planner's split count needs more, fewer splits are used (down to
 * one, which needs none), so every size runs, a little slower than with a workspace.
 * The first call on a device looks the array's address up (set-up work; make it before any
 * stream capture). Calls share the array, so calls that overlap on the GPU race.
 * q_len <= 64; the other arguments are those of bd3_decode_attn. */
BD3_API int bd3_decode_attn_noalloc(const void* q, const void* k, const void* v, void* o,
                                    float* lse_out, int64_t B, int64_t H, int64_t q_len,
                                    int64_t kv_len, int64_t D, const int64_t* strides,
                                    int64_t block_size, int64_t q_pos0, int64_t kv_pos0,
                                    int dtype, int out_dtype, void* stream);

/* Block-sparse decode over a per-(batch, head) list of live KV blocks of kv_block tokens
 * (a multiple of 64). No counterpart kernel in the reference, whose oracle for it is
 * model/modules.py:738 given the expanded (B, H, q_len, kv_len) mask; the block-causal rule
 * above still applies inside the live blocks.
 *   live_idx: (B*H, live_stride) int32 block indices, ascending; live_cnt: (B*H) int32.
 *   q_len <= 64. bd3_decode_live_plan() gives n_splits and the workspace size.
 */
BD3_API int bd3_decode_live_plan(int64_t B, int64_t H, int64_t q_len, int64_t max_live,
                         int64_t kv_block, int64_t* n_splits, size_t* workspace_bytes);
BD3_API int bd3_decode_live_blocks(const void* q, const void* k, const void* v, void* o,
                           float* lse_out, const int32_t* live_idx, const int32_t* live_cnt,
                           int64_t live_stride, int64_t max_live, int64_t kv_block, int64_t B,
                           int64_t H, int64_t q_len, int64_t kv_len, int64_t D,
                           const int64_t* strides, int64_t block_size, int64_t n_splits,
                           int dtype, int out_dtype, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Exchange and merge of sequence-sharded decode in one kernel over NVLink peer memory: each
 * rank stores its partial (O normalised over its keys, fp32; natural-log LSE) straight into
 * every peer's exchange buffer, raises a flag there, waits (at most 1 s, then device status
 * bit 16) for the peers' flags on its own buffer and merges the partials in rank order with
 * the weighting of kernels/SplitKVDecodeAttention.py:109-119 (bd3_lse_merge's). It replaces
 * the NCCL all-gather + bd3_lse_merge pair; the reference itself is single-GPU. Plain stores
 * to peers and loads of the local buffer only (no TMA, no multicast).
 *   part_o: (B*H*rows, 64) fp32, part_lse: (B*H*rows) fp32, this rank's partial.
 *   peer_bufs: host array of `world` device pointers, every rank's exchange buffer as mapped
 *   in this process (symmetric memory), bd3_peer_merge_buffer_bytes() bytes each, zeroed
 *   once before the first call.
 *   epoch: 1, 2, 3, ... advanced by one per call, the same on every rank.
 *   o: (B, H, rows, 64) in out_dtype with o_strides[3]; lse_out optional (B*H, rows) fp32.
 * Every rank must call it with the same sizes and epoch; a rank may be one call ahead of a
 * peer, not two. */
BD3_API size_t bd3_peer_merge_buffer_bytes(int world, int64_t B, int64_t H, int64_t rows);
BD3_API int bd3_peer_merge(const float* part_o, const float* part_lse, const uint64_t* peer_bufs,
                           int world, int rank, uint64_t epoch, void* o, float* lse_out,
                           int64_t B, int64_t H, int64_t rows, const int64_t* o_strides,
                           int out_dtype, void* stream);

/* LSE-weighted merge of G partial results over disjoint key sets (the math of
 * split_kv_reduce_kern, kernels/SplitKVDecodeAttention.py:91-127; here also the merge of
 * per-GPU partials after an all-gather for sequence-sharded decode).
 *   parts: fp32, element (g, bh, r, d) at g*part_g + bh*part_bh + r*64 + d.
 *   lses:  fp32, element (g, bh, r) at g*lse_g + bh*lse_bh + r.
 *   o: (B, H, rows, 64) in out_dtype with o_strides[3]; lse_out optional (B*H, rows) fp32.
 */
BD3_API int bd3_lse_merge(const float* parts, const float* lses, void* o, float* lse_out, int64_t B,
                  int64_t H, int64_t G, int64_t rows, int64_t D, int64_t part_g,
                  int64_t part_bh, int64_t lse_g, int64_t lse_bh, const int64_t* o_strides,
                  int out_dtype, void* stream);

/* Fused QKV split + rotary embedding + in-place KV-cache write for one attention layer.
 * Replaces model/modules.py:395-417 (the rearrange of the fused projection, self.rope on q
 * and k, and the torch.cat of the cached and the new K/V) and KVCache.append
 * (model/kv_cache.py:42-55): k and v go straight into rows [cache_row0, cache_row0 + S) of
 * preallocated cache tensors, so no step or commit copies the cache. RoPE is the reference's
 * rotate-half form with its own tables; results are bit-identical to the reference's ops.
 *   qkv: (B, S, 3*H*D) projection output whose last dim is ordered (three, heads, head_dim)
 *        and contiguous; qkv_strides[2] = (batch, seq) in elements.
 *   positions: device int64 (S,) absolute positions, or NULL for pos0 + s.
 *   cos_table, sin_table: device fp32 (max_pos, D/2) row-major (RoPE.cos_table/sin_table).
 *   q_out: (B, H, S, D) rotated queries, or NULL. k_cache, v_cache: (B, H, cache_rows, D).
 *   strides[9] = q_out, k_cache, v_cache (batch, head, seq) in elements.
 * dtype: BD3_BF16, BD3_F16 or BD3_F32 (all tensors but the tables). head_dim % 16 == 0;
 * pointers and strides 16-byte aligned. A device position outside [0, max_pos) (the
 * reference raises IndexError) leaves its token unwritten and sets device status bit 4.
 * cache_row0 < 0 takes the first cache row from the device value positions[0] (positions
 * required), so a CUDA graph captured once writes each new block at its own rows; a row
 * range outside [0, cache_rows) then writes nothing and sets status bit 4. */
/* fp32 q, k, v onto the fp16 kernels at tf32's precision (the reference's Triton dots round
 * fp32 operands to tf32, kernels/BlockSparseFlashAttention.py:45-70; it has no separate entry).
 * q is (B, H, q_rows, 64), k and v (B, H, kv_rows, 64), fp32 with the last dim contiguous and
 * element strides strides[0..2] (q), [3..5] (k), [6..8] (v); q16, k16, v16 are contiguous fp16
 * outputs of the same shapes. With e_x = floor(log2(max |x|)) (at least -100),
 * a = floor((e_q - e_k) / 2) and c = e_v - 4, writes q * 2^-a and k * 2^a (saturated at
 * +-65504; the scores q . k are unchanged) and v * 2^-c, rounded to nearest, and
 * exps = {a, c, 2^c} (fp32, device). O computed from the fp16 operands is O / 2^c.
 * workspace: 3 uint32 of device memory, zeroed by this call. Enqueued on `stream`. */
BD3_API int bd3_f32_to_f16_scaled(const float* q, const float* k, const float* v,
                                  const int64_t* strides, int64_t B, int64_t H, int64_t q_rows,
                                  int64_t kv_rows, int64_t D, void* q16, void* k16, void* v16,
                                  float* exps, uint32_t* workspace, void* stream);

BD3_API int bd3_qkv_rope_cache(const void* qkv, const int64_t* qkv_strides, int64_t B, int64_t S,
                               int64_t H, int64_t D, const int64_t* positions, int64_t pos0,
                               const float* cos_table, const float* sin_table, int64_t max_pos,
                               void* q_out, void* k_cache, void* v_cache, const int64_t* strides,
                               int64_t cache_row0, int64_t cache_rows, int dtype, void* stream);

/* One ancestral step of the BD3-LM block sampler: SUBS log-probabilities, the update weights
 * and the float64 Gumbel-max draw, fused. Replaces subs_parameterization (model/subs.py:11-43),
 * the step's q = exp(log_probs).double() * (1 - s/t), q[..., mask_index] = s/t,
 * sample_categorical (sample/sampler.py:11-34) and torch.where(block != mask_index, block,
 * new) (sample/sampler.py:114-122).
 *   logits: (B, S, V) in dtype (BD3_BF16 or BD3_F32; with fp16 logits the reference's SUBS
 *           raises, -1e6 overflowing fp16), vocab contiguous;
 *           logit_strides[2] = (batch, seq) in elements. The SUBS log-softmax rounds every
 *           op to that dtype, as the reference's tensors of that dtype do.
 *   xt: device int64 (B, S) tokens; out: device int64 (B, S) next tokens (may alias xt).
 *   t, s: the step's times (t > 0). Tokens that are not mask_index are kept.
 *   uniforms: NULL for the production draw, an exact draw from q / sum(q) by inverse CDF
 *   with one Philox4x32-10 uniform per row (key = seed, counter = (row, offset low 32 bits,
 *   offset high 32 bits, 0x5A3)), or a device float64 (B, S, V) contiguous tensor of
 *   uniforms in [0, 1) to replay the reference's Gumbel-max on a given draw (its
 *   torch.rand_like). */
BD3_API int bd3_subs_sample(const void* logits, const int64_t* logit_strides, int64_t B,
                            int64_t S, int64_t V, const int64_t* xt, int64_t mask_index,
                            double t, double s, uint64_t seed, uint64_t offset,
                            const double* uniforms, int64_t* out, int dtype, void* stream);

/* bd3_subs_sample's production draw with its per-step values in device memory:
 * ts = device float64 (t, s), seed_offset = device uint64 (seed, offset). The launch then
 * does not change from step to step, so a sampling loop captured once in a CUDA graph
 * draws every step afresh once the caller advances them on the device. Same tokens as
 * bd3_subs_sample with those values as host arguments (same sampler.py:100-122 step).
 * A device t <= 0 keeps every token and sets device status bit 2. */
BD3_API int bd3_subs_sample_dev(const void* logits, const int64_t* logit_strides, int64_t B,
                                int64_t S, int64_t V, const int64_t* xt, int64_t mask_index,
                                const double* ts, const uint64_t* seed_offset, int64_t* out,
                                int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * Per-kernel timing for benchmarks. While enabled, every launch is bracketed by a pair of
 * CUDA events on its own stream (at most 8192 launches are kept). bd3_profile_collect()
 * waits for them and writes, per kernel id (0 training forward, 1 prefill forward, 2 backward
 * prep, 3 dQ convert, 4 fused backward, 5 decode, 6 decode combine, 7 QKV RoPE cache write,
 * 8 sampler step), the summed milliseconds
 * and launch counts to
 * total_ms[9] and counts[9]; it returns 9 and forgets the recorded launches.
 */
BD3_API int bd3_profile_enable(int on);
BD3_API int bd3_profile_collect(double* total_ms, int32_t* counts);

/* ---------------------------------------------------------------------------------------
 * Host-only introspection for tests (no GPU needed).
 * bd3_debug_ranges: kind 0 forward/dQ key ranges, 1 dK/dV query ranges, 2 decode key ranges;
 * writes (lo, hi, rule, shift) quadruples to out[16]; returns how many.
 * bd3_debug_tiles: the library's tile sizes: out[0..5] = forward BM, BN; dK/dV BKV, BQ;
 * decode BN; backward query step.
 */
BD3_API int bd3_debug_ranges(int kind, int64_t start, int64_t tile_a, int64_t tile_b, int64_t n_or_qlen,
                     int64_t kv_len, int64_t block_size, int32_t* out);
BD3_API int bd3_debug_tiles(int32_t* out);

/* Self-check of the kernels' bounded waits (tests; no counterpart in the reference, which
 * has no device-side failure handling). One thread initialises an mbarrier expecting one
 * arrival, arrives on it only when `arrive` is non-zero, and waits for it with the limit
 * `limit_ns` (1e3 .. 1e9, else BD3_ERR_INVALID) through the same wait every kernel uses.
 * Without the arrival the wait must give up after limit_ns: the kernel sets status bit 1
 * (read and cleared by bd3_device_status) and exits normally, leaving the context usable.
 * out: a device buffer of 2 uint64, written with (1 if the wait gave up else 0, the wait's
 * duration in ns). Enqueued on `stream`.
 */
BD3_API int bd3_debug_wait_timeout(int64_t limit_ns, int arrive, uint64_t* out, void* stream);

/* Where the first bounded wait that ran out since the last call gave up (no counterpart in
 * the reference): out[0] 1 if one did (else all 0), out[1] its block, out[2] its thread,
 * out[3] the barrier's shared-memory address with the awaited parity in bit 31. Reading
 * clears it. Synchronous. */
BD3_API int bd3_debug_wait_site(uint32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* BD3_ATTN_H_ */
