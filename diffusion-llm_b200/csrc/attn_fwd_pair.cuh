// BD3-LM training attention forward, one CTA per SM over (batch*head, tile pair) items.
//
// Replaces block_sparse_attention_fwd_kern (kernels/BlockSparseFlashAttention.py:76-172) for
// the training layout [x_t | x_0]. An item is the pair of 128-row query tiles i of the two
// copies: the noisy rows [128i, 128i+128) and the clean rows [n+128i, n+128i+128). Both read
// the same clean keys [n, n+128i) unmasked and the same clean diagonal tile under rule 2
// (noisy with shift 1, clean with shift 0); only the noisy tile reads its own noisy keys under
// rule 1. So each K/V tile streamed into shared memory feeds both tiles' MMAs: one K/V load
// per key tile of the pair instead of one per key tile of each query tile. The key ranges of
// each tile are the reference's formulas (fwd_ranges), so the visited tiles are the same.
//
// Roles (320 threads):
//   warps 0-3  softmax of the noisy tile: thread t owns query row t (TMEM lane t), all 128
//              key columns of every S tile; epilogue of the noisy tile (O via TMA, LSE)
//   warps 4-7  the same for the clean tile
//   warp 8     TMA producer: each item's two Q tiles, then the K/V tiles of its steps
//   warp 9     TMEM owner and UMMA issuer (one thread)
// TMEM columns, per query tile x (0 noisy, 1 clean): S_x [128x, 128x+128), P_x (16-bit
// pairs) [256+64x, 256+64x+64), O_x [384+64x, 384+64x+64). P has its own columns, so a
// warpgroup releases S_x as soon as it has loaded the tile into registers, and the issuer
// computes the next S_x while the warpgroup still works on the exponentials: a warpgroup
// finds its next S tile computed when it finishes one, and the two warpgroups wait on
// nothing of each other's. Per step the issuer issues the step's S tiles, then the previous
// step's P V products. Within a diagonal tile, 32-column chunks no row of a warp can see
// skip their exponentials and write P = 0.
#pragma once

#include "attn_fwd.cuh"

namespace bd3 {

constexpr int kPairStages = 4;
constexpr int kPairThreads = 320;
// column pairs (of 64 per row and S tile) whose exponentials run on the FMA pipe (0, 10,
// 20 and 32 measured within 2% of each other; the softmax is latency-bound, not MUFU-bound)
constexpr int kPairPoly = 20;

struct PairSmem {
  static constexpr uint32_t kQ = 0;                                // [item parity][noisy, clean]
  static constexpr uint32_t kK = kQ + 4 * kTile16;
  static constexpr uint32_t kV = kK + kPairStages * kTile16;
  static constexpr uint32_t kOut = kV + kPairStages * kTile16;    // [noisy, clean] O staging
  static constexpr uint32_t kBar = kOut + 2 * kTile16;
  // q_full[2], q_empty[2], k_full[S], v_full[S], kv_empty[S], and per query tile s_full,
  // s_free, p_full, o_done, o_free
  static constexpr uint32_t kNumBars = 4 + 3 * kPairStages + 10;
  static constexpr uint32_t kTmemSlot = kBar + kNumBars * 8;
  static constexpr uint32_t kBytes = kTmemSlot + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;  // room to align the base to 1 KB
};

// Key steps of one item: part A, the noisy tile's rule-1 keys [a_lo, a_hi) (keys < n, noisy
// only); part B, the clean keys [n, max(n_hi, c_hi)) in 128-key steps, each needed by the
// noisy tile below n_hi (rule 0 below n_full, else rule 2 with shift 1) and by the clean
// tile below c_hi (rule 0 below c_full, else rule 2 with shift 0).
struct PairPlan {
  int a_lo, a_hi, n_full, n_hi, c_full, c_hi, na, nb;
};

__device__ __forceinline__ PairPlan pair_plan(int i, int n, int bs) {
  Range n1, n0, n2, c0, c2;
  fwd_ranges_noisy(i * kFwdBM, kFwdBM, kFwdBN, n, bs, n1, n0, n2);
  fwd_ranges_clean(n + i * kFwdBM, kFwdBM, kFwdBN, n, bs, c0, c2);
  PairPlan pl;
  pl.a_lo = n1.lo;
  pl.a_hi = n1.hi;
  pl.n_full = n0.hi;
  pl.n_hi = imax(n2.hi, n0.hi);
  pl.c_full = c0.hi;
  pl.c_hi = imax(c2.hi, c0.hi);
  pl.na = pl.a_hi > pl.a_lo ? cdiv(pl.a_hi - pl.a_lo, kFwdBN) : 0;
  const int hb = imax(pl.n_hi, pl.c_hi);
  pl.nb = hb > n ? cdiv(hb - n, kFwdBN) : 0;
  return pl;
}

struct PairStep {
  int s;            // first key of the step's tile
  bool need[2];     // noisy, clean
  int rule[2];
};

__device__ __forceinline__ PairStep pair_step(const PairPlan& pl, int j, int n) {
  PairStep st;
  if (j < pl.na) {
    st.s = pl.a_lo + j * kFwdBN;
    st.need[0] = true;
    st.need[1] = false;
    st.rule[0] = 1;
    st.rule[1] = 0;
  } else {
    st.s = n + (j - pl.na) * kFwdBN;
    st.need[0] = st.s < pl.n_hi;
    st.rule[0] = st.s < pl.n_full ? 0 : 2;
    st.need[1] = st.s < pl.c_hi;
    st.rule[1] = st.s < pl.c_full ? 0 : 2;
  }
  return st;
}

// Item w of the persistent loop: (batch*head, tile pair), pairs with more keys first.
__device__ __forceinline__ void pair_item(int w, int num_bh, int num_pairs, int* bh, int* i) {
  *bh = w % num_bh;
  *i = num_pairs - 1 - w / num_bh;
}

// Max over the 32 registers x[32c .. 32c+31] as a tree of three-input maxes.
template <int c>
__device__ __forceinline__ float max32_chunk(const float (&x)[128]) {
  float m1[11], m2[4];
#pragma unroll
  for (int i = 0; i < 10; ++i) m1[i] = max3(x[32 * c + 3 * i], x[32 * c + 3 * i + 1], x[32 * c + 3 * i + 2]);
  m1[10] = fmaxf(x[32 * c + 30], x[32 * c + 31]);
#pragma unroll
  for (int i = 0; i < 3; ++i) m2[i] = max3(m1[3 * i], m1[3 * i + 1], m1[3 * i + 2]);
  m2[3] = fmaxf(m1[9], m1[10]);
  return max3(m2[0], m2[1], fmaxf(m2[2], m2[3]));
}

// Max over the chunks of x that bit c of `vis` marks (-inf for none): masked columns
// (outside [lo, hi)) of those chunks are set to -inf first when `masked`.
template <int c>
__device__ __forceinline__ float chunk_max(float (&x)[128], uint32_t vis, bool masked, int lo,
                                           int hi) {
  if (!(vis & (1u << c))) return -INFINITY;
  if (masked) {
#pragma unroll
    for (int k = 0; k < 32; ++k)
      if (32 * c + k < lo || 32 * c + k >= hi) x[32 * c + k] = -INFINITY;
  }
  return max32_chunk<c>(x);
}

template <bool kBF16>
__global__ void __launch_bounds__(kPairThreads, 1)
    attn_fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PairSmem::kBar);
  uint64_t* q_full = bars;                          // [item parity]
  uint64_t* q_empty = bars + 2;                     // [item parity]
  uint64_t* k_full = bars + 4;
  uint64_t* v_full = bars + 4 + kPairStages;
  uint64_t* kv_empty = bars + 4 + 2 * kPairStages;
  // per query tile x; each barrier has one waiting side, which waits for every phase in
  // turn, so a parity wait never meets a barrier two phases ahead
  uint64_t* s_full = bars + 4 + 3 * kPairStages;    // S_x computed
  uint64_t* s_free = s_full + 2;                    // S_x loaded by warpgroup x
  uint64_t* p_full = s_full + 4;                    // P_x written
  uint64_t* o_done = s_full + 6;                    // O_x += P_x V landed
  uint64_t* o_free = s_full + 8;                    // O_x read by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PairSmem::kTmemSlot);

  const int warp = static_cast<int>(warp_id());
  const int num_pairs = p.n / kFwdBM;
  const int num_items = p.num_bh * num_pairs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 128);
    }
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane_id() == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      bool ok = true;
      int J = 0;  // K/V tiles loaded so far by this CTA
      for (int it = 0, w = persistent_item(0); w < num_items && ok; w = persistent_item(++it)) {
        int bh, i;
        pair_item(w, p.num_bh, num_pairs, &bh, &i);
        const int bb = bh / p.H, hh = bh % p.H;
        const PairPlan pl = pair_plan(i, p.n, p.bs);
        const int qb = it & 1;
        if (it >= 2) ok = mbar_wait(&q_empty[qb], ((it >> 1) - 1) & 1);
        if (!ok) break;
        mbar_expect_tx(&q_full[qb], 2 * kTile16);
        uint8_t* qdst = smem + PairSmem::kQ + qb * 2 * kTile16;
        tma_load_4d(&tm_q, &q_full[qb], qdst, 0, i * kFwdBM, hh, bb);
        tma_load_4d(&tm_q, &q_full[qb], qdst + kTile16, 0, p.n + i * kFwdBM, hh, bb);
        for (int j = 0; j < pl.na + pl.nb && ok; ++j, ++J) {
          const int s = pair_step(pl, j, p.n).s;
          const int st = J % kPairStages;
          if (J >= kPairStages) ok = mbar_wait(&kv_empty[st], ((J / kPairStages) - 1) & 1);
          if (!ok) break;
          mbar_expect_tx(&k_full[st], kTile16);
          tma_load_4d(&tm_k, &k_full[st], smem + PairSmem::kK + st * kTile16, 0, s, hh, bb);
          mbar_expect_tx(&v_full[st], kTile16);
          tma_load_4d(&tm_v, &v_full[st], smem + PairSmem::kV + st * kTile16, 0, s, hh, bb);
        }
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------- UMMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_f16(128, 128, false, false, kBF16);
      constexpr uint32_t idesc_pv = idesc_f16(128, 64, false, true, kBF16);
      const uint32_t sbase = smem_u32(smem);
      bool ok = true;
      // P V products of the previous step, noisy first
      struct Pv {
        int x, it, J;
        bool first, last;
      };
      Pv pa{}, pb{};
      int np = 0;
      uint32_t s_issued = 0;  // bit x: an S tile of query tile x has been issued
      uint32_t sf_par = 0;    // bit x: parity of the next s_free[x] phase to wait for
      uint32_t pv_par = 0;    // bit x: parity of the next p_full[x] phase to wait for
      auto issue_pv = [&](const Pv& e) {
        const int st = e.J % kPairStages;
        ok = ok && mbar_wait(&v_full[st], (e.J / kPairStages) & 1);
        if (ok && e.first && e.it > 0) ok = mbar_wait(&o_free[e.x], (e.it - 1) & 1);
        ok = ok && mbar_wait(&p_full[e.x], (pv_par >> e.x) & 1u);
        if (!ok) return;
        pv_par ^= 1u << e.x;
        tc_fence_after();
        const uint64_t vdesc = sw128_desc(sbase + PairSmem::kV + st * kTile16, kTile16, 1024);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + 384 + e.x * 64, tmem + 256 + e.x * 64 + kk * 8,
                  vdesc + ((kk * 2048) >> 4), idesc_pv, (!e.first || kk > 0) ? 1u : 0u);
        umma_commit(&o_done[e.x]);
        if (e.last) umma_commit(&kv_empty[st]);
      };
      int J = 0;
      for (int it = 0, w = persistent_item(0); w < num_items && ok; w = persistent_item(++it)) {
        int bh, i;
        pair_item(w, p.num_bh, num_pairs, &bh, &i);
        const PairPlan pl = pair_plan(i, p.n, p.bs);
        const int qb = it & 1;
        ok = mbar_wait(&q_full[qb], (it >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const int steps = pl.na + pl.nb;
        bool first[2] = {true, true};
        for (int j = 0; j < steps && ok; ++j, ++J) {
          const PairStep ps = pair_step(pl, j, p.n);
          const int st = J % kPairStages;
          ok = mbar_wait(&k_full[st], (J / kPairStages) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint64_t kdesc = sw128_desc(sbase + PairSmem::kK + st * kTile16, 16, 1024);
          const int last_x = ps.need[1] ? 1 : 0;
          Pv c0{}, c1{};
          int nc = 0;
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (!ps.need[x] || !ok) continue;
            if ((s_issued >> x) & 1u) {  // warpgroup x has loaded its previous S tile
              ok = mbar_wait(&s_free[x], (sf_par >> x) & 1u);
              if (!ok) break;
              sf_par ^= 1u << x;
              tc_fence_after();
            }
            s_issued |= 1u << x;
            const uint64_t qdesc =
                sw128_desc(sbase + PairSmem::kQ + (qb * 2 + x) * kTile16, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_ss(tmem + x * 128, qdesc + ((kk * 32) >> 4), kdesc + ((kk * 32) >> 4),
                      idesc_qk, kk > 0 ? 1u : 0u);
            umma_commit(&s_full[x]);
            if (j == steps - 1 && x == last_x) umma_commit(&q_empty[qb]);
            const Pv e{x, it, J, first[x], x == last_x};
            if (nc == 0) c0 = e;
            else c1 = e;
            ++nc;
            first[x] = false;
          }
          if (np >= 1 && ok) issue_pv(pa);
          if (np == 2 && ok) issue_pv(pb);
          pa = c0;
          pb = c1;
          np = nc;
        }
      }
      if (np >= 1 && ok) issue_pv(pa);
      if (np == 2 && ok) issue_pv(pb);
    }
    __syncwarp();
  } else {
    // ---------------- softmax: warpgroup x owns query tile x of the pair ----------------
    const int x = warp >> 2;
    const int row = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + x * 128;
    const uint32_t tP = tmem + lane_base + 256 + x * 64;
    const uint32_t tO = tmem + lane_base + 384 + x * 64;
    const int shift = x == 0 ? 1 : 0;
    bool ok = true;
    int pv = 0;           // P V products of this warpgroup's tile so far
    uint32_t s_par = 0;   // parity of the next s_full[x] phase
    for (int it = 0, w = persistent_item(0); w < num_items; w = persistent_item(++it)) {
      int bh, i;
      pair_item(w, p.num_bh, num_pairs, &bh, &i);
      const int bb = bh / p.H, hh = bh % p.H;
      const int q_row0 = x * p.n + i * kFwdBM;
      const int qi = q_row0 + row;
      const PairPlan pl = pair_plan(i, p.n, p.bs);
      float m_run = -INFINITY, l_run = 0.f;
      int own = 0;
      for (int j = 0; j < pl.na + pl.nb && ok; ++j) {
        const PairStep ps = pair_step(pl, j, p.n);
        if (!ps.need[x]) continue;
        const int rule = ps.rule[x];
        ok = mbar_wait_warp(&s_full[x], s_par);
        if (!ok) break;
        s_par ^= 1u;
        tc_fence_after();
        // this row's visible key columns of the tile, and which 32-column chunks any row of
        // the warp can see
        int lo = 0, hi = kFwdBN;
        if (rule != 0) {
          int vlo, vhi;
          train_row_interval(rule, shift, qi, p.n, p.bs, &vlo, &vhi);
          lo = imax(vlo - ps.s, 0);
          hi = imin(vhi - ps.s, kFwdBN);
        }
        uint32_t vis = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (__any_sync(0xffffffffu, hi > lo && hi > 32 * c && lo < 32 * c + 32)) vis |= 1u << c;
        float xs[128];
        {
          uint32_t r[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32_async(tS + c * 32, r[c]);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            reg_fence(r[c]);
#pragma unroll
            for (int k = 0; k < 32; ++k) xs[c * 32 + k] = __uint_as_float(r[c][k]);
          }
        }
        tc_fence_before();
        mbar_arrive(&s_free[x]);  // S is in registers: the issuer may compute the next one
        // chunks no row of the warp can see are neither masked nor reduced: their
        // exponentials are skipped below and P is 0 there
        const bool masked = rule != 0;
        const float mx = max3(chunk_max<0>(xs, vis, masked, lo, hi),
                              chunk_max<1>(xs, vis, masked, lo, hi),
                              fmaxf(chunk_max<2>(xs, vis, masked, lo, hi),
                                    chunk_max<3>(xs, vis, masked, lo, hi))) *
                         p.scale_log2;
        float alpha = 1.f;
        bool rescale = false;
        const float m_new = fmaxf(m_run, mx);
        if (m_new - m_run > kRescaleLog2) {  // false for NaN (-inf - -inf)
          alpha = ex2(m_run - m_new);        // 0 when m_run = -inf
          rescale = own > 0;
          m_run = m_new;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        const float2 nm2 = make_float2(-m_use, -m_use);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
          if (vis & (1u << c)) {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int gi = c * 16 + k;  // column pair of the row
              const float2 tt =
                  __ffma2_rn(make_float2(xs[2 * gi], xs[2 * gi + 1]), sc2, nm2);
              float2 e;
              if ((gi * kPairPoly) / 64 != ((gi + 1) * kPairPoly) / 64)
                e = exp2_fma2(tt);
              else
                e = make_float2(ex2(tt.x), ex2(tt.y));
              acc[k & 3] = __fadd2_rn(acc[k & 3], e);
              pk[k] = pack2<kBF16>(e.x, e.y);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) pk[k] = 0u;
          }
          if (c == 0 && own > 0) {
            // P_x and O_x are free once the previous O += P V has landed (normally long
            // since: it was issued when this warpgroup published its previous P)
            ok = mbar_wait_warp(&o_done[x], (pv - 1) & 1);
            tc_fence_after();
          }
          tmem_st16(tP + c * 16, pk);
        }
        if (!ok) break;
        const float2 a01 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
        l_run = l_run * alpha + (a01.x + a01.y);
        // the rescale's TMEM load/store is warp-collective: vote, and let the rows that do
        // not need it multiply by alpha = 1
        if (__any_sync(0xffffffffu, rescale)) {
          uint32_t r[2][32];
          tmem_ld32_async(tO, r[0]);
          tmem_ld32_async(tO + 32, r[1]);
          tmem_ld_wait();
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            reg_fence(r[c2]);
#pragma unroll
            for (int k = 0; k < 32; ++k)
              r[c2][k] = __float_as_uint(__uint_as_float(r[c2][k]) * alpha);
            tmem_st32(tO + c2 * 32, r[c2]);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[x]);
        ++pv;
        ++own;
      }
      // ---- epilogue: the tile's last O += P V has landed; O / l out through a swizzled
      // shared-memory tile and one TMA store, the LSE to global memory ----
      if (ok && own > 0) ok = mbar_wait_warp(&o_done[x], (pv - 1) & 1);
      {  // the warpgroup's four warps agree on whether to go on
        uint32_t all;
        asm volatile(
            "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, 128, p;\n"
            " selp.u32 %0, 1, 0, q;\n}\n"
            : "=r"(all)
            : "r"(static_cast<uint32_t>(ok)), "r"(1 + x)
            : "memory");
        ok = all != 0;
      }
      if (!ok) break;
      tc_fence_after();
      uint32_t r[2][32];
      tmem_ld32_async(tO, r[0]);
      tmem_ld32_async(tO + 32, r[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&o_free[x]);  // O is in registers: the next item's P V may overwrite it
      const float inv = 1.f / l_run;
      const bool leader = (row == 0);
      uint8_t* stage = smem + PairSmem::kOut + x * kTile16;
      if (leader) bulk_wait_group_read0_fwd();  // the previous store from this tile has read it
      asm volatile("bar.sync %0, 128;" ::"r"(1 + x) : "memory");
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        reg_fence(r[c2]);
        uint32_t packed[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          packed[k] = pack2<kBF16>(__uint_as_float(r[c2][2 * k]) * inv,
                                   __uint_as_float(r[c2][2 * k + 1]) * inv);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(stage + sw128_offset(row, c2 * 4 + k)) =
              make_uint4(packed[4 * k], packed[4 * k + 1], packed[4 * k + 2], packed[4 * k + 3]);
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync %0, 128;" ::"r"(1 + x) : "memory");
      if (leader) {
        tma_store_4d(&tm_o, stage, 0, q_row0, hh, bb);
        bulk_commit_group_fwd();
      }
      if (p.lse != nullptr)
        p.lse[bb * p.lse_sb + hh * p.lse_sh + qi] =
            (m_run + __log2f(l_run)) * 0.69314718055994530942f;
    }
  }
  if (threadIdx.x == 0 || threadIdx.x == 128) bulk_wait_group0_fwd();  // O stores have landed
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bd3
