// Flash-attention forward, two query tiles per CTA (sm_100a).
//
// Same function as fwd::flash_fwd_kernel (the forward of flash_attention /
// pallas_flash_attention, attnax/kernels/attention.py:209-283 and
// attnax/kernels/pallas.py:118-244), organised so the tensor core never
// waits on one softmax:
//   * CTA = two 128-row query tiles (A, B) of one (batch, query head) that
//     share every K/V tile the TMA warp loads;
//   * warps 0-3 run the softmax of tile A, warps 4-7 of tile B, warp 8 issues
//     TMA, warp 9 issues tcgen05.mma (warps 10-11 complete the warpgroup that
//     hands its registers to the softmax warpgroups);
//   * TMEM: S_A [0,128), S_B [128,256), O_A [256, 256+D), O_B after it.  P
//     (bf16/f16) is written back over the first 64 columns of its S and the
//     PV product reads it straight from TMEM (tcgen05.mma with A in TMEM);
//   * tensor-core order S_A(j), S_B(j), PV_A(j), S_A(j+1), PV_B(j), S_B(j+1),
//     so each softmax overlaps two GEMMs of the other tile;
//   * O is rescaled only when a row maximum grows by more than 2^8 (the
//     stale maximum keeps P <= 256, exact after the final 1/l); kv tiles run
//     from the diagonal downwards, so under ALiBi the first tile already
//     holds the largest bias and rescales become rare;
//   * one exponential in ATTN_FWD2_POLY_EVERY uses a cubic polynomial on the
//     FMA pipe (2^x = 2^n * p(f), n = round(x), |f| <= 1/2, coefficients
//     fitted for this kernel) to take load off the MUFU pipe;
//   * scale/ALiBi/exp-argument/row-sum arithmetic runs as packed f32x2 ops.
#include <cfloat>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace attnb200 {
namespace fwd2 {

constexpr int BM = 128, BN = 128;
constexpr int kThreads = 384;      // 3 warpgroups: softmax A, softmax B, TMA + MMA (+2 idle warps)
// Register split (setmaxnreg): launched at kLaunchRegs per thread; the TMA/MMA
// warpgroup gives registers up, the softmax warpgroups take them:
// 128 * kProducerRegs + 256 * kSoftmaxRegs == 384 * kLaunchRegs.
constexpr int kLaunchRegs = 168, kProducerRegs = 104, kSoftmaxRegs = 200;
static_assert(128 * kProducerRegs + 256 * kSoftmaxRegs == kThreads * kLaunchRegs, "register split");
constexpr float kRescaleThreshold = 8.f;  // log2 units
#ifndef ATTN_FWD2_MAX3
#define ATTN_FWD2_MAX3 0  // three-input max in the row-max tree
#endif
#ifndef ATTN_FWD2_REVERSE
#define ATTN_FWD2_REVERSE 1  // kv tiles from the diagonal down: the first tile holds the row maximum under ALiBi
#endif
#ifndef ATTN_FWD2_POLY_EVERY
#define ATTN_FWD2_POLY_EVERY 0  // one exponential in this many uses the FMA-pipe polynomial (0: none)
#endif

template <int D>
struct Cfg {
  static constexpr int KCH = D / 64;
  static constexpr int STAGES = (D == 64) ? 4 : 2;
  static constexpr int Q_BYTES = KCH * BM * 128;  // one query tile
  static constexpr int KV_BYTES = KCH * BN * 128;
  static constexpr int OFF_Q = 0;                  // Q_A, Q_B
  static constexpr int OFF_K = 2 * Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + STAGES * KV_BYTES;
  static constexpr int NBAR = 1 + 3 * STAGES + 6;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NBAR * 8;
  // Document ids of a boundary kv tile, one 128-entry copy per softmax warp.
  static constexpr int OFF_DOC = (OFF_TMEMPTR + 16 + 15) & ~15;
  static constexpr int SMEM = OFF_DOC + 8 * BN * 4 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  __host__ __device__ static constexpr uint32_t s_col(int x) { return x ? 128u : 0u; }
  __host__ __device__ static constexpr uint32_t o_col(int x) { return x ? 256u + D : 256u; }
};

struct Args {
  int B, Hq, Hkv, Sq, Skv, group, n_ctas;
  float sl2;
  void* out;
  long long o_s0, o_s1, o_s2;
  float* lse;
  attn_mask_t mask;
  const int2* doc_q_tiles;
  const int2* doc_kv_tiles;
  const int2* doc_jrange;  // per q tile: kv tiles whose document ids can match (or null)
  int nq_doc, nk_doc;
  // Document masks: [B][n_ctas] CTA indices, longest first (or null); the
  // grid is then (n_ctas * Hq, 1, B) with heads fastest.
  const int* cta_order;
  // Ring accumulation (acc_o non-null): the launch's normalised rows are
  // folded into a running result by log-sum-exp (the per-step update of
  // ring_attention, attnax/kernels/attention.py:662-671) instead of being
  // stored.  acc_o is [B][Hq][acc_rows][D] fp32, acc_lse [B][Hq][acc_rows]
  // (natural log, -inf = nothing yet; acc_o rows are then not read); launch
  // row r is accumulator row acc_row0 + r.  Rows >= acc_final_from write the
  // merged row to `out` (in the tensor dtype) instead of acc_o; the merged
  // LSE always goes to acc_lse.
  float* acc_o;
  float* acc_lse;
  int acc_rows, acc_row0, acc_final_from;
};

// Cubic fit of 2^f on [-1/2, 1/2] (max relative error 7.6e-5), our own fit.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float y = x + 12582912.f;  // 1.5 * 2^23: the rounded integer lands in the low mantissa bits
  const float f = x - (y - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.05517084f, f, 0.24260935f), f, 0.69326097f), f, 0.99992818f);
  return __int_as_float(__float_as_int(p) + ((__float_as_int(y) - 0x4B400000) << 23));
}

// Boundary tile of a band, prefix or document mask: this thread's row of S in
// TMEM (s_addr, BN columns) gets -inf in every dropped column, 32 columns at a
// time.  dq0 = q - kv and kv0 = global kv at column 0; ncols columns lie inside
// the sequence; doc_ids (or null) holds the tile's column document ids.  Out
// of line, so the full-tile code around the call keeps its registers and
// schedule.
__device__ __noinline__ void mask_boundary_row(uint32_t s_addr, long long dq0, long long kv0, int ncols, bool has_band,
                                               long long band_lo, long long band_hi, bool has_prefix, int pref,
                                               const int* doc_ids, int doc_row) {
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t raw[32];
    tmem_ld32(s_addr + c * 32, raw);
    const long long dc = dq0 - c * 32;  // q - kv at chunk column e is dc - e
    uint32_t keep = bit_range(0, (long long)ncols - c * 32 - 1);  // inside the sequence
    if (has_band) keep &= bit_range(dc - band_hi, dc - band_lo);
    if (has_prefix) keep &= bit_range(0, pref - (kv0 + c * 32) - 1) | bit_range(0, dc);
    if (doc_ids) {
      const int4* ids = reinterpret_cast<const int4*>(doc_ids + c * 32);
      uint32_t same = 0u;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int4 v = ids[u];
        same |= ((uint32_t)(v.x == doc_row) | ((uint32_t)(v.y == doc_row) << 1) | ((uint32_t)(v.z == doc_row) << 2) |
                 ((uint32_t)(v.w == doc_row) << 3))
                << (4 * u);
      }
      keep &= same;
    }
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e)
      if (!((keep >> e) & 1u)) raw[e] = 0xff800000u;  // -inf
    tmem_st32(s_addr + c * 32, raw);
  }
  tmem_wait_st();
}

// ACC: the ring variant that merges into a running result (Args::acc_o); a
// separate instantiation so the plain forward's epilogue stays as it is.
template <int D, bool BF16, bool ACC = false>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Args a) {
  using C = Cfg<D>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t sb = (raw_base + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw_base);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  int ct, hq;
  if (a.cta_order) {
    const int k = (int)blockIdx.x / a.Hq;
    hq = (int)blockIdx.x - k * a.Hq;
    ct = a.cta_order[(long long)b * a.n_ctas + k];
  } else {
    ct = a.n_ctas - 1 - (int)blockIdx.x;  // heavy (late) tiles first
    hq = blockIdx.y;
  }
  const int hkv = hq / a.group;
  int q0[2], q1[2];
  bool act[2];
  for (int x = 0; x < 2; ++x) {
    q0[x] = ct * 2 * BM + x * BM;
    q1[x] = min(q0[x] + BM, a.Sq);
    act[x] = q0[x] < a.Sq;
  }

  const uint32_t bar0 = sb + C::OFF_BAR;
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + S + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (1 + 2 * S + s); };
  auto s_full = [&](int x) { return bar0 + 8u * (1 + 3 * S + x); };
  auto p_full = [&](int x) { return bar0 + 8u * (3 + 3 * S + x); };
  auto o_done = [&](int x) { return bar0 + 8u * (5 + 3 * S + x); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sp + C::OFF_TMEMPTR);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(s_full(x), 1);
      mbar_init(p_full(x), 4);  // one arrival per softmax warp
      mbar_init(o_done(x), 1);
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Union of the two tiles' kv ranges; per-tile state of each kv tile.
  int jl[2], jh[2];
  for (int x = 0; x < 2; ++x) {
    if (act[x]) band_tile_range(a.mask, q0[x], q1[x], a.Skv, BN, &jl[x], &jh[x]);
    else jl[x] = jh[x] = 0;
    if (act[x] && a.doc_jrange) {
      const int2 r = a.doc_jrange[(long long)b * a.nq_doc + q0[x] / kDocTile];
      jl[x] = max(jl[x], r.x);
      jh[x] = max(jl[x], min(jh[x], r.y));
    }
  }
  const int j_lo = act[1] ? min(jl[0], jl[1]) : jl[0];
  const int j_hi = act[1] ? max(jh[0], jh[1]) : jh[0];
  // kv tile visited at position t of the loop (all three roles use the same order).
  auto kv_tile = [&](int t) { return ATTN_FWD2_REVERSE ? j_hi - 1 - t : j_lo + t; };
  const int n_tiles = j_hi - j_lo;
  // State of kv tile j for the query tile (active, kv range [lo, hi), rows [r0, r1)).
  auto state_at = [&](bool x_act, int lo, int hi, int r0, int r1, int j) {
    if (!x_act || j < lo || j >= hi) return (int)kSkip;
    return tile_state(a.mask, a.doc_q_tiles, a.doc_kv_tiles, a.nq_doc, a.nk_doc, b, r0, r1, j * BN,
                      min((j + 1) * BN, a.Skv), BN);
  };
  // x is a compile-time constant at every call (the arrays stay in registers).
  auto state_of = [&](int x, int j) { return state_at(act[x], jl[x], jh[x], q0[x], q1[x], j); };
  // Inside a tile's band range only a prefix or document mask can drop a kv
  // tile; otherwise the TMA and MMA warps need only the range test.
  const bool may_skip = a.mask.prefix_len != nullptr || a.mask.doc_q != nullptr;
  auto kept = [&](int x, int j) {
    return may_skip ? state_of(x, j) != kSkip : (act[x] && j >= jl[x] && j < jh[x]);
  };

  if (warp >= 8) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
   if (warp == 8) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_expect_tx(q_full, 2 * C::Q_BYTES);
      for (int x = 0; x < 2; ++x)
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sb + C::OFF_Q + x * C::Q_BYTES + c * BM * 128, &tm_q, q_full, c * 64, q0[x], hq, b);
      int n = 0;
      for (int t = 0; t < n_tiles; ++t) {
        const int j = kv_tile(t);
        if (!kept(0, j) && !kept(1, j)) continue;
        const int s = n % S;
        if (!mbar_wait(kv_empty(s), ((n / S) & 1) ^ 1, kStatusTimeoutLoad)) break;
        mbar_expect_tx(k_full(s), C::KV_BYTES);
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sb + C::OFF_K + s * C::KV_BYTES + c * BN * 128, &tm_k, k_full(s), c * 64, j * BN, hkv, b);
        mbar_expect_tx(v_full(s), C::KV_BYTES);
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sb + C::OFF_V + s * C::KV_BYTES + c * BN * 128, &tm_v, v_full(s), c * 64, j * BN, hkv, b);
        ++n;
      }
    }
   } else if (warp == 9) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr int FMT = BF16 ? 1 : 0;
      constexpr uint32_t IDESC_QK = idesc_f16(128, BN, FMT, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_f16(128, D, FMT, 0, 1);
      bool ok = mbar_wait(q_full, 0, kStatusTimeoutMma);
      int it[2] = {0, 0};      // S products issued per tile
      int pv[2] = {0, 0};      // PV products issued per tile
      int prev_s = -1, n = 0;  // stage of the previous kv tile, kv tiles consumed
      bool prev_act[2] = {false, false};
      // Descriptor bases; each operand is a base plus a constant offset.
      const uint64_t dQ = sdesc_sw128(sb + C::OFF_Q, 16, 1024);
      const uint64_t dK = sdesc_sw128(sb + C::OFF_K, 16, 1024);
      const uint64_t dV = sdesc_sw128(sb + C::OFF_V, BN * 128, 1024);  // MN-major
      auto issue_s = [&](int x, int s) {
        const uint32_t d = tmem + C::s_col(x);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t ad = sdesc_add(dQ, x * C::Q_BYTES + (k >> 2) * BM * 128 + (k & 3) * 32);
          const uint64_t bd = sdesc_add(dK, s * C::KV_BYTES + (k >> 2) * BN * 128 + (k & 3) * 32);
          umma_f16(d, ad, bd, IDESC_QK, k > 0 ? 1u : 0u);
        }
        umma_commit(s_full(x));
        ++it[x];
      };
      auto issue_pv = [&](int x, int s) -> bool {
        if (!mbar_wait(p_full(x), pv[x] & 1, kStatusTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t pa = tmem + C::s_col(x);  // P: bf16 pairs in the first 64 columns of S
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t bd = sdesc_add(dV, s * C::KV_BYTES + k * 16 * 128);
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem + C::o_col(x)),
              "r"(pa + (uint32_t)(k * 8)), "l"(bd), "r"(IDESC_PV), "r"((pv[x] > 0 || k > 0) ? 1u : 0u)
              : "memory");
        }
        umma_commit(o_done(x));
        ++pv[x];
        return true;
      };
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int j = kv_tile(t);
        const bool ax = kept(0, j), bx = kept(1, j);
        if (!ax && !bx) continue;
        const int s = n % S;
        // PV_A of the previous kv tile needs only that tile's V: it is issued
        // before waiting for this tile's K, so a late K cannot hold it up.
        if (prev_s >= 0) {
          ok = mbar_wait(v_full(prev_s), ((n - 1) / S) & 1, kStatusTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          if (prev_act[0]) ok = issue_pv(0, prev_s);
          if (!ok) break;
        }
        ok = mbar_wait(k_full(s), (n / S) & 1, kStatusTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        if (ax) issue_s(0, s);
        if (prev_act[1]) ok = issue_pv(1, prev_s);
        if (!ok) break;
        // PV_B was the previous stage's last reader: release the stage now
        // (the commit tracks every MMA issued so far), not after S_B, so the
        // next K/V load into it starts one GEMM earlier.
        if (prev_s >= 0) umma_commit(kv_empty(prev_s));
        if (bx) issue_s(1, s);
        prev_s = s;
        prev_act[0] = ax;
        prev_act[1] = bx;
        ++n;
      }
      if (ok && prev_s >= 0) {
        ok = mbar_wait(v_full(prev_s), ((n - 1) / S) & 1, kStatusTimeoutMma);
        if (ok && prev_act[0]) ok = issue_pv(0, prev_s);
        if (ok && prev_act[1]) ok = issue_pv(1, prev_s);
        if (ok) umma_commit(kv_empty(prev_s));
      }
    }
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------------------- softmax --
    const int x = warp >> 2;         // query tile of this warpgroup
    const int r = threadIdx.x & 127; // row within the tile == TMEM lane
    const int my_q0 = x ? q0[1] : q0[0];
    const bool my_act = x ? act[1] : act[0];
    const int my_q1 = x ? q1[1] : q1[0], my_jl = x ? jl[1] : jl[0], my_jh = x ? jh[1] : jh[0];
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    float m_run = -FLT_MAX, l_run = 0.f;
    int i = 0;
    bool ok = true;
    // Per-CTA constants of the full-tile path (no per-tile global loads).
    const bool has_alibi = a.mask.alibi_slopes != nullptr;
    const float slope_l2 = has_alibi ? a.mask.alibi_slopes[hq] * kLog2e : 0.f;
    // With a causal band every kept score has q >= kv, so |q - kv| = q - kv
    // and ALiBi is linear in the column: t = s*sl2 + slope*(c - d0).
    const bool linear_alibi = has_alibi && a.mask.has_band && a.mask.band_lo >= 0;
    const long long qg_row = a.mask.q_offset + my_q0 + r;
    // Bias and boolean masks need per-element loads: their boundary tiles are
    // transformed in TMEM in 32-column chunks (mode 0 below).  Band, prefix
    // and document boundaries are a keep-bit pass instead: a rolled loop over
    // the four chunks sets dropped columns to -inf in TMEM, and the tile then
    // takes the same unrolled code as a full tile.  A row that keeps nothing
    // anywhere still ends with m_run == -FLT_MAX (LSE -inf, fixed up by
    // fix_masked_rows_fwd_kernel), as with -FLT_MAX scores.
    // (Mask parameters are read from the kernel arguments where they are used:
    // only the two per-row values below stay in registers.)
    const bool complex_mask = a.mask.bias || a.mask.bool_mask;
    const bool has_doc = a.mask.doc_q != nullptr;
    const int pref = a.mask.prefix_len ? a.mask.prefix_len[b] : 0;
    const int doc_row = (has_doc && my_act && my_q0 + r < a.Sq)
                            ? a.mask.doc_q[(long long)b * a.mask.doc_q_bstride + a.mask.q_offset + my_q0 + r]
                            : 0;
    int* doc_ids = reinterpret_cast<int*>(sp + C::OFF_DOC) + warp * BN;  // this warp's copy
    for (int t = 0; t < n_tiles; ++t) {
      const int j = kv_tile(t);
      const int st = state_at(my_act, my_jl, my_jh, my_q0, my_q1, j);
      if (st == kSkip) continue;
      const int k0 = j * BN;
      const bool part = st == kPartial;
      // Document ids of a boundary tile's columns: loaded before the wait so
      // the latency hides behind the S MMA.
      int cid[BN / 32];
      if (part && has_doc && !complex_mask) {
        const int32_t* doc_cols = a.mask.doc_kv + (long long)b * a.mask.doc_kv_bstride + a.mask.kv_offset;
#pragma unroll
        for (int u = 0; u < BN / 32; ++u) {
          const int kc = k0 + u * 32 + lane;
          cid[u] = kc < a.Skv ? doc_cols[kc] : 0;
        }
      }
      ok = __all_sync(0xffffffffu, mbar_wait(s_full(x), i & 1, kStatusTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_base + C::s_col(x);
      if (part && !complex_mask) {
        if (has_doc) {
          __syncwarp();
#pragma unroll
          for (int u = 0; u < BN / 32; ++u) doc_ids[u * 32 + lane] = cid[u];
          __syncwarp();
        }
        mask_boundary_row(s_addr, qg_row - (a.mask.kv_offset + k0), a.mask.kv_offset + k0, a.Skv - k0,
                          a.mask.has_band != 0, a.mask.band_lo, a.mask.band_hi, a.mask.prefix_len != nullptr, pref,
                          has_doc ? doc_ids : nullptr, doc_row);
      } else if (part) {
        // Boundary tile: mask/transform 32 columns at a time in TMEM so the
        // per-column mask state never competes with the 128 scores.
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t raw[32];
          float t[32];
          tmem_ld32(s_addr + c * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) t[e] = __uint_as_float(raw[e]);
          const RowCtx rc = make_row_ctx(a.mask, a.sl2, b, hq, my_q0 + r, k0 + c * 32,
                                         max(0, min(32, a.Skv - (k0 + c * 32))), false);
          transform_row<32>(t, rc, true);
#pragma unroll
          for (int e = 0; e < 32; ++e) raw[e] = __float_as_uint(t[e]);
          tmem_st32(s_addr + c * 32, raw);
        }
        tmem_wait_st();
      }
      // Scores into registers: the second half loads while the first is processed.
      float s[BN];
      float mxp[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mxp[e] = -FLT_MAX;
      // Mode: 0 = already transformed (bias/boolean boundary), 1 = plain scale
      // (scale folded into exp2), 2 = linear ALiBi, 3 = general ALiBi.  Dropped
      // columns of band/prefix/document boundary tiles are -inf already.
      const int mode = (part && complex_mask) ? 0 : (!has_alibi ? 1 : (linear_alibi ? 2 : 3));
      const int d0 = clamp_i32(qg_row - (a.mask.kv_offset + k0));
      const float fd0 = (float)d0;
      const float base = -slope_l2 * fd0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t raw[32];
          tmem_ld32(s_addr + (h * 2 + c) * 32, raw);
#pragma unroll
          for (int e = 0; e < 32; ++e) s[(h * 2 + c) * 32 + e] = __uint_as_float(raw[e]);
        }
        tmem_wait_ld();
        if (mode == 2) {
          // t = s*sl2 + (base + slope*c), pairs of columns per f32x2 op; the
          // additive term advances by 8*slope along 4 independent chains.
          const unsigned long long sl2x2 = f2_pack(a.sl2, a.sl2);
          const unsigned long long step = f2_pack(8.f * slope_l2, 8.f * slope_l2);
          unsigned long long addv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int c = h * 64 + 2 * q;
            addv[q] = f2_pack(fmaf(slope_l2, (float)c, base), fmaf(slope_l2, (float)(c + 1), base));
          }
#pragma unroll
          for (int c = h * 64; c < h * 64 + 64; c += 2) {
            const int q = (c >> 1) & 3;
            float lo, hi;
            f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sl2x2, addv[q]), lo, hi);
            s[c] = lo;
            s[c + 1] = hi;
            addv[q] = f2_add(addv[q], step);
          }
        } else if (mode == 3) {
#pragma unroll
          for (int c = h * 64; c < h * 64 + 64; ++c) s[c] = fmaf(-slope_l2, fabsf(fd0 - (float)c), s[c] * a.sl2);
        }
#if ATTN_FWD2_MAX3
#pragma unroll
        for (int c = h * 64; c < h * 64 + 64; c += 2) {
          float m3;
          asm("max.f32 %0, %1, %2, %3;" : "=f"(m3) : "f"(mxp[(c >> 1) & 7]), "f"(s[c]), "f"(s[c + 1]));
          mxp[(c >> 1) & 7] = m3;
        }
#else
#pragma unroll
        for (int c = h * 64; c < h * 64 + 64; ++c) mxp[c & 7] = fmaxf(mxp[c & 7], s[c]);
#endif
      }
      float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                       fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      // Plain tiles were maxed on raw scores; the scale is applied inside exp2 below.
      const float sc = (mode == 1) ? a.sl2 : 1.f;
      if (mode == 1) mx *= a.sl2;
      float alpha = 1.f;
      if (mx > m_run + kRescaleThreshold) {
        alpha = ex2(m_run - mx);
        m_run = mx;
      }
      const float neg_m = -m_run;
      unsigned long long sp[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) sp[e] = f2_pack(0.f, 0.f);
      const unsigned long long sc2 = f2_pack(sc, sc), negm2 = f2_pack(neg_m, neg_m);
      // P in two 64-column halves so the S registers die as P is stored.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const int cc = h * 64 + c;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(s[cc], s[cc + 1]), sc2, negm2), x0, x1);
          const float p0 = ex2(x0);
          const float p1 = (ATTN_FWD2_POLY_EVERY > 0 && ((c >> 1) % (ATTN_FWD2_POLY_EVERY > 0 ? ATTN_FWD2_POLY_EVERY / 2 : 1)) ==
                            (ATTN_FWD2_POLY_EVERY > 0 ? ATTN_FWD2_POLY_EVERY / 2 - 1 : 0))
                               ? exp2_poly(x1)
                               : ex2(x1);
          sp[(c >> 1) & 3] = f2_add(sp[(c >> 1) & 3], f2_pack(p0, p1));
          pk[c >> 1] = pack2(p0, p1, BF16);
        }
        tmem_st32(tmem + lane_base + C::s_col(x) + h * 32, pk);
      }
      float sum = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float lo, hi;
        f2_unpack(sp[e], lo, hi);
        sum += lo + hi;
      }
      l_run = l_run * alpha + sum;
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // PV of the previous tile must be complete before O is rescaled.
        ok = __all_sync(0xffffffffu, mbar_wait(o_done(x), (i - 1) & 1, kStatusTimeoutSoftmax));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          const uint32_t ta = tmem + lane_base + C::o_col(x) + c * 32;
          tmem_ld32(ta, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(ta, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(p_full(x));
      ++i;
    }
    // ------------------------------------------------------------ epilogue --
    if (ok && i > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_done(x), (i - 1) & 1, kStatusTimeoutSoftmax));
    if (ACC && ok && my_act) {
      // ---- ring accumulation: merge this launch's row into the running one ----
      tc_fence_after();
      const bool row_ok = (my_q0 + r) < a.Sq;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const float lp = (m_run == -FLT_MAX || l_run <= 0.f) ? -INFINITY : (m_run + lg2(l_run)) * kLn2;
      const long long arow = ((long long)b * a.Hq + hq) * a.acc_rows + a.acc_row0 + my_q0 + r;
      const float la = row_ok ? a.acc_lse[arow] : -INFINITY;
      const float mm = fmaxf(la, lp);
      float ca = 1.f, cp = 0.f, lnew = la;
      if (mm != -INFINITY) {
        const float wa = la == -INFINITY ? 0.f : ex2((la - mm) * kLog2e);
        const float wp = lp == -INFINITY ? 0.f : ex2((lp - mm) * kLog2e);
        const float tot = wa + wp;
        ca = wa / tot;
        cp = wp / tot * inv;
        lnew = mm + lg2(tot) * kLn2;
      }
      const bool read_acc = la != -INFINITY;
      const bool fin = (my_q0 + r) >= a.acc_final_from;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = reinterpret_cast<T*>(a.out) + (long long)b * a.o_s0 + (long long)hq * a.o_s1 +
                (long long)(my_q0 + r) * a.o_s2;
      float* arow_o = a.acc_o + arow * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (i > 0) {
          tmem_ld32(tmem + lane_base + C::o_col(x) + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (!row_ok) continue;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          float4 av = make_float4(0.f, 0.f, 0.f, 0.f);
          if (read_acc) av = *reinterpret_cast<const float4*>(arow_o + c * 32 + v * 4);
          const float m0 = ca * av.x + cp * __uint_as_float(o[v * 4 + 0]);
          const float m1 = ca * av.y + cp * __uint_as_float(o[v * 4 + 1]);
          const float m2 = ca * av.z + cp * __uint_as_float(o[v * 4 + 2]);
          const float m3 = ca * av.w + cp * __uint_as_float(o[v * 4 + 3]);
          if (fin) {
            uint2 w;
            w.x = pack2(m0, m1, BF16);
            w.y = pack2(m2, m3, BF16);
            *reinterpret_cast<uint2*>(orow + c * 32 + v * 4) = w;
          } else {
            *reinterpret_cast<float4*>(arow_o + c * 32 + v * 4) = make_float4(m0, m1, m2, m3);
          }
        }
      }
      if (row_ok) a.acc_lse[arow] = lnew;
    } else if (ok && my_act) {
      tc_fence_after();
      const bool row_ok = (my_q0 + r) < a.Sq;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = reinterpret_cast<T*>(a.out) + (long long)b * a.o_s0 + (long long)hq * a.o_s1 +
                (long long)(my_q0 + r) * a.o_s2;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (i > 0) {
          tmem_ld32(tmem + lane_base + C::o_col(x) + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack2(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv, BF16);
            w.y = pack2(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv, BF16);
            w.z = pack2(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv, BF16);
            w.w = pack2(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv, BF16);
            *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = w;
          }
        }
      }
      if (row_ok && a.lse)
        a.lse[((long long)b * a.Hq + hq) * a.Sq + my_q0 + r] =
            (m_run == -FLT_MAX || l_run <= 0.f) ? -INFINITY : (m_run + lg2(l_run)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fwd2
}  // namespace attnb200
