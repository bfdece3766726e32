// Flash-attention backward for sm_100a (tcgen05 + TMA).  The reference has
// no hand-written backward: its gradients are JAX autodiff of
// standard_attention (attnax/kernels/attention.py:54-71).  With
// P = softmax(S), dV = P^T dO, dS = P * (dO V^T - rowsum(dO * O)),
// dQ = scale * dS K and dK = scale * dS^T Q; P is recomputed from the LSE of
// the forward.  Head dim 128 runs one kernel (dkdv with fused dQ); other
// head dims run two deterministic kernels (dkdv, then dq):
//
//   dkdv: CTA = 128 kv rows of one (batch, kv head).  Loops over every query
//         head of the GQA group and every 64-row q tile the mask keeps:
//           S^T  = K Q^T,  dP^T = V dO^T      (K and V read from TMEM, where the
//                                              CTA stores them once; S^T/dP^T in TMEM)
//           dV  += P^T dO, dK  += dS^T Q      (TMEM accumulators)
//         so dK/dV of a shared KV head are summed over its query heads, the
//         transpose of the reference's jnp.repeat (attention.py:32-39).
//         Fused dQ (D = 128): also dQ^T = K^T dS^T per tile (M = head dim,
//         N = 64 q; V sits in TMEM as the A operand of dP^T); the elementwise warps stage it as
//         [64 q][D] fp32 in shared memory and one thread adds the 32 KB into
//         an fp32 dQ accumulator with a bulk reduction (L2 performs the
//         adds; summation order across kv tiles is not fixed).  K and V stay
//         in shared memory there, S^T/dP^T are single-buffered.
//   dq:   CTA = 128 q rows of one (batch, query head).  Loops over 128-row kv
//         tiles:  S = Q K^T, dP = dO V^T, dQ += dS K (S/dP single-buffered in
//         TMEM and released as soon as the elementwise warps have loaded them).
//
// Warp roles in both: warps 0-7 do the elementwise math and the epilogue --
// warps w and w+4 share TMEM lanes 32*(w%4).. (one row per thread) and split
// the tile's columns in halves, so two warps per sub-partition hide each
// other's latency (no row reductions are needed: P uses the forward LSE);
// warp 8 issues TMA, warp 9 allocates TMEM and issues MMAs.
#include <cfloat>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace attnb200 {
namespace bwd {

#ifndef ATTN_BWD_KV_STAGES
#define ATTN_BWD_KV_STAGES 3  // dK/dV kernel: Q/dO/lse/delta tiles in flight
#endif
#ifndef ATTN_BWD_P_BUFS
#define ATTN_BWD_P_BUFS 1     // dK/dV kernel: P^T/dS^T shared-memory buffers
#endif
#ifndef ATTN_BWD_Q_STAGES
#define ATTN_BWD_Q_STAGES (ATTN_BWD_DQ_KT == 128 ? 2 : 4)  // dQ kernel: K/V tiles in flight
#endif
#ifndef ATTN_BWD_DS_BUFS
#define ATTN_BWD_DS_BUFS 1    // dQ kernel: dS shared-memory buffers
#endif
constexpr int kThreads = 320;  // warps 0-7 elementwise (two per TMEM lane group), 8 TMA, 9 MMA
constexpr int KROWS = 128;  // kv rows per dkdv CTA (MMA M)
constexpr int QT = 64;      // q rows per dkdv iteration (MMA N)
constexpr int QROWS = 128;  // q rows per dq CTA (MMA M)
#ifndef ATTN_BWD_KV_TMEM
#define ATTN_BWD_KV_TMEM 1    // dK/dV kernel: K and V copied once into TMEM as the A operand of S^T, dP^T
#endif
#ifndef ATTN_BWD_FAST_FULL
#define ATTN_BWD_FAST_FULL 1  // full tiles: hoisted row constants, linear ALiBi, packed f32x2 math
#endif
#ifndef ATTN_BWD_FQ_V_TMEM
#define ATTN_BWD_FQ_V_TMEM 1  // fused dQ: V in TMEM as the A operand of dP^T (dQ^T single-buffered)
#endif
#ifndef ATTN_BWD_DQ_RED
#define ATTN_BWD_DQ_RED 0  // fused dQ: vector fp32 reductions from registers into a [D][q] accumulator
                           // (measured slower than the staged bulk reduction: L2 atomics)
#endif
#ifndef ATTN_BWD_FUSED_DQ
#define ATTN_BWD_FUSED_DQ 1  // head dim 128: dQ accumulated by the dK/dV kernel (no dq kernel)
#endif
#ifndef ATTN_BWD_DQ_KT
#define ATTN_BWD_DQ_KT 128
#endif
#ifndef ATTN_BWD_EW_SPLIT
#define ATTN_BWD_EW_SPLIT 2  // fused dK/dV/dQ kernel: elementwise warps per TMEM lane quarter
                             // (4 measured 7% slower at B4 Hq32 Hkv8 S8192: the warps are not
                             // bound by their own elementwise work)
#endif
#ifndef ATTN_BWD_FQ_STAGES
#define ATTN_BWD_FQ_STAGES 3  // fused kernel: Q/dO stages.  A stage is released when its gradient
                              // GEMMs complete, which is when the S^T GEMM two iterations later is
                              // due: with 2 stages every iteration waits out a TMA load (traced)
#endif
#ifndef ATTN_BWD_DQ_STEPS
#define ATTN_BWD_DQ_STEPS 1   // fused kernel: 1 = one staged bulk add per tile, else one per column group
#endif
#ifndef ATTN_BWD_DQ_WARPS
#define ATTN_BWD_DQ_WARPS 1   // fused kernel: a warpgroup of its own reads dQ^T out of TMEM and stages it
                              // (traced: on the elementwise warps it took ~0.54 us of a ~1.75 us iteration)
#endif
constexpr int KT = ATTN_BWD_DQ_KT;  // kv rows per dq iteration (MMA N): 64 or 128

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

struct Args {
  int B, Hq, Hkv, Sq, Skv, Sq_pad, group;
  float sl2, scale;
  const float* lse2;   // [B][Hq][Sq_pad], +inf for padded / fully masked rows
  const float* delta;  // [B][Hq][Sq_pad]
  void* dq; void* dk; void* dv;
  float* dq_acc;       // fused dQ: [B][Hq][Sq_pad][D] fp32, zeroed before the kernel
  long long dq_s[3], dk_s[3], dv_s[3];
  attn_mask_t mask;
  // Document masks: (min, max) ids per kDocTile tile of q / kv, and the
  // overlapping tile range of the other side per q tile (q_jr) / kv tile
  // (kv_qr), all in kDocTile units (null without a document mask).
  const int2* doc_q_tiles;
  const int2* doc_kv_tiles;
  const int2* doc_q_jr;
  const int2* doc_kv_qr;
  int nq_doc, nk_doc;
  // Document masks: [B][n_kt] kv-tile indices of dkdv_kernel, longest first
  // (or null); its grid is then (n_kt * Hkv, 1, B) with heads fastest.
  const int* kv_order;
  int n_kt;
};

// q-tile index range [lo, hi) (tiles of QT) that the band allows for kv rows [k0, k1).
__device__ __forceinline__ void band_q_range(const attn_mask_t& m, int k0, int k1, int Sq, int* lo, int* hi) {
  const int nq = (Sq + QT - 1) / QT;
  *lo = 0;
  *hi = nq;
  if (m.has_band) {
    const long long klo = m.kv_offset + k0, khi = m.kv_offset + k1 - 1;
    long long r_lo = klo + m.band_lo - m.q_offset;  // q - kv >= lo  ->  q >= kv + lo
    long long r_hi = khi + m.band_hi - m.q_offset;
    r_lo = ll_max(r_lo, 0);
    r_hi = ll_min(r_hi, (long long)Sq - 1);
    if (r_hi < r_lo) {
      *lo = *hi = 0;
      return;
    }
    *lo = (int)(r_lo / QT);
    *hi = (int)(r_hi / QT) + 1;
  }
}

// Launch order of dkdv_kernel's kv tiles under a document mask: per batch, kv
// tile indices ranked by the q tiles they visit (band range intersected with
// the document range kv_qr), largest first (earlier tiles first on ties), so
// the longest CTAs start in the first wave.  One block per batch; n_kt ints
// of dynamic shared memory.
static_assert(KROWS == kDocTile, "kv tiles of dkdv_kernel are the document tiles");
__global__ void doc_kv_order_kernel(attn_mask_t m, const int2* kv_qr, int nk_doc, int Sq, int Skv, int n_kt,
                                    int* order) {
  extern __shared__ int work[];
  const int b = blockIdx.x;
  for (int t = threadIdx.x; t < n_kt; t += blockDim.x) {
    int lo, hi;
    band_q_range(m, t * KROWS, min((t + 1) * KROWS, Skv), Sq, &lo, &hi);
    const int2 r = kv_qr[(long long)b * nk_doc + t];
    work[t] = max(0, min(hi, r.y * (kDocTile / QT)) - max(lo, r.x * (kDocTile / QT)));
  }
  __syncthreads();
  for (int t = threadIdx.x; t < n_kt; t += blockDim.x) {
    const int wt = work[t];
    int rank = 0;
    for (int o = 0; o < n_kt; ++o) rank += (work[o] > wt) || (work[o] == wt && o < t);
    order[(long long)b * n_kt + rank] = t;
  }
}

template <int D, bool FQ>
struct CfgKV {
  static_assert(!FQ || D == 128, "fused dQ needs M = head dim = 128");
  static constexpr int KCH = D / 64;
  static constexpr bool RED = FQ && ATTN_BWD_DQ_RED != 0;  // no shared-memory staging of dQ^T
  // Q/dO stages in flight.  A stage is released when the gradient GEMMs of its
  // iteration complete; the fused kernel fits a third stage only with the dQ
  // staging split into column-group steps (ATTN_BWD_DQ_STEPS).
  static constexpr int ST = (FQ && !RED) ? ATTN_BWD_FQ_STAGES : ATTN_BWD_KV_STAGES;
  static constexpr int PB = ATTN_BWD_P_BUFS;
  static constexpr int KV_BYTES = KCH * KROWS * 128;  // K or V tile
  static constexpr int QD_BYTES = KCH * QT * 128;     // Q or dO tile
  static constexpr int STAGE = ((2 * QD_BYTES + 2 * QT * 4) + 1023) / 1024 * 1024;  // 1024-aligned
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = KV_BYTES;
  static constexpr int OFF_ST = 2 * KV_BYTES;                 // stages: Q, dO, lse2, delta
  static constexpr int OFF_P = OFF_ST + ST * STAGE;           // P^T  [PB][128 kv][64 q] bf16
  static constexpr int OFF_DS = OFF_P + PB * KROWS * 128;     // dS^T [PB][128 kv][64 q] bf16
  // Elementwise warps per TMEM lane quarter: each takes QT / SPLIT columns of
  // every q tile.  The fused kernel (V in TMEM, staged dQ) splits the columns
  // ATTN_BWD_EW_SPLIT ways; the other variants two ways.
  static constexpr bool FQ_STAGED = FQ && !RED && ATTN_BWD_FQ_V_TMEM != 0;
  static constexpr int SPLIT = FQ_STAGED ? ATTN_BWD_EW_SPLIT : 2;
  static_assert(SPLIT == 2 || SPLIT == 4, "elementwise split");
  static constexpr int EW_WARPS = 4 * SPLIT;
  static constexpr int HC = QT / SPLIT;                // columns per elementwise thread
  static constexpr int OFF_COLV = OFF_DS + PB * KROWS * 128;  // per elementwise warp: 32 column terms
  // Fused dQ staging [QT / DQ_STEPS q][D] fp32: with one step every column
  // group stages its q rows and one bulk add covers the tile; with SPLIT
  // steps the groups take turns on a buffer of HC rows.
  static constexpr int DQ_STEPS = ATTN_BWD_DQ_STEPS == 1 ? 1 : SPLIT;
  static constexpr int DQ_ROWS = QT / DQ_STEPS;
  // Dedicated dQ warpgroup (warps EW_WARPS .. EW_WARPS + 3, one per TMEM lane
  // quarter = 32 head-dim rows of dQ^T), then the TMA and MMA warps and two
  // idle warps completing their warpgroup: 16 warps launched at 128
  // registers, split by setmaxnreg as 256 * EW_REGS + 128 * DQ_REGS +
  // 128 * TM_REGS == 512 * LAUNCH_REGS.  Otherwise the elementwise warps
  // flush dQ^T themselves and the CTA is EW_WARPS + 2 warps.
  static constexpr bool DQW = FQ_STAGED && DQ_STEPS == 1 && SPLIT == 2 && ATTN_BWD_DQ_WARPS != 0;
  static constexpr int TMA_WARP = DQW ? EW_WARPS + 4 : EW_WARPS;
  static constexpr int MMA_WARP = TMA_WARP + 1;
  static constexpr int THREADS = DQW ? 512 : (EW_WARPS + 2) * 32;
  static constexpr int LAUNCH_REGS = 128, EW_REGS = 168, DQ_REGS = 96, TM_REGS = 80;
  static_assert(!DQW || 256 * EW_REGS + 128 * DQ_REGS + 128 * TM_REGS == 512 * LAUNCH_REGS, "register split");
  // With V in TMEM its shared-memory tile is dead once the elementwise warps
  // have copied it (before the MMA warp issues anything), so the one-step
  // staging buffer (QT x D fp32 = one V tile) reuses it.
  static constexpr bool DQS_IN_V = FQ_STAGED && DQ_STEPS == 1 && QT * D * 4 <= KV_BYTES;
  static constexpr int OFF_DQS_OWN = OFF_COLV + EW_WARPS * 32 * 4;
  static constexpr int OFF_DQS = DQS_IN_V ? OFF_V : OFF_DQS_OWN;
  static constexpr int DQS_BYTES = (FQ && !RED && !DQS_IN_V) ? DQ_ROWS * D * 4 : 0;
  static constexpr int OFF_BAR = OFF_DQS_OWN + DQS_BYTES;
  static constexpr int NBAR = 1 + 2 * ST + 2 + 2 + 1 + PB + 1 + 1 + 6;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_TMEMPTR + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  // TMEM columns.  With K/V in TMEM: K [0, D/2), V [D/2, D) as bf16 pairs, S^T at 128 and
  // dP^T at 192 (single buffers); otherwise S^T [2] at 0/64 and dP^T [2] at 128/192.
  // Fused dQ: S^T at 0, dP^T at 64 (single buffers), then either V at 128 and
  // dQ^T at 192 (V_TMEM), or dQ^T [2] at 128/192.
  static constexpr bool KV_TMEM = !FQ && ATTN_BWD_KV_TMEM != 0;
  static constexpr bool V_TMEM = KV_TMEM || (FQ && ATTN_BWD_FQ_V_TMEM != 0);
  static constexpr int NDQ = (FQ && V_TMEM) ? 1 : 2;  // dQ^T TMEM buffers
  static constexpr int NSB = (KV_TMEM || FQ) ? 1 : 2;
  static constexpr uint32_t COL_K = 0, COL_V = KV_TMEM ? D / 2 : 128;
  static constexpr uint32_t COL_S = KV_TMEM ? 128 : 0;
  static constexpr uint32_t COL_DP = KV_TMEM ? 192 : (FQ ? 64 : 128);
  static constexpr uint32_t COL_DQ = V_TMEM ? 192 : 128;
  static constexpr uint32_t COL_DV = 256, COL_DK = 256 + D;
  static_assert(SMEM <= 232448, "dkdv kernel shared memory");
};

template <int D, bool BF16, bool FQ>
__global__ void __launch_bounds__(CfgKV<D, FQ>::THREADS, 1)
    dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                const __grid_constant__ Args a) {
  using C = CfgKV<D, FQ>;
  constexpr int ST = C::ST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t sb = (raw_base + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw_base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  int kt, hkv;
  if (a.kv_order) {
    const int k = (int)blockIdx.x / a.Hkv;
    hkv = (int)blockIdx.x - k * a.Hkv;
    kt = a.kv_order[(long long)b * a.n_kt + k];
  } else {
    kt = blockIdx.x;  // early kv tiles carry the most q tiles under causal bands
    hkv = blockIdx.y;
  }
  const int k0 = kt * KROWS, k1 = min(k0 + KROWS, a.Skv);

  const uint32_t bar0 = sb + C::OFF_BAR;
  const uint32_t kv_full = bar0;
  auto st_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto st_free = [&](int s) { return bar0 + 8u * (1 + ST + s); };
  auto s_full = [&](int i) { return bar0 + 8u * (1 + 2 * ST + i); };
  auto s_free = [&](int i) { return bar0 + 8u * (3 + 2 * ST + i); };
  const uint32_t p_full = bar0 + 8u * (5 + 2 * ST);
  auto p_free = [&](int buf) { return bar0 + 8u * (6 + 2 * ST + buf); };
  const uint32_t acc_done = bar0 + 8u * (6 + 2 * ST + C::PB);
  const uint32_t kv_tmem = bar0 + 8u * (7 + 2 * ST + C::PB);  // K/V rows stored into TMEM
  auto dq_full = [&](int x) { return bar0 + 8u * (8 + 2 * ST + C::PB + x); };   // dQ^T[x] computed
  auto dq_free = [&](int x) { return bar0 + 8u * (10 + 2 * ST + C::PB + x); };  // dQ^T[x] read out
  const uint32_t stage_full = bar0 + 8u * (12 + 2 * ST + C::PB);  // dQ staging written
  const uint32_t stage_free = bar0 + 8u * (13 + 2 * ST + C::PB);  // previous reduction has read it
  constexpr int NSB = C::NSB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sp + C::OFF_TMEMPTR);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(st_full(s), 1);
      mbar_init(st_free(s), 1);
    }
    for (int i = 0; i < NSB; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), C::EW_WARPS);  // one arrival per elementwise warp
    }
    mbar_init(p_full, C::EW_WARPS);
    for (int q = 0; q < C::PB; ++q) mbar_init(p_free(q), 1);
    mbar_init(acc_done, 1);
    mbar_init(kv_tmem, C::EW_WARPS);
    for (int x = 0; x < 2; ++x) {
      mbar_init(dq_full(x), 1);
      mbar_init(dq_free(x), C::DQW ? 4 : C::EW_WARPS);
    }
    mbar_init(stage_full, C::DQW ? 4 : C::EW_WARPS / C::DQ_STEPS);  // the warps staging one step
    mbar_init(stage_free, 1);
    fence_mbar_init();
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int t_lo, t_hi;
  band_q_range(a.mask, k0, k1, a.Sq, &t_lo, &t_hi);
  if (a.doc_kv_qr) {
    static_assert(KROWS == kDocTile && kDocTile % QT == 0, "document tiles vs kv / q tiles");
    const int2 r = a.doc_kv_qr[(long long)b * a.nk_doc + kt];
    t_lo = max(t_lo, r.x * (kDocTile / QT));
    t_hi = max(t_lo, min(t_hi, r.y * (kDocTile / QT)));
  }
  const int ntiles = t_hi - t_lo;
  const int iters = a.group * ntiles;  // (g, q tile) pairs, g outer
  auto state_of = [&](int qt) {
    const int q0 = qt * QT;
    return tile_state(a.mask, a.doc_q_tiles, a.doc_kv_tiles, a.nq_doc, a.nk_doc, b, q0, min(q0 + QT, a.Sq), k0,
                      k1, KROWS);
  };
  // Inside [t_lo, t_hi) only a prefix mask (or a document mask) can drop a
  // whole tile; the TMA and MMA warps classify tiles only then.
  const bool may_skip = a.mask.prefix_len != nullptr || a.mask.doc_q != nullptr;
  // (g, qt) advance of the flat (g, q tile) loop.
#define DKDV_NEXT(g, qt) ((qt) + 1 == t_hi ? ((qt) = t_lo, ++(g)) : ++(qt))

  // With the dQ warpgroup, each role branch starts with its setmaxnreg (whole
  // warpgroups, as the instruction requires: the TMA/MMA branch also holds
  // the two idle warps), so the register budget covers that role's code.
  if (warp >= C::TMA_WARP) {
   if constexpr (C::DQW) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::TM_REGS));
   if (warp == C::TMA_WARP) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_expect_tx(kv_full, 2 * C::KV_BYTES);
      for (int c = 0; c < C::KCH; ++c) {
        tma_load_4d(sb + C::OFF_K + c * KROWS * 128, &tm_k, kv_full, c * 64, k0, hkv, b);
        tma_load_4d(sb + C::OFF_V + c * KROWS * 128, &tm_v, kv_full, c * 64, k0, hkv, b);
      }
      int i = 0;
      for (int it = 0, g = 0, qt = t_lo; it < iters; ++it, DKDV_NEXT(g, qt)) {
        if (may_skip && state_of(qt) == kSkip) continue;
        const int hq = hkv * a.group + g, q0 = qt * QT;
        const int s = i % ST;
        if (!mbar_wait(st_free(s), ((i / ST) & 1) ^ 1, kStatusTimeoutLoad)) break;
        const uint32_t base = sb + C::OFF_ST + s * C::STAGE;
        mbar_expect_tx(st_full(s), 2 * C::QD_BYTES + 2 * QT * 4);
        for (int c = 0; c < C::KCH; ++c) {
          tma_load_4d(base + c * QT * 128, &tm_q, st_full(s), c * 64, q0, hq, b);
          tma_load_4d(base + C::QD_BYTES + c * QT * 128, &tm_do, st_full(s), c * 64, q0, hq, b);
        }
        const long long row = ((long long)b * a.Hq + hq) * a.Sq_pad + q0;
        bulk_g2s(base + 2 * C::QD_BYTES, a.lse2 + row, QT * 4, st_full(s));
        bulk_g2s(base + 2 * C::QD_BYTES + QT * 4, a.delta + row, QT * 4, st_full(s));
        ++i;
      }
    }
   } else if (warp == C::MMA_WARP) {
    if (lane == 0) {
      constexpr int FMT = BF16 ? 1 : 0;
      constexpr uint32_t ID_S = idesc_f16(128, QT, FMT, 0, 0);
      constexpr uint32_t ID_G = idesc_f16(128, D, FMT, 0, 1);
      constexpr uint32_t ID_DQ = idesc_f16(128, QT, FMT, 1, 1);  // dQ^T = K^T dS^T: both operands MN-major
      bool ok = mbar_wait(kv_full, 0, kStatusTimeoutMma);
      if (C::V_TMEM) ok = ok && mbar_wait(kv_tmem, 0, kStatusTimeoutMma);
      // Descriptor bases; every operand below is a base plus a constant offset.
      const uint64_t dK_k = sdesc_sw128(sb + C::OFF_K, 16, 1024);             // K, K-major
      const uint64_t dV_k = sdesc_sw128(sb + C::OFF_V, 16, 1024);             // V, K-major
      const uint64_t dK_mn = sdesc_sw128(sb + C::OFF_K, KROWS * 128, 1024);   // K^T, MN-major
      const uint64_t dST_k = sdesc_sw128(sb + C::OFF_ST, 16, 1024);           // Q / dO stages, K-major
      const uint64_t dST_mn = sdesc_sw128(sb + C::OFF_ST, QT * 128, 1024);    // Q / dO stages, MN-major
      const uint64_t dP_k = sdesc_sw128(sb + C::OFF_P, 16, 1024);             // P^T, K-major
      const uint64_t dDS_k = sdesc_sw128(sb + C::OFF_DS, 16, 1024);           // dS^T, K-major
      const uint64_t dDS_mn = sdesc_sw128(sb + C::OFF_DS, KROWS * 128, 1024); // dS^T, MN-major
      auto issue_grads = [&](int j) -> bool {
        const int s = j % ST;
        const uint32_t so = s * C::STAGE, po = (j % C::PB) * KROWS * 128;
        if (!mbar_wait(p_full, j & 1, kStatusTimeoutMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < QT / 16; ++k) {
          const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
          umma_f16(tmem + C::COL_DV, sdesc_add(dP_k, po + k * 32), sdesc_add(dST_mn, so + C::QD_BYTES + k * 2048),
                   ID_G, acc);
          umma_f16(tmem + C::COL_DK, sdesc_add(dDS_k, po + k * 32), sdesc_add(dST_mn, so + k * 2048), ID_G, acc);
        }
        if (FQ) {
          // dQ^T (M = D rows of K^T, N = QT, K = KROWS kv rows); its TMEM buffer
          // was last read out for tile j - NDQ.
          if (!mbar_wait(dq_free(j % C::NDQ), ((j / C::NDQ) & 1) ^ 1, kStatusTimeoutMma)) return false;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < KROWS / 16; ++k)
            umma_f16(tmem + C::COL_DQ + (j % C::NDQ) * QT, sdesc_add(dK_mn, k * 2048),
                     sdesc_add(dDS_mn, po + k * 2048), ID_DQ, k > 0 ? 1u : 0u);
          umma_commit(dq_full(j % C::NDQ));
        }
        umma_commit(st_free(s));
        umma_commit(p_free(j % C::PB));
        return true;
      };
      int i = 0;
      for (int it = 0, g = 0, qt = t_lo; ok && it < iters; ++it, DKDV_NEXT(g, qt)) {
        if (may_skip && state_of(qt) == kSkip) continue;
        const int s = i % ST;
        ok = mbar_wait(st_full(s), (i / ST) & 1, kStatusTimeoutMma) &&
             mbar_wait(s_free(i % NSB), ((i / NSB) & 1) ^ 1, kStatusTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t so = s * C::STAGE;
        const uint32_t cs = C::COL_S + (i % NSB) * QT, cdp = C::COL_DP + (i % NSB) * QT;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * QT * 128 + (k & 3) * 32;   // within a Q / dO tile
          const uint32_t koff = (k >> 2) * KROWS * 128 + (k & 3) * 32;  // within the K / V tile
          const uint64_t qb = sdesc_add(dST_k, so + off), db = sdesc_add(dST_k, so + C::QD_BYTES + off);
          const uint32_t acc = k > 0 ? 1u : 0u;
          if (C::KV_TMEM) {
            umma_f16_ts(tmem + cs, tmem + C::COL_K + k * 8, qb, ID_S, acc);
            umma_f16_ts(tmem + cdp, tmem + C::COL_V + k * 8, db, ID_S, acc);
          } else if (C::V_TMEM) {
            umma_f16(tmem + cs, sdesc_add(dK_k, koff), qb, ID_S, acc);
            umma_f16_ts(tmem + cdp, tmem + C::COL_V + k * 8, db, ID_S, acc);
          } else {
            umma_f16(tmem + cs, sdesc_add(dK_k, koff), qb, ID_S, acc);
            umma_f16(tmem + cdp, sdesc_add(dV_k, koff), db, ID_S, acc);
          }
        }
        umma_commit(s_full(i % NSB));
        if (i > 0) ok = issue_grads(i - 1);
        ++i;
      }
      if (ok && i > 0) ok = issue_grads(i - 1);
      umma_commit(acc_done);
    }
   }
  } else if (warp < C::EW_WARPS) {
    if constexpr (C::DQW) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::EW_REGS));
    const int r = threadIdx.x & 127;  // kv row within the tile == TMEM lane
    const int half = warp >> 2;       // columns [HC*half, HC*half + HC) of each q tile
    constexpr int HC = C::HC;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    uint8_t* PT = sp + C::OFF_P;
    uint8_t* DST = sp + C::OFF_DS;
    float* colv = reinterpret_cast<float*>(sp + C::OFF_COLV) + warp * 32;
    // Full tiles: with no ALiBi, or ALiBi under a causal band (every kept
    // score has q >= kv), t = s*sl2 - slope*(d0 + c) - lse2[c] with
    // d0 = q(column 0) - kv(row); the column part -slope*c - lse2[c] is
    // computed once per warp and shared through shared memory.
    const bool fast_mask = ATTN_BWD_FAST_FULL && (!a.mask.alibi_slopes || (a.mask.has_band && a.mask.band_lo >= 0));
    const long long kg_row = a.mask.kv_offset + k0 + r;
    const unsigned long long sl2x2 = f2_pack(a.sl2, a.sl2);
    // Boundary tiles under band, prefix and document masks take the full-tile
    // arithmetic as well; a keep mask of the thread's HC columns then zeroes P
    // and dS of the dropped ones (a select, so scores the mask drops may
    // overflow freely).  Bias and boolean masks keep the transform_row path.
    const bool bits_mask = fast_mask && !a.mask.bias && !a.mask.bool_mask;
    const bool has_doc = a.mask.doc_q != nullptr;
    const int doc_row =
        (has_doc && k0 + r < a.Skv) ? a.mask.doc_kv[(long long)b * a.mask.doc_kv_bstride + kg_row] : 0;
    const bool row_in_prefix = a.mask.prefix_len && kg_row < (long long)a.mask.prefix_len[b];
    int i = 0;
    bool ok = true;
    if (C::V_TMEM) {
      // Warps 0-3 store their K row, warps 4-7 their V row, into TMEM as bf16
      // pairs; with V alone in TMEM each of the SPLIT column groups stores
      // 64 / SPLIT packed columns (128 / SPLIT features) of its V row.
      ok = __all_sync(0xffffffffu, mbar_wait(kv_full, 0, kStatusTimeoutSoftmax));
      if (ok && !C::KV_TMEM) {
        constexpr int PC = 64 / C::SPLIT;  // packed columns per group
        const int gb = half * PC * 4;      // first byte of the group within the V row
        const uint8_t* src = sp + C::OFF_V + (gb / 128) * KROWS * 128;
        uint32_t w[PC];
#pragma unroll
        for (int u = 0; u < PC / 4; ++u) {
          const int unit = (gb % 128) / 16 + u;
          const uint4 v = *reinterpret_cast<const uint4*>(src + r * 128 + ((unit ^ (r & 7)) << 4));
          w[u * 4 + 0] = v.x; w[u * 4 + 1] = v.y; w[u * 4 + 2] = v.z; w[u * 4 + 3] = v.w;
        }
        tmem_st_cols<PC>(tmem + lane_base + C::COL_V + half * PC, w);
        tmem_wait_st();
      } else if (ok) {
        const uint8_t* src = sp + (half ? C::OFF_V : C::OFF_K);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          uint32_t w[32];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint4 v = *reinterpret_cast<const uint4*>(src + c * KROWS * 128 + r * 128 + ((u ^ (r & 7)) << 4));
            w[u * 4 + 0] = v.x; w[u * 4 + 1] = v.y; w[u * 4 + 2] = v.z; w[u * 4 + 3] = v.w;
          }
          tmem_st32(tmem + lane_base + (half ? C::COL_V : C::COL_K) + c * 32, w);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive_warp(kv_tmem);
    }
    // Fused dQ: tile j's dQ^T (this thread: head-dim row r, q columns
    // [HC*half, HC*half + HC)) -> staging [q][D] fp32 -> one bulk add of the
    // whole [QT][D] block into dq_acc by thread 0.
    float* stg = reinterpret_cast<float*>(sp + C::OFF_DQS);
    auto flush_dq = [&](int j, int hq_j, int q0_j) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(dq_full(j % C::NDQ), (j / C::NDQ) & 1, kStatusTimeoutSoftmax)))
        return false;
      tc_fence_after();
      uint32_t v[HC];
      tmem_ld_cols<HC>(tmem + lane_base + C::COL_DQ + (j % C::NDQ) * QT + half * HC, v);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive_warp(dq_free(j % C::NDQ));
      if constexpr (C::RED) {
        // dq_acc is [B][Hq][D][Sq_pad]: this thread's HC q values are contiguous.
        float* dst = a.dq_acc + (((long long)b * a.Hq + hq_j) * D + r) * a.Sq_pad + q0_j + half * HC;
#pragma unroll
        for (int m = 0; m < HC / 4; ++m)
          atomicAdd(reinterpret_cast<float4*>(dst + 4 * m),
                    make_float4(__uint_as_float(v[4 * m]), __uint_as_float(v[4 * m + 1]),
                                __uint_as_float(v[4 * m + 2]), __uint_as_float(v[4 * m + 3])));
        return true;
      }
      // Staging [DQ_ROWS q][D]: in step h the column groups whose q rows fall
      // in [h*DQ_ROWS, (h+1)*DQ_ROWS) write them and thread 0 adds the buffer
      // into dq_acc once the previous bulk reduction has read it.  Every warp
      // waits every step's stage_free phase in order (a parity wait cannot
      // tell a phase from the one two before it, so no waiter may skip one).
      bool ok0 = true;
      for (int h = 0; h < C::DQ_STEPS; ++h) {
        const uint32_t ph = (uint32_t)(j * C::DQ_STEPS + h) & 1u;
        if (threadIdx.x == 0) {
          bulk_wait_read_all();  // the previous reduction has read the staging buffer
          mbar_arrive(stage_free);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(stage_free, ph, kStatusTimeoutSoftmax))) return false;
        const int row0 = half * HC - h * C::DQ_ROWS;  // this group's first row in the buffer
        if (row0 >= 0 && row0 < C::DQ_ROWS) {
#pragma unroll
          for (int c = 0; c < HC; ++c) stg[(row0 + c) * D + r] = __uint_as_float(v[c]);
          fence_proxy_async_smem();
          mbar_arrive_warp(stage_full);
        }
        if (threadIdx.x == 0 && ok0) {
          ok0 = mbar_wait(stage_full, ph, kStatusTimeoutSoftmax);
          if (ok0) {
            bulk_reduce_add_f32(
                a.dq_acc + (((long long)b * a.Hq + hq_j) * a.Sq_pad + q0_j + h * C::DQ_ROWS) * D,
                smem_u32(stg), C::DQ_ROWS * D * 4);
            bulk_commit();
          }
        }
      }
      return __all_sync(0xffffffffu, ok0);  // warp-uniform
    };
    int prev_hq = 0, prev_q0 = 0;
    for (int it = 0, g = 0, qt = t_lo; it < iters; ++it, DKDV_NEXT(g, qt)) {
      const int st = state_of(qt);
      if (st == kSkip) continue;
      const int hq = hkv * a.group + g, q0 = qt * QT;
      const int s = i % ST;
      const bool part_bits = st == kPartial && bits_mask;
      int cid = 0;  // document id of q column lane of this thread's half (loaded before the wait)
      if (part_bits && has_doc) {
        const int qc = q0 + half * HC + lane;
        cid = (lane < HC && qc < a.Sq)
                  ? a.mask.doc_q[(long long)b * a.mask.doc_q_bstride + a.mask.q_offset + qc]
                  : 0;
      }
      ok = ok && __all_sync(0xffffffffu, mbar_wait(s_full(i % NSB), (i / NSB) & 1, kStatusTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      float sc[HC], dp[HC];
      tmem_ld_cols<HC>(tmem + lane_base + C::COL_S + (i % NSB) * QT + half * HC, reinterpret_cast<uint32_t*>(sc));
      tmem_ld_cols<HC>(tmem + lane_base + C::COL_DP + (i % NSB) * QT + half * HC, reinterpret_cast<uint32_t*>(dp));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive_warp(s_free(i % NSB));
      const int c0 = q0 + half * HC;
      const float* sl = reinterpret_cast<const float*>(sp + C::OFF_ST + s * C::STAGE + 2 * C::QD_BYTES) + half * HC;
      const float* sd = sl + QT;
      if ((st == kFull && fast_mask) || part_bits) {
        // (a full tile has all KROWS kv rows inside the sequence; q columns
        // past the end carry lse2 = +inf and delta = 0, so P = dS = 0 there;
        // a boundary tile's keep mask covers both)
        static_assert(HC <= 32, "one column term per lane");
        const float slope = a.mask.alibi_slopes ? __ldg(a.mask.alibi_slopes + hq) * kLog2e : 0.f;
        __syncwarp();
        if (lane < HC) colv[lane] = fmaf(-slope, (float)lane, -sl[lane]);
        __syncwarp();
        const float base = -slope * (float)clamp_i32(a.mask.q_offset + c0 - kg_row);
        const unsigned long long base2 = f2_pack(base, base);
#pragma unroll
        for (int c = 0; c < HC; c += 4) {
          const float4 v4 = *reinterpret_cast<const float4*>(colv + c);
          const float4 d4 = *reinterpret_cast<const float4*>(sd + c);
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(sc[c + e], sc[c + e + 1]), sl2x2,
                             f2_add(base2, e ? f2_pack(v4.z, v4.w) : f2_pack(v4.x, v4.y))), x0, x1);
            const unsigned long long p2 = f2_pack(ex2(x0), ex2(x1));
            const unsigned long long g2 = f2_mul(p2, f2_sub(f2_pack(dp[c + e], dp[c + e + 1]),
                                                            e ? f2_pack(d4.z, d4.w) : f2_pack(d4.x, d4.y)));
            f2_unpack(p2, sc[c + e], sc[c + e + 1]);
            f2_unpack(g2, dp[c + e], dp[c + e + 1]);
          }
        }
        if (part_bits) {
          const long long dd = a.mask.q_offset + c0 - kg_row;  // q - kv at this thread's column 0
          uint32_t keep = k0 + r < a.Skv ? bit_range(0, (long long)a.Sq - c0 - 1) : 0u;
          if (a.mask.has_band) keep &= bit_range(a.mask.band_lo - dd, a.mask.band_hi - dd);
          if (a.mask.prefix_len && !row_in_prefix) keep &= bit_range(-dd, 31);  // kv < prefix, else kv <= q
          if (has_doc) {
            uint32_t same = 0u;
#pragma unroll
            for (int e = 0; e < HC; ++e) same |= (uint32_t)(__shfl_sync(0xffffffffu, cid, e) == doc_row) << e;
            keep &= same;
          }
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            const bool k = (keep >> c) & 1u;
            sc[c] = k ? sc[c] : 0.f;
            dp[c] = k ? dp[c] : 0.f;
          }
        }
      } else {
        const RowCtx rc = make_row_ctx(a.mask, a.sl2, b, hq, k0 + r, c0, max(0, min(HC, a.Sq - c0)), true);
        transform_row<HC>(sc, rc, st == kPartial || k0 + r >= a.Skv);
        const bool row_ok = k0 + r < a.Skv;
#pragma unroll
        for (int c = 0; c < HC; c += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(sl + c);
          const float4 d4 = *reinterpret_cast<const float4*>(sd + c);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p = row_ok ? ex2(sc[c + e] - lv[e]) : 0.f;
            sc[c + e] = p;
            dp[c + e] = p * (dp[c + e] - dv4[e]);
          }
        }
      }
      if (i >= C::PB) {  // this buffer was last read by the gradient GEMMs of iteration i - PB
        ok = __all_sync(0xffffffffu,
                        mbar_wait(p_free(i % C::PB), ((i / C::PB) - 1) & 1, kStatusTimeoutSoftmax));
        if (!ok) break;
      }
#pragma unroll
      for (int u = 0; u < HC / 8; ++u) {
        const int c = u * 8;
        uint4 pv, dv;
        pv.x = pack2(sc[c], sc[c + 1], BF16); pv.y = pack2(sc[c + 2], sc[c + 3], BF16);
        pv.z = pack2(sc[c + 4], sc[c + 5], BF16); pv.w = pack2(sc[c + 6], sc[c + 7], BF16);
        dv.x = pack2(dp[c], dp[c + 1], BF16); dv.y = pack2(dp[c + 2], dp[c + 3], BF16);
        dv.z = pack2(dp[c + 4], dp[c + 5], BF16); dv.w = pack2(dp[c + 6], dp[c + 7], BF16);
        const int off = r * 128 + (((half * (HC / 8) + u) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(PT + (i % C::PB) * KROWS * 128 + off) = pv;
        *reinterpret_cast<uint4*>(DST + (i % C::PB) * KROWS * 128 + off) = dv;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive_warp(p_full);
      if (FQ && !C::DQW && i > 0) {
        ok = flush_dq(i - 1, prev_hq, prev_q0);
        if (!ok) break;
      }
      prev_hq = hq;
      prev_q0 = q0;
      ++i;
    }
    if (FQ && !C::DQW && ok && i > 0) ok = flush_dq(i - 1, prev_hq, prev_q0);
    if (FQ && !C::DQW && threadIdx.x == 0) bulk_wait_all();
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_done, 0, kStatusTimeoutSoftmax));
    if (ok) {
      tc_fence_after();
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      const bool row_ok = k0 + r < a.Skv;
      T* dvr = reinterpret_cast<T*>(a.dv) + b * a.dv_s[0] + hkv * a.dv_s[1] + (long long)(k0 + r) * a.dv_s[2];
      T* dkr = reinterpret_cast<T*>(a.dk) + b * a.dk_s[0] + hkv * a.dk_s[1] + (long long)(k0 + r) * a.dk_s[2];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        T* dst = which ? dkr : dvr;
        const uint32_t col = which ? C::COL_DK : C::COL_DV;
        const float mul = which ? a.scale : 1.f;
        constexpr int CPP = (D / 32) / C::SPLIT;  // 32-column chunks of dV / dK per column group
        static_assert(CPP >= 1, "epilogue chunks");
#pragma unroll
        for (int c = half * CPP; c < (half + 1) * CPP; ++c) {
          uint32_t o[32];
          if (i > 0) {
            tmem_ld32(tmem + lane_base + col + c * 32, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack2(__uint_as_float(o[v * 8 + 0]) * mul, __uint_as_float(o[v * 8 + 1]) * mul, BF16);
              w.y = pack2(__uint_as_float(o[v * 8 + 2]) * mul, __uint_as_float(o[v * 8 + 3]) * mul, BF16);
              w.z = pack2(__uint_as_float(o[v * 8 + 4]) * mul, __uint_as_float(o[v * 8 + 5]) * mul, BF16);
              w.w = pack2(__uint_as_float(o[v * 8 + 6]) * mul, __uint_as_float(o[v * 8 + 7]) * mul, BF16);
              *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = w;
            }
          }
        }
      }
    }
  } else if (C::DQW && warp < C::EW_WARPS + 4) {
    if constexpr (C::DQW) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::DQ_REGS));
    // ------------------------------------------------------------ dQ^T out --
    // Tile j's dQ^T (this thread: head-dim row r, all QT q columns) -> staging
    // [QT q][D] fp32 in the dead V tile -> one bulk add of the block into
    // dq_acc by the group's first thread, once the previous bulk add has read
    // the staging buffer.  Same (g, q tile) walk and skips as the other roles.
    const int r = threadIdx.x & 127;  // head-dim row of dQ^T == TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const bool leader = threadIdx.x == C::EW_WARPS * 32;
    float* stg = reinterpret_cast<float*>(sp + C::OFF_DQS);
    bool ok = true;
    int j = 0;
    for (int it = 0, g = 0, qt = t_lo; it < iters; ++it, DKDV_NEXT(g, qt)) {
      if (state_of(qt) == kSkip) continue;
      const int hq = hkv * a.group + g, q0 = qt * QT;
      ok = __all_sync(0xffffffffu, mbar_wait(dq_full(j % C::NDQ), (j / C::NDQ) & 1, kStatusTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32(tmem + lane_base + C::COL_DQ + (j % C::NDQ) * QT, v0);
      tmem_ld32(tmem + lane_base + C::COL_DQ + (j % C::NDQ) * QT + 32, v1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive_warp(dq_free(j % C::NDQ));
      const uint32_t ph = (uint32_t)j & 1u;
      if (leader) {
        bulk_wait_read_all();  // the previous reduction has read the staging buffer
        mbar_arrive(stage_free);
      }
      ok = __all_sync(0xffffffffu, mbar_wait(stage_free, ph, kStatusTimeoutSoftmax));
      if (!ok) break;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        stg[c * D + r] = __uint_as_float(v0[c]);
        stg[(c + 32) * D + r] = __uint_as_float(v1[c]);
      }
      fence_proxy_async_smem();
      mbar_arrive_warp(stage_full);
      if (leader) {
        ok = mbar_wait(stage_full, ph, kStatusTimeoutSoftmax);
        if (ok) {
          bulk_reduce_add_f32(a.dq_acc + (((long long)b * a.Hq + hq) * a.Sq_pad + q0) * D, smem_u32(stg),
                              QT * D * 4);
          bulk_commit();
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      ++j;
    }
    if (leader) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == C::MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

#undef DKDV_NEXT

// ------------------------------------------------------------------- dQ ----
template <int D>
struct CfgQ {
  static constexpr int KCH = D / 64;
  static constexpr int ST = ATTN_BWD_Q_STAGES;
  static constexpr int DB = ATTN_BWD_DS_BUFS;
  static constexpr int Q_BYTES = KCH * QROWS * 128;   // Q or dO
  static constexpr int KV_BYTES = KCH * KT * 128;     // K or V tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = Q_BYTES;
  static constexpr int OFF_ST = 2 * Q_BYTES;          // stages: K, V
  static constexpr int DS_BYTES = (KT / 64) * QROWS * 128;   // one dS tile [128 q][KT kv] bf16
  static constexpr int OFF_DS = OFF_ST + ST * 2 * KV_BYTES;   // dS [DB]
  static constexpr int OFF_BAR = OFF_DS + DB * DS_BYTES;
  static constexpr int NSB = (KT == 128) ? 1 : 2;              // TMEM buffers of S and dP
  static constexpr int NBAR = 1 + 2 * ST + 2 * NSB + 1 + DB + 1;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_TMEMPTR + 16 + 1024;
  static_assert(SMEM <= 232448, "dq kernel shared memory");
  static constexpr uint32_t TMEM_COLS = 512;
  // S at [0,128), dP at [128,256) (two 64-column buffers each when KT = 64), dQ at 256
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DQ = 256;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
              const __grid_constant__ Args a) {
  using C = CfgQ<D>;
  constexpr int ST = C::ST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t sb = (raw_base + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw_base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (a.Sq + QROWS - 1) / QROWS;
  const int qt = nqt - 1 - (int)blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / a.group;
  const int q0 = qt * QROWS, q1 = min(q0 + QROWS, a.Sq);

  const uint32_t bar0 = sb + C::OFF_BAR;
  const uint32_t q_full = bar0;
  auto st_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto st_free = [&](int s) { return bar0 + 8u * (1 + ST + s); };
  constexpr int NSB = C::NSB;
  auto s_full = [&](int i) { return bar0 + 8u * (1 + 2 * ST + i); };
  auto s_free = [&](int i) { return bar0 + 8u * (1 + 2 * ST + NSB + i); };
  const uint32_t ds_full = bar0 + 8u * (1 + 2 * ST + 2 * NSB);
  auto ds_free = [&](int buf) { return bar0 + 8u * (2 + 2 * ST + 2 * NSB + buf); };
  const uint32_t acc_done = bar0 + 8u * (2 + 2 * ST + 2 * NSB + C::DB);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sp + C::OFF_TMEMPTR);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(st_full(s), 1);
      mbar_init(st_free(s), 1);
    }
    for (int i = 0; i < NSB; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), 8);  // one arrival per elementwise warp
    }
    mbar_init(ds_full, 8);
    for (int q = 0; q < C::DB; ++q) mbar_init(ds_free(q), 1);
    mbar_init(acc_done, 1);
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

  int j_lo, j_hi;
  band_tile_range(a.mask, q0, q1, a.Skv, KT, &j_lo, &j_hi);
  if (a.doc_q_jr) {
    static_assert(QROWS == kDocTile && kDocTile % KT == 0, "document tiles vs q / kv tiles");
    const int2 r = a.doc_q_jr[(long long)b * a.nq_doc + qt];
    j_lo = max(j_lo, r.x * (kDocTile / KT));
    j_hi = max(j_lo, min(j_hi, r.y * (kDocTile / KT)));
  }
  auto state_of = [&](int j) {
    return tile_state(a.mask, a.doc_q_tiles, a.doc_kv_tiles, a.nq_doc, a.nk_doc, b, q0, q1, j * KT,
                      min((j + 1) * KT, a.Skv), KT);
  };

  if (warp == 8) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_expect_tx(q_full, 2 * C::Q_BYTES);
      for (int c = 0; c < C::KCH; ++c) {
        tma_load_4d(sb + C::OFF_Q + c * QROWS * 128, &tm_q, q_full, c * 64, q0, hq, b);
        tma_load_4d(sb + C::OFF_DO + c * QROWS * 128, &tm_do, q_full, c * 64, q0, hq, b);
      }
      int i = 0;
      for (int j = j_lo; j < j_hi; ++j) {
        if (state_of(j) == kSkip) continue;
        const int s = i % ST;
        if (!mbar_wait(st_free(s), ((i / ST) & 1) ^ 1, kStatusTimeoutLoad)) break;
        const uint32_t base = sb + C::OFF_ST + s * 2 * C::KV_BYTES;
        mbar_expect_tx(st_full(s), 2 * C::KV_BYTES);
        for (int c = 0; c < C::KCH; ++c) {
          tma_load_4d(base + c * KT * 128, &tm_k, st_full(s), c * 64, j * KT, hkv, b);
          tma_load_4d(base + C::KV_BYTES + c * KT * 128, &tm_v, st_full(s), c * 64, j * KT, hkv, b);
        }
        ++i;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr int FMT = BF16 ? 1 : 0;
      constexpr uint32_t ID_S = idesc_f16(128, KT, FMT, 0, 0);
      constexpr uint32_t ID_Q = idesc_f16(128, D, FMT, 0, 1);
      bool ok = mbar_wait(q_full, 0, kStatusTimeoutMma);
      auto issue_dq = [&](int j) -> bool {
        const int s = j % ST;
        const uint32_t base = sb + C::OFF_ST + s * 2 * C::KV_BYTES;
        if (!mbar_wait(ds_full, j & 1, kStatusTimeoutMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < KT / 16; ++k) {
          const uint64_t da =
              sdesc_sw128(sb + C::OFF_DS + (j % C::DB) * C::DS_BYTES + (k >> 2) * QROWS * 128 + (k & 3) * 32, 16, 1024);
          const uint64_t kb = sdesc_sw128(base + k * 16 * 128, KT * 128, 1024);
          umma_f16(tmem + C::COL_DQ, da, kb, ID_Q, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(st_free(s));
        umma_commit(ds_free(j % C::DB));
        return true;
      };
      int i = 0;
      for (int j = j_lo; ok && j < j_hi; ++j) {
        if (state_of(j) == kSkip) continue;
        const int s = i % ST;
        ok = mbar_wait(st_full(s), (i / ST) & 1, kStatusTimeoutMma) &&
             mbar_wait(s_free(i % NSB), ((i / NSB) & 1) ^ 1, kStatusTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t base = sb + C::OFF_ST + s * 2 * C::KV_BYTES;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k & 3) * 32;
          const uint64_t qa = sdesc_sw128(sb + C::OFF_Q + (k >> 2) * QROWS * 128 + off, 16, 1024);
          const uint64_t oa = sdesc_sw128(sb + C::OFF_DO + (k >> 2) * QROWS * 128 + off, 16, 1024);
          const uint64_t kb = sdesc_sw128(base + (k >> 2) * KT * 128 + off, 16, 1024);
          const uint64_t vb = sdesc_sw128(base + C::KV_BYTES + (k >> 2) * KT * 128 + off, 16, 1024);
          umma_f16(tmem + C::COL_S + (i % NSB) * KT, qa, kb, ID_S, k > 0 ? 1u : 0u);
          umma_f16(tmem + C::COL_DP + (i % NSB) * KT, oa, vb, ID_S, k > 0 ? 1u : 0u);
        }
        umma_commit(s_full(i % NSB));
        if (i > 0) ok = issue_dq(i - 1);
        ++i;
      }
      if (ok && i > 0) ok = issue_dq(i - 1);
      umma_commit(acc_done);
    }
  } else if (warp < 8) {
    const int r = threadIdx.x & 127;  // q row within the tile == TMEM lane
    const int half = warp >> 2;       // columns [KT/2*half, KT/2*(half+1)) of each kv tile
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const bool row_ok = q0 + r < a.Sq;
    const long long ridx = ((long long)b * a.Hq + hq) * a.Sq_pad + q0 + r;
    const float lse2 = a.lse2[ridx], delta = a.delta[ridx];
    uint8_t* DS = sp + C::OFF_DS;
    // Full tiles: t = s*sl2 - slope*(d0 - c) - lse2 (d0 = q - kv(column 0) >= c
    // under a causal band), i.e. a per-row constant plus slope*c.
    const float slope_l2 = a.mask.alibi_slopes ? a.mask.alibi_slopes[hq] * kLog2e : 0.f;
    const bool fast_mask = ATTN_BWD_FAST_FULL && (!a.mask.alibi_slopes || (a.mask.has_band && a.mask.band_lo >= 0));
    const long long qg_row = a.mask.q_offset + q0 + r;
    const unsigned long long sl2x2 = f2_pack(a.sl2, a.sl2), delta2 = f2_pack(delta, delta);
    const unsigned long long step2 = f2_pack(8.f * slope_l2, 8.f * slope_l2);
    int i = 0;
    bool ok = true;
    for (int j = j_lo; j < j_hi; ++j) {
      const int st = state_of(j);
      if (st == kSkip) continue;
      ok = __all_sync(0xffffffffu, mbar_wait(s_full(i % NSB), (i / NSB) & 1, kStatusTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      constexpr int HC = KT / 2;  // columns per thread, processed 32 at a time
      if (i >= C::DB) {  // this dS buffer was last read by the dQ GEMM of iteration i - DB
        ok = __all_sync(0xffffffffu,
                        mbar_wait(ds_free(i % C::DB), ((i / C::DB) - 1) & 1, kStatusTimeoutSoftmax));
        if (!ok) break;
      }
      uint8_t* dsb = DS + (i % C::DB) * C::DS_BYTES;
#pragma unroll 1
      for (int cc = 0; cc < HC / 32; ++cc) {
        float sc[32], dp[32];
        tmem_ld32(tmem + lane_base + C::COL_S + (i % NSB) * KT + half * HC + cc * 32,
                  *reinterpret_cast<uint32_t(*)[32]>(sc));
        tmem_ld32(tmem + lane_base + C::COL_DP + (i % NSB) * KT + half * HC + cc * 32,
                  *reinterpret_cast<uint32_t(*)[32]>(dp));
        tmem_wait_ld();
        if (cc == HC / 32 - 1) {
          tc_fence_before();
          mbar_arrive_warp(s_free(i % NSB));
        }
        const int c0 = j * KT + half * HC + cc * 32;
        if (st == kFull && fast_mask) {
          const float rowc = -slope_l2 * (float)clamp_i32(qg_row - (a.mask.kv_offset + c0)) - lse2;
          unsigned long long addv[4];  // rowc + slope*c for the column pairs, 4 independent chains
#pragma unroll
          for (int q = 0; q < 4; ++q)
            addv[q] = f2_pack(fmaf(slope_l2, (float)(2 * q), rowc), fmaf(slope_l2, (float)(2 * q + 1), rowc));
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const int q = (c >> 1) & 3;
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(sc[c], sc[c + 1]), sl2x2, addv[q]), x0, x1);
            addv[q] = f2_add(addv[q], step2);
            const unsigned long long p2 = f2_pack(ex2(x0), ex2(x1));
            f2_unpack(f2_mul(p2, f2_sub(f2_pack(dp[c], dp[c + 1]), delta2)), dp[c], dp[c + 1]);
          }
        } else {
          const RowCtx rc = make_row_ctx(a.mask, a.sl2, b, hq, q0 + r, c0, max(0, min(32, a.Skv - c0)), false);
          transform_row<32>(sc, rc, st == kPartial);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float p = ex2(sc[c] - lse2);
            dp[c] = p * (dp[c] - delta);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = u * 8, ca = half * HC + cc * 32 + c;  // column within the KT-wide tile
          uint4 w;
          w.x = pack2(dp[c], dp[c + 1], BF16); w.y = pack2(dp[c + 2], dp[c + 3], BF16);
          w.z = pack2(dp[c + 4], dp[c + 5], BF16); w.w = pack2(dp[c + 6], dp[c + 7], BF16);
          *reinterpret_cast<uint4*>(dsb + (ca >> 6) * QROWS * 128 + r * 128 + ((((ca & 63) >> 3) ^ (r & 7)) << 4)) = w;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive_warp(ds_full);
      ++i;
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_done, 0, kStatusTimeoutSoftmax));
    if (ok) {
      tc_fence_after();
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* dqr = reinterpret_cast<T*>(a.dq) + b * a.dq_s[0] + hq * a.dq_s[1] + (long long)(q0 + r) * a.dq_s[2];
#pragma unroll
      for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
        uint32_t o[32];
        if (i > 0) {
          tmem_ld32(tmem + lane_base + C::COL_DQ + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack2(__uint_as_float(o[v * 8 + 0]) * a.scale, __uint_as_float(o[v * 8 + 1]) * a.scale, BF16);
            w.y = pack2(__uint_as_float(o[v * 8 + 2]) * a.scale, __uint_as_float(o[v * 8 + 3]) * a.scale, BF16);
            w.z = pack2(__uint_as_float(o[v * 8 + 4]) * a.scale, __uint_as_float(o[v * 8 + 5]) * a.scale, BF16);
            w.w = pack2(__uint_as_float(o[v * 8 + 6]) * a.scale, __uint_as_float(o[v * 8 + 7]) * a.scale, BF16);
            *reinterpret_cast<uint4*>(dqr + c * 32 + v * 8) = w;
          }
        }
      }
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

// dQ = scale * dq_acc^T (fused path with a [B][H][D][S_pad] accumulator):
// one 64-row q tile per block, transposed through shared memory.
template <typename T, int D>
__global__ void dq_convert_t_kernel(const float* acc, T* dq, long long s0, long long s1, long long s2, int H,
                                    int S, int S_pad, float scale) {
  __shared__ float tile[D][65];
  const int q0 = blockIdx.x * 64, h = blockIdx.y, b = blockIdx.z;
  const float* src = acc + ((long long)b * H + h) * D * S_pad + q0;
  for (int i = threadIdx.x; i < D * 64; i += blockDim.x) {
    const int d = i / 64, q = i % 64;
    tile[d][q] = src[(long long)d * S_pad + q];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * (D / 2); i += blockDim.x) {
    const int q = i / (D / 2), d = 2 * (i % (D / 2));
    if (q0 + q < S)
      *reinterpret_cast<uint32_t*>(dq + b * s0 + h * s1 + (long long)(q0 + q) * s2 + d) =
          pack2(tile[d][q] * scale, tile[d + 1][q] * scale, std::is_same<T, __nv_bfloat16>::value);
  }
}

// dQ = scale * dq_acc (fused path), one warp per row, 4 columns per lane.
template <typename T>
__global__ void dq_convert_kernel(const float* acc, T* dq, long long s0, long long s1, long long s2, int H,
                                  int S, int S_pad, int D, float scale) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  if (row >= S) return;
  const float* src = acc + (((long long)b * H + h) * S_pad + row) * D;
  T* dst = dq + b * s0 + h * s1 + (long long)row * s2;
  for (int e = lane * 4; e < D; e += 128) {
    const float4 x = *reinterpret_cast<const float4*>(src + e);
    uint2 w;
    w.x = pack2(x.x * scale, x.y * scale, std::is_same<T, __nv_bfloat16>::value);
    w.y = pack2(x.z * scale, x.w * scale, std::is_same<T, __nv_bfloat16>::value);
    *reinterpret_cast<uint2*>(dst + e) = w;
  }
}

// delta = rowsum(dO * O), lse2 = lse * log2(e) into [B][H][S_pad] with
// padded rows (+inf, 0), and zeroes the row of the fused-dQ accumulator when
// there is one.  D/8 lanes share a row (16 bytes each) and every warp keeps
// kPasses rows-per-pass of loads in flight before reducing.
template <typename T, int D>
__global__ void __launch_bounds__(256) prep_rows_kernel(const T* out, const T* dout, long long os0, long long os1,
                                                        long long os2, long long ds0, long long ds1, long long ds2,
                                                        const float* lse, float* delta, float* lse2, int H, int S,
                                                        int S_pad, float* dq_acc) {
  constexpr int L = D / 8;          // lanes per row
  constexpr int RPP = 32 / L;       // rows per warp pass
  constexpr int kPasses = 4;
  constexpr int RPW = RPP * kPasses;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int row0 = (blockIdx.x * (blockDim.x >> 5) + warp) * RPW + lane / L;
  const int cl = (lane % L) * 8;
  uint4 ov[kPasses], dv[kPasses];
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int row = row0 + p * RPP;
    if (row < S) {
      ov[p] = *reinterpret_cast<const uint4*>(out + b * os0 + h * os1 + (long long)row * os2 + cl);
      dv[p] = *reinterpret_cast<const uint4*>(dout + b * ds0 + h * ds1 + (long long)row * ds2 + cl);
    } else {
      ov[p] = dv[p] = make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const T* oh = reinterpret_cast<const T*>(&ov[p]);
    const T* dh = reinterpret_cast<const T*>(&dv[p]);
    float acc = 0.f;
#pragma unroll
    for (int x = 0; x < 8; ++x) acc = fmaf(to_f32(oh[x]), to_f32(dh[x]), acc);
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const int row = row0 + p * RPP;
    if (dq_acc && row < S_pad) {  // zero this row of the fused-dQ accumulator ([row][D] fp32)
      float4* z = reinterpret_cast<float4*>(dq_acc + (((long long)b * H + h) * S_pad + row) * D + cl);
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (lane % L == 0 && row < S_pad) {
      const long long idx = ((long long)b * H + h) * S_pad + row;
      if (row < S) {
        delta[idx] = acc;
        const float l = lse[((long long)b * H + h) * S + row];
        lse2[idx] = (l == -INFINITY) ? INFINITY : l * kLog2e;
      } else {
        delta[idx] = 0.f;
        lse2[idx] = INFINITY;
      }
    }
  }
}
constexpr int kPrepRowsPerBlock = 8 * 4 * 32;  // 8 warps x 4 passes x 32 lanes, divided by D/8 lanes per row

}  // namespace bwd
}  // namespace attnb200
