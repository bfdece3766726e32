// Flash-attention forward for sm_100a: TMA-staged Q/K/V, tcgen05.mma with the
// S and O accumulators in TMEM, online softmax in registers.
//
// Replaces the forward of flash_attention / pallas_flash_attention
// (attnax/kernels/attention.py:209-283, attnax/kernels/pallas.py:118-244):
// same recurrence as memory_efficient_attention (attention.py:145-199), with
// fully masked KV tiles skipped and the mask/ALiBi/bias terms applied in the
// softmax warps.
//
// CTA = one 128-row query tile of one (batch, query head).  Warp roles:
//   warps 0-3  softmax + O correction + epilogue (thread t owns query row t,
//              which is TMEM lane t)
//   warp 4     TMA producer (Q once, then K/V tiles into a STAGES-deep ring)
//   warp 5     TMEM allocator + single-thread tcgen05.mma issuer
// TMEM columns: S double buffer at [0,128) and [128,256), O at [256, 256+D).
// Issue order on the tensor core: S0, S1, PV0, S2, PV1, ... so the next
// QK^T runs while the softmax warps work on the current tile.
#include <cfloat>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace attnb200 {
namespace fwd {

constexpr int BM = 128, BN = 128;
constexpr int kThreads = 192;

template <int D>
struct Cfg {
  static constexpr int KCH = D / 64;  // 64-element (128-byte) swizzle chunks along head_dim
  static constexpr int STAGES = (D == 64) ? 4 : 2;
  static constexpr int Q_BYTES = KCH * BM * 128;
  static constexpr int KV_BYTES = KCH * BN * 128;
  static constexpr int P_BYTES = (BN / 64) * BM * 128;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_P = OFF_V + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  static constexpr int NBAR = 1 + 3 * STAGES + 2 + 2 + 2;
  static constexpr int OFF_TMEMPTR = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_TMEMPTR + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 256;
};

struct Args {
  int B, Hq, Hkv, Sq, Skv, group, nq_tiles;
  float sl2;  // softmax scale * log2(e)
  void* out;
  long long o_s0, o_s1, o_s2;
  float* lse;
  attn_mask_t mask;
  const int2* doc_q_tiles;
  const int2* doc_kv_tiles;
  const int2* doc_jrange;  // per q tile: kv tiles whose document ids can match (or null)
  int nq_doc, nk_doc;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Args a) {
  using C = Cfg<D>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t sb = (raw_base + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw_base);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = a.nq_tiles - 1 - (int)blockIdx.x;  // heavy (late) tiles first
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / a.group;
  const int q0 = qt * BM, q1 = min(q0 + BM, a.Sq);

  const uint32_t bar0 = sb + C::OFF_BAR;
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + S + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (1 + 2 * S + s); };
  auto s_full = [&](int i) { return bar0 + 8u * (1 + 3 * S + i); };
  auto s_free = [&](int i) { return bar0 + 8u * (3 + 3 * S + i); };
  const uint32_t p_full = bar0 + 8u * (5 + 3 * S);
  const uint32_t pv_done = bar0 + 8u * (6 + 3 * S);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sp + C::OFF_TMEMPTR);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), 4);  // one arrival per softmax warp
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int j_lo, j_hi;
  band_tile_range(a.mask, q0, q1, a.Skv, BN, &j_lo, &j_hi);
  if (a.doc_jrange) {
    static_assert(BM == kDocTile, "one document tile per q tile");
    const int2 r = a.doc_jrange[(long long)b * a.nq_doc + q0 / kDocTile];
    j_lo = max(j_lo, r.x);
    j_hi = max(j_lo, min(j_hi, r.y));
  }
  auto state_of = [&](int j) {
    return tile_state(a.mask, a.doc_q_tiles, a.doc_kv_tiles, a.nq_doc, a.nk_doc, b, q0, q1, j * BN,
                      min((j + 1) * BN, a.Skv), BN);
  };

  if (warp == 4) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_expect_tx(q_full, C::Q_BYTES);
      for (int c = 0; c < C::KCH; ++c)
        tma_load_4d(sb + C::OFF_Q + c * BM * 128, &tm_q, q_full, c * 64, q0, hq, b);
      int i = 0;
      for (int j = j_lo; j < j_hi; ++j) {
        if (state_of(j) == kSkip) continue;
        const int s = i % S;
        if (!mbar_wait(kv_empty(s), ((i / S) & 1) ^ 1, kStatusTimeoutLoad)) break;
        mbar_expect_tx(k_full(s), C::KV_BYTES);
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sb + C::OFF_K + s * C::KV_BYTES + c * BN * 128, &tm_k, k_full(s), c * 64,
                      j * BN, hkv, b);
        mbar_expect_tx(v_full(s), C::KV_BYTES);
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sb + C::OFF_V + s * C::KV_BYTES + c * BN * 128, &tm_v, v_full(s), c * 64,
                      j * BN, hkv, b);
        ++i;
      }
    }
  } else if (warp == 5) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr int FMT = BF16 ? 1 : 0;
      constexpr uint32_t IDESC_QK = idesc_f16(128, BN, FMT, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_f16(128, D, FMT, 0, 1);
      bool ok = mbar_wait(q_full, 0, kStatusTimeoutMma);
      auto issue_pv = [&](int jj) -> bool {
        const int s = jj % S;
        if (!mbar_wait(v_full(s), (jj / S) & 1, kStatusTimeoutMma)) return false;
        if (!mbar_wait(p_full, jj & 1, kStatusTimeoutMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t ad = sdesc_sw128(sb + C::OFF_P + (k >> 2) * BM * 128 + (k & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sb + C::OFF_V + s * C::KV_BYTES + k * 16 * 128, BN * 128, 1024);
          umma_f16(tmem + C::O_COL, ad, bd, IDESC_PV, (jj > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(kv_empty(s));
        umma_commit(pv_done);
        return true;
      };
      int i = 0;
      for (int j = j_lo; ok && j < j_hi; ++j) {
        if (state_of(j) == kSkip) continue;
        const int s = i % S;
        ok = mbar_wait(k_full(s), (i / S) & 1, kStatusTimeoutMma) &&
             mbar_wait(s_free(i & 1), ((i >> 1) & 1) ^ 1, kStatusTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)((i & 1) * BN);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t ad = sdesc_sw128(sb + C::OFF_Q + (k >> 2) * BM * 128 + (k & 3) * 32, 16, 1024);
          const uint64_t bd =
              sdesc_sw128(sb + C::OFF_K + s * C::KV_BYTES + (k >> 2) * BN * 128 + (k & 3) * 32, 16, 1024);
          umma_f16(d, ad, bd, IDESC_QK, k > 0 ? 1u : 0u);
        }
        umma_commit(s_full(i & 1));
        if (i > 0) ok = issue_pv(i - 1);
        ++i;
      }
      if (ok && i > 0) issue_pv(i - 1);
    }
  } else {
    // ------------------------------------------------------------- softmax --
    const int r = threadIdx.x;  // query row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float m_run = -FLT_MAX, l_run = 0.f;
    int i = 0;
    bool ok = true;
    uint8_t* P = sp + C::OFF_P;
    for (int j = j_lo; j < j_hi; ++j) {
      const int st = state_of(j);
      if (st == kSkip) continue;
      ok = __all_sync(0xffffffffu, mbar_wait(s_full(i & 1), (i >> 1) & 1, kStatusTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tmem_ld32(tmem + lane_base + (uint32_t)((i & 1) * BN + c * 32),
                  *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive_warp(s_free(i & 1));

      const int k0 = j * BN;
      const RowCtx rc = make_row_ctx(a.mask, a.sl2, b, hq, q0 + r, k0, min(BN, a.Skv - k0), false);
      transform_row<BN>(s, rc, st == kPartial);
      float mx = m_run;
#pragma unroll
      for (int c = 0; c < BN; ++c) mx = fmaxf(mx, s[c]);
      const float alpha = ex2(m_run - mx);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        s[c] = ex2(s[c] - mx);
        sum += s[c];
      }
      l_run = l_run * alpha + sum;
      m_run = mx;

      // PV of the previous tile must be done before P is overwritten and O rescaled.
      if (i > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (i - 1) & 1, kStatusTimeoutSoftmax));
        if (!ok) break;
        tc_fence_after();
      }
      // P (bf16/f16) into the K-major 128B-swizzled tile the PV MMA reads.
#pragma unroll
      for (int u = 0; u < BN / 8; ++u) {
        const int c = u * 8;
        uint4 val;
        val.x = pack2(s[c + 0], s[c + 1], BF16);
        val.y = pack2(s[c + 2], s[c + 3], BF16);
        val.z = pack2(s[c + 4], s[c + 5], BF16);
        val.w = pack2(s[c + 6], s[c + 7], BF16);
        const int chunk = c >> 6, unit = (c & 63) >> 3;
        *reinterpret_cast<uint4*>(P + chunk * BM * 128 + r * 128 + ((unit ^ (r & 7)) << 4)) = val;
      }
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          const uint32_t ta = tmem + lane_base + C::O_COL + c * 32;
          tmem_ld32(ta, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(ta, o);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive_warp(p_full);
      ++i;
    }
    // ------------------------------------------------------------ epilogue --
    if (ok && i > 0) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (i - 1) & 1, kStatusTimeoutSoftmax));
    if (ok) {
      tc_fence_after();
      const bool row_ok = (q0 + r) < a.Sq;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = reinterpret_cast<T*>(a.out) + (long long)b * a.o_s0 + (long long)hq * a.o_s1 +
                (long long)(q0 + r) * a.o_s2;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (i > 0) {
          tmem_ld32(tmem + lane_base + C::O_COL + c * 32, o);
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
      if (row_ok && a.lse) {
        a.lse[((long long)b * a.Hq + hq) * a.Sq + q0 + r] =
            (m_run == -FLT_MAX || l_run <= 0.f) ? -INFINITY : (m_run + lg2(l_run)) * kLn2;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fwd
}  // namespace attnb200
