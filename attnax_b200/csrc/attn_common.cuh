// Mask semantics shared by every attention kernel.
//
// The flattened mask (attn_mask_t) reproduces the reference's composed
// ScoreMods (attnax/kernels/score_mods.py) and `mask=` argument:
//   causal_mod          keep kv <= q                    (score_mods.py:100-102)
//   sliding_window_mod  keep kv <= q and q - kv < W      (:139-141), or |q-kv| < W (:142)
//   prefix_lm_mod       keep kv < prefix[b] or kv <= q   (:171-174)
//   document_mask_mod   keep ids[b,q] == ids[b,kv]       (:195-209)
//   alibi_mod           s - slope[h] * |q - kv|          (:76-79)
//   additive_bias_mod   s + bias                         (:235)
//   mask=               where(mask, s, finfo.min)        (attention.py:60-62)
// Dropped scores become -FLT_MAX in the log2 domain (the reference's
// finfo.min), so a row with nothing kept still averages V uniformly; key
// columns past the end of the sequence are -inf and never count.
#pragma once
#include <cfloat>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/attnb200.h"

namespace attnb200 {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum TileState : int { kSkip = 0, kPartial = 1, kFull = 2 };

// Tile size of the document-id range tables (both q and kv tiles).
constexpr int kDocTile = 128;

__host__ __device__ inline long long ll_min(long long a, long long b) { return a < b ? a : b; }

// Pool page that block-table entry `e` selects in a pool of `num_blocks`
// pages, read as JAX's array indexing reads pool[block_ids]
// (attnax/paged_cache.py:222-230): a negative entry counts from the end of
// the pool, then the index is clamped into [0, num_blocks).
__host__ __device__ inline long long paged_phys_page(long long e, int num_blocks) {
  if (e < 0) e += num_blocks;
  return e < 0 ? 0 : (e >= num_blocks ? (long long)num_blocks - 1 : e);
}
__host__ __device__ inline long long ll_max(long long a, long long b) { return a > b ? a : b; }

// Classifies the tile [q0,q1) x [k0,k1) of batch b (local positions).
// doc_q_tiles/doc_kv_tiles hold (min,max) ids per kDocTile-row tile; when
// they are null a document mask makes every tile partial.
__host__ __device__ inline int tile_state(const attn_mask_t& m, const int2* doc_q_tiles,
                                          const int2* doc_kv_tiles, int nq_doc, int nk_doc, int b,
                                          int q0, int q1, int k0, int k1, int bn) {
  int st = kFull;
  if (k1 - k0 < bn) st = kPartial;
  const long long qlo = m.q_offset + q0, qhi = m.q_offset + q1 - 1;
  const long long klo = m.kv_offset + k0, khi = m.kv_offset + k1 - 1;
  if (m.has_band) {
    const long long dmin = qlo - khi, dmax = qhi - klo;
    if (dmax < m.band_lo || dmin > m.band_hi) return kSkip;
    if (!(dmin >= m.band_lo && dmax <= m.band_hi)) st = kPartial;
  }
  if (m.prefix_len) {
    const long long pref = m.prefix_len[b];
    if (klo >= pref && klo > qhi) return kSkip;
    if (!(khi < pref || khi <= qlo)) st = kPartial;
  }
  if (m.doc_q) {
    // a tile inside one kDocTile tile uses that tile's (min, max) ids (a
    // superset of its own: skip only if disjoint, full only if one document)
    if (doc_q_tiles && doc_kv_tiles && q0 / kDocTile == (q1 - 1) / kDocTile &&
        k0 / kDocTile == (k1 - 1) / kDocTile) {
      const int2 a = doc_q_tiles[(long long)b * nq_doc + q0 / kDocTile];
      const int2 c = doc_kv_tiles[(long long)b * nk_doc + k0 / kDocTile];
      if (a.y < c.x || c.y < a.x) return kSkip;
      if (!(a.x == a.y && c.x == c.y && a.x == c.x)) st = kPartial;
    } else {
      st = kPartial;
    }
  }
  if (m.bool_mask || m.bias) st = kPartial;
  return st;
}

// Local kv-tile index range [lo, hi) that the band allows for rows [q0, q1).
__host__ __device__ inline void band_tile_range(const attn_mask_t& m, int q0, int q1, int seq_kv,
                                                int bn, int* lo, int* hi) {
  const int nk = (seq_kv + bn - 1) / bn;
  *lo = 0;
  *hi = nk;
  if (m.has_band) {
    const long long qlo = m.q_offset + q0, qhi = m.q_offset + q1 - 1;
    long long c_lo = qlo - m.band_hi - m.kv_offset;   // smallest local kv col kept
    long long c_hi = qhi - m.band_lo - m.kv_offset;   // largest
    c_lo = ll_max(c_lo, 0);
    c_hi = ll_min(c_hi, (long long)seq_kv - 1);
    if (c_hi < c_lo) {
      *lo = *hi = 0;
      return;
    }
    *lo = (int)(c_lo / bn);
    *hi = (int)(c_hi / bn) + 1;
  }
}

__device__ __forceinline__ float load_bias(const void* p, attn_dtype_t dt, long long idx) {
  if (dt == ATTN_F32) return __ldg(reinterpret_cast<const float*>(p) + idx);
  if (dt == ATTN_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
  return __half2float(reinterpret_cast<const __half*>(p)[idx]);
}

// Element transform for one score: raw q.k -> log2-domain score t, with
// every mask and additive term.  `row`/`col` are local positions.
__device__ __forceinline__ float mask_score(const attn_mask_t& m, float raw, float sl2,
                                            float slope_l2, int b, int h, int row, int col,
                                            int seq_kv, bool partial) {
  const long long qg = m.q_offset + row, kvg = m.kv_offset + col;
  float t = raw * sl2;
  if (m.alibi_slopes) t -= slope_l2 * fabsf((float)(int)(qg - kvg));
  if (!partial) return t;
  if (col >= seq_kv) return -INFINITY;
  bool keep = true;
  if (m.has_band) {
    const long long d = qg - kvg;
    keep = keep && d >= m.band_lo && d <= m.band_hi;
  }
  if (m.prefix_len) keep = keep && (kvg < (long long)m.prefix_len[b] || kvg <= qg);
  if (m.doc_q)
    keep = keep && (__ldg(m.doc_q + (long long)b * m.doc_q_bstride + qg) ==
                    __ldg(m.doc_kv + (long long)b * m.doc_kv_bstride + kvg));
  if (m.bool_mask)
    keep = keep && m.bool_mask[b * m.mask_strides[0] + h * m.mask_strides[1] +
                               row * m.mask_strides[2] + col * m.mask_strides[3]] != 0;
  if (m.bias)
    t += kLog2e * load_bias(m.bias, m.bias_dtype,
                            b * m.bias_strides[0] + h * m.bias_strides[1] +
                                row * m.bias_strides[2] + col * m.bias_strides[3]);
  return keep ? t : -FLT_MAX;
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// For every row tile t (of batch b): the range [lo, hi) of column tiles
// whose (min, max) id range overlaps row tile t's, from the per-tile ranges
// of doc_tile_range_kernel -- exact for sorted ids (packed documents), a
// superset otherwise.  One warp per row tile.
__global__ void doc_cross_range_kernel(const int2* row_tiles, int n_row, const int2* col_tiles, int n_col,
                                       int2* out) {
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  if (t >= n_row) return;
  const int2 r = row_tiles[(long long)b * n_row + t];
  int lo = 0x7fffffff, hi = -1;
  for (int c = lane; c < n_col; c += 32) {
    const int2 k = col_tiles[(long long)b * n_col + c];
    if (!(r.y < k.x || k.y < r.x)) {
      lo = min(lo, c);
      hi = max(hi, c);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (lane == 0) out[(long long)b * n_row + t] = hi < 0 ? make_int2(0, 0) : make_int2(lo, hi + 1);
}

// Launch order of the forward's two-query-tile CTAs under a document mask.
// Per batch, CTA indices are ranked by their kv-tile count (the document
// range of q_jr intersected with the band, summed over the CTA's two query
// tiles of bm == kDocTile rows), largest first, later tiles first on ties,
// so the longest CTAs start in the first wave.  One block per batch;
// n_ctas ints of dynamic shared memory.
__global__ void doc_cta_order_kernel(attn_mask_t m, const int2* q_jr, int nq_doc, int seq_q, int seq_kv, int bm,
                                     int bn, int n_ctas, int* order) {
  extern __shared__ int work[];
  const int b = blockIdx.x;
  for (int c = threadIdx.x; c < n_ctas; c += blockDim.x) {
    int tot = 0;
    for (int x = 0; x < 2; ++x) {
      const int q0 = c * 2 * bm + x * bm;
      if (q0 >= seq_q) continue;
      int lo, hi;
      band_tile_range(m, q0, min(q0 + bm, seq_q), seq_kv, bn, &lo, &hi);
      const int2 r = q_jr[(long long)b * nq_doc + q0 / kDocTile];
      tot += max(0, min(hi, r.y) - max(lo, r.x));
    }
    work[c] = tot;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < n_ctas; c += blockDim.x) {
    const int wc = work[c];
    int rank = 0;
    for (int o = 0; o < n_ctas; ++o) rank += (work[o] > wc) || (work[o] == wc && o > c);
    order[(long long)b * n_ctas + rank] = c;
  }
}

// (min, max) of document ids over kDocTile-row tiles of global positions
// offset + [t*kDocTile, min((t+1)*kDocTile, len)).
__global__ void doc_tile_range_kernel(const int32_t* ids, long long bstride, long long offset,
                                      int len, int ntiles, int2* out) {
  const int t = blockIdx.x, b = blockIdx.y;
  int lo = 0x7fffffff, hi = -0x7fffffff - 1;
  for (int i = t * kDocTile + threadIdx.x; i < min((t + 1) * kDocTile, len); i += blockDim.x) {
    const int v = ids[(long long)b * bstride + offset + i];
    lo = min(lo, v);
    hi = max(hi, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  __shared__ int slo[32], shi[32];
  const int w = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) {
    slo[w] = lo;
    shi[w] = hi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)blockDim.x / 32; ++i) {
      lo = min(lo, slo[i]);
      hi = max(hi, shi[i]);
    }
    out[(long long)b * ntiles + t] = make_int2(lo, hi);
  }
}

}  // namespace attnb200

namespace attnb200 {

// Per-thread constants for transforming one row of a score tile held in
// registers.  Columns are kv positions (forward, dQ) or q positions
// (dK/dV, "transposed").  d(c) = q - kv at column c = d0 + dstep * c.
struct RowCtx {
  float sl2;        // softmax scale * log2(e)
  float slope_l2;   // ALiBi slope * log2(e) (0 when no ALiBi)
  int d0, dstep;
  int ncols;        // columns < ncols are inside the sequence
  int band_lo, band_hi;
  int pref_cols;    // prefix: columns c < pref_cols are kept regardless of d (see make_row_ctx)
  int doc_fixed;    // document id of this row
  const int32_t* doc_cols;  // document ids indexed by column
  const uint8_t* bmask;     // bool mask at column 0, column stride bmask_cs
  long long bmask_cs;
  const void* bias;         // bias at column 0, column stride bias_cs
  long long bias_cs;
  attn_dtype_t bias_dtype;
  bool alibi, band, prefix, doc;
};

// Bits e (0..31) of a 32-column chunk with lo <= e <= hi (a keep mask of a
// boundary tile's columns under a band or prefix rule).
__device__ __forceinline__ uint32_t bit_range(long long lo, long long hi) {
  if (hi < 0 || lo > 31 || hi < lo) return 0u;
  const int l = lo < 0 ? 0 : (int)lo, h = hi > 31 ? 31 : (int)hi;
  return (0xffffffffu >> (31 - h)) & (0xffffffffu << l);
}

__device__ __forceinline__ int clamp_i32(long long x) {
  return (int)(x < -(1ll << 30) ? -(1ll << 30) : (x > (1ll << 30) ? (1ll << 30) : x));
}

// row/col0 are local positions of this thread's row and of column 0.
// transposed: the row is a kv position and columns are q positions.
__device__ __forceinline__ RowCtx make_row_ctx(const attn_mask_t& m, float sl2, int b, int hq,
                                               int row, int col0, int ncols, bool transposed) {
  RowCtx r;
  r.sl2 = sl2;
  r.alibi = m.alibi_slopes != nullptr;
  r.slope_l2 = r.alibi ? m.alibi_slopes[hq] * kLog2e : 0.f;
  const long long qg0 = m.q_offset + (transposed ? col0 : row);
  const long long kg0 = m.kv_offset + (transposed ? row : col0);
  r.d0 = clamp_i32(qg0 - kg0);
  r.dstep = transposed ? 1 : -1;
  r.ncols = ncols;
  r.band = m.has_band != 0;
  r.band_lo = clamp_i32(m.has_band ? m.band_lo : -(1ll << 40));
  r.band_hi = clamp_i32(m.has_band ? m.band_hi : (1ll << 40));
  r.prefix = m.prefix_len != nullptr;
  r.pref_cols = 0;
  if (r.prefix) {
    const long long pref = m.prefix_len[b];
    // kept when kv < pref: forward columns c < pref - kg0; transposed: all or none
    r.pref_cols = transposed ? (kg0 < pref ? (1 << 30) : 0) : clamp_i32(pref - kg0);
  }
  r.doc = m.doc_q != nullptr;
  r.doc_fixed = 0;
  r.doc_cols = nullptr;
  if (r.doc) {
    if (transposed) {
      r.doc_fixed = m.doc_kv[(long long)b * m.doc_kv_bstride + kg0];
      r.doc_cols = m.doc_q + (long long)b * m.doc_q_bstride + qg0;
    } else {
      r.doc_fixed = m.doc_q[(long long)b * m.doc_q_bstride + qg0];
      r.doc_cols = m.doc_kv + (long long)b * m.doc_kv_bstride + kg0;
    }
  }
  const int qrow = transposed ? col0 : row, kcol = transposed ? row : col0;
  r.bmask = nullptr;
  r.bmask_cs = 0;
  if (m.bool_mask) {
    r.bmask = m.bool_mask + b * m.mask_strides[0] + hq * m.mask_strides[1] +
              (long long)qrow * m.mask_strides[2] + (long long)kcol * m.mask_strides[3];
    r.bmask_cs = transposed ? m.mask_strides[2] : m.mask_strides[3];
  }
  r.bias = nullptr;
  r.bias_cs = 0;
  r.bias_dtype = m.bias_dtype;
  if (m.bias) {
    const long long off = b * m.bias_strides[0] + hq * m.bias_strides[1] +
                          (long long)qrow * m.bias_strides[2] + (long long)kcol * m.bias_strides[3];
    const int es = m.bias_dtype == ATTN_F32 ? 4 : 2;
    r.bias = reinterpret_cast<const char*>(m.bias) + off * es;
    r.bias_cs = transposed ? m.bias_strides[2] : m.bias_strides[3];
  }
  return r;
}

// Raw q.k scores -> log2-domain masked scores, for N register-resident
// columns.  Each feature is its own branch-free unrolled loop so the common
// (full-tile) path stays short.
template <int N>
__device__ __forceinline__ void transform_row(float (&s)[N], const RowCtx& r, bool partial) {
  if (r.alibi) {
    const float fd0 = (float)r.d0, fstep = (float)r.dstep;
#pragma unroll
    for (int c = 0; c < N; ++c) s[c] = fmaf(-r.slope_l2, fabsf(fmaf(fstep, (float)c, fd0)), s[c] * r.sl2);
  } else {
#pragma unroll
    for (int c = 0; c < N; ++c) s[c] *= r.sl2;
  }
  if (!partial) return;
  if (r.bias) {
    if (r.bias_dtype == ATTN_F32) {
      const float* p = reinterpret_cast<const float*>(r.bias);
#pragma unroll
      for (int c = 0; c < N; ++c)
        if (c < r.ncols) s[c] = fmaf(kLog2e, __ldg(p + c * r.bias_cs), s[c]);
    } else {
#pragma unroll
      for (int c = 0; c < N; ++c)
        if (c < r.ncols) s[c] = fmaf(kLog2e, load_bias(r.bias, r.bias_dtype, c * r.bias_cs), s[c]);
    }
  }
#pragma unroll
  for (int c = 0; c < N; ++c) {
    const int d = r.d0 + r.dstep * c;
    bool keep = !r.band || (d >= r.band_lo && d <= r.band_hi);
    if (r.prefix) keep = keep && (c < r.pref_cols || d >= 0);
    s[c] = c < r.ncols ? (keep ? s[c] : -FLT_MAX) : -INFINITY;
  }
  if (r.doc) {
#pragma unroll
    for (int c = 0; c < N; ++c)
      if (c < r.ncols && __ldg(r.doc_cols + c) != r.doc_fixed) s[c] = -FLT_MAX;
  }
  if (r.bmask) {
#pragma unroll
    for (int c = 0; c < N; ++c)
      if (c < r.ncols && r.bmask[c * r.bmask_cs] == 0) s[c] = -FLT_MAX;
  }
}

}  // namespace attnb200
