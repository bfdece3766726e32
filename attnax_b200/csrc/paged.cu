// Paged KV cache kernels (attnax/paged_cache.py, attnax/kernels/paged.py).
//
// Pool layout (the reference's): [num_blocks, block_size, heads_kv, head_dim],
// token-major with heads interleaved.  Logical token t of sequence s lives in
// physical page block_table[s, t / block_size], row t % block_size
// (paged_cache.py:222-230).  Table entries are read the way JAX's array
// indexing reads them there: a negative entry counts from the end of the
// pool, and the result is clamped into the pool (paged_phys_page).
//
// Decode is split-K: CTA = (split, kv head, sequence, row group).  A TMA
// warp streams each page's K and V slice ([block_size, head_dim] at a
// heads_kv*head_dim stride) into a 128B-swizzled shared-memory ring; four
// consumer warps take interleaved pages and keep an online softmax for the
// R query rows (the heads of the GQA group x query positions) that share
// the KV head, so K/V are read from HBM once per group instead of once per
// query head (the reference repeats K/V to Hq heads, paged.py:61-69).
// Partial (o, lse) per split are merged by paged_combine_kernel.
#include <cfloat>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace attnb200 {
namespace paged {

__device__ __forceinline__ long long phys_page(const int32_t* table_row, int i, int num_blocks) {
  return paged_phys_page(table_row[i], num_blocks);
}

// Logical page `lp` of a sequence bounded by its table row (max_blocks
// entries).  A length beyond max_blocks * block_size (which the reference's
// gather_kv cannot reshape) reads the row's last entry and leaves a notice.
__device__ __forceinline__ int table_col(int lp, int max_blocks) {
  if (lp < max_blocks) return lp;
  atomicCAS(&g_notice, 0, kNoticeTableOverrun);
  return max_blocks - 1;
}

// ------------------------------------------------------------ gather_kv ----
template <typename V>
__global__ void gather_kernel(const V* kp, const V* vp, int bs, int row_vecs,
                              const int32_t* table_row, int seq_len, int num_blocks, V* ko, V* vo) {
  const long long n = (long long)seq_len * row_vecs;
  for (long long x = blockIdx.x * (long long)blockDim.x + threadIdx.x; x < n;
       x += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(x / row_vecs), e = (int)(x % row_vecs);
    const long long src = (phys_page(table_row, t / bs, num_blocks) * bs + t % bs) * row_vecs + e;
    ko[x] = kp[src];
    vo[x] = vp[src];
  }
}

// ------------------------------------------------------------ append_kv ----
// Lowest logical page of the chunk that has no table slot (column past the
// row) or an unallocated one (-1): append_kv raises for both before writing.
__global__ void append_check_kernel(const int32_t* table_row, int max_blocks, int bs, int start, int chunk,
                                    int32_t* bad_slot) {
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < chunk; t += gridDim.x * blockDim.x) {
    const int logical = (start + t) / bs;
    if (logical >= max_blocks || table_row[logical] < 0) atomicMin(bad_slot, logical);
  }
}

// Per-token scatter.  A physical page at or past the end of the pool drops
// its rows, as JAX's .at[].set drops out-of-bounds updates.
template <typename V>
__global__ void append_kernel(V* kp, V* vp, int bs, int row_vecs, const int32_t* table_row, int num_blocks,
                              int max_blocks, int start, int chunk, const V* kn, const V* vn) {
  const long long n = (long long)chunk * row_vecs;
  for (long long x = blockIdx.x * (long long)blockDim.x + threadIdx.x; x < n;
       x += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(x / row_vecs), e = (int)(x % row_vecs);
    const int pos = start + t;
    if (pos / bs >= max_blocks) continue;
    const long long page = table_row[pos / bs];
    if (page < 0 || page >= num_blocks) continue;
    const long long dst = (page * bs + pos % bs) * row_vecs + e;
    kp[dst] = kn[x];
    vp[dst] = vn[x];
  }
}

// --------------------------------------------------------------- decode ----
#ifndef ATTN_PAGED_STAGES
#define ATTN_PAGED_STAGES 8  // pages in flight per CTA (3 CTAs per SM at page 16)
#endif
#ifndef ATTN_PAGED_CHUNK
#define ATTN_PAGED_CHUNK 2048  // tokens per split
#endif
constexpr int NW = 4;                  // consumer warps
constexpr int kThreads = (NW + 1) * 32;
constexpr int kChunkTokens = ATTN_PAGED_CHUNK;

template <int R>
struct DecCfg {
  static constexpr int STAGES = ATTN_PAGED_STAGES;
};

struct DecArgs {
  int num_seqs, Hq, Hkv, Sq, BS, max_blocks, num_blocks, group, rows, row_groups;
  int max_splits, chunk_tokens, box_bytes;  // bytes of one [BS x 64] swizzled box (1024-aligned)
  const void* q;
  const int32_t* block_table;
  const int32_t* seq_lens;
  float* part_o;    // [seq][Hq*Sq][max_splits][D]
  float* part_lse;  // [seq][Hq*Sq][max_splits]
  float sl2;
};

// Head dim fixed at 128 (two 64-wide swizzled boxes per page for K and V).
template <int R, bool BF16>
__global__ void __launch_bounds__(kThreads)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ DecArgs a) {
  constexpr int D = 128;
  constexpr int S = DecCfg<R>::STAGES;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  // Grid (kv head x row group, split, sequence): the CTAs of every kv head of
  // one split are adjacent in launch order, so they stream the same pages
  // (whose token rows hold all kv heads side by side) at the same time.
  const int split = blockIdx.y;
  const int hkv = blockIdx.x / a.row_groups, rg = blockIdx.x % a.row_groups;
  const int seq = blockIdx.z;
  const int ctx = a.seq_lens[seq];
  const int t0 = split * a.chunk_tokens;
  if (t0 >= ctx && !(split == 0 && ctx == 0)) return;
  const int t1 = min(ctx, t0 + a.chunk_tokens);
  const int p0 = t0 / a.BS, p1 = (t1 + a.BS - 1) / a.BS;
  const int npages = max(0, p1 - p0);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t sb = (raw_base + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw_base);
  const int page_bytes = 2 * a.box_bytes;          // K or V slice of one page
  const uint32_t k_base = sb, v_base = sb + S * page_bytes;
  const uint32_t bar0 = sb + 2 * S * page_bytes;
  uint8_t* scratch = sp + 2 * S * page_bytes + 2 * S * 8;  // p staging + merge
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (S + s); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NW) {
    if (lane == 0 && npages > 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int32_t* row = a.block_table + (long long)seq * a.max_blocks;
      for (int i = 0; i < npages; ++i) {
        const int s = i % S;
        if (!mbar_wait(empty(s), ((i / S) & 1) ^ 1, kStatusTimeoutLoad)) break;
        const int pid = (int)phys_page(row, table_col(p0 + i, a.max_blocks), a.num_blocks);
        mbar_expect_tx(full(s), 4 * a.BS * 128);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(k_base + s * page_bytes + c * a.box_bytes, &tm_k, full(s), c * 64, hkv, pid * a.BS);
          tma_load_3d(v_base + s * page_bytes + c * a.box_bytes, &tm_v, full(s), c * 64, hkv, pid * a.BS);
        }
      }
    }
    return;
  }

  // ---- consumers: warp w handles pages w, w+NW, ... of this split ----
  // Scores: 8 lanes per token (4 tokens per pass), lane sub = lane & 7 owns
  // features [16*sub, 16*sub+16).  Softmax: lane -> token lane & 15, rows
  // j = (lane >> 4) (mod 2).  P.V: lane owns features [4*lane, 4*lane+4).
  const int sub = lane & 7;
  float q[R][16];
  float o[R][4];
  const T* qbase = reinterpret_cast<const T*>(a.q);
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int row = rg * R + j;
    const bool okr = row < a.rows;
    const int g = okr ? row % a.group : 0, s_pos = okr ? row / a.group : 0;
    const int hq = hkv * a.group + g;
    const T* qr = qbase + (((long long)seq * a.Hq + hq) * a.Sq + s_pos) * D + sub * 16;
#pragma unroll
    for (int e = 0; e < 16; ++e) q[j][e] = okr ? to_f32(qr[e]) * a.sl2 : 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  }
  float* sc = reinterpret_cast<float*>(scratch) + warp * (16 * R + 3 * R);  // [16][R] scores/p
  float* al = sc + 16 * R;                                                  // [R] alpha
  float* ms = al + R;                                                       // [R] running max
  float* ls = ms + R;                                                       // [R] running sum
  if (lane < R) {
    ms[lane] = -FLT_MAX;
    ls[lane] = 0.f;
  }
  __syncwarp();
  bool ok = true;
  for (int i = warp; i < npages; i += NW) {
    const int s = i % S;
    ok = __all_sync(0xffffffffu, mbar_wait(full(s), (i / S) & 1, kStatusTimeoutSoftmax));
    if (!ok) break;
    const uint8_t* kst = sp + s * page_bytes;
    const uint8_t* vst = sp + S * page_bytes + s * page_bytes;
    const int page_tok0 = (p0 + i) * a.BS;
    for (int g16 = 0; g16 < a.BS; g16 += 16) {
#pragma unroll
      for (int pass = 0; pass < 4; ++pass) {
        const int tk = pass * 4 + (lane >> 3);
        const int r = g16 + tk;
        float dot[R];
#pragma unroll
        for (int j = 0; j < R; ++j) dot[j] = 0.f;
        if (r < a.BS) {
          const uint8_t* krow = kst + (sub >> 2) * a.box_bytes + r * 128;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int chunk = (sub & 3) * 2 + cc;
            const uint4 w = *reinterpret_cast<const uint4*>(krow + ((chunk ^ (r & 7)) << 4));
            const T* h8 = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float kv = to_f32(h8[e]);
#pragma unroll
              for (int j = 0; j < R; ++j) dot[j] = fmaf(q[j][cc * 8 + e], kv, dot[j]);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < R; ++j) {
          dot[j] += __shfl_xor_sync(0xffffffffu, dot[j], 1);
          dot[j] += __shfl_xor_sync(0xffffffffu, dot[j], 2);
          dot[j] += __shfl_xor_sync(0xffffffffu, dot[j], 4);
        }
        const bool valid = r < a.BS && page_tok0 + r >= t0 && page_tok0 + r < t1;
        if (sub == 0) {
#pragma unroll
          for (int j = 0; j < R; ++j) sc[tk * R + j] = valid ? dot[j] : -INFINITY;
        }
      }
      __syncwarp();
      {
        const int tk = lane & 15;
#pragma unroll
        for (int j0 = 0; j0 < R; j0 += 2) {
          const int j = j0 + (lane >> 4);
          if (j < R) {
            const float t = sc[tk * R + j];
            float mx = t;
#pragma unroll
            for (int x = 1; x < 16; x <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
            const float m_old = ms[j];
            const float m_new = fmaxf(m_old, mx);
            const float p = ex2(t - m_new);
            float sum = p;
#pragma unroll
            for (int x = 1; x < 16; x <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, x);
            sc[tk * R + j] = p;
            if (tk == 0) {
              const float alpha = ex2(m_old - m_new);
              al[j] = alpha;
              ls[j] = ls[j] * alpha + sum;
              ms[j] = m_new;
            }
          } else {
            // keep the shuffles convergent for R == 1
#pragma unroll
            for (int x = 1; x < 16; x <<= 1) (void)__shfl_xor_sync(0xffffffffu, 0.f, x);
#pragma unroll
            for (int x = 1; x < 16; x <<= 1) (void)__shfl_xor_sync(0xffffffffu, 0.f, x);
          }
        }
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const float alpha = al[j];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] *= alpha;
      }
      const int nt = min(16, a.BS - g16);
      const int box = lane >> 4, unit = (lane & 15) >> 1, subv = (lane & 1) * 8;
      for (int rr = 0; rr < nt; ++rr) {
        const int row = g16 + rr;
        // (P is 0 there, but a never-written slot may hold NaN: 0 * NaN)
        if (page_tok0 + row < t0 || page_tok0 + row >= t1) continue;
        const uint2 w = *reinterpret_cast<const uint2*>(vst + box * a.box_bytes + row * 128 +
                                                         ((unit ^ (row & 7)) << 4) + subv);
        const T* h4 = reinterpret_cast<const T*>(&w);
        float pr[R];
#pragma unroll
        for (int j = 0; j < R; ++j) pr[j] = sc[rr * R + j];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float vv = to_f32(h4[e]);
#pragma unroll
          for (int j = 0; j < R; ++j) o[j][e] = fmaf(pr[j], vv, o[j][e]);
        }
      }
      __syncwarp();
    }
    if (lane == 0) mbar_arrive(empty(s));
  }
  float m[R], l[R];
#pragma unroll
  for (int j = 0; j < R; ++j) {
    m[j] = ms[j];
    l[j] = ls[j];
  }
  // ---- merge the NW warps' partial states, write this split's (o, lse) ----
  float* mo = reinterpret_cast<float*>(scratch) + NW * (16 * R + 3 * R);  // [NW][R][D]
  float* ml = mo + NW * R * D;                                  // [NW][R][2]
#pragma unroll
  for (int j = 0; j < R; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) mo[(warp * R + j) * D + lane * 4 + e] = o[j][e];
    if (lane == 0) {
      ml[(warp * R + j) * 2 + 0] = m[j];
      ml[(warp * R + j) * 2 + 1] = l[j];
    }
  }
  named_bar_sync(1, NW * 32);
  if (!__all_sync(0xffffffffu, ok)) return;
  // warp w merges rows j = w, w+NW, ...
  for (int j = warp; j < R; j += NW) {
    const int row = rg * R + j;
    if (row >= a.rows) continue;
    float mx = -FLT_MAX;
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, ml[(w * R + j) * 2]);
    float lt = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < NW; ++w) {
      const float sc = ex2(ml[(w * R + j) * 2] - mx);
      lt += sc * ml[(w * R + j) * 2 + 1];
      for (int e = 0; e < 4; ++e) acc[e] += sc * mo[(w * R + j) * D + lane * 4 + e];
    }
    const int g = row % a.group, s_pos = row / a.group;
    const int hq = hkv * a.group + g;
    const long long prow = ((long long)seq * a.Hq * a.Sq + (long long)hq * a.Sq + s_pos);
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    float* po = a.part_o + (prow * a.max_splits + split) * D;
    for (int e = 0; e < 4; ++e) po[lane * 4 + e] = acc[e] * inv;
    if (lane == 0)
      a.part_lse[prow * a.max_splits + split] = (lt > 0.f && mx > -FLT_MAX) ? mx + lg2(lt) : -INFINITY;
  }
}

// ------------------------------------------------- tensor-core consumers ----
// mma.sync m16n8k16 with fp32 accumulation; A row-major (16 x 16), B
// column-major (16 x 8).  The decode is HBM-bound: the tensor core only
// replaces ~1300 scalar FMA/convert instructions per 16-token page slice.
template <bool BF16>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Paged decode with tensor-core consumers (block_size a multiple of 16).
// The TMA ring streams units of U tokens (16 or 32, dividing block_size) of
// one kv head's slice, 128/U stages (64 KB) so every block size up to 256
// keeps 3 CTAs per SM; split-K and outputs as paged_decode_kernel; up to 16
// query rows (GQA group x decode positions of one kv head) per CTA, padded
// to the m16 tile with zero rows.  Per 16 tokens a consumer warp runs
// S = Q K^T (ldmatrix on the swizzled K slice, 16 MMAs), the online softmax
// on the accumulator fragments (rows g and g+8 of lane = 4g + t), and
// O += P V with P re-packed in registers as the A operand (ldmatrix.trans on
// V, 16 MMAs).
template <bool BF16, int U>
__global__ void __launch_bounds__(kThreads, 3)
    paged_decode_mma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ DecArgs a) {
  constexpr int D = 128, RT = 16;
  constexpr int S = 128 / U;  // a.box_bytes == U * 128
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int split = blockIdx.y;
  const int hkv = blockIdx.x / a.row_groups, rg = blockIdx.x % a.row_groups;
  const int seq = blockIdx.z;
  const int ctx = a.seq_lens[seq];
  const int t0 = split * a.chunk_tokens;
  if (t0 >= ctx && !(split == 0 && ctx == 0)) return;
  const int t1 = min(ctx, t0 + a.chunk_tokens);
  const int u0 = t0 / U, u1 = (t1 + U - 1) / U;
  const int nunits = max(0, u1 - u0);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t sb = (raw_base + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw_base);
  const int page_bytes = 2 * a.box_bytes;  // K or V slice of one unit
  const uint32_t k_base = sb, v_base = sb + S * page_bytes;
  const uint32_t bar0 = sb + 2 * S * page_bytes;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (S + s); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NW) {
    if (lane == 0 && nunits > 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int32_t* row = a.block_table + (long long)seq * a.max_blocks;
      for (int i = 0; i < nunits; ++i) {
        const int s = i % S;
        if (!mbar_wait(empty(s), ((i / S) & 1) ^ 1, kStatusTimeoutLoad)) break;
        const int tok = (u0 + i) * U;
        const int pid = (int)phys_page(row, table_col(tok / a.BS, a.max_blocks), a.num_blocks);
        const int prow = pid * a.BS + tok % a.BS;  // pool row of the unit's first token
        mbar_expect_tx(full(s), 4 * U * 128);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(k_base + s * page_bytes + c * a.box_bytes, &tm_k, full(s), c * 64, hkv, prow);
          tma_load_3d(v_base + s * page_bytes + c * a.box_bytes, &tm_v, full(s), c * 64, hkv, prow);
        }
      }
    }
    return;
  }

  const int g = lane >> 2, tig = lane & 3;
  // Q as A fragments: [k-step][row g lo, row g+8 lo, row g hi, row g+8 hi].
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = rg * RT + g + 8 * h;
    const bool okr = row < a.rows;
    const int gq = okr ? row % a.group : 0, s_pos = okr ? row / a.group : 0;
    const T* qr = reinterpret_cast<const T*>(a.q) + (((long long)seq * a.Hq + hkv * a.group + gq) * a.Sq + s_pos) * D;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      qf[kk][h] = okr ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 2 * tig) : 0u;
      qf[kk][2 + h] = okr ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8 + 2 * tig) : 0u;
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-FLT_MAX, -FLT_MAX}, l[2] = {0.f, 0.f};
  // ldmatrix row of this lane: matrix lane >> 3, row lane & 7.
  const int mi = lane >> 3, ri = lane & 7;
  auto sw = [&](uint32_t base, int tok, int d) {  // swizzled [tok][d] in a 2-box page slice
    return base + (d >> 6) * a.box_bytes + tok * 128 + ((((d & 63) >> 3) ^ (tok & 7)) << 4);
  };
  bool ok = true;
  for (int i = warp; i < nunits; i += NW) {
    const int s = i % S;
    ok = __all_sync(0xffffffffu, mbar_wait(full(s), (i / S) & 1, kStatusTimeoutSoftmax));
    if (!ok) break;
    const uint32_t kst = k_base + s * page_bytes, vst = v_base + s * page_bytes;
    const int unit_tok0 = (u0 + i) * U;
    bool zeroed = false;
#pragma unroll
    for (int g16 = 0; g16 < U; g16 += 16) {
      const int tok_a = unit_tok0 + g16;
      if (tok_a < t0 || tok_a + 16 > t1) {
        // V rows of tokens outside [t0, t1) -> 0, so P = 0 there meets finite V.
        for (int x = lane; x < 16 * 16; x += 32) {
          const int r = x >> 4, u = x & 15, tk = tok_a + r;
          if (tk < t0 || tk >= t1)
            *reinterpret_cast<uint4*>(sp + (sw(vst, g16 + r, u * 8) - sb)) = make_uint4(0, 0, 0, 0);
        }
        zeroed = true;
        __syncwarp();
      }
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t b[4];  // (tokens 0-7, d lo), (0-7, hi), (8-15, lo), (8-15, hi)
        ldsm_x4(b, sw(kst, g16 + 8 * (mi >> 1) + ri, 16 * kk + 8 * (mi & 1)));
        mma16816<BF16>(sc[0], qf[kk], b[0], b[1]);
        mma16816<BF16>(sc[1], qf[kk], b[2], b[3]);
      }
      // column (n, e) holds token g16 + 8n + 2*tig + (e & 1); e < 2: row g, else row g + 8
      float mx[2] = {-INFINITY, -INFINITY};
      bool valid[2][2];
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = tok_a + 8 * n + 2 * tig + e;
          valid[n][e] = tk >= t0 && tk < t1;
          if (valid[n][e]) {
            mx[0] = fmaxf(mx[0], sc[n][e]);
            mx[1] = fmaxf(mx[1], sc[n][2 + e]);
          }
        }
      float alpha[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float m_new = fmaxf(m[h], mx[h] * a.sl2);
        alpha[h] = ex2(m[h] - m_new);
        m[h] = m_new;
      }
      float pr[2][4];
      float ps[2] = {0.f, 0.f};
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1;
          pr[n][e] = valid[n][e & 1] ? ex2(fmaf(sc[n][e], a.sl2, -m[h])) : 0.f;
          ps[h] += pr[n][e];
        }
      l[0] = l[0] * alpha[0] + ps[0];
      l[1] = l[1] * alpha[1] + ps[1];
      if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][0] *= alpha[0]; o[n][1] *= alpha[0];
          o[n][2] *= alpha[1]; o[n][3] *= alpha[1];
        }
      }
      const uint32_t pa[4] = {pack2(pr[0][0], pr[0][1], BF16), pack2(pr[0][2], pr[0][3], BF16),
                              pack2(pr[1][0], pr[1][1], BF16), pack2(pr[1][2], pr[1][3], BF16)};
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b[4];  // (tokens 0-7, d tile 2np), (8-15, 2np), (0-7, 2np+1), (8-15, 2np+1)
        ldsm_x4_t(b, sw(vst, g16 + 8 * (mi & 1) + ri, 16 * np + 8 * (mi >> 1)));
        mma16816<BF16>(o[2 * np], pa, b[0], b[1]);
        mma16816<BF16>(o[2 * np + 1], pa, b[2], b[3]);
      }
    }
    if (zeroed) fence_proxy_async_smem();  // generic writes before the next TMA into this stage
    __syncwarp();
    if (lane == 0) mbar_arrive(empty(s));
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  // ---- merge the NW warps' partial states through the drained page ring ----
  named_bar_sync(1, NW * 32);
  constexpr int MS = D + 4;  // padded row stride
  float* mo = reinterpret_cast<float*>(sp);  // [NW][RT][MS]
  float* ml = mo + NW * RT * MS;             // [NW][RT][2]
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    *reinterpret_cast<float2*>(mo + (warp * RT + g) * MS + 8 * n + 2 * tig) = make_float2(o[n][0], o[n][1]);
    *reinterpret_cast<float2*>(mo + (warp * RT + g + 8) * MS + 8 * n + 2 * tig) = make_float2(o[n][2], o[n][3]);
  }
  if (tig == 0) {
    ml[(warp * RT + g) * 2] = m[0];
    ml[(warp * RT + g) * 2 + 1] = l[0];
    ml[(warp * RT + g + 8) * 2] = m[1];
    ml[(warp * RT + g + 8) * 2 + 1] = l[1];
  }
  named_bar_sync(1, NW * 32);
  if (!__all_sync(0xffffffffu, ok)) return;
  for (int j = warp; j < RT; j += NW) {
    const int row = rg * RT + j;
    if (row >= a.rows) continue;
    float mxr = -FLT_MAX;
    for (int w = 0; w < NW; ++w) mxr = fmaxf(mxr, ml[(w * RT + j) * 2]);
    float lt = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < NW; ++w) {
      const float f = ex2(ml[(w * RT + j) * 2] - mxr);
      lt += f * ml[(w * RT + j) * 2 + 1];
      for (int e = 0; e < 4; ++e) acc[e] += f * mo[(w * RT + j) * MS + lane * 4 + e];
    }
    const int gq = row % a.group, s_pos = row / a.group;
    const int hq = hkv * a.group + gq;
    const long long prow = ((long long)seq * a.Hq * a.Sq + (long long)hq * a.Sq + s_pos);
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    float* po = a.part_o + (prow * a.max_splits + split) * D;
    for (int e = 0; e < 4; ++e) po[lane * 4 + e] = acc[e] * inv;
    if (lane == 0)
      a.part_lse[prow * a.max_splits + split] = (lt > 0.f && mxr > -FLT_MAX) ? mxr + lg2(lt) : -INFINITY;
  }
}

// The decode kernel for a launch: tensor-core consumers (R = 16) or scalar ones.
template <int R, bool BF16, bool MMA, int U>
constexpr auto decode_kernel() {
  if constexpr (MMA) return &paged_decode_mma_kernel<BF16, U>;
  else return &paged_decode_kernel<R, BF16>;
}
// Tokens per TMA unit of the tensor-core kernel for a block size (a multiple of 16).
inline int mma_unit(int block_size) { return block_size % 32 == 0 ? 32 : 16; }

// Merges split partials (log2-domain lse): o = sum_i 2^(lse_i - M) o_i / sum_i 2^(lse_i - M).
template <typename T>
__global__ void paged_combine_kernel(const float* part_o, const float* part_lse, const int32_t* seq_lens,
                                     int Hq, int Sq, int D, int max_splits, int chunk_tokens, T* out) {
  const int row = blockIdx.x, seq = blockIdx.y;
  const int ctx = seq_lens[seq];
  const long long prow = (long long)seq * Hq * Sq + row;
  T* orow = out + prow * D;
  // max_context bounds the lengths by contract: a longer sequence is cut to
  // the splits that exist (never read past the partials) and leaves a notice.
  const int need = (ctx + chunk_tokens - 1) / chunk_tokens;
  if (need > max_splits && threadIdx.x == 0) atomicCAS(&g_notice, 0, kNoticeContextOverrun);
  const int n = min(need, max_splits);
  if (n == 0) {  // empty sequence: zeros (paged.py:53-54)
    for (int d = threadIdx.x; d < D; d += blockDim.x) orow[d] = from_f32<T>(0.f);
    return;
  }
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, part_lse[prow * max_splits + i]);
  float tot = 0.f;
  for (int i = 0; i < n; ++i) tot += ex2(part_lse[prow * max_splits + i] - mx);
  const float inv = 1.f / tot;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < n; ++i)
      acc += ex2(part_lse[prow * max_splits + i] - mx) * part_o[(prow * max_splits + i) * D + d];
    orow[d] = from_f32<T>(acc * inv);
  }
}

}  // namespace paged
}  // namespace attnb200
