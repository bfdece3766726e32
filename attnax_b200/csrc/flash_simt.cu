// CUDA-core (FFMA) flash attention: forward and backward in exact fp32
// arithmetic for any supported head_dim and input type.
//
// This is the fp32 path (tcgen05 has no fp32 MMA, and the fp32 parity bar is
// 1e-4 max-abs against standard_attention, attnax/kernels/attention.py:17-71),
// and the path for head dims the tensor-core kernels do not tile.
//
// Layout: a query (or key) row is owned by TPR = max(1, D/32) consecutive
// lanes, each holding EPT = D/TPR contiguous features; dot products reduce
// over those lanes with shuffles.  K/V (or Q/dO) tiles of KT rows are staged
// in shared memory as fp32.
#include <cfloat>

#include "attn_common.cuh"

namespace attnb200 {
namespace simt {

constexpr int kThreads = 128;
constexpr int KT = 32;  // staged rows per tile

template <int D>
struct Lay {
  static constexpr int TPR = D >= 32 ? D / 32 : 1;
  static constexpr int EPT = D / TPR;
  static constexpr int RPB = kThreads / TPR;  // rows per block
};

template <int TPR>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = 1; o < TPR; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

struct FwdArgs {
  int B, Hq, Hkv, Sq, Skv, group;
  const void* q; const void* k; const void* v; void* out;
  long long qs[3], ks[3], vs[3], os[3];
  float* lse;
  float sl2;
  attn_mask_t mask;
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) simt_fwd_kernel(const FwdArgs a) {
  using L = Lay<D>;
  __shared__ float sk[KT][D];
  __shared__ float sv[KT][D];
  const int tid = threadIdx.x;
  const int rloc = tid / L::TPR, part = tid % L::TPR;
  const int hq = blockIdx.y, b = blockIdx.z, hkv = hq / a.group;
  const int q0 = blockIdx.x * L::RPB;
  const int row = q0 + rloc;
  const bool row_ok = row < a.Sq;
  const int q1 = min(q0 + L::RPB, a.Sq);
  const T* Q = reinterpret_cast<const T*>(a.q) + b * a.qs[0] + hq * a.qs[1];
  const T* K = reinterpret_cast<const T*>(a.k) + b * a.ks[0] + hkv * a.ks[1];
  const T* V = reinterpret_cast<const T*>(a.v) + b * a.vs[0] + hkv * a.vs[1];
  float q[L::EPT], o[L::EPT];
#pragma unroll
  for (int e = 0; e < L::EPT; ++e) {
    q[e] = row_ok ? to_f32(Q[(long long)row * a.qs[2] + part * L::EPT + e]) : 0.f;
    o[e] = 0.f;
  }
  const float slope_l2 = a.mask.alibi_slopes ? a.mask.alibi_slopes[hq] * kLog2e : 0.f;
  float m = -FLT_MAX, l = 0.f;
  int j_lo, j_hi;
  band_tile_range(a.mask, q0, q1, a.Skv, KT, &j_lo, &j_hi);
  for (int j = j_lo; j < j_hi; ++j) {
    const int k0 = j * KT, k1 = min(k0 + KT, a.Skv);
    const int st = tile_state(a.mask, nullptr, nullptr, 0, 0, b, q0, q1, k0, k1, KT);
    if (st == kSkip) continue;
    __syncthreads();
    for (int x = tid; x < KT * D; x += kThreads) {
      const int rr = x / D, cc = x % D;
      const bool in = k0 + rr < a.Skv;
      sk[rr][cc] = in ? to_f32(K[(long long)(k0 + rr) * a.ks[2] + cc]) : 0.f;
      sv[rr][cc] = in ? to_f32(V[(long long)(k0 + rr) * a.vs[2] + cc]) : 0.f;
    }
    __syncthreads();
    float t[KT];
    float mx = m;
#pragma unroll
    for (int c = 0; c < KT; ++c) {
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < L::EPT; ++e) acc = fmaf(q[e], sk[c][part * L::EPT + e], acc);
      acc = group_sum<L::TPR>(acc);
      t[c] = mask_score(a.mask, acc, a.sl2, slope_l2, b, hq, row, k0 + c, a.Skv, st == kPartial);
      mx = fmaxf(mx, t[c]);
    }
    const float alpha = exp2f(m - mx);
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < L::EPT; ++e) o[e] *= alpha;
#pragma unroll
    for (int c = 0; c < KT; ++c) {
      const float p = exp2f(t[c] - mx);
      sum += p;
#pragma unroll
      for (int e = 0; e < L::EPT; ++e) o[e] = fmaf(p, sv[c][part * L::EPT + e], o[e]);
    }
    l = l * alpha + sum;
    m = mx;
  }
  if (!row_ok) return;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* O = reinterpret_cast<T*>(a.out) + b * a.os[0] + hq * a.os[1] + (long long)row * a.os[2];
#pragma unroll
  for (int e = 0; e < L::EPT; ++e) O[part * L::EPT + e] = from_f32<T>(o[e] * inv);
  if (a.lse && part == 0)
    a.lse[((long long)b * a.Hq + hq) * a.Sq + row] =
        (m == -FLT_MAX || l <= 0.f) ? -INFINITY : (m + log2f(l)) * kLn2;
}

// ------------------------------------------------------------- backward ----
// delta = rowsum(dO * O); lse2 = lse * log2(e), +inf for rows with no kept
// key (their P is uniform in the reference but their dS is zero; the dV part
// is added by masked_rows_dv_kernel).
template <typename T>
__global__ void bwd_prep_kernel(const T* out, const T* dout, long long os0, long long os1,
                                long long os2, long long ds0, long long ds1, long long ds2,
                                const float* lse, float* delta, float* lse2, int H, int S, int D) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  if (row >= S) return;
  const T* o = out + b * os0 + h * os1 + (long long)row * os2;
  const T* d = dout + b * ds0 + h * ds1 + (long long)row * ds2;
  float acc = 0.f;
  for (int e = lane; e < D; e += 32) acc = fmaf(to_f32(o[e]), to_f32(d[e]), acc);
  for (int x = 16; x > 0; x >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, x);
  if (lane == 0) {
    const long long idx = ((long long)b * H + h) * S + row;
    delta[idx] = acc;
    const float l = lse[idx];
    lse2[idx] = (l == -INFINITY) ? INFINITY : l * kLog2e;
  }
}

struct BwdArgs {
  int B, Hq, Hkv, Sq, Skv, group;
  const void *q, *k, *v, *dout;
  void *dq, *dk, *dv;
  long long qs[3], ks[3], vs[3], dos[3], dqs[3], dks[3], dvs[3];
  const float* lse2;
  const float* delta;
  float scale, sl2;
  attn_mask_t mask;
};

// dQ: one query row per TPR lanes, K/V tiles staged.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) simt_bwd_dq_kernel(const BwdArgs a) {
  using L = Lay<D>;
  __shared__ float sk[KT][D];
  __shared__ float sv[KT][D];
  const int tid = threadIdx.x;
  const int rloc = tid / L::TPR, part = tid % L::TPR;
  const int hq = blockIdx.y, b = blockIdx.z, hkv = hq / a.group;
  const int q0 = blockIdx.x * L::RPB, row = q0 + rloc;
  const bool row_ok = row < a.Sq;
  const int q1 = min(q0 + L::RPB, a.Sq);
  const T* Q = reinterpret_cast<const T*>(a.q) + b * a.qs[0] + hq * a.qs[1];
  const T* DO = reinterpret_cast<const T*>(a.dout) + b * a.dos[0] + hq * a.dos[1];
  const T* K = reinterpret_cast<const T*>(a.k) + b * a.ks[0] + hkv * a.ks[1];
  const T* V = reinterpret_cast<const T*>(a.v) + b * a.vs[0] + hkv * a.vs[1];
  float q[L::EPT], dd[L::EPT], dq[L::EPT];
#pragma unroll
  for (int e = 0; e < L::EPT; ++e) {
    q[e] = row_ok ? to_f32(Q[(long long)row * a.qs[2] + part * L::EPT + e]) : 0.f;
    dd[e] = row_ok ? to_f32(DO[(long long)row * a.dos[2] + part * L::EPT + e]) : 0.f;
    dq[e] = 0.f;
  }
  const long long ridx = ((long long)b * a.Hq + hq) * a.Sq + (row_ok ? row : 0);
  const float lse2 = row_ok ? a.lse2[ridx] : INFINITY;
  const float delta = row_ok ? a.delta[ridx] : 0.f;
  const float slope_l2 = a.mask.alibi_slopes ? a.mask.alibi_slopes[hq] * kLog2e : 0.f;
  int j_lo, j_hi;
  band_tile_range(a.mask, q0, q1, a.Skv, KT, &j_lo, &j_hi);
  for (int j = j_lo; j < j_hi; ++j) {
    const int k0 = j * KT, k1 = min(k0 + KT, a.Skv);
    const int st = tile_state(a.mask, nullptr, nullptr, 0, 0, b, q0, q1, k0, k1, KT);
    if (st == kSkip) continue;
    __syncthreads();
    for (int x = tid; x < KT * D; x += kThreads) {
      const int rr = x / D, cc = x % D;
      const bool in = k0 + rr < a.Skv;
      sk[rr][cc] = in ? to_f32(K[(long long)(k0 + rr) * a.ks[2] + cc]) : 0.f;
      sv[rr][cc] = in ? to_f32(V[(long long)(k0 + rr) * a.vs[2] + cc]) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < KT; ++c) {
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int e = 0; e < L::EPT; ++e) {
        s = fmaf(q[e], sk[c][part * L::EPT + e], s);
        dp = fmaf(dd[e], sv[c][part * L::EPT + e], dp);
      }
      s = group_sum<L::TPR>(s);
      dp = group_sum<L::TPR>(dp);
      const float t = mask_score(a.mask, s, a.sl2, slope_l2, b, hq, row, k0 + c, a.Skv, st == kPartial);
      const float p = (t == -FLT_MAX) ? 0.f : exp2f(t - lse2);
      const float ds = p * (dp - delta);
#pragma unroll
      for (int e = 0; e < L::EPT; ++e) dq[e] = fmaf(ds, sk[c][part * L::EPT + e], dq[e]);
    }
  }
  if (!row_ok) return;
  T* DQ = reinterpret_cast<T*>(a.dq) + b * a.dqs[0] + hq * a.dqs[1] + (long long)row * a.dqs[2];
#pragma unroll
  for (int e = 0; e < L::EPT; ++e) DQ[part * L::EPT + e] = from_f32<T>(dq[e] * a.scale);
}

// dK, dV: one key row per TPR lanes, summed over the query heads of its
// group (the transpose of the reference's jnp.repeat, attention.py:32-39).
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) simt_bwd_dkv_kernel(const BwdArgs a) {
  using L = Lay<D>;
  __shared__ float sq[KT][D];
  __shared__ float sd[KT][D];
  __shared__ float slse[KT], sdelta[KT];
  const int tid = threadIdx.x;
  const int rloc = tid / L::TPR, part = tid % L::TPR;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int k0 = blockIdx.x * L::RPB, col = k0 + rloc;
  const bool col_ok = col < a.Skv;
  const int k1 = min(k0 + L::RPB, a.Skv);
  const T* K = reinterpret_cast<const T*>(a.k) + b * a.ks[0] + hkv * a.ks[1];
  const T* V = reinterpret_cast<const T*>(a.v) + b * a.vs[0] + hkv * a.vs[1];
  float kk[L::EPT], vv[L::EPT], dk[L::EPT], dv[L::EPT];
#pragma unroll
  for (int e = 0; e < L::EPT; ++e) {
    kk[e] = col_ok ? to_f32(K[(long long)col * a.ks[2] + part * L::EPT + e]) : 0.f;
    vv[e] = col_ok ? to_f32(V[(long long)col * a.vs[2] + part * L::EPT + e]) : 0.f;
    dk[e] = dv[e] = 0.f;
  }
  for (int g = 0; g < a.group; ++g) {
    const int hq = hkv * a.group + g;
    const T* Q = reinterpret_cast<const T*>(a.q) + b * a.qs[0] + hq * a.qs[1];
    const T* DO = reinterpret_cast<const T*>(a.dout) + b * a.dos[0] + hq * a.dos[1];
    const float slope_l2 = a.mask.alibi_slopes ? a.mask.alibi_slopes[hq] * kLog2e : 0.f;
    const int nqt = (a.Sq + KT - 1) / KT;
    for (int i = 0; i < nqt; ++i) {
      const int q0 = i * KT, q1 = min(q0 + KT, a.Sq);
      const int st = tile_state(a.mask, nullptr, nullptr, 0, 0, b, q0, q1, k0, k1, L::RPB);
      if (st == kSkip) continue;
      __syncthreads();
      for (int x = tid; x < KT * D; x += kThreads) {
        const int rr = x / D, cc = x % D;
        const bool in = q0 + rr < a.Sq;
        sq[rr][cc] = in ? to_f32(Q[(long long)(q0 + rr) * a.qs[2] + cc]) : 0.f;
        sd[rr][cc] = in ? to_f32(DO[(long long)(q0 + rr) * a.dos[2] + cc]) : 0.f;
      }
      for (int x = tid; x < KT; x += kThreads) {
        const bool in = q0 + x < a.Sq;
        const long long idx = ((long long)b * a.Hq + hq) * a.Sq + q0 + x;
        slse[x] = in ? a.lse2[idx] : INFINITY;
        sdelta[x] = in ? a.delta[idx] : 0.f;
      }
      __syncthreads();
#pragma unroll 4
      for (int rr = 0; rr < KT; ++rr) {
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int e = 0; e < L::EPT; ++e) {
          s = fmaf(sq[rr][part * L::EPT + e], kk[e], s);
          dp = fmaf(sd[rr][part * L::EPT + e], vv[e], dp);
        }
        s = group_sum<L::TPR>(s);
        dp = group_sum<L::TPR>(dp);
        const float t = mask_score(a.mask, s, a.sl2, slope_l2, b, hq, q0 + rr, col, a.Skv,
                                   st == kPartial || q0 + rr >= a.Sq);
        const float p = (t == -FLT_MAX || !col_ok) ? 0.f : exp2f(t - slse[rr]);
        const float ds = p * (dp - sdelta[rr]);
#pragma unroll
        for (int e = 0; e < L::EPT; ++e) {
          dv[e] = fmaf(p, sd[rr][part * L::EPT + e], dv[e]);
          dk[e] = fmaf(ds, sq[rr][part * L::EPT + e], dk[e]);
        }
      }
    }
  }
  if (!col_ok) return;
  T* DK = reinterpret_cast<T*>(a.dk) + b * a.dks[0] + hkv * a.dks[1] + (long long)col * a.dks[2];
  T* DV = reinterpret_cast<T*>(a.dv) + b * a.dvs[0] + hkv * a.dvs[1] + (long long)col * a.dvs[2];
#pragma unroll
  for (int e = 0; e < L::EPT; ++e) {
    DK[part * L::EPT + e] = from_f32<T>(dk[e] * a.scale);
    DV[part * L::EPT + e] = from_f32<T>(dv[e]);
  }
}

}  // namespace simt
}  // namespace attnb200
