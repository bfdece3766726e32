// Ring attention support (attnax/kernels/attention.py:540-691).
//
// The reference carries (m, l, o) through a lax.scan and folds each K/V
// block in with the online-softmax update (:662-671).  Here every ring step
// runs the flash kernel on (local Q, visiting K/V) with global position
// offsets, which returns a normalised partial output and its LSE; this
// kernel folds that partial into the running result.  The K/V rotation
// itself (:673-674) is NCCL send/recv issued by the caller.
#include <cfloat>

#include "attn_common.cuh"

namespace attnb200 {
namespace ring {

// One warp per row; lanes stride over the head_dim features.
template <typename T>
__global__ void lse_merge_kernel(long long rows, int D, float* o_acc, float* lse_acc, const T* o_part,
                                 const float* lse_part, T* out) {
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float la = lse_acc[row], lp = lse_part[row];
  const float m = fmaxf(la, lp);
  float wa = 0.f, wp = 0.f;
  if (m != -INFINITY) {
    wa = (la == -INFINITY) ? 0.f : __expf(la - m);
    wp = (lp == -INFINITY) ? 0.f : __expf(lp - m);
  }
  const float tot = wa + wp;
  const float ca = tot > 0.f ? wa / tot : 1.f, cp = tot > 0.f ? wp / tot : 0.f;
  float* oa = o_acc + row * D;
  const T* op = o_part + row * D;
  for (int e = lane; e < D; e += 32) {
    const float v = ca * oa[e] + cp * to_f32(op[e]);
    oa[e] = v;
    if (out) out[row * D + e] = from_f32<T>(v);
  }
  if (lane == 0) lse_acc[row] = tot > 0.f ? m + __logf(tot) : la;
}

}  // namespace ring
}  // namespace attnb200
