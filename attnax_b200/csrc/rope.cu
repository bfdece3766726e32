// Rotary position embedding (attnax/embeddings.py:126-184): the rotation
// MultiHeadAttention applies to queries and keys before attention.  One
// thread per rotated pair (i, i + half); consecutive threads take
// consecutive i of a row, so loads of both halves are coalesced.  The
// cos/sin rows come from the caller's tables (built in the tensor dtype by
// the reference's recipe) at each token's position id.

namespace attnb200 {
namespace rope {

template <typename T>
__global__ void rope_kernel(attn_rope_params_t p) {
  const int half = p.head_dim / 2;
  const long long total = (long long)p.batch * p.heads * p.seq * half;
  const T* x = reinterpret_cast<const T*>(p.x);
  T* out = reinterpret_cast<T*>(p.out);
  const T* ct = reinterpret_cast<const T*>(p.cos);
  const T* st = reinterpret_cast<const T*>(p.sin);
  for (long long w = blockIdx.x * (long long)blockDim.x + threadIdx.x; w < total;
       w += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(w % half);
    long long r = w / half;
    const int s = (int)(r % p.seq);
    r /= p.seq;
    const int h = (int)(r % p.heads);
    const int b = (int)(r / p.heads);
    int pos = p.positions ? p.positions[(long long)b * p.seq + s] : s;
    if (pos < 0) pos += p.table_len;
    pos = pos < 0 ? 0 : (pos >= p.table_len ? p.table_len - 1 : pos);
    const float c = to_f32(ct[(long long)pos * half + i]), sn = to_f32(st[(long long)pos * half + i]);
    const T* xr = x + b * p.x_strides[0] + h * p.x_strides[1] + (long long)s * p.x_strides[2];
    T* orow = out + b * p.out_strides[0] + h * p.out_strides[1] + (long long)s * p.out_strides[2];
    const float x1 = to_f32(xr[i]), x2 = to_f32(xr[i + half]);
    orow[i] = from_f32<T>(x1 * c - x2 * sn);
    orow[i + half] = from_f32<T>(x1 * sn + x2 * c);
  }
}

}  // namespace rope
}  // namespace attnb200

extern "C" int attn_rope(const attn_rope_params_t* p, void* stream) {
  using namespace attnb200;
  if (!p || !p->x || !p->out || !p->cos || !p->sin) return ATTN_ERR_INVALID;
  if (p->batch < 0 || p->heads < 0 || p->seq < 0 || p->head_dim <= 0 || p->head_dim % 2 ||
      p->table_len <= 0)
    return ATTN_ERR_INVALID;
  const long long total = (long long)p->batch * p->heads * p->seq * (p->head_dim / 2);
  if (total == 0) return ATTN_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((total + 255) / 256 < 148 * 32 ? (total + 255) / 256 : 148 * 32);
  if (p->dtype == ATTN_F32) rope::rope_kernel<float><<<grid, 256, 0, st>>>(*p);
  else if (p->dtype == ATTN_BF16) rope::rope_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(*p);
  else if (p->dtype == ATTN_F16) rope::rope_kernel<__half><<<grid, 256, 0, st>>>(*p);
  else return ATTN_ERR_INVALID;
  return launch_status();
}
