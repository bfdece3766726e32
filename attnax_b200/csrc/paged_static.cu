// Allocation-free variant of the paged decode (attn_paged_decode_static).
//
// Some callers cannot allocate device memory for a workspace: serving loops
// whose allocator forbids cudaMalloc on the decode path (it synchronises the
// device and stalls every stream), embedders that run the library inside a
// fixed device-memory budget, and plugin hosts that hand a kernel only its
// inputs and outputs.  This entry point keeps the split-K partials in a
// file-scope device array instead of a caller workspace.  It launches the
// same decode and combine kernels as attn_paged_decode.
#include <mutex>

namespace attnb200 {
namespace paged_static {

// 8 MiB of split partials (o then lse), shared by every call on a device.
constexpr size_t kScratchFloats = (size_t)2 << 20;
static __device__ __align__(256) float g_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
static float* g_scratch_ptr[kMaxDevices];
static CUcontext g_scratch_ctx[kMaxDevices];
static std::mutex g_scratch_mu;

// The calling thread's current CUDA context (null before the runtime made one).
static CUcontext current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

// Device address of g_scratch for the current device.  In host code the
// symbol is only a host-side stand-in, so the address is looked up with the
// device current (cudaGetSymbolAddress) and cached per device together with
// the context it was looked up in; a call under another context (after a
// cudaDeviceReset, or from a non-primary context, where the module and its
// array may sit elsewhere) looks it up again.
static int scratch_address(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ATTN_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  const CUcontext ctx = current_context();
  if (!g_scratch_ptr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess || !ptr) {
      fprintf(stderr, "attnb200: cudaGetSymbolAddress(scratch) failed: %s\n", cudaGetErrorString(e));
      return ATTN_ERR_CUDA;
    }
    g_scratch_ptr[dev] = static_cast<float*>(ptr);
    g_scratch_ctx[dev] = current_context();  // the lookup made the device's context current
  }
  *out = g_scratch_ptr[dev];
  return ATTN_OK;
}

template <int R, bool BF16, bool MMA = false>
static int launch(const attn_paged_params_t* p, float* scratch, int splits, int chunk, cudaStream_t st) {
  CUtensorMap tk, tv;
  const long long tokens = (long long)p->num_blocks * p->block_size;
  const int box_tokens = MMA ? paged::mma_unit(p->block_size) : p->block_size;
  if (!make_pool_tmap(&tk, p->dtype, p->key_pool, tokens, p->num_heads_kv, 128, box_tokens) ||
      !make_pool_tmap(&tv, p->dtype, p->value_pool, tokens, p->num_heads_kv, 128, box_tokens))
    return ATTN_ERR_INVALID;
  const size_t rows = (size_t)p->num_seqs * p->num_heads_q * p->seq_q;
  paged::DecArgs a;
  a.num_seqs = p->num_seqs; a.Hq = p->num_heads_q; a.Hkv = p->num_heads_kv; a.Sq = p->seq_q;
  a.BS = p->block_size; a.max_blocks = p->max_blocks_per_seq; a.num_blocks = p->num_blocks;
  a.group = p->num_heads_q / p->num_heads_kv;
  a.rows = a.group * p->seq_q;
  a.row_groups = (a.rows + R - 1) / R;
  a.max_splits = splits;
  a.chunk_tokens = chunk;
  a.box_bytes = (int)(((size_t)box_tokens * 128 + 1023) & ~(size_t)1023);
  a.q = p->q; a.block_table = p->block_table; a.seq_lens = p->seq_lengths;
  a.part_o = scratch;                                  // [rows][splits][128]
  a.part_lse = scratch + rows * (size_t)splits * 128;  // [rows][splits]
  a.sl2 = p->softmax_scale * kLog2e;
  const int S = MMA ? 128 / box_tokens : paged::DecCfg<R>::STAGES;
  const size_t smem = 1024 + (size_t)2 * S * 2 * a.box_bytes + 2 * S * 8 +
                      (MMA ? 0 : sizeof(float) * (paged::NW * (19 * R) + paged::NW * R * 128 + paged::NW * R * 2));
  if (smem > 227 * 1024) return ATTN_ERR_UNSUPPORTED;
  auto kern = (MMA && box_tokens == 32) ? paged::decode_kernel<R, BF16, MMA, 32>()
                                          : paged::decode_kernel<R, BF16, MMA, 16>();
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return ATTN_ERR_CUDA;
  kern<<<dim3(p->num_heads_kv * a.row_groups, splits, p->num_seqs), paged::kThreads, smem, st>>>(tk, tv, a);
  int rc = launch_status();
  if (rc != ATTN_OK) return rc;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  paged::paged_combine_kernel<T><<<dim3(p->num_heads_q * p->seq_q, p->num_seqs), 128, 0, st>>>(
      a.part_o, a.part_lse, p->seq_lengths, p->num_heads_q, p->seq_q, 128, splits, chunk,
      reinterpret_cast<T*>(p->out));
  return launch_status();
}

}  // namespace paged_static
}  // namespace attnb200

extern "C" int attn_paged_decode_static(const attn_paged_params_t* p, void* stream) {
  using namespace attnb200;
  if (!p || !p->q || !p->key_pool || !p->value_pool || !p->block_table || !p->seq_lengths || !p->out)
    return ATTN_ERR_INVALID;
  if (p->num_seqs <= 0 || p->num_heads_q <= 0 || p->num_heads_kv <= 0 || p->seq_q <= 0 ||
      p->num_blocks <= 0 || p->block_size <= 0 || p->max_blocks_per_seq <= 0 || p->max_context < 0 ||
      p->num_heads_q % p->num_heads_kv != 0)
    return ATTN_ERR_INVALID;
  if (p->dtype != ATTN_BF16 && p->dtype != ATTN_F16) return ATTN_ERR_UNSUPPORTED;
  if (p->head_dim != 128 || p->block_size > 256) return ATTN_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(p->key_pool) % 16 || reinterpret_cast<uintptr_t>(p->value_pool) % 16)
    return ATTN_ERR_INVALID;
  // Fit the split count to the array: rows * splits * (head_dim + 1) floats.
  const size_t rows = (size_t)p->num_seqs * p->num_heads_q * p->seq_q;
  const size_t per_split = rows * (size_t)(p->head_dim + 1);
  const size_t fit = paged_static::kScratchFloats / per_split;
  if (fit < 1) {
    fprintf(stderr,
            "attnb200: attn_paged_decode_static needs %zu floats of scratch for %zu query rows; the "
            "static array holds %zu (at most %zu rows)\n",
            per_split, rows, paged_static::kScratchFloats,
            paged_static::kScratchFloats / (size_t)(p->head_dim + 1));
    return ATTN_ERR_WORKSPACE;
  }
  int splits = (p->max_context + paged::kChunkTokens - 1) / paged::kChunkTokens;
  if (splits < 1) splits = 1;
  if ((size_t)splits > fit) splits = (int)fit;
  int chunk = p->max_context > 0 ? (p->max_context + splits - 1) / splits : paged::kChunkTokens;
  if (chunk < 1) chunk = 1;
  float* scratch = nullptr;
  const int rc = paged_static::scratch_address(&scratch);
  if (rc != ATTN_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int grp_rows = (p->num_heads_q / p->num_heads_kv) * p->seq_q;
  const bool bf = p->dtype == ATTN_BF16;
  if (p->block_size % 16 == 0)
    return bf ? paged_static::launch<16, true, true>(p, scratch, splits, chunk, st)
              : paged_static::launch<16, false, true>(p, scratch, splits, chunk, st);
  if (grp_rows <= 1)
    return bf ? paged_static::launch<1, true>(p, scratch, splits, chunk, st)
              : paged_static::launch<1, false>(p, scratch, splits, chunk, st);
  if (grp_rows <= 2)
    return bf ? paged_static::launch<2, true>(p, scratch, splits, chunk, st)
              : paged_static::launch<2, false>(p, scratch, splits, chunk, st);
  if (grp_rows <= 4)
    return bf ? paged_static::launch<4, true>(p, scratch, splits, chunk, st)
              : paged_static::launch<4, false>(p, scratch, splits, chunk, st);
  return bf ? paged_static::launch<8, true>(p, scratch, splits, chunk, st)
            : paged_static::launch<8, false>(p, scratch, splits, chunk, st);
}
