// C-ABI entry points (include/attnb200.h).  One translation unit: the kernel
// sources are included here so every kernel shares the device status word.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "../../include/attnb200.h"
#include "attn_common.cuh"
#include "flash_fwd_sm100.cu"
#include "flash_fwd2_sm100.cu"
#include "flash_simt.cu"
#include "flash_bwd_sm100.cu"
#include "paged.cu"
#include "ring.cu"

namespace attnb200 {

// ------------------------------------------------------- masked-row fixes --
// Forward: a row with no kept key is uniform over all of V in the reference
// (every score is finfo.min).  Tile skipping never visits those keys, so
// rows whose LSE came back -inf get mean(V) here.
template <typename T>
__global__ void fix_masked_rows_fwd_kernel(const T* v, long long vs0, long long vs1, long long vs2,
                                           T* out, long long os0, long long os1, long long os2,
                                           const float* lse, int Hq, int Sq, int Skv, int D,
                                           int group) {
  const int q0 = blockIdx.x * 128, hq = blockIdx.y, b = blockIdx.z;
  __shared__ int rows[128];
  __shared__ int nrows;
  if (threadIdx.x == 0) nrows = 0;
  __syncthreads();
  const int r = q0 + threadIdx.x;
  if (threadIdx.x < 128 && r < Sq && lse[((long long)b * Hq + hq) * Sq + r] == -INFINITY)
    rows[atomicAdd(&nrows, 1)] = r;
  __syncthreads();
  if (nrows == 0) return;
  const T* V = v + b * vs0 + (hq / group) * vs1;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int k = 0; k < Skv; ++k) acc += to_f32(V[(long long)k * vs2 + d]);
    const T mean = from_f32<T>(acc / (float)Skv);
    for (int i = 0; i < nrows; ++i) out[b * os0 + hq * os1 + (long long)rows[i] * os2 + d] = mean;
  }
}

// Backward: those rows add dO_row / Skv to every dV row of their KV head
// (uniform P); their dS is zero, so dQ and dK get nothing.
template <typename T>
__global__ void masked_rows_dv_kernel(const T* dout, long long ds0, long long ds1, long long ds2,
                                      T* dv, long long vs0, long long vs1, long long vs2,
                                      const float* lse, int Hq, int Sq, int Skv, int D, int group) {
  const int hkv = blockIdx.y, b = blockIdx.z;
  extern __shared__ float u[];
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  for (int d = threadIdx.x; d < D; d += blockDim.x) u[d] = 0.f;
  __syncthreads();
  for (int g = 0; g < group; ++g) {
    const int hq = hkv * group + g;
    for (int r = 0; r < Sq; ++r) {
      if (lse[((long long)b * Hq + hq) * Sq + r] != -INFINITY) continue;
      if (threadIdx.x == 0) any = 1;
      for (int d = threadIdx.x; d < D; d += blockDim.x)
        u[d] += to_f32(dout[b * ds0 + hq * ds1 + (long long)r * ds2 + d]);
    }
  }
  __syncthreads();
  if (!any) return;
  const int k_per = (Skv + gridDim.x - 1) / gridDim.x;
  for (int k = blockIdx.x * k_per; k < min(Skv, (int)(blockIdx.x + 1) * k_per); ++k)
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      T* p = dv + b * vs0 + hkv * vs1 + (long long)k * vs2 + d;
      *p = from_f32<T>(to_f32(*p) + u[d] / (float)Skv);
    }
}

// -------------------------------------------------------------- helpers ----
static size_t dtype_size(attn_dtype_t t) { return t == ATTN_F32 ? 4 : 2; }

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 4-D tiled map over a (B, H, S, D) tensor with element strides s[0..2] for
// b, h, s; box = 64 features (one 128-byte swizzle row) x box_rows rows.
static bool make_tmap(CUtensorMap* m, attn_dtype_t dt, const void* ptr, int B, int H, int S, int D,
                      const int64_t* s, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const uint64_t es = dtype_size(dt);
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  uint64_t st_s = (uint64_t)s[2] * es, st_h = (uint64_t)s[1] * es, st_b = (uint64_t)s[0] * es;
  // Strides of unit dimensions are never stepped over; give them a legal value.
  if (S == 1) st_s = ((uint64_t)D * es + 15) & ~15ull;
  if (H == 1) st_h = st_s * (uint64_t)S;
  if (B == 1) st_b = st_h * (uint64_t)H;
  cuuint64_t strides[3] = {st_s, st_h, st_b};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16 != 0 || strides[i] >= (1ull << 40)) return false;
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType t =
      dt == ATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(m, t, 4, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool simt_dim_ok(int d) { return d == 8 || d == 16 || d == 32 || d == 64 || d == 128; }

static bool check_mask(const attn_mask_t& m, int B) {
  if (m.has_band && m.band_lo > m.band_hi) return false;
  if ((m.doc_q == nullptr) != (m.doc_kv == nullptr)) return false;
  if (m.bias && m.bias_dtype != ATTN_F32 && m.bias_dtype != ATTN_BF16 && m.bias_dtype != ATTN_F16)
    return false;
  (void)B;
  return true;
}

static std::atomic<unsigned long long> g_launches{0};

// Counts `n` kernel launches and reports the launch error state.
static int launch_status(int n = 1) {
  g_launches.fetch_add(n, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "attnb200: CUDA launch error: %s\n", cudaGetErrorString(e));
    return ATTN_ERR_CUDA;
  }
  return ATTN_OK;
}

// Document-mask tile tables: (min, max) ids per kDocTile tile of q and kv,
// then for each q tile the overlapping kv tile range (q_jr) and, if asked,
// for each kv tile the overlapping q tile range (kv_qr).
static int launch_doc_ranges(const attn_mask_t& m, int batch, int seq_q, int seq_kv, int2* dq_t, int2* dkv_t,
                             int2* q_jr, int2* kv_qr, cudaStream_t st) {
  const int nq = (seq_q + kDocTile - 1) / kDocTile, nk = (seq_kv + kDocTile - 1) / kDocTile;
  doc_tile_range_kernel<<<dim3(nq, batch), 128, 0, st>>>(m.doc_q, m.doc_q_bstride, m.q_offset, seq_q, nq, dq_t);
  doc_tile_range_kernel<<<dim3(nk, batch), 128, 0, st>>>(m.doc_kv, m.doc_kv_bstride, m.kv_offset, seq_kv, nk,
                                                         dkv_t);
  int n = 2;
  if (q_jr) {
    doc_cross_range_kernel<<<dim3((nq + 7) / 8, batch), 256, 0, st>>>(dq_t, nq, dkv_t, nk, q_jr);
    ++n;
  }
  if (kv_qr) {
    doc_cross_range_kernel<<<dim3((nk + 7) / 8, batch), 256, 0, st>>>(dkv_t, nk, dq_t, nq, kv_qr);
    ++n;
  }
  return launch_status(n);
}

struct FwdWorkspace {
  size_t doc_q = 0, doc_kv = 0, doc_jr = 0, doc_order = 0, lse = 0, total = 0;
};

// Document masks: the two-tile forward runs its CTAs longest first
// (doc_cta_order_kernel) when the per-batch ranking fits one block.
constexpr int kMaxOrderedCtas = 4096;
static int fwd2_ctas(int seq_q) { return (seq_q + 2 * fwd2::BM - 1) / (2 * fwd2::BM); }
static bool doc_ordered(const attn_fwd_params_t* p) {
  return p->mask.doc_q && p->seq_q > fwd::BM && fwd2_ctas(p->seq_q) <= kMaxOrderedCtas;
}

static FwdWorkspace fwd_workspace_layout(const attn_fwd_params_t* p) {
  FwdWorkspace w;
  size_t off = 0;
  if (p->mask.doc_q) {
    const int nq = (p->seq_q + kDocTile - 1) / kDocTile, nk = (p->seq_kv + kDocTile - 1) / kDocTile;
    w.doc_q = off;
    off += align256((size_t)p->batch * nq * sizeof(int2));
    w.doc_kv = off;
    off += align256((size_t)p->batch * nk * sizeof(int2));
    w.doc_jr = off;
    off += align256((size_t)p->batch * nq * sizeof(int2));
    if (doc_ordered(p)) {
      w.doc_order = off;
      off += align256((size_t)p->batch * fwd2_ctas(p->seq_q) * sizeof(int));
    }
  }
  if (p->fix_masked_rows && !p->lse) {
    w.lse = off;
    off += align256((size_t)p->batch * p->num_heads_q * p->seq_q * sizeof(float));
  }
  w.total = off;
  return w;
}

template <typename T>
static int launch_simt_fwd(const attn_fwd_params_t* p, float* lse, cudaStream_t st) {
  simt::FwdArgs a;
  a.B = p->batch; a.Hq = p->num_heads_q; a.Hkv = p->num_heads_kv; a.Sq = p->seq_q; a.Skv = p->seq_kv;
  a.group = p->num_heads_q / p->num_heads_kv;
  a.q = p->q; a.k = p->k; a.v = p->v; a.out = p->out;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = p->q_strides[i]; a.ks[i] = p->k_strides[i];
    a.vs[i] = p->v_strides[i]; a.os[i] = p->o_strides[i];
  }
  a.lse = lse; a.sl2 = p->softmax_scale * kLog2e; a.mask = p->mask;
#define ATTN_SIMT_FWD(DD)                                                                   \
  case DD: {                                                                                \
    dim3 g((p->seq_q + simt::Lay<DD>::RPB - 1) / simt::Lay<DD>::RPB, p->num_heads_q, p->batch); \
    simt::simt_fwd_kernel<T, DD><<<g, simt::kThreads, 0, st>>>(a);                          \
    break;                                                                                  \
  }
  switch (p->head_dim) {
    ATTN_SIMT_FWD(8) ATTN_SIMT_FWD(16) ATTN_SIMT_FWD(32) ATTN_SIMT_FWD(64) ATTN_SIMT_FWD(128)
    default: return ATTN_ERR_UNSUPPORTED;
  }
#undef ATTN_SIMT_FWD
  return launch_status();
}

// Accumulation target of a ring step (see fwd2::Args::acc_o); null for a plain forward.
struct RingAcc {
  float* o;
  float* lse;
  int rows, row0, final_from;
};

template <int D, bool BF16>
static int launch_sm100_fwd2(const attn_fwd_params_t* p, float* lse, const int2* dq_t, const int2* dkv_t,
                             const int2* djr, cudaStream_t st, const RingAcc* acc = nullptr,
                             const int* order = nullptr) {
  CUtensorMap tq, tk, tv;
  if (!make_tmap(&tq, p->dtype, p->q, p->batch, p->num_heads_q, p->seq_q, D, p->q_strides, fwd2::BM) ||
      !make_tmap(&tk, p->dtype, p->k, p->batch, p->num_heads_kv, p->seq_kv, D, p->k_strides, fwd2::BN) ||
      !make_tmap(&tv, p->dtype, p->v, p->batch, p->num_heads_kv, p->seq_kv, D, p->v_strides, fwd2::BN))
    return ATTN_ERR_INVALID;
  fwd2::Args a;
  a.B = p->batch; a.Hq = p->num_heads_q; a.Hkv = p->num_heads_kv; a.Sq = p->seq_q; a.Skv = p->seq_kv;
  a.group = p->num_heads_q / p->num_heads_kv;
  a.n_ctas = fwd2_ctas(p->seq_q);
  a.sl2 = p->softmax_scale * kLog2e;
  a.out = p->out;
  a.o_s0 = p->o_strides[0]; a.o_s1 = p->o_strides[1]; a.o_s2 = p->o_strides[2];
  a.lse = lse; a.mask = p->mask;
  a.doc_q_tiles = dq_t; a.doc_kv_tiles = dkv_t; a.doc_jrange = djr;
  a.nq_doc = (p->seq_q + kDocTile - 1) / kDocTile;
  a.nk_doc = (p->seq_kv + kDocTile - 1) / kDocTile;
  a.cta_order = order;
  a.acc_o = acc ? acc->o : nullptr;
  a.acc_lse = acc ? acc->lse : nullptr;
  a.acc_rows = acc ? acc->rows : 0;
  a.acc_row0 = acc ? acc->row0 : 0;
  a.acc_final_from = acc ? acc->final_from : 0;
  constexpr int smem = fwd2::Cfg<D>::SMEM;
  auto kern = acc ? fwd2::flash_fwd2_kernel<D, BF16, true> : fwd2::flash_fwd2_kernel<D, BF16, false>;
  static int attr_dev[2] = {-1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev[acc ? 1 : 0] != dev) {
    // The in-kernel register split assumes this exact launch register count.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs != fwd2::kLaunchRegs)
      return ATTN_ERR_UNSUPPORTED;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return ATTN_ERR_CUDA;
    attr_dev[acc ? 1 : 0] = dev;
  }
  // With an order table, blockIdx.x walks (rank, head) with heads fastest.
  dim3 grid = order ? dim3(a.n_ctas * p->num_heads_q, 1, p->batch) : dim3(a.n_ctas, p->num_heads_q, p->batch);
  kern<<<grid, fwd2::kThreads, smem, st>>>(tq, tk, tv, a);
  return launch_status();
}

template <int D, bool BF16>
static int launch_sm100_fwd(const attn_fwd_params_t* p, float* lse, const int2* dq_t, const int2* dkv_t,
                            const int2* djr, cudaStream_t st, const int* order = nullptr) {
  if (p->seq_q > fwd::BM) {
    const int rc = launch_sm100_fwd2<D, BF16>(p, lse, dq_t, dkv_t, djr, st, nullptr, order);
    if (rc != ATTN_ERR_UNSUPPORTED) return rc;
  }
  CUtensorMap tq, tk, tv;
  if (!make_tmap(&tq, p->dtype, p->q, p->batch, p->num_heads_q, p->seq_q, D, p->q_strides, fwd::BM) ||
      !make_tmap(&tk, p->dtype, p->k, p->batch, p->num_heads_kv, p->seq_kv, D, p->k_strides, fwd::BN) ||
      !make_tmap(&tv, p->dtype, p->v, p->batch, p->num_heads_kv, p->seq_kv, D, p->v_strides, fwd::BN))
    return ATTN_ERR_INVALID;
  fwd::Args a;
  a.B = p->batch; a.Hq = p->num_heads_q; a.Hkv = p->num_heads_kv; a.Sq = p->seq_q; a.Skv = p->seq_kv;
  a.group = p->num_heads_q / p->num_heads_kv;
  a.nq_tiles = (p->seq_q + fwd::BM - 1) / fwd::BM;
  a.sl2 = p->softmax_scale * kLog2e;
  a.out = p->out;
  a.o_s0 = p->o_strides[0]; a.o_s1 = p->o_strides[1]; a.o_s2 = p->o_strides[2];
  a.lse = lse; a.mask = p->mask;
  a.doc_q_tiles = dq_t; a.doc_kv_tiles = dkv_t; a.doc_jrange = djr;
  a.nq_doc = (p->seq_q + kDocTile - 1) / kDocTile;
  a.nk_doc = (p->seq_kv + kDocTile - 1) / kDocTile;
  constexpr int smem = fwd::Cfg<D>::SMEM;
  auto kern = fwd::flash_fwd_kernel<D, BF16>;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return ATTN_ERR_CUDA;
    attr_dev = dev;
  }
  dim3 grid(a.nq_tiles, p->num_heads_q, p->batch);
  kern<<<grid, fwd::kThreads, smem, st>>>(tq, tk, tv, a);
  return launch_status();
}

static bool tc_layout_ok(const attn_fwd_params_t* p) {
  if (p->dtype == ATTN_F32) return false;
  if (p->head_dim != 64 && p->head_dim != 128) return false;
  const void* ptrs[3] = {p->q, p->k, p->v};
  for (auto* x : ptrs)
    if (reinterpret_cast<uintptr_t>(x) % 16) return false;
  if (reinterpret_cast<uintptr_t>(p->out) % 16) return false;
  const int64_t* ss[4] = {p->q_strides, p->k_strides, p->v_strides, p->o_strides};
  for (auto* s : ss)
    for (int i = 0; i < 3; ++i)
      if (s[i] % 8) return false;
  return true;
}

}  // namespace attnb200

using namespace attnb200;

extern "C" {

int attn_version(void) { return 1; }

uint64_t attn_launch_count(void) { return g_launches.load(); }

const char* attn_status_string(int s) {
  switch (s) {
    case ATTN_OK: return "ok";
    case ATTN_ERR_INVALID: return "invalid argument (shape, stride, alignment or pointer)";
    case ATTN_ERR_UNSUPPORTED: return "unsupported configuration";
    case ATTN_ERR_CUDA: return "CUDA error";
    case ATTN_ERR_NCCL: return "NCCL error";
    case ATTN_ERR_WORKSPACE: return "workspace missing or too small";
    case ATTN_ERR_TIMEOUT: return "a bounded device wait timed out";
    default: return "unknown status";
  }
}

int attn_device_status(int32_t* status) {
  int v = 0, n = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return ATTN_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&v, g_status, sizeof(int)) != cudaSuccess) return ATTN_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&n, g_notice, sizeof(int)) != cudaSuccess) return ATTN_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_status, &zero, sizeof(int)) != cudaSuccess) return ATTN_ERR_CUDA;
  if (cudaMemcpyToSymbol(g_notice, &zero, sizeof(int)) != cudaSuccess) return ATTN_ERR_CUDA;
  if (status) *status = v ? v : n;
  return ATTN_OK;
}

int64_t attn_paged_physical_page(int32_t entry, int32_t num_blocks) {
  return num_blocks > 0 ? paged_phys_page(entry, num_blocks) : -1;
}

size_t attn_fwd_workspace_size(const attn_fwd_params_t* p) {
  return p ? fwd_workspace_layout(p).total : 0;
}

int attn_fwd(const attn_fwd_params_t* p, void* stream) {
  if (!p || !p->q || !p->k || !p->v || !p->out) return ATTN_ERR_INVALID;
  if (p->batch <= 0 || p->num_heads_q <= 0 || p->num_heads_kv <= 0 || p->seq_q <= 0 ||
      p->seq_kv <= 0 || p->num_heads_q % p->num_heads_kv != 0)
    return ATTN_ERR_INVALID;
  if (p->dtype != ATTN_F32 && p->dtype != ATTN_BF16 && p->dtype != ATTN_F16) return ATTN_ERR_INVALID;
  if (!check_mask(p->mask, p->batch)) return ATTN_ERR_INVALID;
  const FwdWorkspace w = fwd_workspace_layout(p);
  if (w.total > 0 && (!p->workspace || p->workspace_bytes < w.total)) return ATTN_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(p->workspace);
  float* lse = p->lse ? p->lse : (p->fix_masked_rows ? reinterpret_cast<float*>(ws + w.lse) : nullptr);

  const bool tc = tc_layout_ok(p);
  if (!tc && !simt_dim_ok(p->head_dim)) return ATTN_ERR_UNSUPPORTED;
  int2 *dq_t = nullptr, *dkv_t = nullptr, *djr = nullptr;
  int* order = nullptr;
  if (p->mask.doc_q && tc) {
    dq_t = reinterpret_cast<int2*>(ws + w.doc_q);
    dkv_t = reinterpret_cast<int2*>(ws + w.doc_kv);
    djr = reinterpret_cast<int2*>(ws + w.doc_jr);
    const int lrc = launch_doc_ranges(p->mask, p->batch, p->seq_q, p->seq_kv, dq_t, dkv_t, djr, nullptr, st);
    if (lrc != ATTN_OK) return lrc;
    if (doc_ordered(p)) {
      order = reinterpret_cast<int*>(ws + w.doc_order);
      const int nc = fwd2_ctas(p->seq_q);
      doc_cta_order_kernel<<<p->batch, 256, nc * sizeof(int), st>>>(
          p->mask, djr, (p->seq_q + kDocTile - 1) / kDocTile, p->seq_q, p->seq_kv, fwd2::BM, fwd2::BN, nc, order);
      const int orc = launch_status();
      if (orc != ATTN_OK) return orc;
    }
  }
  int rc;
  if (tc) {
    const bool bf = p->dtype == ATTN_BF16;
    if (p->head_dim == 128)
      rc = bf ? launch_sm100_fwd<128, true>(p, lse, dq_t, dkv_t, djr, st, order)
              : launch_sm100_fwd<128, false>(p, lse, dq_t, dkv_t, djr, st, order);
    else
      rc = bf ? launch_sm100_fwd<64, true>(p, lse, dq_t, dkv_t, djr, st, order)
              : launch_sm100_fwd<64, false>(p, lse, dq_t, dkv_t, djr, st, order);
  } else if (p->dtype == ATTN_F32) {
    rc = launch_simt_fwd<float>(p, lse, st);
  } else if (p->dtype == ATTN_BF16) {
    rc = launch_simt_fwd<__nv_bfloat16>(p, lse, st);
  } else {
    rc = launch_simt_fwd<__half>(p, lse, st);
  }
  if (rc != ATTN_OK) return rc;
  if (p->fix_masked_rows) {
    dim3 g((p->seq_q + 127) / 128, p->num_heads_q, p->batch);
    const int grp = p->num_heads_q / p->num_heads_kv;
#define ATTN_FIX(T)                                                                             \
  fix_masked_rows_fwd_kernel<T><<<g, 128, 0, st>>>(                                             \
      reinterpret_cast<const T*>(p->v), p->v_strides[0], p->v_strides[1], p->v_strides[2],     \
      reinterpret_cast<T*>(p->out), p->o_strides[0], p->o_strides[1], p->o_strides[2], lse,     \
      p->num_heads_q, p->seq_q, p->seq_kv, p->head_dim, grp)
    if (p->dtype == ATTN_F32) ATTN_FIX(float);
    else if (p->dtype == ATTN_BF16) ATTN_FIX(__nv_bfloat16);
    else ATTN_FIX(__half);
#undef ATTN_FIX
    rc = launch_status();
  }
  return rc;
}

}  // extern "C"

namespace attnb200 {
static bool bwd_tc_ok(const attn_bwd_params_t* p) {
  if (p->dtype == ATTN_F32 || (p->head_dim != 64 && p->head_dim != 128)) return false;
  const void* ptrs[9] = {p->q, p->k, p->v, p->out, p->d_out, p->dq, p->dk, p->dv, p->lse};
  for (auto* x : ptrs)
    if (reinterpret_cast<uintptr_t>(x) % 16) return false;
  const int64_t* ss[8] = {p->q_strides, p->k_strides, p->v_strides, p->o_strides, p->do_strides,
                          p->dq_strides, p->dk_strides, p->dv_strides};
  for (auto* s : ss)
    for (int i = 0; i < 3; ++i)
      if (s[i] % 8) return false;
  return true;
}

static int bwd_seq_pad(const attn_bwd_params_t* p) { return (p->seq_q + 127) / 128 * 128; }

static bool bwd_fused_dq(const attn_bwd_params_t* p) { return ATTN_BWD_FUSED_DQ && p->head_dim == 128; }

struct BwdWorkspace {
  size_t lse2 = 0, dq_acc = 0, doc_q = 0, doc_kv = 0, doc_q_jr = 0, doc_kv_qr = 0, doc_kv_order = 0,
         total = 0;  // delta at 0
};

// Document masks: dkdv_kernel runs its kv tiles longest first (doc_kv_order_kernel)
// when the per-batch ranking fits one block.
static int bwd_kv_tiles(int seq_kv) { return (seq_kv + bwd::KROWS - 1) / bwd::KROWS; }
static bool bwd_doc_ordered(const attn_bwd_params_t* p) {
  return p->mask.doc_q && bwd_kv_tiles(p->seq_kv) <= kMaxOrderedCtas;
}

static BwdWorkspace bwd_workspace_layout(const attn_bwd_params_t* p) {
  BwdWorkspace w;
  const bool tc = bwd_tc_ok(p);
  const size_t rows = (size_t)p->batch * p->num_heads_q * (tc ? bwd_seq_pad(p) : p->seq_q);
  w.lse2 = align256(rows * sizeof(float));
  w.dq_acc = 2 * w.lse2;
  size_t off = w.dq_acc + ((tc && bwd_fused_dq(p)) ? align256(rows * p->head_dim * sizeof(float)) : 0);
  if (tc && p->mask.doc_q) {
    const size_t nq = (p->seq_q + kDocTile - 1) / kDocTile, nk = (p->seq_kv + kDocTile - 1) / kDocTile;
    w.doc_q = off;
    off += align256(p->batch * nq * sizeof(int2));
    w.doc_kv = off;
    off += align256(p->batch * nk * sizeof(int2));
    w.doc_q_jr = off;
    off += align256(p->batch * nq * sizeof(int2));
    w.doc_kv_qr = off;
    off += align256(p->batch * nk * sizeof(int2));
    if (bwd_doc_ordered(p)) {
      w.doc_kv_order = off;
      off += align256((size_t)p->batch * bwd_kv_tiles(p->seq_kv) * sizeof(int));
    }
  }
  w.total = off;
  return w;
}

struct BwdDocTables {
  const int2 *q_t = nullptr, *kv_t = nullptr, *q_jr = nullptr, *kv_qr = nullptr;
  const int* kv_order = nullptr;
};

// Sets the kernel's dynamic shared-memory limit once per device.
template <typename K>
static bool smem_attr_once(K kernel, int bytes, int* cached_dev) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (*cached_dev == dev) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  *cached_dev = dev;
  return true;
}

template <int D, bool BF16>
static int launch_sm100_bwd(const attn_bwd_params_t* p, float* delta, float* lse2, float* dq_acc,
                            const BwdDocTables& doc, cudaStream_t st) {
  using namespace bwd;
  const int Sq_pad = bwd_seq_pad(p);
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  {
    constexpr int rows_per_block = kPrepRowsPerBlock / (D / 8);
    prep_rows_kernel<T, D><<<dim3((Sq_pad + rows_per_block - 1) / rows_per_block, p->num_heads_q, p->batch), 256, 0,
                             st>>>(
        reinterpret_cast<const T*>(p->out), reinterpret_cast<const T*>(p->d_out), p->o_strides[0], p->o_strides[1],
        p->o_strides[2], p->do_strides[0], p->do_strides[1], p->do_strides[2], p->lse, delta, lse2,
        p->num_heads_q, p->seq_q, Sq_pad, (D == 128 && bwd_fused_dq(p) && !CfgKV<128, true>::RED) ? dq_acc : nullptr);
  }
  Args a;
  a.B = p->batch; a.Hq = p->num_heads_q; a.Hkv = p->num_heads_kv; a.Sq = p->seq_q; a.Skv = p->seq_kv;
  a.Sq_pad = Sq_pad; a.group = p->num_heads_q / p->num_heads_kv;
  a.sl2 = p->softmax_scale * kLog2e; a.scale = p->softmax_scale;
  a.lse2 = lse2; a.delta = delta;
  a.dq = p->dq; a.dk = p->dk; a.dv = p->dv; a.dq_acc = dq_acc;
  for (int i = 0; i < 3; ++i) {
    a.dq_s[i] = p->dq_strides[i]; a.dk_s[i] = p->dk_strides[i]; a.dv_s[i] = p->dv_strides[i];
  }
  a.mask = p->mask;
  a.doc_q_tiles = doc.q_t; a.doc_kv_tiles = doc.kv_t; a.doc_q_jr = doc.q_jr; a.doc_kv_qr = doc.kv_qr;
  a.nq_doc = (p->seq_q + kDocTile - 1) / kDocTile;
  a.nk_doc = (p->seq_kv + kDocTile - 1) / kDocTile;
  a.kv_order = doc.kv_order;
  a.n_kt = bwd_kv_tiles(p->seq_kv);
  CUtensorMap q64, do64, k128, v128, q128, do128, k64, v64;
  const int B = p->batch, Hq = p->num_heads_q, Hkv = p->num_heads_kv, Sq = p->seq_q, Skv = p->seq_kv;
  if (!make_tmap(&q64, p->dtype, p->q, B, Hq, Sq, D, p->q_strides, QT) ||
      !make_tmap(&do64, p->dtype, p->d_out, B, Hq, Sq, D, p->do_strides, QT) ||
      !make_tmap(&k128, p->dtype, p->k, B, Hkv, Skv, D, p->k_strides, KROWS) ||
      !make_tmap(&v128, p->dtype, p->v, B, Hkv, Skv, D, p->v_strides, KROWS) ||
      !make_tmap(&q128, p->dtype, p->q, B, Hq, Sq, D, p->q_strides, QROWS) ||
      !make_tmap(&do128, p->dtype, p->d_out, B, Hq, Sq, D, p->do_strides, QROWS) ||
      !make_tmap(&k64, p->dtype, p->k, B, Hkv, Skv, D, p->k_strides, KT) ||
      !make_tmap(&v64, p->dtype, p->v, B, Hkv, Skv, D, p->v_strides, KT))
    return ATTN_ERR_INVALID;
  // With an order table, blockIdx.x walks (rank, kv head) with heads fastest.
  const dim3 grid_kv = a.kv_order ? dim3(a.n_kt * Hkv, 1, B) : dim3(a.n_kt, Hkv, B);
  if constexpr (D == 128) {
    if (bwd_fused_dq(p)) {
      // dQ accumulated in fp32 by the dK/dV kernel, then scaled and converted.
      static int attr_dev_f = -1;
      auto kf = dkdv_kernel<D, BF16, true>;
      if (attr_dev_f < 0 && CfgKV<D, true>::DQW) {
        // The in-kernel setmaxnreg split draws on exactly LAUNCH_REGS registers per
        // thread: with any other launch count the growing warps could wait forever.
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, kf) != cudaSuccess || fa.numRegs != CfgKV<D, true>::LAUNCH_REGS)
          return ATTN_ERR_UNSUPPORTED;
      }
      if (!smem_attr_once(kf, CfgKV<D, true>::SMEM, &attr_dev_f)) return ATTN_ERR_CUDA;
      // (dq_acc rows were zeroed by prep_rows_kernel; the transposed layout is cleared here)
      if (CfgKV<D, true>::RED &&
          cudaMemsetAsync(dq_acc, 0, (size_t)B * Hq * Sq_pad * D * sizeof(float), st) != cudaSuccess)
        return ATTN_ERR_CUDA;
      kf<<<grid_kv, CfgKV<D, true>::THREADS, CfgKV<D, true>::SMEM, st>>>(q64, k128, v128, do64, a);
      if (CfgKV<D, true>::RED)
        dq_convert_t_kernel<T, D><<<dim3((Sq + 63) / 64, Hq, B), 256, 0, st>>>(
            dq_acc, reinterpret_cast<T*>(p->dq), p->dq_strides[0], p->dq_strides[1], p->dq_strides[2], Hq, Sq,
            Sq_pad, p->softmax_scale);
      else
        dq_convert_kernel<T><<<dim3((Sq + 7) / 8, Hq, B), 256, 0, st>>>(
            dq_acc, reinterpret_cast<T*>(p->dq), p->dq_strides[0], p->dq_strides[1], p->dq_strides[2], Hq, Sq,
            Sq_pad, D, p->softmax_scale);
      return launch_status(3);
    }
  }
  static int attr_dev_kv = -1, attr_dev_q = -1;
  auto kkv = dkdv_kernel<D, BF16, false>;
  auto kq = dq_kernel<D, BF16>;
  if (!smem_attr_once(kkv, CfgKV<D, false>::SMEM, &attr_dev_kv) || !smem_attr_once(kq, CfgQ<D>::SMEM, &attr_dev_q))
    return ATTN_ERR_CUDA;
  kkv<<<grid_kv, CfgKV<D, false>::THREADS, CfgKV<D, false>::SMEM, st>>>(q64, k128, v128, do64, a);
  kq<<<dim3((Sq + QROWS - 1) / QROWS, Hq, B), kThreads, CfgQ<D>::SMEM, st>>>(q128, k64, v64, do128, a);
  return launch_status(3);
}

}  // namespace attnb200

extern "C" {

size_t attn_bwd_workspace_size(const attn_bwd_params_t* p) {
  if (!p) return 0;
  return bwd_workspace_layout(p).total;
}

int attn_bwd(const attn_bwd_params_t* p, void* stream) {
  if (!p || !p->q || !p->k || !p->v || !p->out || !p->d_out || !p->lse || !p->dq || !p->dk || !p->dv)
    return ATTN_ERR_INVALID;
  if (p->batch <= 0 || p->num_heads_q <= 0 || p->num_heads_kv <= 0 || p->seq_q <= 0 ||
      p->seq_kv <= 0 || p->num_heads_q % p->num_heads_kv != 0)
    return ATTN_ERR_INVALID;
  if (!check_mask(p->mask, p->batch)) return ATTN_ERR_INVALID;
  const bool tc = bwd_tc_ok(p);
  if (!tc && !simt_dim_ok(p->head_dim)) return ATTN_ERR_UNSUPPORTED;
  const size_t need = attn_bwd_workspace_size(p);
  if (!p->workspace || p->workspace_bytes < need) return ATTN_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const BwdWorkspace wl = bwd_workspace_layout(p);
  float* delta = reinterpret_cast<float*>(p->workspace);
  float* lse2 = reinterpret_cast<float*>(reinterpret_cast<char*>(p->workspace) + wl.lse2);
  float* dq_acc = reinterpret_cast<float*>(reinterpret_cast<char*>(p->workspace) + wl.dq_acc);
  const int grp = p->num_heads_q / p->num_heads_kv;

  simt::BwdArgs a;
  a.B = p->batch; a.Hq = p->num_heads_q; a.Hkv = p->num_heads_kv; a.Sq = p->seq_q; a.Skv = p->seq_kv;
  a.group = grp;
  a.q = p->q; a.k = p->k; a.v = p->v; a.dout = p->d_out; a.dq = p->dq; a.dk = p->dk; a.dv = p->dv;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = p->q_strides[i]; a.ks[i] = p->k_strides[i]; a.vs[i] = p->v_strides[i];
    a.dos[i] = p->do_strides[i]; a.dqs[i] = p->dq_strides[i]; a.dks[i] = p->dk_strides[i];
    a.dvs[i] = p->dv_strides[i];
  }
  a.lse2 = lse2; a.delta = delta;
  a.scale = p->softmax_scale; a.sl2 = p->softmax_scale * kLog2e; a.mask = p->mask;

  if (tc) {
    int rc;
    BwdDocTables doc;
    if (p->mask.doc_q) {
      char* wb = reinterpret_cast<char*>(p->workspace);
      int2* q_t = reinterpret_cast<int2*>(wb + wl.doc_q);
      int2* kv_t = reinterpret_cast<int2*>(wb + wl.doc_kv);
      int2* q_jr = reinterpret_cast<int2*>(wb + wl.doc_q_jr);
      int2* kv_qr = reinterpret_cast<int2*>(wb + wl.doc_kv_qr);
      rc = launch_doc_ranges(p->mask, p->batch, p->seq_q, p->seq_kv, q_t, kv_t, q_jr, kv_qr, st);
      if (rc != ATTN_OK) return rc;
      doc.q_t = q_t; doc.kv_t = kv_t; doc.q_jr = q_jr; doc.kv_qr = kv_qr;
      if (bwd_doc_ordered(p)) {
        int* kv_order = reinterpret_cast<int*>(wb + wl.doc_kv_order);
        const int nkt = bwd_kv_tiles(p->seq_kv);
        bwd::doc_kv_order_kernel<<<p->batch, 256, nkt * sizeof(int), st>>>(
            p->mask, kv_qr, (p->seq_kv + kDocTile - 1) / kDocTile, p->seq_q, p->seq_kv, nkt, kv_order);
        rc = launch_status();
        if (rc != ATTN_OK) return rc;
        doc.kv_order = kv_order;
      }
    }
    const bool bf = p->dtype == ATTN_BF16;
    if (p->head_dim == 128)
      rc = bf ? launch_sm100_bwd<128, true>(p, delta, lse2, dq_acc, doc, st)
              : launch_sm100_bwd<128, false>(p, delta, lse2, dq_acc, doc, st);
    else
      rc = bf ? launch_sm100_bwd<64, true>(p, delta, lse2, dq_acc, doc, st)
              : launch_sm100_bwd<64, false>(p, delta, lse2, dq_acc, doc, st);
    if (rc != ATTN_OK || !p->fix_masked_rows) return rc;
    auto fix = [&](auto tag) {
      using T = decltype(tag);
      masked_rows_dv_kernel<T><<<dim3(16, p->num_heads_kv, p->batch), 128, p->head_dim * sizeof(float), st>>>(
          reinterpret_cast<const T*>(p->d_out), p->do_strides[0], p->do_strides[1], p->do_strides[2],
          reinterpret_cast<T*>(p->dv), p->dv_strides[0], p->dv_strides[1], p->dv_strides[2], p->lse,
          p->num_heads_q, p->seq_q, p->seq_kv, p->head_dim, grp);
    };
    if (bf) fix(__nv_bfloat16{});
    else fix(__half{});
    return launch_status();
  }
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    simt::bwd_prep_kernel<T><<<dim3((p->seq_q + 3) / 4, p->num_heads_q, p->batch), 128, 0, st>>>(
        reinterpret_cast<const T*>(p->out), reinterpret_cast<const T*>(p->d_out), p->o_strides[0],
        p->o_strides[1], p->o_strides[2], p->do_strides[0], p->do_strides[1], p->do_strides[2], p->lse,
        delta, lse2, p->num_heads_q, p->seq_q, p->head_dim);
#define ATTN_SIMT_BWD(DD)                                                                         \
  case DD: {                                                                                      \
    using L = simt::Lay<DD>;                                                                      \
    simt::simt_bwd_dq_kernel<T, DD>                                                               \
        <<<dim3((p->seq_q + L::RPB - 1) / L::RPB, p->num_heads_q, p->batch), simt::kThreads, 0, st>>>(a); \
    simt::simt_bwd_dkv_kernel<T, DD>                                                              \
        <<<dim3((p->seq_kv + L::RPB - 1) / L::RPB, p->num_heads_kv, p->batch), simt::kThreads, 0, st>>>(a); \
    break;                                                                                        \
  }
    switch (p->head_dim) {
      ATTN_SIMT_BWD(8) ATTN_SIMT_BWD(16) ATTN_SIMT_BWD(32) ATTN_SIMT_BWD(64) ATTN_SIMT_BWD(128)
      default: return ATTN_ERR_UNSUPPORTED;
    }
#undef ATTN_SIMT_BWD
    if (p->fix_masked_rows) {
      masked_rows_dv_kernel<T><<<dim3(16, p->num_heads_kv, p->batch), 128, p->head_dim * sizeof(float), st>>>(
          reinterpret_cast<const T*>(p->d_out), p->do_strides[0], p->do_strides[1], p->do_strides[2],
          reinterpret_cast<T*>(p->dv), p->dv_strides[0], p->dv_strides[1], p->dv_strides[2], p->lse,
          p->num_heads_q, p->seq_q, p->seq_kv, p->head_dim, grp);
    }
    return launch_status(p->fix_masked_rows ? 4 : 3);
  };
  if (p->dtype == ATTN_F32) return run(float{});
  if (p->dtype == ATTN_BF16) return run(__nv_bfloat16{});
  if (p->dtype == ATTN_F16) return run(__half{});
  return ATTN_ERR_INVALID;
}

}  // extern "C"

// ------------------------------------------------------------ paged cache --
namespace attnb200 {
static int paged_vec_bytes(int row_bytes) {
  return row_bytes % 16 == 0 ? 16 : row_bytes % 8 == 0 ? 8 : row_bytes % 4 == 0 ? 4 : 2;
}
}  // namespace attnb200

extern "C" {

int attn_paged_gather(attn_dtype_t dtype, const void* key_pool, const void* value_pool,
                      int32_t num_blocks, int32_t block_size, int32_t heads_kv, int32_t head_dim,
                      const int32_t* block_table_row, int32_t max_blocks, int32_t seq_len, void* keys_out,
                      void* values_out, void* stream) {
  if (!key_pool || !value_pool || !block_table_row || num_blocks <= 0 || block_size <= 0 || heads_kv <= 0 ||
      head_dim <= 0 || max_blocks <= 0 || seq_len < 0)
    return ATTN_ERR_INVALID;
  if (seq_len == 0) return ATTN_OK;
  // gather_kv cannot reshape fewer table entries than the length needs.
  if ((long long)seq_len > (long long)max_blocks * block_size) return ATTN_ERR_INVALID;
  if (!keys_out || !values_out) return ATTN_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int row_bytes = heads_kv * head_dim * (int)dtype_size(dtype);
  int vb = paged_vec_bytes(row_bytes);
  const uintptr_t al = reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool) |
                       reinterpret_cast<uintptr_t>(keys_out) | reinterpret_cast<uintptr_t>(values_out);
  while (vb > 2 && al % vb) vb /= 2;
  const int row_vecs = row_bytes / vb;
  const long long n = (long long)seq_len * row_vecs;
  const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
#define ATTN_GATHER(V)                                                                          \
  paged::gather_kernel<V><<<grid, 256, 0, st>>>(                                               \
      reinterpret_cast<const V*>(key_pool), reinterpret_cast<const V*>(value_pool), block_size, \
      row_vecs, block_table_row, seq_len, num_blocks, reinterpret_cast<V*>(keys_out),           \
      reinterpret_cast<V*>(values_out))
  if (vb == 16) ATTN_GATHER(uint4);
  else if (vb == 8) ATTN_GATHER(uint2);
  else if (vb == 4) ATTN_GATHER(uint32_t);
  else ATTN_GATHER(uint16_t);
#undef ATTN_GATHER
  return launch_status();
}

int attn_paged_append(attn_dtype_t dtype, void* key_pool, void* value_pool, int32_t num_blocks,
                      int32_t block_size, int32_t heads_kv, int32_t head_dim, const int32_t* block_table_row,
                      int32_t max_blocks, int32_t start, int32_t chunk, const void* keys_new,
                      const void* values_new, int32_t* bad_slot, void* stream) {
  if (!key_pool || !value_pool || !block_table_row || num_blocks <= 0 || block_size <= 0 || heads_kv <= 0 ||
      head_dim <= 0 || max_blocks <= 0 || start < 0 || chunk < 0)
    return ATTN_ERR_INVALID;
  if (chunk == 0) return ATTN_OK;
  if (!keys_new || !values_new) return ATTN_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (bad_slot) {
    // Check pass only: the caller reads bad_slot (pre-set to INT_MAX) and
    // calls again with bad_slot == NULL to write, so a failed append writes
    // nothing (append_kv raises before any update, paged_cache.py:180-188).
    paged::append_check_kernel<<<(chunk + 255) / 256, 256, 0, st>>>(block_table_row, max_blocks, block_size,
                                                                      start, chunk, bad_slot);
    return launch_status();
  }
  const int row_bytes = heads_kv * head_dim * (int)dtype_size(dtype);
  int vb = paged_vec_bytes(row_bytes);
  const uintptr_t al = reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool) |
                       reinterpret_cast<uintptr_t>(keys_new) | reinterpret_cast<uintptr_t>(values_new);
  while (vb > 2 && al % vb) vb /= 2;
  const int row_vecs = row_bytes / vb;
  const long long n = (long long)chunk * row_vecs;
  const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
#define ATTN_APPEND(V)                                                                          \
  paged::append_kernel<V><<<grid, 256, 0, st>>>(                                               \
      reinterpret_cast<V*>(key_pool), reinterpret_cast<V*>(value_pool), block_size, row_vecs,   \
      block_table_row, num_blocks, max_blocks, start, chunk, reinterpret_cast<const V*>(keys_new), \
      reinterpret_cast<const V*>(values_new))
  if (vb == 16) ATTN_APPEND(uint4);
  else if (vb == 8) ATTN_APPEND(uint2);
  else if (vb == 4) ATTN_APPEND(uint32_t);
  else ATTN_APPEND(uint16_t);
#undef ATTN_APPEND
  return launch_status();
}

}  // extern "C"

namespace attnb200 {
struct PagedWs {
  size_t part_o = 0, part_lse = 0, total = 0;
  int max_splits = 0;
};
static PagedWs paged_ws_layout(const attn_paged_params_t* p) {
  PagedWs w;
  w.max_splits = (p->max_context + paged::kChunkTokens - 1) / paged::kChunkTokens;
  if (w.max_splits < 1) w.max_splits = 1;
  const size_t rows = (size_t)p->num_seqs * p->num_heads_q * p->seq_q;
  w.part_o = 0;
  w.part_lse = align256(rows * w.max_splits * p->head_dim * sizeof(float));
  w.total = w.part_lse + align256(rows * w.max_splits * sizeof(float));
  return w;
}

// 3-D map over a pool [blocks*block_size tokens, heads_kv, head_dim]:
// box = 64 features x 1 head x box_tokens tokens, 128B swizzle.
static bool make_pool_tmap(CUtensorMap* m, attn_dtype_t dt, const void* pool, long long tokens,
                           int heads_kv, int head_dim, int box_tokens) {
  auto enc = encode_fn();
  if (!enc) return false;
  const uint64_t es = dtype_size(dt);
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)heads_kv, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)head_dim * es, (cuuint64_t)heads_kv * head_dim * es};
  if (heads_kv == 1) strides[0] = strides[1];
  for (int i = 0; i < 2; ++i)
    if (strides[i] % 16 != 0) return false;
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_tokens};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType t =
      dt == ATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(m, t, 3, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// MMA: tensor-core consumers (block_size % 16 == 0), R = 16 rows per CTA.
template <int R, bool BF16, bool MMA = false>
static int launch_paged(const attn_paged_params_t* p, const PagedWs& w, char* ws, cudaStream_t st) {
  CUtensorMap tk, tv;
  const long long tokens = (long long)p->num_blocks * p->block_size;
  const int box_tokens = MMA ? paged::mma_unit(p->block_size) : p->block_size;
  if (!make_pool_tmap(&tk, p->dtype, p->key_pool, tokens, p->num_heads_kv, 128, box_tokens) ||
      !make_pool_tmap(&tv, p->dtype, p->value_pool, tokens, p->num_heads_kv, 128, box_tokens))
    return ATTN_ERR_INVALID;
  paged::DecArgs a;
  a.num_seqs = p->num_seqs; a.Hq = p->num_heads_q; a.Hkv = p->num_heads_kv; a.Sq = p->seq_q;
  a.BS = p->block_size; a.max_blocks = p->max_blocks_per_seq; a.num_blocks = p->num_blocks;
  a.group = p->num_heads_q / p->num_heads_kv;
  a.rows = a.group * p->seq_q;
  a.row_groups = (a.rows + R - 1) / R;
  a.max_splits = w.max_splits;
  a.chunk_tokens = paged::kChunkTokens;
  a.box_bytes = (int)(((size_t)box_tokens * 128 + 1023) & ~(size_t)1023);
  a.q = p->q; a.block_table = p->block_table; a.seq_lens = p->seq_lengths;
  a.part_o = reinterpret_cast<float*>(ws + w.part_o);
  a.part_lse = reinterpret_cast<float*>(ws + w.part_lse);
  a.sl2 = p->softmax_scale * kLog2e;
  const int S = MMA ? 128 / box_tokens : paged::DecCfg<R>::STAGES;
  // (the MMA kernel merges its warps through the drained page ring instead of extra scratch)
  const size_t smem = 1024 + (size_t)2 * S * 2 * a.box_bytes + 2 * S * 8 +
                      (MMA ? 0 : sizeof(float) * (paged::NW * (19 * R) + paged::NW * R * 128 + paged::NW * R * 2));
  if (smem > 227 * 1024) return ATTN_ERR_UNSUPPORTED;
  auto kern = (MMA && box_tokens == 32) ? paged::decode_kernel<R, BF16, MMA, 32>()
                                          : paged::decode_kernel<R, BF16, MMA, 16>();
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return ATTN_ERR_CUDA;
  dim3 grid(p->num_heads_kv * a.row_groups, w.max_splits, p->num_seqs);
  kern<<<grid, paged::kThreads, smem, st>>>(tk, tv, a);
  int rc = launch_status();
  if (rc != ATTN_OK) return rc;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  paged::paged_combine_kernel<T><<<dim3(p->num_heads_q * p->seq_q, p->num_seqs), 128, 0, st>>>(
      a.part_o, a.part_lse, p->seq_lengths, p->num_heads_q, p->seq_q, 128, w.max_splits,
      paged::kChunkTokens, reinterpret_cast<T*>(p->out));
  return launch_status();
}
}  // namespace attnb200

extern "C" {

size_t attn_paged_decode_workspace_size(const attn_paged_params_t* p) {
  return p ? paged_ws_layout(p).total : 0;
}

int attn_paged_decode(const attn_paged_params_t* p, void* stream) {
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
  const PagedWs w = paged_ws_layout(p);
  if (!p->workspace || p->workspace_bytes < w.total) return ATTN_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(p->workspace);
  const int rows = (p->num_heads_q / p->num_heads_kv) * p->seq_q;
  const bool bf = p->dtype == ATTN_BF16;
  if (p->block_size % 16 == 0)
    return bf ? launch_paged<16, true, true>(p, w, ws, st) : launch_paged<16, false, true>(p, w, ws, st);
  if (rows <= 1) return bf ? launch_paged<1, true>(p, w, ws, st) : launch_paged<1, false>(p, w, ws, st);
  if (rows <= 2) return bf ? launch_paged<2, true>(p, w, ws, st) : launch_paged<2, false>(p, w, ws, st);
  if (rows <= 4) return bf ? launch_paged<4, true>(p, w, ws, st) : launch_paged<4, false>(p, w, ws, st);
  return bf ? launch_paged<8, true>(p, w, ws, st) : launch_paged<8, false>(p, w, ws, st);
}

}  // extern "C"

#include "paged_static.cu"
#include "rope.cu"
#include "ring_host.cu"

extern "C" int attn_lse_merge(attn_dtype_t dtype, int64_t rows, int32_t head_dim, float* o_acc,
                              float* lse_acc, const void* o_part, const float* lse_part, void* out,
                              void* stream) {
  using namespace attnb200;
  if (rows < 0 || head_dim <= 0 || !o_acc || !lse_acc || !o_part || !lse_part) return ATTN_ERR_INVALID;
  if (rows == 0) return ATTN_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((rows + 7) / 8);
#define ATTN_MERGE(T)                                                                         \
  ring::lse_merge_kernel<T><<<grid, 256, 0, st>>>(rows, head_dim, o_acc, lse_acc,             \
                                                  reinterpret_cast<const T*>(o_part), lse_part, \
                                                  reinterpret_cast<T*>(out))
  if (dtype == ATTN_F32) ATTN_MERGE(float);
  else if (dtype == ATTN_BF16) ATTN_MERGE(__nv_bfloat16);
  else if (dtype == ATTN_F16) ATTN_MERGE(__half);
  else return ATTN_ERR_INVALID;
#undef ATTN_MERGE
  return launch_status();
}
