// XLA FFI handlers over the attnb200 C ABI: the custom-call layer through
// which JAX code calls the sm_100a kernels (jax.ffi.ffi_call on the targets
// registered by jax_binding.py).  Each handler adapts XLA buffers, the
// stream and the scratch allocator to one C-ABI entry point:
//
//   attnb200_fwd          attn_fwd            flash_attention forward
//                                             (attnax/kernels/attention.py:209-283)
//   attnb200_bwd          attn_bwd            its VJP (JAX autodiff in the reference)
//   attnb200_paged_decode attn_paged_decode   paged_attention over a PagedKVCache
//                                             (attnax/kernels/paged.py:17-84)
//   attnb200_ring_fwd     attn_ring_fwd       ring_attention (attention.py:540-691)
//
// Mask chains are passed as attributes: a band (causal / sliding window on
// global positions) and ALiBi; the Python side flattens the built-in
// ScoreMods into them.  Workspaces come from XLA's scratch allocator, so
// the handlers allocate nothing themselves.
//
// Build: compiled only where jaxlib's FFI headers are present
// (python -c "import jax.ffi; print(jax.ffi.include_dir())"); see Makefile.
#if __has_include("xla/ffi/api/ffi.h")

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "attnb200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error status_error(int rc, const char* what) {
  if (rc == ATTN_OK) return ffi::Error::Success();
  std::string msg = std::string(what) + ": " + attn_status_string(rc);
  const ffi::ErrorCode code = rc == ATTN_ERR_INVALID       ? ffi::ErrorCode::kInvalidArgument
                              : rc == ATTN_ERR_UNSUPPORTED ? ffi::ErrorCode::kUnimplemented
                                                           : ffi::ErrorCode::kInternal;
  return ffi::Error(code, msg);
}

bool dtype_of(ffi::DataType t, attn_dtype_t* out) {
  switch (t) {
    case ffi::DataType::BF16: *out = ATTN_BF16; return true;
    case ffi::DataType::F16: *out = ATTN_F16; return true;
    case ffi::DataType::F32: *out = ATTN_F32; return true;
    default: return false;
  }
}

// Contiguous (b, h, s) element strides of a rank-4 (B, H, S, D) buffer.
void strides4(const ffi::AnyBuffer& x, int64_t out[3]) {
  auto d = x.dimensions();
  out[2] = d[3];
  out[1] = d[2] * d[3];
  out[0] = d[1] * d[2] * d[3];
}

// The reference's per-head ALiBi slopes (attnax/kernels/score_mods.py:14-45).
std::vector<float> alibi_slopes(int n) {
  auto pow2 = [](int m) {
    std::vector<double> v(m);
    const double start = std::pow(2.0, -std::pow(2.0, -(std::log2((double)m) - 3)));
    for (int i = 0; i < m; ++i) v[i] = start * std::pow(start, i);
    return v;
  };
  std::vector<double> s;
  if ((n & (n - 1)) == 0) {
    s = pow2(n);
  } else {
    const int closest = 1 << (int)std::floor(std::log2((double)n));
    s = pow2(closest);
    const std::vector<double> extra = pow2(2 * closest);
    for (int i = 0; (int)s.size() < n; i += 2) s.push_back(extra[i]);
  }
  return std::vector<float>(s.begin(), s.end());
}

// Slopes copied into scratch memory (the kernels read them from the device).
ffi::Error upload_slopes(ffi::ScratchAllocator& scratch, cudaStream_t st, int heads, const float** out) {
  const std::vector<float> h = alibi_slopes(heads);
  auto mem = scratch.Allocate(h.size() * sizeof(float), 256);
  if (!mem.has_value()) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "attnb200: scratch for ALiBi slopes");
  // pageable source: the copy is staged before the call returns
  if (cudaMemcpyAsync(*mem, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess)
    return ffi::Error(ffi::ErrorCode::kInternal, "attnb200: slope upload");
  *out = static_cast<const float*>(*mem);
  return ffi::Error::Success();
}

void set_band(attn_mask_t* m, int64_t has_band, int64_t lo, int64_t hi) {
  m->has_band = has_band != 0;
  m->band_lo = lo;
  m->band_hi = hi;
}

}  // namespace

// ---- forward --------------------------------------------------------------
static ffi::Error AttnFwdImpl(cudaStream_t st, ffi::ScratchAllocator scratch, ffi::AnyBuffer q, ffi::AnyBuffer k,
                              ffi::AnyBuffer v, int64_t has_band, int64_t band_lo, int64_t band_hi, bool alibi,
                              float softmax_scale, ffi::Result<ffi::AnyBuffer> out,
                              ffi::Result<ffi::Buffer<ffi::F32>> lse) {
  attn_fwd_params_t p;
  std::memset(&p, 0, sizeof(p));
  if (q.dimensions().size() != 4 || !dtype_of(q.element_type(), &p.dtype))
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "attnb200_fwd: q must be rank-4 f32/bf16/f16");
  auto qd = q.dimensions(), kd = k.dimensions();
  p.batch = qd[0]; p.num_heads_q = qd[1]; p.seq_q = qd[2]; p.head_dim = qd[3];
  p.num_heads_kv = kd[1]; p.seq_kv = kd[2];
  p.q = q.untyped_data(); p.k = k.untyped_data(); p.v = v.untyped_data(); p.out = out->untyped_data();
  strides4(q, p.q_strides); strides4(k, p.k_strides); strides4(v, p.v_strides); strides4(q, p.o_strides);
  p.lse = lse->typed_data();
  p.softmax_scale = softmax_scale;
  p.fix_masked_rows = 1;
  set_band(&p.mask, has_band, band_lo, band_hi);
  if (alibi) {
    ffi::Error e = upload_slopes(scratch, st, p.num_heads_q, &p.mask.alibi_slopes);
    if (e.failure()) return e;
  }
  const size_t ws = attn_fwd_workspace_size(&p);
  if (ws) {
    auto mem = scratch.Allocate(ws, 256);
    if (!mem.has_value()) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "attnb200_fwd: workspace");
    p.workspace = *mem;
    p.workspace_bytes = ws;
  }
  return status_error(attn_fwd(&p, st), "attn_fwd");
}

XLA_FFI_DEFINE_HANDLER_SYMBOL(AttnFwd, AttnFwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::AnyBuffer>()  // q (B, Hq, Sq, D)
                                  .Arg<ffi::AnyBuffer>()  // k (B, Hkv, Skv, D)
                                  .Arg<ffi::AnyBuffer>()  // v
                                  .Attr<int64_t>("has_band")
                                  .Attr<int64_t>("band_lo")
                                  .Attr<int64_t>("band_hi")
                                  .Attr<bool>("alibi")
                                  .Attr<float>("softmax_scale")
                                  .Ret<ffi::AnyBuffer>()              // out
                                  .Ret<ffi::Buffer<ffi::F32>>());     // lse (B, Hq, Sq)

// ---- backward -------------------------------------------------------------
static ffi::Error AttnBwdImpl(cudaStream_t st, ffi::ScratchAllocator scratch, ffi::AnyBuffer q, ffi::AnyBuffer k,
                              ffi::AnyBuffer v, ffi::AnyBuffer o, ffi::Buffer<ffi::F32> lse, ffi::AnyBuffer dout,
                              int64_t has_band, int64_t band_lo, int64_t band_hi, bool alibi, float softmax_scale,
                              ffi::Result<ffi::AnyBuffer> dq, ffi::Result<ffi::AnyBuffer> dk,
                              ffi::Result<ffi::AnyBuffer> dv) {
  attn_bwd_params_t p;
  std::memset(&p, 0, sizeof(p));
  if (q.dimensions().size() != 4 || !dtype_of(q.element_type(), &p.dtype))
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "attnb200_bwd: q must be rank-4 f32/bf16/f16");
  auto qd = q.dimensions(), kd = k.dimensions();
  p.batch = qd[0]; p.num_heads_q = qd[1]; p.seq_q = qd[2]; p.head_dim = qd[3];
  p.num_heads_kv = kd[1]; p.seq_kv = kd[2];
  p.q = q.untyped_data(); p.k = k.untyped_data(); p.v = v.untyped_data();
  p.out = o.untyped_data(); p.d_out = dout.untyped_data(); p.lse = lse.typed_data();
  p.dq = dq->untyped_data(); p.dk = dk->untyped_data(); p.dv = dv->untyped_data();
  strides4(q, p.q_strides); strides4(k, p.k_strides); strides4(v, p.v_strides);
  strides4(q, p.o_strides); strides4(q, p.do_strides);
  strides4(q, p.dq_strides); strides4(k, p.dk_strides); strides4(v, p.dv_strides);
  p.softmax_scale = softmax_scale;
  p.fix_masked_rows = 1;
  set_band(&p.mask, has_band, band_lo, band_hi);
  if (alibi) {
    ffi::Error e = upload_slopes(scratch, st, p.num_heads_q, &p.mask.alibi_slopes);
    if (e.failure()) return e;
  }
  const size_t ws = attn_bwd_workspace_size(&p);
  auto mem = scratch.Allocate(ws > 16 ? ws : 16, 256);
  if (!mem.has_value()) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "attnb200_bwd: workspace");
  p.workspace = *mem;
  p.workspace_bytes = ws > 16 ? ws : 16;
  return status_error(attn_bwd(&p, st), "attn_bwd");
}

XLA_FFI_DEFINE_HANDLER_SYMBOL(AttnBwd, AttnBwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::AnyBuffer>()          // q
                                  .Arg<ffi::AnyBuffer>()          // k
                                  .Arg<ffi::AnyBuffer>()          // v
                                  .Arg<ffi::AnyBuffer>()          // out (saved by the forward)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // lse (saved by the forward)
                                  .Arg<ffi::AnyBuffer>()          // d_out
                                  .Attr<int64_t>("has_band")
                                  .Attr<int64_t>("band_lo")
                                  .Attr<int64_t>("band_hi")
                                  .Attr<bool>("alibi")
                                  .Attr<float>("softmax_scale")
                                  .Ret<ffi::AnyBuffer>()          // dq
                                  .Ret<ffi::AnyBuffer>()          // dk
                                  .Ret<ffi::AnyBuffer>());        // dv

// ---- paged decode ---------------------------------------------------------
static ffi::Error PagedDecodeImpl(cudaStream_t st, ffi::ScratchAllocator scratch, ffi::AnyBuffer q,
                                  ffi::AnyBuffer key_pool, ffi::AnyBuffer value_pool,
                                  ffi::Buffer<ffi::S32> block_table, ffi::Buffer<ffi::S32> seq_lengths,
                                  int64_t max_context, float softmax_scale, ffi::Result<ffi::AnyBuffer> out) {
  attn_paged_params_t p;
  std::memset(&p, 0, sizeof(p));
  if (q.dimensions().size() != 4 || !dtype_of(q.element_type(), &p.dtype))
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "attnb200_paged_decode: q must be rank-4 bf16/f16");
  auto qd = q.dimensions(), pd = key_pool.dimensions(), td = block_table.dimensions();
  p.num_seqs = qd[0]; p.num_heads_q = qd[1]; p.seq_q = qd[2]; p.head_dim = qd[3];
  p.num_blocks = pd[0]; p.block_size = pd[1]; p.num_heads_kv = pd[2];
  p.max_blocks_per_seq = td[1];
  p.max_context = (int32_t)max_context;
  p.q = q.untyped_data(); p.key_pool = key_pool.untyped_data(); p.value_pool = value_pool.untyped_data();
  p.block_table = block_table.typed_data(); p.seq_lengths = seq_lengths.typed_data();
  p.out = out->untyped_data();
  p.softmax_scale = softmax_scale;
  const size_t ws = attn_paged_decode_workspace_size(&p);
  auto mem = scratch.Allocate(ws > 16 ? ws : 16, 256);
  if (!mem.has_value()) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "attnb200_paged_decode: workspace");
  p.workspace = *mem;
  p.workspace_bytes = ws > 16 ? ws : 16;
  return status_error(attn_paged_decode(&p, st), "attn_paged_decode");
}

XLA_FFI_DEFINE_HANDLER_SYMBOL(PagedDecode, PagedDecodeImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::AnyBuffer>()          // q (num_seqs, Hq, Sq, D)
                                  .Arg<ffi::AnyBuffer>()          // key pool (num_blocks, block, Hkv, D)
                                  .Arg<ffi::AnyBuffer>()          // value pool
                                  .Arg<ffi::Buffer<ffi::S32>>()   // block table (num_seqs, max_blocks)
                                  .Arg<ffi::Buffer<ffi::S32>>()   // seq lengths (num_seqs,)
                                  .Attr<int64_t>("max_context")
                                  .Attr<float>("softmax_scale")
                                  .Ret<ffi::AnyBuffer>());        // out

// ---- ring forward ---------------------------------------------------------
// `comm` is the attn_comm_t of this process (made once by the Python side
// with attn_comm_unique_id / attn_comm_init), passed as an integer.  The
// ring's NCCL traffic shares XLA's stream with the attention here.
static ffi::Error RingFwdImpl(cudaStream_t st, ffi::ScratchAllocator scratch, ffi::AnyBuffer q, ffi::AnyBuffer k,
                              ffi::AnyBuffer v, int64_t comm, int64_t world, int64_t has_band, int64_t band_lo,
                              int64_t band_hi, bool alibi, int64_t zigzag, float softmax_scale,
                              ffi::Result<ffi::AnyBuffer> out, ffi::Result<ffi::Buffer<ffi::F32>> lse) {
  attn_ring_params_t p;
  std::memset(&p, 0, sizeof(p));
  if (q.dimensions().size() != 4 || !dtype_of(q.element_type(), &p.dtype))
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "attnb200_ring_fwd: q must be rank-4 bf16/f16");
  auto qd = q.dimensions(), kd = k.dimensions();
  p.batch = qd[0]; p.num_heads_q = qd[1]; p.seq_local = qd[2]; p.head_dim = qd[3];
  p.num_heads_kv = kd[1];
  p.q = q.untyped_data(); p.k = k.untyped_data(); p.v = v.untyped_data();
  p.out = out->untyped_data(); p.lse = lse->typed_data();
  p.softmax_scale = softmax_scale;
  p.has_band = has_band != 0; p.band_lo = band_lo; p.band_hi = band_hi;
  p.zigzag = (int32_t)zigzag;
  if (alibi) {
    ffi::Error e = upload_slopes(scratch, st, p.num_heads_q, &p.alibi_slopes);
    if (e.failure()) return e;
  }
  const size_t ws = attn_ring_fwd_workspace_size(&p, (int32_t)world);
  auto mem = scratch.Allocate(ws > 16 ? ws : 16, 256);
  if (!mem.has_value()) return ffi::Error(ffi::ErrorCode::kResourceExhausted, "attnb200_ring_fwd: workspace");
  p.workspace = *mem;
  p.workspace_bytes = ws > 16 ? ws : 16;
  return status_error(attn_ring_fwd(&p, reinterpret_cast<attn_comm_t>(comm), st, st), "attn_ring_fwd");
}

XLA_FFI_DEFINE_HANDLER_SYMBOL(RingFwd, RingFwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::AnyBuffer>()  // q shard (B, Hq, S/P, D)
                                  .Arg<ffi::AnyBuffer>()  // k shard
                                  .Arg<ffi::AnyBuffer>()  // v shard
                                  .Attr<int64_t>("comm")
                                  .Attr<int64_t>("world")
                                  .Attr<int64_t>("has_band")
                                  .Attr<int64_t>("band_lo")
                                  .Attr<int64_t>("band_hi")
                                  .Attr<bool>("alibi")
                                  .Attr<int64_t>("zigzag")
                                  .Attr<float>("softmax_scale")
                                  .Ret<ffi::AnyBuffer>()              // out shard
                                  .Ret<ffi::Buffer<ffi::F32>>());     // lse shard

#endif  // __has_include("xla/ffi/api/ffi.h")
