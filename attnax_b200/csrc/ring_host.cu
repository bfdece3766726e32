// Sequence-parallel ring attention as C-ABI entry points (attn_comm_*,
// attn_ring_plan, attn_ring_fwd) -- the ring of ring_attention
// (attnax/kernels/attention.py:540-691) driven from the host without Python.
//
// One process per GPU.  NCCL is loaded at run time (dlopen of libnccl.so.2,
// which resolves to the copy a host framework already loaded), so the
// library itself links only the CUDA runtime.  Rank r holds the contiguous
// shard [r*S, (r+1)*S) of the global sequence, as in the reference.
//
// Schedule.  With a causal band the work of a contiguous ring is lopsided, so
// the sequence is cut into 2P chunks of C = S/2 rows and rank r works on
// chunks (2r, 2P-1-2r): it keeps the first chunk of its own shard and swaps
// the second with its mirror rank P-1-r (one exchange, overlapped with the
// diagonal block of the kept chunk).  Every hop after that has exactly two
// kept chunk pairs per rank.  At hop i rank r holds the K/V of rank
// (r - i) mod P (attention.py:640) and sends them on to r+1 while the
// attention of the hop runs (the ppermute of :673-674 as NCCL send/recv on a
// communication stream, double-buffered).  Each chunk-pair launch of the
// forward kernel folds its rows into an fp32 running result by log-sum-exp
// in its epilogue (the per-step update of :662-671); the last launch that
// touches a q chunk writes the finished rows in the tensor dtype.  Pairs the
// band keeps whole, with no position-dependent term, are batched into one
// launch over both q chunks or both kv chunks.
#include <dlfcn.h>
#include <nccl.h>  // types and prototypes only; the functions are resolved with dlsym

#include <vector>

namespace attnb200 {
namespace ringhost {

// ------------------------------------------------------------------ NCCL --
struct NcclFns {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

static const NcclFns* nccl() {
  static NcclFns f;
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      fprintf(stderr, "attnb200: NCCL not found (libnccl.so.2): %s\n", dlerror());
      return;
    }
#define ATTN_NCCL_SYM(field, name) f.field = reinterpret_cast<decltype(f.field)>(dlsym(h, name))
    ATTN_NCCL_SYM(get_unique_id, "ncclGetUniqueId");
    ATTN_NCCL_SYM(init_rank, "ncclCommInitRank");
    ATTN_NCCL_SYM(destroy, "ncclCommDestroy");
    ATTN_NCCL_SYM(abort, "ncclCommAbort");
    ATTN_NCCL_SYM(send, "ncclSend");
    ATTN_NCCL_SYM(recv, "ncclRecv");
    ATTN_NCCL_SYM(group_start, "ncclGroupStart");
    ATTN_NCCL_SYM(group_end, "ncclGroupEnd");
    ATTN_NCCL_SYM(all_gather, "ncclAllGather");
    ATTN_NCCL_SYM(error_string, "ncclGetErrorString");
#undef ATTN_NCCL_SYM
    ok = f.get_unique_id && f.init_rank && f.destroy && f.send && f.recv && f.group_start && f.group_end &&
         f.all_gather && f.error_string;
  });
  return ok ? &f : nullptr;
}

static int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return ATTN_OK;
  const NcclFns* f = nccl();
  fprintf(stderr, "attnb200: %s: %s\n", what, f ? f->error_string(r) : "NCCL unavailable");
  return ATTN_ERR_NCCL;
}

// ------------------------------------------------------------ schedule --
// One launch of the forward kernel: q rows [q_slot*C, (q_slot+q_n)*C) of
// the ring buffer against kv rows [kv_slot*C, (kv_slot+kv_n)*C) of the K/V
// visiting at `hop`.  `masked`: pass the band / ALiBi with the global
// positions q_start / kv_start (otherwise the pair is whole and position
// free); `final_from`: first launch row that is final; `local`: needs no
// data from the re-deal (the diagonal block of the kept chunk at hop 0).
struct Launch {
  int hop, q_slot, q_n, kv_slot, kv_n;
  long long q_start, kv_start;
  int masked, final_from, local;
};

struct Sched {
  int P, r, zig, C;
  bool has_band;
  long long lo, hi;
  std::vector<int> held(int rank) const {
    if (!zig) return {rank};
    return {2 * rank, 2 * P - 1 - 2 * rank};
  }
  int mirror() const { return zig ? P - 1 - r : r; }
  // no kept pair between chunk cq (queries) and chunk ck (keys)?
  bool all_masked(int cq, int ck) const {
    if (!has_band) return false;
    const long long q0 = (long long)cq * C, k0 = (long long)ck * C;
    const long long dmax = (q0 + C - 1) - k0, dmin = q0 - (k0 + C - 1);
    return dmax < lo || dmin > hi;
  }
  bool whole(int cq, int ck) const {
    if (!has_band) return true;
    const long long q0 = (long long)cq * C, k0 = (long long)ck * C;
    return q0 - (k0 + C - 1) >= lo && (q0 + C - 1) - k0 <= hi;
  }
};

// The launches of one rank's ring forward, in issue order.
static std::vector<Launch> plan(const Sched& s, bool position_free) {
  struct Pair { int hop, qi, ki; };
  std::vector<Pair> pairs;
  const std::vector<int> mine = s.held(s.r);
  for (int i = 0; i < s.P; ++i) {
    const std::vector<int> kv = s.held(((s.r - i) % s.P + s.P) % s.P);
    for (int qi = 0; qi < (int)mine.size(); ++qi)
      for (int ki = 0; ki < (int)kv.size(); ++ki)
        if (!s.all_masked(mine[qi], kv[ki])) pairs.push_back({i, qi, ki});
  }
  // last pair of each q chunk writes the finished rows
  int last[2] = {-1, -1};
  for (int n = 0; n < (int)pairs.size(); ++n) last[pairs[n].qi] = n;
  std::vector<Launch> out;
  auto single = [&](int n, int local) {
    const Pair& p = pairs[n];
    const std::vector<int> kv = s.held(((s.r - p.hop) % s.P + s.P) % s.P);
    Launch l;
    l.hop = p.hop; l.q_slot = p.qi; l.q_n = 1; l.kv_slot = p.ki; l.kv_n = 1;
    l.q_start = (long long)mine[p.qi] * s.C;
    l.kv_start = (long long)kv[p.ki] * s.C;
    l.masked = 1;
    l.final_from = (n == last[p.qi]) ? 0 : s.C;
    l.local = local;
    out.push_back(l);
  };
  size_t n = 0;
  while (n < pairs.size()) {
    const int hop = pairs[n].hop;
    size_t e = n;
    while (e < pairs.size() && pairs[e].hop == hop) ++e;
    const std::vector<int> kv = s.held(((s.r - hop) % s.P + s.P) % s.P);
    if (hop == 0 && s.zig) {
      // the diagonal block of the kept chunk first: it needs no exchanged data
      for (size_t m = n; m < e; ++m)
        if (pairs[m].qi == 0 && pairs[m].ki == 0) single((int)m, 1);
      for (size_t m = n; m < e; ++m)
        if (!(pairs[m].qi == 0 && pairs[m].ki == 0)) single((int)m, 0);
      n = e;
      continue;
    }
    bool batched = false;
    if (position_free && e - n == 2 && s.whole(mine[pairs[n].qi], kv[pairs[n].ki]) &&
        s.whole(mine[pairs[n + 1].qi], kv[pairs[n + 1].ki])) {
      const Pair &a = pairs[n], &b = pairs[n + 1];
      const bool f0 = (int)n == last[0] || (int)n + 1 == last[0];
      const bool f1 = (int)n == last[1] || (int)n + 1 == last[1];
      // Both q chunks against one kv chunk are batched only when the launch
      // finishes both chunks' rows.  Measured per hop at 131072 tokens on 4
      // GPUs: a batched launch that folds rows into the fp32 running result
      // took 9.8-10.0 ms against 9.3 for two separate launches, while a
      // batched launch that finishes them took 8.4, and one q chunk against
      // both kv chunks 8.7.
      if (a.ki == b.ki && a.qi != b.qi && f0 && f1) {
        Launch l;
        l.hop = hop; l.q_slot = 0; l.q_n = 2; l.kv_slot = a.ki; l.kv_n = 1;
        l.q_start = l.kv_start = 0;
        l.masked = 0;
        l.final_from = 0;
        l.local = 0;
        out.push_back(l);
        batched = true;
      } else if (a.qi == b.qi && a.ki != b.ki) {
        Launch l;
        l.hop = hop; l.q_slot = a.qi; l.q_n = 1; l.kv_slot = 0; l.kv_n = 2;
        l.q_start = l.kv_start = 0;
        l.masked = 0;
        l.final_from = ((int)n == last[a.qi] || (int)n + 1 == last[a.qi]) ? 0 : s.C;
        l.local = 0;
        out.push_back(l);
        batched = true;
      }
    }
    if (!batched)
      for (size_t m = n; m < e; ++m) single((int)m, 0);
    n = e;
  }
  return out;
}

// ------------------------------------------------------------- buffers --
struct RingWs {
  size_t q = 0, kv0 = 0, kv1 = 0, o_acc = 0, lse_acc = 0, send = 0, recv = 0, total = 0;
};

static RingWs ring_ws(const attn_ring_params_t* p, int world) {
  RingWs w;
  const size_t es = dtype_size(p->dtype);
  const size_t B = p->batch, Hq = p->num_heads_q, Hkv = p->num_heads_kv, S = p->seq_local, D = p->head_dim;
  const bool zig = p->zigzag && world > 1;
  const size_t C = zig ? S / 2 : S;
  size_t off = 0;
  auto take = [&](size_t& at, size_t bytes) { at = off; off += align256(bytes); };
  take(w.q, zig ? B * Hq * S * D * es : 0);
  take(w.kv0, 2 * B * Hkv * S * D * es);
  take(w.kv1, 2 * B * Hkv * S * D * es);
  take(w.o_acc, B * Hq * S * D * 4);
  take(w.lse_acc, B * Hq * S * 4);
  const size_t chunk = zig ? (B * Hq * C * D + 2 * B * Hkv * C * D) * es + B * Hq * C * 4 : 0;
  take(w.send, chunk);
  take(w.recv, chunk);
  w.total = off;
  return w;
}

__global__ void fill_f32_kernel(float* x, long long n, float v) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    x[i] = v;
}

// rows [row0, row0 + n) of every (b, h) plane of a [planes][S][width] tensor <-> a packed [planes][n][width] buffer
static cudaError_t copy_rows(void* dst, size_t dst_rows, size_t dst_row0, const void* src, size_t src_rows,
                             size_t src_row0, size_t n, size_t planes, size_t row_bytes, cudaStream_t st) {
  return cudaMemcpy2DAsync(static_cast<char*>(dst) + dst_row0 * row_bytes, dst_rows * row_bytes,
                           static_cast<const char*>(src) + src_row0 * row_bytes, src_rows * row_bytes,
                           n * row_bytes, planes, cudaMemcpyDeviceToDevice, st);
}

}  // namespace ringhost
}  // namespace attnb200

struct attn_comm_s {
  ncclComm_t comm;
  int world, rank, device;
  cudaEvent_t ev[8];
  // Copy-engine K/V rotation (attnb200::ringhost::ce_ensure): two receive
  // slots of ce_slot bytes and a flags page of this rank, IPC-shared; the
  // next rank's slots and flags opened here.  Flags: [0] ready = hops whose
  // K/V have landed in this rank's slots, [kFlagDone] done = hops this rank
  // has finished with (compute and outgoing copy); both only grow, counted
  // from ce_epoch, which every rank advances alike.
  int ce_state = 0;  // 0 not set up, 1 in use, -1 unavailable (NCCL rotation)
  char* ce_buf = nullptr;
  size_t ce_slot = 0;
  unsigned long long* ce_flags = nullptr;
  char* ce_peer_buf = nullptr;
  unsigned long long* ce_peer_flags = nullptr;
  unsigned long long ce_epoch = 0;
};

namespace attnb200 {
namespace ringhost {

constexpr int kFlagDone = 16;          // done counter one 128-byte line after ready
constexpr size_t kFlagBytes = 256;

// Waits (one thread) until *flag >= target; gives up after ATTN_WAIT_NS, or
// when another wait already failed, recording a status code instead.
__global__ void ce_wait_kernel(const unsigned long long* flag, unsigned long long target) {
  const uint64_t t0 = globaltimer();
  while (true) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    if (v >= target) return;
    if (status_now() != 0) return;
    if (globaltimer() - t0 > ATTN_WAIT_NS) {
      atomicCAS(&g_status, 0, kStatusTimeoutOther);
      return;
    }
    __nanosleep(256);
  }
}

// *flag = value with release semantics at system scope (flag may be a peer's):
// everything this stream did before -- a copy into the peer's slot -- is
// visible to whoever acquires the new value.
__global__ void ce_signal_kernel(unsigned long long* flag, unsigned long long value) {
  __threadfence_system();
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(value) : "memory");
}

// All-gather of one fixed-size host record per rank through the comm (setup
// only: synchronous).
static int ce_all_gather(attn_comm_s* c, const void* rec, size_t bytes, void* all, cudaStream_t st) {
  const NcclFns* f = nccl();
  char* d = nullptr;
  if (cudaMalloc(&d, bytes * (c->world + 1)) != cudaSuccess) return ATTN_ERR_CUDA;
  int rc = ATTN_OK;
  if (cudaMemcpyAsync(d, rec, bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) rc = ATTN_ERR_CUDA;
  if (rc == ATTN_OK) rc = nccl_status(f->all_gather(d, d + bytes, bytes, ncclUint8, c->comm, st), "ncclAllGather");
  if (rc == ATTN_OK && cudaMemcpyAsync(all, d + bytes, bytes * c->world, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    rc = ATTN_ERR_CUDA;
  if (rc == ATTN_OK && cudaStreamSynchronize(st) != cudaSuccess) rc = ATTN_ERR_CUDA;
  cudaFree(d);
  return rc;
}

static void ce_release(attn_comm_s* c) {
  if (c->ce_peer_buf) cudaIpcCloseMemHandle(c->ce_peer_buf);
  if (c->ce_peer_flags) cudaIpcCloseMemHandle(c->ce_peer_flags);
  if (c->ce_buf) cudaFree(c->ce_buf);
  c->ce_peer_buf = nullptr;
  c->ce_peer_flags = nullptr;
  c->ce_buf = nullptr;
  c->ce_slot = 0;
}

// Makes the copy-engine rotation ready for slots of `slot` bytes: a collective
// call (every rank of the comm, same sizes, same order).  Returns ATTN_OK with
// c->ce_state == 1 when every rank has its slots and its next rank's slots
// and flags mapped, ATTN_OK with ce_state == -1 when some rank could not (the
// caller then rotates with NCCL), or an error code.
static int ce_ensure(attn_comm_s* c, size_t slot, cudaStream_t st) {
  if (c->world < 2 || c->ce_state < 0) return ATTN_OK;
  if (c->ce_state == 1 && slot <= c->ce_slot) return ATTN_OK;
  // Nobody may still be copying into or reading the old slots.
  if (cudaDeviceSynchronize() != cudaSuccess) return ATTN_ERR_CUDA;
  struct Rec {
    cudaIpcMemHandle_t buf, flags;
    int ok;
  } mine{}, *all = new Rec[c->world];
  int rc = ce_all_gather(c, &mine, sizeof(Rec), all, st);  // barrier: every rank is past its old slots
  if (rc != ATTN_OK) {
    delete[] all;
    return rc;
  }
  ce_release(c);
  bool ok = true;
  if (!c->ce_flags) {
    ok = cudaMalloc(&c->ce_flags, kFlagBytes) == cudaSuccess && cudaMemset(c->ce_flags, 0, kFlagBytes) == cudaSuccess;
    if (!ok) c->ce_flags = nullptr;
  }
  ok = ok && cudaMalloc(&c->ce_buf, 2 * slot) == cudaSuccess;
  ok = ok && cudaIpcGetMemHandle(&mine.buf, c->ce_buf) == cudaSuccess;
  ok = ok && cudaIpcGetMemHandle(&mine.flags, c->ce_flags) == cudaSuccess;
  mine.ok = ok ? 1 : 0;
  rc = ce_all_gather(c, &mine, sizeof(Rec), all, st);
  if (rc == ATTN_OK && ok) {
    const Rec& nx = all[(c->rank + 1) % c->world];
    void* pb = nullptr;
    void* pf = nullptr;
    ok = nx.ok && cudaIpcOpenMemHandle(&pb, nx.buf, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    if (ok) c->ce_peer_buf = static_cast<char*>(pb);
    ok = ok && cudaIpcOpenMemHandle(&pf, nx.flags, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    if (ok) c->ce_peer_flags = static_cast<unsigned long long*>(pf);
  }
  cudaGetLastError();  // a failed IPC call is answered below, not left pending
  // Every rank must take the same rotation: agree on the outcome.
  mine.ok = (rc == ATTN_OK && ok) ? 1 : 0;
  if (rc == ATTN_OK) rc = ce_all_gather(c, &mine, sizeof(Rec), all, st);
  bool all_ok = rc == ATTN_OK;
  for (int i = 0; all_ok && i < c->world; ++i) all_ok = all[i].ok != 0;
  delete[] all;
  if (rc != ATTN_OK) return rc;
  if (!all_ok) {
    ce_release(c);
    c->ce_state = -1;
    fprintf(stderr, "attnb200: ring K/V over copy engines unavailable; rotating with NCCL\n");
    return ATTN_OK;
  }
  c->ce_slot = slot;
  c->ce_state = 1;
  return ATTN_OK;
}

}  // namespace ringhost
}  // namespace attnb200

extern "C" {

int attn_comm_unique_id(void* id, size_t bytes) {
  using namespace attnb200::ringhost;
  if (!id || bytes < sizeof(ncclUniqueId)) return ATTN_ERR_INVALID;
  const NcclFns* f = nccl();
  if (!f) return ATTN_ERR_NCCL;
  ncclUniqueId u;
  const int rc = nccl_status(f->get_unique_id(&u), "ncclGetUniqueId");
  if (rc != ATTN_OK) return rc;
  memcpy(id, &u, sizeof(u));
  return ATTN_OK;
}

int attn_comm_init(attn_comm_t* out, int32_t world, int32_t rank, const void* id, size_t bytes) {
  using namespace attnb200::ringhost;
  if (!out || !id || bytes < sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world) return ATTN_ERR_INVALID;
  *out = nullptr;
  const NcclFns* f = nccl();
  if (!f) return ATTN_ERR_NCCL;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ATTN_ERR_CUDA;
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  attn_comm_s* c = new attn_comm_s();
  c->world = world;
  c->rank = rank;
  c->device = dev;
  for (auto& e : c->ev) {
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      delete c;
      return ATTN_ERR_CUDA;
    }
  }
  const int rc = nccl_status(f->init_rank(&c->comm, world, u, rank), "ncclCommInitRank");
  if (rc != ATTN_OK) {
    for (auto& e : c->ev) cudaEventDestroy(e);
    delete c;
    return rc;
  }
  *out = c;
  return ATTN_OK;
}

int attn_comm_destroy(attn_comm_t c) {
  using namespace attnb200::ringhost;
  if (!c) return ATTN_ERR_INVALID;
  const NcclFns* f = nccl();
  int rc = ATTN_OK;
  ce_release(c);
  if (c->ce_flags) cudaFree(c->ce_flags);
  if (f) rc = nccl_status(f->destroy(c->comm), "ncclCommDestroy");
  for (auto& e : c->ev) cudaEventDestroy(e);
  delete c;
  return rc;
}

int attn_ring_plan(int32_t world, int32_t rank, int32_t seq_local, int32_t zigzag, int32_t has_band, int64_t band_lo,
                   int64_t band_hi, int32_t position_free, int64_t* launches, int32_t max_launches) {
  using namespace attnb200::ringhost;
  if (world < 1 || rank < 0 || rank >= world || seq_local < 1 || (zigzag && world > 1 && seq_local % 2) ||
      max_launches < 0 || (max_launches > 0 && !launches))
    return -ATTN_ERR_INVALID;
  Sched s{world, rank, zigzag && world > 1 ? 1 : 0, 0, has_band != 0, band_lo, band_hi};
  s.C = s.zig ? seq_local / 2 : seq_local;
  const std::vector<Launch> L = plan(s, position_free != 0);
  for (int n = 0; n < (int)L.size() && n < max_launches; ++n) {
    int64_t* o = launches + 10 * n;
    o[0] = L[n].hop; o[1] = L[n].q_slot; o[2] = L[n].q_n; o[3] = L[n].kv_slot; o[4] = L[n].kv_n;
    o[5] = L[n].q_start; o[6] = L[n].kv_start; o[7] = L[n].masked; o[8] = L[n].final_from; o[9] = L[n].local;
  }
  return (int)L.size();
}

size_t attn_ring_fwd_workspace_size(const attn_ring_params_t* p, int32_t world) {
  return p && world >= 1 ? attnb200::ringhost::ring_ws(p, world).total : 0;
}

}  // extern "C"

namespace attnb200 {
namespace ringhost {

template <int D, bool BF16>
static int launch_pair(const attn_ring_params_t* p, const Launch& l, int C, const void* qbuf, const char* kvbuf,
                       void* outbuf, float* o_acc, float* lse_acc, cudaStream_t st) {
  const size_t es = 2;
  const int64_t S = p->seq_local;
  attn_fwd_params_t f;
  memset(&f, 0, sizeof(f));
  f.dtype = p->dtype;
  f.batch = p->batch; f.num_heads_q = p->num_heads_q; f.num_heads_kv = p->num_heads_kv;
  f.seq_q = l.q_n * C; f.seq_kv = l.kv_n * C; f.head_dim = D;
  const size_t kv_plane = (size_t)p->batch * p->num_heads_kv * S * D * es;  // K then V in one buffer
  f.q = static_cast<const char*>(qbuf) + (size_t)l.q_slot * C * D * es;
  f.k = kvbuf + (size_t)l.kv_slot * C * D * es;
  f.v = kvbuf + kv_plane + (size_t)l.kv_slot * C * D * es;
  f.out = static_cast<char*>(outbuf) + (size_t)l.q_slot * C * D * es;
  const int64_t qs[3] = {p->num_heads_q * S * D, S * D, D}, ks[3] = {p->num_heads_kv * S * D, S * D, D};
  for (int i = 0; i < 3; ++i) {
    f.q_strides[i] = qs[i]; f.o_strides[i] = qs[i]; f.k_strides[i] = ks[i]; f.v_strides[i] = ks[i];
  }
  f.softmax_scale = p->softmax_scale;
  if (l.masked) {
    f.mask.has_band = p->has_band;
    f.mask.band_lo = p->band_lo;
    f.mask.band_hi = p->band_hi;
    f.mask.alibi_slopes = p->alibi_slopes;
    f.mask.q_offset = l.q_start;
    f.mask.kv_offset = l.kv_start;
  }
  RingAcc acc{o_acc, lse_acc, (int)S, l.q_slot * C, l.final_from};
  return launch_sm100_fwd2<D, BF16>(&f, nullptr, nullptr, nullptr, nullptr, st, &acc);
}

static int launch_pair_any(const attn_ring_params_t* p, const Launch& l, int C, const void* qbuf, const char* kvbuf,
                           void* outbuf, float* o_acc, float* lse_acc, cudaStream_t st) {
  const bool bf = p->dtype == ATTN_BF16;
  if (p->head_dim == 128)
    return bf ? launch_pair<128, true>(p, l, C, qbuf, kvbuf, outbuf, o_acc, lse_acc, st)
              : launch_pair<128, false>(p, l, C, qbuf, kvbuf, outbuf, o_acc, lse_acc, st);
  return bf ? launch_pair<64, true>(p, l, C, qbuf, kvbuf, outbuf, o_acc, lse_acc, st)
            : launch_pair<64, false>(p, l, C, qbuf, kvbuf, outbuf, o_acc, lse_acc, st);
}

}  // namespace ringhost
}  // namespace attnb200

extern "C" int attn_ring_fwd(const attn_ring_params_t* p, attn_comm_t comm, void* compute_stream, void* comm_stream) {
  using namespace attnb200;
  using namespace attnb200::ringhost;
  if (!p || !comm || !p->q || !p->k || !p->v || !p->out) return ATTN_ERR_INVALID;
  if (p->batch <= 0 || p->num_heads_q <= 0 || p->num_heads_kv <= 0 || p->seq_local <= 0 ||
      p->num_heads_q % p->num_heads_kv)
    return ATTN_ERR_INVALID;
  if ((p->dtype != ATTN_BF16 && p->dtype != ATTN_F16) || (p->head_dim != 64 && p->head_dim != 128))
    return ATTN_ERR_UNSUPPORTED;
  // Every query must keep its own key (the diagonal block is always kept), so
  // every row of the result is written by some launch.
  if (p->has_band && (p->band_lo > 0 || p->band_hi < 0)) return ATTN_ERR_UNSUPPORTED;
  const int P = comm->world, r = comm->rank;
  const bool zig = p->zigzag && P > 1;
  if (zig && p->seq_local % 2) return ATTN_ERR_INVALID;
  const RingWs w = ring_ws(p, P);
  if (!p->workspace || p->workspace_bytes < w.total) return ATTN_ERR_WORKSPACE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(p->q) | reinterpret_cast<uintptr_t>(p->k) |
                       reinterpret_cast<uintptr_t>(p->v) | reinterpret_cast<uintptr_t>(p->out) |
                       reinterpret_cast<uintptr_t>(p->workspace);
  if (al % 16) return ATTN_ERR_INVALID;
  const NcclFns* f = nccl();
  if (!f) return ATTN_ERR_NCCL;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(compute_stream);
  cudaStream_t ms = reinterpret_cast<cudaStream_t>(comm_stream);
  char* ws = static_cast<char*>(p->workspace);
  const size_t es = dtype_size(p->dtype);
  const size_t B = p->batch, Hq = p->num_heads_q, Hkv = p->num_heads_kv, S = p->seq_local, D = p->head_dim;
  const int C = zig ? (int)(S / 2) : (int)S;
  const size_t row = D * es;
  const size_t kv_plane = B * Hkv * S * D * es;
  // K/V slots: the copy-engine rotation's IPC-shared slots when every rank
  // has them (the next hop's K/V goes straight into the next rank's slot
  // with cudaMemcpyAsync, no SMs), else the workspace with NCCL send/recv.
  {
    const int crc = ce_ensure(comm, 2 * kv_plane, ms);
    if (crc != ATTN_OK) return crc;
  }
  const bool ce = P > 1 && comm->ce_state == 1;
  char* kvb[2] = {ce ? comm->ce_buf : ws + w.kv0, ce ? comm->ce_buf + comm->ce_slot : ws + w.kv1};
  float* o_acc = reinterpret_cast<float*>(ws + w.o_acc);
  float* lse_acc = reinterpret_cast<float*>(ws + w.lse_acc);
  void* qbuf = zig ? static_cast<void*>(ws + w.q) : const_cast<void*>(p->q);
  // Finished rows are written in place: ring slot 0 is the caller's rows
  // [0, C); slot 1's rows pass through out rows [C, 2C) on their way to the
  // mirror rank, whose chunk then replaces them (all on the comm stream).
  void* obuf = p->out;
  cudaEvent_t ev_in = comm->ev[0], ev_redeal = comm->ev[1], ev_hop[2] = {comm->ev[2], comm->ev[3]},
              ev_recv[2] = {comm->ev[4], comm->ev[5]}, ev_local = comm->ev[6], ev_back = comm->ev[7];
  const ncclDataType_t u8 = ncclUint8;
  int rc = ATTN_OK;
#define ATTN_CK(x)                        \
  do {                                    \
    if ((x) != cudaSuccess) return ATTN_ERR_CUDA; \
  } while (0)
#define ATTN_NK(x, what)                  \
  do {                                    \
    rc = nccl_status((x), what);          \
    if (rc != ATTN_OK) return rc;         \
  } while (0)

  // ---- running result: empty (lse -inf); acc rows are not read until written ----
  {
    const long long n = (long long)(B * Hq * S);
    fill_f32_kernel<<<(unsigned)std::min<long long>((n + 255) / 256, 1184), 256, 0, cs>>>(lse_acc, n, -INFINITY);
    if ((rc = launch_status()) != ATTN_OK) return rc;
  }
  // ---- re-deal into the ring layout: q, k, v rows [0, C) stay, [C, 2C) come from the mirror ----
  ATTN_CK(cudaEventRecord(ev_in, cs));
  if (zig) {
    ATTN_CK(copy_rows(qbuf, S, 0, p->q, S, 0, C, B * Hq, row, cs));
    ATTN_CK(copy_rows(kvb[0], S, 0, p->k, S, 0, C, B * Hkv, row, cs));
    ATTN_CK(copy_rows(kvb[0] + kv_plane, S, 0, p->v, S, 0, C, B * Hkv, row, cs));
    const int m = r == P - 1 - r ? r : P - 1 - r;
    ATTN_CK(cudaStreamWaitEvent(ms, ev_in, 0));
    if (m == r) {  // middle rank of an odd ring: both chunks are its own
      ATTN_CK(copy_rows(qbuf, S, C, p->q, S, C, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(kvb[0], S, C, p->k, S, C, C, B * Hkv, row, ms));
      ATTN_CK(copy_rows(kvb[0] + kv_plane, S, C, p->v, S, C, C, B * Hkv, row, ms));
    } else {
      char* snd = ws + w.send;
      char* rcv = ws + w.recv;
      const size_t qb = B * Hq * C * row, kb = B * Hkv * C * row;
      ATTN_CK(copy_rows(snd, C, 0, p->q, S, C, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(snd + qb, C, 0, p->k, S, C, C, B * Hkv, row, ms));
      ATTN_CK(copy_rows(snd + qb + kb, C, 0, p->v, S, C, C, B * Hkv, row, ms));
      ATTN_NK(f->group_start(), "ncclGroupStart");
      ATTN_NK(f->send(snd, qb + 2 * kb, u8, m, comm->comm, ms), "ncclSend");
      ATTN_NK(f->recv(rcv, qb + 2 * kb, u8, m, comm->comm, ms), "ncclRecv");
      ATTN_NK(f->group_end(), "ncclGroupEnd");
      ATTN_CK(copy_rows(qbuf, S, C, rcv, C, 0, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(kvb[0], S, C, rcv + qb, C, 0, C, B * Hkv, row, ms));
      ATTN_CK(copy_rows(kvb[0] + kv_plane, S, C, rcv + qb + kb, C, 0, C, B * Hkv, row, ms));
    }
    ATTN_CK(cudaEventRecord(ev_redeal, ms));
  } else {
    ATTN_CK(cudaMemcpyAsync(kvb[0], p->k, kv_plane, cudaMemcpyDeviceToDevice, cs));
    ATTN_CK(cudaMemcpyAsync(kvb[0] + kv_plane, p->v, kv_plane, cudaMemcpyDeviceToDevice, cs));
  }
  ATTN_CK(cudaEventRecord(ev_local, cs));  // this rank's own K/V rows are in the ring buffer

  // ---- hops ----
  Sched s{P, r, zig ? 1 : 0, C, p->has_band != 0, p->band_lo, p->band_hi};
  const bool position_free = p->alibi_slopes == nullptr;
  const std::vector<Launch> L = plan(s, position_free);
  size_t n = 0;
  bool redeal_waited = !zig;
  // Copy-engine counters of this call: hop i's K/V has landed in a rank's
  // slot i&1 when its ready >= base + i; a rank is done with hop i (compute
  // and its outgoing copy) when its done >= base + i + 1.
  const unsigned long long base = comm->ce_epoch;
  if (ce) comm->ce_epoch += P;
  for (int i = 0; i < P; ++i) {
    // start moving this hop's K/V on to rank r+1
    if (i + 1 < P) {
      // (the re-deal's rows were written on the comm stream itself)
      if (i == 0) ATTN_CK(cudaStreamWaitEvent(ms, ev_local, 0));
      if (ce) {
        // slot i&1 holds this hop's K/V once it has landed (hop 0: own rows);
        // rank r+1's slot (i+1)&1 is free once it is done with hop i-1
        if (i > 0) ce_wait_kernel<<<1, 1, 0, ms>>>(comm->ce_flags, base + i);
        ce_wait_kernel<<<1, 1, 0, ms>>>(comm->ce_peer_flags + kFlagDone, base + i);
        ATTN_CK(cudaMemcpyAsync(comm->ce_peer_buf + ((i + 1) & 1) * comm->ce_slot, kvb[i & 1], 2 * kv_plane,
                                cudaMemcpyDeviceToDevice, ms));
        ce_signal_kernel<<<1, 1, 0, ms>>>(comm->ce_peer_flags, base + i + 1);
        if ((rc = launch_status(i > 0 ? 3 : 2)) != ATTN_OK) return rc;
      } else {
        // (the buffer it lands in was last read by hop i-1)
        if (i > 0) ATTN_CK(cudaStreamWaitEvent(ms, ev_hop[(i - 1) & 1], 0));
        ATTN_NK(f->group_start(), "ncclGroupStart");
        ATTN_NK(f->send(kvb[i & 1], 2 * kv_plane, u8, (r + 1) % P, comm->comm, ms), "ncclSend");
        ATTN_NK(f->recv(kvb[(i + 1) & 1], 2 * kv_plane, u8, (r - 1 + P) % P, comm->comm, ms), "ncclRecv");
        ATTN_NK(f->group_end(), "ncclGroupEnd");
      }
      ATTN_CK(cudaEventRecord(ev_recv[i & 1], ms));  // CE: this hop's outgoing copy; NCCL: next hop's K/V
    }
    if (ce && i > 0) {
      ce_wait_kernel<<<1, 1, 0, cs>>>(comm->ce_flags, base + i);  // this hop's K/V has landed
      if ((rc = launch_status()) != ATTN_OK) return rc;
    }
    for (; n < L.size() && L[n].hop == i; ++n) {
      if (!L[n].local && !redeal_waited) {
        ATTN_CK(cudaStreamWaitEvent(cs, ev_redeal, 0));
        redeal_waited = true;
      }
      rc = launch_pair_any(p, L[n], C, qbuf, kvb[i & 1], obuf, o_acc, lse_acc, cs);
      if (rc != ATTN_OK) return rc;
    }
    ATTN_CK(cudaEventRecord(ev_hop[i & 1], cs));
    if (i + 1 < P) ATTN_CK(cudaStreamWaitEvent(cs, ev_recv[i & 1], 0));
    if (ce) {
      ce_signal_kernel<<<1, 1, 0, cs>>>(comm->ce_flags + kFlagDone, base + i + 1);
      if ((rc = launch_status()) != ATTN_OK) return rc;
    }
  }

  // ---- results back to the public layout ----
  if (zig) {
    const int m = r == P - 1 - r ? r : P - 1 - r;
    // rows [0, C) are this rank's own and already in place
    if (p->lse) ATTN_CK(copy_rows(p->lse, S, 0, lse_acc, S, 0, C, B * Hq, 4, cs));
    ATTN_CK(cudaEventRecord(ev_hop[0], cs));
    ATTN_CK(cudaStreamWaitEvent(ms, ev_hop[0], 0));
    if (m == r) {
      if (p->lse) ATTN_CK(copy_rows(p->lse, S, C, lse_acc, S, C, C, B * Hq, 4, ms));
    } else {
      char* snd = ws + w.send;
      char* rcv = ws + w.recv;
      const size_t ob = B * Hq * C * row, lb = B * Hq * C * 4;
      ATTN_CK(copy_rows(snd, C, 0, obuf, S, C, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(snd + ob, C, 0, lse_acc, S, C, C, B * Hq, 4, ms));
      ATTN_NK(f->group_start(), "ncclGroupStart");
      ATTN_NK(f->send(snd, ob + lb, u8, m, comm->comm, ms), "ncclSend");
      ATTN_NK(f->recv(rcv, ob + lb, u8, m, comm->comm, ms), "ncclRecv");
      ATTN_NK(f->group_end(), "ncclGroupEnd");
      ATTN_CK(copy_rows(p->out, S, C, rcv, C, 0, C, B * Hq, row, ms));
      if (p->lse) ATTN_CK(copy_rows(p->lse, S, C, rcv + ob, C, 0, C, B * Hq, 4, ms));
    }
    ATTN_CK(cudaEventRecord(ev_back, ms));
    ATTN_CK(cudaStreamWaitEvent(cs, ev_back, 0));
  } else if (p->lse) {
    ATTN_CK(cudaMemcpyAsync(p->lse, lse_acc, B * Hq * S * 4, cudaMemcpyDeviceToDevice, cs));
  }
#undef ATTN_CK
#undef ATTN_NK
  return ATTN_OK;
}

// ------------------------------------------------------------- backward --
namespace attnb200 {
namespace ringhost {

// dst[plane][row0 + r][:] += src[plane][r][:] (fp32 += tensor dtype), r < rows.
template <typename T>
__global__ void add_rows_kernel(float* dst, long long dst_plane, long long row0, const T* src, long long rows,
                                int D, long long planes) {
  const long long per = rows * D, n = planes * per;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long pl = i / per, w = i % per;
    dst[pl * dst_plane + row0 * D + w] += to_f32(src[i]);
  }
}
__global__ void add_f32_kernel(float* dst, const float* src, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] += src[i];
}
template <typename T>
__global__ void to_dtype_kernel(T* dst, const float* src, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = from_f32<T>(src[i]);
}

static unsigned grid_for(long long n) { return (unsigned)std::min<long long>((n + 255) / 256, 148 * 16); }

struct RingBwdWs {
  size_t q = 0, o = 0, dout = 0, lse = 0, lse_slot = 0, kv0 = 0, kv1 = 0, acc0 = 0, acc1 = 0, loc0 = 0, loc1 = 0,
         dq_acc = 0, dq_p = 0, dk_p = 0, dv_p = 0, bwd = 0, send = 0, recv = 0, total = 0;
  size_t bwd_bytes = 0;
};

static attn_bwd_params_t pair_params(const attn_ring_bwd_params_t* p, int nq, int nkv) {
  attn_bwd_params_t b;
  memset(&b, 0, sizeof(b));
  b.dtype = p->dtype;
  b.batch = p->batch; b.num_heads_q = p->num_heads_q; b.num_heads_kv = p->num_heads_kv;
  b.seq_q = nq; b.seq_kv = nkv; b.head_dim = p->head_dim;
  b.softmax_scale = p->softmax_scale;
  return b;
}

static RingBwdWs ring_bwd_ws(const attn_ring_bwd_params_t* p, int world) {
  RingBwdWs w;
  const size_t es = dtype_size(p->dtype);
  const size_t B = p->batch, Hq = p->num_heads_q, Hkv = p->num_heads_kv, S = p->seq_local, D = p->head_dim;
  const bool zig = p->zigzag && world > 1;
  const size_t C = zig ? S / 2 : S;
  const size_t qt = B * Hq * S * D * es, kvt = B * Hkv * S * D * es;
  size_t off = 0;
  auto take = [&](size_t& at, size_t bytes) { at = off; off += align256(bytes); };
  take(w.q, zig ? qt : 0);
  take(w.o, zig ? qt : 0);
  take(w.dout, zig ? qt : 0);
  take(w.lse, B * Hq * S * 4);
  take(w.lse_slot, B * Hq * S * 4);  // [slot][B][Hq][C]
  take(w.kv0, 2 * kvt);
  take(w.kv1, 2 * kvt);
  take(w.acc0, 2 * B * Hkv * S * D * 4);
  take(w.acc1, 2 * B * Hkv * S * D * 4);
  take(w.loc0, 2 * B * Hkv * S * D * 4);
  take(w.loc1, 2 * B * Hkv * S * D * 4);
  take(w.dq_acc, B * Hq * S * D * 4);
  take(w.dq_p, qt);
  take(w.dk_p, kvt);
  take(w.dv_p, kvt);
  attn_bwd_params_t b = pair_params(p, (int)S, (int)S);
  b.q = b.k = b.v = b.out = b.d_out = b.dq = b.dk = b.dv = reinterpret_cast<void*>(256);
  for (int i = 0; i < 3; ++i) {
    const int64_t qs[3] = {(int64_t)(Hq * S * D), (int64_t)(S * D), (int64_t)D},
                  ks[3] = {(int64_t)(Hkv * S * D), (int64_t)(S * D), (int64_t)D};
    b.q_strides[i] = b.o_strides[i] = b.do_strides[i] = b.dq_strides[i] = qs[i];
    b.k_strides[i] = b.v_strides[i] = b.dk_strides[i] = b.dv_strides[i] = ks[i];
  }
  b.mask.has_band = p->has_band;
  b.mask.band_lo = p->band_lo;
  b.mask.band_hi = p->band_hi;
  w.bwd_bytes = std::max<size_t>(attn_bwd_workspace_size(&b), 16);
  take(w.bwd, w.bwd_bytes);
  const size_t in_chunk = zig ? (3 * B * Hq * C * D + 2 * B * Hkv * C * D) * es + B * Hq * C * 4 : 0;
  const size_t out_chunk = zig ? (B * Hq * C * D + 2 * B * Hkv * C * D) * es : 0;
  take(w.send, std::max(in_chunk, out_chunk));
  take(w.recv, std::max(in_chunk, out_chunk));
  w.total = off;
  return w;
}

}  // namespace ringhost
}  // namespace attnb200

extern "C" size_t attn_ring_bwd_workspace_size(const attn_ring_bwd_params_t* p, int32_t world) {
  return p && world >= 1 ? attnb200::ringhost::ring_bwd_ws(p, world).total : 0;
}

extern "C" int attn_ring_bwd(const attn_ring_bwd_params_t* p, attn_comm_t comm, void* compute_stream,
                             void* comm_stream) {
  using namespace attnb200;
  using namespace attnb200::ringhost;
  if (!p || !comm || !p->q || !p->k || !p->v || !p->out || !p->lse || !p->d_out || !p->dq || !p->dk || !p->dv)
    return ATTN_ERR_INVALID;
  if (p->batch <= 0 || p->num_heads_q <= 0 || p->num_heads_kv <= 0 || p->seq_local <= 0 ||
      p->num_heads_q % p->num_heads_kv)
    return ATTN_ERR_INVALID;
  if ((p->dtype != ATTN_BF16 && p->dtype != ATTN_F16) || (p->head_dim != 64 && p->head_dim != 128))
    return ATTN_ERR_UNSUPPORTED;
  if (p->has_band && (p->band_lo > 0 || p->band_hi < 0)) return ATTN_ERR_UNSUPPORTED;
  const int P = comm->world, r = comm->rank;
  const bool zig = p->zigzag && P > 1;
  if (zig && p->seq_local % 2) return ATTN_ERR_INVALID;
  const RingBwdWs w = ring_bwd_ws(p, P);
  if (!p->workspace || p->workspace_bytes < w.total) return ATTN_ERR_WORKSPACE;
  const NcclFns* f = nccl();
  if (!f) return ATTN_ERR_NCCL;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(compute_stream);
  cudaStream_t ms = reinterpret_cast<cudaStream_t>(comm_stream);
  char* ws = static_cast<char*>(p->workspace);
  const size_t es = dtype_size(p->dtype);
  const size_t B = p->batch, Hq = p->num_heads_q, Hkv = p->num_heads_kv, S = p->seq_local, D = p->head_dim;
  const int C = zig ? (int)(S / 2) : (int)S;
  const size_t row = D * es, frow = D * 4;
  const size_t kv_plane = B * Hkv * S * D * es, acc_plane = B * Hkv * S * D;  // bytes / floats
  const void* qb = zig ? static_cast<const void*>(ws + w.q) : p->q;
  const void* ob = zig ? static_cast<const void*>(ws + w.o) : p->out;
  const void* db = zig ? static_cast<const void*>(ws + w.dout) : p->d_out;
  float* lse_r = reinterpret_cast<float*>(ws + w.lse);
  float* lse_s = reinterpret_cast<float*>(ws + w.lse_slot);
  char* kvb[2] = {ws + w.kv0, ws + w.kv1};
  float* acc[2] = {reinterpret_cast<float*>(ws + w.acc0), reinterpret_cast<float*>(ws + w.acc1)};
  float* loc[2] = {reinterpret_cast<float*>(ws + w.loc0), reinterpret_cast<float*>(ws + w.loc1)};
  float* dq_acc = reinterpret_cast<float*>(ws + w.dq_acc);
  char* dq_p = ws + w.dq_p;
  char* dk_p = ws + w.dk_p;
  char* dv_p = ws + w.dv_p;
  cudaEvent_t ev_in = comm->ev[0], ev_redeal = comm->ev[1], ev_hop[2] = {comm->ev[2], comm->ev[3]},
              ev_recv[2] = {comm->ev[4], comm->ev[5]}, ev_local = comm->ev[6], ev_back = comm->ev[7];
  // (the accumulator chain reuses ev_hop: a hop's partials are done when its
  // compute is, and the chain's last add of a local buffer precedes its reuse
  // two hops later on the comm stream, which the compute stream waits for
  // through ev_recv of the hop in between)
  const ncclDataType_t u8 = ncclUint8;
  int rc = ATTN_OK;
  const bool bf = p->dtype == ATTN_BF16;
#define ATTN_CK(x)                                \
  do {                                            \
    if ((x) != cudaSuccess) return ATTN_ERR_CUDA; \
  } while (0)
#define ATTN_NK(x, what)          \
  do {                            \
    rc = nccl_status((x), what);  \
    if (rc != ATTN_OK) return rc; \
  } while (0)
  const int m = zig ? (r == P - 1 - r ? r : P - 1 - r) : r;

  // ---- ring layout of q, out, d_out, lse (query side) and k, v ----
  ATTN_CK(cudaEventRecord(ev_in, cs));
  ATTN_CK(cudaMemsetAsync(dq_acc, 0, B * Hq * S * D * 4, cs));
  ATTN_CK(cudaMemsetAsync(acc[0], 0, 2 * acc_plane * 4, ms));
  if (zig) {
    ATTN_CK(copy_rows(const_cast<void*>(qb), S, 0, p->q, S, 0, C, B * Hq, row, cs));
    ATTN_CK(copy_rows(const_cast<void*>(ob), S, 0, p->out, S, 0, C, B * Hq, row, cs));
    ATTN_CK(copy_rows(const_cast<void*>(db), S, 0, p->d_out, S, 0, C, B * Hq, row, cs));
    ATTN_CK(copy_rows(lse_r, S, 0, p->lse, S, 0, C, B * Hq, 4, cs));
    ATTN_CK(copy_rows(kvb[0], S, 0, p->k, S, 0, C, B * Hkv, row, cs));
    ATTN_CK(copy_rows(kvb[0] + kv_plane, S, 0, p->v, S, 0, C, B * Hkv, row, cs));
    ATTN_CK(cudaStreamWaitEvent(ms, ev_in, 0));
    if (m == r) {
      ATTN_CK(copy_rows(const_cast<void*>(qb), S, C, p->q, S, C, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(const_cast<void*>(ob), S, C, p->out, S, C, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(const_cast<void*>(db), S, C, p->d_out, S, C, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(lse_r, S, C, p->lse, S, C, C, B * Hq, 4, ms));
      ATTN_CK(copy_rows(kvb[0], S, C, p->k, S, C, C, B * Hkv, row, ms));
      ATTN_CK(copy_rows(kvb[0] + kv_plane, S, C, p->v, S, C, C, B * Hkv, row, ms));
    } else {
      char* snd = ws + w.send;
      char* rcv = ws + w.recv;
      const size_t qc = B * Hq * C * row, kc = B * Hkv * C * row, lc = B * Hq * C * 4;
      const void* qsrc[3] = {p->q, p->out, p->d_out};
      void* qdst[3] = {const_cast<void*>(qb), const_cast<void*>(ob), const_cast<void*>(db)};
      for (int t = 0; t < 3; ++t) ATTN_CK(copy_rows(snd + t * qc, C, 0, qsrc[t], S, C, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(snd + 3 * qc, C, 0, p->lse, S, C, C, B * Hq, 4, ms));
      ATTN_CK(copy_rows(snd + 3 * qc + lc, C, 0, p->k, S, C, C, B * Hkv, row, ms));
      ATTN_CK(copy_rows(snd + 3 * qc + lc + kc, C, 0, p->v, S, C, C, B * Hkv, row, ms));
      const size_t bytes = 3 * qc + lc + 2 * kc;
      ATTN_NK(f->group_start(), "ncclGroupStart");
      ATTN_NK(f->send(snd, bytes, u8, m, comm->comm, ms), "ncclSend");
      ATTN_NK(f->recv(rcv, bytes, u8, m, comm->comm, ms), "ncclRecv");
      ATTN_NK(f->group_end(), "ncclGroupEnd");
      for (int t = 0; t < 3; ++t) ATTN_CK(copy_rows(qdst[t], S, C, rcv + t * qc, C, 0, C, B * Hq, row, ms));
      ATTN_CK(copy_rows(lse_r, S, C, rcv + 3 * qc, C, 0, C, B * Hq, 4, ms));
      ATTN_CK(copy_rows(kvb[0], S, C, rcv + 3 * qc + lc, C, 0, C, B * Hkv, row, ms));
      ATTN_CK(copy_rows(kvb[0] + kv_plane, S, C, rcv + 3 * qc + lc + kc, C, 0, C, B * Hkv, row, ms));
    }
    ATTN_CK(cudaEventRecord(ev_redeal, ms));
    ATTN_CK(cudaStreamWaitEvent(cs, ev_redeal, 0));
  } else {
    ATTN_CK(cudaMemcpyAsync(lse_r, p->lse, B * Hq * S * 4, cudaMemcpyDeviceToDevice, cs));
    ATTN_CK(cudaMemcpyAsync(kvb[0], p->k, kv_plane, cudaMemcpyDeviceToDevice, cs));
    ATTN_CK(cudaMemcpyAsync(kvb[0] + kv_plane, p->v, kv_plane, cudaMemcpyDeviceToDevice, cs));
  }
  // per-slot contiguous LSE ([B][Hq][C] each) for launches over one q chunk
  for (int s = 0; s < (zig ? 2 : 1); ++s)
    ATTN_CK(copy_rows(lse_s + (size_t)s * B * Hq * C, C, 0, lse_r, S, (size_t)s * C, C, B * Hq, 4, cs));
  ATTN_CK(cudaEventRecord(ev_local, cs));

  Sched sc{P, r, zig ? 1 : 0, C, p->has_band != 0, p->band_lo, p->band_hi};
  const std::vector<Launch> L = plan(sc, p->alibi_slopes == nullptr);
  size_t n = 0;
  for (int i = 0; i < P; ++i) {
    float* lb = loc[i & 1];
    if (i + 1 < P) {
      if (i == 0) ATTN_CK(cudaStreamWaitEvent(ms, ev_local, 0));
      if (i > 0) ATTN_CK(cudaStreamWaitEvent(ms, ev_hop[(i - 1) & 1], 0));
      ATTN_NK(f->group_start(), "ncclGroupStart");
      ATTN_NK(f->send(kvb[i & 1], 2 * kv_plane, u8, (r + 1) % P, comm->comm, ms), "ncclSend");
      ATTN_NK(f->recv(kvb[(i + 1) & 1], 2 * kv_plane, u8, (r - 1 + P) % P, comm->comm, ms), "ncclRecv");
      ATTN_NK(f->group_end(), "ncclGroupEnd");
      ATTN_CK(cudaEventRecord(ev_recv[i & 1], ms));
    }
    // this hop's partial dK | dV of the visiting K/V
    ATTN_CK(cudaMemsetAsync(lb, 0, 2 * acc_plane * 4, cs));
    for (; n < L.size() && L[n].hop == i; ++n) {
      const Launch& l = L[n];
      const int nq = l.q_n * C, nkv = l.kv_n * C;
      attn_bwd_params_t b = pair_params(p, nq, nkv);
      b.q = static_cast<const char*>(qb) + (size_t)l.q_slot * C * row;
      b.out = static_cast<const char*>(ob) + (size_t)l.q_slot * C * row;
      b.d_out = static_cast<const char*>(db) + (size_t)l.q_slot * C * row;
      b.lse = l.q_n == 2 ? lse_r : lse_s + (size_t)l.q_slot * B * Hq * C;
      b.k = kvb[i & 1] + (size_t)l.kv_slot * C * row;
      b.v = kvb[i & 1] + kv_plane + (size_t)l.kv_slot * C * row;
      b.dq = dq_p; b.dk = dk_p; b.dv = dv_p;
      const int64_t qs[3] = {(int64_t)(Hq * S * D), (int64_t)(S * D), (int64_t)D},
                    ks[3] = {(int64_t)(Hkv * S * D), (int64_t)(S * D), (int64_t)D},
                    pq[3] = {(int64_t)Hq * nq * (int64_t)D, (int64_t)nq * (int64_t)D, (int64_t)D},
                    pk[3] = {(int64_t)Hkv * nkv * (int64_t)D, (int64_t)nkv * (int64_t)D, (int64_t)D};
      for (int t = 0; t < 3; ++t) {
        b.q_strides[t] = b.o_strides[t] = b.do_strides[t] = qs[t];
        b.k_strides[t] = b.v_strides[t] = ks[t];
        b.dq_strides[t] = pq[t];
        b.dk_strides[t] = b.dv_strides[t] = pk[t];
      }
      if (l.masked) {
        b.mask.has_band = p->has_band;
        b.mask.band_lo = p->band_lo;
        b.mask.band_hi = p->band_hi;
        b.mask.alibi_slopes = p->alibi_slopes;
        b.mask.q_offset = l.q_start;
        b.mask.kv_offset = l.kv_start;
      }
      b.workspace = ws + w.bwd;
      b.workspace_bytes = w.bwd_bytes;
      if ((rc = attn_bwd(&b, cs)) != ATTN_OK) return rc;
      const long long qrows = (long long)nq, krows = (long long)nkv;
      if (bf) {
        add_rows_kernel<__nv_bfloat16><<<grid_for(B * Hq * qrows * D), 256, 0, cs>>>(
            dq_acc, (long long)S * D, (long long)l.q_slot * C, reinterpret_cast<const __nv_bfloat16*>(dq_p), qrows,
            (int)D, (long long)(B * Hq));
        add_rows_kernel<__nv_bfloat16><<<grid_for(B * Hkv * krows * D), 256, 0, cs>>>(
            lb, (long long)S * D, (long long)l.kv_slot * C, reinterpret_cast<const __nv_bfloat16*>(dk_p), krows,
            (int)D, (long long)(B * Hkv));
        add_rows_kernel<__nv_bfloat16><<<grid_for(B * Hkv * krows * D), 256, 0, cs>>>(
            lb + acc_plane, (long long)S * D, (long long)l.kv_slot * C,
            reinterpret_cast<const __nv_bfloat16*>(dv_p), krows, (int)D, (long long)(B * Hkv));
      } else {
        add_rows_kernel<__half><<<grid_for(B * Hq * qrows * D), 256, 0, cs>>>(
            dq_acc, (long long)S * D, (long long)l.q_slot * C, reinterpret_cast<const __half*>(dq_p), qrows, (int)D,
            (long long)(B * Hq));
        add_rows_kernel<__half><<<grid_for(B * Hkv * krows * D), 256, 0, cs>>>(
            lb, (long long)S * D, (long long)l.kv_slot * C, reinterpret_cast<const __half*>(dk_p), krows, (int)D,
            (long long)(B * Hkv));
        add_rows_kernel<__half><<<grid_for(B * Hkv * krows * D), 256, 0, cs>>>(
            lb + acc_plane, (long long)S * D, (long long)l.kv_slot * C, reinterpret_cast<const __half*>(dv_p),
            krows, (int)D, (long long)(B * Hkv));
      }
      if ((rc = launch_status(3)) != ATTN_OK) return rc;
    }
    ATTN_CK(cudaEventRecord(ev_hop[i & 1], cs));
    // accumulator chain: acc[i&1] (arrived for this K/V) += this hop's
    // partials, then on to the next rank, which holds this K/V next hop;
    // after the P-th exchange each rank holds its own shard's dK | dV
    ATTN_CK(cudaStreamWaitEvent(ms, ev_hop[i & 1], 0));
    add_f32_kernel<<<grid_for(2 * acc_plane), 256, 0, ms>>>(acc[i & 1], lb, (long long)(2 * acc_plane));
    if ((rc = launch_status()) != ATTN_OK) return rc;
    if (P > 1) {
      ATTN_NK(f->group_start(), "ncclGroupStart");
      ATTN_NK(f->send(acc[i & 1], 2 * acc_plane * 4, u8, (r + 1) % P, comm->comm, ms), "ncclSend");
      ATTN_NK(f->recv(acc[(i + 1) & 1], 2 * acc_plane * 4, u8, (r - 1 + P) % P, comm->comm, ms), "ncclRecv");
      ATTN_NK(f->group_end(), "ncclGroupEnd");
    }
    if (i + 1 < P) {
      ATTN_CK(cudaStreamWaitEvent(cs, ev_recv[i & 1], 0));
      // the local buffer of hop i+1 was last added by the chain at hop i-1
      // (enqueued on the comm stream before the K/V exchange just waited for)
    }
  }
  float* own = acc[P & 1];  // this rank's dK | dV, ring layout (after P exchanges; P == 1: acc[1]? see below)
  if (P == 1) own = acc[0];

  // ---- results: convert, and return the mirror's rows ----
  ATTN_CK(cudaEventRecord(ev_back, ms));
  ATTN_CK(cudaStreamWaitEvent(cs, ev_back, 0));
  const long long nq_all = (long long)(B * Hq * S * D), nk_all = (long long)acc_plane;
  char* dq_t = dq_p;  // the partial buffers hold the converted ring-layout results now
  if (bf) {
    to_dtype_kernel<__nv_bfloat16><<<grid_for(nq_all), 256, 0, cs>>>(reinterpret_cast<__nv_bfloat16*>(dq_t), dq_acc,
                                                                      nq_all);
    to_dtype_kernel<__nv_bfloat16><<<grid_for(nk_all), 256, 0, cs>>>(reinterpret_cast<__nv_bfloat16*>(dk_p), own,
                                                                      nk_all);
    to_dtype_kernel<__nv_bfloat16><<<grid_for(nk_all), 256, 0, cs>>>(reinterpret_cast<__nv_bfloat16*>(dv_p),
                                                                      own + acc_plane, nk_all);
  } else {
    to_dtype_kernel<__half><<<grid_for(nq_all), 256, 0, cs>>>(reinterpret_cast<__half*>(dq_t), dq_acc, nq_all);
    to_dtype_kernel<__half><<<grid_for(nk_all), 256, 0, cs>>>(reinterpret_cast<__half*>(dk_p), own, nk_all);
    to_dtype_kernel<__half><<<grid_for(nk_all), 256, 0, cs>>>(reinterpret_cast<__half*>(dv_p), own + acc_plane,
                                                               nk_all);
  }
  if ((rc = launch_status(3)) != ATTN_OK) return rc;
  if (!zig) {
    ATTN_CK(cudaMemcpyAsync(p->dq, dq_t, (size_t)nq_all * es, cudaMemcpyDeviceToDevice, cs));
    ATTN_CK(cudaMemcpyAsync(p->dk, dk_p, (size_t)nk_all * es, cudaMemcpyDeviceToDevice, cs));
    ATTN_CK(cudaMemcpyAsync(p->dv, dv_p, (size_t)nk_all * es, cudaMemcpyDeviceToDevice, cs));
    return ATTN_OK;
  }
  ATTN_CK(copy_rows(p->dq, S, 0, dq_t, S, 0, C, B * Hq, row, cs));
  ATTN_CK(copy_rows(p->dk, S, 0, dk_p, S, 0, C, B * Hkv, row, cs));
  ATTN_CK(copy_rows(p->dv, S, 0, dv_p, S, 0, C, B * Hkv, row, cs));
  ATTN_CK(cudaEventRecord(ev_local, cs));
  ATTN_CK(cudaStreamWaitEvent(ms, ev_local, 0));
  if (m == r) {
    ATTN_CK(copy_rows(p->dq, S, C, dq_t, S, C, C, B * Hq, row, ms));
    ATTN_CK(copy_rows(p->dk, S, C, dk_p, S, C, C, B * Hkv, row, ms));
    ATTN_CK(copy_rows(p->dv, S, C, dv_p, S, C, C, B * Hkv, row, ms));
  } else {
    char* snd = ws + w.send;
    char* rcv = ws + w.recv;
    const size_t qc = B * Hq * C * row, kc = B * Hkv * C * row;
    ATTN_CK(copy_rows(snd, C, 0, dq_t, S, C, C, B * Hq, row, ms));
    ATTN_CK(copy_rows(snd + qc, C, 0, dk_p, S, C, C, B * Hkv, row, ms));
    ATTN_CK(copy_rows(snd + qc + kc, C, 0, dv_p, S, C, C, B * Hkv, row, ms));
    ATTN_NK(f->group_start(), "ncclGroupStart");
    ATTN_NK(f->send(snd, qc + 2 * kc, u8, m, comm->comm, ms), "ncclSend");
    ATTN_NK(f->recv(rcv, qc + 2 * kc, u8, m, comm->comm, ms), "ncclRecv");
    ATTN_NK(f->group_end(), "ncclGroupEnd");
    ATTN_CK(copy_rows(p->dq, S, C, rcv, C, 0, C, B * Hq, row, ms));
    ATTN_CK(copy_rows(p->dk, S, C, rcv + qc, C, 0, C, B * Hkv, row, ms));
    ATTN_CK(copy_rows(p->dv, S, C, rcv + qc + kc, C, 0, C, B * Hkv, row, ms));
  }
  ATTN_CK(cudaEventRecord(ev_back, ms));
  ATTN_CK(cudaStreamWaitEvent(cs, ev_back, 0));
  (void)frow;
#undef ATTN_CK
#undef ATTN_NK
  return ATTN_OK;
}
