/*
 * attnb200 — C ABI of the B200 (sm_100a) attention hot path.
 *
 * Plain C: device pointers, element strides, sizes, and CUDA streams passed
 * as `void*` (a `cudaStream_t`).  Every entry point returns an attn_status_t
 * (0 = success) and never allocates device memory: work buffers come from
 * the caller through `workspace`, sized by the matching *_workspace_size().
 * Tensors use the reference's (batch, heads, seq, head_dim) layout with a
 * unit stride on head_dim; the other strides are free but must be multiples
 * of 16 bytes for the tensor-core paths.
 *
 * Reference interfaces replaced (attnax, paths inside the project):
 *   attn_fwd            flash_attention / pallas_flash_attention /
 *                       memory_efficient_attention / standard_attention
 *                       (attnax/kernels/attention.py:17-283,
 *                        attnax/kernels/pallas.py:27-244), forward
 *   attn_bwd            JAX autodiff of the same functions (the reference
 *                       has no hand-written backward; pallas.py:45-47)
 *   attn_paged_decode   paged_attention (attnax/kernels/paged.py:17-84) over
 *                       PagedKVCache block tables (attnax/paged_cache.py:12-48)
 *   attn_paged_gather   gather_kv (attnax/paged_cache.py:201-231)
 *   attn_paged_append   append_kv (attnax/paged_cache.py:144-198)
 *   attn_lse_merge      the per-step softmax merge of ring_attention
 *                       (attnax/kernels/attention.py:662-671); the K/V
 *                       rotation (:673-674) is NCCL send/recv on the caller's
 *                       process group
 *   attn_rope           apply_rope with cos/sin gathered by position ids
 *                       (attnax/embeddings.py:126-184), the rotation
 *                       MultiHeadAttention applies to Q and K before attention
 *                       (attnax/attention.py:340-381)
 */
#ifndef ATTNB200_H_
#define ATTNB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  ATTN_OK = 0,
  ATTN_ERR_INVALID = 1,      /* bad shape, stride, alignment or pointer */
  ATTN_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement */
  ATTN_ERR_CUDA = 3,         /* a CUDA runtime call failed */
  ATTN_ERR_NCCL = 4,         /* an NCCL call failed or the communicator broke */
  ATTN_ERR_WORKSPACE = 5,    /* workspace missing or too small */
  ATTN_ERR_TIMEOUT = 6       /* a bounded device wait gave up (see attn_device_status) */
} attn_status_t;

typedef enum { ATTN_F32 = 0, ATTN_BF16 = 1, ATTN_F16 = 2 } attn_dtype_t;

/*
 * Flattened score modification: the built-in ScoreMods of
 * attnax/kernels/score_mods.py composed left to right
 * (attnax/kernels/_api.py:166-196) plus the boolean `mask=` argument.
 * Selections AND together; additive terms sum.  An entry is kept iff
 *   band_lo <= q - kv <= band_hi                        (has_band)
 *   and (kv < prefix_len[b] or kv <= q)                 (prefix_len)
 *   and doc_q[b, q] == doc_kv[b, kv]                    (doc_q, doc_kv)
 *   and bool_mask[b, h, q, kv] != 0                     (bool_mask)
 * where q, kv are global positions (row + q_offset, col + kv_offset).
 * A dropped entry gets the score finfo(float32).min, as in the reference.
 * Kept scores are  s = scale * q.k - alibi_slopes[h] * |q - kv| + bias[...].
 */
typedef struct {
  int32_t has_band;
  int64_t band_lo, band_hi;
  const int32_t* prefix_len;     /* [batch] or NULL */
  const int32_t* doc_q;          /* [batch, *] ids indexed by global q, or NULL */
  const int32_t* doc_kv;         /* [batch, *] ids indexed by global kv */
  int64_t doc_q_bstride, doc_kv_bstride;
  const float* alibi_slopes;     /* [num_heads_q] or NULL */
  const void* bias;              /* broadcastable (b, h, q, kv) or NULL */
  attn_dtype_t bias_dtype;
  int64_t bias_strides[4];       /* element strides, 0 where broadcast */
  const uint8_t* bool_mask;      /* broadcastable (b, h, q, kv) or NULL */
  int64_t mask_strides[4];
  int64_t q_offset, kv_offset;   /* global position of local row/col 0 */
} attn_mask_t;

typedef struct {
  attn_dtype_t dtype;            /* of q, k, v, out */
  int32_t batch, num_heads_q, num_heads_kv, seq_q, seq_kv, head_dim;
  const void* q; const void* k; const void* v; void* out;
  int64_t q_strides[3], k_strides[3], v_strides[3], o_strides[3]; /* b, h, s */
  float* lse;                    /* [batch, heads_q, seq_q] natural log, or NULL */
  float softmax_scale;           /* rsqrt(head_dim) for the reference */
  int32_t fix_masked_rows;       /* 1: rows with no kept key average all of V */
  attn_mask_t mask;
  void* workspace; size_t workspace_bytes;
} attn_fwd_params_t;

typedef struct {
  attn_dtype_t dtype;
  int32_t batch, num_heads_q, num_heads_kv, seq_q, seq_kv, head_dim;
  const void* q; const void* k; const void* v; const void* out; const void* d_out;
  const float* lse;              /* from attn_fwd */
  void* dq; void* dk; void* dv;  /* same layout/dtype as q, k, v */
  int64_t q_strides[3], k_strides[3], v_strides[3], o_strides[3], do_strides[3];
  int64_t dq_strides[3], dk_strides[3], dv_strides[3];
  float softmax_scale;
  int32_t fix_masked_rows;       /* 1: rows with no kept key add dO/seq_kv to all of dV */
  attn_mask_t mask;
  void* workspace; size_t workspace_bytes;
} attn_bwd_params_t;

typedef struct {
  attn_dtype_t dtype;
  int32_t num_seqs, num_heads_q, num_heads_kv, head_dim, seq_q;
  int32_t num_blocks, block_size, max_blocks_per_seq;
  int32_t max_context;           /* upper bound of seq_lengths, for split planning */
  const void* q;                 /* [num_seqs, heads_q, seq_q, head_dim] contiguous */
  const void* key_pool;          /* [num_blocks, block_size, heads_kv, head_dim] */
  const void* value_pool;
  const int32_t* block_table;    /* [num_seqs, max_blocks_per_seq], -1 unused */
  const int32_t* seq_lengths;    /* [num_seqs] */
  void* out;                     /* like q */
  float softmax_scale;
  void* workspace; size_t workspace_bytes;
} attn_paged_params_t;

/* ---- flash attention ---------------------------------------------------- */
size_t attn_fwd_workspace_size(const attn_fwd_params_t* p);
int attn_fwd(const attn_fwd_params_t* p, void* stream);
size_t attn_bwd_workspace_size(const attn_bwd_params_t* p);
int attn_bwd(const attn_bwd_params_t* p, void* stream);

/* ---- paged KV cache ----------------------------------------------------- */
size_t attn_paged_decode_workspace_size(const attn_paged_params_t* p);
int attn_paged_decode(const attn_paged_params_t* p, void* stream);
/* Allocation-free paged decode.  No counterpart in the reference.  Same
 * inputs, outputs and results as attn_paged_decode, but its split partials
 * live in an 8 MiB array inside the library (one per GPU that loads it,
 * held until the process exits), so callers that cannot allocate device
 * memory can still decode: serving loops whose allocator forbids cudaMalloc
 * on the decode path (it synchronises the device), embedders running inside
 * a fixed device-memory budget, and plugin hosts that pass a kernel only its
 * inputs and outputs.  `workspace` is ignored.  The first call on each
 * device (and in each new context) looks up the array's device address
 * with cudaGetSymbolAddress, so make that first call before any stream
 * capture.  The split count shrinks to fit the array; requests whose
 * num_seqs * num_heads_q * seq_q * (head_dim + 1) floats exceed 8 MiB
 * (16256 query rows at head_dim 128) are rejected with ATTN_ERR_WORKSPACE.
 * All calls share the array: calls that overlap on the GPU (different
 * streams, no ordering between them) race and corrupt each other. */
int attn_paged_decode_static(const attn_paged_params_t* p, void* stream);
/* Contiguous copy of one sequence: keys/values [seq_len, heads_kv, head_dim]
 * from the pages block_table_row[0 .. ceil(seq_len / block_size)).  Entries
 * are read as the reference's pool[block_ids] reads them: negative entries
 * count from the end of the pool, then indices clamp into [0, num_blocks)
 * (attn_paged_physical_page).  A seq_len above max_blocks * block_size is
 * ATTN_ERR_INVALID (gather_kv cannot reshape it either). */
int attn_paged_gather(attn_dtype_t dtype, const void* key_pool, const void* value_pool,
                      int32_t num_blocks, int32_t block_size, int32_t heads_kv, int32_t head_dim,
                      const int32_t* block_table_row, int32_t max_blocks, int32_t seq_len,
                      void* keys_out, void* values_out, void* stream);
/* Writes `chunk` new tokens of one sequence at positions start.. (block
 * table already populated).  With bad_slot non-NULL (pre-set to INT32_MAX)
 * only checks: the lowest logical page that has no table column
 * (>= max_blocks) or an unallocated entry (-1) is stored there, and nothing
 * is written; append_kv raises for both before writing.  Pages at or past
 * num_blocks drop their rows, as JAX's .at[].set drops out-of-bounds
 * updates. */
int attn_paged_append(attn_dtype_t dtype, void* key_pool, void* value_pool, int32_t num_blocks,
                      int32_t block_size, int32_t heads_kv, int32_t head_dim,
                      const int32_t* block_table_row, int32_t max_blocks, int32_t start, int32_t chunk,
                      const void* keys_new, const void* values_new, int32_t* bad_slot, void* stream);
/* The pool page a block-table entry selects (host copy of the kernels' rule):
 * entry < 0 -> entry + num_blocks, then clamped into [0, num_blocks). */
int64_t attn_paged_physical_page(int32_t entry, int32_t num_blocks);

/* ---- ring attention ------------------------------------------------------ */
/* Merges one partial attention result into a running one, row by row, by
 * log-sum-exp (the per-step online-softmax update of ring_attention,
 * attnax/kernels/attention.py:662-671, done once per K/V block):
 *   m = max(lse_acc, lse_part); w_a = e^(lse_acc - m); w_p = e^(lse_part - m)
 *   o_acc = (w_a o_acc + w_p o_part) / (w_a + w_p); lse_acc = m + log(w_a + w_p)
 * Rows with lse_part = -inf (no kept key) leave the running result unchanged.
 * o_acc is float32 [rows, head_dim]; o_part has `dtype`; with `out` non-NULL
 * the merged rows are also written there in `dtype` (the final step). */
int attn_lse_merge(attn_dtype_t dtype, int64_t rows, int32_t head_dim, float* o_acc, float* lse_acc,
                   const void* o_part, const float* lse_part, void* out, void* stream);

/* ---- ring attention over NCCL (one process per GPU) ----------------------- */
/* Replaces ring_attention (attnax/kernels/attention.py:540-691) run under
 * shard_map/pmap with axis_name bound: each rank passes its contiguous
 * shard of the global sequence and gets its output shard back.  NCCL is
 * loaded at run time (libnccl.so.2).  A communicator is made once per group:
 * one rank calls attn_comm_unique_id and hands the ATTN_COMM_ID_BYTES bytes
 * to every rank (the host framework's own broadcast), then every rank calls
 * attn_comm_init with its device current. */
#define ATTN_COMM_ID_BYTES 128
typedef struct attn_comm_s* attn_comm_t;
int attn_comm_unique_id(void* id, size_t bytes);
int attn_comm_init(attn_comm_t* comm, int32_t world, int32_t rank, const void* id, size_t bytes);
int attn_comm_destroy(attn_comm_t comm);

/* The ring's launch plan for one rank (no GPU work; used by tests and
 * tools): writes up to max_launches records of 10 int64 each --
 * hop, q_slot, q_chunks, kv_slot, kv_chunks, q_start, kv_start, masked,
 * final_from, local -- and returns the number of launches (or -status).
 * Slots index the rank's ring buffer in chunks of C = seq_local / 2 rows
 * (zigzag) or seq_local rows. */
int attn_ring_plan(int32_t world, int32_t rank, int32_t seq_local, int32_t zigzag, int32_t has_band,
                   int64_t band_lo, int64_t band_hi, int32_t position_free, int64_t* launches,
                   int32_t max_launches);

typedef struct {
  attn_dtype_t dtype;            /* bf16 or f16 */
  int32_t batch, num_heads_q, num_heads_kv, seq_local, head_dim;  /* head_dim 64 or 128 */
  const void* q;                 /* [batch, heads_q, seq_local, head_dim] contiguous: this rank's shard */
  const void* k;                 /* [batch, heads_kv, seq_local, head_dim] contiguous */
  const void* v;
  void* out;                     /* like q; must not alias q, k, v */
  float* lse;                    /* [batch, heads_q, seq_local] natural log, or NULL */
  float softmax_scale;
  /* selection on global positions: keep band_lo <= q - kv <= band_hi
   * (causal_mod: 0..INT64_MAX; sliding_window_mod(W): 0..W-1; non-causal
   * window: -(W-1)..W-1); band_lo <= 0 <= band_hi is required */
  int32_t has_band;
  int64_t band_lo, band_hi;
  const float* alibi_slopes;     /* [heads_q] or NULL (alibi_mod) */
  int32_t zigzag;                /* 1: balanced chunk assignment (causal bands; even seq_local) */
  void* workspace; size_t workspace_bytes;
} attn_ring_params_t;

size_t attn_ring_fwd_workspace_size(const attn_ring_params_t* p, int32_t world);
/* Enqueues the whole ring on compute_stream (attention) and comm_stream
 * (transfers); the results are ready in stream order of compute_stream.
 * Every rank of the communicator must call it with the same shapes and band.
 * The per-hop K/V rotation runs on the copy engines: the communicator owns
 * two receive slots of 2 x K/V shard bytes and a flags page on each rank,
 * shared with the previous rank through CUDA IPC.  The first call, and any
 * later call that needs larger slots, sets them up collectively: it
 * synchronizes the device, allocates with cudaMalloc and exchanges handles
 * over NCCL, so that call must be made by all ranks and outside any stream
 * capture.  If any rank cannot map its neighbour's slots (no peer access, or
 * two ranks on one GPU), all ranks rotate with NCCL send/recv instead.  A
 * higher-priority comm_stream lets its work start while the attention
 * kernels hold every SM.  attn_comm_destroy frees the slots. */
int attn_ring_fwd(const attn_ring_params_t* p, attn_comm_t comm, void* compute_stream, void* comm_stream);

/* Gradients of attn_ring_fwd (the reference differentiates its lax.scan /
 * ppermute ring with JAX autodiff).  The K/V shards travel the ring again;
 * every kept chunk pair gives exact partial gradients from the saved global
 * LSE, dQ accumulates in place and dK/dV accumulate in fp32 buffers that
 * follow their K/V one hop behind the attention, so the last exchange
 * brings every rank its own dK/dV.  Same shapes, band and zigzag as the
 * forward call whose `out` and `lse` are passed here. */
typedef struct {
  attn_dtype_t dtype;
  int32_t batch, num_heads_q, num_heads_kv, seq_local, head_dim;
  const void* q; const void* k; const void* v;   /* this rank's shards, contiguous */
  const void* out;               /* attn_ring_fwd output shard */
  const float* lse;              /* attn_ring_fwd LSE shard [batch, heads_q, seq_local] */
  const void* d_out;             /* like out */
  void* dq; void* dk; void* dv;  /* like q, k, v */
  float softmax_scale;
  int32_t has_band;
  int64_t band_lo, band_hi;
  const float* alibi_slopes;
  int32_t zigzag;
  void* workspace; size_t workspace_bytes;
} attn_ring_bwd_params_t;

size_t attn_ring_bwd_workspace_size(const attn_ring_bwd_params_t* p, int32_t world);
int attn_ring_bwd(const attn_ring_bwd_params_t* p, attn_comm_t comm, void* compute_stream, void* comm_stream);

/* ---- rotary position embedding ------------------------------------------- */
/* Split-half RoPE on x (batch, heads, seq, head_dim), head_dim even and unit
 * stride:  out[..., i] = x1 cos - x2 sin,  out[..., i + half] = x1 sin + x2 cos
 * with x1 = x[..., i], x2 = x[..., i + half] and cos/sin the row of the
 * [table_len][head_dim/2] tables (in `dtype`, as the reference builds them)
 * at positions[b][s] (NULL: position s).  Positions wrap once when negative
 * and clamp to the table, like the reference's array indexing.  Math in fp32;
 * out may alias x. */
typedef struct {
  attn_dtype_t dtype;        /* x, out, cos, sin */
  int32_t batch, heads, seq, head_dim;
  int64_t x_strides[3];      /* elements: batch, head, seq */
  int64_t out_strides[3];
  const void* x;
  void* out;
  const void* cos;
  const void* sin;
  int32_t table_len;
  const int32_t* positions;  /* [batch][seq] or NULL */
} attn_rope_params_t;

int attn_rope(const attn_rope_params_t* p, void* stream);

/* ---- diagnostics -------------------------------------------------------- */
/* Reads and clears the device status words (0 = none).  Synchronises the
 * current device.  Codes 0x101-0x104: a bounded wait timed out (the kernel
 * unwound; results are invalid).  0x201: a paged decode met a seq_lengths
 * entry above max_context and attended only its first splits.  0x202: a
 * paged decode met a sequence longer than max_blocks_per_seq * block_size
 * and reused the row's last entry for the pages past it.  A timeout code
 * takes precedence over a notice. */
int attn_device_status(int32_t* status);
const char* attn_status_string(int status);
int attn_version(void);
/* Number of kernels this library has launched in this process. */
uint64_t attn_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* ATTNB200_H_ */
