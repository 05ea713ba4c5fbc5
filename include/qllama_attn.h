/*
 * qllama_attn.h -- C ABI of the B200 (sm_100a) attention hot path for Qllama.
 *
 * The path: RoPE on Q/K -> append into a device-resident, paged KV cache ->
 * causal scaled-dot-product attention with GQA head mapping -> softmax.V.
 * It replaces steps 3-7 of the reference's operator
 *   Attention::forward_with_cache(&self, hidden_states, start_pos, kv_cache, layer_idx)
 *   (src/transformer/layers.rs:371-459)
 * and the KvCache it drives (src/kv_cache/cache.rs:31-248).  The Q/K/V and
 * output projections stay with the caller (layers.rs:388-395, 458).
 *
 * Conventions
 *  - Every entry point returns QL_OK (0) or a QL_ERR_* status; nothing throws
 *    or aborts across this boundary.  A human-readable message for the last
 *    failure is available from ql_last_error().  Message texts follow the
 *    reference's Err(String) wording (e.g. "must continue", "exceeds cache
 *    capacity", "divisible") so callers' substring checks keep working.
 *  - Validation is transactional, as in cache.rs:80-82: every argument,
 *    shape and position is checked before any device work is queued; on a
 *    validation error nothing is written and no sequence length moves.
 *  - One context per device, used by one host thread at a time (the
 *    reference's &mut KvCache exclusivity).  Work is queued on the context's
 *    stream (or the stream passed in), so calls are asynchronous unless a
 *    host buffer is involved.
 *  - Pointers are plain device or host pointers; `mem` says which.  Shapes
 *    are row-major and contiguous.
 */
#ifndef QLLAMA_ATTN_H
#define QLLAMA_ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define QL_OK 0
#define QL_ERR_INVALID 1     /* argument / shape / position rejected (nothing written) */
#define QL_ERR_CUDA 2        /* a CUDA runtime call failed */
#define QL_ERR_OOM 3         /* device memory could not be allocated */
#define QL_ERR_NO_DEVICE 4   /* no usable CUDA device */
#define QL_ERR_UNSUPPORTED 5 /* valid request this build does not implement */
#define QL_ERR_DEVICE 6      /* a kernel reported a fault through its status word */

/* ---- element types ---- */
#define QL_F32 0
#define QL_F16 1
#define QL_BF16 2
#define QL_Q8_0 3 /* GGUF Q8_0: blocks of 32 int8 values with one f16 scale (cache only) */

/* ---- memory kinds for the buffers of one call ---- */
#define QL_MEM_DEVICE 0
#define QL_MEM_HOST 1

typedef struct ql_ctx ql_ctx;
typedef struct ql_kv ql_kv;

/* Library version string. */
const char* ql_version(void);

/* Message of the last failed call on this host thread (never NULL). */
const char* ql_last_error(void);

/* ---- context: one CUDA device, one stream, a reusable workspace ---- */
int ql_ctx_create(int device, ql_ctx** out);
int ql_ctx_destroy(ql_ctx* ctx);
/* Use `stream` (a cudaStream_t; NULL = the context's own stream) for later calls. */
int ql_ctx_set_stream(ql_ctx* ctx, void* stream);
/* Wait for all work queued by this context; returns QL_ERR_DEVICE if a
 * kernel set its status word since the last call. */
int ql_ctx_synchronize(ql_ctx* ctx);

/* ---- KV cache --------------------------------------------------------------
 * Mirrors KvCache::new(num_layers, max_seq_len, num_kv_heads, head_dim)
 * (cache.rs:47-67), extended with a sequence dimension (max_batch slots,
 * each the reference's single-sequence cache), a storage type and paging.
 * Layout per layer: pages of `page_size` positions, each page holding
 * [num_kv_heads][page_size][head_dim] elements of K (post-RoPE, cache.rs:3-6)
 * and the same of V.  Q8_0 keeps the int8 values and the f16 block scales in
 * two planes with the same page geometry.  Sequence `s` owns pages through a
 * block table shared by all layers.
 */
typedef struct {
  int32_t num_layers;
  int32_t max_seq_len;  /* positions per sequence (capacity, cache.rs:138-143) */
  int32_t num_kv_heads;
  int32_t head_dim;     /* even; the fast kernels take 64 or 128 */
  int32_t dtype;        /* QL_F32, QL_F16, QL_BF16 or QL_Q8_0 */
  int32_t page_size;    /* positions per page, a multiple of 64 (0 = 64) */
  int32_t max_batch;    /* sequence slots (0 = 1) */
  int32_t num_pages;    /* pages in the pool (0 = max_batch * ceil(max_seq_len/page_size)) */
} ql_kv_config;

int ql_kv_create(ql_ctx* ctx, const ql_kv_config* cfg, ql_kv** out);
int ql_kv_destroy(ql_kv* kv);
/* KvCache::clear (cache.rs:235-239): every layer of every sequence back to
 * length 0.  Like the reference, buffers are kept: sequences keep their pages. */
int ql_kv_clear(ql_kv* kv);
/* Clear one sequence slot and return its pages to the pool. */
int ql_kv_clear_seq(ql_kv* kv, int32_t seq);
/* Shorten sequence `seq` to `new_len` positions in every layer (each layer must
 * hold at least that many); pages are kept and later writes continue from
 * new_len.  No counterpart in the reference, whose cache only appends or
 * clears; it serves roll-back (a rejected speculative draft, a replayed step). */
int ql_kv_truncate(ql_kv* kv, int32_t seq, int64_t new_len);
/* KvCache::seq_len (cache.rs:245-247): written prefix of layer 0 of `seq`. */
int ql_kv_seq_len(const ql_kv* kv, int32_t seq, int64_t* out_len);
/* Written prefix of one layer of one sequence. */
int ql_kv_layer_len(const ql_kv* kv, int32_t layer, int32_t seq, int64_t* out_len);

/* KvCache::update (cache.rs:83-170) for sequence `seq`: k and v are
 * [n, num_kv_heads, head_dim] (K already rotated), given with their shapes so
 * that rank and shape errors are reported as the reference does.  positions
 * must continue the layer's prefix (positions[i] == current_len + i) and stay
 * below max_seq_len.  The values are converted to the cache's storage type. */
int ql_kv_update(ql_ctx* ctx, ql_kv* kv, int32_t layer, int32_t seq, const void* k,
                 const int64_t* k_dims, int32_t k_rank, const void* v, const int64_t* v_dims,
                 int32_t v_rank, int32_t in_dtype, const int32_t* positions, int64_t n_positions,
                 int32_t mem);

/* KvCache::get (cache.rs:185-229): rows for `positions` (each < current_len),
 * in request order, duplicates allowed, dequantised to f32 into
 * k_out/v_out [n, num_kv_heads, head_dim].  Synchronous when mem is HOST. */
int ql_kv_get(ql_ctx* ctx, const ql_kv* kv, int32_t layer, int32_t seq,
              const int32_t* positions, int64_t n_positions, float* k_out, float* v_out,
              int32_t mem);

/* ---- the attention operator ----------------------------------------------
 * Steps 3-7 of Attention::forward_with_cache (layers.rs:397-455) for a
 * batch of sequences, each receiving `new_len` new tokens at its own
 * start_pos:
 *   q: [batch, new_len, num_heads, head_dim]      (pre-RoPE, in_dtype)
 *   k, v: [batch, new_len, num_kv_heads, head_dim] (pre-RoPE, in_dtype)
 *   out: [batch, new_len, num_heads*head_dim]      (out_dtype), head h in
 *        columns [h*head_dim, (h+1)*head_dim) (layers.rs:447-455)
 * RoPE is the adjacent-pair rotation with angles (start_pos+i)*theta^(-2p/hd)
 * in f64 (src/tensor/ops.rs:168-220).  Query head h reads KV head
 * h / (num_heads/num_kv_heads) (layers.rs:436).  Scores are scaled by
 * 1/sqrt(head_dim) and masked causally with offset start_pos (layers.rs:509-531).
 * start_pos[b] must equal the current length of (layer_idx, seq_ids[b]), as
 * KvCache::update demands ("must continue", cache.rs:132-137).
 */
typedef struct {
  int32_t layer_idx;
  int32_t batch;             /* sequences in this call (>= 1) */
  int32_t new_len;           /* new tokens per sequence (>= 0; 0 is a no-op) */
  const int32_t* seq_ids;    /* host array [batch]: cache slot of each sequence */
  const int64_t* start_pos;  /* host array [batch] */
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float rope_theta;
  int32_t in_dtype;          /* QL_F32, QL_F16 or QL_BF16 */
  int32_t out_dtype;         /* QL_F32, QL_F16 or QL_BF16 */
  int32_t mem;               /* QL_MEM_DEVICE or QL_MEM_HOST for q, k, v and out */
  const void* q;
  const void* k;
  const void* v;
  void* out;
} ql_attn_args;

int ql_attn_forward(ql_ctx* ctx, ql_kv* kv, const ql_attn_args* args);

/* ---- single-token decode that allocates nothing ----------------------------
 * No counterpart in the reference; an addition for callers that must not
 * allocate device memory while they serve, such as a host runtime that hands
 * the GPU's memory to its own allocator at start-up, or a serving loop that
 * promises no cudaMalloc/cudaFree between warm-up and shutdown.
 *
 * It decodes one token per sequence like ql_attn_forward (RoPE, fused append,
 * causal GQA attention), but keeps its scratch (split partials and merge
 * counters) in one static device array of QL_NOALLOC_SCRATCH_BYTES that every
 * GPU loading the library holds until the process exits.  It calls no
 * cudaMalloc, cudaFree or allocating library routine.  The cache itself is
 * allocated earlier, by ql_kv_create.
 *
 * Limits (rejected with QL_ERR_INVALID or QL_ERR_UNSUPPORTED and a message):
 * new_len must be 1; q/k/v/out must be device memory (QL_MEM_DEVICE); the
 * cache must be f16 or bf16 with head_dim 64 or 128, or Q8_0 with head_dim
 * 128, with at most 8 query heads per KV head; batch*num_kv_heads must not
 * exceed QL_NOALLOC_MAX_PAIRS.  When the partials would not fit the array,
 * fewer KV splits are used.  RoPE angles are evaluated on the device in f64,
 * so results can differ from ql_attn_forward in the last bits.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Every call shares the array and each call clears its counters, so calls
 * that overlap on the GPU (other streams or contexts on the same device)
 * race and corrupt each other's results: serialise them.
 */
#define QL_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
#define QL_NOALLOC_MAX_PAIRS 16384
int ql_attn_decode_noalloc(ql_ctx* ctx, ql_kv* kv, const ql_attn_args* args);

/* ---- head-sharded layers across GPUs ---------------------------------------
 * No counterpart in the reference, a single-process CPU program.  A layer's
 * KV heads are split evenly over `nranks` GPUs, one process per GPU: rank r
 * owns KV heads [r*Hkv/n, (r+1)*Hkv/n) with their query heads, keeps its own
 * ql_kv for them and receives only their Q/K/V.  ql_attn_forward_sharded
 * computes the rank's heads and all-gathers the outputs, so every rank ends
 * with the whole [batch, new_len, Hq*head_dim] in the layout of
 * layers.rs:447-455 (rank r's heads in columns [r*Hq/n*hd, (r+1)*Hq/n*hd)).
 *
 * Exchange (QL_COMM_P2P): a single-token decode on the split-KV kernel stores
 * each output row straight into every rank's output buffer over NVLink, from
 * the attention kernel itself; the buffers are mapped between the processes
 * with CUDA IPC when the communicator is created, and completion is signalled
 * with flags whose waits are bounded.  Other calls compute locally, then a
 * copy kernel pushes the rows the same way.  QL_COMM_NCCL selects the library
 * baseline instead (ncclAllGather, then a rank-major to head-major permute).
 * NCCL (libnccl.so.2) is loaded at ql_comm_create; nothing else needs it.
 *
 * Collective semantics: every rank makes the same sequence of sharded calls
 * on the same shapes.  The ranks must issue each call within 5 seconds of one
 * another; a rank that does not shows up as QL_ERR_DEVICE ("another GPU")
 * at the next ql_ctx_synchronize.  q, k, v and out are device buffers.
 */
#define QL_COMM_ID_BYTES 128
typedef struct {
  char bytes[QL_COMM_ID_BYTES];
} ql_comm_id;
typedef struct ql_comm ql_comm;
#define QL_COMM_P2P 0
#define QL_COMM_NCCL 1
#define QL_COMM_MAX_RANKS 8

/* Made on one rank and handed to the others out of band (e.g. a broadcast). */
int ql_comm_unique_id(ql_comm_id* out);
/* Collective over the nranks processes; max_out_bytes bounds the whole output
 * of one sharded call (batch*new_len*Hq*head_dim*element size). */
int ql_comm_create(ql_ctx* ctx, int nranks, int rank, const ql_comm_id* id,
                   uint64_t max_out_bytes, int mode, ql_comm** out);
/* Collective; every rank's calls must have finished (ql_ctx_synchronize). */
int ql_comm_destroy(ql_comm* comm);
/* This rank's symmetric output buffer.  Passing it as args->out of a sharded
 * call skips the final device-to-device copy. */
int ql_comm_buffer(ql_comm* comm, void** out, uint64_t* bytes);
/* args: num_heads / num_kv_heads are this rank's counts, q/k/v this rank's
 * heads; out holds batch*new_len rows of num_heads*nranks*head_dim. */
int ql_attn_forward_sharded(ql_ctx* ctx, ql_kv* kv, ql_comm* comm, const ql_attn_args* args);

#ifdef __cplusplus
}
#endif
#endif
