// ql_kernels.cuh -- launch interfaces of the attention kernels (host + device).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ql {

// Sequences one launch can carry in its parameter block.
constexpr int kMaxBatch = 256;
// Positions per KV tile of the split-KV kernels; pages hold a multiple of it.
constexpr int kTile = 64;

// GPUs that can share one head-sharded call.
constexpr int kMaxRanks = 8;
// Largest thread-block cluster of the decode kernel's split merge (its
// gather area holds this many CTAs); above 8 the launch needs the
// non-portable cluster size.
#ifndef QL_MAX_CLUSTER
#define QL_MAX_CLUSTER 16
#endif
constexpr int kMaxClusterCtas = QL_MAX_CLUSTER;
static_assert(kMaxClusterCtas >= 2 && kMaxClusterCtas <= 16, "cluster size");

// Head-sharded output exchange over NVLink peer memory (no collective
// library on this path).  Rank r computes query heads [head_base,
// head_base + hq) of hq_total and stores them straight into every rank's
// symmetric output [rows][hq_total][hd].  Each rank's flag block holds, per
// source rank s, entered[s] (flags[.][s]: s passed its stream dependencies
// for this call and may be written to) and done[s] (flags[.][kMaxRanks + s]:
// every store of s into this rank has been made visible).  Flags are call
// numbers that only grow: a launch's number is *epoch + 1, read once its
// stream dependencies are met, and its last CTA stores it back, so a
// captured CUDA graph replays correctly.
struct PeerOut {
  int32_t nranks;    // 0: unsharded, the output goes to the call's own buffer
  int32_t rank;
  int32_t hq_total;  // query heads of the whole layer (output row width / hd)
  int32_t head_base; // first global query head of this rank
  int32_t total_ctas;  // CTAs of the launch; the last to arrive signals done
  int32_t* arrivals;   // this rank's CTA arrival counter, zero between calls
  uint32_t* epoch;     // this rank's count of sharded calls (device)
  void* out[kMaxRanks];       // every rank's output region
  uint32_t* flags[kMaxRanks]; // every rank's flag block
};

// Per-call sequence table, passed by value in the kernel parameters.
struct SeqTable {
  int32_t seq[kMaxBatch];    // cache slot
  int32_t start[kMaxBatch];  // position of the first new token
};

// Geometry and storage of one layer of the paged KV cache.
struct CacheView {
  void* k;               // K values: [pages][hkv][page][hd] (int8 for Q8_0)
  void* v;               // V values, same geometry
  uint16_t* k_scale;     // Q8_0 only: [pages][hkv][page][hd/32] f16 bits
  uint16_t* v_scale;
  const int32_t* block_table;  // [max_batch][pages_per_seq]
  int32_t pages_per_seq;
  int32_t num_pages;
  int32_t page;          // positions per page
  int32_t hkv;
  int32_t hd;
  int32_t dtype;         // kF32 / kF16 / kBF16 / kQ8_0
};

// Appends new K (rotated unless rope == nullptr) and V rows into the cache.
struct AppendArgs {
  const void* k;
  const void* v;
  int32_t in_dtype;
  int32_t batch;
  int32_t new_len;
  const double2* rope;  // [max_seq][hd/2] (cos, sin) or nullptr
  CacheView cache;
  uint32_t* status;
  SeqTable seqs;
};

// Attention of `new_len` query tokens per sequence over the cached prefix.
struct AttnArgs {
  const void* q;  // [batch, new_len, hq, hd] pre-RoPE
  const void* k;  // new K/V, used when fuse_append (new_len == 1)
  const void* v;
  int32_t in_dtype;
  void* out;  // [batch, new_len, hq*hd]
  int32_t out_dtype;
  const double2* rope;
  int32_t rope_stride;  // table entries per position: head_dim/2, or 0 (one identity row
                        // for queries that arrive rotated)
  float rope_theta;  // used instead of `rope` by the device-RoPE variant
  CacheView cache;
  int32_t hq;
  int32_t group;  // hq / hkv
  int32_t batch;
  int32_t new_len;
  float scale;       // 1/sqrt(hd), computed as the reference does
  int32_t fuse_append;
  int32_t tiles_per_split;
  int32_t max_splits;
  float* part_o;     // [jobs][hkv][max_splits][8][hd]
  float* part_ml;    // [jobs][hkv][max_splits][8][2]
  int32_t* counters; // [jobs][hkv], zero between launches
  float* scratch;    // generic kernel: scores / probabilities
  double* scratch_d; // generic kernel: f64 contributions
  int32_t max_len;   // generic kernel: scratch row length
  int32_t out_vec;   // `out` (and every peer output) is 16-byte aligned
  int32_t wide;      // split-KV kernel: the variant whose consumer groups share a split
  int32_t cluster;   // split-KV kernel: CTAs per cluster along the splits (0/1: none)
  PeerOut peer;      // split-KV kernel: head-sharded output exchange
  uint32_t* status;
  SeqTable seqs;
};

// Multi-token causal attention on the tcgen05 tensor cores (f16 or bf16 cache, hd 64 or 128).
struct PrefillArgs {
  const void* q;       // [batch, new_len, hq, hd] pre-RoPE
  int32_t in_dtype;
  __half* q_rot;       // scratch [batch][hq][q_rows][hd] f16, rotated q divided by q_scale
  float* q_scale;      // scratch [batch][hq][q_rows]: 2^e per row, 1 unless |q| >= 2^15
  int32_t q_rows;      // new_len rounded up to the 128-row tile
  void* out;           // [batch, new_len, hq*hd]
  int32_t out_dtype;
  const double2* rope;
  int32_t rope_stride;  // as in AttnArgs
  CacheView cache;
  int32_t hq;
  int32_t group;
  int32_t batch;
  int32_t new_len;
  float scale;
  int32_t num_sms;     // SMs of the device (chooses one or two heads per CTA)
  uint32_t* status;
  SeqTable seqs;
  // bf16 caches: the keys the call sees, copied as f16 operands by a
  // conversion pass into a dense scratch [batch][hkv][kv_rows][hd] (K, and V
  // alike), each 128-key tile divided by 2^tile_exp; the attention kernel's
  // tensor maps cover these copies.  tile_exp: [K, V][batch][hkv][kv_rows/128].
  __half* k_copy;
  __half* v_copy;
  int8_t* tile_exp;
  int32_t kv_rows;     // keys per (sequence, KV head) in the copies, a multiple of 128
};

struct GatherArgs {
  const int32_t* positions;  // device [n]
  int32_t n;
  int32_t seq;
  float* k_out;
  float* v_out;
  CacheView cache;
};

// Block-table entries a call changed, carried in a kernel's parameter block
// (copied at launch, so the host may reuse its arrays at once and nothing
// waits for the copy).  table[idx[i]] = val[i].
constexpr int kTablePatchMax = 1024;
struct TablePatch {
  int32_t* table;
  int32_t n;
  int32_t idx[kTablePatchMax];
  int32_t val[kTablePatchMax];
};

// Dynamic shared memory the split-KV kernel needs for a configuration.
size_t splitkv_smem_bytes(int hd, int dtype);
// Whether the split-KV tensor-core kernel handles this configuration.
bool splitkv_supported(int hd, int dtype, int group, int page);
// Resident CTAs per SM of the split-KV kernel for a configuration on the
// current device (0 if the query failed); configures the kernel as well.
int splitkv_ctas_per_sm(int hd, int dtype, bool device_rope);
// Consumer groups of the split-KV kernel's wide variant (one CTA per SM, the
// groups take alternate tiles of a split), 0 when the configuration has none.
int splitkv_wide_groups(int hd, int dtype);

cudaError_t launch_append(const AppendArgs& a, cudaStream_t s);
// pdl: launch with programmatic dependent launch (the kernel's set-up and its
// block-table reads overlap the previous kernel).  Pass false when the
// previous launch in the stream patched the block table.
cudaError_t launch_splitkv(const AttnArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap,
                           int grid_jobs, cudaStream_t s, bool pdl = true);
// Same kernel, with the RoPE angles computed on the device (f64 pow/sincos)
// instead of read from the host-built table; needs fuse_append and new_len 1.
cudaError_t launch_splitkv_device_rope(const AttnArgs& a, const CUtensorMap* kmap,
                                       const CUtensorMap* vmap, int jobs, cudaStream_t s);
cudaError_t launch_generic(const AttnArgs& a, cudaStream_t s);
// Head-sharded calls that are not fused single-token decodes: copies this
// rank's compact output rows [rows][row_bytes] into every rank's symmetric
// output at byte offset (row * hq_total + head_base) * hd * elem, with the
// entered/done protocol of PeerOut.  row_bytes must be a multiple of 4.
cudaError_t launch_peer_push(const void* src, int64_t rows, int row_bytes, int head_bytes,
                             PeerOut po, int num_sms, uint32_t* status, cudaStream_t s);
// All-gather baseline: rank-major [nranks][rows][row_bytes] -> head-major
// [rows][nranks * row_bytes].
cudaError_t launch_rank_to_head_major(const void* src, void* dst, int nranks, int64_t rows,
                                      int row_bytes, cudaStream_t s);
cudaError_t launch_gather(const GatherArgs& a, cudaStream_t s);
// Writes the entries of `p` into the device block table, in stream order, as
// an ordinary launch: a kernel queued after it sees the entries once its
// stream dependency is met.  A split-KV launch that follows must not use
// programmatic dependent launch, because that kernel reads the table before
// its grid dependency wait.
cudaError_t launch_table_patch(const TablePatch& p, cudaStream_t s);

// tcgen05 prefill: when it applies, rows of the rotated-q scratch it needs,
// and the launch: one prologue kernel (q rotated into the scratch, new K/V
// rotated and appended into the cache as `ap` describes), then the attention
// kernel.
bool prefill_tc_supported(int hd, int dtype, int new_len);
size_t prefill_q_rows(int new_len);
cudaError_t launch_prefill_tc(const PrefillArgs& a, const AppendArgs& ap, const CUtensorMap* qmap,
                              const CUtensorMap* kmap, const CUtensorMap* vmap, cudaStream_t s);


}  // namespace ql
