// ql_api.cu -- the C ABI (include/qllama_attn.h): contexts, the paged KV cache,
// transactional validation and kernel dispatch.
//
// Validation mirrors the reference before any device work is queued:
//   Attention::new head checks          src/transformer/layers.rs:254-275
//   rope parameter checks               src/tensor/ops.rs:170-188
//   i32 position conversion             src/transformer/layers.rs:403-422
//   KvCache::update / get checks        src/kv_cache/cache.rs:90-144, 186-208
// and uses the same message wording, so substring checks written against the
// reference ("must continue", "exceeds cache capacity", "divisible", ...)
// hold here too.  Sequence lengths advance only after the work is queued.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <atomic>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/qllama_attn.h"
#include "ql_device.cuh"
#include "ql_internal.h"
#include "ql_kernels.cuh"

namespace {

thread_local std::string g_error = "";

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? QL_ERR_OOM : QL_ERR_CUDA, "%s: %s", what,
              cudaGetErrorString(e));
}

#define QL_CUDA(call, what)                 \
  do {                                      \
    cudaError_t e_ = (call);                \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

size_t elem_bytes(int dt) { return dt == QL_F32 ? 4 : (dt == QL_Q8_0 ? 1 : 2); }

bool valid_io_dtype(int dt) { return dt == QL_F32 || dt == QL_F16 || dt == QL_BF16; }

std::string dims_str(const int64_t* d, int rank) {
  std::string s = "[";
  for (int i = 0; i < rank; ++i) {
    if (i) s += ", ";
    s += std::to_string(static_cast<long long>(d[i]));
  }
  return s + "]";
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

// --------------------------------------------------------------- context --
// struct ql_ctx is defined in ql_internal.h (the model host uses it too).
int ql_fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

struct ql_kv {
  ql_ctx* ctx = nullptr;
  ql_kv_config cfg{};
  int pages_per_seq = 0;
  std::vector<void*> k, v;             // per layer
  std::vector<uint16_t*> ks, vs;       // per layer, Q8_0 scales
  std::vector<CUtensorMap> kmap, vmap;  // per layer, split-KV kernel descriptors
  bool have_maps = false;
  int32_t* d_table = nullptr;          // [max_batch][pages_per_seq]
  std::vector<int32_t> table;          // host mirror
  std::vector<int32_t> seq_pages;      // pages owned per sequence
  std::vector<int32_t> free_pages;     // stack of free page ids
  std::vector<int64_t> len;            // [layer][seq] written prefix
  double2* d_rope = nullptr;           // [max_seq_len][head_dim/2] (cos, sin)
  double2* d_rope_id = nullptr;        // [head_dim/2] (1, 0): queries that arrive rotated
  float rope_theta = 0.f;
  // Duplicate-sequence check of a call without per-call allocation: slot s
  // was named by the current call when seen_mark[s] == seen_epoch.
  std::vector<uint32_t> seen_mark;
  uint32_t seen_epoch = 0;
  // Block-table entries handed out by the current call (index into `table`):
  // the roll-back log on pool exhaustion and the list the table patch kernel
  // uploads.  Reserved to the table's size at creation, so a call never
  // grows it.
  std::vector<int32_t> patch_idx;
};

namespace {

int ensure_ws(ql_ctx* c, size_t bytes) {
  if (bytes <= c->ws_bytes) return QL_OK;
  QL_CUDA(cudaStreamSynchronize(c->stream), "synchronize before growing workspace");
  if (c->ws) cudaFree(c->ws);
  c->ws = nullptr;
  c->ws_bytes = 0;
  size_t want = bytes + bytes / 4 + (1 << 20);
  QL_CUDA(cudaMalloc(&c->ws, want), "allocate workspace");
  c->ws_bytes = want;
  return QL_OK;
}

int ensure_counters(ql_ctx* c, size_t n) {
  if (n <= c->counters_n) return QL_OK;
  QL_CUDA(cudaStreamSynchronize(c->stream), "synchronize before growing counters");
  if (c->counters) cudaFree(c->counters);
  c->counters = nullptr;
  c->counters_n = 0;
  size_t want = n + n / 2 + 1024;
  QL_CUDA(cudaMalloc(&c->counters, want * sizeof(int32_t)), "allocate counters");
  QL_CUDA(cudaMemsetAsync(c->counters, 0, want * sizeof(int32_t), c->stream), "zero counters");
  c->counters_n = want;
  return QL_OK;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

ql::CacheView view_of(const ql_kv* kv, int layer) {
  ql::CacheView c;
  c.k = kv->k[layer];
  c.v = kv->v[layer];
  c.k_scale = kv->cfg.dtype == QL_Q8_0 ? kv->ks[layer] : nullptr;
  c.v_scale = kv->cfg.dtype == QL_Q8_0 ? kv->vs[layer] : nullptr;
  c.block_table = kv->d_table;
  c.pages_per_seq = kv->pages_per_seq;
  c.num_pages = kv->cfg.num_pages;
  c.page = kv->cfg.page_size;
  c.hkv = kv->cfg.num_kv_heads;
  c.hd = kv->cfg.head_dim;
  c.dtype = kv->cfg.dtype;
  return c;
}

int encode_map(CUtensorMap* m, void* base, int dtype, int hd, uint64_t rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(QL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const bool q8 = dtype == QL_Q8_0;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(hd), rows};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(hd) * (q8 ? 1 : 2)};
  cuuint32_t box[2] = {q8 ? 128u : 64u, static_cast<cuuint32_t>(ql::kTile)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, q8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base,
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QL_OK;
}

// Tensor map over the rotated-q scratch [rows][hd] f16, boxes of 64 columns x
// 128 rows with the 128-byte swizzle the tcgen05 descriptors expect.
int encode_q_map(CUtensorMap* m, void* base, int hd, uint64_t rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(QL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(hd), rows};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(hd) * 2};
  cuuint32_t box[2] = {64u, 128u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QL_OK;
}

// Builds (once per theta) the f64 (cos, sin) table of every position with the
// reference formula: freq_i = theta^(-2i/hd) via pow, angle = pos * freq_i
// (src/tensor/ops.rs:193-207), evaluated by the host libm as the reference does.
int ensure_rope(ql_kv* kv, float theta) {
  if (kv->d_rope && kv->rope_theta == theta) return QL_OK;
  const int hd = kv->cfg.head_dim, pairs = hd / 2, n = kv->cfg.max_seq_len;
  std::vector<double> freq(pairs);
  for (int p = 0; p < pairs; ++p)
    freq[p] = std::pow(static_cast<double>(theta), -2.0 * static_cast<double>(p) / hd);
  std::vector<double2> tab(static_cast<size_t>(n) * pairs);
  for (int pos = 0; pos < n; ++pos)
    for (int p = 0; p < pairs; ++p) {
      const double ang = static_cast<double>(pos) * freq[p];
      tab[static_cast<size_t>(pos) * pairs + p] = make_double2(std::cos(ang), std::sin(ang));
    }
  if (!kv->d_rope) {
    QL_CUDA(cudaMalloc(&kv->d_rope, std::max<size_t>(1, tab.size()) * sizeof(double2)),
            "allocate rope table");
    // the identity rotation (cos 1, sin 0 leaves a pair exactly as it is)
    std::vector<double2> id(std::max(1, pairs), make_double2(1.0, 0.0));
    QL_CUDA(cudaMalloc(&kv->d_rope_id, id.size() * sizeof(double2)), "allocate rope table");
    QL_CUDA(cudaMemcpyAsync(kv->d_rope_id, id.data(), id.size() * sizeof(double2),
                            cudaMemcpyHostToDevice, kv->ctx->stream),
            "upload the identity rotation");
    QL_CUDA(cudaStreamSynchronize(kv->ctx->stream), "wait for the identity rotation");
  }
  // On the context's stream (the kernels that read the table run there), and
  // waited for before the host vector goes away.
  QL_CUDA(cudaMemcpyAsync(kv->d_rope, tab.data(), tab.size() * sizeof(double2),
                          cudaMemcpyHostToDevice, kv->ctx->stream),
          "upload rope table");
  QL_CUDA(cudaStreamSynchronize(kv->ctx->stream), "wait for the rope table upload");
  kv->rope_theta = theta;
  return QL_OK;
}

// Queues the upload of the block-table entries listed in idx[0..n) (their
// values taken from the host mirror) as table patch launches on the
// context's stream: stream-ordered, with no host synchronisation.
int upload_table_entries(ql_kv* kv, const int32_t* idx, size_t n) {
  ql::TablePatch p;
  p.table = kv->d_table;
  for (size_t i0 = 0; i0 < n; i0 += ql::kTablePatchMax) {
    const size_t m = std::min<size_t>(ql::kTablePatchMax, n - i0);
    p.n = static_cast<int32_t>(m);
    for (size_t i = 0; i < m; ++i) {
      p.idx[i] = idx[i0 + i];
      p.val[i] = kv->table[static_cast<size_t>(idx[i0 + i])];
    }
    QL_CUDA(ql::launch_table_patch(p, kv->ctx->stream), "launch block-table patch");
  }
  return QL_OK;
}

// Gives every listed sequence the pages its new length needs; rolls back on
// exhaustion so that the call stays transactional.  New entries reach the
// device through a table patch launch queued on the context's stream (no
// host synchronisation, no per-call allocation); *patched tells the caller
// that a split-KV launch following it must not use programmatic dependent
// launch (that kernel reads the table before its grid dependency wait).
int reserve_pages(ql_kv* kv, const int32_t* seqs, const int64_t* ends, int count, bool* patched) {
  const int P = kv->cfg.page_size, pps = kv->pages_per_seq;
  *patched = false;
  kv->patch_idx.clear();  // capacity reserved at creation: no allocation
  for (int i = 0; i < count; ++i) {
    const int s = seqs[i];
    const int need = static_cast<int>((ends[i] + P - 1) / P);
    while (kv->seq_pages[s] < need) {
      if (kv->free_pages.empty()) {
        for (auto it = kv->patch_idx.rbegin(); it != kv->patch_idx.rend(); ++it) {
          kv->free_pages.push_back(kv->table[static_cast<size_t>(*it)]);
          kv->table[static_cast<size_t>(*it)] = -1;
          kv->seq_pages[*it / pps]--;
        }
        kv->patch_idx.clear();
        return fail(QL_ERR_OOM, "KV page pool exhausted (%d pages of %d positions)",
                    kv->cfg.num_pages, P);
      }
      const int page = kv->free_pages.back();
      kv->free_pages.pop_back();
      const int32_t idx = s * pps + kv->seq_pages[s];
      kv->table[static_cast<size_t>(idx)] = page;
      kv->patch_idx.push_back(idx);
      kv->seq_pages[s]++;
    }
  }
  if (!kv->patch_idx.empty()) {
    const int r = upload_table_entries(kv, kv->patch_idx.data(), kv->patch_idx.size());
    if (r != QL_OK) return r;
    *patched = true;
  }
  return QL_OK;
}

// A fresh mark for the duplicate check of one call (the marks are cleared
// when the counter wraps).
uint32_t next_seen_epoch(ql_kv* kv) {
  if (++kv->seen_epoch == 0) {
    std::fill(kv->seen_mark.begin(), kv->seen_mark.end(), 0u);
    kv->seen_epoch = 1;
  }
  return kv->seen_epoch;
}

int64_t& len_at(ql_kv* kv, int layer, int seq) {
  return kv->len[static_cast<size_t>(layer) * kv->cfg.max_batch + seq];
}

}  // namespace

int ql_ctx_workspace(ql_ctx* c, size_t bytes, void** out) {
  const int r = ensure_ws(c, bytes);
  if (r != QL_OK) return r;
  *out = c->ws;
  return QL_OK;
}

int ql_check_status(ql_ctx* c) {
  uint32_t st = 0;
  QL_CUDA(cudaMemcpy(&st, c->status, sizeof st, cudaMemcpyDeviceToHost), "read status word");
  if (st) {
    cudaMemsetAsync(c->status, 0, sizeof(uint32_t), c->stream);
    return fail(QL_ERR_DEVICE, "a kernel reported status 0x%x (%s)", st,
                (st & ql::kStatusPeerTimeout)   ? "another GPU of a head-sharded call did not "
                                                  "signal within the wait limit"
                : (st & ql::kStatusWaitTimeout) ? "a pipeline wait timed out"
                : (st & ql::kStatusBadLogits)   ? "the sampler met a non-finite logit"
                : (st & ql::kStatusBadToken)    ? "a token id was outside the vocabulary"
                                                : "a block-table entry was out of range");
  }
  return QL_OK;
}

namespace {

// Split plan of the split-KV decode kernel: the 64-position tiles each CTA
// streams, and the most splits any (token, KV head) job is cut into.
struct SplitPlan {
  int tps;
  int splits;
};

// tiles[b]: the most tiles a token of batch row b sees; per_row: the (token,
// KV head) jobs of each row; slots: CTAs the whole GPU holds at once.
// 1. While the jobs alone do not fill the slots twice, the KV length is split
//    so that they do, keeping at least kMinSplitTiles tiles per split and at
//    most kMaxSplits splits; then the splits are evened out.  A CTA's fixed
//    work (q rotation, pipeline fill, its merge share) is worth about as much
//    as a dozen tiles, so short splits cost more than the wave they fill:
//    with 16 instead of 4, 32 sequences of 500 positions (head_dim 64) decode
//    in about half the time.
// 2. Equal CTAs finish together, so a last wave that leaves slots idle is time
//    lost.  While it would leave more than a tenth of them idle, up to four
//    times as many splits are tried; the first that fills 90% is kept, else
//    the fullest.
SplitPlan plan_splits(const int* tiles, int rows, long long per_row, long long slots) {
  constexpr int kMinSplitTiles = 16, kMaxSplits = 64;
  int max_tiles = 1;
  long long total = 0;
  for (int r = 0; r < rows; ++r) {
    const int t = tiles[r];
    max_tiles = std::max(max_tiles, t);
    total += t * per_row;
  }
  const long long jobs = per_row * static_cast<long long>(rows);
  slots = std::max(1LL, slots);
  int tps = max_tiles;
  if (jobs < 2 * slots) {
    tps = static_cast<int>(std::max(1LL, (total + 2 * slots - 1) / (2 * slots)));
    tps = std::max(tps, kMinSplitTiles);
    tps = std::max(tps, (max_tiles + kMaxSplits - 1) / kMaxSplits);
  }
  int splits = (max_tiles + tps - 1) / tps;
  tps = (max_tiles + splits - 1) / splits;
  auto fill = [&](int t) {
    long long ctas = 0;
    for (int r = 0; r < rows; ++r) ctas += (tiles[r] + t - 1) / t * per_row;
    const long long waves = (ctas + slots - 1) / slots;
    return static_cast<double>(ctas) / static_cast<double>(waves * slots);
  };
  SplitPlan plan{tps, splits};
  double best = fill(tps);
  for (int sp = splits + 1; best < 0.9 && sp <= std::min(kMaxSplits, 4 * splits); ++sp) {
    const int t = (max_tiles + sp - 1) / sp;
    if (t < kMinSplitTiles) break;
    if ((max_tiles + t - 1) / t != sp) continue;  // the same split as a smaller count
    const double f = fill(t);
    if (f > best) {
      best = f;
      plan = {t, sp};
    }
  }
  return plan;
}

// Tiles per split of the wide kernel: up to kWideTilesPerGroup tiles per
// consumer group (each group runs its tiles one after another, the groups in
// parallel), with at most one CTA per SM over all `pairs` (token, KV head)
// jobs; one split per job whenever that covers the sequence, so no merge
// across CTAs is needed.
#ifndef QL_WIDE_TILES_PER_GROUP
#define QL_WIDE_TILES_PER_GROUP 4
#endif
int wide_tiles_per_split(int max_tiles, int groups, long long pairs, int num_sms) {
  constexpr int kWideTilesPerGroup = QL_WIDE_TILES_PER_GROUP;
  long long splits = (max_tiles + 1LL * groups * kWideTilesPerGroup - 1) /
                     (1LL * groups * kWideTilesPerGroup);
  splits = std::min<long long>(splits, std::max<long long>(1, num_sms / std::max(1LL, pairs)));
  splits = std::max<long long>(1, std::min<long long>(splits, 64));
  return static_cast<int>((max_tiles + splits - 1) / splits);
}

}  // namespace

// ---------------------------------------------------- no-allocation decode --
// Fixed device scratch for ql_attn_decode_noalloc: the merge counters, then
// the split partials (m, l) and O.  Every GPU that loads this library holds
// it until the process exits; it starts zeroed and every call clears the
// counters again before use.  In host code `g_noalloc_scratch` is only a
// stand-in symbol: kernels get the device address from cudaGetSymbolAddress.
namespace {

constexpr size_t kNoAllocBytes = QL_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocPairs = QL_NOALLOC_MAX_PAIRS;
constexpr size_t kNoAllocCounterBytes = static_cast<size_t>(kNoAllocPairs) * sizeof(int32_t);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of the array, per device (null until looked up).  Atomic,
// because two host threads may make their first call on one device at once;
// both then store the same address.
std::atomic<char*> g_noalloc_addr[kMaxDevices] = {};

// Called with `device` current.  The lookup runs once per device.
int noalloc_scratch(int device, char** out) {
  if (device < 0 || device >= kMaxDevices)
    return fail(QL_ERR_UNSUPPORTED, "device %d is beyond the %d devices the scratch table covers",
                device, kMaxDevices);
  char* addr = g_noalloc_addr[device].load(std::memory_order_acquire);
  if (!addr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "look up the no-allocation scratch");
    addr = static_cast<char*>(p);
    g_noalloc_addr[device].store(addr, std::memory_order_release);
  }
  *out = addr;
  return QL_OK;
}

}  // namespace

extern "C" {

const char* ql_version(void) { return "qllama_b200 0.1 (sm_100a)"; }

const char* ql_last_error(void) { return g_error.c_str(); }

int ql_ctx_create(int device, ql_ctx** out) {
  if (!out) return fail(QL_ERR_INVALID, "ql_ctx_create: out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return fail(QL_ERR_NO_DEVICE, "no CUDA device is available (%s)",
                e == cudaSuccess ? "none found" : cudaGetErrorString(e));
  if (device < 0 || device >= n)
    return fail(QL_ERR_INVALID, "device %d out of range (%d devices)", device, n);
  cudaDeviceProp prop;
  QL_CUDA(cudaGetDeviceProperties(&prop, device), "query device");
  if (prop.major != 10)
    return fail(QL_ERR_UNSUPPORTED, "this build targets sm_100a (B200); device %d is sm_%d%d",
                device, prop.major, prop.minor);
  QL_CUDA(cudaSetDevice(device), "set device");
  ql_ctx* c = new ql_ctx;
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->status, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemsetAsync(c->status, 0, sizeof(uint32_t), c->own);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->own);
  if (e != cudaSuccess) {
    ql_ctx_destroy(c);
    return cuda_fail(e, "create context");
  }
  c->stream = c->own;
  *out = c;
  return QL_OK;
}

int ql_ctx_destroy(ql_ctx* c) {
  if (!c) return QL_OK;
  cudaSetDevice(c->device);
  if (c->own) cudaStreamSynchronize(c->own);
  if (c->ws) cudaFree(c->ws);
  if (c->counters) cudaFree(c->counters);
  if (c->status) cudaFree(c->status);
  if (c->own) cudaStreamDestroy(c->own);
  delete c;
  return QL_OK;
}

int ql_ctx_set_stream(ql_ctx* c, void* stream) {
  if (!c) return fail(QL_ERR_INVALID, "ql_ctx_set_stream: ctx is NULL");
  c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own;
  return QL_OK;
}

int ql_ctx_synchronize(ql_ctx* c) {
  if (!c) return fail(QL_ERR_INVALID, "ql_ctx_synchronize: ctx is NULL");
  QL_CUDA(cudaSetDevice(c->device), "set device");
  QL_CUDA(cudaStreamSynchronize(c->stream), "synchronize");
  return ql_check_status(c);
}

int ql_kv_create(ql_ctx* c, const ql_kv_config* cfg_in, ql_kv** out) {
  if (!c || !cfg_in || !out) return fail(QL_ERR_INVALID, "ql_kv_create: NULL argument");
  *out = nullptr;
  ql_kv_config cfg = *cfg_in;
  if (cfg.page_size == 0) cfg.page_size = ql::kTile;
  if (cfg.max_batch == 0) cfg.max_batch = 1;
  if (cfg.num_layers < 0 || cfg.max_seq_len < 0 || cfg.num_kv_heads <= 0 || cfg.head_dim <= 0 ||
      cfg.max_batch < 0 || cfg.num_pages < 0)
    return fail(QL_ERR_INVALID,
                "KV cache needs num_layers >= 0, max_seq_len >= 0, num_kv_heads > 0, head_dim > 0");
  if (cfg.dtype < QL_F32 || cfg.dtype > QL_Q8_0)
    return fail(QL_ERR_INVALID, "unknown KV cache dtype %d", cfg.dtype);
  if (cfg.page_size % ql::kTile != 0)
    return fail(QL_ERR_INVALID, "page_size %d must be a positive multiple of %d", cfg.page_size,
                ql::kTile);
  if (cfg.dtype == QL_Q8_0 && cfg.head_dim % 32 != 0)
    return fail(QL_ERR_INVALID, "Q8_0 storage needs head_dim divisible by 32, got %d",
                cfg.head_dim);
  QL_CUDA(cudaSetDevice(c->device), "set device");
  ql_kv* kv = new ql_kv;
  kv->ctx = c;
  kv->pages_per_seq = (cfg.max_seq_len + cfg.page_size - 1) / cfg.page_size;
  if (cfg.num_pages == 0) cfg.num_pages = cfg.max_batch * std::max(1, kv->pages_per_seq);
  kv->cfg = cfg;
  const size_t rows = static_cast<size_t>(cfg.num_pages) * cfg.num_kv_heads * cfg.page_size;
  const size_t bytes = rows * cfg.head_dim * elem_bytes(cfg.dtype);
  auto cleanup = [&](int code) {
    ql_kv_destroy(kv);
    return code;
  };
  for (int l = 0; l < cfg.num_layers; ++l) {
    void *kp = nullptr, *vp = nullptr;
    cudaError_t e = cudaMalloc(&kp, std::max<size_t>(bytes, 256));
    if (e == cudaSuccess) e = cudaMalloc(&vp, std::max<size_t>(bytes, 256));
    if (e == cudaSuccess) e = cudaMemset(kp, 0, std::max<size_t>(bytes, 256));
    if (e == cudaSuccess) e = cudaMemset(vp, 0, std::max<size_t>(bytes, 256));
    kv->k.push_back(kp);
    kv->v.push_back(vp);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "allocate KV pool"));
    if (cfg.dtype == QL_Q8_0) {
      const size_t sb = std::max<size_t>(rows * (cfg.head_dim / 32) * 2, 256);
      uint16_t *a = nullptr, *b = nullptr;
      e = cudaMalloc(&a, sb);
      if (e == cudaSuccess) e = cudaMalloc(&b, sb);
      if (e == cudaSuccess) e = cudaMemset(a, 0, sb);
      if (e == cudaSuccess) e = cudaMemset(b, 0, sb);
      kv->ks.push_back(a);
      kv->vs.push_back(b);
      if (e != cudaSuccess) return cleanup(cuda_fail(e, "allocate Q8_0 scales"));
    }
  }
  kv->table.assign(static_cast<size_t>(cfg.max_batch) * std::max(1, kv->pages_per_seq), -1);
  kv->patch_idx.reserve(kv->table.size());
  kv->seq_pages.assign(cfg.max_batch, 0);
  kv->seen_mark.assign(cfg.max_batch, 0);
  kv->free_pages.reserve(cfg.num_pages);
  for (int p = cfg.num_pages - 1; p >= 0; --p) kv->free_pages.push_back(p);
  kv->len.assign(static_cast<size_t>(std::max(1, cfg.num_layers)) * cfg.max_batch, 0);
  cudaError_t e = cudaMalloc(&kv->d_table, kv->table.size() * sizeof(int32_t));
  // Every entry -1 (all bytes 0xff).  The pool memsets above ran on the legacy
  // stream, which the context's non-blocking stream does not wait for: the
  // device synchronisation orders all of them before any later launch.
  if (e == cudaSuccess) e = cudaMemset(kv->d_table, 0xff, kv->table.size() * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cleanup(cuda_fail(e, "allocate block table"));
  if (ql::splitkv_supported(cfg.head_dim, cfg.dtype, 1, cfg.page_size) && rows > 0) {
    kv->kmap.resize(cfg.num_layers);
    kv->vmap.resize(cfg.num_layers);
    for (int l = 0; l < cfg.num_layers; ++l) {
      int r = encode_map(&kv->kmap[l], kv->k[l], cfg.dtype, cfg.head_dim, rows);
      if (r == QL_OK) r = encode_map(&kv->vmap[l], kv->v[l], cfg.dtype, cfg.head_dim, rows);
      if (r != QL_OK) return cleanup(r);
    }
    kv->have_maps = true;
  }
  *out = kv;
  return QL_OK;
}

int ql_kv_destroy(ql_kv* kv) {
  if (!kv) return QL_OK;
  cudaSetDevice(kv->ctx->device);
  cudaStreamSynchronize(kv->ctx->stream);
  for (void* p : kv->k) cudaFree(p);
  for (void* p : kv->v) cudaFree(p);
  for (void* p : kv->ks) cudaFree(p);
  for (void* p : kv->vs) cudaFree(p);
  if (kv->d_table) cudaFree(kv->d_table);
  if (kv->d_rope) cudaFree(kv->d_rope);
  if (kv->d_rope_id) cudaFree(kv->d_rope_id);
  delete kv;
  return QL_OK;
}

int ql_kv_clear(ql_kv* kv) {
  if (!kv) return fail(QL_ERR_INVALID, "ql_kv_clear: kv is NULL");
  // Lengths back to zero; buffers (and pages) stay, as in cache.rs:231-239.
  std::fill(kv->len.begin(), kv->len.end(), 0);
  return QL_OK;
}

int ql_kv_clear_seq(ql_kv* kv, int32_t seq) {
  if (!kv) return fail(QL_ERR_INVALID, "ql_kv_clear_seq: kv is NULL");
  if (seq < 0 || seq >= kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", seq,
                kv->cfg.max_batch);
  // Stale rows stay in the pages; lengths make them unreachable (cache.rs:231-234).
  for (int l = 0; l < kv->cfg.num_layers; ++l) len_at(kv, l, seq) = 0;
  const int pps = kv->pages_per_seq;
  if (kv->seq_pages[seq] > 0) {
    QL_CUDA(cudaSetDevice(kv->ctx->device), "set device");
    QL_CUDA(cudaStreamSynchronize(kv->ctx->stream), "synchronize before releasing pages");
    kv->patch_idx.clear();
    for (int i = kv->seq_pages[seq] - 1; i >= 0; --i) {
      const int32_t idx = seq * pps + i;
      kv->free_pages.push_back(kv->table[static_cast<size_t>(idx)]);
      kv->table[static_cast<size_t>(idx)] = -1;
      kv->patch_idx.push_back(idx);
    }
    kv->seq_pages[seq] = 0;
    // the device table follows the mirror (-1: the slot owns no page)
    const int r = upload_table_entries(kv, kv->patch_idx.data(), kv->patch_idx.size());
    kv->patch_idx.clear();
    if (r != QL_OK) return r;
  }
  return QL_OK;
}

int ql_kv_truncate(ql_kv* kv, int32_t seq, int64_t new_len) {
  if (!kv) return fail(QL_ERR_INVALID, "ql_kv_truncate: kv is NULL");
  if (seq < 0 || seq >= kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", seq,
                kv->cfg.max_batch);
  for (int l = 0; l < kv->cfg.num_layers; ++l)
    if (new_len < 0 || new_len > len_at(kv, l, seq))
      return fail(QL_ERR_INVALID, "cannot truncate layer %d of sequence %d to %lld positions "
                  "(it holds %lld)", l, seq, (long long)new_len, (long long)len_at(kv, l, seq));
  for (int l = 0; l < kv->cfg.num_layers; ++l) len_at(kv, l, seq) = new_len;
  return QL_OK;
}

int ql_kv_seq_len(const ql_kv* kv, int32_t seq, int64_t* out_len) {
  if (!kv || !out_len) return fail(QL_ERR_INVALID, "ql_kv_seq_len: NULL argument");
  if (seq < 0 || seq >= kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", seq,
                kv->cfg.max_batch);
  *out_len = kv->cfg.num_layers ? kv->len[seq] : 0;
  return QL_OK;
}

int ql_kv_layer_len(const ql_kv* kv, int32_t layer, int32_t seq, int64_t* out_len) {
  if (!kv || !out_len) return fail(QL_ERR_INVALID, "ql_kv_layer_len: NULL argument");
  if (layer < 0 || layer >= kv->cfg.num_layers)
    return fail(QL_ERR_INVALID, "KV cache layer index %d out of range (cache has %d layers)",
                layer, kv->cfg.num_layers);
  if (seq < 0 || seq >= kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", seq,
                kv->cfg.max_batch);
  *out_len = kv->len[static_cast<size_t>(layer) * kv->cfg.max_batch + seq];
  return QL_OK;
}

int ql_kv_update(ql_ctx* c, ql_kv* kv, int32_t layer, int32_t seq, const void* k,
                 const int64_t* k_dims, int32_t k_rank, const void* v, const int64_t* v_dims,
                 int32_t v_rank, int32_t in_dtype, const int32_t* positions, int64_t n_positions,
                 int32_t mem) {
  if (!c || !kv || (!k_dims && k_rank) || (!v_dims && v_rank))
    return fail(QL_ERR_INVALID, "ql_kv_update: NULL argument");
  const int hkv = kv->cfg.num_kv_heads, hd = kv->cfg.head_dim;
  if (layer < 0 || layer >= kv->cfg.num_layers)
    return fail(QL_ERR_INVALID, "KV cache layer index %d out of range (cache has %d layers)",
                layer, kv->cfg.num_layers);
  if (seq < 0 || seq >= kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", seq,
                kv->cfg.max_batch);
  const std::string kd = dims_str(k_dims, k_rank), vd = dims_str(v_dims, v_rank);
  if (k_rank != 3 || k_dims[1] != hkv || k_dims[2] != hd)
    return fail(QL_ERR_INVALID, "K shape %s does not match cache [_, %d, %d]", kd.c_str(), hkv,
                hd);
  bool same = v_rank == k_rank;
  for (int i = 0; same && i < k_rank; ++i) same = v_dims[i] == k_dims[i];
  if (!same) return fail(QL_ERR_INVALID, "K/V shape mismatch: K %s, V %s", kd.c_str(), vd.c_str());
  const int64_t n = k_dims[0];
  if (n_positions != n)
    return fail(QL_ERR_INVALID, "K batch is %lld token(s) but got %lld position(s)",
                (long long)n, (long long)n_positions);
  if (!valid_io_dtype(in_dtype)) return fail(QL_ERR_INVALID, "unknown input dtype %d", in_dtype);
  if (n > 0 && (!positions || !k || !v)) return fail(QL_ERR_INVALID, "ql_kv_update: NULL data");
  const int64_t cur = len_at(kv, layer, seq);
  for (int64_t i = 0; i < n; ++i) {
    const int32_t p = positions[i];
    if (p < 0) return fail(QL_ERR_INVALID, "positions[%lld] = %d is negative", (long long)i, p);
    if (p != cur + i)
      return fail(QL_ERR_INVALID,
                  "positions[%lld] = %d must continue from current_len (expected %lld); "
                  "skipping, backward, or double writes are not allowed",
                  (long long)i, p, (long long)(cur + i));
    if (p >= kv->cfg.max_seq_len)
      return fail(QL_ERR_INVALID, "positions[%lld] = %d exceeds cache capacity %d", (long long)i,
                  p, kv->cfg.max_seq_len);
  }
  if (n == 0) return QL_OK;  // empty batch: no-op (cache.rs:77-78)
  if (n > INT32_MAX / (hkv * 32)) return fail(QL_ERR_INVALID, "batch too large");
  QL_CUDA(cudaSetDevice(c->device), "set device");
  const int32_t one_seq = seq;
  const int64_t one_end = cur + n;
  bool patched = false;  // append_kernel is an ordinary launch: it sees the patch
  int r = reserve_pages(kv, &one_seq, &one_end, 1, &patched);
  if (r != QL_OK) return r;
  const size_t in_bytes = static_cast<size_t>(n) * hkv * hd * elem_bytes(in_dtype);
  const void *kd_ptr = k, *vd_ptr = v;
  if (mem == QL_MEM_HOST) {
    r = ensure_ws(c, 2 * align256(in_bytes));
    if (r != QL_OK) return r;
    char* w = static_cast<char*>(c->ws);
    QL_CUDA(cudaMemcpyAsync(w, k, in_bytes, cudaMemcpyHostToDevice, c->stream), "copy K");
    QL_CUDA(cudaMemcpyAsync(w + align256(in_bytes), v, in_bytes, cudaMemcpyHostToDevice,
                            c->stream),
            "copy V");
    kd_ptr = w;
    vd_ptr = w + align256(in_bytes);
  }
  ql::AppendArgs a{};
  a.k = kd_ptr;
  a.v = vd_ptr;
  a.in_dtype = in_dtype;
  a.batch = 1;
  a.new_len = static_cast<int32_t>(n);
  a.rope = nullptr;  // update() stores K as given (already rotated)
  a.cache = view_of(kv, layer);
  a.status = c->status;
  a.seqs.seq[0] = seq;
  a.seqs.start[0] = static_cast<int32_t>(cur);
  QL_CUDA(ql::launch_append(a, c->stream), "launch append");
  if (mem == QL_MEM_HOST) QL_CUDA(cudaStreamSynchronize(c->stream), "synchronize update");
  len_at(kv, layer, seq) = cur + n;
  return QL_OK;
}

int ql_kv_get(ql_ctx* c, const ql_kv* kv, int32_t layer, int32_t seq, const int32_t* positions,
              int64_t n_positions, float* k_out, float* v_out, int32_t mem) {
  if (!c || !kv) return fail(QL_ERR_INVALID, "ql_kv_get: NULL argument");
  if (layer < 0 || layer >= kv->cfg.num_layers)
    return fail(QL_ERR_INVALID, "KV cache layer index %d out of range (cache has %d layers)",
                layer, kv->cfg.num_layers);
  if (seq < 0 || seq >= kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", seq,
                kv->cfg.max_batch);
  const int64_t cur = kv->len[static_cast<size_t>(layer) * kv->cfg.max_batch + seq];
  for (int64_t i = 0; i < n_positions; ++i) {
    const int32_t p = positions[i];
    if (p < 0) return fail(QL_ERR_INVALID, "positions[%lld] = %d is negative", (long long)i, p);
    if (p >= cur)
      return fail(QL_ERR_INVALID,
                  "positions[%lld] = %d is at or beyond the written prefix (current_len %lld)",
                  (long long)i, p, (long long)cur);
  }
  if (n_positions == 0) return QL_OK;
  if (!k_out || !v_out) return fail(QL_ERR_INVALID, "ql_kv_get: NULL output");
  QL_CUDA(cudaSetDevice(c->device), "set device");
  const size_t ob = static_cast<size_t>(n_positions) * kv->cfg.num_kv_heads * kv->cfg.head_dim *
                    sizeof(float);
  const size_t pb = static_cast<size_t>(n_positions) * sizeof(int32_t);
  int r = ensure_ws(c, align256(pb) + (mem == QL_MEM_HOST ? 2 * align256(ob) : 0));
  if (r != QL_OK) return r;
  char* w = static_cast<char*>(c->ws);
  QL_CUDA(cudaMemcpyAsync(w, positions, pb, cudaMemcpyHostToDevice, c->stream), "copy positions");
  ql::GatherArgs g{};
  g.positions = reinterpret_cast<const int32_t*>(w);
  g.n = static_cast<int32_t>(n_positions);
  g.seq = seq;
  g.k_out = mem == QL_MEM_HOST ? reinterpret_cast<float*>(w + align256(pb)) : k_out;
  g.v_out = mem == QL_MEM_HOST ? reinterpret_cast<float*>(w + align256(pb) + align256(ob)) : v_out;
  g.cache = view_of(kv, layer);
  QL_CUDA(ql::launch_gather(g, c->stream), "launch gather");
  if (mem == QL_MEM_HOST) {
    QL_CUDA(cudaMemcpyAsync(k_out, g.k_out, ob, cudaMemcpyDeviceToHost, c->stream), "copy K out");
    QL_CUDA(cudaMemcpyAsync(v_out, g.v_out, ob, cudaMemcpyDeviceToHost, c->stream), "copy V out");
  }
  QL_CUDA(cudaStreamSynchronize(c->stream), "synchronize get");
  return QL_OK;
}

// The operator.  With `peer` (a head-sharded single-token decode), the
// split-KV kernel stores its rows into every rank's output instead of a->out.
// appended: the call's K/V rows are already in the cache (written by
// ql_qkv_rope_append at positions start_pos .. start_pos+new_len-1) and q
// arrives rotated, so nothing is appended and q is not rotated again.
static int attn_forward_impl(ql_ctx* c, ql_kv* kv, const ql_attn_args* a,
                             const ql::PeerOut* peer, bool appended = false) {
  if (!c || !kv || !a) return fail(QL_ERR_INVALID, "ql_attn_forward: NULL argument");
  const int hq = a->num_heads, hkv = a->num_kv_heads, hd = a->head_dim;
  // Attention::new (layers.rs:254-261)
  if (hq <= 0 || hkv <= 0 || hd <= 0)
    return fail(QL_ERR_INVALID, "Attention head counts and head_dim must be positive");
  if (hq % hkv != 0)
    return fail(QL_ERR_INVALID, "num_heads %d must be divisible by num_kv_heads %d", hq, hkv);
  if (a->batch < 1 || a->new_len < 0)
    return fail(QL_ERR_INVALID, "batch must be >= 1 and new_len >= 0 (got %d, %d)", a->batch,
                a->new_len);
  if (a->batch > ql::kMaxBatch || a->batch > kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "batch %d exceeds the limit (%d per call, %d cache slots)",
                a->batch, ql::kMaxBatch, kv->cfg.max_batch);
  if (!a->seq_ids || !a->start_pos) return fail(QL_ERR_INVALID, "seq_ids/start_pos are NULL");
  // rope parameters (ops.rs:170-182)
  if ((hd & 1) != 0)
    return fail(QL_ERR_INVALID,
                "RoPE requires shape [seq_len, ..., head_dim] with a positive even head_dim");
  if (!std::isfinite(a->rope_theta) || a->rope_theta <= 0.f)
    return fail(QL_ERR_INVALID, "RoPE theta must be finite and positive");
  if (!valid_io_dtype(a->in_dtype) || !valid_io_dtype(a->out_dtype))
    return fail(QL_ERR_INVALID, "unknown input/output dtype (%d, %d)", a->in_dtype, a->out_dtype);
  if (a->mem != QL_MEM_DEVICE && a->mem != QL_MEM_HOST)
    return fail(QL_ERR_INVALID, "unknown memory kind %d", a->mem);
  const int layer = a->layer_idx;
  if (layer < 0 || layer >= kv->cfg.num_layers)
    return fail(QL_ERR_INVALID, "KV cache layer index %d out of range (cache has %d layers)",
                layer, kv->cfg.num_layers);
  const int n = a->new_len;
  if (hkv != kv->cfg.num_kv_heads || hd != kv->cfg.head_dim)
    return fail(QL_ERR_INVALID, "K shape [%d, %d, %d] does not match cache [_, %d, %d]", n, hkv,
                hd, kv->cfg.num_kv_heads, kv->cfg.head_dim);
  int32_t seqs[ql::kMaxBatch];
  int64_t ends[ql::kMaxBatch];
  const uint32_t mark = next_seen_epoch(kv);
  for (int b = 0; b < a->batch; ++b) {
    const int s = a->seq_ids[b];
    if (s < 0 || s >= kv->cfg.max_batch)
      return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", s,
                  kv->cfg.max_batch);
    if (kv->seen_mark[s] == mark)
      return fail(QL_ERR_INVALID, "sequence %d appears twice in one call", s);
    kv->seen_mark[s] = mark;
    const int64_t start = a->start_pos[b];
    if (start < 0) return fail(QL_ERR_INVALID, "start_pos %lld is negative", (long long)start);
    const int64_t last = start + (n > 0 ? n - 1 : 0);
    if (last > INT32_MAX)
      return fail(QL_ERR_INVALID, "position %lld exceeds the i32 range the cache uses",
                  (long long)last);
    const int64_t cur = len_at(kv, layer, s);
    if (n > 0 && appended) {
      if (start + n != cur)
        return fail(QL_ERR_INVALID,
                    "the rows of positions %lld..%lld are not the last ones appended "
                    "(current_len %lld)", (long long)start, (long long)(start + n - 1),
                    (long long)cur);
    } else if (n > 0) {
      if (start != cur)
        return fail(QL_ERR_INVALID,
                    "positions[0] = %lld must continue from current_len (expected %lld); "
                    "skipping, backward, or double writes are not allowed",
                    (long long)start, (long long)cur);
      if (start + n > kv->cfg.max_seq_len)
        return fail(QL_ERR_INVALID, "positions[%lld] = %lld exceeds cache capacity %d",
                    (long long)(kv->cfg.max_seq_len - start),
                    (long long)kv->cfg.max_seq_len, kv->cfg.max_seq_len);
    } else if (start > cur) {
      return fail(QL_ERR_INVALID,
                  "positions[%lld] = %lld is at or beyond the written prefix (current_len %lld)",
                  (long long)cur, (long long)cur, (long long)cur);
    }
    seqs[b] = s;
    ends[b] = start + n;
  }
  if (n == 0) return QL_OK;  // empty batch (transformer_forward.rs:919-946)
  if (!a->q || (!appended && (!a->k || !a->v)) || !a->out)
    return fail(QL_ERR_INVALID, "q/k/v/out is NULL");
  if (appended && peer)
    return fail(QL_ERR_UNSUPPORTED, "a head-sharded call appends its own rows");
  if (peer && !(n == 1 && a->mem == QL_MEM_DEVICE && kv->have_maps &&
                ql::splitkv_supported(hd, kv->cfg.dtype, hq / hkv, kv->cfg.page_size)))
    return fail(QL_ERR_UNSUPPORTED, "the fused head-sharded exchange needs a single-token "
                "decode on the split-KV kernel");
  QL_CUDA(cudaSetDevice(c->device), "set device");
  bool patched = false;
  int r = appended ? QL_OK : reserve_pages(kv, seqs, ends, a->batch, &patched);
  if (r != QL_OK) return r;
  r = ensure_rope(kv, a->rope_theta);
  if (r != QL_OK) return r;

  const int group = hq / hkv;
  const int jobs = a->batch * n;
  const size_t qn = static_cast<size_t>(jobs) * hq * hd, kn = static_cast<size_t>(jobs) * hkv * hd;
  const size_t ib = elem_bytes(a->in_dtype), obb = elem_bytes(a->out_dtype);
  const bool fast = kv->have_maps && ql::splitkv_supported(hd, kv->cfg.dtype, group,
                                                          kv->cfg.page_size);
  const bool tc_prefill = kv->have_maps && n > 1 &&
                          ql::prefill_tc_supported(hd, kv->cfg.dtype, n);
  // split planning for the tensor-core kernel
  int max_tiles = 0;
  int max_len = 0;
  int row_tiles[ql::kMaxBatch];
  for (int b = 0; b < a->batch; ++b) {
    const int64_t end = ends[b];
    max_len = std::max<int>(max_len, static_cast<int>(end));
    row_tiles[b] = static_cast<int>((end + ql::kTile - 1) / ql::kTile);
    max_tiles = std::max(max_tiles, row_tiles[b]);
  }
  int tps = max_tiles, max_splits = 1;
  // Too few (token, KV head) jobs to fill half the SMs: the wide kernel, whose
  // consumer groups share each split's tiles, one CTA per SM (latency).
  const int wide_kg = fast ? ql::splitkv_wide_groups(hd, kv->cfg.dtype) : 0;
  const bool latency = fast && 2LL * jobs * hkv <= c->num_sms;
  // A short context in that regime: each job's tiles spread over up to
  // kMaxCluster CTAs (one tile each when every CTA of the launch then has an
  // SM of its own, more otherwise), as one thread-block cluster that merges
  // through distributed shared memory (each CTA streams its tiles on its own
  // SM; one SM's TMA alone moves a few tens of GB/s).
  // Clusters above the portable 8 CTAs only while there are few of them, so
  // that each finds a GPC with that many free SMs; at most 8 tiles per CTA
  // (longer contexts use every SM through the kernels below).
  const long long pairs = 1LL * jobs * hkv;
  const int max_cluster = pairs <= 4 ? ql::kMaxClusterCtas : std::min(8, ql::kMaxClusterCtas);
  const long long pair_tiles = 1LL * max_tiles * pairs;
  const int cta_tiles = static_cast<int>(
      std::max<long long>((pair_tiles + c->num_sms - 1) / c->num_sms,
                          (max_tiles + max_cluster - 1) / max_cluster));
  const int cluster_ctas = (max_tiles + cta_tiles - 1) / cta_tiles;
  const bool clustered = latency && cluster_ctas >= 2 && cta_tiles <= 8;
  const bool wide = !clustered && latency && wide_kg > 0;
  int cluster = 0;
  if (clustered) {
    tps = (max_tiles + cluster_ctas - 1) / cluster_ctas;
    max_splits = (max_tiles + tps - 1) / tps;
    cluster = max_splits;
  } else if (wide) {
    tps = wide_tiles_per_split(max_tiles, wide_kg, 1LL * jobs * hkv, c->num_sms);
    max_splits = (max_tiles + tps - 1) / tps;
  } else if (fast) {
    const int per_sm = std::max(1, ql::splitkv_ctas_per_sm(hd, kv->cfg.dtype, false));
    const SplitPlan plan =
        plan_splits(row_tiles, a->batch, static_cast<long long>(n) * hkv,
                    1LL * per_sm * c->num_sms);
    tps = plan.tps;
    max_splits = plan.splits;
  }
  // workspace: [staged q][k][v][out][part_o][part_ml][rotated q][its row scales]
  //            [bf16 caches: f16 copies of K and V, tile exponents]
  //            [generic scratch f32][f64]
  size_t off = 0;
  const size_t o_q = off; off += align256(a->mem == QL_MEM_HOST ? qn * ib : 0);
  const size_t o_k = off; off += align256(a->mem == QL_MEM_HOST ? kn * ib : 0);
  const size_t o_v = off; off += align256(a->mem == QL_MEM_HOST ? kn * ib : 0);
  const size_t o_o = off; off += align256(a->mem == QL_MEM_HOST ? qn * obb : 0);
  const size_t o_po = off;
  if (fast && max_splits > 1)
    off += align256(static_cast<size_t>(jobs) * hkv * max_splits * 8 * hd * sizeof(float));
  const size_t o_pm = off;
  if (fast && max_splits > 1)
    off += align256(static_cast<size_t>(jobs) * hkv * max_splits * 8 * 2 * sizeof(float));
  const size_t q_rows = ql::prefill_q_rows(n);
  const size_t o_qr = off;
  if (tc_prefill) off += align256(static_cast<size_t>(a->batch) * hq * q_rows * hd * 2);
  const size_t o_qs = off;
  if (tc_prefill) off += align256(static_cast<size_t>(a->batch) * hq * q_rows * sizeof(float));
  // bf16 and Q8_0: every key the call sees, per (sequence, KV head), padded to 128
  const bool bf_copy = tc_prefill && (kv->cfg.dtype == QL_BF16 || kv->cfg.dtype == QL_Q8_0);
  const size_t kv_rows = static_cast<size_t>((max_len + 127) / 128) * 128;
  const size_t copy_bytes = static_cast<size_t>(a->batch) * hkv * kv_rows * hd * 2;
  const size_t o_kc = off;
  if (bf_copy) off += align256(copy_bytes);
  const size_t o_vc = off;
  if (bf_copy) off += align256(copy_bytes);
  const size_t o_te = off;
  if (bf_copy) off += align256(2 * static_cast<size_t>(a->batch) * hkv * (kv_rows / 128));
  const int gjobs = std::min(jobs, 65535);
  const size_t o_gs = off;
  if (!fast) off += align256(static_cast<size_t>(gjobs) * hq * max_len * sizeof(float));
  const size_t o_gd = off;
  if (!fast) off += align256(static_cast<size_t>(gjobs) * hq * max_len * sizeof(double));
  r = ensure_ws(c, off);
  if (r != QL_OK) return r;
  if (fast && max_splits > 1) {
    r = ensure_counters(c, static_cast<size_t>(jobs) * hkv);
    if (r != QL_OK) return r;
  }
  char* w = static_cast<char*>(c->ws);
  const void *q = a->q, *k = a->k, *v = a->v;
  void* out = a->out;
  if (a->mem == QL_MEM_HOST) {
    QL_CUDA(cudaMemcpyAsync(w + o_q, a->q, qn * ib, cudaMemcpyHostToDevice, c->stream), "copy q");
    if (!appended) {
      QL_CUDA(cudaMemcpyAsync(w + o_k, a->k, kn * ib, cudaMemcpyHostToDevice, c->stream),
              "copy k");
      QL_CUDA(cudaMemcpyAsync(w + o_v, a->v, kn * ib, cudaMemcpyHostToDevice, c->stream),
              "copy v");
    }
    q = w + o_q;
    k = w + o_k;
    v = w + o_v;
    out = w + o_o;
  }
  ql::CacheView cv = view_of(kv, layer);
  ql::SeqTable st{};
  for (int b = 0; b < a->batch; ++b) {
    st.seq[b] = seqs[b];
    st.start[b] = static_cast<int32_t>(a->start_pos[b]);
  }
  const bool fuse = fast && n == 1 && !appended;
  ql::AppendArgs ap{};
  ap.k = k;
  ap.v = v;
  ap.in_dtype = a->in_dtype;
  ap.batch = a->batch;
  ap.new_len = appended ? 0 : n;  // no rows for the prefill prologue to append
  ap.rope = kv->d_rope;
  ap.cache = cv;
  ap.status = c->status;
  ap.seqs = st;
  // the tcgen05 prefill appends in its prologue kernel; a single-token decode
  // on the split-KV kernel appends inside that kernel
  if (!fuse && !tc_prefill && !appended)
    QL_CUDA(ql::launch_append(ap, c->stream), "launch append");
  // queries: rotated here with the position's row, or taken as they are
  const double2* q_rope = appended ? kv->d_rope_id : kv->d_rope;
  const int32_t q_rope_stride = appended ? 0 : hd / 2;
  if (tc_prefill) {
    ql::PrefillArgs pa{};
    pa.q = q;
    pa.in_dtype = a->in_dtype;
    pa.q_rot = reinterpret_cast<__half*>(w + o_qr);
    pa.q_scale = reinterpret_cast<float*>(w + o_qs);
    pa.q_rows = static_cast<int32_t>(q_rows);
    pa.out = out;
    pa.out_dtype = a->out_dtype;
    pa.rope = q_rope;
    pa.rope_stride = q_rope_stride;
    pa.cache = cv;
    pa.hq = hq;
    pa.group = group;
    pa.batch = a->batch;
    pa.new_len = n;
    pa.scale = 1.0f / std::sqrt(static_cast<float>(hd));  // layers.rs:432
    pa.num_sms = c->num_sms;
    pa.status = c->status;
    pa.seqs = st;
    CUtensorMap qmap;
    r = encode_q_map(&qmap, w + o_qr, hd, static_cast<uint64_t>(a->batch) * hq * q_rows);
    if (r != QL_OK) return r;
    const CUtensorMap* kmap = &kv->kmap[layer];
    const CUtensorMap* vmap = &kv->vmap[layer];
    CUtensorMap kcm, vcm;  // bf16 / Q8_0: the attention kernel reads the f16 copies
    if (bf_copy) {
      pa.k_copy = reinterpret_cast<__half*>(w + o_kc);
      pa.v_copy = reinterpret_cast<__half*>(w + o_vc);
      pa.tile_exp = reinterpret_cast<int8_t*>(w + o_te);
      pa.kv_rows = static_cast<int32_t>(kv_rows);
      const uint64_t rows = static_cast<uint64_t>(a->batch) * hkv * kv_rows;
      r = encode_map(&kcm, w + o_kc, QL_F16, hd, rows);
      if (r == QL_OK) r = encode_map(&vcm, w + o_vc, QL_F16, hd, rows);
      if (r != QL_OK) return r;
      kmap = &kcm;
      vmap = &vcm;
    }
    QL_CUDA(ql::launch_prefill_tc(pa, ap, &qmap, kmap, vmap, c->stream),
            "launch tcgen05 prefill");
    if (a->mem == QL_MEM_HOST) {
      QL_CUDA(cudaMemcpyAsync(a->out, out, qn * obb, cudaMemcpyDeviceToHost, c->stream),
              "copy out");
      QL_CUDA(cudaStreamSynchronize(c->stream), "synchronize forward");
    }
    for (int b = 0; b < a->batch; ++b) len_at(kv, layer, seqs[b]) = ends[b];
    return QL_OK;
  }
  ql::AttnArgs at{};
  at.q = q;
  at.k = k;
  at.v = v;
  at.in_dtype = a->in_dtype;
  at.out = out;
  at.out_dtype = a->out_dtype;
  at.rope = q_rope;
  at.rope_stride = q_rope_stride;
  at.cache = cv;
  at.hq = hq;
  at.group = group;
  at.batch = a->batch;
  at.new_len = n;
  at.scale = 1.0f / std::sqrt(static_cast<float>(hd));  // layers.rs:432
  at.fuse_append = fuse ? 1 : 0;
  at.tiles_per_split = tps;
  at.max_splits = max_splits;
  at.part_o = reinterpret_cast<float*>(w + o_po);
  at.part_ml = reinterpret_cast<float*>(w + o_pm);
  at.counters = c->counters;
  at.scratch = reinterpret_cast<float*>(w + o_gs);
  at.scratch_d = reinterpret_cast<double*>(w + o_gd);
  at.max_len = max_len;
  at.out_vec = (reinterpret_cast<uintptr_t>(out) % 16) == 0;
  at.wide = wide ? 1 : 0;
  at.cluster = cluster;
  at.status = c->status;
  at.seqs = st;
  if (peer) {
    at.peer = *peer;
    at.peer.total_ctas = max_splits * hkv * jobs;
    at.out_vec = 1;  // symmetric buffers are 256-byte aligned
  }
  if (fast)
    QL_CUDA(ql::launch_splitkv(at, &kv->kmap[layer], &kv->vmap[layer], jobs, c->stream,
                               /*pdl=*/!patched),
            "launch split-KV attention");
  else
    QL_CUDA(ql::launch_generic(at, c->stream), "launch attention");
  if (a->mem == QL_MEM_HOST) {
    QL_CUDA(cudaMemcpyAsync(a->out, out, qn * obb, cudaMemcpyDeviceToHost, c->stream),
            "copy out");
    QL_CUDA(cudaStreamSynchronize(c->stream), "synchronize forward");
  }
  for (int b = 0; b < a->batch; ++b) len_at(kv, layer, seqs[b]) = ends[b];
  return QL_OK;
}

int ql_attn_forward(ql_ctx* c, ql_kv* kv, const ql_attn_args* a) {
  return attn_forward_impl(c, kv, a, nullptr);
}

int ql_attn_forward_appended(ql_ctx* c, ql_kv* kv, const ql_attn_args* a) {
  return attn_forward_impl(c, kv, a, nullptr, true);
}

}  // extern "C"

// Library-internal half of ql_qkv_rope_append (ql_model.cu): validates the
// call's positions like KvCache::update (cache.rs:90-144), gives the
// sequences the pages they need (a table patch launch, no host
// synchronisation) and the RoPE table, and reports where the rows go.  The
// caller launches the kernel that writes them, then ql_kv_append_commit.
int ql_kv_append_prepare(ql_ctx* c, ql_kv* kv, const ql_attn_args* a, ql::CacheView* view,
                         const double2** rope, ql::SeqTable* st) {
  if (!c || !kv || !a) return fail(QL_ERR_INVALID, "ql_qkv_rope_append: NULL argument");
  const int hq = a->num_heads, hkv = a->num_kv_heads, hd = a->head_dim;
  if (hq <= 0 || hkv <= 0 || hd <= 0)
    return fail(QL_ERR_INVALID, "Attention head counts and head_dim must be positive");
  if (hq % hkv != 0)
    return fail(QL_ERR_INVALID, "num_heads %d must be divisible by num_kv_heads %d", hq, hkv);
  if ((hd & 1) != 0)
    return fail(QL_ERR_INVALID,
                "RoPE requires shape [seq_len, ..., head_dim] with a positive even head_dim");
  if (!std::isfinite(a->rope_theta) || a->rope_theta <= 0.f)
    return fail(QL_ERR_INVALID, "RoPE theta must be finite and positive");
  if (a->batch < 1 || a->new_len < 0 || a->batch > ql::kMaxBatch || a->batch > kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "batch %d / new_len %d outside the limits", a->batch, a->new_len);
  if (!a->seq_ids || !a->start_pos) return fail(QL_ERR_INVALID, "seq_ids/start_pos are NULL");
  const int layer = a->layer_idx;
  if (layer < 0 || layer >= kv->cfg.num_layers)
    return fail(QL_ERR_INVALID, "KV cache layer index %d out of range (cache has %d layers)",
                layer, kv->cfg.num_layers);
  if (hkv != kv->cfg.num_kv_heads || hd != kv->cfg.head_dim)
    return fail(QL_ERR_INVALID, "K shape [%d, %d, %d] does not match cache [_, %d, %d]",
                a->new_len, hkv, hd, kv->cfg.num_kv_heads, kv->cfg.head_dim);
  if (kv->cfg.dtype == QL_Q8_0)
    return fail(QL_ERR_UNSUPPORTED, "the fused projection appends f32, f16 or bf16 rows; a Q8_0 "
                "cache takes ql_attn_forward");
  const int n = a->new_len;
  int32_t seqs[ql::kMaxBatch];
  int64_t ends[ql::kMaxBatch];
  const uint32_t mark = next_seen_epoch(kv);
  for (int b = 0; b < a->batch; ++b) {
    const int s = a->seq_ids[b];
    if (s < 0 || s >= kv->cfg.max_batch)
      return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", s,
                  kv->cfg.max_batch);
    if (kv->seen_mark[s] == mark)
      return fail(QL_ERR_INVALID, "sequence %d appears twice in one call", s);
    kv->seen_mark[s] = mark;
    const int64_t start = a->start_pos[b], cur = len_at(kv, layer, s);
    if (start != cur)
      return fail(QL_ERR_INVALID,
                  "positions[0] = %lld must continue from current_len (expected %lld); "
                  "skipping, backward, or double writes are not allowed",
                  (long long)start, (long long)cur);
    if (start + n > kv->cfg.max_seq_len)
      return fail(QL_ERR_INVALID, "positions[%lld] = %lld exceeds cache capacity %d",
                  (long long)(kv->cfg.max_seq_len - start), (long long)kv->cfg.max_seq_len,
                  kv->cfg.max_seq_len);
    seqs[b] = s;
    ends[b] = start + n;
    st->seq[b] = s;
    st->start[b] = static_cast<int32_t>(start);
  }
  QL_CUDA(cudaSetDevice(c->device), "set device");
  bool patched = false;
  int r = n > 0 ? reserve_pages(kv, seqs, ends, a->batch, &patched) : QL_OK;
  if (r == QL_OK) r = ensure_rope(kv, a->rope_theta);
  if (r != QL_OK) return r;
  *view = view_of(kv, layer);
  *rope = kv->d_rope;
  return QL_OK;
}

void ql_kv_append_commit(ql_kv* kv, const ql_attn_args* a) {
  for (int b = 0; b < a->batch; ++b)
    len_at(kv, a->layer_idx, a->seq_ids[b]) = a->start_pos[b] + a->new_len;
}

extern "C" {

int ql_attn_decode_noalloc(ql_ctx* c, ql_kv* kv, const ql_attn_args* a) {
  if (!c || !kv || !a) return fail(QL_ERR_INVALID, "ql_attn_decode_noalloc: NULL argument");
  const int hq = a->num_heads, hkv = a->num_kv_heads, hd = a->head_dim;
  if (hq <= 0 || hkv <= 0 || hd <= 0)
    return fail(QL_ERR_INVALID, "Attention head counts and head_dim must be positive");
  if (hq % hkv != 0)
    return fail(QL_ERR_INVALID, "num_heads %d must be divisible by num_kv_heads %d", hq, hkv);
  if (a->new_len != 1)
    return fail(QL_ERR_INVALID, "ql_attn_decode_noalloc decodes one token per sequence "
                "(new_len 1), got new_len %d", a->new_len);
  if (a->mem != QL_MEM_DEVICE)
    return fail(QL_ERR_INVALID, "ql_attn_decode_noalloc takes device buffers only "
                "(host staging would need an allocation)");
  if (a->batch < 1 || a->batch > ql::kMaxBatch || a->batch > kv->cfg.max_batch)
    return fail(QL_ERR_INVALID, "batch %d is outside 1..%d (%d cache slots)", a->batch,
                ql::kMaxBatch, kv->cfg.max_batch);
  if (static_cast<long long>(a->batch) * hkv > kNoAllocPairs)
    return fail(QL_ERR_INVALID, "batch*num_kv_heads = %lld exceeds the no-allocation limit of %d "
                "(sequence, KV head) pairs", static_cast<long long>(a->batch) * hkv,
                kNoAllocPairs);
  if (!a->seq_ids || !a->start_pos || !a->q || !a->k || !a->v || !a->out)
    return fail(QL_ERR_INVALID, "ql_attn_decode_noalloc: NULL buffer");
  if ((hd & 1) != 0)
    return fail(QL_ERR_INVALID,
                "RoPE requires shape [seq_len, ..., head_dim] with a positive even head_dim");
  if (!std::isfinite(a->rope_theta) || a->rope_theta <= 0.f)
    return fail(QL_ERR_INVALID, "RoPE theta must be finite and positive");
  if (!valid_io_dtype(a->in_dtype) || !valid_io_dtype(a->out_dtype))
    return fail(QL_ERR_INVALID, "unknown input/output dtype (%d, %d)", a->in_dtype, a->out_dtype);
  const int layer = a->layer_idx;
  if (layer < 0 || layer >= kv->cfg.num_layers)
    return fail(QL_ERR_INVALID, "KV cache layer index %d out of range (cache has %d layers)",
                layer, kv->cfg.num_layers);
  if (hkv != kv->cfg.num_kv_heads || hd != kv->cfg.head_dim)
    return fail(QL_ERR_INVALID, "K shape [1, %d, %d] does not match cache [_, %d, %d]", hkv, hd,
                kv->cfg.num_kv_heads, kv->cfg.head_dim);
  const int group = hq / hkv;
  if (!kv->have_maps || !ql::splitkv_supported(hd, kv->cfg.dtype, group, kv->cfg.page_size))
    return fail(QL_ERR_UNSUPPORTED, "ql_attn_decode_noalloc needs an f16/bf16 cache with head_dim "
                "64 or 128 or a Q8_0 cache with head_dim 128, and at most 8 query heads per KV "
                "head");
  int32_t seqs[ql::kMaxBatch];
  int64_t ends[ql::kMaxBatch];
  int max_tiles = 0;
  int row_tiles[ql::kMaxBatch];
  const uint32_t mark = next_seen_epoch(kv);
  for (int b = 0; b < a->batch; ++b) {
    const int s = a->seq_ids[b];
    if (s < 0 || s >= kv->cfg.max_batch)
      return fail(QL_ERR_INVALID, "sequence %d out of range (cache has %d slots)", s,
                  kv->cfg.max_batch);
    if (kv->seen_mark[s] == mark)
      return fail(QL_ERR_INVALID, "sequence %d appears twice in one call", s);
    kv->seen_mark[s] = mark;
    const int64_t start = a->start_pos[b], cur = len_at(kv, layer, s);
    if (start < 0) return fail(QL_ERR_INVALID, "start_pos %lld is negative", (long long)start);
    if (start != cur)
      return fail(QL_ERR_INVALID,
                  "positions[0] = %lld must continue from current_len (expected %lld); "
                  "skipping, backward, or double writes are not allowed",
                  (long long)start, (long long)cur);
    if (start + 1 > kv->cfg.max_seq_len)
      return fail(QL_ERR_INVALID, "positions[0] = %lld exceeds cache capacity %d",
                  (long long)start, kv->cfg.max_seq_len);
    seqs[b] = s;
    ends[b] = start + 1;
    row_tiles[b] = static_cast<int>((ends[b] + ql::kTile - 1) / ql::kTile);
    max_tiles = std::max(max_tiles, row_tiles[b]);
  }
  QL_CUDA(cudaSetDevice(c->device), "set device");
  char* scratch = nullptr;
  int r = noalloc_scratch(c->device, &scratch);
  if (r != QL_OK) return r;
  bool patched = false;  // the launch below never uses programmatic dependent launch
  r = reserve_pages(kv, seqs, ends, a->batch, &patched);  // hands out pool pages; allocates nothing
  if (r != QL_OK) return r;
  // Split plan of ql_attn_forward, with fewer splits if the partials would not fit.
  const int jobs = a->batch;
  const int per_sm = std::max(1, ql::splitkv_ctas_per_sm(hd, kv->cfg.dtype, true));
  int tps = plan_splits(row_tiles, a->batch, hkv, 1LL * per_sm * c->num_sms).tps;
  auto part_bytes = [&](int splits) {
    return align256(static_cast<size_t>(jobs) * hkv * splits * 8 * 2 * sizeof(float)) +
           static_cast<size_t>(jobs) * hkv * splits * 8 * hd * sizeof(float);
  };
  int max_splits = (max_tiles + tps - 1) / tps;
  while (max_splits > 1 && part_bytes(max_splits) > kNoAllocBytes - kNoAllocCounterBytes) {
    ++tps;
    max_splits = (max_tiles + tps - 1) / tps;
  }
  int32_t* counters = reinterpret_cast<int32_t*>(scratch);
  float* part_ml = reinterpret_cast<float*>(scratch + kNoAllocCounterBytes);
  float* part_o = reinterpret_cast<float*>(
      scratch + kNoAllocCounterBytes +
      align256(static_cast<size_t>(jobs) * hkv * max_splits * 8 * 2 * sizeof(float)));
  // The array keeps the previous call's contents: the counters must start at zero.
  QL_CUDA(cudaMemsetAsync(counters, 0, static_cast<size_t>(jobs) * hkv * sizeof(int32_t),
                          c->stream),
          "clear the no-allocation counters");
  ql::AttnArgs at{};
  at.q = a->q;
  at.k = a->k;
  at.v = a->v;
  at.in_dtype = a->in_dtype;
  at.out = a->out;
  at.out_dtype = a->out_dtype;
  at.rope = nullptr;
  at.rope_theta = a->rope_theta;
  at.cache = view_of(kv, layer);
  at.hq = hq;
  at.group = group;
  at.batch = a->batch;
  at.new_len = 1;
  at.scale = 1.0f / std::sqrt(static_cast<float>(hd));
  at.fuse_append = 1;
  at.tiles_per_split = tps;
  at.max_splits = max_splits;
  at.part_o = part_o;
  at.part_ml = part_ml;
  at.counters = counters;
  at.out_vec = (reinterpret_cast<uintptr_t>(a->out) % 16) == 0;
  at.status = c->status;
  for (int b = 0; b < a->batch; ++b) {
    at.seqs.seq[b] = seqs[b];
    at.seqs.start[b] = static_cast<int32_t>(a->start_pos[b]);
  }
  QL_CUDA(ql::launch_splitkv_device_rope(at, &kv->kmap[layer], &kv->vmap[layer], jobs, c->stream),
          "launch no-allocation decode");
  for (int b = 0; b < a->batch; ++b) len_at(kv, layer, seqs[b]) = ends[b];
  return QL_OK;
}

}  // extern "C"


// ------------------------------------------------ head-sharded layers --
// NCCL is opened on first use, so that single-GPU callers never need it.
namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl_api() {
  static const NcclApi api = [] {
    NcclApi x;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      x.why = e ? e : "dlopen failed";
      return x;
    }
    x.get_unique_id = reinterpret_cast<decltype(x.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    x.comm_init_rank = reinterpret_cast<decltype(x.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    x.comm_destroy = reinterpret_cast<decltype(x.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    x.all_gather = reinterpret_cast<decltype(x.all_gather)>(dlsym(h, "ncclAllGather"));
    x.error_string = reinterpret_cast<decltype(x.error_string)>(dlsym(h, "ncclGetErrorString"));
    x.ok = x.get_unique_id && x.comm_init_rank && x.comm_destroy && x.all_gather && x.error_string;
    if (!x.ok) x.why = "libnccl.so.2 lacks an entry point this library calls";
    return x;
  }();
  return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
  return fail(QL_ERR_CUDA, "%s: %s", what, nccl_api().error_string(r));
}

// Each rank's symmetric buffer starts with this many bytes of flags
// (PeerOut: entered[kMaxRanks], done[kMaxRanks]); the output follows.
constexpr size_t kCommFlagBytes = 4096;
static_assert(sizeof(ncclUniqueId) == QL_COMM_ID_BYTES, "unique id size");
static_assert(QL_COMM_MAX_RANKS == ql::kMaxRanks, "rank limit");

}  // namespace

struct ql_comm {
  ql_ctx* ctx = nullptr;
  int nranks = 1;
  int rank = 0;
  int mode = QL_COMM_P2P;
  ncclComm_t nccl = nullptr;
  char* sym = nullptr;                      // this rank's [flags][output]
  size_t out_bytes = 0;
  char* base[ql::kMaxRanks] = {};           // every rank's symmetric buffer, mapped here
  int32_t* arrivals = nullptr;              // device: CTA arrival counter, then the call count
  void* stage = nullptr;                    // compact local rows of non-fused calls
  void* gather = nullptr;                   // QL_COMM_NCCL: rank-major gathered rows
};

namespace {

void release_comm(ql_comm* cm) {
  for (int p = 0; p < cm->nranks; ++p)
    if (p != cm->rank && cm->base[p]) cudaIpcCloseMemHandle(cm->base[p]);
  if (cm->sym) cudaFree(cm->sym);
  if (cm->arrivals) cudaFree(cm->arrivals);
  if (cm->stage) cudaFree(cm->stage);
  if (cm->gather) cudaFree(cm->gather);
  if (cm->nccl) nccl_api().comm_destroy(cm->nccl);
  delete cm;
}

}  // namespace

int ql_comm_unique_id(ql_comm_id* out) {
  if (!out) return fail(QL_ERR_INVALID, "ql_comm_unique_id: NULL argument");
  const NcclApi& nc = nccl_api();
  if (!nc.ok) return fail(QL_ERR_UNSUPPORTED, "NCCL is not available: %s", nc.why.c_str());
  ncclUniqueId id;
  const ncclResult_t r = nc.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(out->bytes, &id, sizeof id);
  return QL_OK;
}

int ql_comm_create(ql_ctx* c, int nranks, int rank, const ql_comm_id* id,
                   uint64_t max_out_bytes, int mode, ql_comm** out) {
  if (!c || !id || !out) return fail(QL_ERR_INVALID, "ql_comm_create: NULL argument");
  if (nranks < 1 || nranks > ql::kMaxRanks)
    return fail(QL_ERR_INVALID, "nranks %d is outside 1..%d", nranks, ql::kMaxRanks);
  if (rank < 0 || rank >= nranks)
    return fail(QL_ERR_INVALID, "rank %d is outside 0..%d", rank, nranks - 1);
  if (mode != QL_COMM_P2P && mode != QL_COMM_NCCL)
    return fail(QL_ERR_INVALID, "unknown communicator mode %d", mode);
  if (max_out_bytes == 0) return fail(QL_ERR_INVALID, "max_out_bytes must be positive");
  const NcclApi& nc = nccl_api();
  if (!nc.ok) return fail(QL_ERR_UNSUPPORTED, "NCCL is not available: %s", nc.why.c_str());
  QL_CUDA(cudaSetDevice(c->device), "set device");
  ql_comm* cm = new ql_comm;
  cm->ctx = c;
  cm->nranks = nranks;
  cm->rank = rank;
  cm->mode = mode;
  cm->out_bytes = align256(static_cast<size_t>(max_out_bytes));
  auto bail = [&](int code) {
    release_comm(cm);
    return code;
  };
  ncclUniqueId uid;
  std::memcpy(&uid, id->bytes, sizeof uid);
  ncclResult_t nr = nc.comm_init_rank(&cm->nccl, nranks, uid, rank);
  if (nr != ncclSuccess) {
    cm->nccl = nullptr;
    return bail(nccl_fail(nr, "ncclCommInitRank"));
  }
  cudaError_t e = cudaMalloc(&cm->sym, kCommFlagBytes + cm->out_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&cm->arrivals, 256);
  if (e == cudaSuccess) e = cudaMalloc(&cm->stage, cm->out_bytes);
  if (e == cudaSuccess && mode == QL_COMM_NCCL) e = cudaMalloc(&cm->gather, cm->out_bytes);
  if (e == cudaSuccess) e = cudaMemset(cm->sym, 0, kCommFlagBytes);
  if (e == cudaSuccess) e = cudaMemset(cm->arrivals, 0, 256);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return bail(cuda_fail(e, "allocate the communicator's buffers"));
  cm->base[rank] = cm->sym;
  if (nranks > 1) {
    // One all-gather of every rank's buffer handle, size and mode: every rank
    // must have made the same buffer (remote stores assume it) and mode.
    struct Card {
      cudaIpcMemHandle_t handle;
      uint64_t out_bytes;
      int64_t mode;
    };
    Card mine{};
    mine.out_bytes = cm->out_bytes;
    mine.mode = mode;
    if (mode == QL_COMM_P2P) {
      e = cudaIpcGetMemHandle(&mine.handle, cm->sym);
      if (e != cudaSuccess) return bail(cuda_fail(e, "export the output buffer"));
    }
    std::vector<Card> all(nranks);
    char* dh = nullptr;
    e = cudaMalloc(&dh, nranks * sizeof(Card));
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dh + rank * sizeof(Card), &mine, sizeof(Card), cudaMemcpyHostToDevice,
                          c->stream);  // ordered before the all-gather on the same stream
    if (e != cudaSuccess) {
      if (dh) cudaFree(dh);
      return bail(cuda_fail(e, "stage the buffer cards"));
    }
    nr = nc.all_gather(dh + rank * sizeof(Card), dh, sizeof(Card), ncclUint8, cm->nccl,
                       c->stream);
    if (nr == ncclSuccess) {
      e = cudaStreamSynchronize(c->stream);
      if (e == cudaSuccess)
        e = cudaMemcpy(all.data(), dh, nranks * sizeof(Card), cudaMemcpyDeviceToHost);
    }
    cudaFree(dh);
    if (nr != ncclSuccess) return bail(nccl_fail(nr, "exchange the buffer cards"));
    if (e != cudaSuccess) return bail(cuda_fail(e, "exchange the buffer cards"));
    for (int p = 0; p < nranks; ++p)
      if (all[p].out_bytes != cm->out_bytes || all[p].mode != mode)
        return bail(fail(QL_ERR_INVALID, "rank %d made its communicator with %llu output bytes "
                         "and mode %lld, rank %d with %zu and %d: every rank must pass the same",
                         p, static_cast<unsigned long long>(all[p].out_bytes),
                         static_cast<long long>(all[p].mode), rank, cm->out_bytes, mode));
    for (int p = 0; p < nranks && mode == QL_COMM_P2P; ++p) {
      if (p == rank) continue;
      void* ptr = nullptr;
      e = cudaIpcOpenMemHandle(&ptr, all[p].handle, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) return bail(cuda_fail(e, "map another rank's output buffer"));
      cm->base[p] = static_cast<char*>(ptr);
    }
  }
  *out = cm;
  return QL_OK;
}

int ql_comm_destroy(ql_comm* cm) {
  if (!cm) return fail(QL_ERR_INVALID, "ql_comm_destroy: NULL argument");
  QL_CUDA(cudaSetDevice(cm->ctx->device), "set device");
  QL_CUDA(cudaStreamSynchronize(cm->ctx->stream), "synchronize before destroying");
  if (cm->nranks > 1) {
    // No rank unmaps or frees while another may still store into it.
    const ncclResult_t nr = nccl_api().all_gather(
        static_cast<char*>(cm->stage) + cm->rank * 4, cm->stage, 4, ncclUint8, cm->nccl,
        cm->ctx->stream);
    if (nr != ncclSuccess) return nccl_fail(nr, "barrier before destroying");
    QL_CUDA(cudaStreamSynchronize(cm->ctx->stream), "barrier before destroying");
  }
  release_comm(cm);
  return QL_OK;
}

int ql_comm_buffer(ql_comm* cm, void** out, uint64_t* bytes) {
  if (!cm || !out) return fail(QL_ERR_INVALID, "ql_comm_buffer: NULL argument");
  *out = cm->sym + kCommFlagBytes;
  if (bytes) *bytes = cm->out_bytes;
  return QL_OK;
}

int ql_attn_forward_sharded(ql_ctx* c, ql_kv* kv, ql_comm* cm, const ql_attn_args* a) {
  if (!c || !kv || !cm || !a) return fail(QL_ERR_INVALID, "ql_attn_forward_sharded: NULL argument");
  if (cm->ctx != c)
    return fail(QL_ERR_INVALID, "the communicator belongs to another context");
  if (a->mem != QL_MEM_DEVICE)
    return fail(QL_ERR_INVALID, "ql_attn_forward_sharded takes device buffers only");
  if (!valid_io_dtype(a->out_dtype))
    return fail(QL_ERR_INVALID, "unknown input/output dtype (%d, %d)", a->in_dtype, a->out_dtype);
  if (a->num_heads <= 0 || a->num_kv_heads <= 0 || a->head_dim <= 0 || a->batch < 1 ||
      a->new_len < 0)
    return attn_forward_impl(c, kv, a, nullptr);  // the operator's own messages
  const int nranks = cm->nranks, hq_l = a->num_heads, hd = a->head_dim;
  const size_t eb = elem_bytes(a->out_dtype);
  const int64_t rows = static_cast<int64_t>(a->batch) * a->new_len;
  const size_t row_bytes = static_cast<size_t>(hq_l) * hd * eb;  // this rank's part of a row
  if (static_cast<size_t>(rows) * row_bytes * nranks > cm->out_bytes)
    return fail(QL_ERR_INVALID, "the output (%lld rows of %zu bytes) exceeds the communicator's "
                "buffer of %zu bytes", static_cast<long long>(rows), row_bytes * nranks,
                cm->out_bytes);
  if (nranks == 1 || rows == 0) return attn_forward_impl(c, kv, a, nullptr);
  char* symout = cm->sym + kCommFlagBytes;
  ql::PeerOut po{};
  po.nranks = nranks;
  po.rank = cm->rank;
  po.hq_total = hq_l * nranks;
  po.head_base = cm->rank * hq_l;
  po.arrivals = cm->arrivals;
  po.epoch = reinterpret_cast<uint32_t*>(cm->arrivals) + 16;  // its own 64-byte line
  for (int p = 0; p < nranks; ++p) {
    po.out[p] = cm->base[p] + kCommFlagBytes;
    po.flags[p] = reinterpret_cast<uint32_t*>(cm->base[p]);
  }
  const bool fused = cm->mode == QL_COMM_P2P && a->new_len == 1 && kv->have_maps &&
                     a->num_heads % a->num_kv_heads == 0 &&
                     ql::splitkv_supported(hd, kv->cfg.dtype, a->num_heads / a->num_kv_heads,
                                           kv->cfg.page_size);
  int r;
  if (fused) {
    r = attn_forward_impl(c, kv, a, &po);
    if (r != QL_OK) return r;
  } else {
    ql_attn_args local = *a;
    local.out = cm->stage;
    r = attn_forward_impl(c, kv, &local, nullptr);
    if (r != QL_OK) return r;
    if (cm->mode == QL_COMM_P2P) {
      QL_CUDA(ql::launch_peer_push(cm->stage, rows, static_cast<int>(row_bytes),
                                   static_cast<int>(hd * eb), po, c->num_sms, c->status,
                                   c->stream),
              "launch the output exchange");
    } else {
      const ncclResult_t nr = nccl_api().all_gather(cm->stage, cm->gather, rows * row_bytes,
                                                    ncclUint8, cm->nccl, c->stream);
      if (nr != ncclSuccess) return nccl_fail(nr, "ncclAllGather of the outputs");
      QL_CUDA(ql::launch_rank_to_head_major(cm->gather, a->out, nranks, rows,
                                            static_cast<int>(row_bytes), c->stream),
              "launch the head-major permute");
      return QL_OK;
    }
  }
  if (a->out != symout)
    QL_CUDA(cudaMemcpyAsync(a->out, symout, static_cast<size_t>(rows) * row_bytes * nranks,
                            cudaMemcpyDeviceToDevice, c->stream),
            "copy the gathered output");
  return QL_OK;
}
