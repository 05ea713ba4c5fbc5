// ql_model.cu -- the Llama model host around the attention path (qllama_model.h):
// device-resident f32 weights, the non-attention layers as CUDA kernels, the
// sampler on the device, and the generate loop.
//
// Reference (all arithmetic follows it operation for operation):
//   Transformer::forward_with_cache       src/transformer/transformer.rs:238-266
//   TransformerBlock::forward_with_cache  src/transformer/layers.rs:615-631
//   Embedding::forward                    src/transformer/layers.rs:76-100
//   Linear::forward (x @ W^T, W transposed once at construction)
//                                         src/transformer/layers.rs:112-171
//   TensorOps::matmul (f32, sequential inner sum, no fused multiply-add)
//                                         src/tensor/ops.rs:63-94
//   TensorOps::rms_norm (f64 square sum in index order) src/tensor/ops.rs:96-136
//   TensorOps::silu                       src/tensor/ops.rs:222-239
//   Mlp::forward                          src/transformer/layers.rs:573-578
//   generate()                            src/main.rs:387-429
//   Sampler::sample_slice and helpers     src/sampler/sampler.rs:119-325
//
// Kernels:
//   embed_kernel        token rows of the embedding (ids read on the device,
//                       so a generated token feeds the next step without a
//                       host round trip)
//   rmsnorm_kernel      one CTA per row; the f64 square sum runs in index order
//                       as the reference's iterator sum does, the rest in parallel
//   gemm_kernel<R, M>   y = x @ W^T with one thread per output column and R rows
//                       per CTA (the weight column is read once for R rows); the
//                       inner sum is sequential with separately rounded products
//                       (bit-identical to the reference's matmul).  Epilogues:
//                       plain, residual add (TransformerBlock's residual), the
//                       fused Q/K/V split (one GEMM for the three projections),
//                       and the fused SwiGLU (gate and up columns together,
//                       silu(gate) * up)
//   sample_kernel       one CTA: repeat penalty, greedy argmax or temperature,
//                       softmax, top-k, top-p and the draw
#include <cuda_runtime.h>
#include <math_constants.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/qllama_model.h"
#include "ql_device.cuh"
#include "ql_internal.h"
#include "ql_kernels.cuh"

// ql_api.cu: the cache side of the fused projection
int ql_kv_append_prepare(ql_ctx* c, ql_kv* kv, const ql_attn_args* a, ql::CacheView* view,
                         const double2** rope, ql::SeqTable* st);
void ql_kv_append_commit(ql_kv* kv, const ql_attn_args* a);

namespace {

#define QLM_CUDA(call, what)                                                                   \
  do {                                                                                         \
    cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess)                                                                     \
      return ql_fail(e_ == cudaErrorMemoryAllocation ? QL_ERR_OOM : QL_ERR_CUDA, "%s: %s",    \
                     what, cudaGetErrorString(e_));                                            \
  } while (0)

// ------------------------------------------------------------------ kernels --

__global__ void __launch_bounds__(256) embed_kernel(const int32_t* ids, int n, const float* emb,
                                                    int vocab, int hidden, float* x,
                                                    uint32_t* status) {
  const int row = blockIdx.x;
  if (row >= n) return;
  const int id = ids[row];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) atomicOr(status, ql::kStatusBadToken);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    x[static_cast<size_t>(row) * hidden + i] = ok ? emb[static_cast<size_t>(id) * hidden + i] : 0.f;
}

// TensorOps::rms_norm: square_sum = sum of f64(x)^2 in index order,
// den = sqrt(square_sum / hidden + f64(eps)), out = f32(f64(x) / den * f64(w)).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* x, const float* w, int hidden,
                                                      float eps, float* out) {
  extern __shared__ float xs[];
  __shared__ double den_s;
  const size_t base = static_cast<size_t>(blockIdx.x) * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) xs[i] = x[base + i];
  __syncthreads();
  if (threadIdx.x == 0) {
    double ss = 0.0;
    for (int i = 0; i < hidden; ++i) {
      const double d = static_cast<double>(xs[i]);
      ss = __dadd_rn(ss, __dmul_rn(d, d));
    }
    den_s = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, static_cast<double>(hidden)),
                                 static_cast<double>(eps)));
  }
  __syncthreads();
  const double den = den_s;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const double v = static_cast<double>(xs[i]);
    const double nv = den == 0.0 ? v : __ddiv_rn(v, den);
    out[base + i] = __double2float_rn(__dmul_rn(nv, static_cast<double>(w[i])));
  }
}

// exp in single precision as the reference's libm expf computes it: the
// correctly rounded value (f64 exp rounded once to f32; the two agree except
// when the exact value lies within the f64 error of a rounding midpoint).
__device__ __forceinline__ float expf_ref(float v) {
  return __double2float_rn(exp(static_cast<double>(v)));
}

// TensorOps::silu (ops.rs:222-239), branch for branch.
__device__ __forceinline__ float silu_ref(float v) {
  if (v == -CUDART_INF_F) return -0.0f;
  if (v >= 0.f) return __fdiv_rn(v, __fadd_rn(1.f, expf_ref(-v)));
  const float e = expf_ref(v);
  return __fdiv_rn(__fmul_rn(v, e), __fadd_rn(1.f, e));
}

enum GemmMode : int { kPlain = 0, kResidual = 1, kQkv = 2, kSwiglu = 3 };

struct GemmArgs {
  const float* x;    // [n, K]
  const float* wt;   // [K, N] (the reference's transposed weight)
  const float* wt2;  // kSwiglu: the up projection [K, N]
  int n, K, N;
  float* y;          // [n, N] (kPlain, kResidual: y += x @ W^T, kSwiglu)
  // kQkv: columns [0, q_cols) to q, then kv_cols to k, then kv_cols to v
  float* q;
  float* k;
  float* v;
  int q_cols, kv_cols;
};

constexpr int kGemmThreads = 128;
constexpr int kGemmKChunk = 512;  // x rows staged in shared memory this many columns at a time

template <int R, int M>
__global__ void __launch_bounds__(kGemmThreads) gemm_kernel(const GemmArgs g) {
  __shared__ float xs[R][kGemmKChunk];
  const int c = blockIdx.x * kGemmThreads + threadIdx.x;
  const int r0 = blockIdx.y * R;
  float acc[R], acc2[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = acc2[r] = 0.f;
  for (int k0 = 0; k0 < g.K; k0 += kGemmKChunk) {
    const int kc = min(kGemmKChunk, g.K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < R * kc; i += kGemmThreads) {
      const int r = i / kc, kk = i % kc;
      xs[r][kk] = r0 + r < g.n ? g.x[static_cast<size_t>(r0 + r) * g.K + k0 + kk] : 0.f;
    }
    __syncthreads();
    if (c < g.N) {
      const float* wcol = g.wt + static_cast<size_t>(k0) * g.N + c;
      const float* wcol2 = M == kSwiglu ? g.wt2 + static_cast<size_t>(k0) * g.N + c : nullptr;
      for (int kk = 0; kk < kc; ++kk) {
        const float w = __ldg(wcol + static_cast<size_t>(kk) * g.N);
        float w2 = 0.f;
        if constexpr (M == kSwiglu) w2 = __ldg(wcol2 + static_cast<size_t>(kk) * g.N);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          acc[r] = __fadd_rn(acc[r], __fmul_rn(xs[r][kk], w));
          if constexpr (M == kSwiglu) acc2[r] = __fadd_rn(acc2[r], __fmul_rn(xs[r][kk], w2));
        }
      }
    }
  }
  if (c >= g.N) return;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = r0 + r;
    if (row >= g.n) break;
    if constexpr (M == kPlain) {
      g.y[static_cast<size_t>(row) * g.N + c] = acc[r];
    } else if constexpr (M == kResidual) {
      float* p = g.y + static_cast<size_t>(row) * g.N + c;
      *p = __fadd_rn(*p, acc[r]);  // residual.add(out): hidden + attended
    } else if constexpr (M == kSwiglu) {
      g.y[static_cast<size_t>(row) * g.N + c] = __fmul_rn(silu_ref(acc[r]), acc2[r]);
    } else {
      if (c < g.q_cols)
        g.q[static_cast<size_t>(row) * g.q_cols + c] = acc[r];
      else if (c < g.q_cols + g.kv_cols)
        g.k[static_cast<size_t>(row) * g.kv_cols + c - g.q_cols] = acc[r];
      else
        g.v[static_cast<size_t>(row) * g.kv_cols + c - g.q_cols - g.kv_cols] = acc[r];
    }
  }
}

template <int M>
cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t s) {
  if (g.n <= 0 || g.N <= 0) return cudaSuccess;
  const unsigned cols = static_cast<unsigned>((g.N + kGemmThreads - 1) / kGemmThreads);
  if (g.n == 1) {
    gemm_kernel<1, M><<<dim3(cols, 1), kGemmThreads, 0, s>>>(g);
  } else {
    gemm_kernel<4, M><<<dim3(cols, (g.n + 3) / 4), kGemmThreads, 0, s>>>(g);
  }
  return cudaGetLastError();
}

// ------------------------------------------------- fused projection + RoPE --
// One thread per adjacent column pair (2c, 2c+1) of the fused output
// [q | k | v], R token rows per CTA: two sequential f32 dot products as in
// gemm_kernel, then the pair is rotated (q and k, f64 as rope_pair) and q is
// stored to q_rot, k and v into the cache rows of their positions.
struct QkvArgs {
  const float* x;   // [rows, K]
  const float* wt;  // [K, N], N = (hq + 2 hkv) * hd
  int rows, K, N;
  int hq, hkv, hd, new_len;
  float* q_rot;     // [rows, hq * hd]
  const double2* rope;
  ql::CacheView cache;
  uint32_t* status;
  ql::SeqTable seqs;
};

template <int R>
__global__ void __launch_bounds__(kGemmThreads) qkv_rope_append_kernel(const QkvArgs g) {
  __shared__ float xs[R][kGemmKChunk];
  const int c = 2 * (blockIdx.x * kGemmThreads + threadIdx.x);
  const int r0 = blockIdx.y * R;
  float a0[R], a1[R];
#pragma unroll
  for (int r = 0; r < R; ++r) a0[r] = a1[r] = 0.f;
  for (int k0 = 0; k0 < g.K; k0 += kGemmKChunk) {
    const int kc = min(kGemmKChunk, g.K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < R * kc; i += kGemmThreads) {
      const int r = i / kc, kk = i % kc;
      xs[r][kk] = r0 + r < g.rows ? g.x[static_cast<size_t>(r0 + r) * g.K + k0 + kk] : 0.f;
    }
    __syncthreads();
    if (c < g.N) {
      const float* wcol = g.wt + static_cast<size_t>(k0) * g.N + c;
      for (int kk = 0; kk < kc; ++kk) {
        const float2 w = __ldg(reinterpret_cast<const float2*>(wcol + static_cast<size_t>(kk) * g.N));
#pragma unroll
        for (int r = 0; r < R; ++r) {
          a0[r] = __fadd_rn(a0[r], __fmul_rn(xs[r][kk], w.x));
          a1[r] = __fadd_rn(a1[r], __fmul_rn(xs[r][kk], w.y));
        }
      }
    }
  }
  if (c >= g.N) return;
  const int qcols = g.hq * g.hd, kvcols = g.hkv * g.hd;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = r0 + r;
    if (row >= g.rows) break;
    const int b = row / g.new_len, t = row % g.new_len;
    const int pos = g.seqs.start[b] + t;
    float y0 = a0[r], y1 = a1[r];
    if (c < qcols + kvcols) {  // q and k rotate by their position's angles
      const int d = (c < qcols ? c : c - qcols) % g.hd;
      ql::rope_pair(y0, y1, g.rope[static_cast<size_t>(pos) * (g.hd / 2) + d / 2], y0, y1);
    }
    if (c < qcols) {
      g.q_rot[static_cast<size_t>(row) * qcols + c] = y0;
      g.q_rot[static_cast<size_t>(row) * qcols + c + 1] = y1;
      continue;
    }
    const bool is_k = c < qcols + kvcols;
    const int ck = is_k ? c - qcols : c - qcols - kvcols;
    const int h = ck / g.hd, d = ck % g.hd;
    const ql::CacheView& cv = g.cache;
    const int page = cv.block_table[static_cast<size_t>(g.seqs.seq[b]) * cv.pages_per_seq +
                                    pos / cv.page];
    if (page < 0 || page >= cv.num_pages) {
      atomicOr(g.status, ql::kStatusBadPage);
      continue;
    }
    const size_t e =
        ((static_cast<size_t>(page) * cv.hkv + h) * cv.page + pos % cv.page) * cv.hd + d;
    void* dst = is_k ? cv.k : cv.v;
    ql::store_elem(dst, e, cv.dtype, y0);
    ql::store_elem(dst, e + 1, cv.dtype, y1);
  }
}

// ------------------------------------------------------------------ sampler --
// One CTA of kSampleThreads.  Keys: an f32 logit in total order (the
// reference's total_cmp) and an f64 probability (non-negative, so its bits
// order like its values).
constexpr int kSampleThreads = 1024;
constexpr int kMaxCand = 2048;  // candidates sorted in shared memory

struct SampleArgs {
  const float* logits;
  int vocab;
  const int32_t* context;
  int n_context;
  float temperature;
  int top_k;
  float top_p;
  float penalty;
  double r;
  float* work;        // [vocab]
  double* prob;       // [vocab]
  uint64_t* skey;     // [pow2(vocab)] large-set sort keys
  int32_t* sid;       // [pow2(vocab)] their ids
  int sort_n;         // pow2 >= vocab
  int32_t* token_out;
  uint32_t* status;
};

__device__ __forceinline__ uint32_t total_order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ uint64_t dbits(double d) {
  return static_cast<uint64_t>(__double_as_longlong(d));
}

// Block-wide reductions (every thread gets the result).
__device__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  if (w == 0) {
    t = l < (blockDim.x >> 5) ? red[l] : 0.0;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__device__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    unsigned long long t = l < (blockDim.x >> 5) ? red[l] : 0ull;
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long u = __shfl_xor_sync(0xffffffffu, t, o);
      t = u > t ? u : t;
    }
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__device__ int block_or(int v, int* red) {
  v = __any_sync(0xffffffffu, v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int t = 0;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t |= red[i];
  __syncthreads();
  return t;
}

// "a before b" in the reference's sorted_indices: probability descending,
// then id ascending.
__device__ __forceinline__ bool before(uint64_t ka, int ia, uint64_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Bitonic sort of n (a power of two) (key, id) pairs in place by `before`
// (by_id: id ascending instead).
template <typename K>
__device__ void bitonic(K* key, int* id, int n, bool by_id) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool asc = (lo & size) == 0;
        const bool hi_first = by_id ? id[hi] < id[lo] : before(key[hi], id[hi], key[lo], id[lo]);
        if (hi_first == asc) {
          const K tk = key[lo];
          key[lo] = key[hi];
          key[hi] = tk;
          const int ti = id[lo];
          id[lo] = id[hi];
          id[hi] = ti;
        }
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleArgs a) {
  extern __shared__ uint32_t seen[];  // vocab bits
  __shared__ double red_d[32];
  __shared__ unsigned long long red_u[32];
  __shared__ int red_i[32];
  __shared__ uint64_t ckey[kMaxCand];
  __shared__ int cid[kMaxCand];
  __shared__ double cp[kMaxCand];
  __shared__ int n_cand, hist[256], sel_s, need_s;
  int* scan = cid;    // the top-k tie ranks use cid before the candidates fill it
  double* ctot = cp;  // the large-set draw does not use cp
  const int V = a.vocab, tid = threadIdx.x;
  // finite logits (sample_slice's first check)
  int bad = 0;
  for (int i = tid; i < V; i += blockDim.x) {
    const float x = a.logits[i];
    a.work[i] = x;
    bad |= !isfinite(x);
  }
  __syncthreads();
  if (block_or(bad, red_i)) {
    if (tid == 0) {
      *a.token_out = -1;
      atomicOr(a.status, ql::kStatusBadLogits);
    }
    return;
  }
  // repeat penalty: each context id in range once (apply_repeat_penalty)
  if (a.penalty != 1.0f) {
    for (int i = tid; i < (V + 31) / 32; i += blockDim.x) seen[i] = 0u;
    __syncthreads();
    for (int i = tid; i < a.n_context; i += blockDim.x) {
      const int t = a.context[i];
      if (t < 0 || t >= V) continue;
      const uint32_t bit = 1u << (t & 31);
      if (atomicOr(&seen[t >> 5], bit) & bit) continue;
      const float x = a.work[t];
      a.work[t] = x <= 0.f ? __fmul_rn(x, a.penalty) : __fdiv_rn(x, a.penalty);
    }
    __syncthreads();
    bad = 0;
    for (int i = tid; i < V; i += blockDim.x) bad |= !isfinite(a.work[i]);
    if (block_or(bad, red_i)) {
      if (tid == 0) {
        *a.token_out = -1;
        atomicOr(a.status, ql::kStatusBadLogits);
      }
      return;
    }
  }
  // greedy: the largest logit in total order, ties to the smaller id (argmax)
  if (a.temperature <= 0.f) {
    unsigned long long best = 0;
    for (int i = tid; i < V; i += blockDim.x) {
      const unsigned long long k =
          (static_cast<unsigned long long>(total_order_key(a.work[i])) << 32) |
          (0xffffffffu - static_cast<uint32_t>(i));
      best = k > best ? k : best;
    }
    best = block_max_u64(best, red_u);
    if (tid == 0) *a.token_out = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(best));
    return;
  }
  // temperature, then softmax with an f32 maximum and f64 exponentials
  float mx = -CUDART_INF_F;
  bad = 0;
  for (int i = tid; i < V; i += blockDim.x) {
    const float x = __fdiv_rn(a.work[i], a.temperature);
    a.work[i] = x;
    bad |= !isfinite(x);
    mx = fmaxf(mx, x);
  }
  if (block_or(bad, red_i)) {
    if (tid == 0) {
      *a.token_out = -1;
      atomicOr(a.status, ql::kStatusBadLogits);
    }
    return;
  }
  unsigned long long mk = block_max_u64(total_order_key(mx), red_u);
  {
    const uint32_t b = static_cast<uint32_t>(mk);
    mx = __uint_as_float((b & 0x80000000u) ? (b & 0x7fffffffu) : ~b);
  }
  double part = 0.0;
  for (int i = tid; i < V; i += blockDim.x) {
    const double e = exp(static_cast<double>(a.work[i]) - static_cast<double>(mx));
    a.prob[i] = e;
    part += e;
  }
  const double total = block_sum(part, red_d);
  for (int i = tid; i < V; i += blockDim.x) a.prob[i] = a.prob[i] / total;
  __syncthreads();

  // top-k (apply_top_k): the k most probable, ties to the smaller id, found by
  // a radix select on the probability bits.
  const bool limit_k = a.top_k > 0 && a.top_k < V;
  int cand_all = !limit_k;  // every id stays a candidate
  if (limit_k) {
    uint64_t prefix = 0, mask = 0;
    int need = a.top_k;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0;
      __syncthreads();
      for (int i = tid; i < V; i += blockDim.x) {
        const uint64_t key = dbits(a.prob[i]);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
      }
      __syncthreads();
      if (tid == 0) {
        int c = 0, sel = 0;
        for (int b = 255; b >= 0; --b) {
          if (c + hist[b] >= need) {
            sel = b;
            break;
          }
          c += hist[b];
        }
        sel_s = sel;
        need_s = need - c;
      }
      __syncthreads();
      prefix |= static_cast<uint64_t>(sel_s) << shift;
      mask |= static_cast<uint64_t>(0xff) << shift;
      need = need_s;
      __syncthreads();
    }
    // keys above the threshold, then `need` ties in id order
    const uint64_t T = prefix;
    const int chunk = (V + blockDim.x - 1) / blockDim.x;
    const int c0 = tid * chunk, c1 = min(V, c0 + chunk);
    int eq = 0;
    for (int i = c0; i < c1; ++i) eq += dbits(a.prob[i]) == T;
    // exclusive scan of eq over threads (thread order = id order)
    scan[tid] = eq;
    __syncthreads();
    if (tid == 0) {
      int s = 0;
      for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
        const int x = scan[t];
        scan[t] = s;
        s += x;
      }
    }
    __syncthreads();
    int rank = scan[tid];
    if (tid == 0) n_cand = 0;
    __syncthreads();
    for (int i = c0; i < c1; ++i) {
      const uint64_t key = dbits(a.prob[i]);
      bool keep = key > T;
      if (key == T) keep = rank++ < need;
      if (!keep) a.prob[i] = 0.0;
      else if (a.top_k <= kMaxCand) {
        const int slot = atomicAdd(&n_cand, 1);
        ckey[slot] = key;
        cid[slot] = i;
      }
    }
    __syncthreads();
    cand_all = a.top_k > kMaxCand;
    if (cand_all) {  // renormalise the kept set in place (apply_top_k)
      double kp = 0.0;
      for (int i = tid; i < V; i += blockDim.x) kp += a.prob[i];
      const double t = block_sum(kp, red_d);
      for (int i = tid; i < V; i += blockDim.x) a.prob[i] = a.prob[i] / t;
      __syncthreads();
    }
  } else if (V <= kMaxCand) {
    for (int i = tid; i < V; i += blockDim.x) {
      ckey[i] = dbits(a.prob[i]);
      cid[i] = i;
    }
    if (tid == 0) n_cand = V;
    __syncthreads();
    cand_all = 0;
  }

  if (!cand_all) {
    // ---- small candidate set: exact reference order in shared memory
    const int n = n_cand;
    int np = 1;
    while (np < n) np <<= 1;
    for (int i = n + tid; i < np; i += blockDim.x) {
      ckey[i] = 0;
      cid[i] = 0x7fffffff;
    }
    bitonic<uint64_t>(ckey, cid, np, false);  // probability descending, id ascending
    if (tid == 0) {
      for (int i = 0; i < n; ++i) cp[i] = __longlong_as_double(static_cast<long long>(ckey[i]));
      if (limit_k) {  // renormalise the kept set (sum in sorted order)
        double t = 0.0;
        for (int i = 0; i < n; ++i) t += cp[i];
        for (int i = 0; i < n; ++i) cp[i] = cp[i] / t;
      }
      int keep = n;
      if (a.top_p < 1.0f) {  // apply_top_p: keep through the candidate crossing p
        const double th = static_cast<double>(a.top_p);
        double cum = 0.0;
        for (int i = 0; i < n; ++i) {
          cum += cp[i];
          if (cum >= th) {
            keep = i + 1;
            break;
          }
        }
        double t = 0.0;
        for (int i = 0; i < keep; ++i) t += cp[i];
        for (int i = 0; i < n; ++i) cp[i] = i < keep ? cp[i] / t : 0.0;
      }
      n_cand = keep;
      for (int i = 0; i < n; ++i) ckey[i] = static_cast<uint64_t>(__double_as_longlong(cp[i]));
      for (int i = keep; i < n; ++i) cid[i] = 0x7fffffff;  // dropped: sort past the kept ids
    }
    __syncthreads();
    bitonic<uint64_t>(ckey, cid, np, true);  // id ascending: the draw walks index order
    if (tid == 0) {
      const int keep = n_cand;
      double t = 0.0;
      for (int i = 0; i < keep; ++i) t += __longlong_as_double(static_cast<long long>(ckey[i]));
      const double th = a.r * t;
      double cum = 0.0;
      int tok = -1, last = -1;
      for (int i = 0; i < keep; ++i) {
        const double p = __longlong_as_double(static_cast<long long>(ckey[i]));
        if (p <= 0.0) continue;
        last = cid[i];
        cum += p;
        if (cum >= th) {
          tok = cid[i];
          break;
        }
      }
      *a.token_out = tok >= 0 ? tok : last;
      if (tok < 0 && last < 0) atomicOr(a.status, ql::kStatusBadLogits);
    }
    return;
  }

  // ---- large candidate set (no top-k, or k above kMaxCand): probabilities in
  // a[0, V); top-p over a global-memory sort, then the draw in index order.
  if (a.top_p < 1.0f) {
    for (int i = tid; i < a.sort_n; i += blockDim.x) {
      a.skey[i] = i < V ? dbits(a.prob[i]) : 0;
      a.sid[i] = i < V ? i : 0x7fffffff;
    }
    __syncthreads();
    bitonic<uint64_t>(a.skey, a.sid, a.sort_n, false);
    if (tid == 0) {
      const double th = static_cast<double>(a.top_p);
      double cum = 0.0;
      int keep = V;
      for (int i = 0; i < V; ++i) {
        cum += __longlong_as_double(static_cast<long long>(a.skey[i]));
        if (cum >= th) {
          keep = i + 1;
          break;
        }
      }
      double t = 0.0;
      for (int i = 0; i < keep; ++i) t += __longlong_as_double(static_cast<long long>(a.skey[i]));
      red_d[0] = t;
      need_s = keep;
    }
    __syncthreads();
    const double t = red_d[0];
    const int keep = need_s;
    for (int i = tid; i < V; i += blockDim.x) {
      if (i < keep) {
        const int id = a.sid[i];
        a.prob[id] = a.prob[id] / t;
      } else {
        a.prob[a.sid[i]] = 0.0;
      }
    }
    __syncthreads();
  }
  // draw: each thread sums its contiguous chunk; the chunk totals are added
  // in order, and the chunk where the running sum reaches the threshold is
  // walked element by element (sample_from_distribution, index order).
  {
    const int chunk = (V + blockDim.x - 1) / blockDim.x;
    const int c0 = tid * chunk, c1 = min(V, c0 + chunk);
    double s = 0.0;
    for (int i = c0; i < c1; ++i) s += a.prob[i];
    ctot[tid] = s;
    __syncthreads();
    if (tid == 0) {
      const int nch = static_cast<int>(blockDim.x);
      double t = 0.0;
      for (int c = 0; c < nch; ++c) t += ctot[c];
      const double th = a.r * t;
      double cum = 0.0;
      int tok = -1;
      for (int c = 0; c < nch && tok < 0; ++c) {
        if (cum + ctot[c] < th && c + 1 < nch) {
          cum += ctot[c];
          continue;
        }
        for (int i = c * chunk; i < min(V, (c + 1) * chunk); ++i) {
          const double p = a.prob[i];
          if (p <= 0.0) continue;
          cum += p;
          if (cum >= th) {
            tok = i;
            break;
          }
        }
      }
      if (tok < 0)  // rounding kept the sum below the threshold: the last positive
        for (int i = V - 1; i >= 0; --i)
          if (a.prob[i] > 0.0) {
            tok = i;
            break;
          }
      *a.token_out = tok;
      if (tok < 0) atomicOr(a.status, ql::kStatusBadLogits);
    }
  }
}

size_t sample_smem(int vocab) { return static_cast<size_t>((vocab + 31) / 32) * 4; }

int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

size_t sample_scratch_bytes(int vocab) {
  const size_t np = static_cast<size_t>(pow2_at_least(vocab));
  return 4 * static_cast<size_t>(vocab) + 8 * static_cast<size_t>(vocab) + 8 * np + 4 * np + 1024;
}

int check_sampler_config(const ql_sampler_config* c, int vocab) {
  // SamplerConfig::validate (sampler.rs:40-60)
  if (!std::isfinite(c->temperature))
    return ql_fail(QL_ERR_INVALID, "Sampler temperature must be finite, got %g",
                   static_cast<double>(c->temperature));
  if (!std::isfinite(c->top_p))
    return ql_fail(QL_ERR_INVALID, "Sampler top_p must be finite, got %g",
                   static_cast<double>(c->top_p));
  if (!std::isfinite(c->repeat_penalty) || c->repeat_penalty <= 0.f)
    return ql_fail(QL_ERR_INVALID, "Sampler repeat_penalty must be finite and positive, got %g",
                   static_cast<double>(c->repeat_penalty));
  if (c->top_k < 0) return ql_fail(QL_ERR_INVALID, "Sampler top_k must not be negative");
  if (vocab <= 0) return ql_fail(QL_ERR_INVALID, "Sampling requires a non-empty logits slice");
  if (vocab > (1 << 22))
    return ql_fail(QL_ERR_UNSUPPORTED, "vocabulary of %d exceeds the device sampler's limit", vocab);
  return QL_OK;
}

cudaError_t launch_sample(const ql_sampler_config& c, const float* logits, int vocab,
                          const int32_t* context, int n_context, double r, char* scratch,
                          int32_t* token_out, uint32_t* status, cudaStream_t s) {
  SampleArgs a{};
  const int np = pow2_at_least(vocab);
  a.logits = logits;
  a.vocab = vocab;
  a.context = context;
  a.n_context = n_context;
  a.temperature = c.temperature;
  a.top_k = c.top_k;
  a.top_p = c.top_p;
  a.penalty = c.repeat_penalty;
  a.r = r;
  char* p = scratch;
  a.prob = reinterpret_cast<double*>(p);
  p += 8 * static_cast<size_t>(vocab);
  a.skey = reinterpret_cast<uint64_t*>(p);
  p += 8 * static_cast<size_t>(np);
  a.work = reinterpret_cast<float*>(p);
  p += 4 * static_cast<size_t>(vocab);
  a.sid = reinterpret_cast<int32_t*>(p);
  a.sort_n = np;
  a.token_out = token_out;
  a.status = status;
  const size_t smem = sample_smem(vocab);
  cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  sample_kernel<<<1, kSampleThreads, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

// -------------------------------------------------------------------- model --
struct ql_llama {
  ql_ctx* ctx = nullptr;
  ql_llama_config cfg{};
  int hd = 0, kvd = 0, qkv_cols = 0;
  float* embd = nullptr;      // [V, E]
  float* lm_t = nullptr;      // [E, V]: output.weight transposed (or the tied embedding)
  bool have_lm = false;
  float* out_norm = nullptr;  // [E]
  struct Layer {
    float* attn_norm = nullptr;  // [E]
    float* ffn_norm = nullptr;   // [E]
    float* wqkv_t = nullptr;     // [E, E + 2 kvd]: Wq^T | Wk^T | Wv^T
    float* wo_t = nullptr;       // [E, E]
    float* wg_t = nullptr;       // [E, F]
    float* wu_t = nullptr;       // [E, F]
    float* wd_t = nullptr;       // [F, E]
  };
  std::vector<Layer> layers;
  // workspace for `rows` tokens
  // projections fused with RoPE and the append (ql_qkv_rope_append); off:
  // the Q/K/V GEMM, then ql_attn_forward appends (same results, bit for bit)
  bool fused_qkv = true;
  int rows = 0;
  float *x = nullptr, *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
        *g = nullptr, *logits = nullptr;
  int32_t* ids = nullptr;   // [max_pos + 1] token ids of the call / the generated context
  char* sample_scratch = nullptr;
  std::vector<void*> allocations;
};

namespace {

int alloc_dev(ql_llama* m, void** p, size_t bytes) {
  QLM_CUDA(cudaMalloc(p, std::max<size_t>(bytes, 256)), "allocate model memory");
  m->allocations.push_back(*p);
  QLM_CUDA(cudaMemsetAsync(*p, 0, std::max<size_t>(bytes, 256), m->ctx->stream),
           "clear model memory");
  return QL_OK;
}

void free_work(ql_llama* m) {
  for (float* p : {m->x, m->h, m->q, m->k, m->v, m->att, m->g, m->logits})
    if (p) cudaFree(p);
  m->x = m->h = m->q = m->k = m->v = m->att = m->g = m->logits = nullptr;
  m->rows = 0;
}

int ensure_rows(ql_llama* m, int rows) {
  if (rows <= m->rows) return QL_OK;
  QLM_CUDA(cudaStreamSynchronize(m->ctx->stream), "synchronize before growing the workspace");
  free_work(m);
  const size_t E = m->cfg.hidden_size, F = m->cfg.intermediate_size, V = m->cfg.vocab_size;
  const size_t R = static_cast<size_t>(rows);
  struct {
    float** p;
    size_t n;
  } bufs[] = {{&m->x, R * E}, {&m->h, R * E}, {&m->q, R * E}, {&m->k, R * m->kvd},
              {&m->v, R * m->kvd}, {&m->att, R * E}, {&m->g, R * F}, {&m->logits, R * V}};
  for (auto& b : bufs) {
    cudaError_t e = cudaMalloc(b.p, std::max<size_t>(b.n * sizeof(float), 256));
    if (e != cudaSuccess) {
      free_work(m);
      return ql_fail(e == cudaErrorMemoryAllocation ? QL_ERR_OOM : QL_ERR_CUDA,
                     "allocate the model workspace: %s", cudaGetErrorString(e));
    }
  }
  m->rows = rows;
  return QL_OK;
}

// Uploads host [rows, cols] as the transposed [cols, rows] block at column
// `col0` of a device matrix with `ld` columns.
int upload_transposed(ql_llama* m, float* dst, int ld, int col0, const float* src, int rows,
                      int cols) {
  std::vector<float> t(static_cast<size_t>(rows) * cols);
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c)
      t[static_cast<size_t>(c) * rows + r] = src[static_cast<size_t>(r) * cols + c];
  QLM_CUDA(cudaMemcpy2DAsync(dst + col0, static_cast<size_t>(ld) * sizeof(float), t.data(),
                             static_cast<size_t>(rows) * sizeof(float),
                             static_cast<size_t>(rows) * sizeof(float), cols,
                             cudaMemcpyHostToDevice, m->ctx->stream),
           "upload a weight");
  QLM_CUDA(cudaStreamSynchronize(m->ctx->stream), "wait for a weight upload");
  return QL_OK;
}

int upload_plain(ql_llama* m, float* dst, const float* src, size_t n) {
  QLM_CUDA(cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyHostToDevice, m->ctx->stream),
           "upload a weight");
  QLM_CUDA(cudaStreamSynchronize(m->ctx->stream), "wait for a weight upload");
  return QL_OK;
}

// Transformer::forward_with_cache with the token ids already on the device
// (ids[0..n)); logits of the last `logit_rows` rows go to m->logits.
int forward_device(ql_llama* m, ql_kv* kv, int32_t seq, const int32_t* ids, int n,
                   int64_t start_pos, int logit_rows) {
  ql_ctx* c = m->ctx;
  cudaStream_t s = c->stream;
  const ql_llama_config& cf = m->cfg;
  const int E = cf.hidden_size, F = cf.intermediate_size, V = cf.vocab_size;
  embed_kernel<<<n, 256, 0, s>>>(ids, n, m->embd, V, E, m->x, c->status);
  QLM_CUDA(cudaGetLastError(), "launch embedding");
  const size_t norm_smem = static_cast<size_t>(E) * sizeof(float);
  for (int l = 0; l < cf.num_layers; ++l) {
    const ql_llama::Layer& L = m->layers[l];
    rmsnorm_kernel<<<n, 256, norm_smem, s>>>(m->x, L.attn_norm, E, cf.rms_norm_eps, m->h);
    QLM_CUDA(cudaGetLastError(), "launch rms_norm");
    ql_attn_args a{};
    a.layer_idx = l;
    a.batch = 1;
    a.new_len = n;
    a.seq_ids = &seq;
    a.start_pos = &start_pos;
    a.num_heads = cf.num_heads;
    a.num_kv_heads = cf.num_kv_heads;
    a.head_dim = m->hd;
    a.rope_theta = cf.rope_theta;
    a.in_dtype = QL_F32;
    a.out_dtype = QL_F32;
    a.mem = QL_MEM_DEVICE;
    a.q = m->q;
    a.k = m->k;
    a.v = m->v;
    a.out = m->att;
    // Projections, RoPE and the append in one launch, then attention over the
    // appended rows; a Q8_0 cache takes the projection GEMM and the operator,
    // which quantises whole 32-value blocks as it appends.
    int r = m->fused_qkv ? ql_qkv_rope_append(c, kv, &a, m->h, E, L.wqkv_t, m->q) : QL_ERR_UNSUPPORTED;
    if (r == QL_OK) {
      r = ql_attn_forward_appended(c, kv, &a);
    } else if (r == QL_ERR_UNSUPPORTED) {
      GemmArgs g{};
      g.x = m->h;
      g.wt = L.wqkv_t;
      g.n = n;
      g.K = E;
      g.N = m->qkv_cols;
      g.q = m->q;
      g.k = m->k;
      g.v = m->v;
      g.q_cols = E;
      g.kv_cols = m->kvd;
      QLM_CUDA(launch_gemm<kQkv>(g, s), "launch the Q/K/V projection");
      r = ql_attn_forward(c, kv, &a);
    }
    if (r != QL_OK) {
      std::string msg = ql_last_error();
      return ql_fail(r, "Layer %d failed: %s", l, msg.c_str());
    }
    GemmArgs g{};
    g.x = m->att;
    g.wt = L.wo_t;
    g.n = n;
    g.K = E;
    g.N = E;
    g.y = m->x;
    QLM_CUDA(launch_gemm<kResidual>(g, s), "launch the output projection");
    rmsnorm_kernel<<<n, 256, norm_smem, s>>>(m->x, L.ffn_norm, E, cf.rms_norm_eps, m->h);
    QLM_CUDA(cudaGetLastError(), "launch rms_norm");
    g = GemmArgs{};
    g.x = m->h;
    g.wt = L.wg_t;
    g.wt2 = L.wu_t;
    g.n = n;
    g.K = E;
    g.N = F;
    g.y = m->g;
    QLM_CUDA(launch_gemm<kSwiglu>(g, s), "launch the SwiGLU projections");
    g = GemmArgs{};
    g.x = m->g;
    g.wt = L.wd_t;
    g.n = n;
    g.K = F;
    g.N = E;
    g.y = m->x;
    QLM_CUDA(launch_gemm<kResidual>(g, s), "launch the down projection");
  }
  if (logit_rows <= 0) return QL_OK;
  const int first = n - logit_rows;
  rmsnorm_kernel<<<logit_rows, 256, norm_smem, s>>>(m->x + static_cast<size_t>(first) * E,
                                                   m->out_norm, E, cf.rms_norm_eps, m->h);
  QLM_CUDA(cudaGetLastError(), "launch rms_norm");
  GemmArgs g{};
  g.x = m->h;
  g.wt = m->lm_t;
  g.n = logit_rows;
  g.K = E;
  g.N = V;
  g.y = m->logits;
  QLM_CUDA(launch_gemm<kPlain>(g, s), "launch lm_head");
  return QL_OK;
}

int check_positions(const ql_llama* m, int n, int64_t start_pos) {
  // transformer.rs:244-257
  const int64_t last = start_pos + (n > 0 ? n - 1 : 0);
  if (start_pos < 0) return ql_fail(QL_ERR_INVALID, "start_pos %lld is negative", (long long)start_pos);
  if (last >= m->cfg.max_position_embeddings)
    return ql_fail(QL_ERR_INVALID, "Last position %lld exceeds max_position_embeddings %d",
                   (long long)last, m->cfg.max_position_embeddings);
  return QL_OK;
}

}  // namespace

extern "C" {

int ql_llama_create(ql_ctx* c, const ql_llama_config* cfg, ql_llama** out) {
  if (!c || !cfg || !out) return ql_fail(QL_ERR_INVALID, "ql_llama_create: NULL argument");
  *out = nullptr;
  const ql_llama_config& f = *cfg;
  if (f.vocab_size <= 0 || f.hidden_size <= 0 || f.intermediate_size <= 0 || f.num_heads <= 0 ||
      f.num_kv_heads <= 0 || f.num_layers < 0 || f.max_position_embeddings <= 0)
    return ql_fail(QL_ERR_INVALID, "model dimensions must be positive");
  if (f.hidden_size % f.num_heads != 0)
    return ql_fail(QL_ERR_INVALID, "embedding_length %d is not divisible by attention.head_count %d",
                   f.hidden_size, f.num_heads);
  if (f.num_heads % f.num_kv_heads != 0)  // Attention::new (layers.rs:254-261)
    return ql_fail(QL_ERR_INVALID, "num_heads %d must be divisible by num_kv_heads %d",
                   f.num_heads, f.num_kv_heads);
  if ((f.hidden_size / f.num_heads) % 2 != 0)
    return ql_fail(QL_ERR_INVALID,
                   "RoPE requires shape [seq_len, ..., head_dim] with a positive even head_dim");
  if (!std::isfinite(f.rms_norm_eps) || f.rms_norm_eps < 0.f)
    return ql_fail(QL_ERR_INVALID, "RMSNorm eps must be finite and nonnegative");
  if (!std::isfinite(f.rope_theta) || f.rope_theta <= 0.f)
    return ql_fail(QL_ERR_INVALID, "RoPE theta must be finite and positive");
  QLM_CUDA(cudaSetDevice(c->device), "set device");
  ql_llama* m = new ql_llama;
  m->ctx = c;
  m->cfg = f;
  m->hd = f.hidden_size / f.num_heads;
  m->kvd = f.num_kv_heads * m->hd;
  m->qkv_cols = f.hidden_size + 2 * m->kvd;
  const size_t E = f.hidden_size, F = f.intermediate_size, V = f.vocab_size;
  auto bail = [&](int code) {
    ql_llama_destroy(m);
    return code;
  };
  int r = alloc_dev(m, reinterpret_cast<void**>(&m->embd), V * E * 4);
  if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&m->lm_t), E * V * 4);
  if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&m->out_norm), E * 4);
  if (r == QL_OK)
    r = alloc_dev(m, reinterpret_cast<void**>(&m->ids),
                  (static_cast<size_t>(f.max_position_embeddings) + 1) * 4);
  if (r == QL_OK)
    r = alloc_dev(m, reinterpret_cast<void**>(&m->sample_scratch), sample_scratch_bytes(f.vocab_size));
  m->layers.resize(f.num_layers);
  for (int l = 0; l < f.num_layers && r == QL_OK; ++l) {
    ql_llama::Layer& L = m->layers[l];
    r = alloc_dev(m, reinterpret_cast<void**>(&L.attn_norm), E * 4);
    if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&L.ffn_norm), E * 4);
    if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&L.wqkv_t), E * m->qkv_cols * 4);
    if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&L.wo_t), E * E * 4);
    if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&L.wg_t), E * F * 4);
    if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&L.wu_t), E * F * 4);
    if (r == QL_OK) r = alloc_dev(m, reinterpret_cast<void**>(&L.wd_t), F * E * 4);
  }
  if (r == QL_OK) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) r = ql_fail(QL_ERR_CUDA, "clear model memory: %s", cudaGetErrorString(e));
  }
  if (r != QL_OK) return bail(r);
  *out = m;
  return QL_OK;
}

int ql_llama_destroy(ql_llama* m) {
  if (!m) return QL_OK;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  free_work(m);
  for (void* p : m->allocations) cudaFree(p);
  delete m;
  return QL_OK;
}

int ql_llama_get_config(const ql_llama* m, ql_llama_config* out) {
  if (!m || !out) return ql_fail(QL_ERR_INVALID, "ql_llama_get_config: NULL argument");
  *out = m->cfg;
  return QL_OK;
}

int ql_llama_set_tensor(ql_llama* m, const char* name, const float* data, int64_t n) {
  if (!m || !name || !data) return ql_fail(QL_ERR_INVALID, "ql_llama_set_tensor: NULL argument");
  QLM_CUDA(cudaSetDevice(m->ctx->device), "set device");
  const ql_llama_config& f = m->cfg;
  const int E = f.hidden_size, F = f.intermediate_size, V = f.vocab_size, kvd = m->kvd;
  auto expect = [&](int64_t want) {
    if (n != want)
      return ql_fail(QL_ERR_INVALID, "tensor %s has %lld elements, expected %lld", name,
                     (long long)n, (long long)want);
    return QL_OK;
  };
  const std::string s = name;
  int r;
  if (s == "token_embd.weight") {
    if ((r = expect(static_cast<int64_t>(V) * E)) != QL_OK) return r;
    if ((r = upload_plain(m, m->embd, data, static_cast<size_t>(V) * E)) != QL_OK) return r;
    if (!m->have_lm) return upload_transposed(m, m->lm_t, V, 0, data, V, E);  // tied lm_head
    return QL_OK;
  }
  if (s == "output.weight") {
    if ((r = expect(static_cast<int64_t>(V) * E)) != QL_OK) return r;
    m->have_lm = true;
    return upload_transposed(m, m->lm_t, V, 0, data, V, E);
  }
  if (s == "output_norm.weight") {
    if ((r = expect(E)) != QL_OK) return r;
    return upload_plain(m, m->out_norm, data, E);
  }
  int layer = -1, used = 0;
  char suffix[64] = {0};
  if (std::sscanf(name, "blk.%d.%63s%n", &layer, suffix, &used) != 2 || layer < 0 ||
      layer >= f.num_layers || name[used] != '\0')
    return ql_fail(QL_ERR_INVALID, "unknown tensor name %s", name);
  ql_llama::Layer& L = m->layers[layer];
  const std::string t = suffix;
  if (t == "attn_norm.weight") {
    if ((r = expect(E)) != QL_OK) return r;
    return upload_plain(m, L.attn_norm, data, E);
  }
  if (t == "ffn_norm.weight") {
    if ((r = expect(E)) != QL_OK) return r;
    return upload_plain(m, L.ffn_norm, data, E);
  }
  // projections: host [out, in] -> device [in, out] (Linear::new transposes once)
  if (t == "attn_q.weight") {
    if ((r = expect(static_cast<int64_t>(E) * E)) != QL_OK) return r;
    return upload_transposed(m, L.wqkv_t, m->qkv_cols, 0, data, E, E);
  }
  if (t == "attn_k.weight") {
    if ((r = expect(static_cast<int64_t>(kvd) * E)) != QL_OK) return r;
    return upload_transposed(m, L.wqkv_t, m->qkv_cols, E, data, kvd, E);
  }
  if (t == "attn_v.weight") {
    if ((r = expect(static_cast<int64_t>(kvd) * E)) != QL_OK) return r;
    return upload_transposed(m, L.wqkv_t, m->qkv_cols, E + kvd, data, kvd, E);
  }
  if (t == "attn_output.weight") {
    if ((r = expect(static_cast<int64_t>(E) * E)) != QL_OK) return r;
    return upload_transposed(m, L.wo_t, E, 0, data, E, E);
  }
  if (t == "ffn_gate.weight") {
    if ((r = expect(static_cast<int64_t>(F) * E)) != QL_OK) return r;
    return upload_transposed(m, L.wg_t, F, 0, data, F, E);
  }
  if (t == "ffn_up.weight") {
    if ((r = expect(static_cast<int64_t>(F) * E)) != QL_OK) return r;
    return upload_transposed(m, L.wu_t, F, 0, data, F, E);
  }
  if (t == "ffn_down.weight") {
    if ((r = expect(static_cast<int64_t>(E) * F)) != QL_OK) return r;
    return upload_transposed(m, L.wd_t, E, 0, data, E, F);
  }
  return ql_fail(QL_ERR_INVALID, "unknown tensor name %s", name);
}

int ql_llama_forward(ql_llama* m, ql_kv* kv, int32_t seq, const int32_t* ids, int32_t n,
                     int64_t start_pos, float* logits, int32_t mem) {
  if (!m || !kv || (n > 0 && !ids)) return ql_fail(QL_ERR_INVALID, "ql_llama_forward: NULL argument");
  if (n < 0) return ql_fail(QL_ERR_INVALID, "token count %d is negative", n);
  if (mem != QL_MEM_DEVICE && mem != QL_MEM_HOST)
    return ql_fail(QL_ERR_INVALID, "unknown memory kind %d", mem);
  int r = check_positions(m, n, start_pos);
  if (r != QL_OK) return r;
  for (int i = 0; i < n; ++i) {  // Embedding::forward (layers.rs:80-92)
    if (ids[i] < 0)
      return ql_fail(QL_ERR_INVALID, "Token id %d at position %d is negative", ids[i], i);
    if (ids[i] >= m->cfg.vocab_size)
      return ql_fail(QL_ERR_INVALID, "Token id %d at position %d exceeds vocabulary size %d",
                     ids[i], i, m->cfg.vocab_size);
  }
  if (n == 0) return QL_OK;
  QLM_CUDA(cudaSetDevice(m->ctx->device), "set device");
  if ((r = ensure_rows(m, n)) != QL_OK) return r;
  cudaStream_t s = m->ctx->stream;
  QLM_CUDA(cudaMemcpyAsync(m->ids, ids, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, s),
           "copy token ids");
  if ((r = forward_device(m, kv, seq, m->ids, n, start_pos, logits ? n : 0)) != QL_OK) return r;
  if (logits) {
    const size_t bytes = static_cast<size_t>(n) * m->cfg.vocab_size * sizeof(float);
    QLM_CUDA(cudaMemcpyAsync(logits, m->logits, bytes,
                             mem == QL_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice,
                             s),
             "copy logits");
  }
  // the ids buffer is reused by the next call: the host copy above must land first
  QLM_CUDA(cudaStreamSynchronize(s), "synchronize forward");
  return ql_check_status(m->ctx);
}

int ql_qkv_rope_append(ql_ctx* c, ql_kv* kv, const ql_attn_args* a, const float* x,
                       int32_t in_features, const float* wqkv_t, float* q_rot) {
  if (!c || !kv || !a) return ql_fail(QL_ERR_INVALID, "ql_qkv_rope_append: NULL argument");
  if (a->new_len > 0 && (!x || !wqkv_t || !q_rot))
    return ql_fail(QL_ERR_INVALID, "ql_qkv_rope_append: NULL buffer");
  if (in_features <= 0) return ql_fail(QL_ERR_INVALID, "in_features must be positive");
  QkvArgs g{};
  int r = ql_kv_append_prepare(c, kv, a, &g.cache, &g.rope, &g.seqs);
  if (r != QL_OK || a->new_len == 0) return r;
  g.x = x;
  g.wt = wqkv_t;
  g.rows = a->batch * a->new_len;
  g.K = in_features;
  g.hq = a->num_heads;
  g.hkv = a->num_kv_heads;
  g.hd = a->head_dim;
  g.N = (g.hq + 2 * g.hkv) * g.hd;
  g.new_len = a->new_len;
  g.q_rot = q_rot;
  g.status = c->status;
  const unsigned cols = static_cast<unsigned>((g.N / 2 + kGemmThreads - 1) / kGemmThreads);
  if (g.rows == 1)
    qkv_rope_append_kernel<1><<<dim3(cols, 1), kGemmThreads, 0, c->stream>>>(g);
  else
    qkv_rope_append_kernel<4><<<dim3(cols, (g.rows + 3) / 4), kGemmThreads, 0, c->stream>>>(g);
  QLM_CUDA(cudaGetLastError(), "launch the fused projection");
  ql_kv_append_commit(kv, a);
  return QL_OK;
}

int ql_sample(ql_ctx* c, const float* logits, int32_t vocab, const int32_t* context,
              int32_t n_context, const ql_sampler_config* cfg, double r, int32_t* token_out) {
  if (!c || !logits || !cfg || !token_out || (n_context > 0 && !context))
    return ql_fail(QL_ERR_INVALID, "ql_sample: NULL argument");
  int rc = check_sampler_config(cfg, vocab);
  if (rc != QL_OK) return rc;
  if (!(r >= 0.0 && r < 1.0)) return ql_fail(QL_ERR_INVALID, "the uniform draw must lie in [0, 1)");
  QLM_CUDA(cudaSetDevice(c->device), "set device");
  void* scratch = nullptr;
  rc = ql_ctx_workspace(c, sample_scratch_bytes(vocab), &scratch);
  if (rc != QL_OK) return rc;
  QLM_CUDA(launch_sample(*cfg, logits, vocab, context, n_context, r, static_cast<char*>(scratch),
                         token_out, c->status, c->stream),
           "launch the sampler");
  return QL_OK;
}

int ql_llama_generate(ql_llama* m, ql_kv* kv, int32_t seq, const int32_t* prompt,
                      int32_t n_prompt, int32_t steps, int32_t eos_id,
                      const ql_sampler_config* cfg, const double* uniforms, int32_t* out_tokens,
                      int32_t* n_out) {
  if (!m || !kv || !cfg || !n_out || (n_prompt > 0 && !prompt) || (steps > 0 && !out_tokens))
    return ql_fail(QL_ERR_INVALID, "ql_llama_generate: NULL argument");
  *n_out = 0;
  if (n_prompt <= 0) return ql_fail(QL_ERR_INVALID, "generate needs a non-empty prompt");
  if (steps < 0) return ql_fail(QL_ERR_INVALID, "steps must not be negative");
  int r = check_sampler_config(cfg, m->cfg.vocab_size);
  if (r != QL_OK) return r;
  if (cfg->temperature > 0.f) {
    if (!uniforms) return ql_fail(QL_ERR_INVALID, "sampling with temperature > 0 needs uniforms");
    for (int i = 0; i < steps; ++i)
      if (!(uniforms[i] >= 0.0 && uniforms[i] < 1.0))
        return ql_fail(QL_ERR_INVALID, "uniform %d does not lie in [0, 1)", i);
  }
  for (int i = 0; i < n_prompt; ++i)
    if (prompt[i] < 0 || prompt[i] >= m->cfg.vocab_size)
      return ql_fail(QL_ERR_INVALID, "Token id %d at position %d is outside the vocabulary",
                     prompt[i], i);
  if (steps == 0) return QL_OK;
  // the positions generate() reaches (its loop stops at the context limit)
  const int64_t total = static_cast<int64_t>(n_prompt) + steps - 1;
  if (total > m->cfg.max_position_embeddings)
    return ql_fail(QL_ERR_INVALID, "Last position %lld exceeds max_position_embeddings %d",
                   (long long)(total - 1), m->cfg.max_position_embeddings);
  int64_t cur = 0;
  if ((r = ql_kv_layer_len(kv, 0, seq, &cur)) != QL_OK) return r;
  if (cur != 0)
    return ql_fail(QL_ERR_INVALID, "generate starts at position 0; sequence %d holds %lld", seq,
                   (long long)cur);
  QLM_CUDA(cudaSetDevice(m->ctx->device), "set device");
  if ((r = ensure_rows(m, n_prompt)) != QL_OK) return r;
  cudaStream_t s = m->ctx->stream;
  // m->ids holds the whole context: prompt, then each sampled token
  QLM_CUDA(cudaMemcpyAsync(m->ids, prompt, static_cast<size_t>(n_prompt) * 4,
                           cudaMemcpyHostToDevice, s),
           "copy the prompt");
  int64_t position = 0;
  int len = n_prompt, batch_first = 0, batch_n = n_prompt, produced = 0;
  for (int step = 0; step < steps; ++step) {
    if ((r = forward_device(m, kv, seq, m->ids + batch_first, batch_n, position, 1)) != QL_OK)
      return r;
    const double u = cfg->temperature > 0.f ? uniforms[step] : 0.0;
    QLM_CUDA(launch_sample(*cfg, m->logits, m->cfg.vocab_size, m->ids, len, u, m->sample_scratch,
                           m->ids + len, m->ctx->status, s),
             "launch the sampler");
    if (eos_id >= 0) {  // the loop must stop at EOS: look at each token
      int32_t tok = -1;
      QLM_CUDA(cudaMemcpyAsync(&tok, m->ids + len, 4, cudaMemcpyDeviceToHost, s), "read a token");
      QLM_CUDA(cudaStreamSynchronize(s), "synchronize generate");
      if ((r = ql_check_status(m->ctx)) != QL_OK) return r;
      if (tok == eos_id) break;
    }
    ++produced;
    position += batch_n;
    batch_first = len;
    batch_n = 1;
    ++len;
  }
  if (produced > 0)
    QLM_CUDA(cudaMemcpyAsync(out_tokens, m->ids + n_prompt, static_cast<size_t>(produced) * 4,
                             cudaMemcpyDeviceToHost, s),
             "copy the generated tokens");
  QLM_CUDA(cudaStreamSynchronize(s), "synchronize generate");
  if ((r = ql_check_status(m->ctx)) != QL_OK) return r;
  *n_out = produced;
  return QL_OK;
}

}  // extern "C"
