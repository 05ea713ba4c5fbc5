// ql_kernels.cu -- the attention hot path kernels for B200 (sm_100a).
//
//  append_kernel    RoPE on new K rows + conversion/quantisation of K and V into
//                   the paged cache (reference: ops.rs:168-220 rope,
//                   cache.rs:146-163 update writes).
//  splitkv_kernel   causal GQA attention of one query token per CTA job over
//                   the cached prefix, split along the KV length.  K/V tiles
//                   are streamed by TMA into swizzled shared memory behind an
//                   mbarrier pipeline (one producer warp, four consumer warps);
//                   QK^T and PV run on the tensor cores with f32 accumulation;
//                   online softmax in registers; the last CTA of a job merges
//                   the splits.  For single-token decode the same CTA also
//                   rotates and appends the new K/V (fused prologue).
//                   (reference: layers.rs:425-455 with cache.rs:185-229 get)
//  generic_kernel   CUDA-core path for f32 caches and other head sizes; it keeps
//                   the reference's operation order (sequential f32 dot
//                   products without FMA, f64 softmax with a sequential sum,
//                   sequential f32 P.V) so its results track the reference to
//                   the last bit in all but rare f64-exp rounding cases.
//  gather_kernel    KvCache::get (cache.rs:185-229) into f32.
#include <math_constants.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "ql_append.cuh"
#include "ql_device.cuh"
#include "ql_kernels.cuh"

namespace ql {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float cache_value(const CacheView& c, const void* base,
                                             const uint16_t* scale, int64_t row, int d) {
  const size_t e = static_cast<size_t>(row) * c.hd + d;
  if (c.dtype == kQ8_0) {
    float s = __half2float(__ushort_as_half(scale[static_cast<size_t>(row) * (c.hd / 32) + d / 32]));
    return s * static_cast<float>(static_cast<const int8_t*>(base)[e]);
  }
  return load_elem(base, e, c.dtype);
}

}  // namespace

// ---------------------------------------------------------------- append --
// TOKENS (head_dim 64 or 128, f32/f16/bf16 cache): one warp per new token,
// every KV head's row (append_token); otherwise one warp per (token, KV head)
// row (append_kv_row, which also quantises Q8_0 blocks).
template <int TOKENS>
__global__ void __launch_bounds__(128) append_kernel(const __grid_constant__ AppendArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if constexpr (TOKENS != 0) {
    if (warp >= a.batch * a.new_len) return;
    append_token<TOKENS>(a, warp, lane);
  } else {
    if (warp >= a.batch * a.new_len * a.cache.hkv) return;
    append_kv_row(a, warp, lane);
  }
}

cudaError_t launch_append(const AppendArgs& a, cudaStream_t s) {
  const bool tokens = a.cache.dtype != kQ8_0 && (a.cache.hd == 64 || a.cache.hd == 128);
  const int warps = a.batch * a.new_len * (tokens ? 1 : a.cache.hkv);
  if (warps == 0) return cudaSuccess;
  const int blocks = (warps + 3) / 4;
  if (!tokens)
    append_kernel<0><<<blocks, 128, 0, s>>>(a);
  else if (a.cache.hd == 64)
    append_kernel<64><<<blocks, 128, 0, s>>>(a);
  else
    append_kernel<128><<<blocks, 128, 0, s>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- gather --
__global__ void __launch_bounds__(128) gather_kernel(const __grid_constant__ GatherArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int hkv = a.cache.hkv, hd = a.cache.hd;
  if (warp >= a.n * hkv) return;
  const int i = warp / hkv, h = warp % hkv;
  bool ok;
  const int64_t row = cache_row(a.cache, a.seq, a.positions[i], h, nullptr, ok);
  const size_t o = (static_cast<size_t>(i) * hkv + h) * hd;
  for (int d = lane; d < hd; d += 32) {
    a.k_out[o + d] = ok ? cache_value(a.cache, a.cache.k, a.cache.k_scale, row, d) : 0.f;
    a.v_out[o + d] = ok ? cache_value(a.cache, a.cache.v, a.cache.v_scale, row, d) : 0.f;
  }
}

cudaError_t launch_gather(const GatherArgs& a, cudaStream_t s) {
  const int rows = a.n * a.cache.hkv;
  if (rows == 0) return cudaSuccess;
  gather_kernel<<<(rows + 3) / 4, 128, 0, s>>>(a);
  return cudaGetLastError();
}

// ----------------------------------------------------------- table patch --
__global__ void __launch_bounds__(256) table_patch_kernel(const __grid_constant__ TablePatch p) {
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) p.table[p.idx[i]] = p.val[i];
}

cudaError_t launch_table_patch(const TablePatch& p, cudaStream_t s) {
  if (p.n <= 0) return cudaSuccess;
  table_patch_kernel<<<1, 256, 0, s>>>(p);
  return cudaGetLastError();
}

// --------------------------------------------------------------- generic --
// One CTA per (query head, query token).  Bit-level restatement of the
// reference's per-head loop (layers.rs:434-445) on the GPU.
__global__ void __launch_bounds__(256) generic_kernel(const __grid_constant__ AttnArgs a,
                                                      int job0) {
  const int h = blockIdx.x;
  const int job = job0 + blockIdx.y;
  const int b = job / a.new_len, t = job % a.new_len;
  const int hd = a.cache.hd;
  const int kvh = h / a.group;
  const int qpos = a.seqs.start[b] + t;
  const int L = qpos + 1;
  const int seq = a.seqs.seq[b];
  extern __shared__ float sh[];  // q [hd], reduction [32]
  float* q = sh;
  float* red = sh + hd;
  const double2* rope_row = a.rope + static_cast<size_t>(qpos) * a.rope_stride;
  const size_t qoff = (static_cast<size_t>(job) * a.hq + h) * hd;
  for (int p = threadIdx.x; p < hd / 2; p += blockDim.x) {
    float y0, y1;
    rope_pair(load_elem(a.q, qoff + 2 * p, a.in_dtype), load_elem(a.q, qoff + 2 * p + 1, a.in_dtype),
              rope_row[p], y0, y1);
    q[2 * p] = y0;
    q[2 * p + 1] = y1;
  }
  __syncthreads();
  const size_t srow = (static_cast<size_t>(blockIdx.y) * a.hq + h) * a.max_len;
  float* sc = a.scratch + srow;
  double* cd = a.scratch_d + srow;
  // scores, scaled (matmul then scale, ops.rs:63-94 and :257-261)
  float mx = -CUDART_INF_F;
  for (int j = threadIdx.x; j < L; j += blockDim.x) {
    bool ok;
    const int64_t row = cache_row(a.cache, seq, j, kvh, a.status, ok);
    float acc = 0.f;
    for (int d = 0; d < hd; ++d)
      acc = __fadd_rn(acc, __fmul_rn(q[d], ok ? cache_value(a.cache, a.cache.k, a.cache.k_scale,
                                                               row, d)
                                               : 0.f));
    acc = __fmul_rn(acc, a.scale);
    sc[j] = acc;
    mx = fmaxf(mx, acc);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -CUDART_INF_F;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mx = red[0];
  // contributions in f64 (ops.rs:298-310)
  for (int j = threadIdx.x; j < L; j += blockDim.x) {
    const float v = sc[j];
    double c;
    if (mx == -CUDART_INF_F) c = 1.0;
    else if (mx == CUDART_INF_F) c = (v == CUDART_INF_F) ? 1.0 : 0.0;
    else c = exp(static_cast<double>(v) - static_cast<double>(mx));
    cd[j] = c;
  }
  __syncthreads();
  __shared__ double denom_s;
  if (threadIdx.x == 0) {
    double den = 0.0;
    for (int j = 0; j < L; ++j) den += cd[j];  // sequential, as the reference sums
    denom_s = den;
  }
  __syncthreads();
  const double den = denom_s;
  for (int j = threadIdx.x; j < L; j += blockDim.x) sc[j] = static_cast<float>(cd[j] / den);
  __syncthreads();
  // P.V, sequential over keys (ops.rs:81-91 i-k-j order)
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < L; ++j) {
      bool ok;
      const int64_t row = cache_row(a.cache, seq, j, kvh, nullptr, ok);
      const float vv = ok ? cache_value(a.cache, a.cache.v, a.cache.v_scale, row, d) : 0.f;
      acc = __fadd_rn(acc, __fmul_rn(sc[j], vv));
    }
    store_elem(a.out, (static_cast<size_t>(job) * a.hq + h) * hd + d, a.out_dtype, acc);
  }
}

cudaError_t launch_generic(const AttnArgs& a, cudaStream_t s) {
  const int jobs = a.batch * a.new_len;
  const size_t smem = (a.cache.hd + 32) * sizeof(float);
  for (int j0 = 0; j0 < jobs; j0 += 65535) {
    dim3 grid(a.hq, min(65535, jobs - j0));
    generic_kernel<<<grid, 256, smem, s>>>(a, j0);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// ---------------------------------------------------------------- splitkv --
namespace {

template <int HD, int DT, int KG = 1>
struct SplitCfg {
  // KG groups of four consumer warps per CTA: KG == 1 streams one split per
  // CTA at two or three CTAs per SM (throughput); KG > 1 (f16/bf16 only) lets
  // the groups take alternate tiles of one split in parallel, one CTA per SM,
  // for calls with too few (token, KV head) jobs to fill the GPU (latency).
  static constexpr int kConsumerWarps = 4 * KG;
  static constexpr int kConsumers = 32 * kConsumerWarps;
  static constexpr int kThreads = kConsumers + 32;
  static constexpr bool kQ8 = DT == kQ8_0;
  static constexpr bool kBF = DT == kBF16;
  // K and V tile bytes of one 64-position stage
  static constexpr int kKBytes = kQ8 ? kTile * HD : kTile * HD * 2;
  static constexpr int kScaleBytes = kQ8 ? kTile * (HD / 32) * 2 : 0;
  static constexpr int kRaw = 2 * kKBytes + 2 * kScaleBytes;
  static constexpr int kStageBytes = (kRaw + 1023) / 1024 * 1024;
  // Q8_0 keeps three stages so that three CTAs (15 warps) fit on an SM; the
  // wide variant fills most of the SM's shared memory with stages.
  static constexpr int kStages = KG > 1 ? 192 * 1024 / kStageBytes
                                        : (kQ8 ? 3 : (HD == 128 ? 3 : 6));
  static constexpr int kMinCtas = KG > 1 ? 1 : (kQ8 ? 3 : 2);  // resident CTAs per SM
  static constexpr int kTx = kRaw;
  static constexpr int kQLd = HD + 8;  // q tile row stride (elements), padded
  // the new token's converted K/V row (fused append), 16-byte aligned
  static constexpr int kRowOff = ((16 * kQLd * 2 + 16 * kConsumerWarps * 4 + 16 +
                                   (2 * kStages + 1) * 8) + 15) / 16 * 16;
  static constexpr int kRowBytes = kQ8 ? 2 * HD + 2 * (HD / 32) * 2 : 4 * HD;
  static constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * kStageBytes + kRowOff +
                                  (kRowBytes + 15) / 16 * 16;
  // Cluster mode (KG == 1): rank 0's gather area past the regular layout,
  // for clusters of `ctas` CTAs: rows [ctas][8][HD] and (max, sum)
  // [ctas][8][2], f32, then rank 0's mbarrier that counts the bytes the other
  // CTAs store.  Only clustered launches request these bytes.
  static constexpr int kMaxCluster = kMaxClusterCtas;
  static constexpr size_t kGatherOff = (kSmem - 1024 + 15) / 16 * 16;
  static constexpr size_t gather_bytes(int ctas) {
    return (static_cast<size_t>(ctas) * 8 * HD + ctas * 16) * 4 + 16;
  }
  // a launch with clusters of `ctas` CTAs requests the gather area for that many
  static constexpr size_t smem_cluster(int ctas) { return 1024 + kGatherOff + gather_bytes(ctas); }
  static constexpr size_t kSmemCluster = smem_cluster(kMaxCluster);
  // warp partials [warps][8][HD], the output rows [8][HD], (max, sum) [8][2] and
  // the per-(warp, head) weights [warps][8], f32
  static_assert(((kConsumerWarps + 1) * 8 * HD + 16 + 8 * kConsumerWarps + 16 * 8 + 64) * 4 <=
                    kStages * kStageBytes,
                "merge buffer must fit the stages");
  static_assert(KG == 1 || (!kQ8 && kStages >= KG), "wide variant: f16/bf16, a stage per group");
  // Q8_0 int8 q fragments [HD/32][32][4 words], per-head factors [8] and
  // half-row maxima [8][HD/64] in the q tile's space
  static_assert(!kQ8 || (HD / 32) * 512 + (8 + 8 * (HD / 64)) * 4 <= 16 * kQLd * 2,
                "Q8_0 q fragments must fit the q tile");
};

// Q8_0 QK^T runs on the integer tensor path: q is quantised per head to
// int8 hi + lo/254 (scale max|q| / 127), hi in A rows 0-7 and lo in rows
// 8-15, one m16n8k32 MMA per 32-element Q8_0 block.  A thread's B fragment
// is then the 8 consecutive K bytes 8t..8t+7 of its block (MMA k 4t..4t+3
// and 16+4t..16+4t+3), so q follows the same order: byte d of head h goes to
// the fragment word of lane 4h + t that MMA k index of d falls in.  The
// fragments sit in lane order, [block][lane][4 words], one 16-byte load each.
__device__ __forceinline__ int q8_frag_byte(int h, int d, bool lo) {
  const int blk = d >> 5, w = d & 31, t = w >> 3, half = (w >> 2) & 1;
  return ((blk * 32 + h * 4 + t) * 4 + 2 * half + (lo ? 1 : 0)) * 4 + (d & 3);
}

// The decode kernel's fused append of the new token's row (one warp): all
// loads first, then the converted row into shared memory and the release of
// the consumers, then the same bytes into the cache.  Same conversion as
// append_row_t; the cache is f16, bf16 or Q8_0 here.
template <int HD, bool DEV, int IN = -1>
__device__ __forceinline__ void append_fused(const AttnArgs& a, const RopeSrc& rope,
                                             size_t in_off, bool ok, int64_t dst, int lane,
                                             uint8_t* stage, uint64_t* released) {
  const int in_dt = IN >= 0 ? IN : a.in_dtype;  // IN: the type known at compile time
  static_assert(HD % 64 == 0, "whole pairs per lane");
  constexpr int kIt = HD / 64;  // pairs per lane
  const bool kvec = pair_aligned(a.k, in_dt), vvec = pair_aligned(a.v, in_dt);
  float2 kx[kIt], vx[kIt];
  double2 cs[kIt];
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    const int p = it * 32 + lane;
    kx[it] = load_pair(a.k, in_off + 2 * p, in_dt, kvec);
    vx[it] = load_pair(a.v, in_off + 2 * p, in_dt, vvec);
    cs[it] = rope_cs<DEV>(rope, p, HD);
  }
#pragma unroll
  for (int it = 0; it < kIt; ++it) rope_pair(kx[it].x, kx[it].y, cs[it], kx[it].x, kx[it].y);
  const CacheView& c = a.cache;
  if (c.dtype == kQ8_0) {
    int8_t qk[kIt][2], qv[kIt][2];
    __half sk[kIt], sv[kIt];
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      q8_0_pair(kx[it].x, kx[it].y, qk[it][0], qk[it][1], sk[it]);
      q8_0_pair(vx[it].x, vx[it].y, qv[it][0], qv[it][1], sv[it]);
      const int p = it * 32 + lane;
      *reinterpret_cast<char2*>(stage + 2 * p) = make_char2(qk[it][0], qk[it][1]);
      *reinterpret_cast<char2*>(stage + HD + 2 * p) = make_char2(qv[it][0], qv[it][1]);
      if ((lane & 15) == 0) {
        uint16_t* ss = reinterpret_cast<uint16_t*>(stage + 2 * HD);
        ss[(2 * p) / 32] = __half_as_ushort(sk[it]);
        ss[HD / 32 + (2 * p) / 32] = __half_as_ushort(sv[it]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(released);
    if (ok) {
#pragma unroll
      for (int it = 0; it < kIt; ++it) {
        const int p = it * 32 + lane;
        const size_t e = static_cast<size_t>(dst) * HD + 2 * p;
        *reinterpret_cast<char2*>(static_cast<int8_t*>(c.k) + e) = make_char2(qk[it][0], qk[it][1]);
        *reinterpret_cast<char2*>(static_cast<int8_t*>(c.v) + e) = make_char2(qv[it][0], qv[it][1]);
        if ((lane & 15) == 0) {
          const size_t si = static_cast<size_t>(dst) * (HD / 32) + (2 * p) / 32;
          c.k_scale[si] = __half_as_ushort(sk[it]);
          c.v_scale[si] = __half_as_ushort(sv[it]);
        }
      }
    }
  } else {
    const bool bf = c.dtype == kBF16;
    uint32_t kk[kIt], vv[kIt];
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      kk[it] = bf ? pack2<true>(kx[it].x, kx[it].y) : pack2<false>(kx[it].x, kx[it].y);
      vv[it] = bf ? pack2<true>(vx[it].x, vx[it].y) : pack2<false>(vx[it].x, vx[it].y);
      const int p = it * 32 + lane;
      reinterpret_cast<uint32_t*>(stage)[p] = kk[it];
      reinterpret_cast<uint32_t*>(stage + 2 * HD)[p] = vv[it];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(released);
    if (ok) {
#pragma unroll
      for (int it = 0; it < kIt; ++it) {
        const size_t e = static_cast<size_t>(dst) * HD + 2 * (it * 32 + lane);
        *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(c.k) + e) = kk[it];
        *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(c.v) + e) = vv[it];
      }
    }
  }
}

// Pairs (2p, 2p+1) of the q rows of one KV head's group, item idx = tid +
// it * NCT -> head idx / (HD/2), pair idx % (HD/2) (zero past the group).
// The input type is resolved once, outside the loads, so that every load is
// issued before the first is used.
template <int N, int NCT, int HD, typename LD>
__device__ __forceinline__ void gather_q_pairs(int group, size_t row0, int tid, float2 (&x)[N],
                                               LD ld) {
#pragma unroll
  for (int it = 0; it < N; ++it) {
    const int idx = tid + it * NCT, hg = idx / (HD / 2), p = idx % (HD / 2);
    x[it] = idx < 8 * (HD / 2) && hg < group ? ld(row0 + static_cast<size_t>(hg) * HD + 2 * p)
                                             : make_float2(0.f, 0.f);
  }
}

template <int N, int NCT, int HD, int IN = -1, int GRP = 0>
__device__ __forceinline__ void load_q_pairs(const AttnArgs& a, size_t row0, int tid,
                                             float2 (&x)[N]) {
  const void* q = a.q;
  const int gsize = GRP ? GRP : a.group;  // GRP: the group size known at compile time
  const int in_dt = IN >= 0 ? IN : a.in_dtype;  // IN: the type known at compile time
  if (in_dt == kF16 && pair_aligned(q, kF16)) {
    gather_q_pairs<N, NCT, HD>(gsize, row0, tid, x, [q](size_t i) {
      return __half22float2(*reinterpret_cast<const __half2*>(static_cast<const __half*>(q) + i));
    });
  } else if (in_dt == kBF16 && pair_aligned(q, kBF16)) {
    gather_q_pairs<N, NCT, HD>(gsize, row0, tid, x, [q](size_t i) {
      return __bfloat1622float2(
          *reinterpret_cast<const __nv_bfloat162*>(static_cast<const __nv_bfloat16*>(q) + i));
    });
  } else if (in_dt == kF32 && pair_aligned(q, kF32)) {
    gather_q_pairs<N, NCT, HD>(gsize, row0, tid, x, [q](size_t i) {
      return *reinterpret_cast<const float2*>(static_cast<const float*>(q) + i);
    });
  } else {
    const int dt = in_dt;
    gather_q_pairs<N, NCT, HD>(gsize, row0, tid, x, [q, dt](size_t i) {
      return make_float2(load_elem(q, i, dt), load_elem(q, i + 1, dt));
    });
  }
}

// Decode softmax: the running maximum used as reference lags the true one by
// at most this much (log2 units), so probabilities stay below 2^8.
constexpr float kLazyLog2 = 8.f;

__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  // byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128B-swizzled box
  return static_cast<uint32_t>(row * 128 + (((chunk ^ (row & 7))) << 4));
}

// Barrier of the consumer warps only (the producer warp may have returned).
template <int N>
__device__ __forceinline__ void bar_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}

// ---- head-sharded output exchange (PeerOut) ----
// One thread, after the stream dependencies are met: every rank may now store
// into this rank's output for this call.
__device__ __forceinline__ uint32_t peer_epoch(const PeerOut& po) {  // this call's number
  return __ldcg(po.epoch) + 1u;
}
__device__ __forceinline__ void peer_enter(const PeerOut& po, uint32_t e) {
  for (int p = 0; p < po.nranks; ++p) st_release_sys(po.flags[p] + po.rank, e);
}
// Before the first store into the other ranks: have they all entered?
__device__ __forceinline__ bool peer_wait_entered(const PeerOut& po, uint32_t e,
                                                  uint32_t* status) {
  bool ok = true;
  for (int p = 0; p < po.nranks && ok; ++p) ok = wait_epoch(po.flags[po.rank] + p, e, status);
  return ok;
}
// One thread per CTA, after a CTA barrier that follows the CTA's stores:
// counts the CTA.  The
// last CTA of the launch tells every rank that this rank's stores are
// visible, waits until every rank has told it the same (so the output is
// complete when the kernel ends), re-arms the counter and records the call.
// Ordering without a system-wide fence: the CTA barrier before this call
// orders the CTA's row stores (to this and the other GPUs) before this
// thread's arrival; the arrival is a GPU-scope release/acquire add, so the
// last CTA to arrive has every CTA's stores ordered before its own `done`
// stores, which are system-scope releases; another GPU that reads `done` with
// a system-scope acquire then sees the rows (release/acquire chains are
// cumulative).
__device__ __forceinline__ void peer_arrive(const PeerOut& po, uint32_t e, uint32_t* status) {
  if (atom_add_acq_rel_gpu(po.arrivals, 1) != po.total_ctas - 1) return;
  for (int p = 0; p < po.nranks; ++p) st_release_sys(po.flags[p] + kMaxRanks + po.rank, e);
  bool ok = true;
  for (int p = 0; p < po.nranks && ok; ++p)
    ok = wait_epoch(po.flags[po.rank] + kMaxRanks + p, e, status);
  atomicExch(po.arrivals, 0);
  atomicExch(po.epoch, e);
}

// The 128 consumer threads write the group's output rows res[hg][0..HD): to
// the call's output, or, for a head-sharded call, into every rank's output
// (after every rank has entered the call), then count the CTA.
template <int HD, int NCT, bool PEER, int OUT = -1, int GRP = 0>
__device__ __forceinline__ void emit_rows(const AttnArgs& a, const float* res, int job, int kvh,
                                          int tid, int* flag) {
  const PeerOut& po = a.peer;
  const bool vec = a.out_vec != 0;
  const int out_dt = OUT >= 0 ? OUT : a.out_dtype;  // OUT: the type known at compile time
  const int gsize = GRP ? GRP : a.group;
  if (!PEER || po.nranks == 0) {
    for (int c = tid; c < gsize * (HD / 8); c += NCT) {
      const int hg = c / (HD / 8), d0 = (c % (HD / 8)) * 8;
      store8(a.out, (static_cast<size_t>(job) * a.hq + kvh * gsize + hg) * HD + d0,
             out_dt, res + hg * HD + d0, vec);
    }
    return;
  }
  const uint32_t e = peer_epoch(po);
  if (tid == 0) flag[1] = peer_wait_entered(po, e, a.status);
  bar_consumers<NCT>();
  if (flag[1]) {
    for (int c = tid; c < gsize * (HD / 8); c += NCT) {
      const int hg = c / (HD / 8), d0 = (c % (HD / 8)) * 8;
      const size_t off =
          (static_cast<size_t>(job) * po.hq_total + po.head_base + kvh * gsize + hg) * HD + d0;
      for (int p = 0; p < po.nranks; ++p)
        store8(po.out[p], off, out_dt, res + hg * HD + d0, vec);
    }
  }
  // The barrier orders every thread's stores before thread 0's arrival in
  // peer_arrive, whose release covers them (a release is cumulative).
  bar_consumers<NCT>();
  if (tid == 0) peer_arrive(po, e, a.status);
}

}  // namespace

// CL: the launch is clustered (a.cluster > 1); PEER: a head-sharded call
// (a.peer.nranks > 0); IO: the input and output type when both are known
// (-1: read from the arguments); GRP: the query heads per KV head when known
// (0: read from the arguments).  Compile-time facts, so that each form holds
// only its own merge, exchange and conversions: the code a launch runs is
// fetched cold, and less of it is faster.
template <int HD, int DT, bool DEVROPE, int KG, bool CL, bool PEER, int IO, int GRP>
__global__ void __launch_bounds__(SplitCfg<HD, DT, KG>::kThreads, SplitCfg<HD, DT, KG>::kMinCtas)
    splitkv_kernel(const __grid_constant__ AttnArgs a, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, int job0) {
  using C = SplitCfg<HD, DT, KG>;
  const int gsize = GRP ? GRP : a.group;  // GRP: the group size known at compile time
  constexpr int NCW = C::kConsumerWarps;  // consumer warps; warp NCW is the producer
  constexpr int NCT = C::kConsumers;
  constexpr bool Q8 = C::kQ8;
  constexpr bool BF = C::kBF;  // bf16 operands for both MMAs; f16 otherwise
  constexpr int NKS = HD / 16;  // k-steps of QK^T
  constexpr int NO = HD / 8;    // n-tiles of the output

  const int split = blockIdx.x, kvh = blockIdx.y, job = job0 + blockIdx.z;
  const int b = job / a.new_len, t_tok = job % a.new_len;
  const int seq = a.seqs.seq[b];
  const int qpos = a.seqs.start[b] + t_tok;
  const int L = qpos + 1;
  const int ntiles = (L + kTile - 1) / kTile;
  const int nsplit = (ntiles + a.tiles_per_split - 1) / a.tiles_per_split;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  // The CTA's merged rows [8][HD] (normalised) and their (max, sum) [8][2]:
  // what the cluster merge reads from every CTA's shared memory.
  float* res = reinterpret_cast<float*>(stages) + NCW * 8 * HD;
  float* cml = res + 8 * HD;
  // Cluster mode: the splits of one (token, KV head) form a thread-block
  // cluster along x and merge through distributed shared memory; every CTA of
  // the cluster reaches both cluster barriers below on every path.
  constexpr bool cl = CL;  // the host launches CL exactly when a.cluster > 1
  float* grows = reinterpret_cast<float*>(smem + C::kGatherOff);  // rank 0: [rank][8][HD]
  float* gml = grows + a.cluster * 8 * HD;                         // [rank][16] (max, sum)
  uint64_t* gbar = reinterpret_cast<uint64_t*>(gml + a.cluster * 16);  // counts their bytes

  if (split >= nsplit) {
    // In a clustered launch such a CTA sends rank 0 nothing (rank 0 expects
    // the bytes of the live splits only); it still arrives on the cluster
    // barrier that the others wait on.
    if (cl) cluster_arrive_relaxed();
    if (PEER && a.peer.nranks) {  // still counted, once the previous call is done with the counters
      griddep_wait();
      if (threadIdx.x == 0) peer_arrive(a.peer, peer_epoch(a.peer), a.status);
    }
    return;
  }
  const int tile0 = split * a.tiles_per_split;
  const int my_tiles = min(ntiles, tile0 + a.tiles_per_split) - tile0;
  const int hkv = a.cache.hkv;

  uint16_t* qs = reinterpret_cast<uint16_t*>(smem + C::kStages * C::kStageBytes);
  float* ml = reinterpret_cast<float*>(qs + 16 * C::kQLd);  // [NCW][8][2] (m, l)
  int* flag = reinterpret_cast<int*>(ml + 16 * NCW);
  uint64_t* full = reinterpret_cast<uint64_t*>(flag + 4);
  uint64_t* empty = full + C::kStages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  // consumer group, and the 16-position slice of a tile the warp takes
  const int grp = KG == 1 ? 0 : warp >> 2, slice = KG == 1 ? warp : warp & 3;

  uint64_t* appended = empty + C::kStages;  // the fused append is written and fenced
  uint8_t* newrow = reinterpret_cast<uint8_t*>(qs) + C::kRowOff;  // its converted K/V row
  const bool appends = a.fuse_append && split == nsplit - 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    mbar_init(appended, 1);
    if (cl && split == 0) mbar_init(gbar, 1);  // rank 0's expect_tx; the bytes complete it
    fence_mbar_init();
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  __syncthreads();
  if (cl) cluster_arrive_relaxed();  // after the init fence: the others may now arrive on gbar
  // Page ids of the first 32 tiles, one per producer lane, fetched before the
  // stream dependency is met: the block table is written only by the table
  // patch kernel, and a launch that follows a patch is an ordinary one (no
  // programmatic dependency), so the entries are in place when this runs.
  const int* bt = a.cache.block_table + static_cast<size_t>(seq) * a.cache.pages_per_seq;
  int lane_page = 0;
  if (warp == NCW && lane < my_tiles) lane_page = __ldg(bt + (tile0 + lane) * kTile / a.cache.page);
  // What the CTA reads first once the dependency is met is fetched into L2
  // now (prefetches read nothing into the CTA; lines written meanwhile are
  // updated in L2): the first stages' tiles, q of this KV head's group, the
  // rotation row and, for the appending CTA, the new K and V rows.
  // The appending CTA's block-table entry for the new row (same rule).
  int app_page = -1;
  if (warp == NCW && appends)
    app_page = __ldg(bt + static_cast<size_t>(qpos) / a.cache.page);
  if (warp == NCW) {
    if (lane < min(my_tiles, C::kStages) && lane_page >= 0 && lane_page < a.cache.num_pages) {
      const int row =
          (lane_page * hkv + kvh) * a.cache.page + ((tile0 + lane) * kTile) % a.cache.page;
      if constexpr (Q8) {
        tma_prefetch_2d(&kmap, 0, row);
        tma_prefetch_2d(&vmap, 0, row);
        bulk_prefetch_l2(a.cache.k_scale + static_cast<size_t>(row) * (HD / 32), C::kScaleBytes);
        bulk_prefetch_l2(a.cache.v_scale + static_cast<size_t>(row) * (HD / 32), C::kScaleBytes);
      } else {
#pragma unroll
        for (int box = 0; box < HD / 64; ++box) {
          tma_prefetch_2d(&kmap, box * 64, row);
          tma_prefetch_2d(&vmap, box * 64, row);
        }
      }
    }
  } else if (warp < 4) {
    const int ib = (IO >= 0 ? IO : a.in_dtype) == kF32 ? 4 : 2;
    const size_t kv_off = (static_cast<size_t>(job) * hkv + kvh) * HD * ib;
    const char* base = nullptr;
    int bytes = 0;
    if (warp == 0) {
      base = static_cast<const char*>(a.q) +
             (static_cast<size_t>(job) * a.hq + kvh * gsize) * HD * ib;
      bytes = gsize * HD * ib;
    } else if (warp == 1 && !DEVROPE) {
      base = reinterpret_cast<const char*>(a.rope + static_cast<size_t>(qpos) * a.rope_stride);
      bytes = HD / 2 * 16;
    } else if (warp >= 2 && appends) {
      base = static_cast<const char*>(warp == 2 ? a.k : a.v) + kv_off;
      bytes = HD * ib;
    }
    if (bytes > 0) {
      const uintptr_t l0 = reinterpret_cast<uintptr_t>(base) & ~static_cast<uintptr_t>(127);
      const int lines = static_cast<int>((reinterpret_cast<uintptr_t>(base) + bytes - l0 + 127) / 128);
      for (int t = lane; t < lines; t += 32) prefetch_l2(reinterpret_cast<const void*>(l0 + 128 * t));
    }
  }
  // Programmatic dependent launch: everything above overlaps the previous
  // kernel; Q/K/V and the cache may come from it, so they are read only after
  // this wait.  The next kernel may start its own set-up from here on.
  griddep_wait();
  griddep_launch_dependents();
  // A sharded call's number (*epoch + 1) is read where it is used rather than
  // kept live through the tile loop: no CTA stores the new count before every
  // CTA of the launch has arrived, and each CTA reads it before arriving.
  if (PEER && a.peer.nranks && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 &&
      blockIdx.z == 0)
    peer_enter(a.peer, peer_epoch(a.peer));

  const RopeSrc rsrc{DEVROPE ? nullptr : a.rope + static_cast<size_t>(qpos) * a.rope_stride,
                     static_cast<double>(qpos), static_cast<double>(a.rope_theta)};

  // ------------------------------------------------------------ producer --
  // Streams this split's tiles right away, while the consumers rotate q; only
  // the tile holding the new token waits until its K/V row has been appended.
  if (warp == NCW) {
    // Tile i of the split into stage i % kStages (lane 0).
    auto issue = [&](int i, int page) {
      const int st = i % C::kStages;
      const int p0 = (tile0 + i) * kTile;
      if (page < 0 || page >= a.cache.num_pages) {
        atomicOr(a.status, kStatusBadPage);
        page = 0;  // keep the pipeline consistent; the result is flagged
      }
      const int row = (page * hkv + kvh) * a.cache.page + p0 % a.cache.page;
      uint8_t* sb = stages + st * C::kStageBytes;
      mbar_arrive_expect_tx(&full[st], C::kTx);
      if constexpr (Q8) {
        tma_load_2d(sb, &kmap, 0, row, &full[st]);
        tma_load_2d(sb + C::kKBytes, &vmap, 0, row, &full[st]);
        bulk_load(sb + 2 * C::kKBytes, a.cache.k_scale + static_cast<size_t>(row) * (HD / 32),
                  C::kScaleBytes, &full[st]);
        bulk_load(sb + 2 * C::kKBytes + C::kScaleBytes,
                  a.cache.v_scale + static_cast<size_t>(row) * (HD / 32), C::kScaleBytes,
                  &full[st]);
      } else {
#pragma unroll
        for (int box = 0; box < HD / 64; ++box) {
          tma_load_2d(sb + box * 8192, &kmap, box * 64, row, &full[st]);
          tma_load_2d(sb + C::kKBytes + box * 8192, &vmap, box * 64, row, &full[st]);
        }
      }
    };
    // The lanes hold the page ids of 32 tiles at a time, so no dependent
    // global load sits between two copies; lane 0 waits for free stages and
    // issues.  The tile holding the new token is copied at once too: its new
    // row is patched in shared memory by the consumers.
    // Single-token decode: the CTA holding the last tile writes the new K/V
    // row (rotated K) to the cache and to shared memory, then releases the
    // consumer warp that patches it into its tile.  The producer does this
    // right after its first burst of copies, while the consumers rotate q.
    // The consumers need only the shared-memory row, so they are released
    // before the proxy fence that orders the cache writes before later TMA
    // reads (the fence may wait for this warp's copies in flight).
    auto append_new_row = [&]() {
      const bool ok = app_page >= 0 && app_page < a.cache.num_pages;
      if (!ok && lane == 0) atomicOr(a.status, kStatusBadPage);
      const int64_t dst =
          ok ? (static_cast<int64_t>(app_page) * hkv + kvh) * a.cache.page + qpos % a.cache.page
             : 0;
      append_fused<HD, DEVROPE, IO>(a, rsrc, (static_cast<size_t>(job) * hkv + kvh) * HD, ok, dst,
                                lane, newrow, appended);
      fence_proxy_async_global();
    };
    bool alive = true, append_due = appends;
    const int burst = min(my_tiles, C::kStages);
    for (int i0 = 0; i0 < my_tiles && alive; i0 += 32) {
      if (i0 > 0)
        lane_page = i0 + lane < my_tiles ? __ldg(bt + (tile0 + i0 + lane) * kTile / a.cache.page)
                                         : 0;
      const int n = min(32, my_tiles - i0);
      for (int j = 0; j < n && alive; ++j) {
        const int page = __shfl_sync(0xffffffffu, lane_page, j);
        if (lane == 0) {
          const int i = i0 + j, st = i % C::kStages;
          if (i >= C::kStages && !mbar_wait(&empty[st], ((i / C::kStages) - 1) & 1, a.status))
            alive = false;
          else
            issue(i, page);
        }
        alive = __shfl_sync(0xffffffffu, alive, 0);
        if (append_due && i0 + j + 1 == burst) {
          append_new_row();
          append_due = false;
        }
      }
    }
    if (append_due) append_new_row();  // the copies stopped early; still release the consumers
    return;
  }

  // Rotated query rows of this KV head's group.  f16/bf16: split hi/lo, row
  // g the high part of head g, row g+8 the remainder.  Q8_0: int8 fragments
  // (q8_frag_byte) and the per-head factor that turns the integer dot
  // products back into scores.
  const size_t qrow0 = (static_cast<size_t>(job) * a.hq + kvh * gsize) * HD;
  uint32_t* qfrag = reinterpret_cast<uint32_t*>(qs);                  // Q8_0: [HD/32][32][4]
  float* qfac = reinterpret_cast<float*>(qfrag + (HD / 32) * 32 * 4);  // Q8_0: [8]
  if constexpr (Q8) {
    static_assert(KG == 1 && NCT == 128 && (HD / 2) % 32 == 0, "Q8_0 q staging layout");
    constexpr int kIt = 8 * (HD / 2) / NCT;  // pairs per thread; a warp stays inside one head
    float* qmax = qfac + 8;                   // [8 heads][HD / 64 warps]
    float y[kIt][2];
    float2 xq[kIt];
    load_q_pairs<kIt, NCT, HD, IO, GRP>(a, qrow0, threadIdx.x, xq);
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int idx = threadIdx.x + it * NCT, hg = idx / (HD / 2), p = idx % (HD / 2);
      y[it][0] = y[it][1] = 0.f;
      if (hg < gsize) rope_pair(xq[it].x, xq[it].y, rope_cs<DEVROPE>(rsrc, p, HD), y[it][0], y[it][1]);
      float mx = fmaxf(fabsf(y[it][0]), fabsf(y[it][1]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) qmax[hg * (HD / 64) + p / 32] = mx;
    }
    bar_consumers<NCT>();
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int idx = threadIdx.x + it * NCT, hg = idx / (HD / 2), p = idx % (HD / 2);
      float mx = 0.f;
#pragma unroll
      for (int w = 0; w < HD / 64; ++w) mx = fmaxf(mx, qmax[hg * (HD / 64) + w]);
      const float inv = mx > 0.f ? 127.f / mx : 0.f;
      uint32_t hi2 = 0, lo2 = 0;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float u = y[it][e] * inv;  // |u| <= 127
        const int h = __float2int_rn(u);
        const int l = __float2int_rn((u - static_cast<float>(h)) * 254.f);  // |l| <= 127
        hi2 |= (static_cast<uint32_t>(h) & 0xffu) << (8 * e);
        lo2 |= (static_cast<uint32_t>(l) & 0xffu) << (8 * e);
      }
      uint8_t* fb = reinterpret_cast<uint8_t*>(qfrag);
      *reinterpret_cast<uint16_t*>(fb + q8_frag_byte(hg, 2 * p, false)) = static_cast<uint16_t>(hi2);
      *reinterpret_cast<uint16_t*>(fb + q8_frag_byte(hg, 2 * p, true)) = static_cast<uint16_t>(lo2);
      if (p == 0) qfac[hg] = mx * (1.f / (127.f * 254.f));
    }
  } else {
    constexpr int kQIt = (8 * (HD / 2) + NCT - 1) / NCT;
    float2 xq[kQIt];
    load_q_pairs<kQIt, NCT, HD, IO, GRP>(a, qrow0, threadIdx.x, xq);
#pragma unroll
    for (int it = 0; it < kQIt; ++it) {
      const int idx = threadIdx.x + it * NCT, hg = idx / (HD / 2), p = idx % (HD / 2);
      if (idx >= 8 * (HD / 2)) break;
      float y0 = 0.f, y1 = 0.f;
      if (hg < gsize) rope_pair(xq[it].x, xq[it].y, rope_cs<DEVROPE>(rsrc, p, HD), y0, y1);
      float h0, l0, h1, l1;
      split16<BF>(y0, h0, l0);
      split16<BF>(y1, h1, l1);
      const uint32_t hh = pack2<BF>(h0, h1), ll = pack2<BF>(l0, l1);
      qs[hg * C::kQLd + 2 * p] = static_cast<uint16_t>(hh & 0xffff);
      qs[hg * C::kQLd + 2 * p + 1] = static_cast<uint16_t>(hh >> 16);
      qs[(hg + 8) * C::kQLd + 2 * p] = static_cast<uint16_t>(ll & 0xffff);
      qs[(hg + 8) * C::kQLd + 2 * p + 1] = static_cast<uint16_t>(ll >> 16);
    }
  }
  bar_consumers<NCT>();

  // ----------------------------------------------------------- consumers --
  // A fragments of q (f16/bf16): k-step ks starts 32 bytes after k-step
  // ks-1, all of them held in registers.  Q8_0 reloads its int8 fragments
  // from shared memory, one 16-byte load per block.
  const uint32_t qaddr =
      smem_u32(qs + (((lane >> 3) & 1) * 8 + (lane & 7)) * C::kQLd + (lane >> 4) * 8);
  uint32_t qa[Q8 ? 1 : NKS][4];
  if constexpr (!Q8) {
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks)
      ldmatrix_x4(qaddr + ks * 32, qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }

  float o[NO][4];
#pragma unroll
  for (int j = 0; j < NO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m = -CUDART_INF_F, l = 0.f;
  const float sl2 = a.scale * kLog2e;
  // Q8_0 scores come out of the integer MMAs in units of this head's q scale / 254
  const float sl2q = Q8 ? sl2 * qfac[g] : sl2;

  for (int i = grp; i < my_tiles; i += KG) {  // the group's tiles of this split
    const int st = i % C::kStages;
    const bool ok = mbar_wait(&full[st], (i / C::kStages) & 1, a.status);
    if (__any_sync(0xffffffffu, !ok)) break;
    uint8_t* sb = stages + st * C::kStageBytes;
    const int valid = L - (tile0 + i) * kTile - 16 * slice;  // live positions in my slice
    if (valid > 0) {
      if (valid < 16) {
        // Rows past the sequence end hold stale data; zero their V so that
        // 0 * stale never reaches the accumulators.
        if constexpr (Q8) {
          uint16_t* vsc = reinterpret_cast<uint16_t*>(sb + 2 * C::kKBytes + C::kScaleBytes);
          for (int r = valid + lane / (HD / 32); r < 16; r += 32 / (HD / 32))
            vsc[(16 * slice + r) * (HD / 32) + lane % (HD / 32)] = 0;
        } else {
          for (int idx = lane; idx < (16 - valid) * (HD / 8); idx += 32) {
            const int r = 16 * slice + valid + idx / (HD / 8), c = idx % (HD / 8);
            *reinterpret_cast<uint4*>(sb + C::kKBytes + (c >> 3) * 8192 + swz128(r, c & 7)) =
                make_uint4(0, 0, 0, 0);
          }
        }
        __syncwarp();
      }
      if (appends && i == my_tiles - 1 && (qpos - (tile0 + i) * kTile) / 16 == slice) {
        // This slice holds the new token: its row in the tile may be older
        // than the append, so it is copied in from the fused append's
        // shared-memory row (the same bytes the cache now holds).
        const int rt = qpos - (tile0 + i) * kTile;
        if (mbar_wait(appended, 0, a.status)) {
          if constexpr (Q8) {
            if (lane < 8) {
              *reinterpret_cast<uint4*>(sb + swz128(rt, lane)) =
                  reinterpret_cast<const uint4*>(newrow)[lane];
              *reinterpret_cast<uint4*>(sb + C::kKBytes + swz128(rt, lane)) =
                  reinterpret_cast<const uint4*>(newrow + HD)[lane];
            } else if (lane < 8 + HD / 32) {
              const int j = lane - 8;
              const uint16_t* ss = reinterpret_cast<const uint16_t*>(newrow + 2 * HD);
              reinterpret_cast<uint16_t*>(sb + 2 * C::kKBytes)[rt * (HD / 32) + j] = ss[j];
              reinterpret_cast<uint16_t*>(sb + 2 * C::kKBytes + C::kScaleBytes)[rt * (HD / 32) + j] =
                  ss[HD / 32 + j];
            }
          } else if (lane < HD / 8) {  // 16-byte chunk `lane`: box lane/8, chunk lane%8
            const uint32_t off = (lane >> 3) * 8192 + swz128(rt, lane & 7);
            *reinterpret_cast<uint4*>(sb + off) = reinterpret_cast<const uint4*>(newrow)[lane];
            *reinterpret_cast<uint4*>(sb + C::kKBytes + off) =
                reinterpret_cast<const uint4*>(newrow + 2 * HD)[lane];
          }
        }
        __syncwarp();
      }
      // ---- S = Q K^T over this warp's 16 positions (two n-tiles of 8)
      float x[4];  // head g at positions 2tq, 2tq+1, 8+2tq, 9+2tq
      if constexpr (Q8) {
        // One integer MMA per block and n-tile; 254 * hi + lo rows give the
        // block's dot product, scaled by the positions' K scales.
        const uint16_t* ksc = reinterpret_cast<const uint16_t*>(sb + 2 * C::kKBytes);
        uint2 sc[2][2];  // [n-tile][position]: the HD/32 block scales of one row
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e)
            sc[nt][e] = *reinterpret_cast<const uint2*>(ksc + (16 * slice + 8 * nt + 2 * tq + e) *
                                                                  (HD / 32));
        x[0] = x[1] = x[2] = x[3] = 0.f;
#pragma unroll
        for (int blk = 0; blk < HD / 32; ++blk) {
          const uint4 qf = *reinterpret_cast<const uint4*>(qfrag + (blk * 32 + lane) * 4);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int r = 16 * slice + 8 * nt + g;
            const int byte = 32 * blk + 8 * tq;
            const uint2 kb = *reinterpret_cast<const uint2*>(sb + swz128(r, byte >> 4) + (byte & 15));
            int c[4] = {0, 0, 0, 0};
            mma16832_s8(c, qf, kb.x, kb.y);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const uint32_t w = blk < 2 ? sc[nt][e].x : sc[nt][e].y;
              const float d = __half2float(__ushort_as_half(
                  static_cast<uint16_t>((blk & 1) ? (w >> 16) : (w & 0xffffu))));
              x[2 * nt + e] = fmaf(static_cast<float>(c[e] * 254 + c[e + 2]), d, x[2 * nt + e]);
            }
          }
        }
      } else {
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const uint32_t kbase = smem_u32(sb);
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
          const int r = 16 * slice + (lane >> 4) * 8 + (lane & 7);
          const int c = 2 * ks + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kbase + (c >> 3) * 8192 + swz128(r, c & 7), b0, b1, b2, b3);
          mma16816<BF>(s[0], qa[ks], b0, b1);
          mma16816<BF>(s[1], qa[ks], b2, b3);
        }
        // rows g and g+8 hold the high and low parts of head g
        x[0] = s[0][0] + s[0][2];
        x[1] = s[0][1] + s[0][3];
        x[2] = s[1][0] + s[1][2];
        x[3] = s[1][1] + s[1][3];
      }
      // ---- online softmax for head g over positions 2tq, 2tq+1, 8+2tq, 9+2tq
      const int pp[4] = {2 * tq, 2 * tq + 1, 8 + 2 * tq, 9 + 2 * tq};
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x[e] = pp[e] < valid ? x[e] * sl2q : -CUDART_INF_F;
        mx = fmaxf(mx, x[e]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      // The reference maximum moves only when the tile's maximum exceeds it
      // by more than 2^kLazyLog2, so P stays below 2^kLazyLog2 and (m, l, O)
      // stay consistent; the rescale of O then happens a few times per split
      // instead of whenever one of the eight heads sees a new maximum.
      const bool bump = mx > m + kLazyLog2;  // always taken while m is -inf and mx is not
      const float corr = bump ? exp2f(m - mx) : 1.f;  // 0 when m was -inf
      if (bump) m = mx;
      const float base = m == -CUDART_INF_F ? 0.f : m;
      float p[4], psum = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[e] = exp2f(x[e] - base);
        psum += p[e];
      }
      l = l * corr + psum;
      if (__any_sync(0xffffffffu, bump)) {
#pragma unroll
        for (int j = 0; j < NO; ++j) {
          o[j][0] *= corr;
          o[j][1] *= corr;
          o[j][2] *= corr;
          o[j][3] *= corr;
        }
      }
      // P as the A operand: row g = high part, row g+8 = remainder.
      constexpr bool PBF = BF;  // Q8_0 dequantises V to f16
      float ph[4], pl[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) split16<PBF>(p[e], ph[e], pl[e]);
      const uint32_t pa[4] = {pack2<PBF>(ph[0], ph[1]), pack2<PBF>(pl[0], pl[1]),
                              pack2<PBF>(ph[2], ph[3]), pack2<PBF>(pl[2], pl[3])};
      // ---- O += P V
      if constexpr (Q8) {
        const uint8_t* vq = sb + C::kKBytes;
        const uint16_t* vsc =
            reinterpret_cast<const uint16_t*>(sb + 2 * C::kKBytes + C::kScaleBytes);
        const int rA = 16 * slice + 2 * tq;
        const uint4 A = *reinterpret_cast<const uint4*>(vq + swz128(rA, g));
        const uint4 B = *reinterpret_cast<const uint4*>(vq + swz128(rA + 1, g));
        const uint4 Cq = *reinterpret_cast<const uint4*>(vq + swz128(rA + 8, g));
        const uint4 D = *reinterpret_cast<const uint4*>(vq + swz128(rA + 9, g));
        const int sbk = g >> 1;  // this thread's 16 columns lie in Q8_0 block g/2
        const __half2 dAB = __halves2half2(__ushort_as_half(vsc[rA * (HD / 32) + sbk]),
                                           __ushort_as_half(vsc[(rA + 1) * (HD / 32) + sbk]));
        const __half2 dCD = __halves2half2(__ushort_as_half(vsc[(rA + 8) * (HD / 32) + sbk]),
                                           __ushort_as_half(vsc[(rA + 9) * (HD / 32) + sbk]));
        const uint32_t aw[4] = {A.x, A.y, A.z, A.w}, bw[4] = {B.x, B.y, B.z, B.w};
        const uint32_t cw[4] = {Cq.x, Cq.y, Cq.z, Cq.w}, dw[4] = {D.x, D.y, D.z, D.w};
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) {
          uint32_t ab01, ab23, cd01, cd23;
          asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(ab01) : "r"(aw[w4]), "r"(bw[w4]));
          asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(ab23) : "r"(aw[w4]), "r"(bw[w4]));
          asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(cd01) : "r"(cw[w4]), "r"(dw[w4]));
          asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(cd23) : "r"(cw[w4]), "r"(dw[w4]));
          uint32_t x0, x1, x2, x3, y0, y1, y2, y3;
          i8x4_to_h2x2(ab01, x0, x1);
          i8x4_to_h2x2(ab23, x2, x3);
          i8x4_to_h2x2(cd01, y0, y1);
          i8x4_to_h2x2(cd23, y2, y3);
          const uint32_t xs[4] = {x0, x1, x2, x3}, ys[4] = {y0, y1, y2, y3};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __half2 bx = __hmul2(*reinterpret_cast<const __half2*>(&xs[e]), dAB);
            __half2 by = __hmul2(*reinterpret_cast<const __half2*>(&ys[e]), dCD);
            mma16816<false>(o[4 * w4 + e], pa, *reinterpret_cast<uint32_t*>(&bx),
                            *reinterpret_cast<uint32_t*>(&by));
          }
        }
      } else {
        const uint32_t vbase = smem_u32(sb + C::kKBytes);
#pragma unroll
        for (int jj = 0; jj < HD / 16; ++jj) {
          const int r = 16 * slice + ((lane >> 3) & 1) * 8 + (lane & 7);
          const int c = 2 * jj + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(vbase + (c >> 3) * 8192 + swz128(r, c & 7), b0, b1, b2, b3);
          mma16816<BF>(o[2 * jj], pa, b0, b1);
          mma16816<BF>(o[2 * jj + 1], pa, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  // ------------------------------------------------------------- epilogue --
  // Each warp leaves its (max, sum) per head and its raw O rows; weights
  // exp2(m_w - M) / L per (warp, head) are formed once; each output row is
  // then a weighted sum over the warps, four columns per thread.
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  bar_consumers<NCT>();  // every consumer is done reading the stages
  float* ob = reinterpret_cast<float*>(stages);  // [NCW warps][8 heads][HD]
  if (tq == 0) {
    ml[(warp * 8 + g) * 2] = m;
    ml[(warp * 8 + g) * 2 + 1] = l;
  }
#pragma unroll
  for (int j = 0; j < NO; ++j) {
    // Q8_0 columns were permuted: n-tile j, column n -> head-dim 16n + j.
    const int c0 = Q8 ? 16 * (2 * tq) + j : 8 * j + 2 * tq;
    const int c1 = Q8 ? 16 * (2 * tq + 1) + j : 8 * j + 2 * tq + 1;
    ob[(warp * 8 + g) * HD + c0] = o[j][0] + o[j][2];
    ob[(warp * 8 + g) * HD + c1] = o[j][1] + o[j][3];
  }
  bar_consumers<NCT>();
  const int tid = threadIdx.x;
  const size_t pslot = (static_cast<size_t>(job) * hkv + kvh) * a.max_splits;
  // Cluster mode: every split but rank 0 sends its rows and (max, sum) per
  // head straight from the merge below into rank 0's shared memory, by
  // asynchronous remote stores that count their bytes on rank 0's mbarrier.
  const bool sender = cl && split != 0;
  uint32_t rbar = 0, drow = 0, dml = 0;
  if (sender) {
    cluster_wait();  // rank 0's mbarrier is initialised
    rbar = mapa_shared(smem_u32(gbar), 0);
    drow = mapa_shared(smem_u32(grows + split * 8 * HD), 0);
    dml = mapa_shared(smem_u32(gml + split * 16), 0);
  }
  // Each thread forms its head's weights itself (a few exponentials, no
  // serial step and no barrier) and sums four columns over the warps.
  for (int c = tid; c < gsize * (HD / 4); c += NCT) {
    const int hg = c / (HD / 4), d0 = (c % (HD / 4)) * 4;
    float M = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < NCW; ++w) M = fmaxf(M, ml[(w * 8 + hg) * 2]);
    const float Mb = M == -CUDART_INF_F ? 0.f : M;
    float Lh = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < NCW; ++w) {
      const float e = exp2f(ml[(w * 8 + hg) * 2] - Mb);
      Lh = fmaf(ml[(w * 8 + hg) * 2 + 1], e, Lh);
      const float4 v = *reinterpret_cast<const float4*>(ob + (w * 8 + hg) * HD + d0);
      acc.x = fmaf(v.x, e, acc.x);
      acc.y = fmaf(v.y, e, acc.y);
      acc.z = fmaf(v.z, e, acc.z);
      acc.w = fmaf(v.w, e, acc.w);
    }
    const float inv = Lh > 0.f ? 1.f / Lh : 0.f;
    acc.x *= inv;
    acc.y *= inv;
    acc.z *= inv;
    acc.w *= inv;
    if (sender) {
      st_async_v4(drow + 4 * (hg * HD + d0), acc, rbar);
      if (d0 == 0) st_async_v2(dml + 8 * hg, make_float2(M, Lh), rbar);
    } else if (nsplit == 1 || cl) {
      *reinterpret_cast<float4*>(res + hg * HD + d0) = acc;
      if (d0 == 0) {
        cml[2 * hg] = M;
        cml[2 * hg + 1] = Lh;
      }
    } else {
      *reinterpret_cast<float4*>(a.part_o + ((pslot + split) * 8 + hg) * HD + d0) = acc;
      if (d0 == 0) {
        a.part_ml[((pslot + split) * 8 + hg) * 2] = M;
        a.part_ml[((pslot + split) * 8 + hg) * 2 + 1] = Lh;
      }
    }
  }
  if (cl) {
    if (sender) {
      if (PEER && tid == 0 && a.peer.nranks) peer_arrive(a.peer, peer_epoch(a.peer), a.status);
      return;
    }
    // Rank 0 expects the bytes of every live split but itself (rows and
    // (max, sum) of the group's heads); once they have landed (bounded wait,
    // acquire at cluster scope) it merges the live splits by LSE weight, each
    // thread forming its head's weights, and stores its four columns.
    const uint32_t push_bytes = gsize * (HD * 4 + 8);
    bar_consumers<NCT>();  // its own res and cml are complete
    if (tid == 0) mbar_arrive_expect_tx(gbar, (nsplit - 1) * push_bytes);
    mbar_wait_cluster(gbar, 0, a.status);
    // A single GPU's output is stored from registers; a head-sharded call's
    // goes through emit_rows, which writes every rank's buffer in protocol.
    const bool direct = !PEER || a.peer.nranks == 0;
    // The LSE weights once per (split, head), not once per output column:
    // thread t takes split t / 8 and head t % 8 (NCT = 128 covers 16 splits
    // x 8 heads); each head's maximum and denominator are reduced over the
    // splits a warp holds by shuffles, then over the four warps through
    // shared memory (the stages are free by now).  Each thread then sums its
    // four columns over the live splits with those weights.
    // (Clusters run with one group of four consumer warps only: KG == 1.)
    static_assert(KG > 1 || (NCT == 128 && C::kMaxCluster <= 16), "one thread per (split, head)");
    float* mw = cml + 16;      // [16 splits][8 heads] weights
    float* mh = mw + 16 * 8;   // [2][4 warps][8 heads]: maxima, then denominators
    if constexpr (KG == 1) {
      const int r = tid >> 3, hg = tid & 7, cw = tid >> 5;
      const bool live = r < nsplit && hg < gsize;
      const float m_r = live ? (r == 0 ? cml[2 * hg] : gml[r * 16 + 2 * hg]) : -CUDART_INF_F;
      const float l_r = live ? (r == 0 ? cml[2 * hg + 1] : gml[r * 16 + 2 * hg + 1]) : 0.f;
      float M = fmaxf(m_r, __shfl_xor_sync(0xffffffffu, m_r, 8));
      M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
      if (lane < 8) mh[cw * 8 + lane] = M;
      bar_consumers<NCT>();
      M = fmaxf(fmaxf(mh[hg], mh[8 + hg]), fmaxf(mh[16 + hg], mh[24 + hg]));
      const float w = live ? l_r * exp2f(m_r - (M == -CUDART_INF_F ? 0.f : M)) : 0.f;
      mw[r * 8 + hg] = w;
      float den = w + __shfl_xor_sync(0xffffffffu, w, 8);
      den += __shfl_xor_sync(0xffffffffu, den, 16);
      if (lane < 8) mh[32 + cw * 8 + lane] = den;
      bar_consumers<NCT>();
    }
    auto merge = [&](auto width) {
      constexpr int N = decltype(width)::value;
      for (int c = tid; c < gsize * (HD / 4); c += NCT) {
        const int hg = c / (HD / 4), d0 = (c % (HD / 4)) * 4;
        const float den = (mh[32 + hg] + mh[40 + hg]) + (mh[48 + hg] + mh[56 + hg]);
        // two accumulators halve the dependent chain of multiply-adds
        float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll
        for (int r = 0; r < N; ++r) {
          if (r >= nsplit) break;
          const float w = mw[r * 8 + hg];
          const float4 v = r == 0 ? *reinterpret_cast<const float4*>(res + hg * HD + d0)
                                  : *reinterpret_cast<const float4*>(grows + (r * 8 + hg) * HD + d0);
          float4& o = acc[r & 1];
          o.x = fmaf(v.x, w, o.x);
          o.y = fmaf(v.y, w, o.y);
          o.z = fmaf(v.z, w, o.z);
          o.w = fmaf(v.w, w, o.w);
        }
        const float inv = den > 0.f ? 1.f / den : 0.f;
        const float4 out = make_float4((acc[0].x + acc[1].x) * inv, (acc[0].y + acc[1].y) * inv,
                                       (acc[0].z + acc[1].z) * inv, (acc[0].w + acc[1].w) * inv);
        if (direct)
          store4(a.out, (static_cast<size_t>(job) * a.hq + kvh * gsize + hg) * HD + d0,
                 IO >= 0 ? IO : a.out_dtype, out, a.out_vec != 0);
        else
          *reinterpret_cast<float4*>(res + hg * HD + d0) = out;
      }
    };
    if (C::kMaxCluster > 8 && nsplit > 8)
      merge(std::integral_constant<int, (C::kMaxCluster > 8 ? C::kMaxCluster : 8)>{});
    else
      merge(std::integral_constant<int, 8>{});
    if (!direct) {
      bar_consumers<NCT>();
      emit_rows<HD, NCT, PEER, IO, GRP>(a, res, job, kvh, tid, flag);
    }
    return;
  }
  if (nsplit == 1) {
    bar_consumers<NCT>();
    emit_rows<HD, NCT, PEER, IO, GRP>(a, res, job, kvh, tid, flag);
    return;
  }
  // ---- the last CTA of this (job, kv head) merges the splits
  // The barrier orders every thread's partial rows before thread 0's count,
  // whose release makes them visible at GPU scope; its acquire makes the
  // other splits' rows visible to the last CTA, whose threads the second
  // barrier orders after it.
  bar_consumers<NCT>();
  if (tid == 0) {
    const int prev = atom_add_acq_rel_gpu(&a.counters[static_cast<size_t>(job) * hkv + kvh], 1);
    flag[0] = prev == nsplit - 1;
  }
  bar_consumers<NCT>();
  if (!flag[0]) {
    if (PEER && a.peer.nranks && tid == 0) peer_arrive(a.peer, peer_epoch(a.peer), a.status);
    return;
  }
  // Each thread sums four output columns over the splits with a running
  // maximum, loading kU splits' (max, sum) and rows at a time: one round
  // trip to L2 per kU splits.
  for (int c = tid; c < gsize * (HD / 4); c += NCT) {
    const int hg = c / (HD / 4), d0 = (c % (HD / 4)) * 4;
    const float4* po = reinterpret_cast<const float4*>(a.part_o + (pslot * 8 + hg) * HD + d0);
    const float2* pm = reinterpret_cast<const float2*>(a.part_ml + (pslot * 8 + hg) * 2);
    constexpr int kStride = 8 * HD / 4;  // float4s from one split's rows to the next's
    constexpr int kU = KG > 2 ? 4 : 16;  // the four-group variant has 96 registers
    float M = -CUDART_INF_F, den = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < nsplit; s0 += kU) {
      float4 v[kU];
      float2 ml[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const bool live = s0 + u < nsplit;
        v[u] = live ? __ldcg(po + static_cast<size_t>(s0 + u) * kStride)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
        ml[u] = live ? __ldcg(pm + static_cast<size_t>(s0 + u) * 8) : make_float2(-CUDART_INF_F, 0.f);
      }
      float cm = M;
#pragma unroll
      for (int u = 0; u < kU; ++u) cm = fmaxf(cm, ml[u].x);
      const float cb = cm == -CUDART_INF_F ? 0.f : cm;
      const float r = M == -CUDART_INF_F ? 0.f : exp2f(M - cb);  // rescale what came before
      acc.x *= r;
      acc.y *= r;
      acc.z *= r;
      acc.w *= r;
      den *= r;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const float w = ml[u].y * exp2f(ml[u].x - cb);  // 0 past the live splits
        den += w;
        acc.x = fmaf(v[u].x, w, acc.x);
        acc.y = fmaf(v[u].y, w, acc.y);
        acc.z = fmaf(v[u].z, w, acc.z);
        acc.w = fmaf(v[u].w, w, acc.w);
      }
      M = cm;
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    *reinterpret_cast<float4*>(res + hg * HD + d0) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
  if (tid == 0) a.counters[static_cast<size_t>(job) * hkv + kvh] = 0;
  bar_consumers<NCT>();
  emit_rows<HD, NCT, PEER, IO, GRP>(a, res, job, kvh, tid, flag);
}

// ------------------------------------------------ head-sharded exchange --
// Copies this rank's compact output rows into every rank's symmetric output
// (PeerOut protocol); used when the attention itself could not store there.
__global__ void __launch_bounds__(256)
    peer_push_kernel(const uint8_t* src, int64_t rows, int row_bytes, int head_bytes,
                     const __grid_constant__ PeerOut po, uint32_t* status) {
  __shared__ int go;
  const uint32_t e = peer_epoch(po);
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) peer_enter(po, e);
    go = peer_wait_entered(po, e, status);
  }
  __syncthreads();
  if (go) {
    const int64_t row_stride = static_cast<int64_t>(po.hq_total) * head_bytes;
    const int64_t dst0 = static_cast<int64_t>(po.head_base) * head_bytes;
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    if (row_bytes % 16 == 0 && row_stride % 16 == 0 && dst0 % 16 == 0) {
      const int per_row = row_bytes / 16;
      for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
           i < rows * per_row; i += step) {
        const int64_t r = i / per_row, c = i % per_row;
        const uint4 v = *reinterpret_cast<const uint4*>(src + r * row_bytes + c * 16);
        for (int p = 0; p < po.nranks; ++p)
          *reinterpret_cast<uint4*>(static_cast<uint8_t*>(po.out[p]) + r * row_stride + dst0 +
                                    c * 16) = v;
      }
    } else {
      const int per_row = row_bytes / 4;
      for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
           i < rows * per_row; i += step) {
        const int64_t r = i / per_row, c = i % per_row;
        const uint32_t v = *reinterpret_cast<const uint32_t*>(src + r * row_bytes + c * 4);
        for (int p = 0; p < po.nranks; ++p)
          *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(po.out[p]) + r * row_stride + dst0 +
                                       c * 4) = v;
      }
    }
  }
  __syncthreads();  // thread 0's release in peer_arrive then covers every thread's stores
  if (threadIdx.x == 0) peer_arrive(po, e, status);
}

cudaError_t launch_peer_push(const void* src, int64_t rows, int row_bytes, int head_bytes,
                             PeerOut po, int num_sms, uint32_t* status, cudaStream_t s) {
  const int64_t units = rows * (row_bytes / 4);
  const int blocks = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>((units + 255) / 256, 2LL * std::max(num_sms, 1))));
  po.total_ctas = blocks;
  peer_push_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(src), rows, row_bytes,
                                          head_bytes, po, status);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(256)
    rank_to_head_major_kernel(const uint32_t* src, uint32_t* dst, int nranks, int64_t rows,
                              int row_words) {
  const int64_t total = static_cast<int64_t>(nranks) * rows * row_words;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = i % row_words, r = (i / row_words) % rows, k = i / (row_words * rows);
    dst[(r * nranks + k) * row_words + c] = src[i];
  }
}

cudaError_t launch_rank_to_head_major(const void* src, void* dst, int nranks, int64_t rows,
                                      int row_bytes, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(nranks) * rows * (row_bytes / 4);
  if (total == 0) return cudaSuccess;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  rank_to_head_major_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint32_t*>(src),
                                                   static_cast<uint32_t*>(dst), nranks, rows,
                                                   row_bytes / 4);
  return cudaGetLastError();
}

size_t splitkv_smem_bytes(int hd, int dtype) {  // the KG == 1 variant
  if (dtype == kQ8_0) return SplitCfg<128, kQ8_0>::kSmem;
  if (hd == 128) return dtype == kBF16 ? SplitCfg<128, kBF16>::kSmem : SplitCfg<128, kF16>::kSmem;
  return dtype == kBF16 ? SplitCfg<64, kBF16>::kSmem : SplitCfg<64, kF16>::kSmem;
}

bool splitkv_supported(int hd, int dtype, int group, int page) {
  if (group < 1 || group > 8 || page % kTile != 0) return false;
  if (dtype == kQ8_0) return hd == 128;
  return (dtype == kF16 || dtype == kBF16) && (hd == 64 || hd == 128);
}

using SplitKvFn = void (*)(const AttnArgs, const CUtensorMap, const CUtensorMap, int);

// The compiled form for a launch: clustered or not, head-sharded or not, and
// (single-GPU calls with the table's RoPE) I/O of the cache's own 16-bit type,
// then also eight query heads per KV head when the call has that.
template <int HD, int DT, bool DEVROPE, int KG>
static SplitKvFn splitkv_form(bool clustered, bool peer, bool io, bool g8) {
  constexpr int kIO = DT == kQ8_0 ? -1 : DT;
  if constexpr (KG == 1) {
    if (clustered) {
      if (peer) return splitkv_kernel<HD, DT, DEVROPE, KG, true, true, -1, 0>;
      if (io && !DEVROPE)
        return g8 ? splitkv_kernel<HD, DT, DEVROPE, KG, true, false, kIO, 8>
                  : splitkv_kernel<HD, DT, DEVROPE, KG, true, false, kIO, 0>;
      return splitkv_kernel<HD, DT, DEVROPE, KG, true, false, -1, 0>;
    }
  }
  if (peer) return splitkv_kernel<HD, DT, DEVROPE, KG, false, true, -1, 0>;
  if (io && !DEVROPE)
    return g8 ? splitkv_kernel<HD, DT, DEVROPE, KG, false, false, kIO, 8>
              : splitkv_kernel<HD, DT, DEVROPE, KG, false, false, kIO, 0>;
  return splitkv_kernel<HD, DT, DEVROPE, KG, false, false, -1, 0>;
}

// Sets every form's shared-memory limit on the current device (once per
// device) and reports how many of the kernel's CTAs an SM holds.
template <int HD, int DT, bool DEVROPE, int KG>
static cudaError_t configure_splitkv_t(int* ctas_per_sm) {
  using C = SplitCfg<HD, DT, KG>;
  constexpr int kMaxDev = 64;
  static std::atomic<int> occupancy[kMaxDev];  // 0 = not configured yet
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < kMaxDev && occupancy[dev].load(std::memory_order_acquire) > 0) {
    if (ctas_per_sm) *ctas_per_sm = occupancy[dev].load(std::memory_order_relaxed);
    return cudaSuccess;
  }
  // every compiled form: shared memory (clustered forms add the gather area)
  // and, for clusters above 8 CTAs, the non-portable size
  for (int form = 0; form < 16 && e == cudaSuccess; ++form) {
    const bool clustered = form & 1, peer = form & 2, io = form & 4, g8 = form & 8;
    if (clustered && KG != 1) continue;
    SplitKvFn k = splitkv_form<HD, DT, DEVROPE, KG>(clustered, peer, io, g8);
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(clustered ? C::kSmemCluster : C::kSmem));
    if (e == cudaSuccess && clustered && C::kMaxCluster > 8)
      e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  }
  if (e != cudaSuccess) return e;
  int n = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &n, splitkv_form<HD, DT, DEVROPE, KG>(false, false, false, false), C::kThreads, C::kSmem);
  if (e != cudaSuccess) return e;
  n = max(n, 1);
  if (dev < kMaxDev) occupancy[dev].store(n, std::memory_order_release);
  if (ctas_per_sm) *ctas_per_sm = n;
  return cudaSuccess;
}

template <int HD, int DT, bool DEVROPE, int KG>
static cudaError_t launch_splitkv_t(const AttnArgs& a, const CUtensorMap* kmap,
                                    const CUtensorMap* vmap, int jobs, cudaStream_t s, bool pdl) {
  using C = SplitCfg<HD, DT, KG>;
  cudaError_t e = configure_splitkv_t<HD, DT, DEVROPE, KG>(nullptr);
  if (e != cudaSuccess) return e;
  const bool io = DT != kQ8_0 && a.in_dtype == DT && a.out_dtype == DT;
  const SplitKvFn kernel = splitkv_form<HD, DT, DEVROPE, KG>(KG == 1 && a.cluster > 1,
                                                             a.peer.nranks > 0, io, a.group == 8);
  for (int j0 = 0; j0 < jobs; j0 += 65535) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.max_splits, a.cache.hkv, min(65535, jobs - j0));
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = a.cluster > 1 ? C::smem_cluster(a.cluster) : C::kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
      attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[na].val.programmaticStreamSerializationAllowed = 1;
      ++na;
    }
    if (a.cluster > 1) {  // the splits of one job as one cluster (grid x == cluster size)
      attr[na].id = cudaLaunchAttributeClusterDimension;
      attr[na].val.clusterDim.x = a.cluster;
      attr[na].val.clusterDim.y = 1;
      attr[na].val.clusterDim.z = 1;
      ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    e = cudaLaunchKernelEx(&cfg, kernel, a, *kmap, *vmap, j0);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Consumer groups of the wide (latency) variant for a configuration, 0 if it
// has none: four at head_dim 64, two at 128 (the register file bounds it).
constexpr int wide_groups(int hd, int dt) {
  return dt == kQ8_0 ? 0 : (hd == 64 ? 4 : (hd == 128 ? 2 : 0));
}

template <bool DEVROPE>
static cudaError_t dispatch_splitkv(const AttnArgs& a, const CUtensorMap* kmap,
                                    const CUtensorMap* vmap, int jobs, cudaStream_t s, bool pdl) {
  const int hd = a.cache.hd, dt = a.cache.dtype;
  if constexpr (!DEVROPE) {
    if (a.wide && wide_groups(hd, dt)) {
      if (hd == 128)
        return dt == kBF16 ? launch_splitkv_t<128, kBF16, false, 2>(a, kmap, vmap, jobs, s, pdl)
                           : launch_splitkv_t<128, kF16, false, 2>(a, kmap, vmap, jobs, s, pdl);
      return dt == kBF16 ? launch_splitkv_t<64, kBF16, false, 4>(a, kmap, vmap, jobs, s, pdl)
                         : launch_splitkv_t<64, kF16, false, 4>(a, kmap, vmap, jobs, s, pdl);
    }
  }
  if (dt == kQ8_0) return launch_splitkv_t<128, kQ8_0, DEVROPE, 1>(a, kmap, vmap, jobs, s, pdl);
  if (hd == 128)
    return dt == kBF16 ? launch_splitkv_t<128, kBF16, DEVROPE, 1>(a, kmap, vmap, jobs, s, pdl)
                       : launch_splitkv_t<128, kF16, DEVROPE, 1>(a, kmap, vmap, jobs, s, pdl);
  return dt == kBF16 ? launch_splitkv_t<64, kBF16, DEVROPE, 1>(a, kmap, vmap, jobs, s, pdl)
                     : launch_splitkv_t<64, kF16, DEVROPE, 1>(a, kmap, vmap, jobs, s, pdl);
}

template <bool DEVROPE>
static int ctas_per_sm_t(int hd, int dt) {
  int n = 0;
  cudaError_t e;
  if (dt == kQ8_0)
    e = configure_splitkv_t<128, kQ8_0, DEVROPE, 1>(&n);
  else if (hd == 128)
    e = dt == kBF16 ? configure_splitkv_t<128, kBF16, DEVROPE, 1>(&n)
                    : configure_splitkv_t<128, kF16, DEVROPE, 1>(&n);
  else
    e = dt == kBF16 ? configure_splitkv_t<64, kBF16, DEVROPE, 1>(&n)
                    : configure_splitkv_t<64, kF16, DEVROPE, 1>(&n);
  return e == cudaSuccess ? n : 0;
}

int splitkv_wide_groups(int hd, int dtype) { return wide_groups(hd, dtype); }

int splitkv_ctas_per_sm(int hd, int dtype, bool device_rope) {
  return device_rope ? ctas_per_sm_t<true>(hd, dtype) : ctas_per_sm_t<false>(hd, dtype);
}

cudaError_t launch_splitkv(const AttnArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap,
                           int jobs, cudaStream_t s, bool pdl) {
  return dispatch_splitkv<false>(a, kmap, vmap, jobs, s, pdl);
}

cudaError_t launch_splitkv_device_rope(const AttnArgs& a, const CUtensorMap* kmap,
                                       const CUtensorMap* vmap, int jobs, cudaStream_t s) {
  return dispatch_splitkv<true>(a, kmap, vmap, jobs, s, false);
}

}  // namespace ql
