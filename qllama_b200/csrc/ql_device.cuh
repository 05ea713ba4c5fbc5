// ql_device.cuh -- device helpers shared by the attention kernels (sm_100a).
//
// Inline-PTX wrappers for mbarriers, TMA (tensor and plain bulk copies, never
// with cluster multicast), ldmatrix and the m16n8k16 tensor-core MMA, plus
// element conversions and the f64 RoPE rotation that reproduces the
// reference bit for bit (src/tensor/ops.rs:207-215).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ql {

enum : int { kF32 = 0, kF16 = 1, kBF16 = 2, kQ8_0 = 3 };

// Bits of the context status word that kernels raise instead of trapping.
enum : uint32_t {
  kStatusWaitTimeout = 1u,  // an mbarrier wait ran out of iterations
  kStatusBadPage = 2u,      // a block-table entry pointed outside the pool
  kStatusPeerTimeout = 4u,  // another GPU of a head-sharded call did not signal in time
  kStatusBadLogits = 8u,    // the sampler met a non-finite logit
  kStatusBadToken = 16u,    // a token id read on the device was outside the vocabulary
};

// Time bound for every spin on an mbarrier, in nanoseconds of %globaltimer:
// far above any legitimate wait (a TMA tile lands in microseconds), short
// enough that a copy that never completes ends the kernel in about a second.
constexpr uint64_t kWaitLimitNs = 1000000000ull;
// Bound for waits on another GPU's flags in a head-sharded call: the ranks
// must issue their calls within this many nanoseconds of each other.
constexpr uint64_t kPeerWaitLimitNs = 5000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: returns false (and raises the status bit) if the phase has not
// flipped within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  if (status) atomicOr(status, kStatusWaitTimeout);
  return false;
}

// ------------------------------------------------- thread-block clusters --
// Split arrive/wait of the hardware cluster barrier (every thread of every CTA
// arrives once, right after its mbarriers are initialised; waiting later
// costs nothing), stores into another CTA's shared memory that complete on
// its mbarrier, and a bounded wait that acquires at cluster scope.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait;" ::: "memory");
}
// Address of the same shared-memory location in CTA `cta_rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t cta_rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(cta_rank));
  return r;
}
// Asynchronous 16-byte store into another CTA's shared memory (both
// addresses from mapa_shared) whose completion counts its bytes on that CTA's
// mbarrier; the issuing thread does not wait for it.
__device__ __forceinline__ void st_async_v4(uint32_t remote_addr, const float4& v,
                                            uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::
          "r"(remote_addr),
      "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar)
      : "memory");
}
// The 8-byte form of st_async_v4.
__device__ __forceinline__ void st_async_v2(uint32_t remote_addr, const float2& v,
                                            uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
          remote_addr),
      "f"(v.x), "f"(v.y), "r"(remote_bar)
      : "memory");
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  uint32_t* status) {
  auto try_wait = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_wait()) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (try_wait()) return true;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  if (status) atomicOr(status, kStatusWaitTimeout);
  return false;
}

// Atomic add at GPU scope with acquire and release semantics; returns the
// old value.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(reinterpret_cast<uint64_t>(p)), "r"(v)
               : "memory");
  return old;
}

// ------------------------------------------- programmatic dependent launch --
// Waits until the grids this one depends on have completed and their memory
// is visible (a no-op when the launch carried no programmatic dependency).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next grid in the stream begin launching (its pre-wait part).
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------- TMA --
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// L2 prefetches: a 128-byte line, one box of a tensor map, or a plain range
// (16-byte aligned, a multiple of 16 bytes).  The L2 is the GPU's point of
// coherence, so a line fetched early is updated there by later writes.
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)),
               "r"(bytes)
               : "memory");
}

// 2-D tiled load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Plain (untiled) bulk copy global -> shared; both addresses 16-byte aligned,
// size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------- ldmatrix / mma --
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D(16x8,f32) += A(16x16, row) * B(16x8, col); A/B f16 (BF = false) or bf16.
template <bool BF>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (BF) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// D(16x8,s32) += A(16x32, row) * B(32x8, col), A/B signed 8-bit.  Register
// a0 holds A[g][4t..4t+3], a1 A[g+8][4t..], a2 A[g][16+4t..], a3
// A[g+8][16+4t..]; b0 holds B[4t..4t+3][g], b1 B[16+4t..][g]; d as for
// mma16816 (g = lane / 4, t = lane % 4).
__device__ __forceinline__ void mma16832_s8(int (&d)[4], const uint4& a, uint32_t b0,
                                            uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// -------------------------------------------------------------- elements --
// f16 operand range of a block of values whose largest magnitude has the f32
// bits `bits` (a non-negative value): the power of two 2^e to divide them by.
// e = 0 while that magnitude lies in [2^-10, 2^15) (the values are used as
// they are); otherwise e = floor(log2(magnitude)) - 14, which brings it into
// [2^14, 2^15): below f16's overflow, and with small values kept off f16's
// subnormal range.  Clamped to [-100, 113]; 0 for Inf/NaN (kept as they are).
__device__ __forceinline__ int f16_range_exp(uint32_t bits) {
  if (bits >= 0x7f800000u) return 0;
  const int E = static_cast<int>(bits >> 23) - 127;
  if (E >= -10 && E <= 14) return 0;
  return E - 14 < -100 ? -100 : E - 14;
}
// 2^e as an f32, exactly, for -126 <= e <= 127.
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }

template <bool BF>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <bool BF>
__device__ __forceinline__ float round16(float x) {
  if constexpr (BF) return __bfloat162float(__float2bfloat16_rn(x));
  else return __half2float(__float2half_rn(x));
}

// Splits x into hi + lo, both representable in the 16-bit type, so that two
// MMAs recover about twice the significand of one.
template <bool BF>
__device__ __forceinline__ void split16(float x, float& hi, float& lo) {
  hi = round16<BF>(x);
  lo = x - hi;
}

__device__ __forceinline__ float load_elem(const void* base, size_t i, int dt) {
  if (dt == kF32) return static_cast<const float*>(base)[i];
  if (dt == kF16) return __half2float(static_cast<const __half*>(base)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
}

// Elements i and i+1 (i even) in one access when `vec` says the base pointer
// is aligned to two elements, else one at a time.
__device__ __forceinline__ float2 load_pair(const void* base, size_t i, int dt, bool vec) {
  if (!vec) return make_float2(load_elem(base, i, dt), load_elem(base, i + 1, dt));
  if (dt == kF32) return *reinterpret_cast<const float2*>(static_cast<const float*>(base) + i);
  if (dt == kF16)
    return __half22float2(*reinterpret_cast<const __half2*>(static_cast<const __half*>(base) + i));
  return __bfloat1622float2(
      *reinterpret_cast<const __nv_bfloat162*>(static_cast<const __nv_bfloat16*>(base) + i));
}

__device__ __forceinline__ bool pair_aligned(const void* base, int dt) {
  return (reinterpret_cast<uintptr_t>(base) & (dt == kF32 ? 7u : 3u)) == 0;
}

__device__ __forceinline__ void store_elem(void* base, size_t i, int dt, float x) {
  if (dt == kF32) static_cast<float*>(base)[i] = x;
  else if (dt == kF16) static_cast<__half*>(base)[i] = __float2half_rn(x);
  else static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(x);
}

// Elements i..i+7 (i a multiple of 8) from x[0..8): one 16-byte store for
// f16/bf16, two for f32, when `vec` says the base is 16-byte aligned; else
// element by element.  Rounding is the same either way (to nearest even).
__device__ __forceinline__ void store8(void* base, size_t i, int dt, const float* x, bool vec) {
  if (!vec) {
#pragma unroll
    for (int e = 0; e < 8; ++e) store_elem(base, i + e, dt, x[e]);
    return;
  }
  if (dt == kF32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + i);
    p[0] = make_float4(x[0], x[1], x[2], x[3]);
    p[1] = make_float4(x[4], x[5], x[6], x[7]);
    return;
  }
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    w[e] = dt == kF16 ? pack2<false>(x[2 * e], x[2 * e + 1]) : pack2<true>(x[2 * e], x[2 * e + 1]);
  *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + i) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Four consecutive output elements (i a multiple of 4) in one store when
// `vec` says the base is 16-byte aligned.
__device__ __forceinline__ void store4(void* base, size_t i, int dt, const float4& x, bool vec) {
  if (!vec) {
    store_elem(base, i, dt, x.x);
    store_elem(base, i + 1, dt, x.y);
    store_elem(base, i + 2, dt, x.z);
    store_elem(base, i + 3, dt, x.w);
    return;
  }
  if (dt == kF32) {
    *reinterpret_cast<float4*>(static_cast<float*>(base) + i) = x;
    return;
  }
  const uint32_t w0 = dt == kF16 ? pack2<false>(x.x, x.y) : pack2<true>(x.x, x.y);
  const uint32_t w1 = dt == kF16 ? pack2<false>(x.z, x.w) : pack2<true>(x.z, x.w);
  *reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + i) = make_uint2(w0, w1);
}

// ------------------------------------------- flags shared between GPUs --
// System-scope release store / acquire load, for flags that another GPU
// writes or reads over NVLink.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait until the epoch counter *p reaches `epoch` (wrap-safe); raises
// kStatusPeerTimeout and returns false after kPeerWaitLimitNs.  Once a wait of
// the context has given up (the bit is set until the host reads it), later
// waits return at once, so that a rank that left costs one wait limit, not
// one per remaining call.
__device__ __forceinline__ bool wait_epoch(const uint32_t* p, uint32_t epoch, uint32_t* status) {
  if (static_cast<int32_t>(ld_acquire_sys(p) - epoch) >= 0) return true;
  if (status && (*reinterpret_cast<volatile uint32_t*>(status) & kStatusPeerTimeout)) return false;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 16; ++i) {
      if (static_cast<int32_t>(ld_acquire_sys(p) - epoch) >= 0) return true;
      __nanosleep(64);
    }
    if (global_ns() - t0 > kPeerWaitLimitNs) break;
  }
  if (status) atomicOr(status, kStatusPeerTimeout);
  return false;
}

// int8x4 in one word -> two f16x2 holding (b0,b1) and (b2,b3), exactly.
// Each byte is biased to an unsigned value u = x + 128 placed in the low
// mantissa bits of an f16 with exponent 10 (value 1024 + u); subtracting
// 1152 leaves x.
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t w, uint32_t& h01, uint32_t& h23) {
  uint32_t u = w ^ 0x80808080u;
  uint32_t lo, hi;
  asm("prmt.b32 %0, %1, %2, 0x7170;" : "=r"(lo) : "r"(u), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x7372;" : "=r"(hi) : "r"(u), "r"(0x64646464u));
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  __half2 a = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
  __half2 b = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
  h01 = *reinterpret_cast<uint32_t*>(&a);
  h23 = *reinterpret_cast<uint32_t*>(&b);
}

// ------------------------------------------------------------------ RoPE --
// The reference rotates each adjacent pair in f64 and casts to f32:
//   y0 = (x0*cos - x1*sin) as f32, y1 = (x0*sin + x1*cos) as f32
// (src/tensor/ops.rs:212-215).  The explicit _rn intrinsics keep the
// compiler from contracting the products into FMAs, so the result equals
// the reference's bit for bit given the same f64 cos/sin (taken from a table
// the host builds with the reference's formula).
__device__ __forceinline__ void rope_pair(float x0, float x1, double2 cs, float& y0,
                                          float& y1) {
  double a = __dmul_rn(static_cast<double>(x0), cs.x);
  double b = __dmul_rn(static_cast<double>(x1), cs.y);
  double c = __dmul_rn(static_cast<double>(x0), cs.y);
  double d = __dmul_rn(static_cast<double>(x1), cs.x);
  y0 = __double2float_rn(__dsub_rn(a, b));
  y1 = __double2float_rn(__dadd_rn(c, d));
}

// Q8_0 quantisation of one 32-value block held as 16 pairs by 16 consecutive
// lanes (lane & 15 = pair index within the block).  Same rule as the GGUF
// reference quantiser: d = amax/127, id = 1/d (0 if d == 0), q = round(x*id)
// with ties away from zero, scale stored as f16(d).
__device__ __forceinline__ void q8_0_pair(float x0, float x1, int8_t& q0, int8_t& q1,
                                          __half& scale) {
  float amax = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  float r0 = roundf(x0 * id), r1 = roundf(x1 * id);
  q0 = static_cast<int8_t>(r0 == r0 ? static_cast<int>(r0) : 0);
  q1 = static_cast<int8_t>(r1 == r1 ? static_cast<int>(r1) : 0);
  scale = __float2half_rn(d);
}

}  // namespace ql
