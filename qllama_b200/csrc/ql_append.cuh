// ql_append.cuh -- the cache append shared by the append and prologue kernels:
// block-table lookup, RoPE source and the conversion of one new K/V row into
// the cache's storage type (reference: ops.rs:168-220 rope, cache.rs:146-163
// update writes).
#pragma once

#include "ql_device.cuh"
#include "ql_kernels.cuh"

namespace ql {

__device__ __forceinline__ int64_t cache_row(const CacheView& c, int seq, int pos, int h,
                                             uint32_t* status, bool& ok) {
  int page = c.block_table[static_cast<size_t>(seq) * c.pages_per_seq + pos / c.page];
  if (page < 0 || page >= c.num_pages) {
    ok = false;
    if (status) atomicOr(status, kStatusBadPage);
    return 0;
  }
  ok = true;
  return (static_cast<int64_t>(page) * c.hkv + h) * c.page + pos % c.page;
}

// Source of the RoPE (cos, sin) pairs of one position: the host-built table
// row, or (DEV) f64 pow/sincos evaluated on the device for callers that have
// no table (the no-allocation decode entry point).
struct RopeSrc {
  const double2* row;  // table row of the position, or nullptr for "no rotation"
  double pos;
  double theta;
};

template <bool DEV>
__device__ __forceinline__ double2 rope_cs(const RopeSrc& r, int p, int hd) {
  if constexpr (DEV) {
    const double f = pow(r.theta, -2.0 * static_cast<double>(p) / static_cast<double>(hd));
    double sn, cs;
    sincos(r.pos * f, &sn, &cs);
    return make_double2(cs, sn);
  } else {
    return r.row[p];
  }
}

// One warp writes one cache row (one position of one KV head): K rotated
// by the table row when one is given, V as is, both converted to the cache
// type.
__device__ __forceinline__ void append_row(const void* kin, const void* vin, int in_dt,
                                           size_t in_off, const double2* rope_row,
                                           const CacheView& c, int64_t dst, int lane) {
  const int hd = c.hd;
  const int pairs = hd / 2;
  const RopeSrc rope{rope_row, 0.0, 0.0};
  for (int base = 0; base < pairs; base += 32) {
    const int p = base + lane;
    const bool valid = p < pairs;
    float k0 = 0.f, k1 = 0.f, v0 = 0.f, v1 = 0.f;
    if (valid) {
      k0 = load_elem(kin, in_off + 2 * p, in_dt);
      k1 = load_elem(kin, in_off + 2 * p + 1, in_dt);
      v0 = load_elem(vin, in_off + 2 * p, in_dt);
      v1 = load_elem(vin, in_off + 2 * p + 1, in_dt);
      if (rope_row) rope_pair(k0, k1, rope_cs<false>(rope, p, hd), k0, k1);
    }
    const size_t e = static_cast<size_t>(dst) * hd + 2 * p;
    if (c.dtype == kQ8_0) {
      int8_t qk0, qk1, qv0, qv1;
      __half sk, sv;
      q8_0_pair(k0, k1, qk0, qk1, sk);
      q8_0_pair(v0, v1, qv0, qv1, sv);
      if (valid) {
        *reinterpret_cast<char2*>(static_cast<int8_t*>(c.k) + e) = make_char2(qk0, qk1);
        *reinterpret_cast<char2*>(static_cast<int8_t*>(c.v) + e) = make_char2(qv0, qv1);
        if ((lane & 15) == 0) {
          const size_t si = static_cast<size_t>(dst) * (hd / 32) + (2 * p) / 32;
          c.k_scale[si] = __half_as_ushort(sk);
          c.v_scale[si] = __half_as_ushort(sv);
        }
      }
    } else if (valid) {
      store_elem(c.k, e, c.dtype, k0);
      store_elem(c.k, e + 1, c.dtype, k1);
      store_elem(c.v, e, c.dtype, v0);
      store_elem(c.v, e + 1, c.dtype, v1);
    }
  }
}

// N consecutive input elements (N = 2 or 4, i a multiple of N) as f32, in one
// access when `vec` says the base is aligned to it, else one at a time.
template <int N>
__device__ __forceinline__ void load_vec(const void* base, size_t i, int dt, bool vec,
                                         float (&x)[N]) {
  static_assert(N == 2 || N == 4, "two or four elements");
  if (!vec) {
#pragma unroll
    for (int k = 0; k < N; ++k) x[k] = load_elem(base, i + k, dt);
    return;
  }
  if (dt == kF32) {
    if constexpr (N == 4) {
      const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
      x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
    } else {
      const float2 v = *reinterpret_cast<const float2*>(static_cast<const float*>(base) + i);
      x[0] = v.x, x[1] = v.y;
    }
    return;
  }
  uint32_t w[N / 2];
  if constexpr (N == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + i);
    w[0] = v.x, w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(static_cast<const uint16_t*>(base) + i);
  }
#pragma unroll
  for (int k = 0; k < N / 2; ++k) {
    const float2 f = dt == kF16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[k]))
                                : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
    x[2 * k] = f.x, x[2 * k + 1] = f.y;
  }
}

// N consecutive values into an f32, f16 or bf16 cache row at element i (a
// multiple of N; cache rows are aligned), in one store.
template <int N>
__device__ __forceinline__ void store_vec(void* base, size_t i, int dt, const float (&x)[N]) {
  if (dt == kF32) {
    if constexpr (N == 4)
      *reinterpret_cast<float4*>(static_cast<float*>(base) + i) = make_float4(x[0], x[1], x[2], x[3]);
    else
      *reinterpret_cast<float2*>(static_cast<float*>(base) + i) = make_float2(x[0], x[1]);
    return;
  }
  uint32_t w[N / 2];
#pragma unroll
  for (int k = 0; k < N / 2; ++k)
    w[k] = dt == kF16 ? pack2<false>(x[2 * k], x[2 * k + 1]) : pack2<true>(x[2 * k], x[2 * k + 1]);
  if constexpr (N == 4)
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + i) = make_uint2(w[0], w[1]);
  else
    *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(base) + i) = w[0];
}

// One warp appends every KV head's row of one new token r (= b * new_len +
// t) into an f32, f16 or bf16 cache with head_dim HD (64 or 128): the
// position's page and (cos, sin) pairs are looked up once for all heads, and
// each lane moves HD/32 consecutive values of a row.  Same rotation and
// conversion as append_row.
template <int HD>
__device__ __forceinline__ void append_token(const AppendArgs& a, int r, int lane) {
  constexpr int kN = HD / 32;  // values per lane: 2 or 4
  const CacheView& c = a.cache;
  const int b = r / a.new_len, t = r - b * a.new_len;
  const int pos = a.seqs.start[b] + t;
  const int page = c.block_table[static_cast<size_t>(a.seqs.seq[b]) * c.pages_per_seq + pos / c.page];
  if (page < 0 || page >= c.num_pages) {
    if (lane == 0 && a.status) atomicOr(a.status, kStatusBadPage);
    return;
  }
  double2 cs[kN / 2];
  if (a.rope) {
#pragma unroll
    for (int i = 0; i < kN / 2; ++i)
      cs[i] = a.rope[static_cast<size_t>(pos) * (HD / 2) + lane * (kN / 2) + i];
  }
  const uintptr_t align = static_cast<uintptr_t>(kN) * (a.in_dtype == kF32 ? 4 : 2);
  const bool kvec = reinterpret_cast<uintptr_t>(a.k) % align == 0;
  const bool vvec = reinterpret_cast<uintptr_t>(a.v) % align == 0;
  const size_t row0 = (static_cast<size_t>(page) * c.hkv) * c.page + pos % c.page;
  // kG heads' rows loaded before any is written: one memory round trip per
  // group of heads, not one per head
  constexpr int kG = 4;
  for (int h0 = 0; h0 < c.hkv; h0 += kG) {
    float k[kG][kN], v[kG][kN];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (h0 + g >= c.hkv) break;
      const size_t in = (static_cast<size_t>(r) * c.hkv + h0 + g) * HD + kN * lane;
      load_vec<kN>(a.k, in, a.in_dtype, kvec, k[g]);
      load_vec<kN>(a.v, in, a.in_dtype, vvec, v[g]);
    }
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (h0 + g >= c.hkv) break;
      if (a.rope) {
#pragma unroll
        for (int i = 0; i < kN / 2; ++i)
          rope_pair(k[g][2 * i], k[g][2 * i + 1], cs[i], k[g][2 * i], k[g][2 * i + 1]);
      }
      const size_t dst = (row0 + static_cast<size_t>(h0 + g) * c.page) * HD + kN * lane;
      store_vec<kN>(c.k, dst, c.dtype, k[g]);
      store_vec<kN>(c.v, dst, c.dtype, v[g]);
    }
  }
}

__device__ __forceinline__ void append_kv_row(const AppendArgs& a, int warp, int lane) {
  const int hkv = a.cache.hkv;
  const int h = warp % hkv;
  const int t = (warp / hkv) % a.new_len;
  const int b = warp / (hkv * a.new_len);
  const int pos = a.seqs.start[b] + t;
  bool ok;
  const int64_t dst = cache_row(a.cache, a.seqs.seq[b], pos, h, a.status, ok);
  if (!ok) return;
  const size_t in_off = (static_cast<size_t>(b * a.new_len + t) * hkv + h) * a.cache.hd;
  const double2* rope = a.rope ? a.rope + static_cast<size_t>(pos) * (a.cache.hd / 2) : nullptr;
  append_row(a.k, a.v, a.in_dtype, in_off, rope, a.cache, dst, lane);
}

}  // namespace ql
