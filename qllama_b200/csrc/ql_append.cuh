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
