// bench_driver.cpp -- drives a whole prefill + decode job through the C ABI.
//
// Benchmark harness for bench.py: the reference's generate loop
// (src/main.rs:387-429) issues one Attention::forward_with_cache per layer
// per step; this loop makes the same sequence of ql_attn_forward calls from
// native code, so the measured time is the library's, not an interpreter's.
// `prefill` tokens are written at positions 0..prefill-1, then `steps` single
// tokens, sequence b from position decode_starts[b] on (either phase may be
// empty).  With a communicator, every call is ql_attn_forward_sharded: hq and
// hkv are this rank's heads and the outputs hold out_heads (all ranks' query
// heads) per row.  The calls go to cache layers layer0 .. layer0+layers-1.
// Buffers are device pointers laid out as
//   prefill q/k/v: [layers][batch][prefill][heads][hd]
//   decode  q/k/v: [steps][layers][batch][1][heads][hd]
//   outputs       : same layouts with out_heads*hd columns
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "../../include/qllama_attn.h"

extern "C" int qlb_run_job(ql_ctx* ctx, ql_kv* kv, int32_t layers, int32_t batch,
                           int32_t prefill, int32_t steps, const int64_t* decode_starts,
                           int32_t hq,
                           int32_t hkv, int32_t hd,
                           float theta, int32_t in_dtype, int32_t out_dtype, const void* pq,
                           const void* pk, const void* pv, void* pout, const void* dq,
                           const void* dk, const void* dv, void* dout, ql_comm* comm,
                           int32_t out_heads, int32_t layer0) {
  auto call = [&](const ql_attn_args* a) {
    return comm ? ql_attn_forward_sharded(ctx, kv, comm, a) : ql_attn_forward(ctx, kv, a);
  };
  const size_t in_b = in_dtype == QL_F32 ? 4 : 2, out_b = out_dtype == QL_F32 ? 4 : 2;
  std::vector<int32_t> seqs(batch);
  std::vector<int64_t> starts(batch, 0);
  for (int b = 0; b < batch; ++b) seqs[b] = b;
  ql_attn_args a{};
  a.batch = batch;
  a.seq_ids = seqs.data();
  a.start_pos = starts.data();
  a.num_heads = hq;
  a.num_kv_heads = hkv;
  a.head_dim = hd;
  a.rope_theta = theta;
  a.in_dtype = in_dtype;
  a.out_dtype = out_dtype;
  a.mem = QL_MEM_DEVICE;
  auto at = [](const void* base, size_t off) {
    return static_cast<const void*>(static_cast<const char*>(base) + off);
  };
  if (prefill > 0) {
    a.new_len = prefill;
    const size_t qs = (size_t)batch * prefill * hq * hd, ks = (size_t)batch * prefill * hkv * hd;
    const size_t os = (size_t)batch * prefill * out_heads * hd;
    for (int l = 0; l < layers; ++l) {
      a.layer_idx = layer0 + l;
      a.q = at(pq, l * qs * in_b);
      a.k = at(pk, l * ks * in_b);
      a.v = at(pv, l * ks * in_b);
      a.out = const_cast<void*>(at(pout, l * os * out_b));
      int rc = call(&a);
      if (rc != QL_OK) return rc;
    }
  }
  for (int b = 0; b < batch; ++b) starts[b] = decode_starts[b];
  a.new_len = 1;
  const size_t qs = (size_t)batch * hq * hd, ks = (size_t)batch * hkv * hd;
  const size_t os = (size_t)batch * out_heads * hd;
  for (int s = 0; s < steps; ++s) {
    for (int l = 0; l < layers; ++l) {
      const size_t i = (size_t)s * layers + l;
      a.layer_idx = layer0 + l;
      a.q = at(dq, i * qs * in_b);
      a.k = at(dk, i * ks * in_b);
      a.v = at(dv, i * ks * in_b);
      a.out = const_cast<void*>(at(dout, i * os * out_b));
      int rc = call(&a);
      if (rc != QL_OK) return rc;
    }
    for (int b = 0; b < batch; ++b) starts[b] += 1;
  }
  return QL_OK;
}
