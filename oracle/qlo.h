/*
 * qlo.h -- CPU ORACLE for the Qllama attention hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's CPU arithmetic for
 *   RoPE on Q/K -> append into the KV cache -> causal GQA attention -> softmax.V
 * (Qllama `Attention::forward_with_cache`, src/transformer/layers.rs:371-459).
 * It exists to check the CUDA path and to serve as the timed CPU baseline.
 * Nothing in the product library links, loads or calls it; only the tests,
 * the smoke check and the benchmark's CPU-baseline leg do.
 *
 * Numerics follow the reference step for step:
 *   - rope: f64 powf/sin/cos, f64 rotation, cast to f32      (src/tensor/ops.rs:168-220)
 *   - matmul: f32, i-k-j order, sequential in k, no FMA      (src/tensor/ops.rs:63-94)
 *   - scale: f32 multiply                                    (src/tensor/ops.rs:257-261)
 *   - causal mask with offset                                (src/transformer/layers.rs:509-531)
 *   - softmax: f32 max, f64 exp and sum                      (src/tensor/ops.rs:138-166, 292-319)
 *   - KV cache update/get/clear/seq_len                      (src/kv_cache/cache.rs:47-247)
 * Build with -ffp-contract=off so that no multiply-add is fused.
 *
 * The reference's cache stores f32.  The device cache also stores f16, bf16
 * and GGUF-style Q8_0; the oracle models those formats with the same
 * rounding the device applies on append (round-to-nearest-even for f16/bf16,
 * the Q8_0 rule in qlo_q8_0_quantize) so that the comparison isolates the
 * attention arithmetic.  QLO_F32 storage is the reference's own behaviour.
 *
 * Parity pins: tests/test_oracle_kats.py checks this file against the
 * known-answer tests of the reference's tests/tensor_ops.rs,
 * tests/transformer_layers.rs and tests/kv_cache.rs, and against golden
 * vectors generated from the reference's scripts/numpy_forward_reference.py.
 */
#ifndef QLO_H
#define QLO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { QLO_F32 = 0, QLO_F16 = 1, QLO_BF16 = 2, QLO_Q8_0 = 3 };

/* ---- element formats (define the device cache's rounding) ---- */
uint16_t qlo_f32_to_f16(float x);          /* round to nearest even */
float qlo_f16_to_f32(uint16_t h);
uint16_t qlo_f32_to_bf16(float x);         /* round to nearest even */
float qlo_bf16_to_f32(uint16_t h);
/* Q8_0: blocks of 32 values, one f16 scale each.  d = amax/127, id = 1/d
 * (0 when d == 0), q = roundf(x*id) (half away from zero; NaN -> 0),
 * stored scale = f16(d).  Dequantised value = f32(scale) * q. */
void qlo_q8_0_quantize(const float* x, size_t n_blocks, int8_t* qs, uint16_t* scales);
void qlo_q8_0_dequantize(const int8_t* qs, const uint16_t* scales, size_t n_blocks, float* out);
/* Round-trip through a storage format (what a read-back of a cached row returns). */
void qlo_store_roundtrip(int storage, const float* x, size_t n, size_t head_dim, float* out);

/* ---- tensor ops (src/tensor/ops.rs) ---- */
/* x: [seq, inner] with inner = (product of middle dims) * head_dim. */
int qlo_rope(const float* x, size_t seq, size_t inner, size_t head_dim, size_t start_pos,
             float theta, float* out, char* err, size_t errlen);
void qlo_matmul(const float* a, const float* b, size_t m, size_t k, size_t n, float* out);
void qlo_scale(const float* x, size_t n, float factor, float* out);
/* Softmax over the last axis of a [rows, cols] matrix. Errors on NaN. */
int qlo_softmax_rows(const float* x, size_t rows, size_t cols, float* out, char* err, size_t errlen);
/* Softmax along `axis` of a row-major tensor of rank `rank` (ops.rs:138-166). */
int qlo_softmax_axis(const float* x, const size_t* dims, size_t rank, size_t axis, float* out,
                     char* err, size_t errlen);
int qlo_causal_mask_offset(float* scores, size_t rows, size_t cols, size_t offset, char* err,
                           size_t errlen);

/* ---- KV cache (src/kv_cache/cache.rs) ---- */
typedef struct qlo_kv qlo_kv;
qlo_kv* qlo_kv_new(size_t num_layers, size_t max_seq_len, size_t num_kv_heads, size_t head_dim,
                   int storage);
void qlo_kv_free(qlo_kv* kv);
/* k_dims/v_dims: the tensors' shapes (rank may be wrong, which is reported). */
int qlo_kv_update(qlo_kv* kv, size_t layer, const float* k, const size_t* k_dims, size_t k_rank,
                  const float* v, const size_t* v_dims, size_t v_rank, const int32_t* positions,
                  size_t n_positions, char* err, size_t errlen);
int qlo_kv_get(const qlo_kv* kv, size_t layer, const int32_t* positions, size_t n, float* k_out,
               float* v_out, char* err, size_t errlen);
void qlo_kv_clear(qlo_kv* kv);
size_t qlo_kv_seq_len(const qlo_kv* kv);
size_t qlo_kv_layer_len(const qlo_kv* kv, size_t layer);

/* ---- attention core: layers.rs:397-455 (steps 3-7; projections excluded) ----
 * q: [new_len, Hq, hd], k/v: [new_len, Hkv, hd], pre-RoPE, f32.
 * out: [new_len, Hq*hd].  Returns 0 or nonzero with a message in err. */
int qlo_attention_with_cache(qlo_kv* kv, size_t layer, const float* q, const float* k,
                             const float* v, size_t new_len, size_t start_pos, size_t num_heads,
                             size_t num_kv_heads, size_t head_dim, float theta, float* out,
                             char* err, size_t errlen);
/* Uncached twin, layers.rs:293-351 (steps 3-6). */
int qlo_attention_full(const float* q, const float* k, const float* v, size_t seq_len,
                       size_t start_pos, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                       float theta, float* out, char* err, size_t errlen);
/* Attention of one query row block over already-roped, already-cached keys
 * (steps 5-7 of layers.rs:425-455).  qr: [new_len, Hq, hd] post-RoPE;
 * kc/vc: [total_len, Hkv, hd] as read back from the cache. */
int qlo_attention_core(const float* qr, const float* kc, const float* vc, size_t new_len,
                       size_t total_len, size_t start_pos, size_t num_heads, size_t num_kv_heads,
                       size_t head_dim, float* out, char* err, size_t errlen);

/* Threads used by qlo_matmul's row loop (rayon's role in ops.rs:81).  1 = serial. */
void qlo_set_threads(int n);
int qlo_get_threads(void);

/* Batched driver for the CPU baseline: runs `batch` independent sequences'
 * attention cores (one reference call each) on `threads` host threads.
 * qr: [batch][new_len, Hq, hd]; kc/vc: [batch][total_len, Hkv, hd] with the
 * per-sequence total lengths in total_lens; out: [batch][new_len, Hq*hd]. */
int qlo_batch_attention_core(const float* qr, const float* const* kc, const float* const* vc,
                             const size_t* total_lens, size_t batch, size_t new_len,
                             size_t num_heads, size_t num_kv_heads, size_t head_dim,
                             float* out, int threads);

/* ---- model-host pieces outside attention (end-to-end parity only) ---- */
/* TensorOps::silu (ops.rs:222-239): -inf -> -0.0; x >= 0: x / (1 + expf(-x));
 * else e = expf(x), x * e / (1 + e); f32 with libm expf, as Rust's f32::exp. */
void qlo_silu(const float* x, size_t n, float* out);

/* Sampler::sample_slice (src/sampler/sampler.rs:119-325) with the uniform
 * draw `r` in [0, 1) given instead of drawn from the seeded generator:
 * repeat penalty (each context id once, out-of-range ids ignored), greedy
 * argmax (total order, ties to the smaller id) when temperature <= 0, else
 * temperature, softmax (f32 max, f64 exp, sequential f64 sum), top-k, top-p
 * (sorted by probability descending then id ascending, sums in that order)
 * and the draw in index order.  Returns 0 and the id, or nonzero with the
 * reference's message. */
int qlo_sample(const float* logits, size_t vocab, const int32_t* context, size_t n_context,
               float temperature, size_t top_k, float top_p, float repeat_penalty, double r,
               int32_t* out, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
