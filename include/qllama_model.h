/*
 * qllama_model.h -- C ABI of the Llama model host around the attention path
 * (B200, sm_100a): the layers on either side of the attention operator, a
 * GGUF loader that puts the weights on the device, and the sampler.
 *
 * It replaces, for a device-resident model:
 *   Transformer::forward_with_cache   src/transformer/transformer.rs:238-266
 *   TransformerBlock::forward_with_cache  src/transformer/layers.rs:615-631
 *   Embedding / Linear / RmsNorm / Mlp  src/transformer/layers.rs:57-205, 538-579
 *   TensorOps::rms_norm / silu          src/tensor/ops.rs:96-136, 222-239
 *   Transformer::from_gguf, TransformerConfig::from_gguf
 *                                       src/transformer/transformer.rs:142-197,
 *                                       src/transformer/config.rs:71-164
 *   GgufFile::from_path / load_tensor   src/gguf/parser.rs:40-99, src/gguf/loader.rs:47-132
 *   generate (prefill, then one token per step)  src/main.rs:387-429
 *   Sampler::sample_slice               src/sampler/sampler.rs:119-325
 * The attention steps of each layer go through ql_attn_forward
 * (qllama_attn.h) on the caller's ql_kv.
 *
 * Conventions are those of qllama_attn.h: every entry point returns QL_OK or
 * a QL_ERR_* status with a message in ql_last_error(); validation happens
 * before device work; one host thread per context at a time.
 *
 * Arithmetic: weights and activations are f32.  Every matrix product keeps
 * the reference's order (one output element = a sequential f32 sum over the
 * inner dimension, each product rounded separately, no fused multiply-add);
 * RMSNorm sums squares in f64 in index order; SiLU evaluates exp in f64 and
 * rounds it to f32 (the correctly rounded single-precision exp; the
 * reference's libm expf is within 0.502 ulp, so about one value in a few
 * hundred differs in its last bit).  With an f32 KV cache the logits agree
 * with the reference's CPU path to about 1e-5, and bit for bit where the
 * host's SiLU rounds the same way; greedy tokens are identical.
 * Each layer's Q/K/V projections run fused with RoPE and the cache append
 * (ql_qkv_rope_append, below) for f32, f16 and bf16 caches.
 */
#ifndef QLLAMA_MODEL_H
#define QLLAMA_MODEL_H

#include <stdint.h>

#include "qllama_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* TransformerConfig (src/transformer/config.rs:12-31); head_dim =
 * hidden_size / num_heads. */
typedef struct {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t num_layers;
  int32_t max_position_embeddings;
  float rms_norm_eps;
  float rope_theta;
} ql_llama_config;

typedef struct ql_llama ql_llama;

/* Transformer::from_parts: allocates the device weights (zeros) and the
 * workspace for up to max_position_embeddings tokens per call.  The checks of
 * Attention::new / Mlp::new (layers.rs:244-286, 550-570) apply. */
int ql_llama_create(ql_ctx* ctx, const ql_llama_config* cfg, ql_llama** out);
int ql_llama_destroy(ql_llama* m);
int ql_llama_get_config(const ql_llama* m, ql_llama_config* out);

/* Sets one weight by its GGUF name (llama.cpp's LLM_TENSOR names, as
 * Transformer::from_gguf assembles them): token_embd.weight, output_norm.weight,
 * output.weight, blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,
 * ffn_gate,ffn_up,ffn_down}.weight.  `data` is host f32 in the reference's
 * logical layout after the GGUF dimension reversal: [out_features,
 * in_features] for projections, [vocab, hidden] for the embedding.  `n` must
 * equal the tensor's element count.  Without output.weight the lm_head shares
 * the embedding (tied embeddings, transformer.rs:150-155). */
int ql_llama_set_tensor(ql_llama* m, const char* name, const float* data, int64_t n);

/* GgufFile::from_path + Transformer::from_gguf: parses the file (GGUF v2/v3,
 * little-endian), derives the configuration from its metadata as
 * TransformerConfig::from_gguf does, and loads F32 and F16 tensors (F16
 * widened exactly to f32).  Quantised tensor types are rejected with the
 * reference's message ("not yet supported"). */
int ql_llama_load_gguf(ql_ctx* ctx, const char* path, ql_llama** out);

/* Transformer::forward_with_cache for sequence slot `seq` of `kv` (created
 * with the model's num_layers, num_kv_heads, head_dim; f32 storage keeps the
 * reference's arithmetic): ids [n] (host), logits [n, vocab] written to
 * `logits` (host or device memory as `mem` says; NULL computes only the
 * cache update).  start_pos must continue the cache (cache.rs:132-137) and
 * the last position must stay below max_position_embeddings
 * ("exceeds max_position_embeddings", transformer.rs:250-257). */
int ql_llama_forward(ql_llama* m, ql_kv* kv, int32_t seq, const int32_t* ids, int32_t n,
                     int64_t start_pos, float* logits, int32_t mem);

/* The projections fused with RoPE and the append: one launch computes the
 * Q, K and V projections of `x` (layers.rs:388-390), rotates q and k
 * (layers.rs:397-402, ops.rs:168-220) and writes K and V into the cache at the
 * call's positions (layers.rs:403-413, KvCache::update cache.rs:83-170).
 * args gives layer_idx, batch, new_len, seq_ids, start_pos, num_heads,
 * num_kv_heads, head_dim and rope_theta as for ql_attn_forward (q, k, v, out,
 * dtypes and mem are not read).  x: device f32 [batch*new_len, in_features];
 * wqkv_t: device f32 [in_features, (num_heads + 2*num_kv_heads)*head_dim],
 * the transposed weights of q, k and v side by side; q_rot: device f32
 * [batch, new_len, num_heads, head_dim], the rotated queries.  The cache
 * must store f32, f16 or bf16; positions must continue each sequence
 * ("must continue"), and the sequences' lengths advance.  Every product is an
 * f32 sequential sum in the reference's order. */
int ql_qkv_rope_append(ql_ctx* ctx, ql_kv* kv, const ql_attn_args* args, const float* x,
                       int32_t in_features, const float* wqkv_t, float* q_rot);

/* Steps 5-7 of forward_with_cache (layers.rs:425-455) over rows that
 * ql_qkv_rope_append has just written: args as for ql_attn_forward with
 * q = the rotated queries (in_dtype f32) and k, v unused; start_pos[b] +
 * new_len must equal the sequence's current length. */
int ql_attn_forward_appended(ql_ctx* ctx, ql_kv* kv, const ql_attn_args* args);

/* SamplerConfig (src/sampler/sampler.rs:15-25).  temperature <= 0 is greedy
 * (argmax after the repeat penalty, ties to the smaller id). */
typedef struct {
  float temperature;
  int32_t top_k;        /* 0 = no limit */
  float top_p;          /* >= 1 = no limit */
  float repeat_penalty; /* 1 = none */
} ql_sampler_config;

/* Sampler::sample_slice on the device for one row of logits: repeat penalty
 * over `context` (ids outside the vocabulary ignored, each id once), then
 * greedy argmax, or temperature, softmax (f64), top-k, top-p and the draw at
 * `r` (a uniform number in [0, 1) the caller supplies: the reference draws it
 * from its seeded generator, rng.gen::<f64>()).  logits [vocab] f32 and
 * context [n_context] int32 are device pointers; the token id is written to
 * the device int32 at token_out.  Invalid configurations are rejected as
 * SamplerConfig::validate does; a non-finite logit makes the kernel write -1
 * and raise the context's status (QL_ERR_DEVICE at the next synchronize). */
int ql_sample(ql_ctx* ctx, const float* logits, int32_t vocab, const int32_t* context,
              int32_t n_context, const ql_sampler_config* cfg, double r, int32_t* token_out);

/* generate() (src/main.rs:387-429) on the device: the prompt is prefilled at
 * position 0 of slot `seq`, then each step feeds back the sampled token.  The
 * whole loop is queued without a host round trip per step (the embedding of
 * a step reads the token the previous step's sampler wrote), unless eos_id >=
 * 0, in which case every step is checked and generation stops at EOS (not
 * counted, as in the reference).  `uniforms` holds one draw in [0, 1) per
 * step (NULL for greedy).  out_tokens (host, `steps` entries) receives the
 * generated ids, *n_out their count. */
int ql_llama_generate(ql_llama* m, ql_kv* kv, int32_t seq, const int32_t* prompt,
                      int32_t n_prompt, int32_t steps, int32_t eos_id,
                      const ql_sampler_config* cfg, const double* uniforms, int32_t* out_tokens,
                      int32_t* n_out);

#ifdef __cplusplus
}
#endif
#endif
