/*
 * qlo.c -- CPU ORACLE (test infrastructure only) for the Qllama attention hot path.
 *
 * A restatement, in C, of the reference's CPU arithmetic; see qlo.h for the
 * list of reference functions followed and for who may use this file.
 * Compile with -ffp-contract=off: the reference's Rust code never fuses a
 * multiply with an add, and bit-level agreement depends on that.
 */
#include "qlo.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;

void qlo_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int qlo_get_threads(void) { return g_threads; }

static int fail(char* err, size_t errlen, const char* fmt, ...) {
  if (err && errlen) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
  }
  return 1;
}

/* ------------------------------------------------------------------ */
/* element formats                                                     */
/* ------------------------------------------------------------------ */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t qlo_f32_to_f16(float f) {
  uint32_t x = f2u(f);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) /* inf or NaN */
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x0200u : 0u));
  if (ax >= 0x477FF000u) /* >= 65520 rounds to infinity */
    return (uint16_t)(sign | 0x7C00u);
  if (ax < 0x38800000u) { /* below 2^-14: f16 subnormal or zero */
    if (ax < 0x33000000u) return sign; /* below 2^-25 (2^-25 itself ties to 0) */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - e; /* value / 2^-24 = m >> shift */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q += 1u;
    return (uint16_t)(sign | q);
  }
  uint32_t r = ax + 0xFFFu + ((ax >> 13) & 1u); /* round mantissa 23 -> 10 bits, ties to even */
  r -= (112u << 23);                            /* rebias exponent 127 -> 15 */
  return (uint16_t)(sign | (r >> 13));
}

float qlo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  if (e == 0x1Fu) return u2f(sign | 0x7F800000u | (m << 13));
  if (e == 0) {
    if (m == 0) return u2f(sign);
    float v = (float)m * 0x1p-24f; /* exact */
    return sign ? -v : v;
  }
  return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

uint16_t qlo_f32_to_bf16(float f) {
  uint32_t x = f2u(f);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x0040u); /* quiet NaN */
  x += 0x7FFFu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

float qlo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

void qlo_q8_0_quantize(const float* x, size_t n_blocks, int8_t* qs, uint16_t* scales) {
  for (size_t b = 0; b < n_blocks; ++b) {
    const float* xb = x + b * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(xb[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    scales[b] = qlo_f32_to_f16(d);
    for (int i = 0; i < 32; ++i) {
      float r = roundf(xb[i] * id);
      qs[b * 32 + i] = (int8_t)(r == r ? (int)r : 0);
    }
  }
}

void qlo_q8_0_dequantize(const int8_t* qs, const uint16_t* scales, size_t n_blocks, float* out) {
  for (size_t b = 0; b < n_blocks; ++b) {
    float d = qlo_f16_to_f32(scales[b]);
    for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)qs[b * 32 + i];
  }
}

void qlo_store_roundtrip(int storage, const float* x, size_t n, size_t head_dim, float* out) {
  switch (storage) {
    case QLO_F16:
      for (size_t i = 0; i < n; ++i) out[i] = qlo_f16_to_f32(qlo_f32_to_f16(x[i]));
      break;
    case QLO_BF16:
      for (size_t i = 0; i < n; ++i) out[i] = qlo_bf16_to_f32(qlo_f32_to_bf16(x[i]));
      break;
    case QLO_Q8_0: {
      size_t nb = n / 32;
      int8_t* q = (int8_t*)malloc(n ? n : 1);
      uint16_t* s = (uint16_t*)malloc((nb ? nb : 1) * sizeof(uint16_t));
      qlo_q8_0_quantize(x, nb, q, s);
      qlo_q8_0_dequantize(q, s, nb, out);
      free(q);
      free(s);
      (void)head_dim;
      break;
    }
    default:
      if (out != x) memcpy(out, x, n * sizeof(float));
  }
}

/* ------------------------------------------------------------------ */
/* tensor ops                                                          */
/* ------------------------------------------------------------------ */

/* ops.rs:168-220.  Frequencies theta^(-2i/hd) in f64 via pow; angle
 * (start_pos + s) * freq in f64; sin/cos in f64; rotation of the adjacent
 * pair (x[2i], x[2i+1]) in f64, cast to f32.  All heads of one position
 * share the angles. */
int qlo_rope(const float* x, size_t seq, size_t inner, size_t head_dim, size_t start_pos,
             float theta, float* out, char* err, size_t errlen) {
  if (head_dim == 0 || (head_dim & 1) || inner % head_dim != 0)
    return fail(err, errlen,
                "RoPE requires shape [seq_len, ..., head_dim] with a positive even head_dim");
  if (!isfinite(theta) || theta <= 0.0f)
    return fail(err, errlen, "RoPE theta must be finite and positive");
  if (seq != 0 && start_pos > SIZE_MAX - (seq - 1))
    return fail(err, errlen, "RoPE last position overflows usize");
  if (seq == 0 || inner == 0) return 0;
  size_t pairs = head_dim / 2;
  double* freq = (double*)malloc(pairs * sizeof(double));
  for (size_t p = 0; p < pairs; ++p)
    freq[p] = pow((double)theta, -2.0 * (double)p / (double)head_dim);
  size_t heads = inner / head_dim;
  for (size_t s = 0; s < seq; ++s) {
    double position = (double)(start_pos + s);
    for (size_t p = 0; p < pairs; ++p) {
      double angle = position * freq[p];
      double sn = sin(angle), cs = cos(angle);
      for (size_t h = 0; h < heads; ++h) {
        const float* xi = x + s * inner + h * head_dim;
        float* xo = out + s * inner + h * head_dim;
        double first = (double)xi[2 * p];
        double second = (double)xi[2 * p + 1];
        double a = first * cs;
        double b = second * sn;
        double c = first * sn;
        double d = second * cs;
        xo[2 * p] = (float)(a - b);
        xo[2 * p + 1] = (float)(c + d);
      }
    }
  }
  free(freq);
  return 0;
}

/* ops.rs:63-94: [m,k] x [k,n], rows in parallel (rayon there, OpenMP here),
 * i-k-j order within a row, f32 multiply then add, sequential in k. */
void qlo_matmul(const float* a, const float* b, size_t m, size_t k, size_t n, float* out) {
  long long rows = (long long)m;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && rows > 1 && !omp_in_parallel())
#endif
  for (long long i = 0; i < rows; ++i) {
    float* orow = out + (size_t)i * n;
    for (size_t j = 0; j < n; ++j) orow[j] = 0.0f;
    if (k == 0) continue;
    const float* arow = a + (size_t)i * k;
    for (size_t kk = 0; kk < k; ++kk) {
      float left = arow[kk];
      const float* brow = b + kk * n;
      for (size_t j = 0; j < n; ++j) {
        float prod = left * brow[j];
        orow[j] = orow[j] + prod;
      }
    }
  }
}

/* ops.rs:257-261 */
void qlo_scale(const float* x, size_t n, float factor, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = x[i] * factor;
}

/* ops.rs:292-319: one slice with the given stride. */
static void softmax_slice(const float* in, float* out, size_t len, size_t stride) {
  float maximum = -INFINITY;
  for (size_t i = 0; i < len; ++i) maximum = fmaxf(maximum, in[i * stride]);
  double denom = 0.0;
  for (size_t i = 0; i < len; ++i) {
    float v = in[i * stride];
    double c;
    if (maximum == -INFINITY) c = 1.0;
    else if (maximum == INFINITY) c = (v == INFINITY) ? 1.0 : 0.0;
    else c = exp((double)v - (double)maximum);
    denom += c;
  }
  for (size_t i = 0; i < len; ++i) {
    float v = in[i * stride];
    double c;
    if (maximum == -INFINITY) c = 1.0;
    else if (maximum == INFINITY) c = (v == INFINITY) ? 1.0 : 0.0;
    else c = exp((double)v - (double)maximum);
    out[i * stride] = (float)(c / denom);
  }
}

/* ops.rs:138-166 */
int qlo_softmax_axis(const float* x, const size_t* dims, size_t rank, size_t axis, float* out,
                     char* err, size_t errlen) {
  if (axis >= rank)
    return fail(err, errlen, "Softmax axis %zu is out of bounds for rank %zu", axis, rank);
  size_t total = 1;
  for (size_t i = 0; i < rank; ++i) total *= dims[i];
  for (size_t i = 0; i < total; ++i)
    if (isnan(x[i])) return fail(err, errlen, "Softmax input must not contain NaN");
  if (total == 0) return 0;
  size_t inner = 1;
  for (size_t i = axis + 1; i < rank; ++i) inner *= dims[i];
  size_t block = dims[axis] * inner;
  for (size_t base = 0; base < total; base += block)
    for (size_t off = 0; off < inner; ++off)
      softmax_slice(x + base + off, out + base + off, dims[axis], inner);
  return 0;
}

int qlo_softmax_rows(const float* x, size_t rows, size_t cols, float* out, char* err,
                     size_t errlen) {
  size_t dims[2] = {rows, cols};
  return qlo_softmax_axis(x, dims, 2, 1, out, err, errlen);
}

/* layers.rs:509-531 */
int qlo_causal_mask_offset(float* scores, size_t rows, size_t cols, size_t offset, char* err,
                           size_t errlen) {
  if (cols < rows + offset)
    return fail(err, errlen,
                "Causal mask got [%zu, %zu]: %zu key column(s) cannot cover %zu query row(s) "
                "starting at offset %zu",
                rows, cols, cols, rows, offset);
  for (size_t q = 0; q < rows; ++q)
    for (size_t k = offset + q + 1; k < cols; ++k) scores[q * cols + k] = -INFINITY;
  return 0;
}

/* ------------------------------------------------------------------ */
/* KV cache (cache.rs)                                                 */
/* ------------------------------------------------------------------ */

struct qlo_kv {
  size_t num_layers, max_seq_len, num_kv_heads, head_dim;
  int storage;
  float** k; /* per layer [max_seq_len, Hkv, hd] as stored (read-back values) */
  float** v;
  size_t* current_len;
};

/* cache.rs:47-67 */
qlo_kv* qlo_kv_new(size_t num_layers, size_t max_seq_len, size_t num_kv_heads, size_t head_dim,
                   int storage) {
  qlo_kv* kv = (qlo_kv*)calloc(1, sizeof(qlo_kv));
  kv->num_layers = num_layers;
  kv->max_seq_len = max_seq_len;
  kv->num_kv_heads = num_kv_heads;
  kv->head_dim = head_dim;
  kv->storage = storage;
  kv->k = (float**)calloc(num_layers ? num_layers : 1, sizeof(float*));
  kv->v = (float**)calloc(num_layers ? num_layers : 1, sizeof(float*));
  kv->current_len = (size_t*)calloc(num_layers ? num_layers : 1, sizeof(size_t));
  size_t n = max_seq_len * num_kv_heads * head_dim;
  for (size_t l = 0; l < num_layers; ++l) {
    kv->k[l] = (float*)calloc(n ? n : 1, sizeof(float));
    kv->v[l] = (float*)calloc(n ? n : 1, sizeof(float));
  }
  return kv;
}

void qlo_kv_free(qlo_kv* kv) {
  if (!kv) return;
  for (size_t l = 0; l < kv->num_layers; ++l) {
    free(kv->k[l]);
    free(kv->v[l]);
  }
  free(kv->k);
  free(kv->v);
  free(kv->current_len);
  free(kv);
}

static void fmt_dims(char* buf, size_t len, const size_t* dims, size_t rank) {
  size_t o = 0;
  o += (size_t)snprintf(buf + o, len - o, "[");
  for (size_t i = 0; i < rank && o < len; ++i)
    o += (size_t)snprintf(buf + o, len - o, i ? ", %zu" : "%zu", dims[i]);
  if (o < len) snprintf(buf + o, len - o, "]");
}

/* cache.rs:83-170: validate everything, then write, then advance current_len. */
int qlo_kv_update(qlo_kv* kv, size_t layer, const float* k, const size_t* k_dims, size_t k_rank,
                  const float* v, const size_t* v_dims, size_t v_rank, const int32_t* positions,
                  size_t n_positions, char* err, size_t errlen) {
  if (layer >= kv->num_layers)
    return fail(err, errlen, "KV cache layer index %zu out of range (cache has %zu layers)",
                layer, kv->num_layers);
  char kd[96], vd[96];
  fmt_dims(kd, sizeof kd, k_dims, k_rank);
  fmt_dims(vd, sizeof vd, v_dims, v_rank);
  if (k_rank != 3 || k_dims[1] != kv->num_kv_heads || k_dims[2] != kv->head_dim)
    return fail(err, errlen, "K shape %s does not match cache [_, %zu, %zu]", kd,
                kv->num_kv_heads, kv->head_dim);
  int same = (v_rank == k_rank);
  for (size_t i = 0; same && i < k_rank; ++i) same = (v_dims[i] == k_dims[i]);
  if (!same) return fail(err, errlen, "K/V shape mismatch: K %s, V %s", kd, vd);
  size_t new_len = k_dims[0];
  if (n_positions != new_len)
    return fail(err, errlen, "K batch is %zu token(s) but got %zu position(s)", new_len,
                n_positions);
  size_t cur = kv->current_len[layer];
  for (size_t i = 0; i < n_positions; ++i) {
    int32_t p = positions[i];
    if (p < 0) return fail(err, errlen, "positions[%zu] = %d is negative", i, (int)p);
    size_t expected = cur + i;
    if ((size_t)p != expected)
      return fail(err, errlen,
                  "positions[%zu] = %d must continue from current_len (expected %zu); skipping, "
                  "backward, or double writes are not allowed",
                  i, (int)p, expected);
    if ((size_t)p >= kv->max_seq_len)
      return fail(err, errlen, "positions[%zu] = %d exceeds cache capacity %zu", i, (int)p,
                  kv->max_seq_len);
  }
  size_t row = kv->num_kv_heads * kv->head_dim;
  for (size_t t = 0; t < n_positions; ++t) {
    size_t pos = (size_t)positions[t];
    qlo_store_roundtrip(kv->storage, k + t * row, row, kv->head_dim, kv->k[layer] + pos * row);
    qlo_store_roundtrip(kv->storage, v + t * row, row, kv->head_dim, kv->v[layer] + pos * row);
  }
  if (n_positions) {
    size_t last = (size_t)positions[n_positions - 1] + 1;
    if (last > kv->current_len[layer]) kv->current_len[layer] = last;
  }
  return 0;
}

/* cache.rs:185-229: rows in request order, duplicates allowed. */
int qlo_kv_get(const qlo_kv* kv, size_t layer, const int32_t* positions, size_t n, float* k_out,
               float* v_out, char* err, size_t errlen) {
  if (layer >= kv->num_layers)
    return fail(err, errlen, "KV cache layer index %zu out of range (cache has %zu layers)",
                layer, kv->num_layers);
  size_t row = kv->num_kv_heads * kv->head_dim;
  for (size_t i = 0; i < n; ++i) {
    int32_t p = positions[i];
    if (p < 0) return fail(err, errlen, "positions[%zu] = %d is negative", i, (int)p);
    if ((size_t)p >= kv->current_len[layer])
      return fail(err, errlen,
                  "positions[%zu] = %d is at or beyond the written prefix (current_len %zu)", i,
                  (int)p, kv->current_len[layer]);
  }
  for (size_t i = 0; i < n; ++i) {
    size_t p = (size_t)positions[i];
    memcpy(k_out + i * row, kv->k[layer] + p * row, row * sizeof(float));
    memcpy(v_out + i * row, kv->v[layer] + p * row, row * sizeof(float));
  }
  return 0;
}

/* cache.rs:235-239 */
void qlo_kv_clear(qlo_kv* kv) {
  for (size_t l = 0; l < kv->num_layers; ++l) kv->current_len[l] = 0;
}

/* cache.rs:245-247 */
size_t qlo_kv_seq_len(const qlo_kv* kv) { return kv->num_layers ? kv->current_len[0] : 0; }

size_t qlo_kv_layer_len(const qlo_kv* kv, size_t layer) {
  return layer < kv->num_layers ? kv->current_len[layer] : 0;
}

/* ------------------------------------------------------------------ */
/* attention                                                           */
/* ------------------------------------------------------------------ */

/* layers.rs:254-261 (Attention::new's head checks) */
static int check_heads(size_t hq, size_t hkv, size_t hd, char* err, size_t errlen) {
  if (hq == 0 || hkv == 0 || hd == 0)
    return fail(err, errlen, "Attention head counts and head_dim must be positive");
  if (hq % hkv != 0)
    return fail(err, errlen, "num_heads %zu must be divisible by num_kv_heads %zu", hq, hkv);
  return 0;
}

/* [rows, H, hd] -> [H, rows, hd], a copy like tensor.rs:157-183. */
static void to_head_major(const float* x, size_t rows, size_t heads, size_t hd, float* out) {
  for (size_t r = 0; r < rows; ++r)
    for (size_t h = 0; h < heads; ++h)
      memcpy(out + (h * rows + r) * hd, x + (r * heads + h) * hd, hd * sizeof(float));
}

/* layers.rs:425-455 (steps 5-7).  qr post-RoPE [new_len, Hq, hd]; kc/vc
 * cache read-back [total_len, Hkv, hd]; mask offset = start_pos. */
int qlo_attention_core(const float* qr, const float* kc, const float* vc, size_t new_len,
                       size_t total_len, size_t start_pos, size_t num_heads, size_t num_kv_heads,
                       size_t head_dim, float* out, char* err, size_t errlen) {
  if (check_heads(num_heads, num_kv_heads, head_dim, err, errlen)) return 1;
  size_t hd = head_dim;
  float* qh = (float*)malloc((num_heads * new_len * hd + 1) * sizeof(float));
  float* kh = (float*)malloc((num_kv_heads * total_len * hd + 1) * sizeof(float));
  float* vh = (float*)malloc((num_kv_heads * total_len * hd + 1) * sizeof(float));
  float* kt = (float*)malloc((total_len * hd + 1) * sizeof(float));
  float* scores = (float*)malloc((new_len * total_len + 1) * sizeof(float));
  float* probs = (float*)malloc((new_len * total_len + 1) * sizeof(float));
  float* head_out = (float*)malloc((num_heads * new_len * hd + 1) * sizeof(float));
  int rc = 0;
  to_head_major(qr, new_len, num_heads, hd, qh);
  to_head_major(kc, total_len, num_kv_heads, hd, kh);
  to_head_major(vc, total_len, num_kv_heads, hd, vh);
  size_t group = num_heads / num_kv_heads;
  float scale = 1.0f / sqrtf((float)hd);
  for (size_t h = 0; h < num_heads && !rc; ++h) {
    size_t kvh = h / group;
    const float* q_h = qh + h * new_len * hd;
    const float* k_h = kh + kvh * total_len * hd;
    const float* v_h = vh + kvh * total_len * hd;
    /* k_h.transpose(0, 1): [total_len, hd] -> [hd, total_len] */
    for (size_t t = 0; t < total_len; ++t)
      for (size_t d = 0; d < hd; ++d) kt[d * total_len + t] = k_h[t * hd + d];
    qlo_matmul(q_h, kt, new_len, hd, total_len, scores);
    qlo_scale(scores, new_len * total_len, scale, scores);
    rc = qlo_causal_mask_offset(scores, new_len, total_len, start_pos, err, errlen);
    if (rc) break;
    rc = qlo_softmax_rows(scores, new_len, total_len, probs, err, errlen);
    if (rc) break;
    qlo_matmul(probs, v_h, new_len, total_len, hd, head_out + h * new_len * hd);
  }
  if (!rc) /* merge heads: head h occupies columns [h*hd, (h+1)*hd) */
    for (size_t p = 0; p < new_len; ++p)
      for (size_t h = 0; h < num_heads; ++h)
        memcpy(out + (p * num_heads + h) * hd, head_out + (h * new_len + p) * hd,
               hd * sizeof(float));
  free(qh);
  free(kh);
  free(vh);
  free(kt);
  free(scores);
  free(probs);
  free(head_out);
  return rc;
}

/* layers.rs:397-455 */
int qlo_attention_with_cache(qlo_kv* kv, size_t layer, const float* q, const float* k,
                             const float* v, size_t new_len, size_t start_pos, size_t num_heads,
                             size_t num_kv_heads, size_t head_dim, float theta, float* out,
                             char* err, size_t errlen) {
  if (check_heads(num_heads, num_kv_heads, head_dim, err, errlen)) return 1;
  size_t hd = head_dim;
  size_t qn = new_len * num_heads * hd, kn = new_len * num_kv_heads * hd;
  float* qr = (float*)malloc((qn + 1) * sizeof(float));
  float* kr = (float*)malloc((kn + 1) * sizeof(float));
  int32_t* positions = (int32_t*)malloc((new_len + 1) * sizeof(int32_t));
  float *kc = NULL, *vc = NULL;
  int32_t* all_positions = NULL;
  int rc = 0;
  /* 3. RoPE of the new segment from start_pos (layers.rs:398-399) */
  rc = qlo_rope(q, new_len, num_heads * hd, hd, start_pos, theta, qr, err, errlen);
  if (!rc) rc = qlo_rope(k, new_len, num_kv_heads * hd, hd, start_pos, theta, kr, err, errlen);
  /* 4. positions -> update -> get all (layers.rs:403-423) */
  for (size_t i = 0; !rc && i < new_len; ++i) {
    size_t pos = start_pos + i;
    if (pos > 0x7FFFFFFFu)
      rc = fail(err, errlen, "position %zu exceeds the i32 range the cache uses", pos);
    else
      positions[i] = (int32_t)pos;
  }
  if (!rc) {
    size_t dims[3] = {new_len, num_kv_heads, hd};
    rc = qlo_kv_update(kv, layer, kr, dims, 3, v, dims, 3, positions, new_len, err, errlen);
  }
  size_t total_len = start_pos + new_len;
  if (!rc) {
    all_positions = (int32_t*)malloc((total_len + 1) * sizeof(int32_t));
    for (size_t i = 0; !rc && i < total_len; ++i) {
      if (i > 0x7FFFFFFFu)
        rc = fail(err, errlen, "position %zu exceeds the i32 range the cache uses", i);
      else
        all_positions[i] = (int32_t)i;
    }
  }
  if (!rc) {
    size_t cn = total_len * num_kv_heads * hd;
    kc = (float*)malloc((cn + 1) * sizeof(float));
    vc = (float*)malloc((cn + 1) * sizeof(float));
    rc = qlo_kv_get(kv, layer, all_positions, total_len, kc, vc, err, errlen);
  }
  /* 5-7. head-major attention, merge (layers.rs:425-455) */
  if (!rc)
    rc = qlo_attention_core(qr, kc, vc, new_len, total_len, start_pos, num_heads, num_kv_heads,
                            hd, out, err, errlen);
  free(qr);
  free(kr);
  free(positions);
  free(all_positions);
  free(kc);
  free(vc);
  return rc;
}

/* layers.rs:293-351 (steps 3-6 of the uncached forward). */
int qlo_attention_full(const float* q, const float* k, const float* v, size_t seq_len,
                       size_t start_pos, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                       float theta, float* out, char* err, size_t errlen) {
  if (check_heads(num_heads, num_kv_heads, head_dim, err, errlen)) return 1;
  size_t hd = head_dim;
  float* qr = (float*)malloc((seq_len * num_heads * hd + 1) * sizeof(float));
  float* kr = (float*)malloc((seq_len * num_kv_heads * hd + 1) * sizeof(float));
  int rc = qlo_rope(q, seq_len, num_heads * hd, hd, start_pos, theta, qr, err, errlen);
  if (!rc) rc = qlo_rope(k, seq_len, num_kv_heads * hd, hd, start_pos, theta, kr, err, errlen);
  /* square causal mask (layers.rs:482-497) == offset mask with offset 0 */
  if (!rc)
    rc = qlo_attention_core(qr, kr, v, seq_len, seq_len, 0, num_heads, num_kv_heads, hd, out,
                            err, errlen);
  free(qr);
  free(kr);
  return rc;
}

int qlo_batch_attention_core(const float* qr, const float* const* kc, const float* const* vc,
                             const size_t* total_lens, size_t batch, size_t new_len,
                             size_t num_heads, size_t num_kv_heads, size_t head_dim,
                             float* out, int threads) {
  long long nb = (long long)batch;
  int failed = 0;
  int saved = g_threads;
  g_threads = 1; /* one sequence per thread; each call's matmul then runs serially */
  size_t qstride = new_len * num_heads * head_dim;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads < 1 ? 1 : threads) reduction(| : failed)
#endif
  for (long long b = 0; b < nb; ++b) {
    char err[256];
    size_t total = total_lens[b];
    failed |= qlo_attention_core(qr + (size_t)b * qstride, kc[b], vc[b], new_len, total,
                                 total - new_len, num_heads, num_kv_heads, head_dim,
                                 out + (size_t)b * qstride, err, sizeof err);
  }
  g_threads = saved;
  (void)threads;
  return failed;
}

/* ---- model-host pieces outside attention --------------------------------- */

/* ops.rs:222-239 */
void qlo_silu(const float* x, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) {
    const float v = x[i];
    if (v == -INFINITY) {
      out[i] = -0.0f;
    } else if (v >= 0.0f) {
      const float d = 1.0f + expf(-v);
      out[i] = v / d;
    } else {
      const float e = expf(v);
      const float num = v * e;
      const float d = 1.0f + e;
      out[i] = num / d;
    }
  }
}

/* f32::total_cmp as an integer key: negative values reversed below positive. */
static int32_t total_key(float f) {
  int32_t b;
  memcpy(&b, &f, 4);
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

/* sorted_indices (sampler.rs:296-304): probability descending, id ascending. */
static const double* g_sort_p;
static int cmp_prob_desc(const void* a, const void* b) {
  const size_t ia = *(const size_t*)a, ib = *(const size_t*)b;
  const double pa = g_sort_p[ia], pb = g_sort_p[ib];
  if (pa > pb) return -1;
  if (pa < pb) return 1;
  return ia < ib ? -1 : (ia > ib ? 1 : 0);
}

static size_t* sorted_indices(const double* p, size_t n) {
  size_t* order = (size_t*)malloc(n * sizeof(size_t));
  for (size_t i = 0; i < n; ++i) order[i] = i;
  g_sort_p = p;
  qsort(order, n, sizeof(size_t), cmp_prob_desc);
  return order;
}

/* apply_top_k / apply_top_p share this: keep order[0..keep), renormalise. */
static void keep_prefix(double* p, size_t n, const size_t* order, size_t keep) {
  double total = 0.0;
  for (size_t i = 0; i < keep; ++i) total += p[order[i]];
  unsigned char* flags = (unsigned char*)calloc(n, 1);
  for (size_t i = 0; i < keep; ++i) flags[order[i]] = 1;
  for (size_t i = 0; i < n; ++i) p[i] = flags[i] ? p[i] / total : 0.0;
  free(flags);
}

int qlo_sample(const float* logits, size_t vocab, const int32_t* context, size_t n_context,
               float temperature, size_t top_k, float top_p, float repeat_penalty, double r,
               int32_t* out, char* err, size_t errlen) {
  if (vocab == 0) return fail(err, errlen, "Sampling requires a non-empty logits slice");
  for (size_t i = 0; i < vocab; ++i)
    if (!isfinite(logits[i]))
      return fail(err, errlen, "Logits must be finite, but element %zu is %g", i,
                  (double)logits[i]);
  if (!isfinite(temperature))
    return fail(err, errlen, "Sampler temperature must be finite, got %g", (double)temperature);
  if (!isfinite(top_p)) return fail(err, errlen, "Sampler top_p must be finite, got %g", (double)top_p);
  if (!isfinite(repeat_penalty) || repeat_penalty <= 0.0f)
    return fail(err, errlen, "Sampler repeat_penalty must be finite and positive, got %g",
                (double)repeat_penalty);
  float* w = (float*)malloc(vocab * sizeof(float));
  memcpy(w, logits, vocab * sizeof(float));
  if (repeat_penalty != 1.0f) { /* apply_repeat_penalty */
    unsigned char* seen = (unsigned char*)calloc(vocab, 1);
    for (size_t i = 0; i < n_context; ++i) {
      const int32_t t = context[i];
      if (t < 0 || (size_t)t >= vocab || seen[t]) continue;
      seen[t] = 1;
      if (w[t] <= 0.0f) w[t] = w[t] * repeat_penalty;
      else w[t] = w[t] / repeat_penalty;
    }
    free(seen);
    for (size_t i = 0; i < vocab; ++i)
      if (!isfinite(w[i])) {
        free(w);
        return fail(err, errlen, "Repeat penalty produced a non-finite logit at element %zu", i);
      }
  }
  if (temperature <= 0.0f) { /* argmax: total order, ties to the smaller id */
    size_t best = 0;
    for (size_t i = 1; i < vocab; ++i)
      if (total_key(w[i]) > total_key(w[best])) best = i;
    free(w);
    *out = (int32_t)best;
    return 0;
  }
  for (size_t i = 0; i < vocab; ++i) {
    w[i] = w[i] / temperature;
    if (!isfinite(w[i])) {
      free(w);
      return fail(err, errlen, "Temperature %g produced a non-finite logit at element %zu",
                  (double)temperature, i);
    }
  }
  /* softmax (sampler.rs:226-235) */
  float mx = -INFINITY;
  for (size_t i = 0; i < vocab; ++i) mx = fmaxf(mx, w[i]);
  double* p = (double*)malloc(vocab * sizeof(double));
  double total = 0.0;
  for (size_t i = 0; i < vocab; ++i) p[i] = exp((double)w[i] - (double)mx);
  for (size_t i = 0; i < vocab; ++i) total += p[i];
  for (size_t i = 0; i < vocab; ++i) p[i] = p[i] / total;
  free(w);
  if (top_k != 0 && top_k < vocab) { /* apply_top_k */
    size_t* order = sorted_indices(p, vocab);
    keep_prefix(p, vocab, order, top_k);
    free(order);
  }
  if (top_p < 1.0f) { /* apply_top_p */
    size_t* order = sorted_indices(p, vocab);
    const double th = (double)top_p;
    double cum = 0.0;
    size_t keep = vocab;
    for (size_t i = 0; i < vocab; ++i) {
      cum += p[order[i]];
      if (cum >= th) {
        keep = i + 1;
        break;
      }
    }
    keep_prefix(p, vocab, order, keep);
    free(order);
  }
  /* sample_from_distribution (sampler.rs:306-325) */
  double t = 0.0;
  for (size_t i = 0; i < vocab; ++i) t += p[i];
  const double threshold = r * t;
  double cum = 0.0;
  long found = -1, last = -1;
  for (size_t i = 0; i < vocab; ++i) {
    if (p[i] <= 0.0) continue;
    cum += p[i];
    if (cum >= threshold) {
      found = (long)i;
      break;
    }
  }
  if (found < 0)
    for (size_t i = vocab; i-- > 0;)
      if (p[i] > 0.0) {
        last = (long)i;
        break;
      }
  free(p);
  if (found < 0 && last < 0)
    return fail(err, errlen, "Sampling failed: the distribution has no positive probability");
  *out = (int32_t)(found >= 0 ? found : last);
  return 0;
}
