/*
 * sx_oracle.c -- CPU restatement of the Sullux/ai-research decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker).  See sx_oracle.h.  Nothing in the
 * product library links or loads this file.  Citations are file:line in the
 * reference project (Zig sources and WGSL shaders).
 *
 * Parity anchor: the reference cannot be built here (Zig, Vulkan absent), so this
 * restatement is pinned to the reference's own known-answer tests
 * (kernels.zig:176-183, tensor.zig:30-41, ring_buffer.zig:149-187, gpu.zig:30-59,
 * test_q4_exec.zig:16-101, test_gpu_suite.zig:9-102) by tests/test_oracle_kat.py.
 */
#include "sx_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* small parallel-for (the reference splits rows into 16 jobs, kernels.zig:76-92) */
typedef void (*orc_range_fn)(void *ctx, size_t begin, size_t end);
typedef struct {
  orc_range_fn fn;
  void *ctx;
  size_t begin, end;
} orc_job;

static void *orc_job_run(void *p) {
  orc_job *j = (orc_job *)p;
  j->fn(j->ctx, j->begin, j->end);
  return NULL;
}

static void orc_parallel_for(size_t n, int threads, orc_range_fn fn, void *ctx) {
  if (threads <= 1 || n < 64) {
    fn(ctx, 0, n);
    return;
  }
  if (threads > 64) threads = 64;
  pthread_t tid[64];
  orc_job jobs[64];
  size_t chunk = (n + (size_t)threads - 1) / (size_t)threads;
  int spawned = 0;
  for (int t = 0; t < threads; ++t) {
    size_t b = (size_t)t * chunk;
    if (b >= n) break;
    size_t e = b + chunk < n ? b + chunk : n;
    jobs[t].fn = fn;
    jobs[t].ctx = ctx;
    jobs[t].begin = b;
    jobs[t].end = e;
    if (pthread_create(&tid[t], NULL, orc_job_run, &jobs[t]) != 0) {
      fn(ctx, b, e);
      jobs[t].fn = NULL;
    }
    spawned = t + 1;
  }
  for (int t = 0; t < spawned; ++t)
    if (jobs[t].fn) pthread_join(tid[t], NULL);
}

static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* ------------------------------------------------------------------------- */
/* tensor.zig:7-18 -- bf16 round-to-nearest-even and widening */
uint16_t orc_bf16_from_f32(float v) {
  uint32_t u = f2u(v);
  uint32_t bias = 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)((u + bias) >> 16);
}
float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* f32 -> f16 -> f32 round trip (round to nearest even, subnormals kept).  Used only
 * for the synthetic scales: BASELINE configs store fp16-representable scales. */
float orc_f16_round(float v) {
  uint32_t x = f2u(v);
  uint32_t sign = x & 0x80000000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return v;
  if (ax >= 0x477FF000u) return u2f(sign | 0x7F800000u);
  if (ax < 0x38800000u) {
    float a = u2f(ax) * 16777216.0f; /* exact power-of-two scaling */
    float r = rintf(a) * (1.0f / 16777216.0f);
    return u2f(sign | f2u(r));
  }
  uint32_t lsb = (ax >> 13) & 1u;
  ax = (ax + 0xFFFu + lsb) & ~0x1FFFu;
  return u2f(sign | ax);
}

/* ------------------------------------------------------------------------- */
/* quant.zig:18-51 -- Q8_0: 9 words per 32 values: f32 d = amax/127, 32 x i8 */
void orc_quantize_row_q8_0(uint32_t *dst, const uint16_t *src, size_t n) {
  size_t nb = n / 32;
  for (size_t b = 0; b < nb; ++b) {
    const uint16_t *s = src + b * 32;
    uint32_t *d = dst + b * 9;
    float amax = 0.0f, vals[32];
    for (int i = 0; i < 32; ++i) {
      vals[i] = orc_bf16_to_f32(s[i]);
      float a = fabsf(vals[i]);
      if (a > amax) amax = a;
    }
    float dd = amax / 127.0f;
    float id = amax > 0.0f ? 127.0f / amax : 0.0f;
    d[0] = f2u(dd);
    uint8_t bytes[32];
    for (int i = 0; i < 32; ++i) {
      /* std.math.round: half away from zero (C round()) */
      int q = (int)roundf(vals[i] * id);
      if (q < -128) q = -128;
      if (q > 127) q = 127;
      bytes[i] = (uint8_t)(int8_t)q;
    }
    for (int w = 0; w < 8; ++w)
      d[1 + w] = (uint32_t)bytes[w * 4] | ((uint32_t)bytes[w * 4 + 1] << 8) |
                 ((uint32_t)bytes[w * 4 + 2] << 16) | ((uint32_t)bytes[w * 4 + 3] << 24);
  }
}

/* quant.zig:53-90 -- Q4_0: 5 words per 32 values: f32 d = amax/7, nibble n of word w is
 * element w*8+n, stored as clamp(round(v*7/amax), -8, 7) + 8 */
void orc_quantize_row_q4_0(uint32_t *dst, const uint16_t *src, size_t n) {
  size_t nb = n / 32;
  for (size_t b = 0; b < nb; ++b) {
    const uint16_t *s = src + b * 32;
    uint32_t *d = dst + b * 5;
    float amax = 0.0f, vals[32];
    for (int i = 0; i < 32; ++i) {
      vals[i] = orc_bf16_to_f32(s[i]);
      float a = fabsf(vals[i]);
      if (a > amax) amax = a;
    }
    float dd = amax / 7.0f;
    float id = amax > 0.0f ? 7.0f / amax : 0.0f;
    d[0] = f2u(dd);
    uint8_t nib[32];
    for (int i = 0; i < 32; ++i) {
      int q = (int)roundf(vals[i] * id);
      if (q < -8) q = -8;
      if (q > 7) q = 7;
      nib[i] = (uint8_t)(q + 8);
    }
    for (int w = 0; w < 4; ++w) {
      uint32_t word = 0;
      for (int k = 0; k < 8; ++k) word |= (uint32_t)nib[w * 8 + k] << (k * 4);
      d[1 + w] = word;
    }
  }
}

/* quant.zig:164-171 */
size_t orc_quantized_row_words(size_t cols, int mode) {
  size_t nb = (cols + 31) / 32;
  if (mode == ORC_QUANT_Q8) return nb * 9;
  if (mode == ORC_QUANT_Q4) return nb * 5;
  return cols / 2;
}

typedef struct {
  uint32_t *dst;
  const uint16_t *src;
  size_t cols, row_words;
  int mode;
} orc_qm_ctx;
static void orc_qm_range(void *p, size_t b, size_t e) {
  orc_qm_ctx *c = (orc_qm_ctx *)p;
  for (size_t r = b; r < e; ++r) {
    if (c->mode == ORC_QUANT_Q8)
      orc_quantize_row_q8_0(c->dst + r * c->row_words, c->src + r * c->cols, c->cols);
    else
      orc_quantize_row_q4_0(c->dst + r * c->row_words, c->src + r * c->cols, c->cols);
  }
}
/* quant.zig:92-162 (row split across up to 16 threads) */
void orc_quantize_matrix(uint32_t *dst, const uint16_t *src, size_t rows, size_t cols, int mode,
                         int threads) {
  if (rows == 0 || cols == 0) return;
  orc_qm_ctx c = {dst, src, cols, orc_quantized_row_words(cols, mode), mode};
  orc_parallel_for(rows, threads, orc_qm_range, &c);
}

/* ------------------------------------------------------------------------- */
/* test_q4_exec.zig:56-74 -- dequantised value (nib - 8) * d at element b*32 + w*8 + n */
void orc_dequant_q4(float *out, const uint32_t *w, size_t rows, size_t cols) {
  size_t nb = cols / 32, rw = nb * 5;
  for (size_t r = 0; r < rows; ++r)
    for (size_t b = 0; b < nb; ++b) {
      const uint32_t *blk = w + r * rw + b * 5;
      float d = u2f(blk[0]);
      for (int wi = 0; wi < 4; ++wi)
        for (int n = 0; n < 8; ++n) {
          uint32_t nib = (blk[1 + wi] >> (n * 4)) & 0xFu;
          out[r * cols + b * 32 + wi * 8 + n] = ((float)nib - 8.0f) * d;
        }
    }
}

/* gemv_q8.wgsl:113-119 -- dequantised value i8 * d, element b*32 + w*4 + byte */
void orc_dequant_q8(float *out, const uint32_t *w, size_t rows, size_t cols) {
  size_t nb = cols / 32, rw = nb * 9;
  for (size_t r = 0; r < rows; ++r)
    for (size_t b = 0; b < nb; ++b) {
      const uint32_t *blk = w + r * rw + b * 9;
      float d = u2f(blk[0]);
      for (int wi = 0; wi < 8; ++wi)
        for (int k = 0; k < 4; ++k) {
          int8_t q = (int8_t)((blk[1 + wi] >> (k * 8)) & 0xFFu);
          out[r * cols + b * 32 + wi * 4 + k] = (float)q * d;
        }
    }
}

typedef struct {
  float *y;
  const uint32_t *w, *w2;
  const float *x;
  size_t cols;
  int wbf16; /* Q4 weights rounded to bf16 after the dequant (the prefill GEMM's operand) */
} orc_gemv_ctx;

/* test_q4_exec.zig:56-74: row_sum += ((nib - 8) * d) * x[elem], sequential over b, w, n;
 * wbf16: the dequantised weight is rounded to bf16 (RNE) first */
static float orc_row_q4(const uint32_t *row, const float *x, size_t cols, int wbf16) {
  size_t nb = cols / 32;
  float sum = 0.0f;
  for (size_t b = 0; b < nb; ++b) {
    const uint32_t *blk = row + b * 5;
    float d = u2f(blk[0]);
    for (int wi = 0; wi < 4; ++wi) {
      uint32_t pk = blk[1 + wi];
      for (int n = 0; n < 8; ++n) {
        float wt = ((float)((pk >> (n * 4)) & 0xFu) - 8.0f) * d;
        if (wbf16) wt = orc_bf16_to_f32(orc_bf16_from_f32(wt));
        sum += wt * x[b * 32 + wi * 8 + n];
      }
    }
  }
  return sum;
}

static float orc_row_q8(const uint32_t *row, const float *x, size_t cols) {
  size_t nb = cols / 32;
  float sum = 0.0f;
  for (size_t b = 0; b < nb; ++b) {
    const uint32_t *blk = row + b * 9;
    float d = u2f(blk[0]);
    for (int wi = 0; wi < 8; ++wi) {
      uint32_t pk = blk[1 + wi];
      for (int k = 0; k < 4; ++k) {
        int8_t q = (int8_t)((pk >> (k * 8)) & 0xFFu);
        sum += ((float)q * d) * x[b * 32 + wi * 4 + k];
      }
    }
  }
  return sum;
}

static void orc_gemv_q4_range(void *p, size_t b, size_t e) {
  orc_gemv_ctx *c = (orc_gemv_ctx *)p;
  size_t rw = (c->cols / 32) * 5;
  for (size_t r = b; r < e; ++r) c->y[r] = orc_row_q4(c->w + r * rw, c->x, c->cols, c->wbf16);
}
static void orc_gemv_q8_range(void *p, size_t b, size_t e) {
  orc_gemv_ctx *c = (orc_gemv_ctx *)p;
  size_t rw = (c->cols / 32) * 9;
  for (size_t r = b; r < e; ++r) c->y[r] = orc_row_q8(c->w + r * rw, c->x, c->cols);
}
void orc_gemv_q4(float *y, const uint32_t *w, const float *x, size_t rows, size_t cols,
                 int threads) {
  orc_gemv_ctx c = {y, w, NULL, x, cols, 0};
  orc_parallel_for(rows, threads, orc_gemv_q4_range, &c);
}
static void orc_gemv_q4_w(float *y, const uint32_t *w, const float *x, size_t rows, size_t cols,
                          int threads, int wbf16) {
  orc_gemv_ctx c = {y, w, NULL, x, cols, wbf16};
  orc_parallel_for(rows, threads, orc_gemv_q4_range, &c);
}
void orc_gemv_q8(float *y, const uint32_t *w, const float *x, size_t rows, size_t cols,
                 int threads) {
  orc_gemv_ctx c = {y, w, NULL, x, cols, 0};
  orc_parallel_for(rows, threads, orc_gemv_q8_range, &c);
}

/* kernels.zig:94-97 */
float orc_gelu_tanh(float x) {
  float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}

/* fused_mlp_q4.wgsl:184-282 / kernels.zig:110-115: act[r] = gelu_tanh(Wg[r].x) * (Wu[r].x) */
static void orc_geglu_range(void *p, size_t b, size_t e) {
  orc_gemv_ctx *c = (orc_gemv_ctx *)p;
  size_t rw = (c->cols / 32) * 5;
  for (size_t r = b; r < e; ++r) {
    float g = orc_row_q4(c->w + r * rw, c->x, c->cols, c->wbf16);
    float u = orc_row_q4(c->w2 + r * rw, c->x, c->cols, c->wbf16);
    c->y[r] = orc_gelu_tanh(g) * u;
  }
}
void orc_gate_up_geglu_q4(float *y, const uint32_t *wg, const uint32_t *wu, const float *x,
                          size_t rows, size_t cols, int threads) {
  orc_gemv_ctx c = {y, wg, wu, x, cols, 0};
  orc_parallel_for(rows, threads, orc_geglu_range, &c);
}
/* fused_mlp_q8.wgsl:1-127 (dequantised i8 * d times x, the Q8 GEMV's row order) */
static void orc_geglu_q8_range(void *p, size_t b, size_t e) {
  orc_gemv_ctx *c = (orc_gemv_ctx *)p;
  size_t rw = (c->cols / 32) * 9;
  for (size_t r = b; r < e; ++r) {
    float g = orc_row_q8(c->w + r * rw, c->x, c->cols);
    float u = orc_row_q8(c->w2 + r * rw, c->x, c->cols);
    c->y[r] = orc_gelu_tanh(g) * u;
  }
}
void orc_gate_up_geglu_q8(float *y, const uint32_t *wg, const uint32_t *wu, const float *x,
                          size_t rows, size_t cols, int threads) {
  orc_gemv_ctx c = {y, wg, wu, x, cols, 0};
  orc_parallel_for(rows, threads, orc_geglu_q8_range, &c);
}
static void orc_geglu_w(float *y, const uint32_t *wg, const uint32_t *wu, const float *x,
                        size_t rows, size_t cols, int threads, int wbf16) {
  orc_gemv_ctx c = {y, wg, wu, x, cols, wbf16};
  orc_parallel_for(rows, threads, orc_geglu_range, &c);
}

/* ------------------------------------------------------------------------- */
/* kernels.zig:24-43 -- 8-lane accumulation, then a horizontal sum, then the tail */
static float orc_dot_bf16(const uint16_t *w, const float *x, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int k = 0; k < 8; ++k) acc[k] += orc_bf16_to_f32(w[i + k]) * x[i + k];
  float s = 0.0f;
  for (int k = 0; k < 8; ++k) s += acc[k];
  for (; i < n; ++i) s += orc_bf16_to_f32(w[i]) * x[i];
  return s;
}
/* kernels.zig:6-22 */
static float orc_dot_f32(const float *a, const float *b, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int k = 0; k < 8; ++k) acc[k] += a[i + k] * b[i + k];
  float s = 0.0f;
  for (int k = 0; k < 8; ++k) s += acc[k];
  for (; i < n; ++i) s += a[i] * b[i];
  return s;
}

/* kernels.zig:68-73 */
void orc_gemv_bf16(float *y, const float *x, const uint16_t *w, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; ++r) y[r] = orc_dot_bf16(w + r * cols, x, cols);
}
typedef struct {
  float *y;
  const uint16_t *w, *w2;
  const float *x;
  size_t cols;
} orc_bf16_ctx;
static void orc_gemv_bf16_range(void *p, size_t b, size_t e) {
  orc_bf16_ctx *c = (orc_bf16_ctx *)p;
  for (size_t r = b; r < e; ++r) c->y[r] = orc_dot_bf16(c->w + r * c->cols, c->x, c->cols);
}
/* kernels.zig:76-92: the row split of gemvParallel */
void orc_gemv_bf16_mt(float *y, const float *x, const uint16_t *w, size_t rows, size_t cols,
                      int threads) {
  orc_bf16_ctx c = {y, w, NULL, x, cols};
  orc_parallel_for(rows, threads, orc_gemv_bf16_range, &c);
}
/* kernels.zig:100-115 gatedMlp's gate/up products with bf16 weights */
static void orc_geglu_bf16_range(void *p, size_t b, size_t e) {
  orc_bf16_ctx *c = (orc_bf16_ctx *)p;
  for (size_t r = b; r < e; ++r) {
    float g = orc_dot_bf16(c->w + r * c->cols, c->x, c->cols);
    float u = orc_dot_bf16(c->w2 + r * c->cols, c->x, c->cols);
    c->y[r] = orc_gelu_tanh(g) * u;
  }
}

/* kernels.zig:46-52 (norm weights already widened to f32, model_gpu.zig:64-73) */
void orc_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; ++i) ss += in[i] * in[i];
  float r = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; ++i) out[i] = in[i] * r * w[i];
}

/* kernels.zig:55-61 */
void orc_unit_rmsnorm(float *out, const float *in, size_t n, float eps) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; ++i) ss += in[i] * in[i];
  float r = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; ++i) out[i] = in[i] * r;
}

/* add_rmsnorm.wgsl:303-338: X = (X + R) * scalar; Y = X * rsqrt(mean(X^2) + eps) * W */
void orc_add_rmsnorm(float *x, const float *r, const float *w, float *y, size_t n, float eps,
                     float scalar) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    x[i] = (x[i] + r[i]) * scalar;
    ss += x[i] * x[i];
  }
  float rs = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; ++i) y[i] = x[i] * rs * w[i];
}

/* kernels.zig:138: freq_i = 1 / pow(theta, 2i / rotary_dim) */
void orc_rope_inv_freq(float *out, size_t rotary_dim, float theta) {
  for (size_t i = 0; i < rotary_dim / 2; ++i)
    out[i] = 1.0f / powf(theta, (float)(2 * i) / (float)rotary_dim);
}

/* kernels.zig:132-150: rotate pairs (i, i + rot/2) for i < rot/2 by angle pos * freq_i */
void orc_apply_rope_partial(float *vec, size_t len, uint64_t pos, size_t head_dim,
                            size_t rotary_dim, const float *inv_freq) {
  size_t heads = len / head_dim, half = rotary_dim / 2;
  for (size_t h = 0; h < heads; ++h) {
    float *v = vec + h * head_dim;
    for (size_t i = 0; i < half; ++i) {
      float angle = (float)pos * inv_freq[i];
      float c = cosf(angle), s = sinf(angle);
      float v0 = v[i], v1 = v[i + half];
      v[i] = v0 * c - v1 * s;
      v[i + half] = v0 * s + v1 * c;
    }
  }
}

/* kernels.zig:152-162 */
void orc_softmax(float *v, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = v[i] > mx ? v[i] : mx;
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    v[i] = expf(v[i] - mx);
    sum += v[i];
  }
  float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) v[i] *= inv;
}

/* kernels.zig:164-174: first index of the maximum (strict >) */
uint32_t orc_argmax(const float *v, size_t n) {
  uint32_t bi = 0;
  float bv = v[0];
  for (size_t i = 1; i < n; ++i)
    if (v[i] > bv) {
      bv = v[i];
      bi = (uint32_t)i;
    }
  return bi;
}

/* ------------------------------------------------------------------------- */
static inline float orc_store_kv(float v, int bf16) {
  return bf16 ? orc_bf16_to_f32(orc_bf16_from_f32(v)) : v;
}

/* qkv_rope.wgsl:133-288 / forward.zig:127-142: per q head RMSNorm(q_norm) + partial RoPE
 * (in place); per kv head RMSNorm(k_norm) + RoPE -> K_cache[slot], unit RMSNorm(v or k when
 * k_eq_v) -> V_cache[slot].  Cache layout [slot][kv_head][head_dim] (model_gpu.zig:133). */
void orc_qkv_rope(float *q, const float *k_in, const float *v_in, const float *q_norm_w,
                  const float *k_norm_w, float *k_cache, float *v_cache, int cache_bf16,
                  uint32_t num_q, uint32_t num_kv, uint32_t head_dim, uint32_t rotary_dim,
                  uint32_t k_eq_v, const float *inv_freq, float eps, uint64_t clock,
                  uint32_t slot, uint32_t total_slots) {
  (void)total_slots;
  size_t D = head_dim;
  for (uint32_t h = 0; h < num_q; ++h) orc_rmsnorm(q + h * D, q + h * D, q_norm_w, D, eps);
  orc_apply_rope_partial(q, (size_t)num_q * D, clock, D, rotary_dim, inv_freq);
  float *tmp = (float *)malloc(sizeof(float) * D);
  size_t kv_dim = (size_t)num_kv * D;
  for (uint32_t h = 0; h < num_kv; ++h) {
    orc_rmsnorm(tmp, k_in + h * D, k_norm_w, D, eps);
    orc_apply_rope_partial(tmp, D, clock, D, rotary_dim, inv_freq);
    float *kc = k_cache + (size_t)slot * kv_dim + h * D;
    for (size_t i = 0; i < D; ++i) kc[i] = orc_store_kv(tmp[i], cache_bf16);
    orc_unit_rmsnorm(tmp, (k_eq_v ? k_in : v_in) + h * D, D, eps);
    float *vc = v_cache + (size_t)slot * kv_dim + h * D;
    for (size_t i = 0; i < D; ++i) vc[i] = orc_store_kv(tmp[i], cache_bf16);
  }
  free(tmp);
}

/* forward.zig:77-104 (runAttentionHeads) / decode_attn.wgsl:19-108 */
void orc_decode_attn(float *out, const float *q, const float *k_cache, const float *v_cache,
                     const uint32_t *slots, uint32_t n_slots, uint32_t num_q, uint32_t num_kv,
                     uint32_t head_dim, uint32_t total_slots, float scale) {
  (void)total_slots;
  size_t D = head_dim, kv_dim = (size_t)num_kv * D;
  uint32_t group = num_q / num_kv;
  float *sc = (float *)malloc(sizeof(float) * (n_slots ? n_slots : 1));
  for (uint32_t h = 0; h < num_q; ++h) {
    uint32_t kvh = h / group;
    const float *qh = q + h * D;
    for (uint32_t i = 0; i < n_slots; ++i)
      sc[i] = orc_dot_f32(qh, k_cache + (size_t)slots[i] * kv_dim + kvh * D, D) * scale;
    if (n_slots) orc_softmax(sc, n_slots);
    float *o = out + h * D;
    for (size_t d = 0; d < D; ++d) o[d] = 0.0f;
    for (uint32_t i = 0; i < n_slots; ++i) {
      const float *vh = v_cache + (size_t)slots[i] * kv_dim + kvh * D;
      for (size_t d = 0; d < D; ++d) o[d] += sc[i] * vh[d];
    }
  }
  free(sc);
}

/* ------------------------------------------------------------------------- */
/* ring_buffer.zig:8-146 -- slot bookkeeping */
struct orc_ring {
  uint32_t num_layers, num_anchors, window_size, num_recall, total_slots;
  uint64_t *clocks;
  uint8_t *active;
  uint64_t total_ingested;
};

orc_ring *orc_ring_create(uint32_t num_layers, uint32_t num_anchors, uint32_t window_size,
                          uint32_t num_recall) {
  orc_ring *r = (orc_ring *)calloc(1, sizeof(orc_ring));
  r->num_layers = num_layers;
  r->num_anchors = num_anchors;
  r->window_size = window_size;
  r->num_recall = num_recall;
  r->total_slots = num_anchors + window_size + num_recall;
  r->clocks = (uint64_t *)calloc((size_t)num_layers * r->total_slots, sizeof(uint64_t));
  r->active = (uint8_t *)calloc((size_t)num_layers * r->total_slots, 1);
  return r;
}
void orc_ring_destroy(orc_ring *r) {
  if (!r) return;
  free(r->clocks);
  free(r->active);
  free(r);
}
void orc_ring_reset(orc_ring *r) {
  memset(r->clocks, 0, sizeof(uint64_t) * r->num_layers * r->total_slots);
  memset(r->active, 0, (size_t)r->num_layers * r->total_slots);
  r->total_ingested = 0;
}
uint32_t orc_ring_total_slots(const orc_ring *r) { return r->total_slots; }

/* ring_buffer.zig:56-59 */
uint32_t orc_ring_slot_index(const orc_ring *r, uint64_t clock) {
  if (clock < r->num_anchors) return (uint32_t)clock;
  return r->num_anchors + (uint32_t)((clock - r->num_anchors) % r->window_size);
}

/* ring_buffer.zig:61-68 (writeKV :70-80 has the same bookkeeping) */
uint32_t orc_ring_activate_slot(orc_ring *r, uint32_t layer, uint64_t clock) {
  uint32_t slot = orc_ring_slot_index(r, clock);
  size_t gi = (size_t)layer * r->total_slots + slot;
  r->clocks[gi] = clock;
  r->active[gi] = 1;
  if (layer == 0 && clock >= r->total_ingested) r->total_ingested = clock + 1;
  return slot;
}

/* Equivalent to activate_slot(0, c) for every c < upto: the last W clocks own the window. */
void orc_ring_prefill(orc_ring *r, uint32_t layer, uint64_t upto) {
  for (uint64_t c = 0; c < upto && c < r->num_anchors; ++c) orc_ring_activate_slot(r, layer, c);
  uint64_t lo = upto > r->num_anchors + (uint64_t)r->window_size ? upto - r->window_size
                                                                  : (uint64_t)r->num_anchors;
  for (uint64_t c = lo; c < upto; ++c) orc_ring_activate_slot(r, layer, c);
}

/* ring_buffer.zig:90-99 */
void orc_ring_write_recall(orc_ring *r, uint32_t layer, uint32_t rank, uint64_t clock) {
  uint32_t slot = r->num_anchors + r->window_size + rank;
  size_t gi = (size_t)layer * r->total_slots + slot;
  r->clocks[gi] = clock;
  r->active[gi] = 1;
}

/* ring_buffer.zig:82-88 */
void orc_ring_clear_recall(orc_ring *r) {
  uint32_t start = r->num_anchors + r->window_size;
  for (uint32_t l = 0; l < r->num_layers; ++l)
    memset(r->active + (size_t)l * r->total_slots + start, 0, r->num_recall);
}

/* ring_buffer.zig:101-136: anchors [0, min(clock+1, A)), then window slots whose clock lies
 * in [max(clock-W+1 | A), clock], then recall slots with clock <= current clock */
uint32_t orc_ring_active_slots(const orc_ring *r, uint32_t layer, uint64_t clock,
                               uint32_t *out) {
  size_t off = (size_t)layer * r->total_slots;
  uint32_t count = 0;
  uint64_t anchor_limit = clock + 1 < r->num_anchors ? clock + 1 : r->num_anchors;
  for (uint32_t s = 0; s < anchor_limit; ++s)
    if (r->active[off + s]) out[count++] = s;
  uint32_t recall_start = r->num_anchors + r->window_size;
  if (clock >= r->num_anchors) {
    uint64_t min_valid =
        clock >= r->window_size ? clock - r->window_size + 1 : (uint64_t)r->num_anchors;
    for (uint32_t s = r->num_anchors; s < recall_start; ++s) {
      if (!r->active[off + s]) continue;
      uint64_t sc = r->clocks[off + s];
      if (sc >= min_valid && sc <= clock) out[count++] = s;
    }
  }
  for (uint32_t s = recall_start; s < r->total_slots; ++s) {
    if (!r->active[off + s]) continue;
    if (r->clocks[off + s] <= clock) out[count++] = s;
  }
  return count;
}

/* ------------------------------------------------------------------------- */
/* Synthetic inputs.  Integer-only generator so that the CUDA library and this oracle
 * produce bit-identical weights; BASELINE distributions: Q4 scales fp16(|N(0,1)|*0.02),
 * uniform nibbles; Q8 scales likewise with uniform int8; norm gains 1 + N(0, 0.1). */
static inline uint64_t orc_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
uint64_t orc_hash(uint64_t seed, uint64_t stream, uint64_t idx) {
  return orc_mix64(orc_mix64(seed ^ (stream * 0xD1B54A32D192ED03ull)) + idx);
}
/* Irwin-Hall(4) of 16-bit uniforms, standardised; exact integer sum, one IEEE division */
float orc_synth_normal(uint64_t seed, uint64_t stream, uint64_t idx) {
  uint64_t h = orc_hash(seed, stream, idx);
  int32_t s = (int32_t)((h & 0xFFFFu) + ((h >> 16) & 0xFFFFu) + ((h >> 32) & 0xFFFFu) +
                        ((h >> 48) & 0xFFFFu)) -
              131070;
  return (float)s / 37837.23f;
}

/* Synthetic blocks, rows in parallel (the values depend only on (seed, stream, block index),
 * so the split does not change them). */
typedef struct {
  uint32_t *dst;
  size_t nb;
  uint64_t seed, stream;
  int q8;
} orc_synth_ctx;

static void orc_synth_rows(void *p, size_t r0, size_t r1) {
  const orc_synth_ctx *c = (const orc_synth_ctx *)p;
  const int words = c->q8 ? 9 : 5, step = c->q8 ? 16 : 8;
  for (size_t r = r0; r < r1; ++r)
    for (size_t b = 0; b < c->nb; ++b) {
      uint64_t idx = r * c->nb + b;
      uint32_t *blk = c->dst + idx * (size_t)words;
      float z = orc_synth_normal(c->seed, c->stream, idx * (uint64_t)step);
      blk[0] = f2u(orc_f16_round(fabsf(z) * 0.02f));
      for (int j = 1; j < words; ++j)
        blk[j] = (uint32_t)orc_hash(c->seed, c->stream, idx * (uint64_t)step + (uint64_t)j);
    }
}

static int g_synth_threads = 1;
void orc_set_synth_threads(int threads) { g_synth_threads = threads < 1 ? 1 : threads; }

void orc_synth_q4(uint32_t *dst, size_t rows, size_t cols, uint64_t seed, uint64_t stream) {
  orc_synth_ctx c = {dst, cols / 32, seed, stream, 0};
  orc_parallel_for(rows, g_synth_threads, orc_synth_rows, &c);
}

void orc_synth_q8(uint32_t *dst, size_t rows, size_t cols, uint64_t seed, uint64_t stream) {
  orc_synth_ctx c = {dst, cols / 32, seed, stream, 1};
  orc_parallel_for(rows, g_synth_threads, orc_synth_rows, &c);
}

void orc_synth_bf16_normal(uint16_t *dst, size_t n, uint64_t seed, uint64_t stream,
                           float mean, float std) {
  for (size_t i = 0; i < n; ++i)
    dst[i] = orc_bf16_from_f32(fmaf(std, orc_synth_normal(seed, stream, i), mean));
}

/* norm gains: bf16(1 + 0.1 z) widened to f32 (model_gpu.zig:64-73) */
void orc_synth_gain_f32(float *dst, size_t n, uint64_t seed, uint64_t stream) {
  for (size_t i = 0; i < n; ++i)
    dst[i] = orc_bf16_to_f32(
        orc_bf16_from_f32(fmaf(0.1f, orc_synth_normal(seed, stream, i), 1.0f)));
}

/* forward.zig:33-37: x = bf16 embedding row * sqrt(H) */
void orc_synth_embed_row(float *x, uint32_t hidden, uint32_t token, uint64_t seed) {
  float sc = sqrtf((float)hidden);
  for (uint32_t j = 0; j < hidden; ++j) {
    float e = orc_bf16_to_f32(
        orc_bf16_from_f32(orc_synth_normal(seed, 1, (uint64_t)token * hidden + j)));
    x[j] = e * sc;
  }
}

/* ------------------------------------------------------------------------- */
/* Whole-model decode in the op order of the pre-recorded GPU graph
 * (model_dispatch.zig:10-43 per layer, :121-127 tail), with the GPU token dispatch
 * semantics of forward.zig:41-45 (layer 0's active-slot list used for every layer). */
enum {
  ORC_T_INPUT_NORM = 0,
  ORC_T_Q = 1,
  ORC_T_K = 2,
  ORC_T_V = 3,
  ORC_T_O = 4,
  ORC_T_QNORM = 5,
  ORC_T_KNORM = 6,
  ORC_T_POST_ATTN = 7,
  ORC_T_PRE_FFN = 8,
  ORC_T_GATE = 9,
  ORC_T_UP = 10,
  ORC_T_DOWN = 11,
  ORC_T_POST_FFN = 12,
  ORC_T_SCALAR = 13,
};
static uint64_t orc_stream(uint32_t layer, uint32_t kind) { return (uint64_t)(layer + 1) * 64 + kind; }

typedef struct {
  uint32_t head_dim, rot, num_kv, q_dim, kv_dim, k_eq_v;
  float theta, layer_scalar;
  uint32_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  float *in_norm, *q_norm, *k_norm, *post_attn, *pre_ffn, *post_ffn;
  float *inv_freq;
  float *k_cache, *v_cache;
} orc_layer;

struct orc_model {
  orc_model_config c;
  float *x_prev;        /* [num_layers][H] quiescence-gate history (model_gpu.zig:132) */
  float *gate_mean_sq;  /* [num_layers] last forward's gate statistic */
  uint32_t *gate_active;
  int threads;
  uint64_t seed;
  orc_layer *layers;
  uint32_t *lm_head;
  float *final_norm;
  orc_ring *ring;
  float *x, *normed, *q, *k, *v, *attn, *mlp, *act, *logits;
  uint32_t *slots;
  int act_bf16; /* round every projection input to bf16 (the batched-prefill GEMM path) */
};

static uint32_t *orc_alloc_q(size_t rows, size_t cols, int mode) {
  return (uint32_t *)malloc(sizeof(uint32_t) * rows * orc_quantized_row_words(cols, mode));
}

/* a layer matrix in the model's layer format: quantised blocks (synthetic, quant.zig layout)
 * or bf16 values bf16(0.02 N(0,1)) (the mode-none checkpoint stand-in) */
static uint32_t *orc_layer_matrix(const orc_model_config *c, size_t rows, size_t cols,
                                  uint64_t seed, uint64_t stream) {
  uint32_t *w = orc_alloc_q(rows, cols, (int)c->layer_quant);
  if (c->layer_quant == ORC_QUANT_Q8)
    orc_synth_q8(w, rows, cols, seed, stream);
  else if (c->layer_quant == ORC_QUANT_NONE)
    orc_synth_bf16_normal((uint16_t *)w, rows * cols, seed, stream, 0.0f, 0.02f);
  else
    orc_synth_q4(w, rows, cols, seed, stream);
  return w;
}

/* y = W x in the layer format (gemv_q4.wgsl / gemv_q8.wgsl / gemv_bf16.wgsl) */
static void orc_proj(const orc_model *m, float *y, const uint32_t *w, const float *x, size_t rows,
                     size_t cols);
static void orc_proj_geglu(const orc_model *m, float *y, const uint32_t *wg, const uint32_t *wu,
                           const float *x, size_t rows, size_t cols);

orc_model *orc_model_create(const orc_model_config *cfg, uint64_t seed, int threads) {
  orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
  m->c = *cfg;
  m->threads = threads;
  m->seed = seed;
  orc_set_synth_threads(threads);
  const orc_model_config *c = &m->c;
  uint32_t H = c->hidden_size, I = c->intermediate_size;
  uint32_t total_slots = c->num_anchors + c->window_size + c->num_recall;
  m->layers = (orc_layer *)calloc(c->num_layers, sizeof(orc_layer));
  uint32_t max_q = 0, max_kv = 0;
  for (uint32_t l = 0; l < c->num_layers; ++l) {
    orc_layer *L = &m->layers[l];
    /* loader.zig:36-42 / types.zig:109 */
    int full = c->full_every && ((l + 1) % c->full_every == 0);
    L->head_dim = full ? c->global_head_dim : c->head_dim;
    L->rot = full ? L->head_dim / 4 : L->head_dim;
    L->num_kv = full ? c->num_global_kv_heads : c->num_kv_heads;
    L->q_dim = c->num_q_heads * L->head_dim;
    L->kv_dim = L->num_kv * L->head_dim;
    L->k_eq_v = full && c->attention_k_eq_v;
    L->theta = full ? c->rope_theta_full : c->rope_theta;
    if (L->q_dim > max_q) max_q = L->q_dim;
    if (L->kv_dim > max_kv) max_kv = L->kv_dim;
    L->wq = orc_layer_matrix(c, L->q_dim, H, seed, orc_stream(l, ORC_T_Q));
    L->wk = orc_layer_matrix(c, L->kv_dim, H, seed, orc_stream(l, ORC_T_K));
    if (L->k_eq_v) {
      L->wv = orc_alloc_q(L->kv_dim, H, (int)c->layer_quant);
      memcpy(L->wv, L->wk,
             sizeof(uint32_t) * L->kv_dim * orc_quantized_row_words(H, (int)c->layer_quant));
    } else {
      L->wv = orc_layer_matrix(c, L->kv_dim, H, seed, orc_stream(l, ORC_T_V));
    }
    L->wo = orc_layer_matrix(c, H, L->q_dim, seed, orc_stream(l, ORC_T_O));
    L->wg = orc_layer_matrix(c, I, H, seed, orc_stream(l, ORC_T_GATE));
    L->wu = orc_layer_matrix(c, I, H, seed, orc_stream(l, ORC_T_UP));
    L->wd = orc_layer_matrix(c, H, I, seed, orc_stream(l, ORC_T_DOWN));
    L->in_norm = (float *)malloc(sizeof(float) * H);
    L->post_attn = (float *)malloc(sizeof(float) * H);
    L->pre_ffn = (float *)malloc(sizeof(float) * H);
    L->post_ffn = (float *)malloc(sizeof(float) * H);
    L->q_norm = (float *)malloc(sizeof(float) * L->head_dim);
    L->k_norm = (float *)malloc(sizeof(float) * L->head_dim);
    orc_synth_gain_f32(L->in_norm, H, seed, orc_stream(l, ORC_T_INPUT_NORM));
    orc_synth_gain_f32(L->post_attn, H, seed, orc_stream(l, ORC_T_POST_ATTN));
    orc_synth_gain_f32(L->pre_ffn, H, seed, orc_stream(l, ORC_T_PRE_FFN));
    orc_synth_gain_f32(L->post_ffn, H, seed, orc_stream(l, ORC_T_POST_FFN));
    orc_synth_gain_f32(L->q_norm, L->head_dim, seed, orc_stream(l, ORC_T_QNORM));
    orc_synth_gain_f32(L->k_norm, L->head_dim, seed, orc_stream(l, ORC_T_KNORM));
    L->layer_scalar = orc_bf16_to_f32(orc_bf16_from_f32(
        fmaf(0.05f, orc_synth_normal(seed, orc_stream(l, ORC_T_SCALAR), 0), 1.0f)));
    L->inv_freq = (float *)malloc(sizeof(float) * (L->rot / 2 + 1));
    orc_rope_inv_freq(L->inv_freq, L->rot, L->theta);
    L->k_cache = (float *)calloc((size_t)total_slots * L->kv_dim, sizeof(float));
    L->v_cache = (float *)calloc((size_t)total_slots * L->kv_dim, sizeof(float));
  }
  if (c->layer_quant == ORC_QUANT_NONE) {
    m->lm_head = orc_alloc_q(c->vocab_size, H, ORC_QUANT_NONE);
    orc_synth_bf16_normal((uint16_t *)m->lm_head, (size_t)c->vocab_size * H, seed, 2, 0.0f, 0.02f);
  } else {
    m->lm_head = orc_alloc_q(c->vocab_size, H, ORC_QUANT_Q8);
    orc_synth_q8(m->lm_head, c->vocab_size, H, seed, 2);
  }
  m->final_norm = (float *)malloc(sizeof(float) * H);
  orc_synth_gain_f32(m->final_norm, H, seed, 3);
  m->ring = orc_ring_create(1, c->num_anchors, c->window_size, c->num_recall);
  m->x_prev = (float *)calloc((size_t)c->num_layers * H, sizeof(float));
  m->gate_mean_sq = (float *)calloc(c->num_layers, sizeof(float));
  m->gate_active = (uint32_t *)calloc(c->num_layers, sizeof(uint32_t));
  m->x = (float *)malloc(sizeof(float) * H);
  m->normed = (float *)malloc(sizeof(float) * H);
  m->mlp = (float *)malloc(sizeof(float) * H);
  m->q = (float *)malloc(sizeof(float) * max_q);
  m->attn = (float *)malloc(sizeof(float) * max_q);
  m->k = (float *)malloc(sizeof(float) * max_kv);
  m->v = (float *)malloc(sizeof(float) * max_kv);
  m->act = (float *)malloc(sizeof(float) * I);
  m->logits = (float *)malloc(sizeof(float) * c->vocab_size);
  m->slots = (uint32_t *)malloc(sizeof(uint32_t) * total_slots);
  return m;
}

void orc_model_destroy(orc_model *m) {
  if (!m) return;
  for (uint32_t l = 0; l < m->c.num_layers; ++l) {
    orc_layer *L = &m->layers[l];
    free(L->wq); free(L->wk); free(L->wv); free(L->wo); free(L->wg); free(L->wu); free(L->wd);
    free(L->in_norm); free(L->post_attn); free(L->pre_ffn); free(L->post_ffn);
    free(L->q_norm); free(L->k_norm); free(L->inv_freq); free(L->k_cache); free(L->v_cache);
  }
  free(m->layers);
  free(m->x_prev); free(m->gate_mean_sq); free(m->gate_active);
  free(m->lm_head); free(m->final_norm);
  orc_ring_destroy(m->ring);
  free(m->x); free(m->normed); free(m->mlp); free(m->q); free(m->attn); free(m->k);
  free(m->v); free(m->act); free(m->logits); free(m->slots);
  free(m);
}

orc_ring *orc_model_ring(orc_model *m) { return m->ring; }
float *orc_model_kcache(orc_model *m, uint32_t layer) { return m->layers[layer].k_cache; }
float *orc_model_vcache(orc_model *m, uint32_t layer) { return m->layers[layer].v_cache; }
uint32_t orc_model_kv_dim(orc_model *m, uint32_t layer) { return m->layers[layer].kv_dim; }

/* Synthetic past: every slot of every layer gets K = bf16(N(0,1)) and V = bf16 of the
 * unit-RMS-normalised N(0,1) vector of that (slot, kv head).  The sum of squares is a
 * sequential fmaf chain so that the CUDA generator reproduces it bit for bit. */
void orc_model_fill_kv(orc_model *m, uint64_t seed) {
  uint32_t total = m->c.num_anchors + m->c.window_size + m->c.num_recall;
  for (uint32_t l = 0; l < m->c.num_layers; ++l) {
    orc_layer *L = &m->layers[l];
    uint32_t D = L->head_dim;
    size_t rows = (size_t)total * L->num_kv;
    for (size_t row = 0; row < rows; ++row) {
      float ss = 0.0f;
      for (uint32_t d = 0; d < D; ++d) {
        float vz = orc_synth_normal(seed, 0x10001ull + 2ull * l, row * D + d);
        ss = fmaf(vz, vz, ss);
      }
      float r = 1.0f / sqrtf(ss / (float)D + m->c.rms_norm_eps);
      for (uint32_t d = 0; d < D; ++d) {
        float kz = orc_synth_normal(seed, 0x10000ull + 2ull * l, row * D + d);
        float vz = orc_synth_normal(seed, 0x10001ull + 2ull * l, row * D + d);
        L->k_cache[row * D + d] = orc_bf16_to_f32(orc_bf16_from_f32(kz));
        L->v_cache[row * D + d] = orc_bf16_to_f32(orc_bf16_from_f32(vz * r));
      }
    }
  }
}

/* Synthetic recall tier (config 3 / 4): the first n_recall recall slots are active with
 * clocks drawn uniformly below `clock`. */
void orc_model_synth_recall(orc_model *m, uint64_t clock, uint32_t n_recall, uint64_t seed) {
  for (uint32_t r = 0; r < n_recall && r < m->c.num_recall; ++r) {
    uint64_t c = clock ? orc_hash(seed, 6, r) % clock : 0;
    orc_ring_write_recall(m->ring, 0, r, c);
  }
}

/* The tcgen05 prefill path multiplies bf16 operands: each layer projection gets a bf16 copy
 * of its f32 input (the normed residual, the attention output, the GeGLU product) and the
 * dequantised weight (f32)(nib - 8) * d rounded to bf16.  This mode rounds the same values
 * (round to nearest even, tensor.zig:7-18) so that path can be held to the f32 tolerance.
 * The LM head (Q8, f32 input) is unchanged. */
void orc_model_set_act_bf16(orc_model *m, int on) { m->act_bf16 = on; }

static void orc_round_bf16(orc_model *m, float *v, size_t n) {
  if (!m->act_bf16) return;
  for (size_t i = 0; i < n; ++i) v[i] = orc_bf16_to_f32(orc_bf16_from_f32(v[i]));
}

static void orc_proj(const orc_model *m, float *y, const uint32_t *w, const float *x, size_t rows,
                     size_t cols) {
  if (m->c.layer_quant == ORC_QUANT_Q8)
    orc_gemv_q8(y, w, x, rows, cols, m->threads);
  else if (m->c.layer_quant == ORC_QUANT_NONE)
    orc_gemv_bf16_mt(y, x, (const uint16_t *)w, rows, cols, m->threads);
  else
    orc_gemv_q4_w(y, w, x, rows, cols, m->threads, m->act_bf16);
}
static void orc_proj_geglu(const orc_model *m, float *y, const uint32_t *wg, const uint32_t *wu,
                           const float *x, size_t rows, size_t cols) {
  if (m->c.layer_quant == ORC_QUANT_Q8) {
    orc_gate_up_geglu_q8(y, wg, wu, x, rows, cols, m->threads);
  } else if (m->c.layer_quant == ORC_QUANT_NONE) {
    orc_bf16_ctx c = {y, (const uint16_t *)wg, (const uint16_t *)wu, x, cols};
    orc_parallel_for(rows, m->threads, orc_geglu_bf16_range, &c);
  } else {
    orc_geglu_w(y, wg, wu, x, rows, cols, m->threads, m->act_bf16);
  }
}

/* quiescence_gate.wgsl:1-62: lane l sums (X_curr[i] - X_prev[i])^2 over i = l, l + 32, ...
 * (copying X_curr into X_prev), the 32 partial sums are folded 16, 8, 4, 2 and the last two
 * added; the layer runs when mean_sq >= threshold_sq or threshold_sq <= 0 */
int orc_quiescence_gate(const float *x, float *x_prev, uint32_t n, float threshold_sq,
                        float *mean_sq) {
  float s[32];
  for (uint32_t lane = 0; lane < 32; ++lane) {
    float acc = 0.0f;
    for (uint32_t i = lane; i < n; i += 32) {
      float d = x[i] - x_prev[i];
      acc = acc + d * d;
      x_prev[i] = x[i];
    }
    s[lane] = acc;
  }
  for (uint32_t w = 16; w >= 2; w >>= 1)
    for (uint32_t lane = 0; lane < w; ++lane) s[lane] = s[lane] + s[lane + w];
  float ms = (s[0] + s[1]) / (float)n;
  if (mean_sq) *mean_sq = ms;
  return (ms >= threshold_sq) || (threshold_sq <= 0.0f);
}

void orc_model_gate_stats(const orc_model *m, float *mean_sq, uint32_t *active) {
  for (uint32_t l = 0; l < m->c.num_layers; ++l) {
    if (mean_sq) mean_sq[l] = m->gate_mean_sq[l];
    if (active) active[l] = m->gate_active[l];
  }
}

uint32_t orc_model_forward(orc_model *m, const float *x_in, uint64_t clock, int want_logits,
                           float *logits_out, float *x_out) {
  const orc_model_config *c = &m->c;
  uint32_t H = c->hidden_size, I = c->intermediate_size;
  float eps = c->rms_norm_eps;
  uint32_t total_slots = c->num_anchors + c->window_size + c->num_recall;
  memcpy(m->x, x_in, sizeof(float) * H);
  uint32_t slot = orc_ring_activate_slot(m->ring, 0, clock);
  uint32_t n = orc_ring_active_slots(m->ring, 0, clock, m->slots);
  const uint32_t dense_limit = c->num_layers / 3;  /* model_dispatch.zig:107 */
  for (uint32_t l = 0; l < c->num_layers; ++l) {
    orc_layer *L = &m->layers[l];
    m->gate_active[l] = 1;
    m->gate_mean_sq[l] = 0.0f;
    if (l >= dense_limit) {
      /* recordLayerIndirect: the gate sees the residual entering the layer; a quiescent
       * layer's 13 commands dispatch nothing (the residual passes through, no K/V write) */
      m->gate_active[l] = (uint32_t)orc_quiescence_gate(m->x, m->x_prev + (size_t)l * H, H,
                                                        c->quiescence_threshold,
                                                        &m->gate_mean_sq[l]);
      if (!m->gate_active[l]) continue;
    }
    orc_rmsnorm(m->normed, m->x, L->in_norm, H, eps);
    orc_round_bf16(m, m->normed, H);
    orc_proj(m, m->q, L->wq, m->normed, L->q_dim, H);
    orc_proj(m, m->k, L->wk, m->normed, L->kv_dim, H);
    orc_proj(m, m->v, L->wv, m->normed, L->kv_dim, H);
    orc_qkv_rope(m->q, m->k, m->v, L->q_norm, L->k_norm, L->k_cache, L->v_cache, c->kv_bf16,
                 c->num_q_heads, L->num_kv, L->head_dim, L->rot, L->k_eq_v, L->inv_freq, eps,
                 clock, slot, total_slots);
    orc_decode_attn(m->attn, m->q, L->k_cache, L->v_cache, m->slots, n, c->num_q_heads,
                    L->num_kv, L->head_dim, total_slots, c->attn_scale);
    orc_round_bf16(m, m->attn, L->q_dim);
    orc_proj(m, m->mlp, L->wo, m->attn, H, L->q_dim);
    if (c->has_post_norms) orc_rmsnorm(m->mlp, m->mlp, L->post_attn, H, eps);
    orc_add_rmsnorm(m->x, m->mlp, L->pre_ffn, m->normed, H, eps, 1.0f);
    orc_round_bf16(m, m->normed, H);
    orc_proj_geglu(m, m->act, L->wg, L->wu, m->normed, I, H);
    orc_round_bf16(m, m->act, I);
    orc_proj(m, m->mlp, L->wd, m->act, H, I);
    if (c->has_post_norms) orc_rmsnorm(m->mlp, m->mlp, L->post_ffn, H, eps);
    orc_add_rmsnorm(m->x, m->mlp, L->in_norm, m->normed, H, eps, L->layer_scalar);
  }
  if (x_out) memcpy(x_out, m->x, sizeof(float) * H);
  if (!want_logits) return 0;
  orc_rmsnorm(m->normed, m->x, m->final_norm, H, eps);
  if (c->layer_quant == ORC_QUANT_NONE)
    orc_gemv_bf16_mt(m->logits, m->normed, (const uint16_t *)m->lm_head, c->vocab_size, H,
                     m->threads);
  else
    orc_gemv_q8(m->logits, m->lm_head, m->normed, c->vocab_size, H, m->threads);
  if (logits_out) memcpy(logits_out, m->logits, sizeof(float) * c->vocab_size);
  return orc_argmax(m->logits, c->vocab_size);
}

/* ------------------------------------------------------------------------- */
/* memory.zig:19-151 DiffArchive, diff.zig:9-57, memory_inject.zig:17-46 */
struct orc_archive {
  orc_model *m;
  uint32_t dim, capacity, count, write_head, max_kv;
  float alpha, beta, gamma, lambda;
  float *vectors;            /* [capacity][dim] unit-normalised */
  uint64_t *timestamp, *last_accessed;
  uint32_t *access_count;
  float *salience;
  float *kv;                 /* [capacity][layers][2][max_kv] */
  float *scores;             /* scan scratch */
  uint32_t *indices;
  float *prev_normed;        /* scratch.prev_normed_x */
};

orc_archive *orc_archive_create(orc_model *m, uint32_t capacity, float alpha, float beta,
                                float gamma, float lambda) {
  orc_archive *a = (orc_archive *)calloc(1, sizeof(orc_archive));
  a->m = m;
  a->dim = m->c.hidden_size;
  a->capacity = capacity;
  a->alpha = alpha;
  a->beta = beta;
  a->gamma = gamma;
  a->lambda = lambda;
  for (uint32_t l = 0; l < m->c.num_layers; ++l)
    if (m->layers[l].kv_dim > a->max_kv) a->max_kv = m->layers[l].kv_dim;
  a->vectors = (float *)calloc((size_t)capacity * a->dim, sizeof(float));
  a->timestamp = (uint64_t *)calloc(capacity, sizeof(uint64_t));
  a->last_accessed = (uint64_t *)calloc(capacity, sizeof(uint64_t));
  a->access_count = (uint32_t *)calloc(capacity, sizeof(uint32_t));
  a->salience = (float *)calloc(capacity, sizeof(float));
  a->kv = (float *)calloc((size_t)capacity * m->c.num_layers * 2 * a->max_kv, sizeof(float));
  a->scores = (float *)calloc(capacity, sizeof(float));
  a->indices = (uint32_t *)calloc(capacity, sizeof(uint32_t));
  a->prev_normed = (float *)calloc(a->dim, sizeof(float));
  return a;
}

orc_archive *orc_archive_create_dim(uint32_t dim, uint32_t capacity, float alpha, float beta,
                                    float gamma, float lambda) {
  orc_archive *a = (orc_archive *)calloc(1, sizeof(orc_archive));
  a->dim = dim;
  a->capacity = capacity;
  a->alpha = alpha;
  a->beta = beta;
  a->gamma = gamma;
  a->lambda = lambda;
  a->vectors = (float *)calloc((size_t)capacity * dim, sizeof(float));
  a->timestamp = (uint64_t *)calloc(capacity, sizeof(uint64_t));
  a->last_accessed = (uint64_t *)calloc(capacity, sizeof(uint64_t));
  a->access_count = (uint32_t *)calloc(capacity, sizeof(uint32_t));
  a->salience = (float *)calloc(capacity, sizeof(float));
  a->scores = (float *)calloc(capacity, sizeof(float));
  a->indices = (uint32_t *)calloc(capacity, sizeof(uint32_t));
  a->prev_normed = (float *)calloc(dim, sizeof(float));
  return a;
}

void orc_archive_append(orc_archive *a, uint64_t timestamp, float salience, const float *vector) {
  float ss = 0.0f;
  for (uint32_t i = 0; i < a->dim; ++i) ss += vector[i] * vector[i];
  float inv = ss > 1e-12f ? 1.0f / sqrtf(ss) : 0.0f;
  uint32_t idx = a->write_head;
  for (uint32_t i = 0; i < a->dim; ++i) a->vectors[(size_t)idx * a->dim + i] = vector[i] * inv;
  a->timestamp[idx] = timestamp;
  a->last_accessed[idx] = timestamp;
  a->access_count[idx] = 0;
  a->salience[idx] = salience;
  a->write_head = (idx + 1) % a->capacity;
  if (a->count < a->capacity) a->count += 1;
}

uint32_t orc_archive_write_head(const orc_archive *a) { return a->write_head; }

void orc_archive_destroy(orc_archive *a) {
  if (!a) return;
  free(a->vectors); free(a->timestamp); free(a->last_accessed); free(a->access_count);
  free(a->salience); free(a->kv); free(a->scores); free(a->indices); free(a->prev_normed);
  free(a);
}

uint32_t orc_archive_count(const orc_archive *a) { return a->count; }

void orc_archive_entry(const orc_archive *a, uint32_t i, float *vec, uint64_t *timestamp,
                       uint64_t *last_accessed, uint32_t *access_count, float *salience) {
  if (vec) memcpy(vec, a->vectors + (size_t)i * a->dim, sizeof(float) * a->dim);
  if (timestamp) *timestamp = a->timestamp[i];
  if (last_accessed) *last_accessed = a->last_accessed[i];
  if (access_count) *access_count = a->access_count[i];
  if (salience) *salience = a->salience[i];
}

/* memory.zig:145-151 score */
static float orc_archive_score(const orc_archive *a, const float *query, uint64_t now,
                               uint32_t i) {
  const float *row = a->vectors + (size_t)i * a->dim;
  float dot = 0.0f;
  for (uint32_t k = 0; k < a->dim; ++k) dot += query[k] * row[k];
  uint64_t dt = now > a->timestamp[i] ? now - a->timestamp[i] : 0;  /* now -| timestamp */
  float recency = expf(-a->lambda * (float)dt);
  return a->alpha * dot + a->beta * recency + a->gamma * a->salience[i];
}

/* memory.zig:113-143 scan: scores, then k rounds of selection with swaps (strict > keeps the
 * first position of a maximum), then the selected entries' access metadata */
uint32_t orc_archive_scan(orc_archive *a, const float *query, uint64_t now, uint32_t *out,
                          uint32_t top_k) {
  uint32_t n = a->count;
  if (n == 0) return 0;
  for (uint32_t i = 0; i < n; ++i) {
    a->scores[i] = orc_archive_score(a, query, now, i);
    a->indices[i] = i;
  }
  uint32_t k = top_k < n ? top_k : n;
  for (uint32_t slot = 0; slot < k; ++slot) {
    uint32_t best = slot;
    for (uint32_t j = slot + 1; j < n; ++j)
      if (a->scores[j] > a->scores[best]) best = j;
    float ts = a->scores[slot];
    a->scores[slot] = a->scores[best];
    a->scores[best] = ts;
    uint32_t ti = a->indices[slot];
    a->indices[slot] = a->indices[best];
    a->indices[best] = ti;
    out[slot] = a->indices[slot];
  }
  for (uint32_t r = 0; r < k; ++r) {
    a->last_accessed[out[r]] = now;
    a->access_count[out[r]] += 1;
  }
  return k;
}

uint32_t orc_archive_integrate(orc_archive *a, uint64_t clock, uint32_t *selected) {
  orc_model *m = a->m;
  const uint32_t H = a->dim, L = m->c.num_layers;
  const float *cur = m->normed, *prev = a->prev_normed;
  /* diff.zig:9-35 computeDelta (threshold 0): norm = sqrt(sum (cur - prev)^2) */
  float sum_sq = 0.0f;
  for (uint32_t i = 0; i < H; ++i) {
    float d = cur[i] - prev[i];
    sum_sq += d * d;
  }
  float delta_norm = sqrtf(sum_sq);
  /* diff.zig:37-52 cosineSimilarity(prev, cur) */
  float dot = 0.0f, na = 0.0f, nb = 0.0f;
  for (uint32_t i = 0; i < H; ++i) {
    dot += prev[i] * cur[i];
    na += prev[i] * prev[i];
    nb += cur[i] * cur[i];
  }
  float denom = sqrtf(na) * sqrtf(nb);
  float sim = denom < 1e-12f ? 0.0f : dot / denom;
  if (sim < 0.98f) {  /* LANDMARK_SIMILARITY_THRESHOLD */
    uint32_t idx = a->write_head;
    /* memory.zig:91-111 appendWithMeta: unit-normalised copy, metadata */
    float ss = 0.0f;
    for (uint32_t i = 0; i < H; ++i) ss += cur[i] * cur[i];
    float inv = ss > 1e-12f ? 1.0f / sqrtf(ss) : 0.0f;
    for (uint32_t i = 0; i < H; ++i) a->vectors[(size_t)idx * H + i] = cur[i] * inv;
    a->timestamp[idx] = clock;
    a->last_accessed[idx] = clock;
    a->access_count[idx] = 0;
    a->salience[idx] = delta_norm;
    a->write_head = (idx + 1) % a->capacity;
    if (a->count < a->capacity) a->count += 1;
    /* memory.zig:70-79 copyKVFromRing: the token's K/V rows of every layer */
    uint32_t slot = orc_ring_slot_index(m->ring, clock);
    for (uint32_t l = 0; l < L; ++l) {
      orc_layer *Ly = &m->layers[l];
      float *dst = a->kv + (((size_t)idx * L + l) * 2) * a->max_kv;
      memset(dst, 0, sizeof(float) * 2 * a->max_kv);
      memcpy(dst, Ly->k_cache + (size_t)slot * Ly->kv_dim, sizeof(float) * Ly->kv_dim);
      memcpy(dst + a->max_kv, Ly->v_cache + (size_t)slot * Ly->kv_dim, sizeof(float) * Ly->kv_dim);
    }
  }
  memcpy(a->prev_normed, cur, sizeof(float) * H);
  uint32_t recall = m->c.num_recall;
  if (recall == 0) {
    orc_ring_clear_recall(m->ring);
    return 0;
  }
  uint32_t k = orc_archive_scan(a, cur, clock, selected, recall);
  orc_ring_clear_recall(m->ring);
  /* memory.zig:81-89 copyKVToRing -> ring_buffer.zig writeRecallKV (slot recallStart + rank,
   * clock = the entry's timestamp) */
  uint32_t total = m->c.num_anchors + m->c.window_size + m->c.num_recall;
  for (uint32_t rank = 0; rank < k; ++rank) {
    uint32_t mi = selected[rank];
    uint32_t slot = m->c.num_anchors + m->c.window_size + rank;
    for (uint32_t l = 0; l < L; ++l) {
      orc_layer *Ly = &m->layers[l];
      const float *src = a->kv + (((size_t)mi * L + l) * 2) * a->max_kv;
      memcpy(Ly->k_cache + (size_t)slot * Ly->kv_dim, src, sizeof(float) * Ly->kv_dim);
      memcpy(Ly->v_cache + (size_t)slot * Ly->kv_dim, src + a->max_kv, sizeof(float) * Ly->kv_dim);
    }
    /* the model's ring keeps one bookkeeping layer: every layer attends over its slot list */
    orc_ring_write_recall(m->ring, 0, rank, a->timestamp[mi]);
  }
  (void)total;
  return k;
}
