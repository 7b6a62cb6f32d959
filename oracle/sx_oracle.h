/*
 * sx_oracle.h -- CPU restatement of the Sullux/ai-research decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 kernels in ai-research_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference leg may load it.  The product
 * library (libsx.so) never links, loads or calls anything here.
 *
 * Every function cites the reference file:line whose arithmetic it restates
 * (paths relative to the reference project root).  The reference is Zig and
 * cannot be compiled in this image (no zig toolchain), so the restatement is
 * pinned against the reference's own known-answer tests instead
 * (tests/test_oracle_kat.py lists them).
 */
#ifndef SX_ORACLE_H
#define SX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QUANT_NONE 0
#define ORC_QUANT_Q8 1
#define ORC_QUANT_Q4 2

/* ---- tensor.zig ---- */
uint16_t orc_bf16_from_f32(float v);
float orc_bf16_to_f32(uint16_t b);
float orc_f16_round(float v);

/* ---- quant.zig ---- */
void orc_quantize_row_q8_0(uint32_t *dst, const uint16_t *src, size_t n);
void orc_quantize_row_q4_0(uint32_t *dst, const uint16_t *src, size_t n);
void orc_quantize_matrix(uint32_t *dst, const uint16_t *src, size_t rows, size_t cols, int mode,
                         int threads);
size_t orc_quantized_row_words(size_t cols, int mode);

/* ---- dequantised GEMV (test_q4_exec.zig CPU reference) ---- */
void orc_dequant_q4(float *out, const uint32_t *w, size_t rows, size_t cols);
void orc_dequant_q8(float *out, const uint32_t *w, size_t rows, size_t cols);
void orc_gemv_q4(float *y, const uint32_t *w, const float *x, size_t rows, size_t cols,
                 int threads);
void orc_gemv_q8(float *y, const uint32_t *w, const float *x, size_t rows, size_t cols,
                 int threads);
void orc_gate_up_geglu_q4(float *y, const uint32_t *wg, const uint32_t *wu, const float *x,
                          size_t rows, size_t cols, int threads);

/* ---- kernels.zig ---- */
void orc_gemv_bf16(float *y, const float *x, const uint16_t *w, size_t rows, size_t cols);
/* the same on `threads` threads (rows split; each row's sum is unchanged) */
void orc_gemv_bf16_mt(float *y, const float *x, const uint16_t *w, size_t rows, size_t cols,
                      int threads);
/* fused_mlp_q8.wgsl: act[r] = gelu_tanh(Wg[r].x) * (Wu[r].x) with Q8_0 weights */
void orc_gate_up_geglu_q8(float *y, const uint32_t *wg, const uint32_t *wu, const float *x,
                          size_t rows, size_t cols, int threads);
void orc_rmsnorm(float *out, const float *in, const float *w, size_t n, float eps);
void orc_unit_rmsnorm(float *out, const float *in, size_t n, float eps);
void orc_add_rmsnorm(float *x, const float *r, const float *w, float *y, size_t n, float eps,
                     float scalar);
float orc_gelu_tanh(float x);
void orc_rope_inv_freq(float *out, size_t rotary_dim, float theta);
void orc_apply_rope_partial(float *vec, size_t len, uint64_t pos, size_t head_dim,
                            size_t rotary_dim, const float *inv_freq);
void orc_softmax(float *v, size_t n);
uint32_t orc_argmax(const float *v, size_t n);

/* ---- qkv_rope / decode attention on an explicit cache ---- */
void orc_qkv_rope(float *q, const float *k_in, const float *v_in, const float *q_norm_w,
                  const float *k_norm_w, float *k_cache, float *v_cache, int cache_bf16,
                  uint32_t num_q, uint32_t num_kv, uint32_t head_dim, uint32_t rotary_dim,
                  uint32_t k_eq_v, const float *inv_freq, float eps, uint64_t clock,
                  uint32_t slot, uint32_t total_slots);
void orc_decode_attn(float *out, const float *q, const float *k_cache, const float *v_cache,
                     const uint32_t *slots, uint32_t n_slots, uint32_t num_q, uint32_t num_kv,
                     uint32_t head_dim, uint32_t total_slots, float scale);

/* ---- ring_buffer.zig (slot bookkeeping only; K/V live in the caller's cache) ---- */
typedef struct orc_ring orc_ring;
orc_ring *orc_ring_create(uint32_t num_layers, uint32_t num_anchors, uint32_t window_size,
                          uint32_t num_recall);
void orc_ring_destroy(orc_ring *r);
void orc_ring_reset(orc_ring *r);
uint32_t orc_ring_slot_index(const orc_ring *r, uint64_t clock);
uint32_t orc_ring_activate_slot(orc_ring *r, uint32_t layer, uint64_t clock);
void orc_ring_prefill(orc_ring *r, uint32_t layer, uint64_t upto);
void orc_ring_write_recall(orc_ring *r, uint32_t layer, uint32_t rank, uint64_t clock);
void orc_ring_clear_recall(orc_ring *r);
uint32_t orc_ring_active_slots(const orc_ring *r, uint32_t layer, uint64_t clock,
                               uint32_t *out);
uint32_t orc_ring_total_slots(const orc_ring *r);

/* ---- synthetic inputs (identical integer generator to libsx's) ---- */
uint64_t orc_hash(uint64_t seed, uint64_t stream, uint64_t idx);
float orc_synth_normal(uint64_t seed, uint64_t stream, uint64_t idx);
/* threads used by orc_synth_q4 / orc_synth_q8 (orc_model_create sets its own count) */
void orc_set_synth_threads(int threads);
void orc_synth_q4(uint32_t *dst, size_t rows, size_t cols, uint64_t seed, uint64_t stream);
void orc_synth_q8(uint32_t *dst, size_t rows, size_t cols, uint64_t seed, uint64_t stream);
void orc_synth_bf16_normal(uint16_t *dst, size_t n, uint64_t seed, uint64_t stream,
                           float mean, float std);
void orc_synth_gain_f32(float *dst, size_t n, uint64_t seed, uint64_t stream);
void orc_synth_embed_row(float *x, uint32_t hidden, uint32_t token, uint64_t seed);

/* ---- whole-model decode in the GPU graph's op order (model_dispatch.zig) ---- */
typedef struct {
  uint32_t vocab_size, hidden_size, intermediate_size, num_layers;
  uint32_t num_q_heads, num_kv_heads, num_global_kv_heads, head_dim, global_head_dim;
  uint32_t num_anchors, window_size, num_recall;
  uint32_t kv_bf16, has_post_norms, full_every, attention_k_eq_v;
  float rms_norm_eps, rope_theta, rope_theta_full, attn_scale;
  /* layer weight format (kernels.zig:36-41 GpuEngine.init by mode): ORC_QUANT_Q4 (Q4_0
   * layers), ORC_QUANT_Q8 (Q8_0 layers) or ORC_QUANT_NONE (bf16 layers); the LM head is Q8_0
   * in both quantised modes and bf16 otherwise (kernels.zig:38, model_gpu.zig:161) */
  uint32_t layer_quant;
  /* model_gpu.zig:75 quiescence_thresh: layers l >= num_layers / 3 run behind the quiescence
   * gate (model_dispatch.zig:112-118); 0 lets every layer run */
  float quiescence_threshold;
} orc_model_config;

typedef struct orc_model orc_model;
orc_model *orc_model_create(const orc_model_config *cfg, uint64_t seed, int threads);
void orc_model_destroy(orc_model *m);
orc_ring *orc_model_ring(orc_model *m);
uint32_t orc_model_forward(orc_model *m, const float *x_in, uint64_t clock, int want_logits,
                           float *logits_out, float *x_out);
void orc_model_fill_kv(orc_model *m, uint64_t seed);
/* quiescence_gate.wgsl:1-62 on one vector: mean of (x - x_prev)^2 with the shader's 32-lane
 * strided sums and tree; x_prev becomes x; returns 1 when the layer runs */
int orc_quiescence_gate(const float *x, float *x_prev, uint32_t n, float threshold_sq,
                        float *mean_sq);
/* per-layer gate outcome of the last forward: mean_sq[l], active[l] (1 for ungated layers) */
void orc_model_gate_stats(const orc_model *m, float *mean_sq, uint32_t *active);
void orc_model_set_act_bf16(orc_model *m, int on);
void orc_model_synth_recall(orc_model *m, uint64_t clock, uint32_t n_recall, uint64_t seed);
float *orc_model_kcache(orc_model *m, uint32_t layer);
float *orc_model_vcache(orc_model *m, uint32_t layer);
uint32_t orc_model_kv_dim(orc_model *m, uint32_t layer);

/* ---- memory.zig DiffArchive + diff.zig + memory_inject.zig integrateMemory, on a model's
 * ring and caches (layer K/V rows of kv_dim values, f32 or bf16-rounded like the model) ---- */
typedef struct orc_archive orc_archive;
/* initWithKV (memory.zig:28-52); SalienceConfig defaults alpha 1, beta 0.5, gamma 1,
 * lambda 1/2048 (memory.zig:5-7) */
orc_archive *orc_archive_create(orc_model *m, uint32_t capacity, float alpha, float beta,
                                float gamma, float lambda);
void orc_archive_destroy(orc_archive *a);
/* integrateMemory (memory_inject.zig:17-46) after the model's last forward (with logits, whose
 * final normed state it reads) at `clock`; returns the number of recalled entries and their
 * archive indices in rank order */
uint32_t orc_archive_integrate(orc_archive *a, uint64_t clock, uint32_t *selected);
/* DiffArchive.init (memory.zig:24-26): vectors and metadata only, no model, no K/V */
orc_archive *orc_archive_create_dim(uint32_t dim, uint32_t capacity, float alpha, float beta,
                                    float gamma, float lambda);
/* appendWithMeta (memory.zig:91-111) */
void orc_archive_append(orc_archive *a, uint64_t timestamp, float salience, const float *vector);
uint32_t orc_archive_write_head(const orc_archive *a);
uint32_t orc_archive_count(const orc_archive *a);
/* entry i: unit vector (dim floats), timestamp, last access, access count, salience */
void orc_archive_entry(const orc_archive *a, uint32_t i, float *vec, uint64_t *timestamp,
                       uint64_t *last_accessed, uint32_t *access_count, float *salience);
/* scan alone (memory.zig:113-143) with an explicit query: top_k indices in rank order */
uint32_t orc_archive_scan(orc_archive *a, const float *query, uint64_t now, uint32_t *out,
                          uint32_t top_k);

#ifdef __cplusplus
}
#endif
#endif
