/*
 * sx.h -- C ABI of libsx, the B200 (sm_100a) decode hot path of the Sullux/ai-research
 * inference engine.
 *
 * The reference's Zig host drives its GPU through `GpuEngine` (src/gpu/kernels.zig): it
 * records every per-token op into a command buffer once at init (`record*` calls bound to
 * descriptor sets of storage buffers, src/gpu/model_dispatch.zig:10-129) and re-submits that
 * buffer once per token (`submitPreRecorded`).  This header is the drop-in replacement for
 * that API: the same record calls with the same arguments, recorded into a CUDA graph and
 * replayed per token.  Each declaration cites the reference interface it replaces.
 *
 * Conventions: every function that can fail returns an sx_status (0 = success) and never
 * throws; sx_last_error() gives a message for the calling thread.  Record calls return void
 * exactly like the reference; a bad record call poisons the command buffer and the error is
 * returned by sx_cmd_end.  No torch types cross this boundary: plain pointers and sizes.
 */
#ifndef SX_H
#define SX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SX_API __attribute__((visibility("default")))

typedef int32_t sx_status;
#define SX_OK 0
#define SX_ERR_INVALID 1     /* bad argument or unsupported shape                      */
#define SX_ERR_CUDA 2        /* CUDA runtime error (message in sx_last_error)          */
#define SX_ERR_LAUNCH 3      /* kernel launch failed (VkQueueSubmitFailed)             */
#define SX_ERR_TIMEOUT 4     /* submit did not finish in time (VkFenceTimeout)         */
#define SX_ERR_OOM 5         /* device allocation failed                               */
#define SX_ERR_PEER 6        /* multi-GPU exchange failed                              */
#define SX_ERR_UNSUPPORTED 7 /* valid request this build does not implement            */
#define SX_ERR_DEVICE 8      /* a kernel reported a device-side error (bad slot, ...)  */

/* quant.zig:3-13 QuantMode */
typedef enum { SX_QUANT_NONE = 0, SX_QUANT_Q8 = 1, SX_QUANT_Q4 = 2 } sx_quant_mode;

/* engine flags */
#define SX_ENGINE_KV_F32 1u /* keep the KV cache in f32 like model_gpu.zig:133 (default bf16) */

SX_API const char *sx_version(void);
SX_API const char *sx_last_error(void);
SX_API const char *sx_status_string(sx_status s);

/* ---------------------------------------------------------------------------------------
 * Formats (host only, no GPU needed)
 * ------------------------------------------------------------------------------------- */
/* quant.zig:164-171 getQuantizedRowWords */
SX_API uint64_t sx_quantized_row_words(uint32_t cols, sx_quant_mode mode);
/* Bytes of the packed device layout sx_buffer_upload_weights produces for a rows x cols
 * matrix (equal to the reference's 20 B / 36 B per block when rows % 16 == 0 and
 * cols % 64 == 0). */
SX_API uint64_t sx_packed_bytes(uint32_t rows, uint32_t cols, sx_quant_mode mode);
/* kernels.zig:138 RoPE inverse frequencies 1 / pow(theta, 2i / rotary_dim), i < rot/2 */
SX_API void sx_rope_inv_freq(float *out, uint32_t rotary_dim, float theta);
/* forward.zig:33-37 synthetic-checkpoint embedding row times sqrt(hidden) */
SX_API void sx_synth_embed_row(float *x, uint32_t hidden, uint32_t token, uint64_t seed);

/* ---------------------------------------------------------------------------------------
 * Ring buffer bookkeeping (host), ring_buffer.zig:8-146 DynamicRingBuffer.  Only slot
 * clocks and liveness live here; K/V live in device caches.
 * ------------------------------------------------------------------------------------- */
typedef struct sx_ring sx_ring;
/* ring_buffer.zig:20-37 init */
SX_API sx_status sx_ring_create(uint32_t num_layers, uint32_t num_anchors, uint32_t window_size,
                                uint32_t num_recall, sx_ring **out);
/* ring_buffer.zig:39-43 deinit */
SX_API void sx_ring_destroy(sx_ring *r);
/* ring_buffer.zig:45-49 reset */
SX_API void sx_ring_reset(sx_ring *r);
SX_API uint32_t sx_ring_total_slots(const sx_ring *r);
/* ring_buffer.zig:56-59 getSlotIndex */
SX_API uint32_t sx_ring_slot_index(const sx_ring *r, uint64_t clock);
/* ring_buffer.zig:61-68 activateSlot */
SX_API uint32_t sx_ring_activate_slot(sx_ring *r, uint32_t layer, uint64_t clock);
/* activateSlot for every clock below `upto` (history of a session that ran to `upto`) */
SX_API void sx_ring_prefill(sx_ring *r, uint32_t layer, uint64_t upto);
/* ring_buffer.zig:90-99 writeRecallKV (bookkeeping part) */
SX_API void sx_ring_write_recall(sx_ring *r, uint32_t layer, uint32_t rank, uint64_t clock);
/* ring_buffer.zig:82-88 clearRecall */
SX_API void sx_ring_clear_recall(sx_ring *r);
/* ring_buffer.zig:101-136 getActiveSlots; returns the count written to out */
SX_API uint32_t sx_ring_active_slots(const sx_ring *r, uint32_t layer, uint64_t clock,
                                     uint32_t *out);

/* ---------------------------------------------------------------------------------------
 * Engine, buffers, descriptor sets (gpu/context.zig, gpu/buffer.zig, gpu/descriptors.zig)
 * ------------------------------------------------------------------------------------- */
typedef struct sx_engine sx_engine;
typedef struct sx_buffer sx_buffer;
typedef struct sx_set sx_set;
typedef struct sx_cmd sx_cmd;

/* GpuContext.init + GpuEngine.init (context.zig:17, kernels.zig:35-68).  `mode` selects
 * the layer GEMV format; with SX_QUANT_Q4 the logits GEMV is Q8 (kernels.zig:38). */
SX_API sx_status sx_engine_create(int device, sx_quant_mode mode, uint32_t flags,
                                  sx_engine **out);
/* GpuEngine.deinit (kernels.zig:70-78) */
SX_API void sx_engine_destroy(sx_engine *e);
/* Run subsequent work on an external cudaStream_t (NULL restores the engine's own). */
SX_API sx_status sx_engine_set_stream(sx_engine *e, void *cuda_stream);
SX_API void *sx_engine_stream(sx_engine *e);
/* Wait for the engine stream, then report any device-side error word. */
SX_API sx_status sx_engine_sync(sx_engine *e);

/* GpuBuffer.init (buffer.zig:13) -- device memory */
SX_API sx_status sx_buffer_create(sx_engine *e, uint64_t bytes, sx_buffer **out);
/* Wrap caller-owned device memory (not freed by sx_buffer_destroy). */
SX_API sx_status sx_buffer_wrap(sx_engine *e, void *device_ptr, uint64_t bytes,
                                sx_buffer **out);
/* GpuBuffer.deinit (buffer.zig:56) */
SX_API void sx_buffer_destroy(sx_buffer *b);
SX_API void *sx_buffer_device_ptr(sx_buffer *b);
SX_API uint64_t sx_buffer_size(const sx_buffer *b);
/* asSlice writes/reads (buffer.zig:64-67); synchronous on the engine stream */
SX_API sx_status sx_buffer_write(sx_buffer *b, uint64_t offset, const void *src, uint64_t bytes);
SX_API sx_status sx_buffer_read(sx_buffer *b, uint64_t offset, void *dst, uint64_t bytes);
/* createWeightBuffer (model_gpu.zig:51-62): take a rows x cols matrix in the reference's
 * quantised block layout (quantizeMatrix output: Q4 5 words / Q8 9 words per 32 values) and
 * store it in `dst` in the packed device layout (lossless permutation; dst must hold
 * sx_packed_bytes).  mode NONE is rejected. */
SX_API sx_status sx_buffer_upload_weights(sx_buffer *dst, const uint32_t *ref_words,
                                          uint32_t rows, uint32_t cols, sx_quant_mode mode);
/* Weight ingest on the device (quantizeMatrix, quant.zig:92-162, which the reference runs on
 * 16 CPU threads at load): a row-major bf16 matrix already in device memory (16-byte aligned,
 * cols % 32 == 0) quantised to Q4_0 / Q8_0 blocks bit-identical to the CPU quantiser's, then
 * stored packed in `dst` like sx_buffer_upload_weights.  Synchronous; allocates a staging
 * buffer of the reference-layout size for the call. */
SX_API sx_status sx_buffer_quantize_device(sx_buffer *dst, const void *bf16_device, uint32_t rows,
                                           uint32_t cols, sx_quant_mode mode);
/* Same, from reference-layout words already in device memory. */
SX_API sx_status sx_buffer_repack_device(sx_buffer *dst, const void *ref_words_device,
                                         uint32_t rows, uint32_t cols, sx_quant_mode mode);

/* DescriptorManager.allocateSet + bindBuffers (descriptors.zig:27-103): an ordered tuple of
 * buffers; aliasing allowed (model_gpu.zig:144,153-154).  A record call copies the set's
 * device addresses, so the set may be destroyed after recording; the buffers themselves must
 * outlive every command buffer that uses them. */
SX_API sx_status sx_set_create(sx_engine *e, sx_buffer *const *buffers, uint32_t count,
                               sx_set **out);
SX_API void sx_set_destroy(sx_set *s);

/* ---------------------------------------------------------------------------------------
 * Command buffers: record once, submit per token (kernels.zig:80-157)
 * ------------------------------------------------------------------------------------- */
SX_API sx_status sx_cmd_create(sx_engine *e, sx_cmd **out);
SX_API void sx_cmd_destroy(sx_cmd *c);
/* vkBeginCommandBuffer (model_dispatch.zig:110) */
SX_API sx_status sx_cmd_begin(sx_cmd *c);
/* vkEndCommandBuffer (model_dispatch.zig:128): instantiates the CUDA graph */
SX_API sx_status sx_cmd_end(sx_cmd *c);

/* recordGemv (kernels.zig:80-83): set {W, X, Y}, Y[m] = W[m x k] . X[k] in the engine mode */
SX_API void sx_record_gemv(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k);
/* recordGemvLogits (kernels.zig:88-91): set {W, X, Y}; Q8 weights when the mode is Q4 */
SX_API void sx_record_gemv_logits(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k);
/* recordGateUpSwiGlu (kernels.zig:92-95): set {W_gate, W_up, X, Y},
 * Y[r] = gelu_tanh(W_gate[r] . X) * (W_up[r] . X) */
SX_API void sx_record_gate_up(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k);
/* recordAddRmsNorm (kernels.zig:100-103): set {X, R, W, Y}; X = (X + R) * scalar,
 * Y = X * rsqrt(mean(X^2) + eps) * W */
SX_API void sx_record_add_rmsnorm(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h, float eps,
                                  float scalar);
/* recordRmsNorm (kernels.zig:108-111): set {X, W, Y} */
SX_API void sx_record_rmsnorm(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h, float eps);
/* recordDecodeAttn (kernels.zig:116-119): set {Q, K_cache, V_cache, Active_slots, Attn_out,
 * Step_params}; Step_params = u32 {clock, slot, n_active, 0}.  total_slots sizes the caches
 * (the reference hard-codes 1024, model_gpu.zig:86). */
SX_API void sx_record_decode_attn(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t head_dim,
                                  uint32_t kv_dim, uint32_t gqa_ratio, float inv_sqrt_dim,
                                  uint32_t num_q_heads, uint32_t total_slots);
/* recordQkvRope (kernels.zig:124-129): set {Q_in, K_in, V_in, Q_norm_w, K_norm_w, Q_out,
 * K_cache, V_cache, Step_params} */
SX_API void sx_record_qkv_rope(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t num_q,
                               uint32_t num_kv, uint32_t head_dim, uint32_t rotary_dim,
                               uint32_t k_eq_v, float theta, float eps, uint32_t total_slots);
/* kernels.zig:10-16 QuiescenceGatePushConstants */
typedef struct {
  uint32_t hidden_size;
  float threshold_sq;
  uint32_t base_cmd_idx;
  uint32_t num_cmds;
  uint32_t targets[16];
} sx_quiescence_gate_pc;
/* recordQuiescenceGate (kernels.zig:136-138, quiescence_gate.wgsl): set {X_curr, X_prev,
 * Indirect_args}.  mean((X_curr - X_prev)^2) over hidden_size, X_prev = X_curr, then for
 * c < num_cmds the dispatch record {targets[c], 1, 1} (the layer runs: mean >= threshold_sq
 * or threshold_sq <= 0) or {0, 0, 0} at u32 3 (base_cmd_idx + c) of Indirect_args. */
SX_API void sx_record_quiescence_gate(sx_engine *e, sx_cmd *c, sx_set *set,
                                      const sx_quiescence_gate_pc *pc);
/* record*Indirect (kernels.zig:84-87, 96-99, 104-107, 112-115, 120-123, 130-134): the op
 * reads its dispatch record {x, y, z} (three u32 at byte `offset` of `ind`) on the device when
 * it runs and does nothing when any of the three is zero.  CUDA grids are fixed when the op is
 * recorded, so a non-zero record runs the whole op (the reference's workgroup counts come from
 * the gate's `targets`, which only need to be non-zero here).  The attention variant takes
 * num_q_heads, which the reference takes from the record's x. */
SX_API void sx_record_gemv_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k,
                                    sx_buffer *ind, uint64_t offset);
SX_API void sx_record_gate_up_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m,
                                       uint32_t k, sx_buffer *ind, uint64_t offset);
SX_API void sx_record_add_rmsnorm_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h,
                                           float eps, float scalar, sx_buffer *ind,
                                           uint64_t offset);
SX_API void sx_record_rmsnorm_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h,
                                       float eps, sx_buffer *ind, uint64_t offset);
SX_API void sx_record_decode_attn_indirect(sx_engine *e, sx_cmd *c, sx_set *set,
                                           uint32_t head_dim, uint32_t kv_dim, uint32_t gqa_ratio,
                                           float inv_sqrt_dim, uint32_t num_q_heads,
                                           uint32_t total_slots, sx_buffer *ind,
                                           uint64_t offset);
SX_API void sx_record_qkv_rope_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t num_q,
                                        uint32_t num_kv, uint32_t head_dim, uint32_t rotary_dim,
                                        uint32_t k_eq_v, float theta, float eps,
                                        uint32_t total_slots, sx_buffer *ind, uint64_t offset);
/* recordArgmax (kernels.zig:139-142): set {Logits, OutToken}; first index of the maximum
 * (the CPU rule, kernels.zig:164-174) */
SX_API void sx_record_argmax(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t vocab);
/* recordBarrier (kernels.zig:143-146): ordering is implicit in the graph; kept for parity */
SX_API void sx_record_barrier(sx_engine *e, sx_cmd *c);
/* submitPreRecorded (kernels.zig:147-157): launch and poll to a deadline
 * (timeout_ns == 0 -> the reference's 5 s).  SX_ERR_TIMEOUT like VkFenceTimeout. */
SX_API sx_status sx_submit(sx_engine *e, sx_cmd *c, uint64_t timeout_ns);

/* ---------------------------------------------------------------------------------------
 * Immediate-mode dispatch on device pointers (ComputePipeline.dispatch, pipeline.zig:143-158,
 * as used by test_q4_exec.zig:77-85).  Asynchronous on the engine stream.  Packed weights
 * come from sx_buffer_upload_weights / sx_buffer_repack_device.  Batch rows are contiguous
 * with strides k (inputs) and m (outputs).
 * ------------------------------------------------------------------------------------- */
SX_API sx_status sx_dispatch_gemv(sx_engine *e, sx_quant_mode mode, const void *w_packed,
                                  const float *x, float *y, uint32_t m, uint32_t k,
                                  uint32_t batch);
/* Batch-prefill projection (new: the reference prefills token by token through gemv_q4):
 * y[t][n] (f32, row stride n) = sum_k x[t][k] (bf16) * bf16_rne((q[n][k] - 8) * d[n][k / 32])
 * on the tcgen05 tensor cores, for all T tokens at once.  w_packed: packed Q4_0 (n x k) with
 * finite scales; k % 64 == 0; n % 4 == 0; x and y 16-byte aligned. */
SX_API sx_status sx_dispatch_prefill_gemm(sx_engine *e, const void *w_packed, const void *x_bf16,
                                          float *y, uint32_t t, uint32_t n, uint32_t k);
SX_API sx_status sx_dispatch_gate_up(sx_engine *e, const void *wg_packed, const void *wu_packed,
                                     const float *x, float *y, uint32_t m, uint32_t k,
                                     uint32_t batch);
SX_API sx_status sx_dispatch_rmsnorm(sx_engine *e, const float *x, const float *w, float *y,
                                     uint32_t n, uint32_t batch, float eps);
SX_API sx_status sx_dispatch_add_rmsnorm(sx_engine *e, float *x, const float *r, const float *w,
                                         float *y, uint32_t n, uint32_t batch, float eps,
                                         float scalar);
SX_API sx_status sx_dispatch_qkv_rope(sx_engine *e, const float *q_in, const float *k_in,
                                      const float *v_in, const float *q_norm_w,
                                      const float *k_norm_w, float *q_out, void *k_cache,
                                      void *v_cache, const uint32_t *step_params,
                                      uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
                                      uint32_t rotary_dim, uint32_t k_eq_v, float theta,
                                      float eps, uint32_t total_slots);
SX_API sx_status sx_dispatch_decode_attn(sx_engine *e, const float *q, const void *k_cache,
                                         const void *v_cache, const uint32_t *active_slots,
                                         const uint32_t *step_params, float *out,
                                         uint32_t head_dim, uint32_t kv_dim, uint32_t gqa_ratio,
                                         float scale, uint32_t num_q_heads,
                                         uint32_t total_slots);
/* recordQkvRope followed by recordDecodeAttn (kernels.zig:116-129, qkv_rope.wgsl +
 * decode_attn.wgsl) as the one fused kernel the decode graph runs: q heads and the new k
 * RMS-normalised with their gains and rotated over the first rotary_dim elements, v
 * unit-normalised, the new K/V stored at step_params[1] in the engine's KV precision, then
 * attention of every q head over the slot list (the current slot's K/V taken from the values
 * just stored).  q_in is not modified.  `instances` independent problems run in one launch:
 * instance i reads q_in / k_in / v_in at + i * qkv_stride floats, its caches at
 * + i * total_slots * num_kv * head_dim elements, its slot list at + i * total_slots, its step
 * record at + 4 i, and writes out at + i * num_q * head_dim (several instances need a ring of at
 * most 1024 slots).  Vectors and caches 16-byte aligned; head_dim 64/128/256/512; 1, 2, 4 or 8
 * q heads per kv head. */
SX_API sx_status sx_dispatch_qkv_rope_attn(sx_engine *e, const float *q_in, const float *k_in,
                                           const float *v_in, const float *q_norm_w,
                                           const float *k_norm_w, void *k_cache, void *v_cache,
                                           const uint32_t *active_slots,
                                           const uint32_t *step_params, float *out,
                                           uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
                                           uint32_t rotary_dim, uint32_t k_eq_v, float theta,
                                           float eps, float scale, uint32_t total_slots,
                                           uint32_t instances, uint32_t qkv_stride);
/* The quiescence gate alone on device vectors (asynchronous on the engine stream). */
SX_API sx_status sx_dispatch_quiescence_gate(sx_engine *e, const float *x_curr, float *x_prev,
                                             uint32_t *indirect_args,
                                             const sx_quiescence_gate_pc *pc);
SX_API sx_status sx_dispatch_argmax(sx_engine *e, const float *logits, uint32_t n,
                                    uint32_t *out_token);
/* No counterpart in the reference.  Decode attention that allocates nothing, for callers that
 * may not call cudaMalloc while serving (device memory owned by another allocator or a fixed
 * arena, or allocation forbidden after start-up) and so cannot create an engine.  Same math and
 * arguments as sx_dispatch_decode_attn plus the KV precision (kv_bf16: 1 bf16, 0 f32) and the
 * cudaStream_t to run on.  Its split-over-slots partials live in a fixed 1 MiB array inside
 * the library's device image, held by every GPU that loads libsx until the process exits:
 * requests needing num_q_heads * ceil(total_slots / 32) * (head_dim + 2) * 4 bytes above 1 MiB
 * are rejected with SX_ERR_INVALID.  The first call on a device looks the array's address up
 * (cudaGetSymbolAddress) and sets kernel attributes, so make that first call outside any stream
 * capture.  All calls share the array: calls whose GPU work overlaps (different streams, or
 * threads) race on it.  Every partial is written before it is read, so nothing in it needs to
 * start at zero.  Device-side slot checks skip bad slots but have no error word to report to. */
SX_API sx_status sx_decode_attn_noalloc(const float *q, const void *k_cache, const void *v_cache,
                                        const uint32_t *active_slots,
                                        const uint32_t *step_params, float *out,
                                        uint32_t head_dim, uint32_t kv_dim, uint32_t gqa_ratio,
                                        float scale, uint32_t num_q_heads, uint32_t total_slots,
                                        uint32_t kv_bf16, void *cuda_stream);
/* The quantiser alone: reference-layout block words (Q4 5 / Q8 9 words per 32 values) of a
 * device bf16 matrix into device memory, asynchronous on the engine stream. */
SX_API sx_status sx_dispatch_quantize(sx_engine *e, sx_quant_mode mode, const void *bf16_device,
                                     uint32_t *ref_words_device, uint32_t rows, uint32_t cols);
/* Dequantise a packed Q4 matrix to f32 (nib - 8) * d in reference element order. */
SX_API sx_status sx_dispatch_unpack_q4(sx_engine *e, const void *w_packed, float *out,
                                       uint32_t m, uint32_t k);
/* Synthetic reference-layout blocks (BASELINE distributions), rows [row0, row0 + rows). */
SX_API sx_status sx_dispatch_synth_weights(sx_engine *e, sx_quant_mode mode, uint32_t *ref_out,
                                           uint32_t row0, uint32_t rows, uint32_t cols,
                                           uint64_t seed, uint64_t stream_id);

/* ---------------------------------------------------------------------------------------
 * Model: GpuModelContext (model_gpu.zig:35-197) + gpuDispatchForwardToken
 * (model_dispatch.zig:131-147) for a Q4_0 model with a Q8_0 LM head.
 * ------------------------------------------------------------------------------------- */
typedef struct {
  uint32_t vocab_size, hidden_size, intermediate_size, num_layers;
  uint32_t num_q_heads, num_kv_heads, num_global_kv_heads, head_dim, global_head_dim;
  uint32_t num_anchors, window_size, num_recall;
  uint32_t kv_bf16;          /* 1: bf16 KV cache (build default), 0: f32 (reference)    */
  uint32_t has_post_norms;   /* post_attention / post_feedforward layernorms present     */
  uint32_t full_every;       /* layer l is full attention when (l+1) % full_every == 0  */
  uint32_t attention_k_eq_v; /* types.zig:58                                            */
  float rms_norm_eps, rope_theta, rope_theta_full, attn_scale;
  uint32_t reference_graph;  /* graph of one token: 1 = the reference's op-by-op graph through
                                the record API (14 launches per layer); 0 = the fused graph (5
                                launches per layer: q|k|v, attention, o, gate+up, down); 4 = the
                                fused graph with q|k|v, attention and o as one attention-block
                                kernel (3 launches per layer; one session, one GPU, Q4_0
                                layers, else as 0); 2 = the fused graph's kernels as phases of
                                one persistent cooperative launch per token; 3 = the streaming
                                decode kernel: one cooperative launch per token in which a
                                producer warp per SM streams every layer's weights through a
                                shared-memory ring while the other warps compute (one session,
                                one GPU) */
  uint32_t tp_size;          /* tensor-parallel ranks (0 or 1: one GPU); with tp_size > 1 the
                                model holds rank tp_rank's shard (sx_tp_shard_plan) and must be
                                created with sx_model_create_tp */
  uint32_t tp_rank;
  uint32_t num_sessions;     /* independent decode sessions held by the model (0 or 1: one);
                                each has its own KV cache, ring and clock and they share the
                                weights: sx_decode_batch steps n <= num_sessions of them with
                                one batched pass (config 2 batch 8, config 5 sessions).  At
                                most 8; needs the fused graph (reference_graph 0), tp_size <= 1
                                and a ring of at most 1024 slots. */
  float quiescence_threshold; /* model_gpu.zig:75 quiescence_thresh: layers l >= num_layers / 3
                                are recorded behind the quiescence gate and skipped when the
                                residual entering them moved less than this (mean square) since
                                the last token (model_dispatch.zig:45-118); 0 runs every layer.
                                A positive threshold needs the op-by-op graph
                                (reference_graph 1). */
} sx_model_config;

/* sizeof(sx_model_config): bindings check their mirror of the struct against it. */
SX_API uint32_t sx_model_config_bytes(void);

typedef struct sx_model sx_model;
/* GpuModelContext.init without weights: allocates every device buffer and records the
 * decode and prefill graphs (model_gpu.zig:75-185). */
SX_API sx_status sx_model_create(sx_engine *e, const sx_model_config *cfg, sx_model **out);
SX_API void sx_model_destroy(sx_model *m);
/* Fill all weights with the synthetic checkpoint (seeded, BASELINE distributions). */
SX_API sx_status sx_model_synth_weights(sx_model *m, uint64_t seed);
/* Fill every KV slot with a synthetic past (K = bf16 N(0,1), V unit-RMS): session 0. */
SX_API sx_status sx_model_fill_kv(sx_model *m, uint64_t seed);
/* The same for the KV cache of session `session` (< num_sessions). */
SX_API sx_status sx_model_fill_kv_session(sx_model *m, uint32_t session, uint64_t seed);
/* gpuDispatchForwardToken (model_dispatch.zig:131-147): host x[hidden], clock, slot and the
 * active-slot list in; greedy token out (and the logits when logits_out != NULL).
 * want_logits == 0 runs the prefill graph (no LM head).  Host<->device copies included. */
SX_API sx_status sx_forward_token(sx_model *m, const float *x, uint32_t clock, uint32_t slot,
                                  const uint32_t *active_slots, uint32_t n_active,
                                  int want_logits, uint32_t *token_out, float *logits_out);
/* Batch-8 decode (new; the reference runs one session per forwardToken): one token for each
 * of sessions 0..n-1 (n <= num_sessions) in one pass that streams the weights once.  Row i of
 * x[n][hidden], clock[i], slot[i], the active list active[i * total_slots ..][0, n_active[i])
 * and the greedy token tokens[i] belong to session i; logits_out (optional) is [n][vocab].
 * Equal to n calls of sx_forward_token on n single-session models with those caches. */
SX_API sx_status sx_decode_batch(sx_model *m, uint32_t n, const float *x, const uint32_t *clock,
                                 const uint32_t *slot, const uint32_t *active,
                                 const uint32_t *n_active, int want_logits, uint32_t *tokens,
                                 float *logits_out);
/* Batched prefill (new; the reference prefills with one forwardToken per prompt token,
 * forward.zig:19-75): T tokens of any of the model's sessions in one pass per layer, the
 * projections on the tcgen05 Q4_0 GEMM (sx_dispatch_prefill_gemm).  Token t: embedding row
 * x[t][hidden], session[t] (< num_sessions), clock[t], slot[t] and its ring's active list
 * active[t * total_slots ..][0, n_active[t]) -- exactly what sx_forward_token would take for
 * it.  Every token's K/V is written to its session's cache.  The greedy next token (and,
 * with logits_out, the [n_out][vocab] logits) is returned for the n_out <= 8 token rows
 * out_rows (normally the last prompt token of each session).  Equal to calling
 * sx_forward_token token by token, with the activations entering each projection rounded to
 * bf16.  Rejected (SX_ERR_INVALID) when a slot is written twice in the call or a token lists
 * a slot that a later token of its session rewrites: prompts up to anchors + window tokens
 * from a fresh ring go in one call; once a session's window has wrapped, each call holds one
 * token of it.  Hidden, q and intermediate sizes must be multiples of 64. */
SX_API sx_status sx_prefill_batch(sx_model *m, uint32_t T, const float *x,
                                  const uint32_t *session, const uint32_t *clock,
                                  const uint32_t *slot, const uint32_t *active,
                                  const uint32_t *n_active, uint32_t n_out,
                                  const uint32_t *out_rows, uint32_t *tokens, float *logits_out);
/* Device-resident replay: inputs already in the model's device buffers (sx_model_io). */
SX_API sx_status sx_model_launch(sx_model *m, int want_logits);
/* Asynchronous replay of the n-session step of sx_decode_batch on the engine stream, from
 * the inputs its last call staged (benchmarks: the device time of a batched step without the
 * host's per-step work).  The first use of an n records its graph (outside stream capture). */
SX_API sx_status sx_model_launch_batch(sx_model *m, uint32_t n, int want_logits);
typedef struct {
  float *x;            /* device f32[hidden]                  */
  uint32_t *slots;     /* device u32[total_slots]             */
  uint32_t *step;      /* device u32[4] {clock, slot, n, 0}   */
  uint32_t *token;     /* device u32[1]                       */
  float *logits;       /* device f32[vocab]                   */
  float *normed;       /* device f32[hidden]                  */
} sx_model_io;
SX_API sx_status sx_model_get_io(sx_model *m, sx_model_io *io);
/* Device pointers of layer weights / caches (tests and benchmarks). */
SX_API void *sx_model_kcache(sx_model *m, uint32_t layer);
SX_API void *sx_model_vcache(sx_model *m, uint32_t layer);
SX_API uint64_t sx_model_weight_bytes(sx_model *m);
SX_API uint32_t sx_model_kernels_per_token(sx_model *m, int want_logits);

/* ---------------------------------------------------------------------------------------
 * The recall tier on the device: DiffArchive (memory.zig:19-151) and integrateMemory
 * (memory_inject.zig:17-46) over the model's own KV caches (session 0).  The reference keeps
 * its archive on the CPU and copies K/V through the CPU ring, which its GPU decode never reads;
 * here the archive, its K/V rows and the recall slots all live in device memory.
 * ------------------------------------------------------------------------------------- */
/* memory.zig:5-7 SalienceConfig (defaults alpha 1, beta 0.5, gamma 1, lambda 1/2048) */
typedef struct {
  float alpha, beta, gamma, lambda;
} sx_salience_config;
typedef struct sx_archive sx_archive;
/* DiffArchive.initWithKV (memory.zig:28-52) for model m: `capacity` unit vectors of
 * hidden_size floats, their metadata and each entry's K/V rows of every layer in the model's
 * cache format (1 <= capacity <= 16384; the reference uses 8192, main.zig:19).  cfg NULL: the
 * defaults. */
SX_API sx_status sx_archive_create(sx_model *m, uint32_t capacity, const sx_salience_config *cfg,
                                   sx_archive **out);
SX_API void sx_archive_destroy(sx_archive *a);
/* integrateMemory (memory_inject.zig:17-46) after the token at `clock` was decoded with logits
 * (its final normed state is the query): when the state's cosine similarity to the previous
 * token's is below 0.98 it is appended with salience |delta| and the token's K/V rows; the
 * min(num_recall, count) entries of highest score alpha cos + beta exp(-lambda dt) +
 * gamma salience (memory.zig:113-151, the reference's selection order) are copied into recall
 * slots anchors + window + rank of every layer's cache, and `ring`'s recall tier is rewritten
 * with their timestamps (clearRecall + writeRecallKV).  Synchronous.  n_selected / selected
 * (num_recall entries, archive indices in rank order) are optional. */
SX_API sx_status sx_archive_integrate(sx_archive *a, sx_ring *ring, uint64_t clock,
                                     uint32_t *n_selected, uint32_t *selected);
SX_API uint32_t sx_archive_count(const sx_archive *a);
/* entry i: unit vector (hidden_size floats), timestamp, last access, access count, salience
 * (any pointer may be NULL) */
SX_API sx_status sx_archive_entry(sx_archive *a, uint32_t i, float *vec, uint64_t *timestamp,
                                  uint64_t *last_accessed, uint32_t *access_count,
                                  float *salience);

/* ---------------------------------------------------------------------------------------
 * Tensor-parallel decode (new: the reference runs on one GPU).  One engine, communicator and
 * model per GPU.  Column-parallel q (num_q_heads / N heads), k / v (num_kv_heads / N and
 * num_global_kv_heads / N heads: the GQA ratio is preserved), gate / up (intermediate / N
 * rows); row-parallel o and down (their K split the same way) followed by a sum all-reduce
 * of the hidden vector, twice per layer; vocabulary-parallel LM head (vocab / N rows) whose
 * local argmax candidates {value, index} are all-gathered and merged on device (lowest index
 * on ties, logits[0] = NaN -> token 0 as on one GPU).  Norms, residual stream and x are
 * replicated; the KV cache holds the rank's kv heads.  Collectives: NCCL, captured in the
 * per-token graph (graph mode 0).
 * ------------------------------------------------------------------------------------- */
typedef struct {
  uint32_t q_heads, q_head0;                 /* this rank's q heads [q_head0, +q_heads)      */
  uint32_t kv_heads, kv_head0;               /* sliding-layer kv heads                        */
  uint32_t global_kv_heads, global_kv_head0; /* full-attention-layer kv heads                 */
  uint32_t inter, inter0;                    /* intermediate rows / down-projection columns   */
  uint32_t vocab, vocab0;                    /* LM-head rows                                  */
} sx_tp_shard;
/* Host only: the shard of rank cfg->tp_rank of cfg->tp_size; SX_ERR_INVALID when the heads,
 * intermediate size (in 32-column blocks) or vocabulary do not divide evenly. */
SX_API sx_status sx_tp_shard_plan(const sx_model_config *cfg, sx_tp_shard *out);

typedef struct sx_comm sx_comm;
/* NCCL unique id (128 bytes) made on one rank and shared with the others by the caller. */
SX_API sx_status sx_comm_unique_id(uint8_t id[128]);
SX_API sx_status sx_comm_create(sx_engine *e, const uint8_t id[128], uint32_t nranks,
                                uint32_t rank, sx_comm **out);
SX_API void sx_comm_destroy(sx_comm *c);
/* The all-reduce of the row-parallel o / down outputs: NCCL, or (use_nccl = 0) a one-shot
 * peer-to-peer kernel over NVLink -- each rank stores its vector into every rank's workspace
 * (mapped through CUDA IPC when the communicator is made), releases a flag, waits for all the
 * flags with a bounded poll and sums in rank order.  Choose before creating the model (its
 * graphs capture the choice).  sx_comm_create maps the workspaces collectively and all ranks
 * agree on the result, so selecting the peer kernel succeeds on every rank or fails
 * (SX_ERR_UNSUPPORTED) on every rank.  The reference has no multi-GPU path. */
SX_API sx_status sx_comm_set_allreduce(sx_comm *c, int use_nccl);
SX_API int sx_comm_allreduce_is_nccl(const sx_comm *c);
/* The row-parallel all-reduce alone (the op the per-token graph captures twice per layer):
 * in-place sum of count floats at the device pointer buf over all ranks, asynchronous on the
 * engine stream.  With the peer kernel, buf must be 16-byte aligned and count <= 16384; a
 * rank that does not arrive within the wait limit makes the call record a device error
 * (SX_ERR_DEVICE from the next sx_engine_sync) instead of hanging. */
SX_API sx_status sx_comm_allreduce(sx_comm *c, float *buf, uint32_t count);
/* How long the peer all-reduce waits for the other ranks' flags (default 2 s); applies to
 * calls launched or graphs recorded after it. */
SX_API sx_status sx_comm_set_wait_ns(sx_comm *c, uint64_t wait_ns);
/* sx_model_create for a tensor-parallel rank: cfg->tp_size / tp_rank must match the
 * communicator; cfg->reference_graph must be 0. */
SX_API sx_status sx_model_create_tp(sx_engine *e, const sx_model_config *cfg, sx_comm *comm,
                                    sx_model **out);

#ifdef __cplusplus
}
#endif
#endif /* SX_H */
