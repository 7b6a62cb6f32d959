// sx_internal.h -- launchers shared between the kernel files and the host engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sx {

// GEMV input prologues and epilogues (see sx_gemv.cu)
enum GemvPrologue : int { kProNone = 0, kProNorm = 1, kProResid = 2 };
enum GemvEpilogue : int { kEpiPlain = 0, kEpiArgmax = 2 };

struct GemvArgs {
  // up to three row-concatenated matrices (e.g. q | k | v); w[s][1] is the up matrix of the
  // fused GeGLU; y[s] receives the rows of segment s
  const void *w[3][2];
  float *y[3];
  uint32_t rows[3];
  uint32_t tiles[3];      // tiles_of(rows[s]); 0 for unused segments
  uint32_t row_base[3];   // global row index of segment s (argmax ids)
  uint32_t k, batch, ldy;
  const float *x;         // [batch][ldx] input, or the residual stream for kProResid
  uint32_t ldx;
  int pro;
  const float *pro_w;       // norm gain
  const float *pro_mlp;     // kProResid: sublayer output added to x
  const float *pro_post_w;  // kProResid: optional post-norm gain of the sublayer output
  float *pro_x_out;         // kProResid: updated residual stream (must not alias x)
  float *pro_norm_out;      // optional: the normed input rows, written by CTA 0
  // kProResid: the sublayer output is the sum of pro_mlp_parts vectors pro_mlp_ld floats
  // apart, added in order (0 or 1: one vector)
  uint32_t pro_mlp_parts, pro_mlp_ld;
  float pro_scalar;         // kProResid: layer scalar
  float eps;
  int epi;
  uint32_t *token;          // kEpiArgmax: [batch] greedy ids
  uint32_t *cand;           // kEpiArgmax, optional: [batch][4] {value bits, global index,
                            // 1 if this call holds logits row 0 and it is NaN, 0}
  // scratch (engine-owned): split-tile records, per-tile arrival counters (zero at rest),
  // per-worker argmax candidates, the argmax arrival counter (zero at rest)
  float *part;
  uint32_t *tile_cnt;
  float *best_v;
  uint32_t *best_i;
  uint32_t *done_cnt;
  uint32_t *err;
  // optional L2 prefetch issued before the dependency wait (standalone launches): the rows
  // pf_slots[0 .. min(pf_step[2], pf_max)) of pf_base[0] and pf_base[1] (pf_row_bytes each,
  // a multiple of 16), i.e. the live K/V cache rows the following attention reads
  const uint32_t *pf_slots, *pf_step;
  const void *pf_base[2];
  uint32_t pf_row_bytes, pf_max;
  const uint32_t *gate;  // indirect dispatch record {x, y, z}: a zero skips the call (or null)
};

// Per-device kernel attributes (dynamic shared memory limits); called at engine creation,
// never inside a stream capture.
cudaError_t prepare_gemv_kernels();
cudaError_t prepare_ops_kernels();

// qt: 4 or 8.  geglu: fused gate+up with gelu_tanh(gate) * up epilogue.  pdl: launch with
// programmatic stream serialization (the kernel prefetches weights before waiting).
cudaError_t launch_gemv(int qt, bool geglu, const GemvArgs &a, int num_sms, cudaStream_t s,
                        bool pdl);
size_t gemv_smem_bytes(int qt, uint32_t k, uint32_t batch, bool geglu, bool prologue);
size_t gemv_part_bytes(int num_sms);
// The kernel streams the chunks of all segments as one run starting at w[0][m]: segment s
// must begin where segment s - 1 ends.
bool gemv_segments_contiguous(const GemvArgs &a, int qt, int nmat);
size_t gemv_workers(int num_sms);
constexpr uint32_t kGemvPrologueMaxK = 4096;  // fused norm prologues hold K / 512 <= 8 per thread
constexpr uint32_t kMaxGemvTiles = 262144;

// bf16-weight GEMV of the engine's mode none (sx_gemv_bf16.cu): y[b][r] = W[r] . x[b] with
// row-major bf16 W (k % 8 == 0, 16-byte aligned rows and x), or the GeGLU of two matrices
cudaError_t launch_gemv_bf16(bool geglu, const uint16_t *w0, const uint16_t *w1, const float *x,
                             float *y, uint32_t m, uint32_t k, uint32_t batch, int num_sms,
                             cudaStream_t s, const uint32_t *gate = nullptr);
// synthetic bf16(0.02 N(0,1)) weights, element i of (seed, stream)
cudaError_t launch_synth_bf16(uint16_t *dst, uint64_t n, uint64_t seed, uint64_t stream_id,
                              cudaStream_t s);

// quantizeMatrix on the device: nblocks 32-value bf16 blocks -> reference block words
cudaError_t launch_quantize(int qt, const void *bf16, uint32_t *ref, uint64_t nblocks,
                            cudaStream_t s);
cudaError_t launch_repack(int qt, const uint32_t *ref, void *packed, uint32_t m, uint32_t k,
                          cudaStream_t s);
cudaError_t launch_unpack_q4(const void *packed, float *out, uint32_t m, uint32_t k,
                             cudaStream_t s);
// Synthetic reference-layout rows [row0, row0 + rows) x 32-column blocks [blk0, blk0 + k / 32)
// of a matrix with nb_global blocks per row (nb_global = 0: k / 32, the whole row).
cudaError_t launch_synth_ref(int qt, uint32_t *ref, uint32_t row0, uint32_t rows, uint32_t k,
                             uint64_t seed, uint64_t stream_id, cudaStream_t s,
                             uint32_t blk0 = 0, uint32_t nb_global = 0);
cudaError_t launch_synth_gain(float *dst, uint32_t n, uint64_t seed, uint64_t stream_id,
                              cudaStream_t s);
// Synthetic past K/V: rows [slot][local kv head] of a cache holding heads
// [head0, head0 + heads) of heads_global (the values of the one-GPU model's heads).
cudaError_t launch_fill_kv(void *k_cache, void *v_cache, int kv_bf16, uint32_t rows,
                           uint32_t head_dim, float eps, uint64_t seed, uint32_t layer,
                           cudaStream_t s, uint32_t heads = 1, uint32_t head0 = 0,
                           uint32_t heads_global = 1);

struct NormArgs {
  float *x;           // residual stream (add variant: updated in place)
  const float *r;     // added vector (add variant)
  const float *w;     // gain
  float *y;           // output
  uint32_t n, batch, ld;
  float eps, scalar;
  const uint32_t *gate = nullptr;  // indirect dispatch record (see gate_closed)
};
cudaError_t launch_rmsnorm(bool add, const NormArgs &a, cudaStream_t s);

struct QkvRopeArgs {
  const float *q_in, *k_in, *v_in, *q_norm_w, *k_norm_w;
  float *q_out;
  void *k_cache, *v_cache;
  const uint32_t *step;  // {clock, slot, n_active, 0}
  const float *inv_freq;
  uint32_t num_q, num_kv, head_dim, rotary_dim, k_eq_v, kv_bf16, total_slots;
  float eps;
  uint32_t *err;
  const uint32_t *gate = nullptr;  // indirect dispatch record (see gate_closed)
};
cudaError_t launch_qkv_rope(const QkvRopeArgs &a, cudaStream_t s);

// quiescence_gate.wgsl: mean (x - x_prev)^2 over h (32-lane strided sums and tree, as the
// shader), x_prev = x, then num_cmds dispatch records {targets[c], 1, 1} (the layer runs:
// mean >= threshold_sq or threshold_sq <= 0) or {0, 0, 0} at ind + 3 (base + c)
struct GateArgs {
  const float *x;
  float *x_prev;
  uint32_t *ind;
  uint32_t h;
  float threshold_sq;
  uint32_t base, num_cmds;
  uint32_t targets[16];
};
cudaError_t launch_quiescence_gate(const GateArgs &a, cudaStream_t s);

struct AttnArgs {
  const float *q;
  const void *k_cache, *v_cache;
  const uint32_t *slots;
  const uint32_t *step;
  float *out;
  float *part;           // scratch: [num_q][nchunks][head_dim + 2]
  uint32_t head_dim, kv_dim, gqa, num_q, total_slots, kv_bf16;
  float scale;
  uint32_t *err;
  const uint32_t *gate = nullptr;  // indirect dispatch record (see gate_closed)
};
size_t attn_scratch_bytes(uint32_t num_q, uint32_t total_slots, uint32_t head_dim);
cudaError_t launch_decode_attn(const AttnArgs &a, cudaStream_t s);

struct AttnFusedArgs {
  const float *q, *k, *v;          // raw projections of this token
  const float *q_norm_w, *k_norm_w;
  const float *inv_freq;
  void *k_cache, *v_cache;
  const uint32_t *slots, *step;
  float *out;
  float *part;                     // [num_q][nchunks][head_dim + 2]
  uint32_t *cnt;                   // [num_kv], zero at rest
  uint32_t head_dim, kv_dim, num_q, num_kv, rotary_dim, k_eq_v, kv_bf16, total_slots;
  float scale, eps;
  uint32_t *err;
  // independent sessions (cluster form only): session z < sessions reads q/k/v at + z qkv_ld
  // floats, its caches at + z cache_ld elements, slots at + z total_slots, step at + 4 z, and
  // writes out at + z out_ld floats
  uint32_t sessions, qkv_ld, out_ld;
  uint64_t cache_ld;
};
cudaError_t launch_attn_fused(const AttnFusedArgs &a, cudaStream_t s, bool pdl);
// rings up to this many live slots run the cluster form (16 CTAs x 64 slots per kv head)
constexpr uint32_t kAttnClusterMaxSlots = 1024;

// The attention block of one decode layer as one kernel (sx_attn_block.cu): q|k|v projection
// with its residual + input-norm prologue, q/k norm + RoPE + cache write, attention over the
// active slots, and the o projection split by kv-head group into num_kv partial rows.
struct AttnBlockArgs {
  GemvArgs g;         // q|k|v: w[0..2][0] = wq, wk, wv (packed Q4_0), y[0..2] = q, k, v rows,
                      // k = hidden size, batch 1, the input prologue fields
  AttnFusedArgs at;   // q/k/v (= g.y), norm gains, RoPE table, caches, slots, step, scale, ...
  const void *wo;     // packed Q4_0 o projection [o_rows][num_q * head_dim]
  float *opart;       // [num_kv][o_rows]: the o projection of each group's columns
  float *rec;         // [num_kv][ctas][G][head_dim + 2] attention records
  uint32_t *cnt;      // [2 * num_kv + 1] arrival counters, zero at rest (the kernel clears them)
  uint32_t o_rows;    // hidden size
  uint32_t ctas;      // CTAs per kv-head group
  uint32_t max_slots; // active slots per CTA the shared memory holds
  uint32_t o_tiles;   // o-projection tiles per CTA the shared memory holds
  uint64_t wait_ns;   // limit of each counter wait (GPU time)
};
struct AttnBlockPlan {
  uint32_t ctas, max_slots, o_tiles, smem;
};
// false when the shape has no attention-block form (head_dim, GQA ratio, ring or shared memory)
bool attn_block_plan(uint32_t hidden, uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
                     uint32_t total_slots, bool kv_bf16, int num_sms, uint32_t smem_limit,
                     AttnBlockPlan *plan);
cudaError_t launch_attn_block(const AttnBlockArgs &a, cudaStream_t s);
constexpr uint32_t kAttnBlockSmemLimit = 227 * 1024 - 1024;  // dynamic, below the opt-in max

// The cluster attention with the o projection of each kv head's q heads folded in
// (sx_attn_o.cu): one session, one GPU, Q4_0 o projection; the o rows come out as one partial
// vector per kv head, opart[kv head][row], which the gate+up prologue adds in kv-head order.
struct AttnOArgs {
  AttnFusedArgs at;   // the fused attention's arguments (out: the G x head_dim rows per head)
  const void *wo;     // packed Q4_0 o projection [o_rows][num_q * head_dim]
  float *opart;       // [num_kv][o_rows]
  uint32_t o_rows;    // hidden size
  uint32_t o_tiles;   // W_o tiles per CTA the shared memory holds (attn_o_plan)
  uint32_t cta_slots; // ring slots per CTA (attn_o_plan: 40 for rings of up to 640 slots, else 64)
};
bool attn_o_plan(uint32_t o_rows, uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
                 uint32_t total_slots, uint32_t smem_limit, uint32_t *o_tiles,
                 uint32_t *cta_slots);
cudaError_t launch_attn_o(const AttnOArgs &a, cudaStream_t s);
cudaError_t prepare_attn_o_kernels();
cudaError_t prepare_attn_block_kernels();

// ---------------------------------------------------------------------------------------
// Batched prefill (sx_prefill_model.cu): per-token kernels around the tcgen05 GEMMs.
struct PfNormArgs {
  const float *x;        // [rows][n] residual stream (input)
  const float *mlp;      // optional sublayer output: x = (x + post?(mlp)) * scalar first
  const float *post_w;   // optional post-norm gain of mlp
  float scalar;
  float *x_out;          // updated residual stream (may equal x), when mlp is set
  const float *w;        // norm gain
  void *out;             // [rows][n] bf16 or f32
  const uint32_t *rows;  // optional: input row of each output row
  uint32_t n;
  float eps;
};
cudaError_t launch_pf_norm(const PfNormArgs &a, uint32_t rows, bool out_bf16, cudaStream_t s);

struct PfQkvArgs {
  const float *y;  // [tokens][ldy]: q (num_q heads) | k (num_kv) | v (num_kv) projections
  uint32_t ldy;
  const float *q_norm_w, *k_norm_w, *inv_freq;
  float *q_out;    // [tokens][num_q * head_dim]
  void *k_cache, *v_cache;  // [sessions][total_slots][num_kv][head_dim]
  uint64_t cache_ld;        // elements per session
  const uint32_t *sess, *clock, *slot;  // per token
  uint32_t sessions, total_slots, num_q, num_kv, head_dim, rotary_dim, k_eq_v, kv_bf16;
  float eps;
  uint32_t *err;
};
cudaError_t launch_pf_qkv_rope(const PfQkvArgs &a, uint32_t tokens, cudaStream_t s);

struct PfAttnArgs {
  const float *q;           // [tokens][num_q * head_dim]
  const void *k_cache, *v_cache;
  uint64_t cache_ld;
  const uint32_t *sess, *slots, *count;  // per token: session, active list [total_slots], n
  void *out;                // [tokens][num_q * head_dim] bf16
  uint32_t tokens, sessions, total_slots, num_q, num_kv, head_dim, kv_bf16;
  float scale;
  uint32_t *err;
  // tensor-core form (pf_attn_tc_ok): work items {first token, tokens} of at most
  // pf_attn_tc_tokens(G) consecutive tokens of one session; n_items of them
  const uint32_t *items;
  uint32_t n_items;
};
cudaError_t launch_pf_attn(const PfAttnArgs &a, cudaStream_t s);
// whether the prefill attention of this shape runs on the tensor cores (then a.items is read)
bool pf_attn_tc_ok(const PfAttnArgs &a);
// tokens per tensor-core work item for G q heads per kv head (64 query rows per CTA)
inline uint32_t pf_attn_tc_tokens(uint32_t g) { return g ? 64u / g : 0u; }
cudaError_t launch_pf_geglu(const float *g, const float *u, void *h, size_t count, cudaStream_t s);

// ---------------------------------------------------------------------------------------
// Persistent decode kernel (sx_persist.cu): one cooperative launch runs a table of phases on
// one CTA per SM with grid barriers between consecutive phases.
enum PhaseKind : uint32_t { kPhaseGemv = 0, kPhaseAttn = 1 };
struct Phase {
  uint32_t kind;
  uint32_t variant;         // kernel instantiation (persist_gemv_variant / persist_attn_variant)
  uint32_t prefetch_after;  // GEMV: first chunks issued after this phase (kNoPhase: at start)
  uint32_t smem_off;        // GEMV: end of its shared-memory layout; attention: start of
                            // the two work items' shared memory
  GemvArgs g;
  AttnFusedArgs at;
};
constexpr uint32_t kNoPhase = 0xFFFFFFFFu;
// Shared memory of the persistent kernel and where its two attention work items start.
uint32_t persist_smem_bytes();
uint32_t persist_attn_offset(const AttnFusedArgs &a);
// false when the call has no instantiation in the persistent kernel (batch > 4, no ring fits)
bool persist_gemv_variant(int qt, bool geglu, const GemvArgs &a, uint32_t smem_limit,
                          uint32_t *variant, uint32_t *smem_end);
bool persist_attn_variant(const AttnFusedArgs &a, uint32_t *variant);
cudaError_t prepare_persist_kernel();

// Streaming decode kernel (sx_stream.cu): the same phase table as one cooperative launch whose
// producer warp streams every GEMV phase's weights through a shared-memory ring.  ctr: one
// completion counter per phase plus an abort word (n + 1 words), zeroed before every launch.
uint32_t stream_smem_bytes();
uint32_t stream_threads();
// false when the call has no streaming form (batch > 1, fewer than 16 block pairs, ...)
bool stream_gemv_variant(int qt, bool geglu, const GemvArgs &a, int num_sms, uint32_t *variant);
bool stream_attn_variant(const AttnFusedArgs &a, uint32_t *variant);
cudaError_t prepare_stream_kernel();
cudaError_t launch_stream(const Phase *phases, uint32_t n, uint32_t *ctr, uint32_t *err,
                          int num_sms, cudaStream_t s);

// The recall tier on the device (sx_archive.cu): DiffArchive + integrateMemory over the
// model's caches.  Capacity up to kArchiveMaxCapacity entries (the selection holds every score
// in shared memory).
constexpr uint32_t kArchiveMaxCapacity = 16384;
struct ArchiveLayer {
  void *k_cache, *v_cache;  // session 0's cache of the layer, [slot][kv_dim]
  uint32_t kv_dim;
};
struct ArchiveArgs {
  const float *normed;      // the token's final normed state [dim]
  float *prev;              // the previous token's [dim]
  float *vectors;           // [capacity][dim] unit vectors
  uint64_t *timestamp, *last_accessed;
  uint32_t *access_count;
  float *salience;
  void *kv;                 // [capacity][layers][2][max_kv] in the cache format
  float *scores;            // [capacity]
  uint32_t *state;          // count, write_head, appended, append index, selected count
  uint32_t *selected;       // [num_recall] archive indices in rank order
  uint64_t *sel_ts;         // [num_recall] their timestamps
  const ArchiveLayer *layers;
  uint32_t dim, capacity, num_layers, max_kv, kv_bf16, num_recall, recall_start, slot;
  uint64_t clock;
  float alpha, beta, gamma, lambda;
};
cudaError_t prepare_archive_kernels();
cudaError_t launch_archive_integrate(const ArchiveArgs &a, cudaStream_t s);

// Batch-prefill Q4_0 projection GEMM (sx_prefill.cu): y[t][n] = x[t][:] . bf16(deq(w[n][:]))
cudaError_t prepare_prefill_kernel();
cudaError_t launch_prefill_q4(const void *w, const void *x, float *y, uint32_t t, uint32_t n,
                              uint32_t k, uint32_t ldy, uint32_t *err, cudaStream_t s);
// bar: two words (arrival count, abort), cleared by the caller before every launch
cudaError_t launch_persist(const Phase *phases, uint32_t n, uint32_t *bar, uint32_t *err,
                           int num_sms, cudaStream_t s);

cudaError_t launch_argmax(const float *logits, uint32_t n, uint32_t *out, void *scratch,
                          size_t scratch_bytes, cudaStream_t s);
size_t argmax_scratch_bytes();

}  // namespace sx
