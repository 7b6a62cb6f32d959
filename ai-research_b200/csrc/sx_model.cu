// sx_model.cu -- GpuModelContext (src/gpu/model_gpu.zig:35-197) and the per-token dispatch
// (src/gpu/model_dispatch.zig:103-147) on top of the public record API of include/sx.h.
//
// The decode graph is recorded exactly like recordForwardGraph/recordLayerDirect: the same
// descriptor-set bindings (model_gpu.zig:140-168) and the same op order, then captured into
// a CUDA graph that is replayed per token.  Quiescence gating (recordLayerIndirect) runs
// every layer at the reference's default threshold 0.0, so all layers are recorded direct.
#include <cmath>
#include <cstring>
#include <vector>

#include "sx_common.cuh"
#include "sx_host.h"
#include "sx_internal.h"

namespace {

struct LayerBufs {
  uint32_t head_dim = 0, rot = 0, num_kv = 0, q_dim = 0, kv_dim = 0, k_eq_v = 0;
  uint32_t kv_head0 = 0, num_kv_global = 0;  // this rank's kv heads within the layer's
  float theta = 0.0f, layer_scalar = 1.0f;
  sx_buffer *in_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  sx_buffer *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr;
  sx_buffer *wg = nullptr, *wu = nullptr, *wd = nullptr;
  sx_buffer *pre_ffn = nullptr, *post_attn = nullptr, *post_ffn = nullptr;
  sx_buffer *kc = nullptr, *vc = nullptr;
  sx_set *s_input_norm = nullptr, *s_q = nullptr, *s_k = nullptr, *s_v = nullptr;
  sx_set *s_qkv_rope = nullptr, *s_attn = nullptr, *s_o = nullptr, *s_gate_up = nullptr;
  sx_set *s_down = nullptr, *s_pre_ffn = nullptr, *s_post_attn = nullptr, *s_post_ffn = nullptr;
  sx_set *s_post_ffn_add = nullptr;
  sx_buffer *x_prev = nullptr;  // quiescence-gate history (model_gpu.zig:132), zero at start
  sx_set *s_gate = nullptr;     // {x, x_prev, indirect records} (model_gpu.zig:156)
  // the layer's attention block as one kernel (sx_attn_block.cu); ctas == 0: not eligible
  sx::AttnBlockPlan ab{};
  // the cluster attention with the o projection folded in (sx_attn_o.cu); 0: not eligible
  uint32_t ao_tiles = 0, ao_slots = 0;
};

enum Tensor : uint32_t {
  T_INPUT_NORM = 0, T_Q = 1, T_K = 2, T_V = 3, T_O = 4, T_QNORM = 5, T_KNORM = 6,
  T_POST_ATTN = 7, T_PRE_FFN = 8, T_GATE = 9, T_UP = 10, T_DOWN = 11, T_POST_FFN = 12,
  T_SCALAR = 13,
};
uint64_t stream_of(uint32_t layer, uint32_t kind) { return (uint64_t)(layer + 1) * 64 + kind; }

}  // namespace

struct sx_model {
  sx_engine *e = nullptr;
  sx_model_config c{};
  // tensor parallelism: this rank's shard (the whole model when comm == nullptr)
  sx_comm *comm = nullptr;
  sx_tp_shard tp{};
  uint32_t nq = 0, I = 0, V = 0;  // local q heads, intermediate rows, vocabulary rows
  sx_buffer *cand = nullptr, *cand_all = nullptr;  // LM-head argmax candidates (local / all)
  uint32_t total_slots = 0, max_q = 0, max_kv = 0;
  std::vector<LayerBufs> L;
  sx_buffer *x = nullptr, *x2 = nullptr, *normed = nullptr, *q = nullptr, *k = nullptr, *v = nullptr;
  sx_buffer *attn_out = nullptr, *slots = nullptr, *act = nullptr, *mlp_out = nullptr;
  sx_buffer *logits = nullptr, *token = nullptr, *step = nullptr;
  sx_buffer *lm_head = nullptr, *final_norm = nullptr;
  sx_buffer *ind = nullptr;  // 16 dispatch records of 12 bytes per layer (model_gpu.zig:107)
  // attention-block kernels (fused graph, one session, one GPU, Q4_0 layers): the o
  // projection's per-group partial rows, the attention records, per-layer arrival counters
  sx_buffer *ab_opart = nullptr, *ab_rec = nullptr, *ab_cnt = nullptr;
  uint32_t ab_cnt_words = 0;  // counter words per layer
  sx_set *s_final_norm = nullptr, *s_logits = nullptr, *s_argmax = nullptr;
  sx_cmd *cmd[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};  // [want_logits][io]
  // independent sessions: activation rows [S][...], KV caches [S][slots][kv_dim] (session 0
  // first, so the one-session graphs see exactly session 0), q | k | v rows packed per
  // session with the layer's stride; batched graphs [sessions in the step][want_logits]
  uint32_t S = 1, max_base = 0;
  sx_buffer *qkv = nullptr;
  sx_cmd *bcmd[9][2] = {};
  // batched-prefill scratch, grown to the largest call (sx_prefill_batch)
  uint64_t pf_T = 0;
  std::vector<void *> pf;
  float *h_x = nullptr;
  uint32_t *h_slots = nullptr, *h_step = nullptr, *h_token = nullptr;
  std::vector<sx_buffer *> buffers;
  std::vector<sx_set *> sets;
  uint64_t weight_bytes = 0;
  // layer weight format = the engine mode (kernels.zig:36-41): Q4_0, Q8_0 or bf16 (none); the
  // LM head is Q8_0 in the quantised modes and bf16 in mode none (model_gpu.zig:161)
  sx_quant_mode lmode = SX_QUANT_Q4, hmode = SX_QUANT_Q8;
  int lqt = 4;  // GEMV format code of the layers: 4, 8, 0 (bf16)
};

namespace {

sx_status mk_buf(sx_model *m, uint64_t bytes, sx_buffer **out) {
  sx_status st = sx_buffer_create(m->e, bytes ? bytes : 4, out);
  if (st == SX_OK) m->buffers.push_back(*out);
  return st;
}

// a non-owning window [off, off + bytes) of an allocation made with mk_buf
sx_status mk_view(sx_model *m, sx_buffer *base, uint64_t off, uint64_t bytes, sx_buffer **out) {
  sx_status st = sx_buffer_wrap(m->e, static_cast<uint8_t *>(base->d) + off, bytes, out);
  if (st == SX_OK) m->buffers.push_back(*out);
  return st;
}

sx_status mk_set(sx_model *m, std::vector<sx_buffer *> bufs, sx_set **out) {
  sx_status st = sx_set_create(m->e, bufs.data(), (uint32_t)bufs.size(), out);
  if (st == SX_OK) m->sets.push_back(*out);
  return st;
}

#define M_TRY(expr)               \
  do {                            \
    sx_status _s = (expr);        \
    if (_s != SX_OK) return _s;   \
  } while (0)

sx_status alloc_model(sx_model *m) {
  const sx_model_config &c = m->c;
  M_TRY(sx_tp_shard_plan(&c, &m->tp));
  m->nq = m->tp.q_heads;
  m->I = m->tp.inter;
  m->V = m->tp.vocab;
  const uint32_t H = c.hidden_size, I = m->I, V = m->V;
  m->total_slots = c.num_anchors + c.window_size + c.num_recall;
  m->L.resize(c.num_layers);
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    LayerBufs &B = m->L[l];
    // loader.zig:36-42 per-layer shapes
    bool full = c.full_every && ((l + 1) % c.full_every == 0);
    B.head_dim = full ? c.global_head_dim : c.head_dim;
    B.rot = full ? B.head_dim / 4 : B.head_dim;
    B.num_kv = full ? m->tp.global_kv_heads : m->tp.kv_heads;
    B.kv_head0 = full ? m->tp.global_kv_head0 : m->tp.kv_head0;
    B.num_kv_global = full ? c.num_global_kv_heads : c.num_kv_heads;
    B.q_dim = m->nq * B.head_dim;
    B.kv_dim = B.num_kv * B.head_dim;
    B.k_eq_v = (full && c.attention_k_eq_v) ? 1u : 0u;
    B.theta = full ? c.rope_theta_full : c.rope_theta;
    if (B.q_dim > m->max_q) m->max_q = B.q_dim;
    if (B.kv_dim > m->max_kv) m->max_kv = B.kv_dim;
    if (B.q_dim + 2 * B.kv_dim > m->max_base) m->max_base = B.q_dim + 2 * B.kv_dim;
  }
  const uint64_t S = m->S = c.num_sessions > 1 ? c.num_sessions : 1;
  M_TRY(mk_buf(m, 4ull * H * S, &m->x));
  M_TRY(mk_buf(m, 4ull * H * S, &m->x2));
  M_TRY(mk_buf(m, 4ull * H * S, &m->normed));
  M_TRY(mk_buf(m, 4ull * m->max_q, &m->q));
  M_TRY(mk_buf(m, 4ull * m->max_kv, &m->k));
  M_TRY(mk_buf(m, 4ull * m->max_kv, &m->v));
  M_TRY(mk_buf(m, 4ull * m->max_base * S, &m->qkv));
  M_TRY(mk_buf(m, 4ull * m->max_q * S, &m->attn_out));
  M_TRY(mk_buf(m, 4ull * m->total_slots * S, &m->slots));
  M_TRY(mk_buf(m, 4ull * I * S, &m->act));
  M_TRY(mk_buf(m, 4ull * H * S, &m->mlp_out));
  M_TRY(mk_buf(m, 4ull * V * S, &m->logits));
  M_TRY(mk_buf(m, 64, &m->token));
  M_TRY(mk_buf(m, 16, &m->cand));
  M_TRY(mk_buf(m, 16ull * (c.tp_size > 1 ? c.tp_size : 1), &m->cand_all));
  M_TRY(mk_buf(m, 16 * S < 64 ? 64 : 16 * S, &m->step));
  const size_t kvb = c.kv_bf16 ? 2 : 4;
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    LayerBufs &B = m->L[l];
    M_TRY(mk_buf(m, 4ull * H, &B.in_norm));
    M_TRY(mk_buf(m, 4ull * B.head_dim, &B.q_norm));
    M_TRY(mk_buf(m, 4ull * B.head_dim, &B.k_norm));
    M_TRY(mk_buf(m, 4ull * H, &B.pre_ffn));
    M_TRY(mk_buf(m, 4ull * H, &B.post_attn));
    M_TRY(mk_buf(m, 4ull * H, &B.post_ffn));
    // q | k | v back to back: the fused projection streams them as one run of chunks
    const uint64_t qb = sx_packed_bytes(B.q_dim, H, m->lmode);
    const uint64_t kvb_w = sx_packed_bytes(B.kv_dim, H, m->lmode);
    sx_buffer *qkv = nullptr;
    M_TRY(mk_buf(m, qb + 2 * kvb_w, &qkv));
    M_TRY(mk_view(m, qkv, 0, qb, &B.wq));
    M_TRY(mk_view(m, qkv, qb, kvb_w, &B.wk));
    M_TRY(mk_view(m, qkv, qb + kvb_w, kvb_w, &B.wv));
    M_TRY(mk_buf(m, sx_packed_bytes(H, B.q_dim, m->lmode), &B.wo));
    M_TRY(mk_buf(m, sx_packed_bytes(I, H, m->lmode), &B.wg));
    M_TRY(mk_buf(m, sx_packed_bytes(I, H, m->lmode), &B.wu));
    M_TRY(mk_buf(m, sx_packed_bytes(H, I, m->lmode), &B.wd));
    M_TRY(mk_buf(m, (uint64_t)m->total_slots * B.kv_dim * kvb * S, &B.kc));
    M_TRY(mk_buf(m, (uint64_t)m->total_slots * B.kv_dim * kvb * S, &B.vc));
    m->weight_bytes += B.wq->bytes + B.wk->bytes + B.wv->bytes + B.wo->bytes + B.wg->bytes +
                       B.wu->bytes + B.wd->bytes;
  }
  M_TRY(mk_buf(m, 16ull * 12 * c.num_layers, &m->ind));
  // attention + o plans: graph 0 with one session, one GPU and Q4_0 layers
  if (c.reference_graph == 0 && S == 1 && c.tp_size <= 1 && m->lmode == SX_QUANT_Q4) {
    uint64_t opart = 0;
    for (uint32_t l = 0; l < c.num_layers; ++l) {
      LayerBufs &B = m->L[l];
      if (!sx::attn_o_plan(H, m->nq, B.num_kv, B.head_dim, m->total_slots,
                           sx::kAttnBlockSmemLimit, &B.ao_tiles, &B.ao_slots))
        B.ao_tiles = 0;
      if (B.ao_tiles && (uint64_t)B.num_kv * H > opart) opart = (uint64_t)B.num_kv * H;
    }
    if (opart) M_TRY(mk_buf(m, 4 * opart, &m->ab_opart));
  }
  // attention-block plans: graph 4 with one session, one GPU and Q4_0 layers (the rows of the
  // q|k|v projection are regrouped per kv head, which the packed Q4_0 tiles allow)
  if (c.reference_graph == 4 && S == 1 && c.tp_size <= 1 && m->lmode == SX_QUANT_Q4) {
    uint64_t rec = 0, opart = 0;
    uint32_t max_kv_heads = 0;
    for (uint32_t l = 0; l < c.num_layers; ++l) {
      LayerBufs &B = m->L[l];
      if (B.k_eq_v ||
          !sx::attn_block_plan(H, m->nq, B.num_kv, B.head_dim, m->total_slots, c.kv_bf16 != 0,
                               m->e->num_sms, sx::kAttnBlockSmemLimit, &B.ab))
        B.ab = sx::AttnBlockPlan{};
      if (!B.ab.ctas) continue;
      const uint64_t r = (uint64_t)m->nq * B.ab.ctas * (B.head_dim + 2);
      if (r > rec) rec = r;
      if ((uint64_t)B.num_kv * H > opart) opart = (uint64_t)B.num_kv * H;
      if (B.num_kv > max_kv_heads) max_kv_heads = B.num_kv;
    }
    if (rec) {
      M_TRY(mk_buf(m, 4 * rec, &m->ab_rec));
      M_TRY(mk_buf(m, 4 * opart, &m->ab_opart));
      m->ab_cnt_words = 2 * max_kv_heads + 1;
      M_TRY(mk_buf(m, 4ull * m->ab_cnt_words * c.num_layers, &m->ab_cnt));  // zeroed
    }
  }
  for (uint32_t l = 0; l < c.num_layers; ++l) M_TRY(mk_buf(m, 4ull * H, &m->L[l].x_prev));
  M_TRY(mk_buf(m, sx_packed_bytes(V, H, m->hmode), &m->lm_head));
  M_TRY(mk_buf(m, 4ull * H, &m->final_norm));
  m->weight_bytes += m->lm_head->bytes;

  // descriptor sets, model_gpu.zig:140-168
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    LayerBufs &B = m->L[l];
    M_TRY(mk_set(m, {m->x, B.in_norm, m->normed}, &B.s_input_norm));
    M_TRY(mk_set(m, {B.wq, m->normed, m->q}, &B.s_q));
    M_TRY(mk_set(m, {B.wk, m->normed, m->k}, &B.s_k));
    M_TRY(mk_set(m, {B.wv, m->normed, m->v}, &B.s_v));
    M_TRY(mk_set(m, {m->q, m->k, m->v, B.q_norm, B.k_norm, m->q, B.kc, B.vc, m->step},
                 &B.s_qkv_rope));
    M_TRY(mk_set(m, {m->q, B.kc, B.vc, m->slots, m->attn_out, m->step}, &B.s_attn));
    M_TRY(mk_set(m, {B.wo, m->attn_out, m->mlp_out}, &B.s_o));
    M_TRY(mk_set(m, {B.wg, B.wu, m->normed, m->act}, &B.s_gate_up));
    M_TRY(mk_set(m, {B.wd, m->act, m->mlp_out}, &B.s_down));
    M_TRY(mk_set(m, {m->x, m->mlp_out, B.pre_ffn, m->normed}, &B.s_pre_ffn));
    M_TRY(mk_set(m, {m->mlp_out, B.post_attn, m->mlp_out}, &B.s_post_attn));
    M_TRY(mk_set(m, {m->mlp_out, B.post_ffn, m->mlp_out}, &B.s_post_ffn));
    M_TRY(mk_set(m, {m->x, m->mlp_out, B.in_norm, m->normed}, &B.s_post_ffn_add));
    M_TRY(mk_set(m, {m->x, B.x_prev, m->ind}, &B.s_gate));
    M_TRY(sx_host_cuda_status(cudaMemset(B.x_prev->d, 0, 4ull * H), "x_prev zero"));
  }
  M_TRY(sx_host_cuda_status(cudaMemset(m->ind->d, 0, m->ind->bytes), "indirect records zero"));
  M_TRY(mk_set(m, {m->x, m->final_norm, m->normed}, &m->s_final_norm));
  M_TRY(mk_set(m, {m->lm_head, m->normed, m->logits}, &m->s_logits));
  M_TRY(mk_set(m, {m->logits, m->token}, &m->s_argmax));

  const uint64_t step_bytes = 16 * S < 64 ? 64 : 16 * S;
  M_TRY(sx_host_cuda_status(
      cudaHostAlloc((void **)&m->h_x, 4ull * H * S, cudaHostAllocDefault), "pinned x"));
  M_TRY(sx_host_cuda_status(
      cudaHostAlloc((void **)&m->h_slots, 4ull * m->total_slots * S, cudaHostAllocDefault),
      "pinned slots"));
  M_TRY(sx_host_cuda_status(
      cudaHostAlloc((void **)&m->h_step, step_bytes, cudaHostAllocDefault), "pinned step"));
  M_TRY(sx_host_cuda_status(cudaHostAlloc((void **)&m->h_token, 64, cudaHostAllocDefault),
                            "pinned token"));
  memset(m->h_x, 0, 4ull * H * S);
  memset(m->h_slots, 0, 4ull * m->total_slots * S);
  memset(m->h_step, 0, step_bytes);
  memset(m->h_token, 0, 64);
  return SX_OK;
}

// recordLayerDirect (model_dispatch.zig:10-43)
void record_layer(sx_model *m, sx_cmd *cmd, uint32_t l) {
  sx_engine *e = m->e;
  const sx_model_config &c = m->c;
  LayerBufs &B = m->L[l];
  const uint32_t H = c.hidden_size, I = m->I;
  const float eps = c.rms_norm_eps;
  const uint32_t gqa = m->nq / B.num_kv;
  sx_record_rmsnorm(e, cmd, B.s_input_norm, H, eps);
  sx_record_barrier(e, cmd);
  sx_record_gemv(e, cmd, B.s_q, B.q_dim, H);
  sx_record_gemv(e, cmd, B.s_k, B.kv_dim, H);
  sx_record_gemv(e, cmd, B.s_v, B.kv_dim, H);
  sx_record_barrier(e, cmd);
  sx_record_qkv_rope(e, cmd, B.s_qkv_rope, m->nq, B.num_kv, B.head_dim, B.rot, B.k_eq_v,
                     B.theta, eps, m->total_slots);
  sx_record_barrier(e, cmd);
  sx_record_decode_attn(e, cmd, B.s_attn, B.head_dim, B.kv_dim, gqa, c.attn_scale, m->nq,
                        m->total_slots);
  sx_record_barrier(e, cmd);
  sx_record_gemv(e, cmd, B.s_o, H, B.q_dim);
  if (c.has_post_norms) {
    sx_record_barrier(e, cmd);
    sx_record_rmsnorm(e, cmd, B.s_post_attn, H, eps);
  }
  sx_record_barrier(e, cmd);
  sx_record_add_rmsnorm(e, cmd, B.s_pre_ffn, H, eps, 1.0f);
  sx_record_barrier(e, cmd);
  sx_record_gate_up(e, cmd, B.s_gate_up, I, H);
  sx_record_barrier(e, cmd);
  sx_record_gemv(e, cmd, B.s_down, H, I);
  if (c.has_post_norms) {
    sx_record_barrier(e, cmd);
    sx_record_rmsnorm(e, cmd, B.s_post_ffn, H, eps);
  }
  sx_record_barrier(e, cmd);
  sx_record_add_rmsnorm(e, cmd, B.s_post_ffn_add, H, eps, B.layer_scalar);
  sx_record_barrier(e, cmd);
}

// recordLayerIndirect (model_dispatch.zig:45-101): the quiescence gate writes the dispatch
// records of the layer's 13 commands (16 slots per layer), every command reads its record
void record_layer_indirect(sx_model *m, sx_cmd *cmd, uint32_t l) {
  sx_engine *e = m->e;
  const sx_model_config &c = m->c;
  LayerBufs &B = m->L[l];
  const uint32_t H = c.hidden_size, I = m->I;
  const float eps = c.rms_norm_eps;
  const uint32_t gqa = m->nq / B.num_kv;
  sx_quiescence_gate_pc pc{};
  pc.hidden_size = H;
  pc.threshold_sq = c.quiescence_threshold;
  pc.base_cmd_idx = l * 16;
  pc.num_cmds = 13;
  // the reference's workgroup counts (here they only need to be non-zero)
  const uint32_t t[13] = {1, (B.q_dim + 3) / 4, (B.kv_dim + 3) / 4, (B.kv_dim + 3) / 4,
                          m->nq + B.num_kv, m->nq, (H + 3) / 4, 1, 1, (I + 3) / 4,
                          (H + 3) / 4, 1, 1};
  for (int i = 0; i < 13; ++i) pc.targets[i] = t[i];
  sx_record_quiescence_gate(e, cmd, B.s_gate, &pc);
  sx_record_barrier(e, cmd);
  const uint64_t base = (uint64_t)l * 16 * 12;
  sx_buffer *ind = m->ind;
  sx_record_rmsnorm_indirect(e, cmd, B.s_input_norm, H, eps, ind, base + 0 * 12);
  sx_record_barrier(e, cmd);
  sx_record_gemv_indirect(e, cmd, B.s_q, B.q_dim, H, ind, base + 1 * 12);
  sx_record_gemv_indirect(e, cmd, B.s_k, B.kv_dim, H, ind, base + 2 * 12);
  sx_record_gemv_indirect(e, cmd, B.s_v, B.kv_dim, H, ind, base + 3 * 12);
  sx_record_barrier(e, cmd);
  sx_record_qkv_rope_indirect(e, cmd, B.s_qkv_rope, m->nq, B.num_kv, B.head_dim, B.rot, B.k_eq_v,
                              B.theta, eps, m->total_slots, ind, base + 4 * 12);
  sx_record_barrier(e, cmd);
  sx_record_decode_attn_indirect(e, cmd, B.s_attn, B.head_dim, B.kv_dim, gqa, c.attn_scale,
                                 m->nq, m->total_slots, ind, base + 5 * 12);
  sx_record_barrier(e, cmd);
  sx_record_gemv_indirect(e, cmd, B.s_o, H, B.q_dim, ind, base + 6 * 12);
  if (c.has_post_norms) {
    sx_record_barrier(e, cmd);
    sx_record_rmsnorm_indirect(e, cmd, B.s_post_attn, H, eps, ind, base + 7 * 12);
  }
  sx_record_barrier(e, cmd);
  sx_record_add_rmsnorm_indirect(e, cmd, B.s_pre_ffn, H, eps, 1.0f, ind, base + 8 * 12);
  sx_record_barrier(e, cmd);
  sx_record_gate_up_indirect(e, cmd, B.s_gate_up, I, H, ind, base + 9 * 12);
  sx_record_barrier(e, cmd);
  sx_record_gemv_indirect(e, cmd, B.s_down, H, I, ind, base + 10 * 12);
  if (c.has_post_norms) {
    sx_record_barrier(e, cmd);
    sx_record_rmsnorm_indirect(e, cmd, B.s_post_ffn, H, eps, ind, base + 11 * 12);
  }
  sx_record_barrier(e, cmd);
  sx_record_add_rmsnorm_indirect(e, cmd, B.s_post_ffn_add, H, eps, B.layer_scalar, ind,
                                 base + 12 * 12);
  sx_record_barrier(e, cmd);
}

// recordForwardGraph (model_dispatch.zig:103-129), optionally wrapped in the per-token
// host<->device copies of gpuDispatchForwardToken (model_dispatch.zig:136-146).
sx_status record_forward(sx_model *m, sx_cmd *cmd, bool logits, bool io) {
  sx_engine *e = m->e;
  const sx_model_config &c = m->c;
  M_TRY(sx_cmd_begin(cmd));
  if (io) {
    Op a{OP_H2D};
    a.host = m->h_x; a.dev = m->x->d; a.bytes = 4ull * c.hidden_size;
    sx_host_push_op(cmd, a);
    Op b{OP_H2D};
    b.host = m->h_slots; b.dev = m->slots->d; b.bytes = 4ull * m->total_slots;
    sx_host_push_op(cmd, b);
    Op s{OP_H2D};
    s.host = m->h_step; s.dev = m->step->d; s.bytes = 16;
    sx_host_push_op(cmd, s);
  }
  sx_record_barrier(e, cmd);
  // layers below num_layers / 3 are recorded direct, the rest behind the quiescence gate
  // (model_dispatch.zig:107-118)
  const uint32_t dense_limit = c.num_layers / 3;
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    if (l < dense_limit) record_layer(m, cmd, l);
    else record_layer_indirect(m, cmd, l);
  }
  if (logits) {
    sx_record_rmsnorm(e, cmd, m->s_final_norm, c.hidden_size, c.rms_norm_eps);
    sx_record_barrier(e, cmd);
    sx_record_gemv_logits(e, cmd, m->s_logits, m->V, c.hidden_size);
    sx_record_barrier(e, cmd);
    sx_record_argmax(e, cmd, m->s_argmax, m->V);
    if (io) {
      Op t{OP_D2H};
      t.host = m->h_token; t.dev = m->token->d; t.bytes = 4;
      sx_host_push_op(cmd, t);
    }
  }
  return sx_cmd_end(cmd);
}

// The fused decode graph: per layer
//   [prologue: residual update of the previous layer + input RMSNorm] q|k|v GEMV
//   -> fused qkv_rope + decode attention -> o GEMV
//   -> [prologue: residual + pre-FFN RMSNorm] gate+up GeGLU GEMV -> down GEMV
// and a Q8 LM head whose prologue applies the last residual update and the final norm and
// whose epilogue is the argmax.  Same arithmetic as recordLayerDirect, 5 launches per layer
// instead of 14, all chained with programmatic dependent launch.
void push_gemv(sx_model *m, sx_cmd *cmd, const sx::GemvArgs &a, int qt, bool geglu) {
  Op op{OP_GEMV_FUSED};
  op.qt = qt;
  op.geglu = geglu;
  op.gemv = a;
  sx_host_bind_scratch(m->e, op.gemv);
  sx_host_push_op(cmd, op);
}

void push_allreduce(sx_model *m, sx_cmd *cmd, sx_buffer *buf, uint32_t count) {
  Op op{OP_ALLREDUCE};
  op.dev = buf->d;
  op.u[0] = count;
  op.comm = m->comm;
  sx_host_push_op(cmd, op);
}

sx::GemvArgs gemv1(const sx_buffer *w, const sx_buffer *x, sx_buffer *y, uint32_t rows,
                   uint32_t k) {
  sx::GemvArgs a{};
  a.w[0][0] = a.w[0][1] = w->d;
  a.y[0] = (float *)y->d;
  a.rows[0] = rows;
  a.tiles[0] = sx::tiles_of(rows);
  a.k = k;
  a.batch = 1;
  a.ldy = rows;
  a.x = (const float *)x->d;
  a.ldx = k;
  a.pro = sx::kProNone;
  a.epi = sx::kEpiPlain;
  return a;
}

// nb: sessions stepped together (1 for the one-session graphs); every GEMV runs with batch nb
// (row j = session j) and the attention with one grid layer per session.
sx_status record_forward_fused(sx_model *m, sx_cmd *cmd, bool logits, bool io,
                               int persistent, uint32_t nb = 1) {
  const sx_model_config &c = m->c;
  const uint32_t H = c.hidden_size, I = m->I, L = c.num_layers;
  const bool tp = m->comm != nullptr;
  const float eps = c.rms_norm_eps;
  M_TRY(sx_cmd_begin(cmd));
  sx_host_set_persistent(cmd, persistent);
  if (io) {
    Op a{OP_H2D};
    a.host = m->h_x; a.dev = m->x->d; a.bytes = 4ull * H * nb;
    sx_host_push_op(cmd, a);
    Op b{OP_H2D};
    b.host = m->h_slots; b.dev = m->slots->d; b.bytes = 4ull * m->total_slots * nb;
    sx_host_push_op(cmd, b);
    Op s{OP_H2D};
    s.host = m->h_step; s.dev = m->step->d; s.bytes = 16ull * nb;
    sx_host_push_op(cmd, s);
  }
  for (uint32_t l = 0; l < L; ++l) {
    LayerBufs &B = m->L[l];
    // q | k | v with the input norm (and, after layer 0, the previous layer's residual)
    // q | k | v rows of session j at qkv + j * base (base = q_dim + 2 kv_dim of this layer)
    const bool blk = persistent == kPersistNone && nb == 1 && !tp && B.ab.ctas != 0;
    const bool ao = persistent == kPersistNone && nb == 1 && !tp && B.ao_tiles != 0;
    sx::GemvArgs q{};
    const sx_buffer *w3[3] = {B.wq, B.wk, B.wv};
    uint32_t r3[3] = {B.q_dim, B.kv_dim, B.kv_dim};
    uint32_t base = 0;
    for (int s = 0; s < 3; ++s) {
      q.w[s][0] = q.w[s][1] = w3[s]->d;
      q.y[s] = (float *)m->qkv->d + base;
      q.rows[s] = r3[s];
      q.tiles[s] = sx::tiles_of(r3[s]);
      q.row_base[s] = base;
      base += r3[s];
    }
    float *const qp = (float *)m->qkv->d, *const kp = qp + B.q_dim, *const vp = kp + B.kv_dim;
    q.k = H;
    q.batch = nb;
    q.ldy = base;
    q.ldx = H;
    q.eps = eps;
    q.pro_w = (const float *)B.in_norm->d;
    if (l == 0) {
      q.pro = sx::kProNorm;
      q.x = (const float *)m->x->d;
    } else {
      LayerBufs &P = m->L[l - 1];
      q.pro = sx::kProResid;
      q.x = (const float *)m->x2->d;
      q.pro_mlp = (const float *)m->mlp_out->d;
      q.pro_post_w = c.has_post_norms ? (const float *)P.post_ffn->d : nullptr;
      q.pro_scalar = P.layer_scalar;
      q.pro_x_out = (float *)m->x->d;
    }
    q.epi = sx::kEpiPlain;
    // the attention below reads the live K/V rows of this layer's cache, last touched one
    // token ago: start pulling them into L2 while this GEMV runs
    if (B.kv_dim * (c.kv_bf16 ? 2u : 4u) % 16 == 0 && nb == 1)  // bulk: 16-byte multiples
      q.pf_slots = (const uint32_t *)m->slots->d;
    q.pf_step = (const uint32_t *)m->step->d;
    q.pf_base[0] = B.kc->d;
    q.pf_base[1] = B.k_eq_v ? nullptr : B.vc->d;
    q.pf_row_bytes = B.kv_dim * (c.kv_bf16 ? 2u : 4u);
    q.pf_max = m->total_slots;
    if (!blk) {
      M_TRY(sx_host_check_gemv(m->lqt, false, true, B.q_dim + 2 * B.kv_dim, H, nb));
      push_gemv(m, cmd, q, m->lqt, false);
    }

    // fused qkv_rope + attention
    Op at{OP_ATTN_FUSED};
    sx::AttnFusedArgs &A = at.attnf;
    A.q = qp;
    A.k = kp;
    A.v = vp;
    A.q_norm_w = (const float *)B.q_norm->d;
    A.k_norm_w = (const float *)B.k_norm->d;
    A.k_cache = B.kc->d;
    A.v_cache = B.vc->d;
    A.slots = (const uint32_t *)m->slots->d;
    A.step = (const uint32_t *)m->step->d;
    A.out = (float *)m->attn_out->d;
    A.head_dim = B.head_dim;
    A.kv_dim = B.kv_dim;
    A.num_q = m->nq;
    A.num_kv = B.num_kv;
    A.rotary_dim = B.rot;
    A.k_eq_v = B.k_eq_v;
    A.kv_bf16 = c.kv_bf16 ? 1u : 0u;
    A.total_slots = m->total_slots;
    A.scale = c.attn_scale;
    A.eps = eps;
    A.sessions = nb;
    A.qkv_ld = base;
    A.out_ld = B.q_dim;
    A.cache_ld = (uint64_t)m->total_slots * B.kv_dim;
    at.attn_rot = B.rot;
    at.attn_theta = B.theta;
    sx_host_bind_scratch(m->e, A);
    if (sx::attn_scratch_bytes(m->nq, m->total_slots, B.head_dim) > m->e->attn_part_bytes ||
        B.num_kv > 4096) {
      sx_host_set_error("model: attention scratch too small for this ring / head count");
      return SX_ERR_UNSUPPORTED;
    }
    if (blk) {
      // q|k|v projection + qkv_rope + attention + o projection as one kernel; the o rows come
      // out as one partial vector per kv-head group, summed by the gate+up prologue
      Op ab{OP_ATTN_BLOCK};
      sx::AttnBlockArgs &X = ab.ab;
      X.g = q;
      sx_host_bind_scratch(m->e, X.g);
      X.at = A;
      X.wo = B.wo->d;
      X.opart = (float *)m->ab_opart->d;
      X.rec = (float *)m->ab_rec->d;
      X.cnt = (uint32_t *)m->ab_cnt->d + (size_t)l * m->ab_cnt_words;
      X.o_rows = H;
      X.ctas = B.ab.ctas;
      X.max_slots = B.ab.max_slots;
      X.o_tiles = B.ab.o_tiles;
      X.wait_ns = 200000000ull;  // 0.2 s per counter wait
      ab.attn_rot = B.rot;
      ab.attn_theta = B.theta;
      sx_host_push_op(cmd, ab);
    } else if (ao) {
      // qkv_rope + attention + this kv head's share of the o projection as one cluster kernel;
      // the o rows come out as one partial vector per kv head, summed by the gate+up prologue
      Op op{OP_ATTN_O};
      op.ao.at = A;
      op.ao.wo = B.wo->d;
      op.ao.opart = (float *)m->ab_opart->d;
      op.ao.o_rows = H;
      op.ao.o_tiles = B.ao_tiles;
      op.ao.cta_slots = B.ao_slots;
      op.attn_rot = B.rot;
      op.attn_theta = B.theta;
      sx_host_push_op(cmd, op);
    } else {
      sx_host_push_op(cmd, at);

      // o projection
      M_TRY(sx_host_check_gemv(m->lqt, false, false, H, B.q_dim, nb));
      sx::GemvArgs o = gemv1(B.wo, m->attn_out, m->mlp_out, H, B.q_dim);
      o.batch = nb;
      push_gemv(m, cmd, o, m->lqt, false);
      if (tp) push_allreduce(m, cmd, m->mlp_out, H);  // row-parallel o: sum of the ranks' parts
    }

    // gate+up GeGLU with the post-attention residual and pre-FFN norm
    sx::GemvArgs g = gemv1(B.wg, m->x, m->act, I, H);
    g.w[0][1] = B.wu->d;
    g.pro = sx::kProResid;
    g.pro_mlp = (const float *)m->mlp_out->d;
    if (blk || ao) {
      g.pro_mlp = (const float *)m->ab_opart->d;
      g.pro_mlp_parts = B.num_kv;
      g.pro_mlp_ld = H;
    }
    g.pro_post_w = c.has_post_norms ? (const float *)B.post_attn->d : nullptr;
    g.pro_scalar = 1.0f;
    g.pro_w = (const float *)B.pre_ffn->d;
    g.pro_x_out = (float *)m->x2->d;
    g.eps = eps;
    g.batch = nb;
    M_TRY(sx_host_check_gemv(m->lqt, true, true, I, H, nb));
    push_gemv(m, cmd, g, m->lqt, true);

    // down projection
    M_TRY(sx_host_check_gemv(m->lqt, false, false, H, I, nb));
    sx::GemvArgs d = gemv1(B.wd, m->act, m->mlp_out, H, I);
    d.batch = nb;
    push_gemv(m, cmd, d, m->lqt, false);
    if (tp) push_allreduce(m, cmd, m->mlp_out, H);  // row-parallel down
  }
  if (logits) {
    LayerBufs &P = m->L[L - 1];
    sx::GemvArgs h = gemv1(m->lm_head, m->x2, m->logits, m->V, H);
    h.row_base[0] = m->tp.vocab0;  // global vocabulary index of local row 0
    h.pro = sx::kProResid;
    h.pro_mlp = (const float *)m->mlp_out->d;
    h.pro_post_w = c.has_post_norms ? (const float *)P.post_ffn->d : nullptr;
    h.pro_scalar = P.layer_scalar;
    h.pro_w = (const float *)m->final_norm->d;
    h.pro_x_out = (float *)m->x->d;
    h.pro_norm_out = (float *)m->normed->d;  // the final normed state (recall tier's query)
    h.eps = eps;
    h.epi = sx::kEpiArgmax;
    h.token = (uint32_t *)m->token->d;
    h.batch = nb;
    if (tp) h.cand = (uint32_t *)m->cand->d;
    M_TRY(sx_host_check_gemv(8, false, true, m->V, H, nb));
    push_gemv(m, cmd, h, 8, false);
    if (tp) {
      // vocabulary-parallel argmax: all ranks' candidates, merged on device
      Op g{OP_ALLGATHER};
      g.bind = {m->cand->d, m->cand_all->d};
      g.u[0] = 4;  // u32 words per rank
      g.comm = m->comm;
      sx_host_push_op(cmd, g);
      Op mg{OP_TP_ARGMAX};
      mg.bind = {m->cand_all->d, m->token->d};
      mg.u[0] = m->c.tp_size;
      sx_host_push_op(cmd, mg);
    }
    if (io) {
      Op t{OP_D2H};
      t.host = m->h_token; t.dev = m->token->d; t.bytes = 4ull * nb;
      sx_host_push_op(cmd, t);
    }
  }
  return sx_cmd_end(cmd);
}

sx_status record_graph(sx_model *m, sx_cmd *cmd, bool logits, bool io) {
  if (m->c.reference_graph == 1) return record_forward(m, cmd, logits, io);
  const int kind = m->c.reference_graph == 2   ? kPersistPhases
                   : m->c.reference_graph == 3 ? kPersistStream
                                               : kPersistNone;
  return record_forward_fused(m, cmd, logits, io, kind);
}

// rows x cols of the synthetic matrix (seed, stream), starting at global row `grow0` and
// 32-column block `gblk0` of a matrix with `gnb` blocks per row (gnb = 0: cols / 32)
sx_status synth_matrix(sx_model *m, sx_buffer *dst, uint32_t rows, uint32_t cols,
                       sx_quant_mode mode, uint64_t seed, uint64_t stream, void *tmp,
                       uint64_t tmp_bytes, uint32_t grow0 = 0, uint32_t gblk0 = 0,
                       uint32_t gnb = 0) {
  if (mode == SX_QUANT_NONE) {  // bf16 values written in place (one GPU: no slices)
    if (grow0 || gblk0 || (gnb && gnb != cols / 32)) {
      sx_host_set_error("synth: bf16 weights are not sliced for tensor parallelism");
      return SX_ERR_UNSUPPORTED;
    }
    return sx_host_cuda_status(sx::launch_synth_bf16((uint16_t *)dst->d, (uint64_t)rows * cols,
                                                     seed, stream, m->e->stream),
                               "synth bf16");
  }
  const uint64_t row_bytes = sx_quantized_row_words(cols, mode) * 4;
  uint64_t chunk = tmp_bytes / row_bytes;
  chunk = (chunk / 16) * 16;
  if (chunk < 16) {
    sx_host_set_error("synth: staging buffer too small");
    return SX_ERR_INVALID;
  }
  const int qt = mode == SX_QUANT_Q4 ? 4 : 8;
  const uint64_t chunk_bytes = qt == 4 ? sx::kQ4ChunkBytes : sx::kQ8ChunkBytes;
  for (uint64_t r0 = 0; r0 < rows; r0 += chunk) {
    uint32_t n = (uint32_t)((rows - r0) < chunk ? (rows - r0) : chunk);
    M_TRY(sx_host_cuda_status(sx::launch_synth_ref(qt, (uint32_t *)tmp, grow0 + (uint32_t)r0, n,
                                                   cols, seed, stream, m->e->stream, gblk0, gnb),
                              "synth launch"));
    uint8_t *out = (uint8_t *)dst->d + (r0 / 16) * sx::pairs_of(cols) * chunk_bytes;
    M_TRY(sx_host_cuda_status(
        sx::launch_repack(qt, (const uint32_t *)tmp, out, n, cols, m->e->stream), "repack"));
  }
  return SX_OK;
}

}  // namespace

extern "C" {

namespace {

sx_status create_model(sx_engine *e, const sx_model_config *cfg, sx_comm *comm, sx_model **out) {
  if (!e || !cfg || !out) {
    sx_host_set_error("model_create: null argument");
    return SX_ERR_INVALID;
  }
  const sx_model_config &c = *cfg;
  bool ok = c.vocab_size > 0 && c.hidden_size % 32 == 0 && c.intermediate_size % 32 == 0 &&
            c.num_layers > 0 && c.num_q_heads > 0 && c.num_kv_heads > 0 &&
            c.num_q_heads % c.num_kv_heads == 0 && c.window_size > 0 && c.head_dim > 0 &&
            (c.num_q_heads * c.head_dim) % 32 == 0 && c.reference_graph <= 4;
  if (c.full_every)
    ok = ok && c.num_global_kv_heads > 0 && c.num_q_heads % c.num_global_kv_heads == 0 &&
         c.global_head_dim > 0;
  if (!ok) {
    sx_host_set_error("model_create: inconsistent config");
    return SX_ERR_INVALID;
  }
  if (c.num_sessions > 1) {
    const uint32_t slots = c.num_anchors + c.window_size + c.num_recall;
    if (c.num_sessions > 8 || c.reference_graph != 0 || c.tp_size > 1 ||
        slots > sx::kAttnClusterMaxSlots) {
      sx_host_set_error("model_create: num_sessions %u needs <= 8 sessions, the fused graph "
                        "(reference_graph 0), one GPU and a ring of at most %u slots",
                        c.num_sessions, sx::kAttnClusterMaxSlots);
      return SX_ERR_UNSUPPORTED;
    }
  }
  if ((c.kv_bf16 != 0) != e->kv_bf16) {
    sx_host_set_error("model_create: config.kv_bf16 must match the engine's KV precision flag");
    return SX_ERR_INVALID;
  }
  if (c.quiescence_threshold > 0.0f && c.reference_graph != 1) {
    sx_host_set_error("model_create: a positive quiescence threshold needs the op-by-op graph "
                      "(reference_graph 1), whose gated layers read device-side dispatch records");
    return SX_ERR_UNSUPPORTED;
  }
  if (e->mode == SX_QUANT_NONE && c.reference_graph != 1) {
    sx_host_set_error("model_create: bf16 layers (engine mode none) run the reference's op-by-op "
                      "graph (reference_graph 1)");
    return SX_ERR_UNSUPPORTED;
  }
  if (e->mode != SX_QUANT_Q4 && (c.tp_size > 1 || c.num_sessions > 1)) {
    sx_host_set_error("model_create: tensor parallelism and batched sessions need Q4_0 layers");
    return SX_ERR_UNSUPPORTED;
  }
  cudaSetDevice(e->device);
  sx_model *m = new sx_model();
  m->e = e;
  m->c = c;
  m->comm = comm;
  m->lmode = e->mode;
  m->hmode = e->mode == SX_QUANT_NONE ? SX_QUANT_NONE : SX_QUANT_Q8;
  m->lqt = e->mode == SX_QUANT_Q4 ? 4 : e->mode == SX_QUANT_Q8 ? 8 : 0;
  sx_status st = alloc_model(m);
  for (int lg = 0; lg < 2 && st == SX_OK; ++lg)
    for (int io = 0; io < 2 && st == SX_OK; ++io) {
      st = sx_cmd_create(e, &m->cmd[lg][io]);
      if (st == SX_OK) st = record_graph(m, m->cmd[lg][io], lg != 0, io != 0);
    }
  if (st != SX_OK) {
    std::string msg = sx_last_error();
    sx_model_destroy(m);
    sx_host_set_error("%s", msg.c_str());
    return st;
  }
  *out = m;
  return SX_OK;
}

}  // namespace

SX_API uint32_t sx_model_config_bytes(void) { return (uint32_t)sizeof(sx_model_config); }

SX_API sx_status sx_model_create(sx_engine *e, const sx_model_config *cfg, sx_model **out) {
  if (cfg && cfg->tp_size > 1) {
    sx_host_set_error("model_create: tp_size > 1 needs a communicator (sx_model_create_tp)");
    return SX_ERR_INVALID;
  }
  return create_model(e, cfg, nullptr, out);
}

SX_API sx_status sx_model_create_tp(sx_engine *e, const sx_model_config *cfg, sx_comm *comm,
                                    sx_model **out) {
  if (!cfg || !comm) {
    sx_host_set_error("model_create_tp: null argument");
    return SX_ERR_INVALID;
  }
  const uint32_t n = cfg->tp_size > 1 ? cfg->tp_size : 1;
  if (n != sx_host_comm_ranks(comm) || (n > 1 ? cfg->tp_rank : 0) != sx_host_comm_rank(comm)) {
    sx_host_set_error("model_create_tp: tp_size %u / tp_rank %u do not match the communicator "
                      "(%u ranks, rank %u)", cfg->tp_size, cfg->tp_rank,
                      sx_host_comm_ranks(comm), sx_host_comm_rank(comm));
    return SX_ERR_INVALID;
  }
  if (cfg->reference_graph != 0) {
    sx_host_set_error("model_create_tp: tensor parallelism runs the fused graph (reference_graph "
                      "0); the persistent kernel and the record-API graph have no collectives");
    return SX_ERR_UNSUPPORTED;
  }
  return create_model(e, cfg, comm, out);
}

SX_API void sx_model_destroy(sx_model *m) {
  if (!m) return;
  cudaSetDevice(m->e->device);
  cudaStreamSynchronize(m->e->stream);
  for (auto &row : m->cmd)
    for (sx_cmd *c : row) sx_cmd_destroy(c);
  for (auto &row : m->bcmd)
    for (sx_cmd *c : row) sx_cmd_destroy(c);
  for (sx_set *s : m->sets) sx_set_destroy(s);
  for (sx_buffer *b : m->buffers) sx_buffer_destroy(b);
  for (void *p : m->pf) cudaFree(p);
  if (m->h_x) cudaFreeHost(m->h_x);
  if (m->h_slots) cudaFreeHost(m->h_slots);
  if (m->h_step) cudaFreeHost(m->h_step);
  if (m->h_token) cudaFreeHost(m->h_token);
  delete m;
}

SX_API sx_status sx_model_synth_weights(sx_model *m, uint64_t seed) {
  if (!m) {
    sx_host_set_error("model: null");
    return SX_ERR_INVALID;
  }
  sx_engine *e = m->e;
  const sx_model_config &c = m->c;
  const uint32_t H = c.hidden_size, I = m->I;
  const sx_tp_shard &tp = m->tp;
  cudaSetDevice(e->device);
  const uint64_t tmp_bytes = 64ull << 20;
  void *tmp = nullptr;
  M_TRY(sx_host_cuda_status(cudaMalloc(&tmp, tmp_bytes), "synth staging"));
  sx_status st = SX_OK;
  for (uint32_t l = 0; l < c.num_layers && st == SX_OK; ++l) {
    LayerBufs &B = m->L[l];
    auto gain = [&](sx_buffer *b, uint32_t n, uint32_t kind) {
      return sx_host_cuda_status(sx::launch_synth_gain((float *)b->d, n, seed, stream_of(l, kind),
                                                       e->stream),
                                 "synth gain");
    };
    if (st == SX_OK) st = gain(B.in_norm, H, T_INPUT_NORM);
    if (st == SX_OK) st = gain(B.post_attn, H, T_POST_ATTN);
    if (st == SX_OK) st = gain(B.pre_ffn, H, T_PRE_FFN);
    if (st == SX_OK) st = gain(B.post_ffn, H, T_POST_FFN);
    if (st == SX_OK) st = gain(B.q_norm, B.head_dim, T_QNORM);
    if (st == SX_OK) st = gain(B.k_norm, B.head_dim, T_KNORM);
    // this rank's slices of the one-GPU model's matrices: rows of q/k/v/gate/up (its heads
    // and intermediate rows), 32-column blocks of o/down (the same split of their K)
    auto mat = [&](sx_buffer *b, uint32_t rows, uint32_t cols, uint32_t kind, uint32_t grow0,
                   uint32_t gblk0, uint32_t gnb) {
      return synth_matrix(m, b, rows, cols, m->lmode, seed, stream_of(l, kind), tmp, tmp_bytes,
                          grow0, gblk0, gnb);
    };
    const uint32_t hd = B.head_dim, q_glob = c.num_q_heads * hd;
    if (st == SX_OK) st = mat(B.wq, B.q_dim, H, T_Q, tp.q_head0 * hd, 0, 0);
    if (st == SX_OK) st = mat(B.wk, B.kv_dim, H, T_K, B.kv_head0 * hd, 0, 0);
    if (st == SX_OK)
      st = mat(B.wv, B.kv_dim, H, B.k_eq_v ? T_K : T_V, B.kv_head0 * hd, 0, 0);
    if (st == SX_OK) st = mat(B.wo, H, B.q_dim, T_O, 0, tp.q_head0 * hd / 32, q_glob / 32);
    if (st == SX_OK) st = mat(B.wg, I, H, T_GATE, tp.inter0, 0, 0);
    if (st == SX_OK) st = mat(B.wu, I, H, T_UP, tp.inter0, 0, 0);
    if (st == SX_OK)
      st = mat(B.wd, H, I, T_DOWN, 0, tp.inter0 / 32, c.intermediate_size / 32);
    float z = sx::synth_normal(seed, stream_of(l, T_SCALAR), 0);
    B.layer_scalar = sx::bf16_bits_to_f32(sx::bf16_bits_rne(fmaf(0.05f, z, 1.0f)));
  }
  if (st == SX_OK)
    st = synth_matrix(m, m->lm_head, m->V, H, m->hmode, seed, 2, tmp, tmp_bytes, tp.vocab0);
  if (st == SX_OK)
    st = sx_host_cuda_status(
        sx::launch_synth_gain((float *)m->final_norm->d, H, seed, 3, e->stream), "synth gain");
  if (st == SX_OK) st = sx_host_cuda_status(cudaStreamSynchronize(e->stream), "synth sync");
  cudaFree(tmp);
  if (st != SX_OK) return st;
  // layer scalars are recorded into the graphs: re-record them
  for (int lg = 0; lg < 2 && st == SX_OK; ++lg)
    for (int io = 0; io < 2 && st == SX_OK; ++io)
      st = record_graph(m, m->cmd[lg][io], lg != 0, io != 0);
  for (uint32_t n = 2; n <= 8 && st == SX_OK; ++n)
    for (int lg = 0; lg < 2 && st == SX_OK; ++lg)
      if (m->bcmd[n][lg]) st = record_forward_fused(m, m->bcmd[n][lg], lg != 0, true, false, n);
  return st;
}

SX_API sx_status sx_model_fill_kv(sx_model *m, uint64_t seed) {
  return sx_model_fill_kv_session(m, 0, seed);
}

SX_API sx_status sx_model_fill_kv_session(sx_model *m, uint32_t session, uint64_t seed) {
  if (!m) {
    sx_host_set_error("model: null");
    return SX_ERR_INVALID;
  }
  if (session >= m->S) {
    sx_host_set_error("fill_kv: session %u of a model with %u sessions", session, m->S);
    return SX_ERR_INVALID;
  }
  cudaSetDevice(m->e->device);
  const uint64_t eb = m->c.kv_bf16 ? 2 : 4;
  for (uint32_t l = 0; l < m->c.num_layers; ++l) {
    LayerBufs &B = m->L[l];
    const uint64_t off = (uint64_t)session * m->total_slots * B.kv_dim * eb;
    M_TRY(sx_host_cuda_status(
        sx::launch_fill_kv((uint8_t *)B.kc->d + off, (uint8_t *)B.vc->d + off,
                           m->c.kv_bf16 ? 1 : 0, m->total_slots * B.num_kv,
                           B.head_dim, m->c.rms_norm_eps, seed, l, m->e->stream, B.num_kv,
                           B.kv_head0, B.num_kv_global),
        "fill kv"));
  }
  return sx_host_cuda_status(cudaStreamSynchronize(m->e->stream), "fill kv sync");
}

SX_API sx_status sx_forward_token(sx_model *m, const float *x, uint32_t clock, uint32_t slot,
                                  const uint32_t *active_slots, uint32_t n_active,
                                  int want_logits, uint32_t *token_out, float *logits_out) {
  if (!m || !x || (n_active && !active_slots)) {
    sx_host_set_error("forward_token: null argument");
    return SX_ERR_INVALID;
  }
  if (n_active > m->total_slots || slot >= m->total_slots) {
    sx_host_set_error("forward_token: slot list larger than the ring or slot out of range");
    return SX_ERR_INVALID;
  }
  memcpy(m->h_x, x, 4ull * m->c.hidden_size);
  if (n_active) memcpy(m->h_slots, active_slots, 4ull * n_active);
  m->h_step[0] = clock;
  m->h_step[1] = slot;
  m->h_step[2] = n_active;
  m->h_step[3] = 0;
  sx_status st = sx_submit(m->e, m->cmd[want_logits ? 1 : 0][1], 0);
  if (token_out) *token_out = (st == SX_OK && want_logits) ? m->h_token[0] : 0u;
  if (st == SX_OK && want_logits && logits_out)
    st = sx_buffer_read(m->logits, 0, logits_out, 4ull * m->V);
  return st;
}

namespace {
// the graph stepping sessions 0..n-1 (with host staging); recorded on first use
sx_status batch_cmd(sx_model *m, uint32_t n, int lg, sx_cmd **out) {
  if (n == 1) {
    *out = m->cmd[lg][1];
    return SX_OK;
  }
  if (!m->bcmd[n][lg]) {
    M_TRY(sx_cmd_create(m->e, &m->bcmd[n][lg]));
    sx_status st = record_forward_fused(m, m->bcmd[n][lg], lg != 0, true, false, n);
    if (st != SX_OK) {
      sx_cmd_destroy(m->bcmd[n][lg]);
      m->bcmd[n][lg] = nullptr;
      return st;
    }
  }
  *out = m->bcmd[n][lg];
  return SX_OK;
}
}  // namespace

SX_API sx_status sx_decode_batch(sx_model *m, uint32_t n, const float *x, const uint32_t *clock,
                                 const uint32_t *slot, const uint32_t *active,
                                 const uint32_t *n_active, int want_logits, uint32_t *tokens,
                                 float *logits_out) {
  if (!m || !x || !clock || !slot || !active || !n_active) {
    sx_host_set_error("decode_batch: null argument");
    return SX_ERR_INVALID;
  }
  if (n == 0 || n > m->S) {
    sx_host_set_error("decode_batch: %u sessions requested, the model holds %u", n, m->S);
    return SX_ERR_INVALID;
  }
  const uint32_t H = m->c.hidden_size, TS = m->total_slots;
  for (uint32_t i = 0; i < n; ++i)
    if (n_active[i] > TS || slot[i] >= TS) {
      sx_host_set_error("decode_batch: session %u: slot list larger than the ring or slot out "
                        "of range", i);
      return SX_ERR_INVALID;
    }
  const int lg = want_logits ? 1 : 0;
  sx_cmd *cmd = nullptr;
  M_TRY(batch_cmd(m, n, lg, &cmd));
  memcpy(m->h_x, x, 4ull * H * n);
  for (uint32_t i = 0; i < n; ++i) {
    if (n_active[i]) memcpy(m->h_slots + (size_t)i * TS, active + (size_t)i * TS, 4ull * n_active[i]);
    m->h_step[4 * i + 0] = clock[i];
    m->h_step[4 * i + 1] = slot[i];
    m->h_step[4 * i + 2] = n_active[i];
    m->h_step[4 * i + 3] = 0;
  }
  sx_status st = sx_submit(m->e, cmd, 0);
  if (tokens)
    for (uint32_t i = 0; i < n; ++i) tokens[i] = (st == SX_OK && want_logits) ? m->h_token[i] : 0u;
  if (st == SX_OK && want_logits && logits_out)
    st = sx_buffer_read(m->logits, 0, logits_out, 4ull * m->V * n);
  return st;
}

SX_API sx_status sx_model_launch_batch(sx_model *m, uint32_t n, int want_logits) {
  if (!m || n == 0 || n > m->S) {
    sx_host_set_error("model_launch_batch: null model or %u sessions (the model holds %u)", n,
                      m ? m->S : 0);
    return SX_ERR_INVALID;
  }
  sx_cmd *cmd = nullptr;
  M_TRY(batch_cmd(m, n, want_logits ? 1 : 0, &cmd));
  return sx_host_cuda_status(cudaGraphLaunch(cmd->exec, m->e->stream), "graph launch");
}

SX_API sx_status sx_model_launch(sx_model *m, int want_logits) {
  if (!m) {
    sx_host_set_error("model: null");
    return SX_ERR_INVALID;
  }
  sx_cmd *c = m->cmd[want_logits ? 1 : 0][0];
  return sx_host_cuda_status(cudaGraphLaunch(c->exec, m->e->stream), "graph launch");
}

SX_API sx_status sx_model_get_io(sx_model *m, sx_model_io *io) {
  if (!m || !io) {
    sx_host_set_error("model: null");
    return SX_ERR_INVALID;
  }
  io->x = (float *)m->x->d;
  io->slots = (uint32_t *)m->slots->d;
  io->step = (uint32_t *)m->step->d;
  io->token = (uint32_t *)m->token->d;
  io->logits = (float *)m->logits->d;
  io->normed = (float *)m->normed->d;
  return SX_OK;
}

SX_API void *sx_model_kcache(sx_model *m, uint32_t layer) {
  return (m && layer < m->L.size()) ? m->L[layer].kc->d : nullptr;
}
SX_API void *sx_model_vcache(sx_model *m, uint32_t layer) {
  return (m && layer < m->L.size()) ? m->L[layer].vc->d : nullptr;
}
SX_API uint64_t sx_model_weight_bytes(sx_model *m) { return m ? m->weight_bytes : 0; }
SX_API uint32_t sx_model_kernels_per_token(sx_model *m, int want_logits) {
  return m ? m->cmd[want_logits ? 1 : 0][0]->kernels : 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Batched prefill: every token of the call goes through each layer at once (tcgen05 GEMMs for
// the projections, per-token kernels in sx_prefill_model.cu); the LM head runs on the
// requested rows (normally the last prompt token of each session).
namespace {

enum PfBuf { PF_XA, PF_XB, PF_MLP, PF_XN, PF_Y, PF_Y2, PF_Q, PF_META, PF_LISTS, PF_OUT, PF_ITEMS,
             PF_NUM };

sx_status pf_ensure(sx_model *m, uint64_t T) {
  if (T <= m->pf_T) return SX_OK;
  for (void *p : m->pf) cudaFree(p);
  m->pf.assign(PF_NUM, nullptr);
  m->pf_T = 0;
  const uint64_t H = m->c.hidden_size, I = m->I, ts = m->total_slots;
  uint64_t wide = H > I ? H : I;
  if (m->max_q > wide) wide = m->max_q;
  const uint64_t ywide = m->max_base > I ? m->max_base : I;
  const uint64_t bytes[PF_NUM] = {
      4 * T * H, 4 * T * H, 4 * T * H, 2 * T * wide, 4 * T * ywide, 4 * T * I,
      4 * T * m->max_q, 16 * T, 4 * T * ts,
      // out: row ids [8], normed rows [8][H], tokens [8], logits [8][V]
      4 * 8 + 4 * 8 * H + 4 * 8 + 4ull * 8 * m->V,
      // tensor-core attention work items {first token, tokens}: up to two item sets
      16 * T};
  for (int i = 0; i < PF_NUM; ++i)
    M_TRY(sx_host_cuda_status(cudaMalloc(&m->pf[i], bytes[i]), "prefill scratch"));
  m->pf_T = T;
  return SX_OK;
}

}  // namespace

extern "C" SX_API sx_status sx_prefill_batch(sx_model *m, uint32_t T, const float *x,
                                             const uint32_t *session, const uint32_t *clock,
                                             const uint32_t *slot, const uint32_t *active,
                                             const uint32_t *n_active, uint32_t n_out,
                                             const uint32_t *out_rows, uint32_t *tokens,
                                             float *logits_out) {
  if (!m || !x || !session || !clock || !slot || !active || !n_active || T == 0 ||
      (n_out && !out_rows)) {
    sx_host_set_error("prefill_batch: null argument or no tokens");
    return SX_ERR_INVALID;
  }
  const sx_model_config &c = m->c;
  if (m->comm || c.reference_graph == 1 || m->lmode != SX_QUANT_Q4) {
    sx_host_set_error("prefill_batch: runs on one GPU with the fused kernels and Q4_0 layers "
                      "(tp_size <= 1, reference_graph != 1, engine mode Q4)");
    return SX_ERR_UNSUPPORTED;
  }
  const uint32_t H = c.hidden_size, I = m->I, ts = m->total_slots, L = c.num_layers;
  if (n_out > 8) {
    sx_host_set_error("prefill_batch: at most 8 output rows per call (%u asked)", n_out);
    return SX_ERR_INVALID;
  }
  for (uint32_t i = 0; i < n_out; ++i)
    if (out_rows[i] >= T) {
      sx_host_set_error("prefill_batch: output row %u beyond %u tokens", out_rows[i], T);
      return SX_ERR_INVALID;
    }
  // GEMM shapes: K of every projection a multiple of 64, N a multiple of 4
  for (uint32_t l = 0; l < L; ++l) {
    const LayerBufs &B = m->L[l];
    if (H % 64 || B.q_dim % 64 || I % 64 || (B.q_dim + 2 * B.kv_dim) % 4) {
      sx_host_set_error("prefill_batch: hidden, q and intermediate sizes must be multiples of "
                        "64 for the tcgen05 GEMM");
      return SX_ERR_UNSUPPORTED;
    }
  }
  // per-token checks, and causality of the one-pass layers: no token may read a slot that a
  // later token of its session rewrites in this call (and no slot is written twice)
  std::vector<std::vector<uint32_t>> writer(m->S, std::vector<uint32_t>(ts, 0xFFFFFFFFu));
  for (uint32_t t = 0; t < T; ++t) {
    if (session[t] >= m->S || slot[t] >= ts || n_active[t] > ts) {
      sx_host_set_error("prefill_batch: token %u: session %u (of %u), slot %u or %u active "
                        "slots out of range", t, session[t], m->S, slot[t], n_active[t]);
      return SX_ERR_INVALID;
    }
    uint32_t &w = writer[session[t]][slot[t]];
    if (w != 0xFFFFFFFFu) {
      sx_host_set_error("prefill_batch: slot %u of session %u written twice in one call; split "
                        "the prompt", slot[t], session[t]);
      return SX_ERR_INVALID;
    }
    w = clock[t];
  }
  for (uint32_t t = 0; t < T; ++t) {
    const uint32_t *lst = active + (size_t)t * ts;
    for (uint32_t j = 0; j < n_active[t]; ++j) {
      if (lst[j] >= ts) {
        sx_host_set_error("prefill_batch: token %u lists slot %u of a %u-slot ring", t, lst[j], ts);
        return SX_ERR_INVALID;
      }
      const uint32_t w = writer[session[t]][lst[j]];
      if (w != 0xFFFFFFFFu && w > clock[t]) {
        sx_host_set_error("prefill_batch: token %u (clock %u) reads slot %u, which the token at "
                          "clock %u of the same session rewrites in this call; split the prompt",
                          t, clock[t], lst[j], w);
        return SX_ERR_INVALID;
      }
    }
  }
  sx_engine *e = m->e;
  cudaSetDevice(e->device);
  M_TRY(pf_ensure(m, T));
  cudaStream_t s = e->stream;
  float *xa = (float *)m->pf[PF_XA], *xb = (float *)m->pf[PF_XB], *mlp = (float *)m->pf[PF_MLP];
  void *xn = m->pf[PF_XN];
  float *y = (float *)m->pf[PF_Y], *y2 = (float *)m->pf[PF_Y2], *qo = (float *)m->pf[PF_Q];
  uint32_t *meta = (uint32_t *)m->pf[PF_META], *lists = (uint32_t *)m->pf[PF_LISTS];
  uint32_t *d_sess = meta, *d_clock = meta + T, *d_slot = meta + 2 * T, *d_cnt = meta + 3 * T;
  uint32_t *d_rows = (uint32_t *)m->pf[PF_OUT];
  float *d_norm = (float *)(d_rows + 8);
  uint32_t *d_tok = (uint32_t *)(d_norm + 8ull * H);
  float *d_logits = (float *)(d_tok + 8);
  auto cp = [&](void *dst, const void *src, size_t bytes) {
    return sx_host_cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s),
                               "prefill upload");
  };
  M_TRY(cp(xa, x, 4ull * T * H));
  M_TRY(cp(d_sess, session, 4ull * T));
  M_TRY(cp(d_clock, clock, 4ull * T));
  M_TRY(cp(d_slot, slot, 4ull * T));
  M_TRY(cp(d_cnt, n_active, 4ull * T));
  M_TRY(cp(lists, active, 4ull * T * ts));
  if (n_out) M_TRY(cp(d_rows, out_rows, 4ull * n_out));
  // tensor-core prefill attention: runs of up to 64 / G consecutive tokens of one session
  // (G = q heads per kv head of a layer; at most two layer shapes, sliding and full)
  uint32_t *d_items = (uint32_t *)m->pf[PF_ITEMS];
  std::vector<std::pair<uint32_t, std::vector<uint32_t>>> item_sets;  // (tokens per item, items)
  auto items_for = [&](uint32_t g, uint32_t *off, uint32_t *count) -> bool {
    const uint32_t tb = sx::pf_attn_tc_tokens(g);
    if (tb == 0) return false;
    for (size_t i = 0; i < item_sets.size(); ++i)
      if (item_sets[i].first == tb) {
        *off = (uint32_t)i * 2 * T;
        *count = (uint32_t)item_sets[i].second.size() / 2;
        return true;
      }
    if (item_sets.size() == 2) return false;
    std::vector<uint32_t> it;
    for (uint32_t t = 0; t < T;) {
      uint32_t n = 1;
      while (t + n < T && n < tb && session[t + n] == session[t]) ++n;
      it.push_back(t);
      it.push_back(n);
      t += n;
    }
    *off = (uint32_t)item_sets.size() * 2 * T;
    *count = (uint32_t)it.size() / 2;
    item_sets.emplace_back(tb, std::move(it));
    return true;
  };
  std::vector<uint32_t> layer_items(2 * L, 0);  // per layer: offset, count (count 0: CUDA cores)
  for (uint32_t l = 0; l < L; ++l) {
    const LayerBufs &B = m->L[l];
    sx::PfAttnArgs probe{};
    probe.num_q = m->nq;
    probe.num_kv = B.num_kv;
    probe.head_dim = B.head_dim;
    probe.kv_bf16 = c.kv_bf16 ? 1u : 0u;
    probe.total_slots = ts;
    if (sx::pf_attn_tc_ok(probe) && B.num_kv)
      if (!items_for(m->nq / B.num_kv, &layer_items[2 * l], &layer_items[2 * l + 1]))
        layer_items[2 * l + 1] = 0;
  }
  for (size_t i = 0; i < item_sets.size(); ++i)
    M_TRY(cp(d_items + i * 2 * T, item_sets[i].second.data(), 4ull * item_sets[i].second.size()));
  const float eps = c.rms_norm_eps;
  auto run = [&](cudaError_t ce, const char *what) { return sx_host_cuda_status(ce, what); };
  for (uint32_t l = 0; l < L; ++l) {
    LayerBufs &B = m->L[l];
    const uint32_t base = B.q_dim + 2 * B.kv_dim;
    // input norm, after layer 0 with the previous layer's residual update
    sx::PfNormArgs na{};
    na.n = H;
    na.eps = eps;
    na.w = (const float *)B.in_norm->d;
    na.out = xn;
    if (l == 0) {
      na.x = xa;
    } else {
      const LayerBufs &P = m->L[l - 1];
      na.x = xb;
      na.mlp = mlp;
      na.post_w = c.has_post_norms ? (const float *)P.post_ffn->d : nullptr;
      na.scalar = P.layer_scalar;
      na.x_out = xa;
    }
    M_TRY(run(sx::launch_pf_norm(na, T, true, s), "prefill norm"));
    M_TRY(run(sx::launch_prefill_q4(B.wq->d, xn, y, T, base, H, base, e->err_dev, s),
              "prefill qkv gemm"));
    sx_status fst = SX_OK;
    const float *freq = sx_host_inv_freq(e, B.rot, B.theta, &fst);
    if (!freq) return fst;
    sx::PfQkvArgs qa{};
    qa.y = y;
    qa.ldy = base;
    qa.q_norm_w = (const float *)B.q_norm->d;
    qa.k_norm_w = (const float *)B.k_norm->d;
    qa.inv_freq = freq;
    qa.q_out = qo;
    qa.k_cache = B.kc->d;
    qa.v_cache = B.vc->d;
    qa.cache_ld = (uint64_t)ts * B.kv_dim;
    qa.sess = d_sess;
    qa.clock = d_clock;
    qa.slot = d_slot;
    qa.sessions = m->S;
    qa.total_slots = ts;
    qa.num_q = m->nq;
    qa.num_kv = B.num_kv;
    qa.head_dim = B.head_dim;
    qa.rotary_dim = B.rot;
    qa.k_eq_v = B.k_eq_v;
    qa.kv_bf16 = c.kv_bf16 ? 1u : 0u;
    qa.eps = eps;
    qa.err = e->err_dev;
    M_TRY(run(sx::launch_pf_qkv_rope(qa, T, s), "prefill qkv rope"));
    sx::PfAttnArgs aa{};
    aa.q = qo;
    aa.k_cache = B.kc->d;
    aa.v_cache = B.vc->d;
    aa.cache_ld = qa.cache_ld;
    aa.sess = d_sess;
    aa.slots = lists;
    aa.count = d_cnt;
    aa.out = xn;
    aa.tokens = T;
    aa.sessions = m->S;
    aa.total_slots = ts;
    aa.num_q = m->nq;
    aa.num_kv = B.num_kv;
    aa.head_dim = B.head_dim;
    aa.kv_bf16 = qa.kv_bf16;
    aa.scale = c.attn_scale;
    aa.err = e->err_dev;
    if (layer_items[2 * l + 1]) {
      aa.items = d_items + layer_items[2 * l];
      aa.n_items = layer_items[2 * l + 1];
    }
    M_TRY(run(sx::launch_pf_attn(aa, s), "prefill attention"));
    M_TRY(run(sx::launch_prefill_q4(B.wo->d, xn, mlp, T, H, B.q_dim, H, e->err_dev, s),
              "prefill o gemm"));
    // post-attention residual and pre-FFN norm
    sx::PfNormArgs nb{};
    nb.n = H;
    nb.eps = eps;
    nb.x = xa;
    nb.mlp = mlp;
    nb.post_w = c.has_post_norms ? (const float *)B.post_attn->d : nullptr;
    nb.scalar = 1.0f;
    nb.x_out = xb;
    nb.w = (const float *)B.pre_ffn->d;
    nb.out = xn;
    M_TRY(run(sx::launch_pf_norm(nb, T, true, s), "prefill pre-ffn norm"));
    M_TRY(run(sx::launch_prefill_q4(B.wg->d, xn, y, T, I, H, I, e->err_dev, s), "prefill gate"));
    M_TRY(run(sx::launch_prefill_q4(B.wu->d, xn, y2, T, I, H, I, e->err_dev, s), "prefill up"));
    M_TRY(run(sx::launch_pf_geglu(y, y2, xn, (size_t)T * I, s), "prefill geglu"));
    M_TRY(run(sx::launch_prefill_q4(B.wd->d, xn, mlp, T, H, I, H, e->err_dev, s),
              "prefill down gemm"));
  }
  if (n_out) {
    // last residual update and final norm of the output rows, then the Q8 LM head + argmax
    const LayerBufs &P = m->L[L - 1];
    sx::PfNormArgs nf{};
    nf.n = H;
    nf.eps = eps;
    nf.x = xb;
    nf.mlp = mlp;
    nf.post_w = c.has_post_norms ? (const float *)P.post_ffn->d : nullptr;
    nf.scalar = P.layer_scalar;
    nf.x_out = xa;
    nf.w = (const float *)m->final_norm->d;
    nf.out = d_norm;
    nf.rows = d_rows;
    M_TRY(run(sx::launch_pf_norm(nf, n_out, false, s), "prefill final norm"));
    sx::GemvArgs h{};
    h.w[0][0] = h.w[0][1] = m->lm_head->d;
    h.y[0] = d_logits;
    h.rows[0] = m->V;
    h.tiles[0] = sx::tiles_of(m->V);
    h.k = H;
    h.batch = n_out;
    h.ldy = m->V;
    h.x = d_norm;
    h.ldx = H;
    h.pro = sx::kProNone;
    h.epi = sx::kEpiArgmax;
    h.token = d_tok;
    M_TRY(sx_host_check_gemv(8, false, false, m->V, H, n_out));
    sx_host_bind_scratch(e, h);
    M_TRY(run(sx::launch_gemv(8, false, h, e->num_sms, s, false), "prefill lm head"));
    uint32_t tok_h[8];
    M_TRY(sx_host_cuda_status(
        cudaMemcpyAsync(tok_h, d_tok, 4ull * n_out, cudaMemcpyDeviceToHost, s), "tokens"));
    if (logits_out)
      M_TRY(sx_host_cuda_status(cudaMemcpyAsync(logits_out, d_logits, 4ull * n_out * m->V,
                                                cudaMemcpyDeviceToHost, s),
                                "logits"));
    M_TRY(sx_engine_sync(e));
    if (tokens) memcpy(tokens, tok_h, 4ull * n_out);
    return SX_OK;
  }
  return sx_engine_sync(e);
}

// ---------------------------------------------------------------------------------------
// The recall tier on the device (sx_archive.cu): DiffArchive + integrateMemory over this
// model's caches (session 0) and the caller's ring.
struct sx_archive {
  sx_model *m = nullptr;
  sx::ArchiveArgs a{};
  void *block = nullptr;            // one device allocation for everything below
  sx::ArchiveLayer *d_layers = nullptr;
  uint32_t *h_out = nullptr;        // pinned: state[5] | selected[R] | timestamps (u64)[R]
  uint32_t count = 0;
};

extern "C" {

SX_API sx_status sx_archive_create(sx_model *m, uint32_t capacity, const sx_salience_config *cfg,
                                   sx_archive **out) {
  if (!m || !out || capacity == 0 || capacity > sx::kArchiveMaxCapacity) {
    sx_host_set_error("archive_create: need a model and 1 <= capacity <= %u",
                      sx::kArchiveMaxCapacity);
    return SX_ERR_INVALID;
  }
  if (m->c.num_recall > 1024 || m->comm) {
    sx_host_set_error("archive_create: at most 1024 recall slots, one GPU");
    return SX_ERR_UNSUPPORTED;
  }
  sx_engine *e = m->e;
  M_TRY(sx_host_cuda_status(cudaSetDevice(e->device), "cudaSetDevice"));
  const uint32_t H = m->c.hidden_size, L = m->c.num_layers, R = m->c.num_recall;
  uint32_t max_kv = 0;
  for (const LayerBufs &B : m->L) max_kv = B.kv_dim > max_kv ? B.kv_dim : max_kv;
  const size_t eb = m->c.kv_bf16 ? 2 : 4;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  };
  const size_t o_prev = take(4ull * H), o_vec = take(4ull * capacity * H);
  const size_t o_ts = take(8ull * capacity), o_la = take(8ull * capacity);
  const size_t o_ac = take(4ull * capacity), o_sal = take(4ull * capacity);
  const size_t o_kv = take((size_t)capacity * L * 2 * max_kv * eb), o_sc = take(4ull * capacity);
  const size_t o_st = take(64), o_sel = take(4ull * (R + 1)), o_sts = take(8ull * (R + 1));
  const size_t o_lay = take(sizeof(sx::ArchiveLayer) * L);
  sx_archive *a = new sx_archive();
  a->m = m;
  sx_status st = sx_host_cuda_status(cudaMalloc(&a->block, off), "archive memory");
  if (st == SX_OK)
    st = sx_host_cuda_status(cudaMemset(a->block, 0, off), "archive memory");
  if (st == SX_OK)
    st = sx_host_cuda_status(
        cudaHostAlloc((void **)&a->h_out, 4 * (8 + 3 * (R + 1)), cudaHostAllocDefault),
        "archive readback");
  if (st != SX_OK) {
    sx_archive_destroy(a);
    return st;
  }
  uint8_t *b = static_cast<uint8_t *>(a->block);
  std::vector<sx::ArchiveLayer> lay(L);
  for (uint32_t l = 0; l < L; ++l) lay[l] = {m->L[l].kc->d, m->L[l].vc->d, m->L[l].kv_dim};
  a->d_layers = reinterpret_cast<sx::ArchiveLayer *>(b + o_lay);
  st = sx_host_cuda_status(cudaMemcpy(a->d_layers, lay.data(), sizeof(sx::ArchiveLayer) * L,
                                      cudaMemcpyHostToDevice),
                           "archive layers");
  if (st != SX_OK) {
    sx_archive_destroy(a);
    return st;
  }
  sx::ArchiveArgs &A = a->a;
  A.normed = (const float *)m->normed->d;
  A.prev = reinterpret_cast<float *>(b + o_prev);
  A.vectors = reinterpret_cast<float *>(b + o_vec);
  A.timestamp = reinterpret_cast<uint64_t *>(b + o_ts);
  A.last_accessed = reinterpret_cast<uint64_t *>(b + o_la);
  A.access_count = reinterpret_cast<uint32_t *>(b + o_ac);
  A.salience = reinterpret_cast<float *>(b + o_sal);
  A.kv = b + o_kv;
  A.scores = reinterpret_cast<float *>(b + o_sc);
  A.state = reinterpret_cast<uint32_t *>(b + o_st);
  A.selected = reinterpret_cast<uint32_t *>(b + o_sel);
  A.sel_ts = reinterpret_cast<uint64_t *>(b + o_sts);
  A.layers = a->d_layers;
  A.dim = H;
  A.capacity = capacity;
  A.num_layers = L;
  A.max_kv = max_kv;
  A.kv_bf16 = m->c.kv_bf16 ? 1u : 0u;
  A.num_recall = R;
  A.recall_start = m->c.num_anchors + m->c.window_size;
  // SalienceConfig defaults (memory.zig:5-7)
  A.alpha = cfg ? cfg->alpha : 1.0f;
  A.beta = cfg ? cfg->beta : 0.5f;
  A.gamma = cfg ? cfg->gamma : 1.0f;
  A.lambda = cfg ? cfg->lambda : 1.0f / 2048.0f;
  *out = a;
  return SX_OK;
}

SX_API void sx_archive_destroy(sx_archive *a) {
  if (!a) return;
  cudaSetDevice(a->m->e->device);
  cudaStreamSynchronize(a->m->e->stream);
  if (a->block) cudaFree(a->block);
  if (a->h_out) cudaFreeHost(a->h_out);
  delete a;
}

SX_API sx_status sx_archive_integrate(sx_archive *a, sx_ring *ring, uint64_t clock,
                                     uint32_t *n_selected, uint32_t *selected) {
  if (!a || !ring) {
    sx_host_set_error("archive_integrate: null argument");
    return SX_ERR_INVALID;
  }
  if (sx_ring_total_slots(ring) != a->m->total_slots) {
    sx_host_set_error("archive_integrate: the ring does not match the model's slots");
    return SX_ERR_INVALID;
  }
  sx_engine *e = a->m->e;
  M_TRY(sx_host_cuda_status(cudaSetDevice(e->device), "cudaSetDevice"));
  sx::ArchiveArgs A = a->a;
  A.clock = clock;
  A.slot = sx_ring_slot_index(ring, clock);
  M_TRY(sx_host_cuda_status(sx::launch_archive_integrate(A, e->stream), "archive launch"));
  const uint32_t R = A.num_recall;
  uint32_t *h = a->h_out;
  M_TRY(sx_host_cuda_status(cudaMemcpyAsync(h, A.state, 4 * 5, cudaMemcpyDeviceToHost, e->stream),
                            "archive readback"));
  M_TRY(sx_host_cuda_status(
      cudaMemcpyAsync(h + 8, A.selected, 4ull * R, cudaMemcpyDeviceToHost, e->stream),
      "archive readback"));
  M_TRY(sx_host_cuda_status(
      cudaMemcpyAsync(h + 8 + (R + 1), A.sel_ts, 8ull * R, cudaMemcpyDeviceToHost, e->stream),
      "archive readback"));
  M_TRY(sx_engine_sync(e));
  a->count = h[0];
  const uint32_t k = R ? h[4] : 0;
  const uint64_t *ts = reinterpret_cast<const uint64_t *>(h + 8 + (R + 1));
  // clearRecall, then writeRecallKV's bookkeeping for every rank (memory_inject.zig:39-45);
  // the model's ring keeps one bookkeeping layer, read by every layer
  sx_ring_clear_recall(ring);
  for (uint32_t r = 0; r < k; ++r) sx_ring_write_recall(ring, 0, r, ts[r]);
  if (n_selected) *n_selected = k;
  if (selected)
    for (uint32_t r = 0; r < k; ++r) selected[r] = h[8 + r];
  return SX_OK;
}

SX_API uint32_t sx_archive_count(const sx_archive *a) { return a ? a->count : 0; }

SX_API sx_status sx_archive_entry(sx_archive *a, uint32_t i, float *vec, uint64_t *timestamp,
                                  uint64_t *last_accessed, uint32_t *access_count,
                                  float *salience) {
  if (!a || i >= a->a.capacity) {
    sx_host_set_error("archive_entry: index out of range");
    return SX_ERR_INVALID;
  }
  sx_engine *e = a->m->e;
  M_TRY(sx_host_cuda_status(cudaSetDevice(e->device), "cudaSetDevice"));
  M_TRY(sx_host_cuda_status(cudaStreamSynchronize(e->stream), "archive sync"));
  const sx::ArchiveArgs &A = a->a;
  cudaError_t ce = cudaSuccess;
  if (vec && ce == cudaSuccess)
    ce = cudaMemcpy(vec, A.vectors + (size_t)i * A.dim, 4ull * A.dim, cudaMemcpyDeviceToHost);
  if (timestamp && ce == cudaSuccess)
    ce = cudaMemcpy(timestamp, A.timestamp + i, 8, cudaMemcpyDeviceToHost);
  if (last_accessed && ce == cudaSuccess)
    ce = cudaMemcpy(last_accessed, A.last_accessed + i, 8, cudaMemcpyDeviceToHost);
  if (access_count && ce == cudaSuccess)
    ce = cudaMemcpy(access_count, A.access_count + i, 4, cudaMemcpyDeviceToHost);
  if (salience && ce == cudaSuccess)
    ce = cudaMemcpy(salience, A.salience + i, 4, cudaMemcpyDeviceToHost);
  return sx_host_cuda_status(ce, "archive entry readback");
}

}  // extern "C"
