// sx_engine.cu -- host side of libsx: the C ABI declared in include/sx.h.
//
// Mirrors the reference's GPU dispatch layer (src/gpu/kernels.zig GpuEngine,
// src/gpu/model_gpu.zig GpuModelContext, src/gpu/model_dispatch.zig) on CUDA:
//   Vulkan command buffer  -> list of recorded ops, captured into a CUDA graph at end()
//   descriptor set         -> ordered tuple of device buffers
//   vkQueueSubmit + fence  -> cudaGraphLaunch + deadline-bounded cudaStreamQuery poll
// Nothing here falls back to the CPU: every op is a CUDA kernel from csrc/.
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/sx.h"
#include "sx_common.cuh"
#include "sx_internal.h"
#include "sx_host.h"

namespace {

thread_local std::string g_last_error;

void set_error(const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

sx_status cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return SX_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  if (e == cudaErrorMemoryAllocation) return SX_ERR_OOM;
  if (e == cudaErrorLaunchFailure || e == cudaErrorLaunchOutOfResources ||
      e == cudaErrorInvalidConfiguration)
    return SX_ERR_LAUNCH;
  return SX_ERR_CUDA;
}

#define SX_TRY_CUDA(expr, what)                          \
  do {                                                   \
    sx_status _s = cuda_status((expr), (what));          \
    if (_s != SX_OK) return _s;                          \
  } while (0)

#define SX_CHECK_ARG(cond, ...)  \
  do {                           \
    if (!(cond)) {               \
      set_error(__VA_ARGS__);    \
      return SX_ERR_INVALID;     \
    }                            \
  } while (0)

}  // namespace

void sx_host_set_error(const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void sx_host_bind_scratch(sx_engine *e, sx::GemvArgs &a) {
  a.part = e->gemv_part;
  a.tile_cnt = e->tile_cnt;
  a.best_v = e->best_v;
  a.best_i = e->best_i;
  a.done_cnt = e->done_cnt;
  a.err = e->err_dev;
}
void sx_host_bind_scratch(sx_engine *e, sx::AttnFusedArgs &a) {
  a.part = e->attn_part;
  a.cnt = e->attn_cnt;
  a.err = e->err_dev;
}
sx_status sx_host_cuda_status(cudaError_t e, const char *what) { return cuda_status(e, what); }

namespace {

float *engine_inv_freq(sx_engine *e, uint32_t rot, float theta, sx_status *st) {
  uint32_t tb;
  memcpy(&tb, &theta, 4);
  std::lock_guard<std::mutex> lk(e->freq_mu);
  auto key = std::make_pair(rot, tb);
  auto it = e->inv_freq.find(key);
  if (it != e->inv_freq.end()) return it->second;
  std::vector<float> h(rot / 2 + 1, 0.0f);
  sx_rope_inv_freq(h.data(), rot, theta);
  float *d = nullptr;
  cudaError_t ce = cudaMalloc(&d, sizeof(float) * h.size());
  if (ce == cudaSuccess)
    ce = cudaMemcpy(d, h.data(), sizeof(float) * h.size(), cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) {
    *st = cuda_status(ce, "inv_freq table");
    return nullptr;
  }
  e->inv_freq[key] = d;
  return d;
}

}  // namespace
float *sx_host_inv_freq(sx_engine *e, uint32_t rot, float theta, sx_status *st) {
  return engine_inv_freq(e, rot, theta, st);
}
namespace {

int qt_of(sx_quant_mode m) { return m == SX_QUANT_Q4 ? 4 : m == SX_QUANT_Q8 ? 8 : 0; }

sx_status check_gemv_shape(int qt, bool geglu, bool pro, uint32_t m, uint32_t k,
                           uint32_t batch) {
  SX_CHECK_ARG(m > 0 && k > 0 && (k % 32) == 0, "gemv: need m > 0 and k a multiple of 32 (m=%u k=%u)", m, k);
  SX_CHECK_ARG(batch >= 1 && batch <= 8, "gemv: batch must be 1..8 (got %u)", batch);
  SX_CHECK_ARG(sx::tiles_of(m) <= sx::kMaxGemvTiles, "gemv: at most %u rows", sx::kMaxGemvTiles * 16);
  SX_CHECK_ARG(!pro || k <= sx::kGemvPrologueMaxK, "gemv: fused norm prologue needs k <= %u",
               sx::kGemvPrologueMaxK);
  size_t smem = sx::gemv_smem_bytes(qt, k, batch, geglu, pro);
  if (smem > 227 * 1024) {
    set_error("gemv: k=%u with batch %u needs %zu B of shared memory (max 227 KB)", k, batch, smem);
    return SX_ERR_UNSUPPORTED;
  }
  return SX_OK;
}

}  // namespace
sx_status sx_host_check_gemv(int qt, bool geglu, bool pro, uint32_t m, uint32_t k,
                             uint32_t batch) {
  return check_gemv_shape(qt, geglu, pro, m, k, batch);
}
namespace {

sx_status do_gemv(sx_engine *e, cudaStream_t s, int qt, bool geglu, const void *w0,
                  const void *w1, const float *x, float *y, uint32_t m, uint32_t k,
                  uint32_t batch, const uint32_t *gate = nullptr) {
  if (qt == 0) {  // mode none: bf16 weights (gemv_bf16.wgsl)
    SX_CHECK_ARG(m > 0 && k > 0 && k % 8 == 0 && batch >= 1 && batch <= 8,
                 "gemv bf16: need m > 0, k a multiple of 8 and batch 1..8 (m=%u k=%u batch=%u)",
                 m, k, batch);
    SX_CHECK_ARG(w0 && x && y && (!geglu || w1), "gemv: null pointer");
    SX_CHECK_ARG(((uintptr_t)w0 | (uintptr_t)(geglu ? w1 : w0) | (uintptr_t)x) % 16 == 0,
                 "gemv bf16: weights and x must be 16-byte aligned");
    return cuda_status(sx::launch_gemv_bf16(geglu, (const uint16_t *)w0, (const uint16_t *)w1, x,
                                            y, m, k, batch, e->num_sms, s, gate),
                       "gemv bf16 launch");
  }
  SX_CHECK_ARG(qt == 4 || qt == 8, "gemv: unsupported quant mode");
  sx_status st = check_gemv_shape(qt, geglu, false, m, k, batch);
  if (st != SX_OK) return st;
  SX_CHECK_ARG(w0 && x && y && (!geglu || w1), "gemv: null pointer");
  SX_CHECK_ARG(((uintptr_t)w0 | (uintptr_t)(geglu ? w1 : w0) | (uintptr_t)x) % 16 == 0,
               "gemv: packed weights and x must be 16-byte aligned");
  sx::GemvArgs a{};
  a.w[0][0] = w0;
  a.w[0][1] = geglu ? w1 : w0;
  a.y[0] = y;
  a.rows[0] = m;
  a.tiles[0] = sx::tiles_of(m);
  a.k = k;
  a.batch = batch;
  a.ldy = m;
  a.x = x;
  a.ldx = k;
  a.pro = sx::kProNone;
  a.epi = sx::kEpiPlain;
  a.gate = gate;
  sx_host_bind_scratch(e, a);
  return cuda_status(sx::launch_gemv(qt, geglu, a, e->num_sms, s, true), "gemv launch");
}

sx_status do_norm(cudaStream_t s, bool add, float *x, const float *r, const float *w, float *y,
                  uint32_t n, uint32_t batch, float eps, float scalar,
                  const uint32_t *gate = nullptr) {
  SX_CHECK_ARG(n > 0 && batch > 0, "rmsnorm: empty input");
  SX_CHECK_ARG(x && w && y && (!add || r), "rmsnorm: null pointer");
  sx::NormArgs a{x, r, w, y, n, batch, n, eps, scalar};
  a.gate = gate;
  return cuda_status(sx::launch_rmsnorm(add, a, s), "rmsnorm launch");
}

sx_status do_qkv_rope(sx_engine *e, cudaStream_t s, const float *q_in, const float *k_in,
                      const float *v_in, const float *qnw, const float *knw, float *q_out,
                      void *kc, void *vc, const uint32_t *step, uint32_t num_q, uint32_t num_kv,
                      uint32_t head_dim, uint32_t rot, uint32_t k_eq_v, float theta, float eps,
                      uint32_t total_slots, const uint32_t *gate = nullptr) {
  SX_CHECK_ARG(num_q > 0 && head_dim > 0 && head_dim <= 4096 && rot <= head_dim && rot % 2 == 0,
               "qkv_rope: bad shape (num_q=%u head_dim=%u rot=%u)", num_q, head_dim, rot);
  SX_CHECK_ARG(total_slots > 0, "qkv_rope: total_slots must be > 0");
  sx_status st = SX_OK;
  float *freq = engine_inv_freq(e, rot, theta, &st);
  if (!freq) return st;
  sx::QkvRopeArgs a{q_in, k_in, v_in, qnw, knw, q_out, kc, vc, step, freq,
                    num_q, num_kv, head_dim, rot, k_eq_v, e->kv_bf16 ? 1u : 0u, total_slots,
                    eps, e->err_dev};
  a.gate = gate;
  return cuda_status(sx::launch_qkv_rope(a, s), "qkv_rope launch");
}

sx_status do_attn(sx_engine *e, cudaStream_t s, const float *q, const void *kc, const void *vc,
                  const uint32_t *slots, const uint32_t *step, float *out, uint32_t head_dim,
                  uint32_t kv_dim, uint32_t gqa, float scale, uint32_t num_q,
                  uint32_t total_slots, const uint32_t *gate = nullptr) {
  SX_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512,
               "decode_attn: head_dim must be 64/128/256/512 (got %u)", head_dim);
  SX_CHECK_ARG(gqa == 1 || gqa == 2 || gqa == 4 || gqa == 8,
               "decode_attn: gqa ratio must be 1/2/4/8 (got %u)", gqa);
  SX_CHECK_ARG(num_q % gqa == 0 && (num_q / gqa) * head_dim <= kv_dim,
               "decode_attn: num_q_heads/gqa_ratio kv heads do not fit kv_dim");
  SX_CHECK_ARG(total_slots > 0, "decode_attn: total_slots must be > 0");
  SX_CHECK_ARG(q && kc && vc && slots && step && out, "decode_attn: null pointer");
  SX_CHECK_ARG(((uintptr_t)kc | (uintptr_t)vc) % 16 == 0 && kv_dim % 8 == 0,
               "decode_attn: caches must be 16-byte aligned with kv_dim a multiple of 8");
  size_t need = sx::attn_scratch_bytes(num_q, total_slots, head_dim);
  if (need > e->attn_part_bytes) {
    set_error("decode_attn: needs %zu B scratch, engine has %zu", need, e->attn_part_bytes);
    return SX_ERR_UNSUPPORTED;
  }
  sx::AttnArgs a{q, kc, vc, slots, step, out, e->attn_part, head_dim, kv_dim,
                 gqa, num_q, total_slots, e->kv_bf16 ? 1u : 0u, scale, e->err_dev};
  a.gate = gate;
  return cuda_status(sx::launch_decode_attn(a, s), "decode_attn launch");
}

sx_status do_argmax(sx_engine *e, cudaStream_t s, const float *logits, uint32_t n,
                    uint32_t *out) {
  SX_CHECK_ARG(n > 0 && logits && out, "argmax: empty input");
  return cuda_status(
      sx::launch_argmax(logits, n, out, e->argmax_part, sx::argmax_scratch_bytes(), s),
      "argmax launch");
}



sx_status run_op(sx_engine *e, cudaStream_t s, const Op &op, uint32_t *kernels) {
  switch (op.kind) {
    case OP_GEMV:
    case OP_GEMV_LOGITS: {
      // the logits GEMV is Q8 when the layers are quantised, bf16 in mode none
      // (kernels.zig:38: Q8 for q4, the layer format otherwise)
      int qt = op.kind == OP_GEMV_LOGITS ? (e->mode == SX_QUANT_NONE ? 0 : 8) : qt_of(e->mode);
      *kernels += 1;
      return do_gemv(e, s, qt, false, op.bind.at(0), nullptr, (const float *)op.bind.at(1),
                     (float *)op.bind.at(2), op.u[0], op.u[1], 1, op.gate);
    }
    case OP_GATE_UP:
      *kernels += 1;
      return do_gemv(e, s, qt_of(e->mode), true, op.bind.at(0), op.bind.at(1),
                     (const float *)op.bind.at(2), (float *)op.bind.at(3), op.u[0], op.u[1], 1,
                     op.gate);
    case OP_ADD_RMSNORM:
      *kernels += 1;
      return do_norm(s, true, (float *)op.bind.at(0), (const float *)op.bind.at(1),
                     (const float *)op.bind.at(2), (float *)op.bind.at(3), op.u[0], 1, op.f[0],
                     op.f[1], op.gate);
    case OP_RMSNORM:
      *kernels += 1;
      return do_norm(s, false, (float *)op.bind.at(0), nullptr, (const float *)op.bind.at(1),
                     (float *)op.bind.at(2), op.u[0], 1, op.f[0], 1.0f, op.gate);
    case OP_ATTN:
      *kernels += 2;
      return do_attn(e, s, (const float *)op.bind.at(0), op.bind.at(1), op.bind.at(2),
                     (const uint32_t *)op.bind.at(3), (const uint32_t *)op.bind.at(5),
                     (float *)op.bind.at(4), op.u[0], op.u[1], op.u[2], op.f[0], op.u[3], op.u[4],
                     op.gate);
    case OP_QKV_ROPE:
      *kernels += 1;
      return do_qkv_rope(e, s, (const float *)op.bind.at(0), (const float *)op.bind.at(1),
                         (const float *)op.bind.at(2), (const float *)op.bind.at(3),
                         (const float *)op.bind.at(4), (float *)op.bind.at(5), op.bind.at(6),
                         op.bind.at(7), (const uint32_t *)op.bind.at(8), op.u[0], op.u[1],
                         op.u[2], op.u[3], op.u[4], op.f[0], op.f[1], op.u[5], op.gate);
    case OP_QGATE: {
      *kernels += 1;
      sx::GateArgs g = op.qgate;
      g.x = (const float *)op.bind.at(0);
      g.x_prev = (float *)op.bind.at(1);
      g.ind = (uint32_t *)op.bind.at(2);
      return cuda_status(sx::launch_quiescence_gate(g, s), "quiescence gate launch");
    }
    case OP_ARGMAX:
      *kernels += 2;
      return do_argmax(e, s, (const float *)op.bind.at(0), op.u[0], (uint32_t *)op.bind.at(1));
    case OP_GEMV_FUSED:
      *kernels += 1;
      if (!sx::gemv_segments_contiguous(op.gemv, op.qt, op.geglu ? 2 : 1)) {
        set_error("fused gemv: the segments of a multi-segment call must lie back to back");
        return SX_ERR_UNSUPPORTED;
      }
      return cuda_status(sx::launch_gemv(op.qt, op.geglu, op.gemv, e->num_sms, s, true),
                         "fused gemv launch");
    case OP_ATTN_FUSED: {
      *kernels += 1;
      sx::AttnFusedArgs a = op.attnf;
      sx_status fst = SX_OK;
      a.inv_freq = engine_inv_freq(e, op.attn_rot, op.attn_theta, &fst);
      if (!a.inv_freq) return fst;
      return cuda_status(sx::launch_attn_fused(a, s, true), "fused attention launch");
    }
    case OP_ATTN_BLOCK: {
      *kernels += 1;
      sx::AttnBlockArgs a = op.ab;
      sx_status fst = SX_OK;
      a.at.inv_freq = engine_inv_freq(e, op.attn_rot, op.attn_theta, &fst);
      if (!a.at.inv_freq) return fst;
      return cuda_status(sx::launch_attn_block(a, s), "attention block launch");
    }
    case OP_ATTN_O: {
      *kernels += 1;
      sx::AttnOArgs a = op.ao;
      sx_status fst = SX_OK;
      a.at.inv_freq = engine_inv_freq(e, op.attn_rot, op.attn_theta, &fst);
      if (!a.at.inv_freq) return fst;
      return cuda_status(sx::launch_attn_o(a, s), "attention + o launch");
    }
    case OP_ALLREDUCE:
      return sx_host_allreduce(op.comm, static_cast<float *>(op.dev), op.u[0], s);
    case OP_ALLGATHER:
      return sx_host_allgather(op.comm, static_cast<const uint32_t *>(op.bind.at(0)),
                               static_cast<uint32_t *>(op.bind.at(1)), op.u[0], s);
    case OP_TP_ARGMAX:
      *kernels += 1;
      return sx_host_tp_argmax(static_cast<const uint32_t *>(op.bind.at(0)), op.u[0],
                               static_cast<uint32_t *>(op.bind.at(1)), s);
    case OP_STREAM: {
      *kernels += 1;
      SX_TRY_CUDA(cudaMemsetAsync(op.bind.at(0), 0, 4ull * (op.u[0] + 1), s), "counter reset");
      return cuda_status(sx::launch_stream(static_cast<const sx::Phase *>(op.dev), op.u[0],
                                           static_cast<uint32_t *>(op.bind.at(0)), e->err_dev,
                                           e->num_sms, s),
                         "streaming decode launch");
    }
    case OP_PERSIST: {
      *kernels += 1;
      SX_TRY_CUDA(cudaMemsetAsync(e->persist_bar, 0, 8, s), "barrier reset");
      return cuda_status(sx::launch_persist(static_cast<const sx::Phase *>(op.dev), op.u[0],
                                            e->persist_bar, e->err_dev,
                                            e->num_sms, s),
                         "persistent decode launch");
    }
    case OP_H2D:
      return cuda_status(cudaMemcpyAsync(op.dev, op.host, op.bytes, cudaMemcpyHostToDevice, s),
                         "h2d copy");
    case OP_D2H:
      return cuda_status(cudaMemcpyAsync(op.host, op.dev, op.bytes, cudaMemcpyDeviceToHost, s),
                         "d2h copy");
  }
  set_error("unknown op");
  return SX_ERR_INVALID;
}

// set arity per op, as bound in model_gpu.zig:140-156
bool set_ok(sx_set *s, size_t n) {
  if (!s || s->b.size() < n) return false;
  for (size_t i = 0; i < n; ++i)
    if (!s->b[i] || !s->b[i]->d) return false;
  return true;
}

void poison(sx_cmd *c, sx_status st, const char *msg) {
  if (c->poisoned == SX_OK) {
    c->poisoned = st;
    c->poison_msg = msg;
  }
}

bool record_guard(sx_engine *e, sx_cmd *c, sx_set *s, size_t arity, const char *name) {
  if (!c) return false;
  if (!e || c->e != e) {
    poison(c, SX_ERR_INVALID, "record: engine does not own this command buffer");
    return false;
  }
  if (!c->recording) {
    poison(c, SX_ERR_INVALID, "record: command buffer is not recording (call sx_cmd_begin)");
    return false;
  }
  if (arity && !set_ok(s, arity)) {
    std::string m = std::string(name) + ": descriptor set has too few bound buffers";
    poison(c, SX_ERR_INVALID, m.c_str());
    return false;
  }
  return true;
}

sx_status wait_stream(sx_engine *e, cudaStream_t s, uint64_t timeout_ns) {
  // kernels.zig:151-156: spin on the fence, then a bounded wait (5 s) -> VkFenceTimeout
  if (timeout_ns == 0) timeout_ns = 5000000000ull;
  auto t0 = std::chrono::steady_clock::now();
  uint64_t spins = 0;
  for (;;) {
    cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return cuda_status(q, "stream query");
    auto dt = std::chrono::duration_cast<std::chrono::nanoseconds>(
                  std::chrono::steady_clock::now() - t0)
                  .count();
    if ((uint64_t)dt > timeout_ns) {
      set_error("submit: work did not finish within %llu ns", (unsigned long long)timeout_ns);
      return SX_ERR_TIMEOUT;
    }
    if (++spins > 2000) std::this_thread::yield();
  }
  uint32_t err = __atomic_load_n(e->err_host, __ATOMIC_ACQUIRE);
  if (err != 0) {
    __atomic_store_n(e->err_host, 0u, __ATOMIC_RELEASE);
    set_error("device reported error code %u (1=wait timeout, 2=bad params, 3=bad slot)", err);
    return SX_ERR_DEVICE;
  }
  return SX_OK;
}

}  // namespace

// ---------------------------------------------------------------------------------------
// misc
extern "C" {

SX_API const char *sx_version(void) { return "sx 0.1 (sm_100a)"; }
SX_API const char *sx_last_error(void) { return g_last_error.c_str(); }
SX_API const char *sx_status_string(sx_status s) {
  switch (s) {
    case SX_OK: return "ok";
    case SX_ERR_INVALID: return "invalid argument";
    case SX_ERR_CUDA: return "cuda error";
    case SX_ERR_LAUNCH: return "launch failed";
    case SX_ERR_TIMEOUT: return "timeout";
    case SX_ERR_OOM: return "out of device memory";
    case SX_ERR_PEER: return "peer exchange failed";
    case SX_ERR_UNSUPPORTED: return "unsupported";
    case SX_ERR_DEVICE: return "device-side error";
  }
  return "unknown status";
}

SX_API uint64_t sx_quantized_row_words(uint32_t cols, sx_quant_mode mode) {
  uint64_t nb = (cols + 31u) / 32u;
  if (mode == SX_QUANT_Q8) return nb * 9;
  if (mode == SX_QUANT_Q4) return nb * 5;
  return cols / 2;
}

SX_API uint64_t sx_packed_bytes(uint32_t rows, uint32_t cols, sx_quant_mode mode) {
  uint64_t chunks = (uint64_t)sx::tiles_of(rows) * sx::pairs_of(cols);
  if (mode == SX_QUANT_Q4) return chunks * sx::kQ4ChunkBytes;
  if (mode == SX_QUANT_Q8) return chunks * sx::kQ8ChunkBytes;
  return (uint64_t)rows * cols * 2;  // bf16 rows as the reference stores them (mode none)
}

SX_API void sx_rope_inv_freq(float *out, uint32_t rotary_dim, float theta) {
  for (uint32_t i = 0; i < rotary_dim / 2; ++i)
    out[i] = 1.0f / powf(theta, (float)(2 * i) / (float)rotary_dim);
}

SX_API void sx_synth_embed_row(float *x, uint32_t hidden, uint32_t token, uint64_t seed) {
  float sc = sqrtf((float)hidden);
  for (uint32_t j = 0; j < hidden; ++j) {
    float e = sx::bf16_bits_to_f32(
        sx::bf16_bits_rne(sx::synth_normal(seed, 1, (uint64_t)token * hidden + j)));
    x[j] = e * sc;
  }
}

// ---------------------------------------------------------------------------------------
// ring buffer (ring_buffer.zig)
}  // extern "C"

struct sx_ring {
  uint32_t num_layers, num_anchors, window_size, num_recall, total_slots;
  std::vector<uint64_t> clocks;
  std::vector<uint8_t> active;
  uint64_t total_ingested = 0;
};

extern "C" {

SX_API sx_status sx_ring_create(uint32_t num_layers, uint32_t num_anchors, uint32_t window_size,
                                uint32_t num_recall, sx_ring **out) {
  SX_CHECK_ARG(out, "ring: null out");
  SX_CHECK_ARG(num_layers > 0 && window_size > 0, "ring: need num_layers > 0 and window_size > 0");
  sx_ring *r = new sx_ring();
  r->num_layers = num_layers;
  r->num_anchors = num_anchors;
  r->window_size = window_size;
  r->num_recall = num_recall;
  r->total_slots = num_anchors + window_size + num_recall;
  r->clocks.assign((size_t)num_layers * r->total_slots, 0);
  r->active.assign((size_t)num_layers * r->total_slots, 0);
  *out = r;
  return SX_OK;
}
SX_API void sx_ring_destroy(sx_ring *r) { delete r; }
SX_API void sx_ring_reset(sx_ring *r) {
  std::fill(r->clocks.begin(), r->clocks.end(), 0);
  std::fill(r->active.begin(), r->active.end(), 0);
  r->total_ingested = 0;
}
SX_API uint32_t sx_ring_total_slots(const sx_ring *r) { return r->total_slots; }
SX_API uint32_t sx_ring_slot_index(const sx_ring *r, uint64_t clock) {
  if (clock < r->num_anchors) return (uint32_t)clock;
  return r->num_anchors + (uint32_t)((clock - r->num_anchors) % r->window_size);
}
SX_API uint32_t sx_ring_activate_slot(sx_ring *r, uint32_t layer, uint64_t clock) {
  uint32_t slot = sx_ring_slot_index(r, clock);
  size_t gi = (size_t)layer * r->total_slots + slot;
  r->clocks[gi] = clock;
  r->active[gi] = 1;
  if (layer == 0 && clock >= r->total_ingested) r->total_ingested = clock + 1;
  return slot;
}
SX_API void sx_ring_prefill(sx_ring *r, uint32_t layer, uint64_t upto) {
  for (uint64_t c = 0; c < upto && c < r->num_anchors; ++c) sx_ring_activate_slot(r, layer, c);
  uint64_t lo = upto > (uint64_t)r->num_anchors + r->window_size ? upto - r->window_size
                                                                 : (uint64_t)r->num_anchors;
  for (uint64_t c = lo; c < upto; ++c) sx_ring_activate_slot(r, layer, c);
}
SX_API void sx_ring_write_recall(sx_ring *r, uint32_t layer, uint32_t rank, uint64_t clock) {
  if (rank >= r->num_recall) return;
  size_t gi = (size_t)layer * r->total_slots + r->num_anchors + r->window_size + rank;
  r->clocks[gi] = clock;
  r->active[gi] = 1;
}
SX_API void sx_ring_clear_recall(sx_ring *r) {
  uint32_t start = r->num_anchors + r->window_size;
  for (uint32_t l = 0; l < r->num_layers; ++l)
    for (uint32_t s = 0; s < r->num_recall; ++s)
      r->active[(size_t)l * r->total_slots + start + s] = 0;
}
SX_API uint32_t sx_ring_active_slots(const sx_ring *r, uint32_t layer, uint64_t clock,
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

// ---------------------------------------------------------------------------------------
// engine
SX_API sx_status sx_engine_create(int device, sx_quant_mode mode, uint32_t flags,
                                  sx_engine **out) {
  SX_CHECK_ARG(out, "engine: null out");
  SX_CHECK_ARG(mode == SX_QUANT_Q4 || mode == SX_QUANT_Q8 || mode == SX_QUANT_NONE,
               "engine: unknown quant mode %d", (int)mode);
  int n = 0;
  SX_TRY_CUDA(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  SX_CHECK_ARG(device >= 0 && device < n, "engine: device %d out of range (%d devices)", device, n);
  SX_TRY_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  SX_TRY_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10) {
    set_error("engine: libsx is built for sm_100a (B200); device %d is sm_%d%d", device,
              prop.major, prop.minor);
    return SX_ERR_UNSUPPORTED;
  }
  sx_engine *e = new sx_engine();
  e->device = device;
  e->mode = mode;
  e->flags = flags;
  e->kv_bf16 = (flags & SX_ENGINE_KV_F32) == 0;
  e->num_sms = prop.multiProcessorCount;
  sx_status st = SX_OK;
  do {
    st = cuda_status(cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking), "stream");
    if (st) break;
    st = cuda_status(cudaStreamCreateWithFlags(&e->capture_stream, cudaStreamNonBlocking),
                     "capture stream");
    if (st) break;
    e->stream = e->own_stream;
    st = cuda_status(cudaHostAlloc((void **)&e->err_host, sizeof(uint32_t), cudaHostAllocMapped),
                     "error word");
    if (st) break;
    *e->err_host = 0;
    st = cuda_status(cudaHostGetDevicePointer((void **)&e->err_dev, e->err_host, 0),
                     "error word mapping");
    if (st) break;
    {
      // scratch regions, 256-byte aligned
      size_t off = 0;
      auto take = [&](size_t bytes) {
        size_t o = off;
        off = (off + bytes + 255) & ~(size_t)255;
        return o;
      };
      const size_t nw_max = sx::gemv_workers(e->num_sms);
      size_t o_attn = take(e->attn_part_bytes = 8u << 20);
      size_t o_acnt = take(4096 * 4);
      size_t o_gpart = take(sx::gemv_part_bytes(e->num_sms));
      size_t o_tcnt = take((size_t)sx::kMaxGemvTiles * 4);
      size_t o_bv = take(nw_max * 8 * 4);
      size_t o_bi = take(nw_max * 8 * 4);
      size_t o_done = take(256);
      size_t o_amax = take(sx::argmax_scratch_bytes());
      size_t o_pbar = take(256);
      e->scratch_bytes = off;
      st = cuda_status(cudaMalloc(&e->scratch, e->scratch_bytes), "engine scratch");
      if (st) break;
      uint8_t *b = static_cast<uint8_t *>(e->scratch);
      e->attn_part = reinterpret_cast<float *>(b + o_attn);
      e->attn_cnt = reinterpret_cast<uint32_t *>(b + o_acnt);
      e->gemv_part = reinterpret_cast<float *>(b + o_gpart);
      e->tile_cnt = reinterpret_cast<uint32_t *>(b + o_tcnt);
      e->best_v = reinterpret_cast<float *>(b + o_bv);
      e->best_i = reinterpret_cast<uint32_t *>(b + o_bi);
      e->done_cnt = reinterpret_cast<uint32_t *>(b + o_done);
      e->argmax_part = b + o_amax;
      e->persist_bar = reinterpret_cast<uint32_t *>(b + o_pbar);
      st = cuda_status(cudaMemset(e->scratch, 0, e->scratch_bytes), "engine scratch zero");
      if (st) break;
    }
    st = cuda_status(sx::prepare_gemv_kernels(), "gemv kernel attributes");
    if (st) break;
    st = cuda_status(sx::prepare_ops_kernels(), "attention kernel attributes");
    if (st) break;
    st = cuda_status(sx::prepare_attn_block_kernels(), "attention block kernel attributes");
    if (st) break;
    st = cuda_status(sx::prepare_attn_o_kernels(), "attention + o kernel attributes");
    if (st) break;
    st = cuda_status(sx::prepare_persist_kernel(), "persistent kernel attributes");
    if (st) break;
    st = cuda_status(sx::prepare_stream_kernel(), "streaming kernel attributes");
    if (st) break;
    st = cuda_status(sx::prepare_archive_kernels(), "archive kernel attributes");
    if (st) break;
    st = cuda_status(sx::prepare_prefill_kernel(), "prefill kernel attributes");
  } while (0);
  if (st != SX_OK) {
    sx_engine_destroy(e);
    return st;
  }
  *out = e;
  return SX_OK;
}

SX_API void sx_engine_destroy(sx_engine *e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto &kv : e->inv_freq) cudaFree(kv.second);
  if (e->scratch) cudaFree(e->scratch);
  if (e->err_host) cudaFreeHost(e->err_host);
  if (e->capture_stream) cudaStreamDestroy(e->capture_stream);
  if (e->own_stream) cudaStreamDestroy(e->own_stream);
  delete e;
}

SX_API sx_status sx_engine_set_stream(sx_engine *e, void *cuda_stream) {
  SX_CHECK_ARG(e, "engine: null");
  e->stream = cuda_stream ? (cudaStream_t)cuda_stream : e->own_stream;
  return SX_OK;
}
SX_API void *sx_engine_stream(sx_engine *e) { return e ? (void *)e->stream : nullptr; }

SX_API sx_status sx_engine_sync(sx_engine *e) {
  SX_CHECK_ARG(e, "engine: null");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return wait_stream(e, e->stream, 60000000000ull);
}

// ---------------------------------------------------------------------------------------
// buffers
SX_API sx_status sx_buffer_create(sx_engine *e, uint64_t bytes, sx_buffer **out) {
  SX_CHECK_ARG(e && out && bytes > 0, "buffer: bad arguments");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  void *d = nullptr;
  SX_TRY_CUDA(cudaMalloc(&d, bytes), "cudaMalloc");
  cudaError_t ce = cudaMemsetAsync(d, 0, bytes, e->stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
  if (ce != cudaSuccess) {
    cudaFree(d);
    return cuda_status(ce, "buffer zero-fill");
  }
  sx_buffer *b = new sx_buffer();
  b->e = e;
  b->d = d;
  b->bytes = bytes;
  b->owned = true;
  *out = b;
  return SX_OK;
}

SX_API sx_status sx_buffer_wrap(sx_engine *e, void *device_ptr, uint64_t bytes,
                                sx_buffer **out) {
  SX_CHECK_ARG(e && out && device_ptr && bytes > 0, "buffer_wrap: bad arguments");
  sx_buffer *b = new sx_buffer();
  b->e = e;
  b->d = device_ptr;
  b->bytes = bytes;
  b->owned = false;
  *out = b;
  return SX_OK;
}

SX_API void sx_buffer_destroy(sx_buffer *b) {
  if (!b) return;
  if (b->owned && b->d) {
    cudaSetDevice(b->e->device);
    cudaFree(b->d);
  }
  delete b;
}
SX_API void *sx_buffer_device_ptr(sx_buffer *b) { return b ? b->d : nullptr; }
SX_API uint64_t sx_buffer_size(const sx_buffer *b) { return b ? b->bytes : 0; }

SX_API sx_status sx_buffer_write(sx_buffer *b, uint64_t offset, const void *src, uint64_t bytes) {
  SX_CHECK_ARG(b && src && offset + bytes <= b->bytes, "buffer_write: out of range");
  SX_TRY_CUDA(cudaSetDevice(b->e->device), "cudaSetDevice");
  SX_TRY_CUDA(cudaMemcpyAsync((uint8_t *)b->d + offset, src, bytes, cudaMemcpyHostToDevice,
                              b->e->stream),
              "buffer_write");
  SX_TRY_CUDA(cudaStreamSynchronize(b->e->stream), "buffer_write sync");
  return SX_OK;
}

SX_API sx_status sx_buffer_read(sx_buffer *b, uint64_t offset, void *dst, uint64_t bytes) {
  SX_CHECK_ARG(b && dst && offset + bytes <= b->bytes, "buffer_read: out of range");
  SX_TRY_CUDA(cudaSetDevice(b->e->device), "cudaSetDevice");
  SX_TRY_CUDA(cudaMemcpyAsync(dst, (const uint8_t *)b->d + offset, bytes, cudaMemcpyDeviceToHost,
                              b->e->stream),
              "buffer_read");
  SX_TRY_CUDA(cudaStreamSynchronize(b->e->stream), "buffer_read sync");
  return SX_OK;
}

SX_API sx_status sx_buffer_repack_device(sx_buffer *dst, const void *ref_words_device,
                                         uint32_t rows, uint32_t cols, sx_quant_mode mode) {
  SX_CHECK_ARG(dst && ref_words_device, "repack: null argument");
  if (mode == SX_QUANT_NONE) {  // bf16 rows are stored as given
    SX_CHECK_ARG(rows > 0 && cols > 0 && cols % 8 == 0, "repack: bf16 cols must be a multiple of 8");
    SX_CHECK_ARG(sx_packed_bytes(rows, cols, mode) <= dst->bytes, "repack: destination too small");
    SX_TRY_CUDA(cudaSetDevice(dst->e->device), "cudaSetDevice");
    SX_TRY_CUDA(cudaMemcpyAsync(dst->d, ref_words_device, sx_packed_bytes(rows, cols, mode),
                                cudaMemcpyDeviceToDevice, dst->e->stream),
                "bf16 copy");
    return SX_OK;
  }
  SX_CHECK_ARG(mode == SX_QUANT_Q4 || mode == SX_QUANT_Q8, "repack: unknown mode");
  SX_CHECK_ARG(rows > 0 && cols > 0 && cols % 32 == 0, "repack: cols must be a multiple of 32");
  SX_CHECK_ARG(sx_packed_bytes(rows, cols, mode) <= dst->bytes,
               "repack: destination holds %llu B, need %llu", (unsigned long long)dst->bytes,
               (unsigned long long)sx_packed_bytes(rows, cols, mode));
  SX_TRY_CUDA(cudaSetDevice(dst->e->device), "cudaSetDevice");
  SX_TRY_CUDA(sx::launch_repack(qt_of(mode), (const uint32_t *)ref_words_device, dst->d, rows,
                                cols, dst->e->stream),
              "repack launch");
  return SX_OK;
}

SX_API sx_status sx_dispatch_quantize(sx_engine *e, sx_quant_mode mode, const void *bf16_device,
                                     uint32_t *ref_words_device, uint32_t rows, uint32_t cols) {
  SX_CHECK_ARG(e && bf16_device && ref_words_device, "quantize: null argument");
  SX_CHECK_ARG(mode == SX_QUANT_Q4 || mode == SX_QUANT_Q8, "quantize: mode must be Q4 or Q8");
  SX_CHECK_ARG(rows > 0 && cols > 0 && cols % 32 == 0, "quantize: cols must be a multiple of 32");
  SX_CHECK_ARG((uintptr_t)bf16_device % 16 == 0, "quantize: the bf16 matrix must be 16-byte aligned");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  SX_TRY_CUDA(sx::launch_quantize(qt_of(mode), bf16_device, ref_words_device,
                                  (uint64_t)rows * (cols / 32), e->stream),
              "quantize launch");
  return SX_OK;
}

SX_API sx_status sx_buffer_quantize_device(sx_buffer *dst, const void *bf16_device, uint32_t rows,
                                           uint32_t cols, sx_quant_mode mode) {
  SX_CHECK_ARG(dst && bf16_device, "quantize_device: null argument");
  sx_engine *e = dst->e;
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  if (mode == SX_QUANT_NONE) {  // createWeightBuffer in mode none keeps the bf16 values
    sx_status st = sx_buffer_repack_device(dst, bf16_device, rows, cols, mode);
    if (st == SX_OK) st = cuda_status(cudaStreamSynchronize(e->stream), "bf16 copy sync");
    return st;
  }
  SX_CHECK_ARG(mode == SX_QUANT_Q4 || mode == SX_QUANT_Q8, "quantize_device: unknown mode");
  SX_CHECK_ARG(rows > 0 && cols > 0 && cols % 32 == 0,
               "quantize_device: cols must be a multiple of 32");
  SX_CHECK_ARG(sx_packed_bytes(rows, cols, mode) <= dst->bytes,
               "quantize_device: destination holds %llu B, need %llu",
               (unsigned long long)dst->bytes,
               (unsigned long long)sx_packed_bytes(rows, cols, mode));
  const uint64_t bytes = (uint64_t)rows * sx_quantized_row_words(cols, mode) * 4;
  void *tmp = nullptr;
  SX_TRY_CUDA(cudaMalloc(&tmp, bytes), "quantize staging");
  sx_status st = sx_dispatch_quantize(e, mode, bf16_device, (uint32_t *)tmp, rows, cols);
  if (st == SX_OK) st = sx_buffer_repack_device(dst, tmp, rows, cols, mode);
  if (st == SX_OK) st = cuda_status(cudaStreamSynchronize(e->stream), "quantize sync");
  cudaFree(tmp);
  return st;
}

SX_API sx_status sx_buffer_upload_weights(sx_buffer *dst, const uint32_t *ref_words,
                                          uint32_t rows, uint32_t cols, sx_quant_mode mode) {
  SX_CHECK_ARG(dst && ref_words, "upload_weights: null argument");
  SX_CHECK_ARG(mode == SX_QUANT_Q4 || mode == SX_QUANT_Q8 || mode == SX_QUANT_NONE,
               "upload_weights: unknown mode");
  SX_CHECK_ARG(rows > 0 && cols > 0 && cols % (mode == SX_QUANT_NONE ? 8 : 32) == 0,
               "upload_weights: cols must be a multiple of 32 (8 for bf16)");
  sx_engine *e = dst->e;
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  uint64_t bytes = (uint64_t)rows * sx_quantized_row_words(cols, mode) * 4;
  void *tmp = nullptr;
  SX_TRY_CUDA(cudaMalloc(&tmp, bytes), "upload staging");
  sx_status st = cuda_status(cudaMemcpyAsync(tmp, ref_words, bytes, cudaMemcpyHostToDevice,
                                             e->stream),
                             "upload copy");
  if (st == SX_OK) st = sx_buffer_repack_device(dst, tmp, rows, cols, mode);
  if (st == SX_OK) st = cuda_status(cudaStreamSynchronize(e->stream), "upload sync");
  cudaFree(tmp);
  return st;
}

// ---------------------------------------------------------------------------------------
// descriptor sets
SX_API sx_status sx_set_create(sx_engine *e, sx_buffer *const *buffers, uint32_t count,
                               sx_set **out) {
  SX_CHECK_ARG(e && out && (count == 0 || buffers), "set: bad arguments");
  sx_set *s = new sx_set();
  s->b.assign(buffers, buffers + count);
  *out = s;
  return SX_OK;
}
SX_API void sx_set_destroy(sx_set *s) { delete s; }

// ---------------------------------------------------------------------------------------
// command buffers
SX_API sx_status sx_cmd_create(sx_engine *e, sx_cmd **out) {
  SX_CHECK_ARG(e && out, "cmd: bad arguments");
  sx_cmd *c = new sx_cmd();
  c->e = e;
  *out = c;
  return SX_OK;
}

static void cmd_release_graph(sx_cmd *c) {
  if (c->exec) cudaGraphExecDestroy(c->exec);
  if (c->graph) cudaGraphDestroy(c->graph);
  if (c->d_phases) cudaFree(c->d_phases);
  if (c->d_ctr) cudaFree(c->d_ctr);
  c->exec = nullptr;
  c->graph = nullptr;
  c->d_phases = nullptr;
  c->d_ctr = nullptr;
}

// Persistent command buffer: the recorded H2D copies, then the GEMV_FUSED / ATTN_FUSED
// kernels as the phase table of one persistent launch, then the D2H copies.  Phase q (a GEMV)
// issues its first weight copies after phase q - 1, or after q - 2 when q - 1 is attention
// and q's shared-memory layout ends below the attention work items (the o projection).
static sx_status build_persistent(sx_cmd *c) {
  sx_engine *e = c->e;
  const bool stream = c->persistent == kPersistStream;
  std::vector<Op> head, tail;
  std::vector<sx::Phase> ph;
  for (const Op &op : c->ops) {
    if (op.kind == OP_H2D) {
      if (!ph.empty() || !tail.empty()) {
        set_error("persistent graph: host-to-device copies must precede the kernels");
        return SX_ERR_UNSUPPORTED;
      }
      head.push_back(op);
    } else if (op.kind == OP_D2H) {
      tail.push_back(op);
    } else if ((op.kind == OP_GEMV_FUSED || op.kind == OP_ATTN_FUSED) && tail.empty()) {
      sx::Phase p{};
      if (op.kind == OP_GEMV_FUSED) {
        if (!sx::gemv_segments_contiguous(op.gemv, op.qt, op.geglu ? 2 : 1)) {
          set_error("persistent graph: the segments of a multi-segment GEMV must lie back to back");
          return SX_ERR_UNSUPPORTED;
        }
        p.kind = sx::kPhaseGemv;
        p.g = op.gemv;
        if (stream) {
          if (!sx::stream_gemv_variant(op.qt, op.geglu, op.gemv, e->num_sms, &p.variant)) {
            set_error("streaming graph: GEMV k=%u batch=%u has no streaming form", op.gemv.k,
                      op.gemv.batch);
            return SX_ERR_UNSUPPORTED;
          }
          ph.push_back(p);
          continue;
        }
        if (!sx::persist_gemv_variant(op.qt, op.geglu, op.gemv, sx::persist_smem_bytes(),
                                      &p.variant, &p.smem_off)) {
          set_error("persistent graph: GEMV k=%u batch=%u has no persistent instantiation",
                    op.gemv.k, op.gemv.batch);
          return SX_ERR_UNSUPPORTED;
        }
        const uint32_t q = (uint32_t)ph.size();
        bool first = true;
        for (const sx::Phase &x : ph) first = first && x.kind != sx::kPhaseGemv;
        p.prefetch_after = first ? sx::kNoPhase : q - 1;
        if (!first && q >= 2 && ph[q - 1].kind == sx::kPhaseAttn &&
            ph[q - 2].kind == sx::kPhaseGemv && p.smem_off <= ph[q - 1].smem_off)
          p.prefetch_after = q - 2;
      } else {
        p.kind = sx::kPhaseAttn;
        p.at = op.attnf;
        sx_status fst = SX_OK;
        p.at.inv_freq = engine_inv_freq(e, op.attn_rot, op.attn_theta, &fst);
        if (!p.at.inv_freq) return fst;
        if (stream) {
          if (!sx::stream_attn_variant(p.at, &p.variant)) {
            set_error("streaming graph: attention head_dim=%u gqa=%u has no streaming form",
                      p.at.head_dim, p.at.num_q / (p.at.num_kv ? p.at.num_kv : 1));
            return SX_ERR_UNSUPPORTED;
          }
          ph.push_back(p);
          continue;
        }
        if (!sx::persist_attn_variant(p.at, &p.variant)) {
          set_error("persistent graph: attention head_dim=%u gqa=%u has no persistent "
                    "instantiation", p.at.head_dim, p.at.num_q / (p.at.num_kv ? p.at.num_kv : 1));
          return SX_ERR_UNSUPPORTED;
        }
        p.smem_off = sx::persist_attn_offset(p.at);
      }
      ph.push_back(p);
    } else {
      set_error("persistent graph: op %d cannot run as a phase", (int)op.kind);
      return SX_ERR_UNSUPPORTED;
    }
  }
  if (ph.empty()) {
    set_error("persistent graph: no kernels recorded");
    return SX_ERR_UNSUPPORTED;
  }
  const size_t bytes = sizeof(sx::Phase) * ph.size();
  SX_TRY_CUDA(cudaMalloc(&c->d_phases, bytes), "phase table");
  SX_TRY_CUDA(cudaMemcpy(c->d_phases, ph.data(), bytes, cudaMemcpyHostToDevice), "phase table");
  Op run{stream ? OP_STREAM : OP_PERSIST};
  run.u[0] = (uint32_t)ph.size();
  run.dev = c->d_phases;
  if (stream) {
    SX_TRY_CUDA(cudaMalloc(&c->d_ctr, 4 * (ph.size() + 1)), "phase counters");
    run.bind = {c->d_ctr};
  }
  c->ops = head;
  c->ops.push_back(run);
  c->ops.insert(c->ops.end(), tail.begin(), tail.end());
  return SX_OK;
}

SX_API void sx_cmd_destroy(sx_cmd *c) {
  if (!c) return;
  cudaSetDevice(c->e->device);
  cmd_release_graph(c);
  delete c;
}

SX_API sx_status sx_cmd_begin(sx_cmd *c) {
  SX_CHECK_ARG(c, "cmd: null");
  cmd_release_graph(c);
  c->ops.clear();
  c->poisoned = SX_OK;
  c->poison_msg.clear();
  c->recording = true;
  c->kernels = 0;
  c->persistent = kPersistNone;
  return SX_OK;
}

SX_API sx_status sx_cmd_end(sx_cmd *c) {
  SX_CHECK_ARG(c, "cmd: null");
  SX_CHECK_ARG(c->recording, "cmd_end: command buffer is not recording");
  c->recording = false;
  if (c->poisoned != SX_OK) {
    set_error("%s", c->poison_msg.c_str());
    return c->poisoned;
  }
  sx_engine *e = c->e;
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  if (c->persistent) {
    sx_status pst = build_persistent(c);
    if (pst != SX_OK) return pst;
  }
  // device-side tables are created before capture (no allocation inside a capture)
  for (const Op &op : c->ops) {
    sx_status fst = SX_OK;
    if (op.kind == OP_QKV_ROPE && !engine_inv_freq(e, op.u[3], op.f[0], &fst)) return fst;
    if ((op.kind == OP_ATTN_FUSED || op.kind == OP_ATTN_BLOCK || op.kind == OP_ATTN_O) &&
        !engine_inv_freq(e, op.attn_rot, op.attn_theta, &fst))
      return fst;
  }
  cudaStream_t cs = e->capture_stream;
  SX_TRY_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
  sx_status st = SX_OK;
  uint32_t kernels = 0;
  for (const Op &op : c->ops) {
    st = run_op(e, cs, op, &kernels);
    if (st != SX_OK) break;
  }
  cudaGraph_t g = nullptr;
  cudaError_t ce = cudaStreamEndCapture(cs, &g);
  if (st != SX_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  if (ce != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return cuda_status(ce, "end capture");
  }
  cudaGraphExec_t ex = nullptr;
  ce = cudaGraphInstantiate(&ex, g, 0);
  if (ce != cudaSuccess) {
    cudaGraphDestroy(g);
    return cuda_status(ce, "graph instantiate");
  }
  c->graph = g;
  c->exec = ex;
  c->kernels = kernels;
  return SX_OK;
}

extern "C++" void sx_host_push_op(sx_cmd *c, const Op &op) { c->ops.push_back(op); }
static void push_op(sx_cmd *c, Op op, sx_set *set) {
  for (sx_buffer *b : set->b) op.bind.push_back(b ? b->d : nullptr);
  sx_host_push_op(c, op);
}

SX_API void sx_record_gemv(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k) {
  if (!record_guard(e, c, set, 3, "record_gemv")) return;
  Op op{OP_GEMV};
  op.u[0] = m;
  op.u[1] = k;
  push_op(c, op, set);
}
SX_API void sx_record_gemv_logits(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k) {
  if (!record_guard(e, c, set, 3, "record_gemv_logits")) return;
  Op op{OP_GEMV_LOGITS};
  op.u[0] = m;
  op.u[1] = k;
  push_op(c, op, set);
}
SX_API void sx_record_gate_up(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k) {
  if (!record_guard(e, c, set, 4, "record_gate_up")) return;
  Op op{OP_GATE_UP};
  op.u[0] = m;
  op.u[1] = k;
  push_op(c, op, set);
}
SX_API void sx_record_add_rmsnorm(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h, float eps,
                                  float scalar) {
  if (!record_guard(e, c, set, 4, "record_add_rmsnorm")) return;
  Op op{OP_ADD_RMSNORM};
  op.u[0] = h;
  op.f[0] = eps;
  op.f[1] = scalar;
  push_op(c, op, set);
}
SX_API void sx_record_rmsnorm(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h, float eps) {
  if (!record_guard(e, c, set, 3, "record_rmsnorm")) return;
  Op op{OP_RMSNORM};
  op.u[0] = h;
  op.f[0] = eps;
  push_op(c, op, set);
}
SX_API void sx_record_decode_attn(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t head_dim,
                                  uint32_t kv_dim, uint32_t gqa_ratio, float inv_sqrt_dim,
                                  uint32_t num_q_heads, uint32_t total_slots) {
  if (!record_guard(e, c, set, 6, "record_decode_attn")) return;
  Op op{OP_ATTN};
  op.u[0] = head_dim;
  op.u[1] = kv_dim;
  op.u[2] = gqa_ratio;
  op.u[3] = num_q_heads;
  op.u[4] = total_slots;
  op.f[0] = inv_sqrt_dim;
  push_op(c, op, set);
}
SX_API void sx_record_qkv_rope(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t num_q,
                               uint32_t num_kv, uint32_t head_dim, uint32_t rotary_dim,
                               uint32_t k_eq_v, float theta, float eps, uint32_t total_slots) {
  if (!record_guard(e, c, set, 9, "record_qkv_rope")) return;
  Op op{OP_QKV_ROPE};
  op.u[0] = num_q;
  op.u[1] = num_kv;
  op.u[2] = head_dim;
  op.u[3] = rotary_dim;
  op.u[4] = k_eq_v;
  op.u[5] = total_slots;
  op.f[0] = theta;
  op.f[1] = eps;
  push_op(c, op, set);
}
// ---- quiescence gate and indirect records (kernels.zig:84-138, model_dispatch.zig:45-101)
SX_API void sx_record_quiescence_gate(sx_engine *e, sx_cmd *c, sx_set *set,
                                      const sx_quiescence_gate_pc *pc) {
  if (!record_guard(e, c, set, 3, "record_quiescence_gate")) return;
  if (!pc || pc->hidden_size == 0 || pc->num_cmds > 16) {
    poison(c, SX_ERR_INVALID, "record_quiescence_gate: null push constants, hidden_size 0 or "
                              "more than 16 commands");
    return;
  }
  const sx_buffer *xb = set->b[0], *pb = set->b[1], *ib = set->b[2];
  if (xb->bytes < 4ull * pc->hidden_size || pb->bytes < 4ull * pc->hidden_size ||
      ib->bytes < 12ull * ((uint64_t)pc->base_cmd_idx + pc->num_cmds)) {
    poison(c, SX_ERR_INVALID, "record_quiescence_gate: a bound buffer is too small");
    return;
  }
  Op op{OP_QGATE};
  op.qgate.h = pc->hidden_size;
  op.qgate.threshold_sq = pc->threshold_sq;
  op.qgate.base = pc->base_cmd_idx;
  op.qgate.num_cmds = pc->num_cmds;
  for (int i = 0; i < 16; ++i) op.qgate.targets[i] = pc->targets[i];
  push_op(c, op, set);
}

// the dispatch record {x, y, z} at byte `offset` of `ind` (12 bytes, 4-byte aligned)
static const uint32_t *indirect_record(sx_cmd *c, sx_buffer *ind, uint64_t offset,
                                       const char *name) {
  if (!ind || offset % 4 != 0 || offset + 12 > ind->bytes) {
    std::string m = std::string(name) + ": indirect buffer missing, misaligned or too small";
    poison(c, SX_ERR_INVALID, m.c_str());
    return nullptr;
  }
  return reinterpret_cast<const uint32_t *>(static_cast<const uint8_t *>(ind->d) + offset);
}

SX_API void sx_record_gemv_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m, uint32_t k,
                                    sx_buffer *ind, uint64_t offset) {
  if (!record_guard(e, c, set, 3, "record_gemv_indirect")) return;
  const uint32_t *g = indirect_record(c, ind, offset, "record_gemv_indirect");
  if (!g) return;
  Op op{OP_GEMV};
  op.u[0] = m;
  op.u[1] = k;
  op.gate = g;
  push_op(c, op, set);
}
SX_API void sx_record_gate_up_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t m,
                                       uint32_t k, sx_buffer *ind, uint64_t offset) {
  if (!record_guard(e, c, set, 4, "record_gate_up_indirect")) return;
  const uint32_t *g = indirect_record(c, ind, offset, "record_gate_up_indirect");
  if (!g) return;
  Op op{OP_GATE_UP};
  op.u[0] = m;
  op.u[1] = k;
  op.gate = g;
  push_op(c, op, set);
}
SX_API void sx_record_add_rmsnorm_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h,
                                           float eps, float scalar, sx_buffer *ind,
                                           uint64_t offset) {
  if (!record_guard(e, c, set, 4, "record_add_rmsnorm_indirect")) return;
  const uint32_t *g = indirect_record(c, ind, offset, "record_add_rmsnorm_indirect");
  if (!g) return;
  Op op{OP_ADD_RMSNORM};
  op.u[0] = h;
  op.f[0] = eps;
  op.f[1] = scalar;
  op.gate = g;
  push_op(c, op, set);
}
SX_API void sx_record_rmsnorm_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t h,
                                       float eps, sx_buffer *ind, uint64_t offset) {
  if (!record_guard(e, c, set, 3, "record_rmsnorm_indirect")) return;
  const uint32_t *g = indirect_record(c, ind, offset, "record_rmsnorm_indirect");
  if (!g) return;
  Op op{OP_RMSNORM};
  op.u[0] = h;
  op.f[0] = eps;
  op.gate = g;
  push_op(c, op, set);
}
SX_API void sx_record_decode_attn_indirect(sx_engine *e, sx_cmd *c, sx_set *set,
                                           uint32_t head_dim, uint32_t kv_dim, uint32_t gqa_ratio,
                                           float inv_sqrt_dim, uint32_t num_q_heads,
                                           uint32_t total_slots, sx_buffer *ind,
                                           uint64_t offset) {
  if (!record_guard(e, c, set, 6, "record_decode_attn_indirect")) return;
  const uint32_t *g = indirect_record(c, ind, offset, "record_decode_attn_indirect");
  if (!g) return;
  Op op{OP_ATTN};
  op.u[0] = head_dim;
  op.u[1] = kv_dim;
  op.u[2] = gqa_ratio;
  op.u[3] = num_q_heads;
  op.u[4] = total_slots;
  op.f[0] = inv_sqrt_dim;
  op.gate = g;
  push_op(c, op, set);
}
SX_API void sx_record_qkv_rope_indirect(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t num_q,
                                        uint32_t num_kv, uint32_t head_dim, uint32_t rotary_dim,
                                        uint32_t k_eq_v, float theta, float eps,
                                        uint32_t total_slots, sx_buffer *ind, uint64_t offset) {
  if (!record_guard(e, c, set, 9, "record_qkv_rope_indirect")) return;
  const uint32_t *g = indirect_record(c, ind, offset, "record_qkv_rope_indirect");
  if (!g) return;
  Op op{OP_QKV_ROPE};
  op.u[0] = num_q;
  op.u[1] = num_kv;
  op.u[2] = head_dim;
  op.u[3] = rotary_dim;
  op.u[4] = k_eq_v;
  op.u[5] = total_slots;
  op.f[0] = theta;
  op.f[1] = eps;
  op.gate = g;
  push_op(c, op, set);
}

SX_API void sx_record_argmax(sx_engine *e, sx_cmd *c, sx_set *set, uint32_t vocab) {
  if (!record_guard(e, c, set, 2, "record_argmax")) return;
  Op op{OP_ARGMAX};
  op.u[0] = vocab;
  push_op(c, op, set);
}
SX_API void sx_record_barrier(sx_engine *e, sx_cmd *c) {
  // Ops in one command buffer execute in stream order; the barrier is implicit.
  record_guard(e, c, nullptr, 0, "record_barrier");
}

SX_API sx_status sx_submit(sx_engine *e, sx_cmd *c, uint64_t timeout_ns) {
  SX_CHECK_ARG(e && c && c->e == e, "submit: bad arguments");
  SX_CHECK_ARG(c->exec, "submit: command buffer was not ended successfully");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  cudaError_t ce = cudaGraphLaunch(c->exec, e->stream);
  if (ce != cudaSuccess) {
    cuda_status(ce, "graph launch");
    return SX_ERR_LAUNCH;
  }
  return wait_stream(e, e->stream, timeout_ns);
}

// ---------------------------------------------------------------------------------------
// immediate mode
SX_API sx_status sx_dispatch_gemv(sx_engine *e, sx_quant_mode mode, const void *w_packed,
                                  const float *x, float *y, uint32_t m, uint32_t k,
                                  uint32_t batch) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return do_gemv(e, e->stream, qt_of(mode), false, w_packed, nullptr, x, y, m, k, batch);
}
SX_API sx_status sx_dispatch_prefill_gemm(sx_engine *e, const void *w_packed, const void *x_bf16,
                                          float *y, uint32_t t, uint32_t n, uint32_t k) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_CHECK_ARG(w_packed && x_bf16 && y, "prefill_gemm: null pointer");
  SX_CHECK_ARG(t > 0 && n > 0 && n % 4 == 0 && k >= 64 && k % 64 == 0 && t < (1u << 31),
               "prefill_gemm: need t > 0, n a positive multiple of 4 (16-byte rows of y) and k a "
               "positive multiple of 64 (t=%u n=%u k=%u)",
               t, n, k);
  SX_CHECK_ARG(((uintptr_t)w_packed | (uintptr_t)x_bf16 | (uintptr_t)y) % 16 == 0,
               "prefill_gemm: w, x and y must be 16-byte aligned");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return cuda_status(sx::launch_prefill_q4(w_packed, x_bf16, y, t, n, k, n, e->err_dev, e->stream),
                     "prefill gemm launch");
}
SX_API sx_status sx_dispatch_gate_up(sx_engine *e, const void *wg_packed, const void *wu_packed,
                                     const float *x, float *y, uint32_t m, uint32_t k,
                                     uint32_t batch) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return do_gemv(e, e->stream, qt_of(e->mode), true, wg_packed, wu_packed, x, y, m, k, batch);
}
SX_API sx_status sx_dispatch_rmsnorm(sx_engine *e, const float *x, const float *w, float *y,
                                     uint32_t n, uint32_t batch, float eps) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return do_norm(e->stream, false, const_cast<float *>(x), nullptr, w, y, n, batch, eps, 1.0f);
}
SX_API sx_status sx_dispatch_add_rmsnorm(sx_engine *e, float *x, const float *r, const float *w,
                                         float *y, uint32_t n, uint32_t batch, float eps,
                                         float scalar) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return do_norm(e->stream, true, x, r, w, y, n, batch, eps, scalar);
}
SX_API sx_status sx_dispatch_qkv_rope(sx_engine *e, const float *q_in, const float *k_in,
                                      const float *v_in, const float *q_norm_w,
                                      const float *k_norm_w, float *q_out, void *k_cache,
                                      void *v_cache, const uint32_t *step_params,
                                      uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
                                      uint32_t rotary_dim, uint32_t k_eq_v, float theta,
                                      float eps, uint32_t total_slots) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return do_qkv_rope(e, e->stream, q_in, k_in, v_in, q_norm_w, k_norm_w, q_out, k_cache, v_cache,
                     step_params, num_q, num_kv, head_dim, rotary_dim, k_eq_v, theta, eps,
                     total_slots);
}
SX_API sx_status sx_dispatch_decode_attn(sx_engine *e, const float *q, const void *k_cache,
                                         const void *v_cache, const uint32_t *active_slots,
                                         const uint32_t *step_params, float *out,
                                         uint32_t head_dim, uint32_t kv_dim, uint32_t gqa_ratio,
                                         float scale, uint32_t num_q_heads,
                                         uint32_t total_slots) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return do_attn(e, e->stream, q, k_cache, v_cache, active_slots, step_params, out, head_dim,
                 kv_dim, gqa_ratio, scale, num_q_heads, total_slots);
}
SX_API sx_status sx_dispatch_qkv_rope_attn(
    sx_engine *e, const float *q_in, const float *k_in, const float *v_in, const float *q_norm_w,
    const float *k_norm_w, void *k_cache, void *v_cache, const uint32_t *active_slots,
    const uint32_t *step_params, float *out, uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
    uint32_t rotary_dim, uint32_t k_eq_v, float theta, float eps, float scale,
    uint32_t total_slots, uint32_t instances, uint32_t qkv_stride) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_CHECK_ARG(q_in && k_in && v_in && q_norm_w && k_norm_w && k_cache && v_cache &&
                   active_slots && step_params && out,
               "qkv_rope_attn: null pointer");
  SX_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512,
               "qkv_rope_attn: head_dim must be 64/128/256/512 (got %u)", head_dim);
  SX_CHECK_ARG(num_kv > 0 && num_q % num_kv == 0, "qkv_rope_attn: num_q must be a multiple of num_kv");
  const uint32_t g = num_q / num_kv;
  SX_CHECK_ARG(g == 1 || g == 2 || g == 4 || g == 8,
               "qkv_rope_attn: q heads per kv head must be 1/2/4/8 (got %u)", g);
  SX_CHECK_ARG(rotary_dim <= head_dim && rotary_dim % 2 == 0,
               "qkv_rope_attn: rotary_dim must be even and <= head_dim");
  SX_CHECK_ARG(total_slots > 0 && instances >= 1 && num_kv <= 4096,
               "qkv_rope_attn: need total_slots > 0, instances >= 1, num_kv <= 4096");
  SX_CHECK_ARG(instances == 1 || (total_slots <= sx::kAttnClusterMaxSlots &&
                                  qkv_stride >= (num_q + 2 * num_kv) * head_dim &&
                                  qkv_stride % 4 == 0 && instances <= 65535),
               "qkv_rope_attn: several instances need a ring of at most %u slots and a q|k|v "
               "stride of at least (num_q + 2 num_kv) head_dim floats, a multiple of 4",
               sx::kAttnClusterMaxSlots);
  SX_CHECK_ARG(((uintptr_t)q_in | (uintptr_t)k_in | (uintptr_t)v_in | (uintptr_t)q_norm_w |
                (uintptr_t)k_norm_w | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)out) %
                       16 == 0,
               "qkv_rope_attn: vectors and caches must be 16-byte aligned");
  if (total_slots > sx::kAttnClusterMaxSlots &&
      sx::attn_scratch_bytes(num_q, total_slots, head_dim) > e->attn_part_bytes) {
    set_error("qkv_rope_attn: ring of %u slots needs more attention scratch than the engine has",
              total_slots);
    return SX_ERR_UNSUPPORTED;
  }
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  sx_status st = SX_OK;
  sx::AttnFusedArgs a{};
  a.inv_freq = engine_inv_freq(e, rotary_dim, theta, &st);
  if (!a.inv_freq) return st;
  a.q = q_in;
  a.k = k_in;
  a.v = v_in;
  a.q_norm_w = q_norm_w;
  a.k_norm_w = k_norm_w;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.slots = active_slots;
  a.step = step_params;
  a.out = out;
  a.head_dim = head_dim;
  a.kv_dim = num_kv * head_dim;
  a.num_q = num_q;
  a.num_kv = num_kv;
  a.rotary_dim = rotary_dim;
  a.k_eq_v = k_eq_v ? 1u : 0u;
  a.kv_bf16 = e->kv_bf16 ? 1u : 0u;
  a.total_slots = total_slots;
  a.scale = scale;
  a.eps = eps;
  a.sessions = instances;
  a.qkv_ld = qkv_stride;
  a.out_ld = num_q * head_dim;
  a.cache_ld = (uint64_t)total_slots * num_kv * head_dim;
  sx_host_bind_scratch(e, a);
  return cuda_status(sx::launch_attn_fused(a, e->stream, false), "qkv_rope_attn launch");
}
SX_API sx_status sx_dispatch_quiescence_gate(sx_engine *e, const float *x_curr, float *x_prev,
                                             uint32_t *indirect_args,
                                             const sx_quiescence_gate_pc *pc) {
  SX_CHECK_ARG(e && x_curr && x_prev && indirect_args && pc, "quiescence_gate: null argument");
  SX_CHECK_ARG(pc->hidden_size > 0 && pc->num_cmds <= 16,
               "quiescence_gate: hidden_size must be > 0 and num_cmds <= 16");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  sx::GateArgs g{};
  g.x = x_curr;
  g.x_prev = x_prev;
  g.ind = indirect_args;
  g.h = pc->hidden_size;
  g.threshold_sq = pc->threshold_sq;
  g.base = pc->base_cmd_idx;
  g.num_cmds = pc->num_cmds;
  for (int i = 0; i < 16; ++i) g.targets[i] = pc->targets[i];
  return cuda_status(sx::launch_quiescence_gate(g, e->stream), "quiescence gate launch");
}
SX_API sx_status sx_dispatch_argmax(sx_engine *e, const float *logits, uint32_t n,
                                    uint32_t *out_token) {
  SX_CHECK_ARG(e, "dispatch: null engine");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return do_argmax(e, e->stream, logits, n, out_token);
}
SX_API sx_status sx_dispatch_unpack_q4(sx_engine *e, const void *w_packed, float *out,
                                       uint32_t m, uint32_t k) {
  SX_CHECK_ARG(e && w_packed && out && m > 0 && k % 32 == 0, "unpack: bad arguments");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return cuda_status(sx::launch_unpack_q4(w_packed, out, m, k, e->stream), "unpack launch");
}
SX_API sx_status sx_dispatch_synth_weights(sx_engine *e, sx_quant_mode mode, uint32_t *ref_out,
                                           uint32_t row0, uint32_t rows, uint32_t cols,
                                           uint64_t seed, uint64_t stream_id) {
  SX_CHECK_ARG(e && ref_out && rows > 0 && cols % 32 == 0, "synth: bad arguments");
  SX_CHECK_ARG(mode == SX_QUANT_Q4 || mode == SX_QUANT_Q8, "synth: mode must be Q4 or Q8");
  SX_TRY_CUDA(cudaSetDevice(e->device), "cudaSetDevice");
  return cuda_status(
      sx::launch_synth_ref(qt_of(mode), ref_out, row0, rows, cols, seed, stream_id, e->stream),
      "synth launch");
}

}  // extern "C"
