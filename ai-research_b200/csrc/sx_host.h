// sx_host.h -- host object definitions shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/sx.h"
#include "sx_internal.h"

// ---------------------------------------------------------------------------------------
// objects
struct sx_engine {
  int device = 0;
  sx_quant_mode mode = SX_QUANT_Q4;
  uint32_t flags = 0;
  bool kv_bf16 = true;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  cudaStream_t capture_stream = nullptr;
  uint32_t *err_host = nullptr;  // mapped pinned word
  uint32_t *err_dev = nullptr;
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  // carved out of `scratch` (counters are zero at rest; kernels that use them reset them)
  float *attn_part = nullptr;
  size_t attn_part_bytes = 0;
  uint32_t *attn_cnt = nullptr;
  float *gemv_part = nullptr;
  uint32_t *tile_cnt = nullptr;
  float *best_v = nullptr;
  uint32_t *best_i = nullptr;
  uint32_t *done_cnt = nullptr;
  void *argmax_part = nullptr;
  uint32_t *persist_bar = nullptr;  // grid-barrier arrival word of the persistent kernel
  int num_sms = 148;
  std::mutex freq_mu;
  std::map<std::pair<uint32_t, uint32_t>, float *> inv_freq;  // (rot, theta bits)
};

struct sx_buffer {
  sx_engine *e = nullptr;
  void *d = nullptr;
  uint64_t bytes = 0;
  bool owned = true;
};

struct sx_set {
  std::vector<sx_buffer *> b;
};

enum OpKind {
  OP_GEMV,
  OP_GEMV_LOGITS,
  OP_GATE_UP,
  OP_ADD_RMSNORM,
  OP_RMSNORM,
  OP_ATTN,
  OP_QKV_ROPE,
  OP_ARGMAX,
  OP_H2D,
  OP_D2H,
  OP_GEMV_FUSED,  // multi-segment GEMV with fused prologue / epilogue (model graph)
  OP_ATTN_FUSED,  // qkv_rope + decode attention + combine (model graph)
  OP_PERSIST,     // the GEMV_FUSED / ATTN_FUSED run of a persistent command buffer
  OP_STREAM,      // the same run as one streaming decode launch (sx_stream.cu)
  OP_QGATE,       // quiescence gate (quiescence_gate.wgsl)
  OP_ALLREDUCE,   // tensor parallel: in-place sum all-reduce of u[0] floats at dev
  OP_ALLGATHER,   // tensor parallel: bind[0] (u[0] u32 words per rank) -> bind[1]
  OP_TP_ARGMAX,   // tensor parallel: merge u[0] ranks' argmax candidates bind[0] -> bind[1]
  OP_ATTN_BLOCK,  // q|k|v GEMV + qkv_rope + attention + o GEMV as one kernel (model graph)
  OP_ATTN_O,      // qkv_rope + attention + per-kv-head o projection (model graph)
};

struct Op {
  OpKind kind;
  // device addresses of the bound buffers, copied from the descriptor set when the op is
  // recorded (the set itself may be destroyed afterwards; the buffers must stay alive)
  std::vector<void *> bind;
  uint32_t u[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float f[4] = {0, 0, 0, 0};
  void *host = nullptr;    // OP_H2D / OP_D2H
  void *dev = nullptr;
  uint64_t bytes = 0;
  // OP_GEMV_FUSED / OP_ATTN_FUSED: complete kernel arguments fixed at record time
  int qt = 4;
  bool geglu = false;
  sx::GemvArgs gemv{};
  sx::AttnFusedArgs attnf{};
  sx::AttnBlockArgs ab{};   // OP_ATTN_BLOCK
  sx::AttnOArgs ao{};       // OP_ATTN_O
  uint32_t attn_rot = 0;
  float attn_theta = 0.0f;
  sx_comm *comm = nullptr;  // OP_ALLREDUCE / OP_ALLGATHER
  // record*Indirect: device address of the op's dispatch record {x, y, z} (null: always runs)
  const uint32_t *gate = nullptr;
  sx::GateArgs qgate{};     // OP_QGATE
};

struct sx_cmd {
  sx_engine *e = nullptr;
  std::vector<Op> ops;
  bool recording = false;
  sx_status poisoned = SX_OK;
  std::string poison_msg;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint32_t kernels = 0;
  // persistent: the fused kernels run as phases of one cooperative launch -- kPersistPhases
  // (sx_persist.cu, grid barriers) or kPersistStream (sx_stream.cu, producer-warp weight ring)
  int persistent = 0;
  sx::Phase *d_phases = nullptr;
  uint32_t *d_ctr = nullptr;  // kPersistStream: per-phase completion counters + abort word
};
constexpr int kPersistNone = 0, kPersistPhases = 1, kPersistStream = 2;


// Append an op (including the internal host<->device copy ops) to a recording command buffer.
void sx_host_push_op(sx_cmd *c, const Op &op);
// record the command buffer's fused kernels as one persistent launch (sx_persist.cu)
inline void sx_host_set_persistent(sx_cmd *c, int kind) { c->persistent = kind; }
void sx_host_set_error(const char *fmt, ...);  // printf-style
// tensor parallel (sx_tp.cu): collectives and the argmax-candidate merge on stream s
sx_status sx_host_allreduce(sx_comm *c, float *buf, size_t count, cudaStream_t s);
sx_status sx_host_allgather(sx_comm *c, const uint32_t *src, uint32_t *dst, size_t words,
                            cudaStream_t s);
sx_status sx_host_tp_argmax(const uint32_t *cand, uint32_t n, uint32_t *token, cudaStream_t s);
uint32_t sx_host_comm_ranks(const sx_comm *c);
uint32_t sx_host_comm_rank(const sx_comm *c);
// Shape / shared-memory validation of a GEMV launch (sets the error message).
sx_status sx_host_check_gemv(int qt, bool geglu, bool pro, uint32_t m, uint32_t k,
                             uint32_t batch);
// Fill the scratch / error-word fields of GEMV and fused-attention arguments.
void sx_host_bind_scratch(sx_engine *e, sx::GemvArgs &a);
void sx_host_bind_scratch(sx_engine *e, sx::AttnFusedArgs &a);
// Device RoPE inverse-frequency table for (rotary_dim, theta); created on first use, never
// inside a stream capture.
float *sx_host_inv_freq(sx_engine *e, uint32_t rot, float theta, sx_status *st);
sx_status sx_host_cuda_status(cudaError_t e, const char *what);
