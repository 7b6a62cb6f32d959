// sx_host.h -- host object definitions shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/sx.h"

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
};


// Append an op (including the internal host<->device copy ops) to a recording command buffer.
void sx_host_push_op(sx_cmd *c, const Op &op);
void sx_host_set_error(const char *msg);
sx_status sx_host_cuda_status(cudaError_t e, const char *what);
