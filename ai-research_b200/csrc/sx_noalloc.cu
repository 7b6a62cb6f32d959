// sx_noalloc.cu -- decode attention for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at decode time: a runtime whose device
// memory is owned by another allocator (a fixed arena handed out at start-up, a memory pool
// that must not grow, a process that is only allowed to map memory before serving begins).
// The engine-based entry points keep their split-K partials in scratch that sx_engine_create
// allocates; this file offers the same attention with that scratch in a fixed-size array in
// the library's own device image instead, so the call allocates nothing.
//
// The scratch array is a file-scope __device__ variable: every GPU that loads libsx holds it
// (1 MiB) until the process exits.  Its host-side name is only a stand-in for the symbol, not
// a device address, so the address is looked up with cudaGetSymbolAddress once per device.
#include <mutex>

#include "../../include/sx.h"
#include "sx_common.cuh"
#include "sx_host.h"
#include "sx_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;  // 1 MiB of attention partials per GPU

static __device__ __align__(256) float g_noalloc_attn_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
float *g_scratch_ptr[kMaxDevices] = {};

// One-time per-device set-up, run with that device current: resolve the scratch symbol's
// device address and set the attention kernels' shared-memory limits.  Neither allocates.
sx_status noalloc_setup(int device, float **out) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_ptr[device]) {
    *out = g_scratch_ptr[device];
    return SX_OK;
  }
  float *ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void **)&ptr, g_noalloc_attn_scratch);
  if (e != cudaSuccess) return sx_host_cuda_status(e, "noalloc: cudaGetSymbolAddress");
  e = sx::prepare_ops_kernels();
  if (e != cudaSuccess) return sx_host_cuda_status(e, "noalloc: attention kernel attributes");
  g_scratch_ptr[device] = ptr;
  *out = ptr;
  return SX_OK;
}

}  // namespace

extern "C" {

SX_API sx_status sx_decode_attn_noalloc(const float *q, const void *k_cache, const void *v_cache,
                                        const uint32_t *active_slots,
                                        const uint32_t *step_params, float *out,
                                        uint32_t head_dim, uint32_t kv_dim, uint32_t gqa_ratio,
                                        float scale, uint32_t num_q_heads, uint32_t total_slots,
                                        uint32_t kv_bf16, void *cuda_stream) {
  if (!q || !k_cache || !v_cache || !active_slots || !step_params || !out) {
    sx_host_set_error("decode_attn_noalloc: null pointer");
    return SX_ERR_INVALID;
  }
  bool shape_ok = (head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512) &&
                  (gqa_ratio == 1 || gqa_ratio == 2 || gqa_ratio == 4 || gqa_ratio == 8) &&
                  num_q_heads > 0 && num_q_heads % gqa_ratio == 0 &&
                  (num_q_heads / gqa_ratio) * head_dim <= kv_dim && kv_dim % 8 == 0 &&
                  total_slots > 0;
  if (!shape_ok) {
    sx_host_set_error("decode_attn_noalloc: unsupported shape (head_dim 64/128/256/512, gqa "
                      "1/2/4/8, kv heads * head_dim <= kv_dim)");
    return SX_ERR_INVALID;
  }
  if (((uintptr_t)k_cache | (uintptr_t)v_cache) % 16 != 0) {
    sx_host_set_error("decode_attn_noalloc: caches must be 16-byte aligned");
    return SX_ERR_INVALID;
  }
  size_t need = sx::attn_scratch_bytes(num_q_heads, total_slots, head_dim);
  if (need > kNoAllocScratchBytes) {
    sx_host_set_error("decode_attn_noalloc: num_q_heads x ceil(total_slots/32) x "
                      "(head_dim+2) x 4 bytes exceeds the fixed 1 MiB scratch");
    return SX_ERR_INVALID;
  }
  int device = 0;
  cudaError_t ce = cudaGetDevice(&device);
  if (ce != cudaSuccess) return sx_host_cuda_status(ce, "decode_attn_noalloc: cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) {
    sx_host_set_error("decode_attn_noalloc: device ordinal out of range");
    return SX_ERR_INVALID;
  }
  float *scratch = nullptr;
  sx_status st = noalloc_setup(device, &scratch);
  if (st != SX_OK) return st;
  sx::AttnArgs a{q, k_cache, v_cache, active_slots, step_params, out, scratch, head_dim, kv_dim,
                 gqa_ratio, num_q_heads, total_slots, kv_bf16 ? 1u : 0u, scale, nullptr};
  return sx_host_cuda_status(sx::launch_decode_attn(a, (cudaStream_t)cuda_stream),
                             "decode_attn_noalloc launch");
}

}  // extern "C"
