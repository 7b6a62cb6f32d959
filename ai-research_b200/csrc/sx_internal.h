// sx_internal.h -- launchers shared between the kernel files and the host engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sx {

struct GemvArgs {
  const void *w0;      // packed matrix (gate matrix for the fused GeGLU)
  const void *w1;      // packed up matrix (fused GeGLU only)
  const float *x;      // [batch][ldx]
  float *y;            // [batch][ldy]
  uint32_t m, k, batch;
  uint32_t ldx, ldy;
};

// Per-device kernel attributes (dynamic shared memory limits); called at engine creation,
// never inside a stream capture.
cudaError_t prepare_gemv_kernels();
cudaError_t prepare_ops_kernels();

// qt: 4 or 8.  geglu: fused gate+up with gelu_tanh(gate) * up epilogue.
cudaError_t launch_gemv(int qt, bool geglu, const GemvArgs &a, int num_sms, cudaStream_t s);
size_t gemv_smem_bytes(int qt, uint32_t k, uint32_t batch);

cudaError_t launch_repack(int qt, const uint32_t *ref, void *packed, uint32_t m, uint32_t k,
                          cudaStream_t s);
cudaError_t launch_unpack_q4(const void *packed, float *out, uint32_t m, uint32_t k,
                             cudaStream_t s);
cudaError_t launch_synth_ref(int qt, uint32_t *ref, uint32_t row0, uint32_t rows, uint32_t k,
                             uint64_t seed, uint64_t stream_id, cudaStream_t s);
cudaError_t launch_synth_gain(float *dst, uint32_t n, uint64_t seed, uint64_t stream_id,
                              cudaStream_t s);
cudaError_t launch_fill_kv(void *k_cache, void *v_cache, int kv_bf16, uint32_t rows,
                           uint32_t head_dim, float eps, uint64_t seed, uint32_t layer,
                           cudaStream_t s);

struct NormArgs {
  float *x;           // residual stream (add variant: updated in place)
  const float *r;     // added vector (add variant)
  const float *w;     // gain
  float *y;           // output
  uint32_t n, batch, ld;
  float eps, scalar;
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
};
cudaError_t launch_qkv_rope(const QkvRopeArgs &a, cudaStream_t s);

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
};
size_t attn_scratch_bytes(uint32_t num_q, uint32_t total_slots, uint32_t head_dim);
cudaError_t launch_decode_attn(const AttnArgs &a, cudaStream_t s);

cudaError_t launch_argmax(const float *logits, uint32_t n, uint32_t *out, void *scratch,
                          size_t scratch_bytes, cudaStream_t s);
size_t argmax_scratch_bytes();

}  // namespace sx
