// sx_prefill_model.cu -- the per-token kernels of the batched prefill (sx_prefill_batch):
// row norms with the residual update, q/k norm + partial RoPE + KV-cache write, causal
// attention over each token's active-slot list, and the GeGLU product.  The projections run
// on the tcgen05 Q4_0 GEMM (sx_prefill.cu).
//
// The reference prefills a prompt by calling forwardToken once per token
// (src/model/forward.zig:19-75; op order of src/gpu/model_dispatch.zig:10-43).  Here every
// token of every session in the call goes through a layer at once: the K/V of all tokens
// are written before any token attends, and a token attends only over the slots of its own
// ring's active list at its clock (src/ring_buffer.zig:101-136), so the result equals the
// sequential one as long as no token reads a slot that a later token of the call overwrites
// (checked on the host).  Arithmetic follows the decode kernels (rmsnorm / add_rmsnorm /
// qkv_rope / decode_attn semantics); activations entering a GEMM are rounded to bf16.
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr int kPfThreads = 256;

SX_DEV float pf_block_sum(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.0f;
  if (w == 0) {
    s = l < (int)(blockDim.x >> 5) ? red[l] : 0.0f;
    s = warp_sum(s);
    if (l == 0) red[0] = s;
  }
  __syncthreads();
  return red[0];
}

SX_DEV float pf_inv_rms(float ss, uint32_t n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// One row per CTA: (resid) x = (x_in + (post_w ? rmsnorm(mlp) * post_w : mlp)) * scalar, written
// to x_out; then out = rmsnorm(x) * w as bf16 (GEMM input) or f32.  `rows` (optional) maps the
// CTA's output row to its input row (gathering the last token of each session).
constexpr int kPfNormPer = 16;  // elements per thread: n <= 256 * 16
template <bool OUT_BF16>
__global__ void __launch_bounds__(kPfThreads) pf_norm_kernel(PfNormArgs a) {
  __shared__ float red[32];
  const uint32_t r = blockIdx.x, src = a.rows ? a.rows[r] : r;
  const float *x = a.x + (size_t)src * a.n;
  float xv[kPfNormPer];
#pragma unroll
  for (int q = 0; q < kPfNormPer; ++q) {
    const uint32_t i = threadIdx.x + q * kPfThreads;
    xv[q] = i < a.n ? x[i] : 0.0f;
  }
  if (a.mlp) {
    const float *mv = a.mlp + (size_t)src * a.n;
    float m[kPfNormPer];
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < kPfNormPer; ++q) {
      const uint32_t i = threadIdx.x + q * kPfThreads;
      m[q] = i < a.n ? mv[i] : 0.0f;
      ss = fmaf(m[q], m[q], ss);
    }
    float rm = 1.0f;
    if (a.post_w) rm = pf_inv_rms(pf_block_sum(ss, red), a.n, a.eps);
#pragma unroll
    for (int q = 0; q < kPfNormPer; ++q) {
      const uint32_t i = threadIdx.x + q * kPfThreads;
      if (i < a.n) {
        float v = m[q];
        if (a.post_w) v = __fmul_rn(__fmul_rn(v, rm), a.post_w[i]);
        xv[q] = __fmul_rn(__fadd_rn(xv[q], v), a.scalar);
        if (a.x_out) a.x_out[(size_t)src * a.n + i] = xv[q];
      }
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int q = 0; q < kPfNormPer; ++q) ss = fmaf(xv[q], xv[q], ss);
  const float rs = pf_inv_rms(pf_block_sum(ss, red), a.n, a.eps);
#pragma unroll
  for (int q = 0; q < kPfNormPer; ++q) {
    const uint32_t i = threadIdx.x + q * kPfThreads;
    if (i < a.n) {
      const float y = __fmul_rn(__fmul_rn(xv[q], rs), a.w[i]);
      if (OUT_BF16)
        reinterpret_cast<uint16_t *>(a.out)[(size_t)r * a.n + i] = bf16_bits_rne(y);
      else
        reinterpret_cast<float *>(a.out)[(size_t)r * a.n + i] = y;
    }
  }
}

// One token per CTA, one warp per vector (q heads, then per kv head its k and v): RMS norm
// (q / k with their gains, v unit), rotation of the first rotary_dim elements by
// clock * inv_freq, k / v rounded to the cache precision and stored at the token's slot of its
// session's cache; q (f32) goes to q_out for the attention.
template <int DPL, bool BF16>
__global__ void __launch_bounds__(kPfThreads) pf_qkv_rope_kernel(PfQkvArgs a) {
  constexpr uint32_t D = 32 * DPL;
  extern __shared__ float pf_sh[];
  const uint32_t t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sess = a.sess[t], slot = a.slot[t];
  const bool ok = sess < a.sessions && slot < a.total_slots;
  const float fclock = (float)a.clock[t];
  const uint32_t half = a.rotary_dim / 2, nvec = a.num_q + 2 * a.num_kv;
  const float *y = a.y + (size_t)t * a.ldy;
  float *buf = pf_sh + warp * D;
  for (uint32_t vi = warp; vi < nvec; vi += kPfThreads / 32) {
    const bool isq = vi < a.num_q, isk = !isq && (vi - a.num_q) < a.num_kv;
    const uint32_t kvh = isq ? 0 : (isk ? vi - a.num_q : vi - a.num_q - a.num_kv);
    const float *src = isq ? y + (size_t)vi * D
                           : y + a.num_q * D + (size_t)((isk || a.k_eq_v) ? 0 : a.num_kv * D) +
                                 (size_t)kvh * D;
    float x[DPL];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      x[i] = src[lane * DPL + i];
      ss = fmaf(x[i], x[i], ss);
    }
    ss = warp_sum(ss);
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps)));
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const uint32_t d = lane * DPL + i;
      buf[d] = isq ? __fmul_rn(__fmul_rn(x[i], rs), a.q_norm_w[d])
                   : (isk ? __fmul_rn(__fmul_rn(x[i], rs), a.k_norm_w[d]) : __fmul_rn(x[i], rs));
    }
    __syncwarp();
    if (isq || isk) {
      for (uint32_t i = lane; i < half; i += 32) {
        float sn, cs;
        sincosf(__fmul_rn(fclock, a.inv_freq[i]), &sn, &cs);
        const float v0 = buf[i], v1 = buf[i + half];
        buf[i] = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
        buf[i + half] = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
      }
      __syncwarp();
    }
    if (isq) {
      for (uint32_t d = lane; d < D; d += 32) a.q_out[(size_t)t * a.num_q * D + vi * D + d] = buf[d];
    } else if (ok) {
      void *cache = isk ? a.k_cache : a.v_cache;
      const size_t off = ((size_t)sess * a.cache_ld) + ((size_t)slot * a.num_kv + kvh) * D;
      for (uint32_t d = lane; d < D; d += 32) {
        if (BF16)
          reinterpret_cast<uint16_t *>(cache)[off + d] = bf16_bits_rne(buf[d]);
        else
          reinterpret_cast<float *>(cache)[off + d] = buf[d];
      }
    }
    __syncwarp();
  }
  if (!ok && threadIdx.x == 0) raise_error(a.err, kDevBadSlot);
}

// One (token, kv head) per CTA: the G q heads of the kv head attend over the token's active
// slots of its session's cache.  Warp w takes slots w, w + 8, ... in chunks of 4 with an
// online softmax (chunk max, one rescale per chunk); the 8 warps' (m, l, o) merge in shared
// memory; out = O / L rounded to bf16 (the o-projection GEMM input).
constexpr int kPfChunk = 4;
template <int DPL, int G, bool BF16>
__global__ void __launch_bounds__(kPfThreads, 1) pf_attn_kernel(PfAttnArgs a) {
  constexpr uint32_t D = 32 * DPL;
  constexpr int W = kPfThreads / 32;
  extern __shared__ float pf_sh[];
  float *wm = pf_sh, *wl = wm + W * G, *wo = wl + W * G;  // [W][G], [W][G], [W][G][D]
  const uint32_t t = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sess = a.sess[t];
  uint32_t S = a.count[t];
  const bool bad = sess >= a.sessions || S > a.total_slots;
  if (bad) S = 0;
  const uint32_t *list = a.slots + (size_t)t * a.total_slots;
  const size_t cache0 = (size_t)(bad ? 0 : sess) * a.cache_ld;

  float q[G][DPL], o[G][DPL], m[G], l[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float *qs = a.q + ((size_t)t * a.num_q + kvh * G + h) * D + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      q[h][i] = qs[i];
      o[h][i] = 0.0f;
    }
    m[h] = -INFINITY;
    l[h] = 0.0f;
  }
  // the lane's DPL elements of a cached row with the widest aligned loads (rows start on
  // D-element boundaries, so lane * DPL elements is 4 * DPL (f32) or 2 * DPL (bf16) aligned)
  auto load_row = [&](const void *cache, uint32_t sl, float (&out)[DPL]) {
    const size_t idx = cache0 + ((size_t)sl * a.num_kv + kvh) * D + lane * DPL;
    if constexpr (BF16) {
      const uint16_t *p = reinterpret_cast<const uint16_t *>(cache) + idx;
      uint32_t w[DPL / 2];
      if constexpr (DPL == 8) {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
      } else if constexpr (DPL == 4) {
        const uint2 u = *reinterpret_cast<const uint2 *>(p);
        w[0] = u.x; w[1] = u.y;
      } else {
        w[0] = *reinterpret_cast<const uint32_t *>(p);
      }
#pragma unroll
      for (int i = 0; i < DPL / 2; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
    } else {
      const float *p = reinterpret_cast<const float *>(cache) + idx;
#pragma unroll
      for (int i = 0; i < DPL; i += 2) {
        const float2 u = *reinterpret_cast<const float2 *>(p + i);
        out[i] = u.x;
        out[i + 1] = u.y;
      }
    }
  };
  for (uint32_t j0 = warp; j0 < S; j0 += W * kPfChunk) {
    uint32_t sl[kPfChunk];
    bool live[kPfChunk];
#pragma unroll
    for (int p = 0; p < kPfChunk; ++p) {
      const uint32_t j = j0 + p * W;
      sl[p] = j < S ? list[j] : 0xFFFFFFFFu;
      live[p] = sl[p] < a.total_slots;
      if (j < S && !live[p] && lane == 0) raise_error(a.err, kDevBadSlot);
    }
    float kr[kPfChunk][DPL], vr[kPfChunk][DPL];
#pragma unroll
    for (int p = 0; p < kPfChunk; ++p) {
      if (live[p]) {
        load_row(a.k_cache, sl[p], kr[p]);
        load_row(a.v_cache, sl[p], vr[p]);
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) kr[p][i] = vr[p][i] = 0.0f;
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float sc[kPfChunk];
#pragma unroll
      for (int p = 0; p < kPfChunk; ++p) {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) s = fmaf(q[h][i], kr[p][i], s);
        sc[p] = s;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int p = 0; p < kPfChunk; ++p) sc[p] += __shfl_xor_sync(0xffffffffu, sc[p], off);
      float mx = m[h];
#pragma unroll
      for (int p = 0; p < kPfChunk; ++p) {
        sc[p] = live[p] ? sc[p] * a.scale : -INFINITY;
        mx = fmaxf(mx, sc[p]);
      }
      if (mx == -INFINITY) continue;  // nothing live yet for this head
      const float corr = m[h] == -INFINITY ? 0.0f : expf(m[h] - mx);
      float pr[kPfChunk], ps = 0.0f;
#pragma unroll
      for (int p = 0; p < kPfChunk; ++p) {
        pr[p] = live[p] ? expf(sc[p] - mx) : 0.0f;
        ps += pr[p];
      }
      l[h] = fmaf(l[h], corr, ps);
      m[h] = mx;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        float acc = o[h][i] * corr;
#pragma unroll
        for (int p = 0; p < kPfChunk; ++p) acc = fmaf(pr[p], vr[p][i], acc);
        o[h][i] = acc;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (lane == 0) {
      wm[warp * G + h] = m[h];
      wl[warp * G + h] = l[h];
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) wo[(warp * G + h) * D + lane * DPL + i] = o[h][i];
  }
  __syncthreads();
  for (uint32_t idx = threadIdx.x; idx < G * D; idx += kPfThreads) {
    const uint32_t h = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, wm[w * G + h]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float f = wm[w * G + h] == -INFINITY ? 0.0f : expf(wm[w * G + h] - M);
        L = fmaf(wl[w * G + h], f, L);
        O = fmaf(wo[(w * G + h) * D + d], f, O);
      }
    }
    const float out = L > 0.0f ? O / L : 0.0f;
    reinterpret_cast<uint16_t *>(a.out)[((size_t)t * a.num_q + kvh * G + h) * D + d] =
        bf16_bits_rne(out);
  }
}

// h = bf16(gelu_tanh(gate) * up), elementwise over [rows][n] (fused_mlp_q4.wgsl epilogue)
__global__ void pf_geglu_kernel(const float *g, const float *u, uint16_t *h, size_t count) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count;
       i += (size_t)gridDim.x * blockDim.x) {
    const float x = g[i];
    const float x3 = __fmul_rn(__fmul_rn(x, x), x);
    const float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
    const float ge = __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
    h[i] = bf16_bits_rne(__fmul_rn(ge, u[i]));
  }
}

template <int DPL, int G, bool BF16>
cudaError_t launch_attn_t(const PfAttnArgs &a, cudaStream_t s) {
  const size_t smem = sizeof(float) * (2 * 8 * G + 8 * G * 32 * DPL);
  cudaError_t e = cudaFuncSetAttribute(pf_attn_kernel<DPL, G, BF16>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  pf_attn_kernel<DPL, G, BF16><<<dim3(a.tokens, a.num_kv), kPfThreads, smem, s>>>(a);
  return cudaGetLastError();
}

template <int DPL, bool BF16>
cudaError_t launch_attn_g(const PfAttnArgs &a, cudaStream_t s) {
  switch (a.num_q / a.num_kv) {
    case 1: return launch_attn_t<DPL, 1, BF16>(a, s);
    case 2: return launch_attn_t<DPL, 2, BF16>(a, s);
    case 4: return launch_attn_t<DPL, 4, BF16>(a, s);
    case 8: return launch_attn_t<DPL, 8, BF16>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_pf_norm(const PfNormArgs &a, uint32_t rows, bool out_bf16, cudaStream_t s) {
  if (a.n > (uint32_t)(kPfThreads * kPfNormPer) || rows == 0) return cudaErrorInvalidValue;
  if (out_bf16)
    pf_norm_kernel<true><<<rows, kPfThreads, 0, s>>>(a);
  else
    pf_norm_kernel<false><<<rows, kPfThreads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_pf_qkv_rope(const PfQkvArgs &a, uint32_t tokens, cudaStream_t s) {
  const size_t smem = sizeof(float) * (kPfThreads / 32) * a.head_dim;
  switch (a.head_dim) {
#define PF_QKV(DPL)                                                                        \
  case 32 * DPL:                                                                           \
    if (a.kv_bf16)                                                                         \
      pf_qkv_rope_kernel<DPL, true><<<tokens, kPfThreads, smem, s>>>(a);                   \
    else                                                                                   \
      pf_qkv_rope_kernel<DPL, false><<<tokens, kPfThreads, smem, s>>>(a);                  \
    return cudaGetLastError();
    PF_QKV(2)
    PF_QKV(4)
    PF_QKV(8)
#undef PF_QKV
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pf_attn(const PfAttnArgs &a, cudaStream_t s) {
  if (a.num_kv == 0 || a.num_q % a.num_kv) return cudaErrorInvalidValue;
  switch (a.head_dim) {
    case 64: return a.kv_bf16 ? launch_attn_g<2, true>(a, s) : launch_attn_g<2, false>(a, s);
    case 128: return a.kv_bf16 ? launch_attn_g<4, true>(a, s) : launch_attn_g<4, false>(a, s);
    case 256: return a.kv_bf16 ? launch_attn_g<8, true>(a, s) : launch_attn_g<8, false>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pf_geglu(const float *g, const float *u, void *h, size_t count,
                            cudaStream_t s) {
  const uint32_t blocks = (uint32_t)((count + 255) / 256 < 148 * 16 ? (count + 255) / 256 : 148 * 16);
  pf_geglu_kernel<<<blocks ? blocks : 1, 256, 0, s>>>(g, u, static_cast<uint16_t *>(h), count);
  return cudaGetLastError();
}

}  // namespace sx
