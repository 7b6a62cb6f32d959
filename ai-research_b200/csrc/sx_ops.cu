// sx_ops.cu -- RMSNorm / add+RMSNorm, QKV norm + partial RoPE + cache write, GQA decode
// attention over the ring's active-slot list, and the vocabulary argmax (sm_100a).
#include "sx_attn_dev.cuh"
#include "sx_common.cuh"
#include "sx_internal.h"

#include <utility>

namespace sx {

namespace {

// Launch with programmatic stream serialization: every kernel here calls
// griddepcontrol.wait before it touches data written by the previous kernel.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// rmsnorm.wgsl:352-387 and add_rmsnorm.wgsl:303-338.
//   plain: Y = X * (1 / sqrt(mean(X^2) + eps)) * W          (kernels.zig:46-52)
//   add:   X = (X + R) * scalar (written back); Y = X * rsqrt(...) * W
// One CTA per batch row; the per-element products keep the CPU's (x * r) * w order.
template <bool ADD>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(NormArgs a) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  if (gate_closed(a.gate)) return;
  float *x = a.x + (size_t)blockIdx.x * a.ld;
  const float *r = ADD ? a.r + (size_t)blockIdx.x * a.ld : nullptr;
  float *y = a.y + (size_t)blockIdx.x * a.ld;
  float ss = 0.0f;
  for (uint32_t i = threadIdx.x; i < a.n; i += blockDim.x) {
    float v = x[i];
    if (ADD) {
      v = __fmul_rn(__fadd_rn(v, r[i]), a.scalar);
      x[i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.n), a.eps)));
  for (uint32_t i = threadIdx.x; i < a.n; i += blockDim.x)
    y[i] = __fmul_rn(__fmul_rn(x[i], rs), a.w[i]);
}

// ---------------------------------------------------------------------------
// qkv_rope.wgsl:133-288 (semantics of forward.zig:127-142).  CTA h < num_q: q head h is
// RMS-normalised with q_norm_w and rotated in place; CTA num_q + kh: k head kh is normalised
// with k_norm_w, rotated and stored at K_cache[slot], v (k when k_eq_v) is unit-normalised
// and stored at V_cache[slot].  Cache layout [slot][kv_head][head_dim] (model_gpu.zig:133),
// element type bf16 (build default) or f32 (reference).  inv_freq is the host-computed
// table 1/pow(theta, 2i/rot) (kernels.zig:138) so CPU and GPU angles agree bit for bit.
__global__ void __launch_bounds__(128) qkv_rope_kernel(QkvRopeArgs a) {
  extern __shared__ float sh[];  // head_dim floats + 32 reduction slots
  pdl_launch_dependents();
  pdl_wait();
  if (gate_closed(a.gate)) return;
  float *vec = sh;
  float *red = sh + a.head_dim;
  const uint32_t D = a.head_dim, half = a.rotary_dim / 2;
  const uint32_t clock = a.step[0], slot = a.step[1];
  const uint32_t h = blockIdx.x;
  const bool is_q = h < a.num_q;
  if (!is_q && h - a.num_q >= a.num_kv) return;
  if (!is_q && slot >= a.total_slots) {
    if (threadIdx.x == 0) raise_error(a.err, kDevBadSlot);
    return;
  }
  const float *src = is_q ? a.q_in + (size_t)h * D : a.k_in + (size_t)(h - a.num_q) * D;
  const float *nw = is_q ? a.q_norm_w : a.k_norm_w;

  float ss = 0.0f;
  for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
    float v = src[d];
    vec[d] = v;
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps)));
  __syncthreads();
  for (uint32_t d = threadIdx.x; d < D; d += blockDim.x)
    vec[d] = __fmul_rn(__fmul_rn(vec[d], rs), nw[d]);
  __syncthreads();

  float *qdst = a.q_out + (size_t)h * D;
  const uint32_t kh = h - a.num_q;
  const size_t cache_off = ((size_t)slot * a.num_kv + kh) * D;
  auto store = [&](uint32_t d, float v) {
    if (is_q) {
      qdst[d] = v;
    } else if (a.kv_bf16) {
      reinterpret_cast<uint16_t *>(a.k_cache)[cache_off + d] = bf16_bits_rne(v);
    } else {
      reinterpret_cast<float *>(a.k_cache)[cache_off + d] = v;
    }
  };
  const float fclock = (float)clock;
  for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
    float ang = __fmul_rn(fclock, a.inv_freq[i]);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    float v0 = vec[i], v1 = vec[i + half];
    store(i, __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn)));
    store(i + half, __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs)));
  }
  for (uint32_t d = a.rotary_dim + threadIdx.x; d < D; d += blockDim.x) store(d, vec[d]);
  if (is_q) return;

  // v_norm: unit RMSNorm without weight (kernels.zig:55-61)
  const float *vsrc = (a.k_eq_v ? a.k_in : a.v_in) + (size_t)kh * D;
  ss = 0.0f;
  for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
    float v = vsrc[d];
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps)));
  for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
    float v = __fmul_rn(vsrc[d], rs);
    if (a.kv_bf16)
      reinterpret_cast<uint16_t *>(a.v_cache)[cache_off + d] = bf16_bits_rne(v);
    else
      reinterpret_cast<float *>(a.v_cache)[cache_off + d] = v;
  }
}

// ---------------------------------------------------------------------------
// decode_attn.wgsl:19-108 / forward.zig:77-104: for q head h (kv head h / gqa):
//   s_i = (q . K[slot_i]) * scale, p = softmax(s), out = sum_i p_i V[slot_i]
// over the host-built active-slot list.  Split over slots (flash-decoding): CTA (kv head,
// chunk) runs an online softmax for the whole GQA group of q heads over 32 slots and writes
// an unnormalised partial (m, l, o[D]) to scratch; a combine kernel merges the chunks.
constexpr int kAttnWarps = 4;

// Lane `lane` owns elements [lane*DPL, lane*DPL + DPL) of a head row; the load width matches
// DPL so every access is naturally aligned (DPL*2 or DPL*4 bytes per lane).
template <int DPL, bool BF16>
SX_DEV void load_row(const void *cache, size_t off, int lane, float (&v)[DPL]) {
  if (BF16) {
    const uint16_t *p = reinterpret_cast<const uint16_t *>(cache) + off + (size_t)lane * DPL;
    if constexpr (DPL % 8 == 0) {
#pragma unroll
      for (int i = 0; i < DPL; i += 8) {
        uint4 u = *reinterpret_cast<const uint4 *>(p + i);
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          v[i + 2 * k] = u2f(w[k] << 16);
          v[i + 2 * k + 1] = u2f(w[k] & 0xFFFF0000u);
        }
      }
    } else if constexpr (DPL == 4) {
      uint2 u = *reinterpret_cast<const uint2 *>(p);
      v[0] = u2f(u.x << 16); v[1] = u2f(u.x & 0xFFFF0000u);
      v[2] = u2f(u.y << 16); v[3] = u2f(u.y & 0xFFFF0000u);
    } else {
      static_assert(DPL == 2, "head_dim must be 64, 128, 256 or 512");
      uint32_t u = *reinterpret_cast<const uint32_t *>(p);
      v[0] = u2f(u << 16); v[1] = u2f(u & 0xFFFF0000u);
    }
  } else {
    const float *p = reinterpret_cast<const float *>(cache) + off + (size_t)lane * DPL;
    if constexpr (DPL % 4 == 0) {
#pragma unroll
      for (int i = 0; i < DPL; i += 4) {
        float4 u = *reinterpret_cast<const float4 *>(p + i);
        v[i] = u.x; v[i + 1] = u.y; v[i + 2] = u.z; v[i + 3] = u.w;
      }
    } else {
      static_assert(DPL == 2, "head_dim must be 64, 128, 256 or 512");
      float2 u = *reinterpret_cast<const float2 *>(p);
      v[0] = u.x; v[1] = u.y;
    }
  }
}

template <int DPL, int G, bool BF16>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(AttnArgs a) {
  extern __shared__ float sh[];
  pdl_launch_dependents();
  pdl_wait();
  if (gate_closed(a.gate)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t D = a.head_dim;  // == 32 * DPL
  const uint32_t kvh = blockIdx.x, chunk = blockIdx.y, nchunks = gridDim.y;
  uint32_t S = a.step[2];
  if (S > a.total_slots) {
    if (threadIdx.x == 0 && chunk == 0) raise_error(a.err, kDevBadParams);
    S = a.total_slots;
  }
  const uint32_t s0 = chunk * kAttnChunk;
  const uint32_t s1 = min(S, s0 + kAttnChunk);

  float *qs = sh;                          // [G][D]
  float *wm = qs + G * D;                  // [warps][G] running max
  float *wl = wm + kAttnWarps * G;         // [warps][G] running sum
  float *wo = wl + kAttnWarps * G;         // [warps][G][D]
  for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x)
    qs[i] = a.q[(size_t)(kvh * G) * D + i];
  __syncthreads();

  float m[G], l[G], o[G][DPL], qr[G][DPL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      o[h][i] = 0.0f;
      qr[h][i] = qs[h * D + lane * DPL + i];
    }
  }
  for (uint32_t si = s0 + warp; si < s1; si += kAttnWarps) {
    uint32_t slot = a.slots[si];
    if (slot >= a.total_slots) {
      if (lane == 0) raise_error(a.err, kDevBadSlot);
      continue;
    }
    size_t off = (size_t)slot * a.kv_dim + (size_t)kvh * D;
    float kr[DPL], vr[DPL];
    load_row<DPL, BF16>(a.k_cache, off, lane, kr);
    load_row<DPL, BF16>(a.v_cache, off, lane, vr);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float part = 0.0f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) part = fmaf(qr[h][i], kr[i], part);
      float sc = warp_sum(part) * a.scale;
      float mn = fmaxf(m[h], sc);
      float corr = expf(m[h] - mn);
      float p = expf(sc - mn);
      l[h] = fmaf(l[h], corr, p);
#pragma unroll
      for (int i = 0; i < DPL; ++i) o[h][i] = fmaf(o[h][i], corr, p * vr[i]);
      m[h] = mn;
    }
  }
  // merge the warps of this CTA
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
  for (uint32_t idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    uint32_t h = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w * G + h]);
    float Lsum = 0.0f, O = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w) {
      float f = M == -INFINITY ? 0.0f : expf(wm[w * G + h] - M);
      Lsum = fmaf(wl[w * G + h], f, Lsum);
      O = fmaf(wo[(w * G + h) * D + d], f, O);
    }
    uint32_t qh = kvh * G + h;
    float *rec = a.part + ((size_t)qh * nchunks + chunk) * (D + 2);
    rec[2 + d] = O;
    if (d == 0) {
      rec[0] = M;
      rec[1] = Lsum;
    }
  }
}

__global__ void attn_combine_kernel(AttnArgs a, uint32_t nchunks) {
  pdl_launch_dependents();
  pdl_wait();
  if (gate_closed(a.gate)) return;
  const uint32_t qh = blockIdx.x, D = a.head_dim;
  const float *base = a.part + (size_t)qh * nchunks * (D + 2);
  float M = -INFINITY;
  for (uint32_t c = 0; c < nchunks; ++c) M = fmaxf(M, base[(size_t)c * (D + 2)]);
  for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (uint32_t c = 0; c < nchunks; ++c) {
        const float *rec = base + (size_t)c * (D + 2);
        float f = expf(rec[0] - M);
        L = fmaf(rec[1], f, L);
        O = fmaf(rec[2 + d], f, O);
      }
    }
    a.out[(size_t)qh * D + d] = L > 0.0f ? O / L : 0.0f;
  }
}

// ---------------------------------------------------------------------------
// Fused decode attention as a kernel of its own: CTA (kv head, chunk) runs one work item
// (sx_attn_dev.cuh); the dependency wait is griddepcontrol.wait.
template <int DPL, int G, bool BF16>
__global__ void __launch_bounds__(kFusedWarps * 32) attn_fused_kernel(AttnFusedArgs a) {
  extern __shared__ float sh[];
  __shared__ uint32_t last_flag;
  pdl_launch_dependents();
  attn_item<DPL, G, BF16>(a, blockIdx.x, blockIdx.y, gridDim.y, sh, &last_flag,
                          (int)threadIdx.x, 0, true, [] { pdl_wait(); });
}

// Cluster form (rings of up to 16 x 64 slots): one cluster of CL CTAs per kv head.
template <int DPL, int G, bool BF16>
__global__ void __launch_bounds__(kFusedWarps * 32) attn_cluster_kernel(AttnFusedArgs a) {
  extern __shared__ float sh[];
  pdl_launch_dependents();
  // this CTA's session (grid z): the same item over that session's vectors, caches and ring
  AttnFusedArgs s = a;
  const uint32_t z = blockIdx.z;
  const size_t eb = a.kv_bf16 ? 2 : 4;
  s.q += (size_t)z * a.qkv_ld;
  s.k += (size_t)z * a.qkv_ld;
  s.v += (size_t)z * a.qkv_ld;
  s.k_cache = static_cast<uint8_t *>(a.k_cache) + z * a.cache_ld * eb;
  s.v_cache = static_cast<uint8_t *>(a.v_cache) + z * a.cache_ld * eb;
  s.slots += (size_t)z * a.total_slots;
  s.step += 4 * z;
  s.out += (size_t)z * a.out_ld;
  if constexpr (DPL == 8 && G == 8 && BF16)
    attn_cluster_item_tc(s, blockIdx.x, sh, [] { pdl_wait(); });  // tensor-core form
  else
    attn_cluster_item<DPL, G, BF16>(s, blockIdx.x, sh, [] { pdl_wait(); });
}

static_assert(kClusterSlots * kClusterMax == (int)kAttnClusterMaxSlots, "cluster ring limit");

template <int DPL, int G>
cudaError_t launch_attn_fused_t(const AttnFusedArgs &a, cudaStream_t s, bool pdl) {
  const uint32_t ncl = (a.total_slots + kClusterSlots - 1) / kClusterSlots;
  if (ncl <= (uint32_t)kClusterMax) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.num_kv, ncl, a.sessions > 1 ? a.sessions : 1);
    cfg.blockDim = dim3(kFusedWarps * 32);
    cfg.dynamicSmemBytes = (DPL == 8 && G == 8 && a.kv_bf16)
                               ? (size_t)TcaLayout::total
                               : sizeof(float) * attn_cluster_floats(G, 32 * DPL, ncl);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = ncl;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    if (a.kv_bf16) return cudaLaunchKernelEx(&cfg, attn_cluster_kernel<DPL, G, true>, a);
    return cudaLaunchKernelEx(&cfg, attn_cluster_kernel<DPL, G, false>, a);
  }
  if (a.sessions > 1) return cudaErrorInvalidValue;  // sessions: cluster form only
  uint32_t nchunks = (a.total_slots + kAttnChunk - 1) / kAttnChunk;
  size_t D = 32 * DPL;
  size_t smem = sizeof(float) * attn_item_floats(G, D, nchunks);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_kv, nchunks);
  cfg.blockDim = dim3(kFusedWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (a.kv_bf16) return cudaLaunchKernelEx(&cfg, attn_fused_kernel<DPL, G, true>, a);
  return cudaLaunchKernelEx(&cfg, attn_fused_kernel<DPL, G, false>, a);
}

template <int DPL>
cudaError_t launch_attn_fused_d(const AttnFusedArgs &a, cudaStream_t s, bool pdl) {
  switch (a.num_q / a.num_kv) {
    case 1: return launch_attn_fused_t<DPL, 1>(a, s, pdl);
    case 2: return launch_attn_fused_t<DPL, 2>(a, s, pdl);
    case 4: return launch_attn_fused_t<DPL, 4>(a, s, pdl);
    case 8: return launch_attn_fused_t<DPL, 8>(a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int DPL, int G>
cudaError_t prepare_attn_fused_t() {
  for (auto k : {attn_cluster_kernel<DPL, G, true>, attn_cluster_kernel<DPL, G, false>}) {
    cudaError_t e = allow_max_dynamic_smem(k);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  cudaError_t a = allow_max_dynamic_smem(attn_fused_kernel<DPL, G, true>);
  cudaError_t b = allow_max_dynamic_smem(attn_fused_kernel<DPL, G, false>);
  return a != cudaSuccess ? a : b;
}

template <int DPL, int G>
cudaError_t launch_attn_t(const AttnArgs &a, cudaStream_t s) {
  uint32_t num_kv = a.num_q / G;
  uint32_t nchunks = (a.total_slots + kAttnChunk - 1) / kAttnChunk;
  size_t smem = sizeof(float) * (G * a.head_dim + 2 * kAttnWarps * G +
                                 (size_t)kAttnWarps * G * a.head_dim);
  auto kern = a.kv_bf16 ? attn_split_kernel<DPL, G, true> : attn_split_kernel<DPL, G, false>;
  cudaError_t e = launch_pdl(kern, dim3(num_kv, nchunks), dim3(kAttnWarps * 32), smem, s, a);
  if (e != cudaSuccess) return e;
  return launch_pdl(attn_combine_kernel, dim3(a.num_q), dim3(256), 0, s, a, nchunks);
}

template <int DPL, int G>
cudaError_t prepare_attn_t() {
  cudaError_t a = allow_max_dynamic_smem(attn_split_kernel<DPL, G, true>);
  cudaError_t b = allow_max_dynamic_smem(attn_split_kernel<DPL, G, false>);
  return a != cudaSuccess ? a : b;
}

template <int DPL>
cudaError_t prepare_attn_d() {
  cudaError_t r[8] = {prepare_attn_t<DPL, 1>(),       prepare_attn_t<DPL, 2>(),
                      prepare_attn_t<DPL, 4>(),       prepare_attn_t<DPL, 8>(),
                      prepare_attn_fused_t<DPL, 1>(), prepare_attn_fused_t<DPL, 2>(),
                      prepare_attn_fused_t<DPL, 4>(), prepare_attn_fused_t<DPL, 8>()};
  for (cudaError_t x : r)
    if (x != cudaSuccess) return x;
  return cudaSuccess;
}

template <int DPL>
cudaError_t launch_attn_d(const AttnArgs &a, cudaStream_t s) {
  switch (a.gqa) {
    case 1: return launch_attn_t<DPL, 1>(a, s);
    case 2: return launch_attn_t<DPL, 2>(a, s);
    case 4: return launch_attn_t<DPL, 4>(a, s);
    case 8: return launch_attn_t<DPL, 8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// argmax.wgsl:399-435 with the CPU tie rule of kernels.zig:164-174 (first index of the
// maximum): partial (value, index) per CTA, then one CTA merges.  NaNs never win a strict
// comparison, as on the CPU.
constexpr int kArgmaxBlocks = 296;
constexpr int kArgmaxThreads = 512;

SX_DEV bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_partial_kernel(const float *x,
                                                                         uint32_t n,
                                                                         float2 *part) {
  __shared__ float sv[kArgmaxThreads];
  pdl_launch_dependents();
  pdl_wait();
  __shared__ uint32_t si[kArgmaxThreads];
  uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x, stride = gridDim.x * blockDim.x;
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  if (i0 < n) {
    float v = x[i0];
    bv = isnan(v) ? -INFINITY : v;
    bi = i0;
  }
  for (uint32_t i = i0 + stride; i < n; i += stride) {
    float v = x[i];
    if (v > bv) {
      bv = v;
      bi = i;
    }
  }
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      float v = sv[threadIdx.x + s];
      uint32_t i = si[threadIdx.x + s];
      if (i != 0xFFFFFFFFu &&
          (si[threadIdx.x] == 0xFFFFFFFFu || better(v, i, sv[threadIdx.x], si[threadIdx.x]))) {
        sv[threadIdx.x] = v;
        si[threadIdx.x] = i;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = make_float2(sv[0], __uint_as_float(si[0]));
}

__global__ void argmax_final_kernel(const float *x, const float2 *part, uint32_t nparts,
                                    uint32_t *out) {
  __shared__ float sv[kArgmaxThreads];
  pdl_launch_dependents();
  pdl_wait();
  __shared__ uint32_t si[kArgmaxThreads];
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t p = threadIdx.x; p < nparts; p += blockDim.x) {
    float v = part[p].x;
    uint32_t i = __float_as_uint(part[p].y);
    if (i != 0xFFFFFFFFu && (bi == 0xFFFFFFFFu || better(v, i, bv, bi))) {
      bv = v;
      bi = i;
    }
  }
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      float v = sv[threadIdx.x + s];
      uint32_t i = si[threadIdx.x + s];
      if (i != 0xFFFFFFFFu &&
          (si[threadIdx.x] == 0xFFFFFFFFu || better(v, i, sv[threadIdx.x], si[threadIdx.x]))) {
        sv[threadIdx.x] = v;
        si[threadIdx.x] = i;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    uint32_t r = si[0] == 0xFFFFFFFFu ? 0u : si[0];
    // CPU: max starts at logits[0]; a NaN there is never beaten -> index 0.
    if (isnan(x[0])) r = 0;
    // CPU: nothing beats the first value when every later value is <= it.
    *out = r;
  }
}

}  // namespace

cudaError_t prepare_ops_kernels() {
  cudaError_t r[4] = {prepare_attn_d<2>(), prepare_attn_d<4>(), prepare_attn_d<8>(),
                      prepare_attn_d<16>()};
  for (cudaError_t x : r)
    if (x != cudaSuccess) return x;
  return cudaSuccess;
}

// quiescence_gate.wgsl:1-62, one 32-thread CTA with the shader's order of operations: lane l
// accumulates (x[i] - x_prev[i])^2 for i = l, l + 32, ... (no fused multiply-add, like the
// CPU restatement) and copies x into x_prev, the partials fold 16, 8, 4, 2, lane 0 adds the
// last two, divides by h and writes the dispatch records.
__global__ void __launch_bounds__(32) quiescence_gate_kernel(GateArgs a) {
  __shared__ float s[32];
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t lane = threadIdx.x;
  float acc = 0.0f;
  for (uint32_t i = lane; i < a.h; i += 32) {
    const float c = a.x[i];
    const float d = __fsub_rn(c, a.x_prev[i]);
    acc = __fadd_rn(acc, __fmul_rn(d, d));
    a.x_prev[i] = c;
  }
  s[lane] = acc;
  __syncwarp();
  for (uint32_t w = 16; w >= 2; w >>= 1) {
    if (lane < w) s[lane] = __fadd_rn(s[lane], s[lane + w]);
    __syncwarp();
  }
  if (lane == 0) {
    const float mean_sq = __fdiv_rn(__fadd_rn(s[0], s[1]), (float)a.h);
    const bool active = (mean_sq >= a.threshold_sq) || (a.threshold_sq <= 0.0f);
    for (uint32_t c = 0; c < a.num_cmds && c < 16; ++c) {
      uint32_t *rec = a.ind + 3ull * (a.base + c);
      rec[0] = active ? a.targets[c] : 0u;
      rec[1] = active ? 1u : 0u;
      rec[2] = active ? 1u : 0u;
    }
  }
}

cudaError_t launch_quiescence_gate(const GateArgs &a, cudaStream_t s) {
  return launch_pdl(quiescence_gate_kernel, dim3(1), dim3(32), 0, s, a);
}

cudaError_t launch_rmsnorm(bool add, const NormArgs &a, cudaStream_t s) {
  uint32_t threads = a.n >= 1024 ? 1024 : ((a.n + 31) / 32) * 32;
  if (threads == 0) threads = 32;
  if (add) return launch_pdl(rmsnorm_kernel<true>, dim3(a.batch), dim3(threads), 0, s, a);
  return launch_pdl(rmsnorm_kernel<false>, dim3(a.batch), dim3(threads), 0, s, a);
}

cudaError_t launch_qkv_rope(const QkvRopeArgs &a, cudaStream_t s) {
  size_t smem = sizeof(float) * (a.head_dim + 32);
  return launch_pdl(qkv_rope_kernel, dim3(a.num_q + a.num_kv), dim3(128), smem, s, a);
}

size_t attn_scratch_bytes(uint32_t num_q, uint32_t total_slots, uint32_t head_dim) {
  uint32_t nchunks = (total_slots + kAttnChunk - 1) / kAttnChunk;
  return sizeof(float) * (size_t)num_q * nchunks * (head_dim + 2);
}

cudaError_t launch_decode_attn(const AttnArgs &a, cudaStream_t s) {
  switch (a.head_dim) {
    case 64: return launch_attn_d<2>(a, s);
    case 128: return launch_attn_d<4>(a, s);
    case 256: return launch_attn_d<8>(a, s);
    case 512: return launch_attn_d<16>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attn_fused(const AttnFusedArgs &a, cudaStream_t s, bool pdl) {
  if (a.num_kv == 0 || a.num_q % a.num_kv != 0) return cudaErrorInvalidValue;
  switch (a.head_dim) {
    case 64: return launch_attn_fused_d<2>(a, s, pdl);
    case 128: return launch_attn_fused_d<4>(a, s, pdl);
    case 256: return launch_attn_fused_d<8>(a, s, pdl);
    case 512: return launch_attn_fused_d<16>(a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

size_t argmax_scratch_bytes() { return sizeof(float2) * kArgmaxBlocks; }

cudaError_t launch_argmax(const float *logits, uint32_t n, uint32_t *out, void *scratch,
                          size_t scratch_bytes, cudaStream_t s) {
  if (scratch_bytes < argmax_scratch_bytes() || n == 0) return cudaErrorInvalidValue;
  float2 *part = static_cast<float2 *>(scratch);
  cudaError_t e = launch_pdl(argmax_partial_kernel, dim3(kArgmaxBlocks), dim3(kArgmaxThreads), 0,
                             s, logits, n, part);
  if (e != cudaSuccess) return e;
  return launch_pdl(argmax_final_kernel, dim3(1), dim3(kArgmaxThreads), 0, s, logits,
                    (const float2 *)part, (uint32_t)kArgmaxBlocks, out);
}

}  // namespace sx
