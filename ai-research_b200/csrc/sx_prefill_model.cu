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

// ---------------------------------------------------------------------------------------
// Tensor-core form of the prefill attention (head_dim 256, bf16 cache, G = 1, 2, 4 or 8 q heads
// per kv head).  One CTA per (work item, kv head); a work item is a run of up to 64 / G
// consecutive tokens of one session (built on the host), i.e. 64 query rows (token-major,
// row = token * G + head).  The CTA ORs the item's per-token active-slot lists into one
// 64-bit token mask per ring slot, compacts the slots with a nonzero mask into a key list
// (ring-slot order), and streams that list's K/V rows through double-buffered shared-memory
// tiles of 64 keys (cp.async gathers).  Per tile: S = Q K^T and O += P V on mma.m16n8k16 (bf16,
// f32 accumulate), with q and p split into bf16 hi + lo (16 significant bits; K and V are
// exact bf16), a key visible to a row only when its token listed that slot (the ring's own
// causal and window mask), and an online softmax per row in f32.  8 warps: 4 row groups of
// 16 x 2 halves of head_dim (both halves of a row group compute the same scores).  Each row
// ends as bf16(O / L), like the CUDA-core kernel.
constexpr int kTcRows = 64, kTcKeys = 64, kTcD = 256;
constexpr int kTcStride = kTcD * 2 + 16;  // bytes per shared row: fragment loads conflict-free
constexpr int kTcThreads = 256;
constexpr uint32_t kTcMaxSlots = 1024;
constexpr uint32_t kTcRowBytes = kTcRows * kTcStride;
// qh | ql | k[2] | v[2] | tile masks [2][64] u64 | slot masks [1024] u64 | key list [1024] u32 |
// scan [32] u32
constexpr uint32_t kTcSmem = 6 * kTcRowBytes + 2 * kTcKeys * 8 + kTcMaxSlots * 8 +
                             kTcMaxSlots * 4 + 32 * 4;

SX_DEV uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}
// x0, x1 -> bf16 hi pair and the bf16 pair of the residuals
SX_DEV void split_bf16x2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  hi = *reinterpret_cast<const uint32_t *>(&h);
  lo = pack_bf16x2(__fsub_rn(x0, __low2float(h)), __fsub_rn(x1, __high2float(h)));
}
SX_DEV void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <int G>
__global__ void __launch_bounds__(kTcThreads, 1) pf_attn_tc_kernel(PfAttnArgs a) {
  constexpr int TB = kTcRows / G;
  constexpr uint32_t D = kTcD;
  extern __shared__ __align__(128) uint8_t tsm[];
  uint8_t *const qh = tsm, *const ql = qh + kTcRowBytes;
  uint8_t *const kb = ql + kTcRowBytes;          // [2][64 rows]
  uint8_t *const vb = kb + 2 * kTcRowBytes;      // [2][64 rows]
  uint64_t *const tmask = reinterpret_cast<uint64_t *>(vb + 2 * kTcRowBytes);  // [2][64]
  uint64_t *const umask = tmask + 2 * kTcKeys;   // [ts]
  uint32_t *const ulist = reinterpret_cast<uint32_t *>(umask + kTcMaxSlots);
  uint32_t *const scan = ulist + kTcMaxSlots;    // [32]
  const uint32_t item = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const uint32_t ts = a.total_slots;
  const uint32_t t0 = a.items[2 * item], nt = min(a.items[2 * item + 1], (uint32_t)TB);
  const uint32_t sess = a.sess[t0];
  const bool bad = sess >= a.sessions || t0 + nt > a.tokens;
  if (bad && tid == 0) raise_error(a.err, kDevBadParams);
  const size_t cache0 = (size_t)(bad ? 0 : sess) * a.cache_ld;

  // 1. slot masks of the item's tokens, and q (hi / lo bf16) in shared memory
  for (uint32_t i = tid; i < ts; i += kTcThreads) umask[i] = 0ull;
  __syncthreads();
  for (uint32_t r = 0; r < (bad ? 0u : nt); ++r) {
    const uint32_t t = t0 + r, S = min(a.count[t], ts);
    const uint32_t *list = a.slots + (size_t)t * ts;
    for (uint32_t j = tid; j < S; j += kTcThreads) {
      const uint32_t sl = list[j];
      if (sl < ts) atomicOr(reinterpret_cast<unsigned long long *>(umask + sl), 1ull << r);
      else raise_error(a.err, kDevBadSlot);
    }
  }
  for (uint32_t pi = tid; pi < kTcRows * D / 2; pi += kTcThreads) {
    const uint32_t row = pi / (D / 2), dp = pi % (D / 2), tr = row / G, h = row % G;
    float2 x = make_float2(0.0f, 0.0f);
    if (!bad && tr < nt)
      x = *reinterpret_cast<const float2 *>(a.q + ((size_t)(t0 + tr) * a.num_q + kvh * G + h) * D + 2 * dp);
    uint32_t hi, lo;
    split_bf16x2(x.x, x.y, hi, lo);
    *reinterpret_cast<uint32_t *>(qh + row * kTcStride + dp * 4) = hi;
    *reinterpret_cast<uint32_t *>(ql + row * kTcStride + dp * 4) = lo;
  }
  __syncthreads();
  // 2. key list: the slots with a nonzero mask, in slot order (block-wide exclusive scan)
  constexpr uint32_t kPer = kTcMaxSlots / kTcThreads;
  uint32_t cnt = 0;
#pragma unroll
  for (uint32_t k = 0; k < kPer; ++k) {
    const uint32_t i = tid * kPer + k;
    cnt += (i < ts && umask[i] != 0ull) ? 1u : 0u;
  }
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) scan[warp] = incl;
  __syncthreads();
  uint32_t wbase = 0, n_u = 0;
  for (int w = 0; w < kTcThreads / 32; ++w) {
    if (w < warp) wbase += scan[w];
    n_u += scan[w];
  }
  uint32_t pos = wbase + incl - cnt;
#pragma unroll
  for (uint32_t k = 0; k < kPer; ++k) {
    const uint32_t i = tid * kPer + k;
    if (i < ts && umask[i] != 0ull) ulist[pos++] = i;
  }
  __syncthreads();

  // 3. key tiles: K and V rows of 64 keys per tile gathered with cp.async, double-buffered
  const uint32_t ntiles = (n_u + kTcKeys - 1) / kTcKeys;
  const uint8_t *const kc = static_cast<const uint8_t *>(a.k_cache);
  const uint8_t *const vc = static_cast<const uint8_t *>(a.v_cache);
  auto issue = [&](uint32_t tile) {
    const uint32_t buf = tile & 1;
    uint8_t *kd = kb + buf * kTcRowBytes, *vd = vb + buf * kTcRowBytes;
    // 64 rows x 32 chunks of 16 B for each of K and V: 16 copies per thread
    for (uint32_t q = tid; q < kTcKeys * 32; q += kTcThreads) {
      const uint32_t kr = q >> 5, ch = q & 31, u = tile * kTcKeys + kr;
      if (u < n_u) {
        const size_t off = (cache0 + ((size_t)ulist[u] * a.num_kv + kvh) * D) * 2 + ch * 16;
        cp_async16(smem_u32(kd + kr * kTcStride + ch * 16), kc + off);
        cp_async16(smem_u32(vd + kr * kTcStride + ch * 16), vc + off);
      } else {
        *reinterpret_cast<uint4 *>(kd + kr * kTcStride + ch * 16) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(vd + kr * kTcStride + ch * 16) = make_uint4(0, 0, 0, 0);
      }
    }
    if (tid < kTcKeys) {
      const uint32_t u = tile * kTcKeys + tid;
      tmask[buf * kTcKeys + tid] = u < n_u ? umask[ulist[u]] : 0ull;
    }
    cp_async_commit();
  };
  if (ntiles > 0) issue(0);

  const int rg = warp & 3, dh = warp >> 2;
  const uint32_t row0 = 16 * rg + g, row1 = row0 + 8;
  const uint32_t tok0 = row0 / G, tok1 = row1 / G;
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
  const uint8_t *const qh0 = qh + row0 * kTcStride + 4 * c, *const qh1 = qh + row1 * kTcStride + 4 * c;
  const uint8_t *const ql0 = ql + row0 * kTcStride + 4 * c, *const ql1 = ql + row1 * kTcStride + 4 * c;
  for (uint32_t tile = 0; tile < ntiles; ++tile) {
    const uint32_t buf = tile & 1;
    if (tile + 1 < ntiles) issue(tile + 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint8_t *const kd = kb + buf * kTcRowBytes, *const vd = vb + buf * kTcRowBytes;
    // S = Q K^T for this warp's 16 rows x 64 keys
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll 4
    for (int kk = 0; kk < 16; ++kk) {
      const uint32_t off = kk * 32;
      uint32_t ah[4], al[4];
      ah[0] = *reinterpret_cast<const uint32_t *>(qh0 + off);
      ah[1] = *reinterpret_cast<const uint32_t *>(qh1 + off);
      ah[2] = *reinterpret_cast<const uint32_t *>(qh0 + off + 16);
      ah[3] = *reinterpret_cast<const uint32_t *>(qh1 + off + 16);
      al[0] = *reinterpret_cast<const uint32_t *>(ql0 + off);
      al[1] = *reinterpret_cast<const uint32_t *>(ql1 + off);
      al[2] = *reinterpret_cast<const uint32_t *>(ql0 + off + 16);
      al[3] = *reinterpret_cast<const uint32_t *>(ql1 + off + 16);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint8_t *krow = kd + (8 * j + g) * kTcStride + off + 4 * c;
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(krow);
        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(krow + 16);
        mma_bf16_16816(sc[j], ah, b0, b1);
        mma_bf16_16816(sc[j], al, b0, b1);
      }
    }
    // visibility (the token listed the slot) and scale, then the online softmax per row
    const uint64_t *const tm = tmask + buf * kTcKeys;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t key = 8 * j + 2 * c + (e & 1);
        const uint32_t tok = e < 2 ? tok0 : tok1;
        const bool vis = (tm[key] >> tok) & 1ull;
        sc[j][e] = vis ? sc[j][e] * a.scale : -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], sc[j][e]);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m[r], mx[r]);
      corr[r] = m[r] == -INFINITY ? (mn == -INFINITY ? 1.0f : 0.0f) : expf(m[r] - mn);
      m[r] = mn;
    }
    float ps[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = sc[j][e] == -INFINITY ? 0.0f : expf(sc[j][e] - m[e >> 1]);
        sc[j][e] = p;
        ps[e >> 1] += p;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      ps[r] += __shfl_xor_sync(0xffffffffu, ps[r], 1);
      ps[r] += __shfl_xor_sync(0xffffffffu, ps[r], 2);
      l[r] = fmaf(l[r], corr[r], ps[r]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // O += P V over this warp's half of head_dim: 4 key steps of 16, 16 d tiles of 8
    const uint32_t vbase = smem_u32(vd) + (lane & 7) * kTcStride + ((lane >> 3) & 1) * 8 * kTcStride +
                           (dh * 128 + (lane >> 4) * 8) * 2;
#pragma unroll
    for (int s2 = 0; s2 < 4; ++s2) {
      uint32_t ph[4], pl[4];
      split_bf16x2(sc[2 * s2][0], sc[2 * s2][1], ph[0], pl[0]);
      split_bf16x2(sc[2 * s2][2], sc[2 * s2][3], ph[1], pl[1]);
      split_bf16x2(sc[2 * s2 + 1][0], sc[2 * s2 + 1][1], ph[2], pl[2]);
      split_bf16x2(sc[2 * s2 + 1][2], sc[2 * s2 + 1][3], ph[3], pl[3]);
#pragma unroll
      for (int jd = 0; jd < 16; jd += 2) {
        uint32_t b00, b01, b10, b11;
        ldsm_x4_trans(vbase + s2 * 16 * kTcStride + jd * 16, b00, b01, b10, b11);
        mma_bf16_16816(o[jd], ph, b00, b01);
        mma_bf16_16816(o[jd], pl, b00, b01);
        mma_bf16_16816(o[jd + 1], ph, b10, b11);
        mma_bf16_16816(o[jd + 1], pl, b10, b11);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
  cp_async_wait<0>();
  // 4. O / L as bf16
  if (!bad) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t row = r ? row1 : row0, tr = row / G, h = row % G;
      if (tr >= nt) continue;
      uint16_t *out = reinterpret_cast<uint16_t *>(a.out) +
                      ((size_t)(t0 + tr) * a.num_q + kvh * G + h) * D + dh * 128 + 2 * c;
#pragma unroll
      for (int jd = 0; jd < 16; ++jd) {
        const float v0 = l[r] > 0.0f ? o[jd][2 * r] / l[r] : 0.0f;
        const float v1 = l[r] > 0.0f ? o[jd][2 * r + 1] / l[r] : 0.0f;
        const uint32_t pk = (uint32_t)bf16_bits_rne(v0) | ((uint32_t)bf16_bits_rne(v1) << 16);
        *reinterpret_cast<uint32_t *>(out + jd * 8) = pk;
      }
    }
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

template <int G>
cudaError_t launch_attn_tc(const PfAttnArgs &a, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(pf_attn_tc_kernel<G>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
  if (e != cudaSuccess) return e;
  pf_attn_tc_kernel<G><<<dim3(a.n_items, a.num_kv), kTcThreads, kTcSmem, s>>>(a);
  return cudaGetLastError();
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

bool pf_attn_tc_ok(const PfAttnArgs &a) {
  if (a.num_kv == 0 || a.num_q % a.num_kv) return false;
  const uint32_t g = a.num_q / a.num_kv;
  return (g == 1 || g == 2 || g == 4 || g == 8) && a.head_dim == kTcD && a.kv_bf16 &&
         a.total_slots <= kTcMaxSlots;
}

cudaError_t launch_pf_attn(const PfAttnArgs &a, cudaStream_t s) {
  if (a.num_kv == 0 || a.num_q % a.num_kv) return cudaErrorInvalidValue;
  if (a.items != nullptr && pf_attn_tc_ok(a)) {
    if (a.n_items == 0) return cudaSuccess;
    switch (a.num_q / a.num_kv) {
      case 1: return launch_attn_tc<1>(a, s);
      case 2: return launch_attn_tc<2>(a, s);
      case 4: return launch_attn_tc<4>(a, s);
      case 8: return launch_attn_tc<8>(a, s);
      default: return cudaErrorInvalidValue;
    }
  }
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
