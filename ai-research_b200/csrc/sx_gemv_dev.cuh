// sx_gemv_dev.cuh -- device code of the Q4_0 / Q8_0 GEMV, shared by its own kernel
// (sx_gemv.cu) and the persistent decode kernel (sx_persist.cu).
//
//
// Replaces gemv_q4.wgsl, gemv_q8.wgsl, fused_mlp_q4.wgsl and argmax.wgsl (reference dispatch:
// src/gpu/kernels.zig:80-95,139-142).  Semantics: y[r] = sum_b sum_e ((q - 8) * d_b) * x[e]
// for Q4, (q * d_b) * x[e] for Q8; GeGLU: y[r] = gelu_tanh(Wg[r].x) * (Wu[r].x)
// (kernels.zig:94-115); argmax = first index of the maximum (kernels.zig:164-174).
//
// Work split.  The matrix (or the concatenation of up to three matrices, e.g. q|k|v) is a
// sequence of tiles x pairs 640-byte chunks (16 rows x 64 columns; 1152 B for Q8).  One
// persistent 512-thread CTA runs per SM and owns a contiguous run of whole tiles (tile counts
// balanced to within one); its 16 warps split the run's chunks evenly.  Each warp streams its
// chunks through its own shared-memory ring of S stages with 16-byte cp.async copies; the first
// S - 1 chunks are issued before the programmatic-dependent-launch wait, i.e. while the previous
// kernel is still finishing.  The chunks of a call form one contiguous stream (the segments of a
// q|k|v call lie back to back), each lane copies and reads back the same 16 bytes of every quant
// record, and the warp synchronises once per chunk for the shared scale record.  A tile held by
// one warp is written directly; the partial sums of a tile shared by several warps of the CTA
// meet in shared memory after the loop and are added in warp order (deterministic; no global
// scratch, fences or atomics).
//
// Dequantisation.  Nibbles become mma.m16n8k16 A fragments with one shift + one LOP3 per two
// weights (bf16 value 8 + q/2, exact).  The f32 activation enters as the B operand split into
// bf16 hi + lo (16 significant bits), one column pair per batch row, so the tensor core forms
// the 32-element block dot products; the per-block f32 scale and the offset are applied on
// the f32 result: sum_e (q_e - 8) x_e = 2 * (D - 12 * sum_e x_e).  (A 1024-magic f16 form
// needs fewer logic ops but carries an offset ~200x the signal through the f32 sums, costing
// about 1e-3 relative accuracy on the outputs; the bf16 form keeps the offset near 5x.)  Q8
// uses f16 values 1024 + (q + 128) (exact) with a per-vector power-of-two prescale of x.
#pragma once
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr int kThreads = 512;  // one persistent CTA per SM, 16 stream-K workers
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kSmemLimit = 227 * 1024;
// Lane-private scale copies (four per stage) remove the per-chunk warp synchronisation but
// quadruple the scale bytes written to and read from shared memory; the shared copy is used.
constexpr bool kPrivScales = false;

SX_HD uint32_t nv_of(uint32_t batch) {
  return batch <= 1 ? 2u : batch <= 2 ? 4u : batch <= 4 ? 8u : 16u;
}

template <int QT>
struct QTraits;
template <>
struct QTraits<4> {
  static constexpr int kChunk = kQ4ChunkBytes;
  static constexpr int kScaleOff = 512;
  static constexpr int kStage = 512 + 512;  // quants + four copies of the scales
  static constexpr int kStageShared = 512 + 128;  // quants + one shared copy
};
template <>
struct QTraits<8> {
  static constexpr int kChunk = kQ8ChunkBytes;
  static constexpr int kScaleOff = 1024;
  static constexpr int kStage = 1024 + 512;
  static constexpr int kStageShared = 1024 + 128;
};

struct Layout {
  uint32_t xfrag, corr, misc, xin, xin_bytes, ring, total;
};

// xfrag | corr | misc (xscale[8], xexp[8], red[32]) | xin (f32 activation) | ring
SX_HD Layout layout_of(uint32_t k, uint32_t batch, int nmat, int qt, bool with_xin, int stages) {
  Layout L;
  uint32_t nblk = 2 * pairs_of(k);
  L.xfrag = 0;
  L.corr = nblk * nv_of(batch) * 64;
  L.misc = L.corr + ((nblk * batch * 4 + 15) & ~15u);
  L.xin = L.misc + 48 * 4;
  L.xin_bytes = with_xin ? batch * k * 4 : 0;
  L.ring = (L.xin + L.xin_bytes + 127) & ~127u;
  // a ring stage holds the chunk's quants and, for one column set, one copy of its 128 B of
  // scales per lane of a row group (every lane then reads only bytes it copied itself); with
  // two column sets the x fragments are large and the warp shares a single copy
  const bool priv = kPrivScales && batch <= 4;
  uint32_t stage = qt == 4 ? (priv ? QTraits<4>::kStage : QTraits<4>::kStageShared)
                           : (priv ? QTraits<8>::kStage : QTraits<8>::kStageShared);
  L.total = L.ring + kWarps * stages * nmat * stage;
  return L;
}

// Deepest ring (8, 6, 4 or 2 stages per warp) that fits in shared memory; 0 if none does.  x
// gets its own staging area whenever it fits (the fused prologues require it).
SX_HD int stages_for(uint32_t k, uint32_t batch, int nmat, int qt, bool pro) {
  const int opts[4] = {8, 6, 4, 2};
  for (int s : opts)
    if (layout_of(k, batch, nmat, qt, true, s).total <= kSmemLimit) return s;
  if (!pro)
    for (int s : opts)
      if (layout_of(k, batch, nmat, qt, false, s).total <= kSmemLimit) return s;
  return 0;
}
SX_HD Layout layout_for(uint32_t k, uint32_t batch, int nmat, int qt, int s) {
  Layout L = layout_of(k, batch, nmat, qt, true, s);
  return L.total <= kSmemLimit ? L : layout_of(k, batch, nmat, qt, false, s);
}

SX_DEV float gelu_tanh_dev(float x) {
  // kernels.zig:94-97, same operation order
  float x3 = __fmul_rn(__fmul_rn(x, x), x);
  float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

SX_DEV float inv_rms(float ss, uint32_t n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// The threads that run a prologue / x staging and how they synchronise: the whole CTA
// (__syncthreads) in the GEMV kernels, the consumer warps alone (a named barrier) in the
// streaming decode kernel, whose producer warp never joins them.
struct CtaSync {
  SX_DEV void operator()() const { __syncthreads(); }
  SX_DEV uint32_t threads() const { return blockDim.x; }
};

// Sum over the synchronising threads; `red` holds >= 32 floats.  All of them get the result.
template <typename Sync>
SX_DEV float group_block_sum(float v, float *red, const Sync &sync) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (int)(sync.threads() + 31) >> 5;
  v = warp_sum(v);
  sync();
  if (lane == 0) red[wid] = v;
  sync();
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}

// ---------------------------------------------------------------------------------------
// Fused input prologues (replace a separate norm launch).  Each CTA computes the GEMV input
// for all batch rows into shared memory with one round trip to global memory:
//   kProNorm:  xin = rmsnorm(x, w)                                   (rmsnorm.wgsl)
//   kProResid: v = post_w ? rmsnorm(mlp, post_w) : mlp; xn = (x + v) * scalar;
//              CTA 0 writes xn to x_out; xin = rmsnorm(xn, w)         (add_rmsnorm.wgsl)
constexpr int kProPer = 8;  // elements per thread held in registers: K <= 512 * 8
constexpr int kProMaxParts = 8;  // partial vectors a residual prologue adds (pro_mlp_parts)

// The prologue's norm gains (weights: they do not depend on the producer of x, so a caller may
// load them before it waits for that producer).
struct ProGains {
  float nw[kProPer], pw[kProPer];
};
SX_DEV void load_prologue_gains(const GemvArgs &a, uint32_t nthr, ProGains &gn) {
#pragma unroll
  for (int q = 0; q < kProPer; ++q) {
    const uint32_t i = threadIdx.x + q * nthr;
    const bool in = i < a.k;
    gn.nw[q] = in ? a.pro_w[i] : 0.0f;
    gn.pw[q] = (in && a.pro == kProResid && a.pro_post_w) ? a.pro_post_w[i] : 0.0f;
  }
}

template <typename Sync>
SX_DEV void run_prologue_gains(const GemvArgs &a, float *xin, float *red, const Sync &sync,
                               const ProGains &gn) {
  const uint32_t K = a.k, nthr = sync.threads();
  for (uint32_t j = 0; j < a.batch; ++j) {
    float *xo = xin + (size_t)j * K;
    const float *x = a.x + (size_t)j * a.ldx;
    float xv[kProPer], mv[kProPer];
    const float *pw = gn.pw, *nw = gn.nw;
#pragma unroll
    for (int q = 0; q < kProPer; ++q) {
      uint32_t i = threadIdx.x + q * nthr;
      bool in = i < K;
      xv[q] = in ? __ldcg(x + i) : 0.0f;  // activations: through L2 (see stage_x)
      mv[q] = 0.0f;
      if (a.pro == kProResid && in) mv[q] = __ldcg(a.pro_mlp + (size_t)j * a.ldx + i);
    }
    if (a.pro == kProResid && a.pro_mlp_parts > 1) {
      // a sublayer output delivered as partial vectors, added in part order (the Q4 calls of
      // their own kernel take stage_x_q4, which keeps four parts' loads in flight)
#pragma unroll 1
      for (uint32_t p = 1; p < a.pro_mlp_parts; ++p)
#pragma unroll
        for (int q = 0; q < kProPer; ++q) {
          const uint32_t i = threadIdx.x + q * nthr;
          if (i < K) mv[q] += __ldcg(a.pro_mlp + (size_t)p * a.pro_mlp_ld + (size_t)j * a.ldx + i);
        }
    }
    if (a.pro == kProResid) {
      float rm = 1.0f;
      if (a.pro_post_w) {
        float ss = 0.0f;
#pragma unroll
        for (int q = 0; q < kProPer; ++q) ss = fmaf(mv[q], mv[q], ss);
        rm = inv_rms(group_block_sum(ss, red, sync), K, a.eps);
      }
#pragma unroll
      for (int q = 0; q < kProPer; ++q) {
        float v = mv[q];
        if (a.pro_post_w) v = __fmul_rn(__fmul_rn(v, rm), pw[q]);
        xv[q] = __fmul_rn(__fadd_rn(xv[q], v), a.pro_scalar);
      }
      if (blockIdx.x == 0) {
#pragma unroll
        for (int q = 0; q < kProPer; ++q) {
          uint32_t i = threadIdx.x + q * nthr;
          if (i < K) a.pro_x_out[(size_t)j * a.ldx + i] = xv[q];
        }
      }
    }
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < kProPer; ++q) ss = fmaf(xv[q], xv[q], ss);
    float r = inv_rms(group_block_sum(ss, red, sync), K, a.eps);
#pragma unroll
    for (int q = 0; q < kProPer; ++q) {
      uint32_t i = threadIdx.x + q * nthr;
      if (i < K) {
        const float v = __fmul_rn(__fmul_rn(xv[q], r), nw[q]);
        xo[i] = v;
        if (a.pro_norm_out != nullptr && blockIdx.x == 0) a.pro_norm_out[(size_t)j * K + i] = v;
      }
    }
    sync();
  }
}

template <typename Sync = CtaSync>
SX_DEV void run_prologue(const GemvArgs &a, float *xin, float *red, const Sync &sync = Sync()) {
  ProGains gn;
  load_prologue_gains(a, sync.threads(), gn);
  run_prologue_gains(a, xin, red, sync, gn);
}

// Activation -> B fragments.  Item (blk, j, c, jj) converts elements 32*blk + 8*jj + 2c,+1
// of batch row j into the hi/lo pair words and reduces the block sum for the offset term.
template <int QT, typename Sync = CtaSync>
SX_DEV void stage_x(const GemvArgs &a, const float *src, uint32_t ld, uint8_t *smem,
                    const Layout &L, bool src_global, const Sync &sync = Sync()) {
  const uint32_t nthr = sync.threads();
  uint32_t *xf = reinterpret_cast<uint32_t *>(smem + L.xfrag);
  float *corr = reinterpret_cast<float *>(smem + L.corr);
  float *xscale = reinterpret_cast<float *>(smem + L.misc);
  int *xexp = reinterpret_cast<int *>(smem + L.misc + 32);
  float *red = reinterpret_cast<float *>(smem + L.misc + 64);
  const uint32_t nb = a.k / 32, nblk = 2 * pairs_of(a.k), nv = nv_of(a.batch);
  const int tid = threadIdx.x;

  if (QT == 8) {
    // Per-row power-of-two prescale so that the f16 hi/lo split neither overflows nor loses
    // precision: max |x| * 2^e < 2^15.
    for (uint32_t j = 0; j < a.batch; ++j) {
      float mx = 0.0f;
      for (uint32_t i = tid; i < a.k; i += nthr)
        mx = fmaxf(mx, fabsf(src_global ? __ldcg(src + j * ld + i) : src[j * ld + i]));
      mx = warp_max(mx);
      sync();
      if ((tid & 31) == 0) red[tid >> 5] = mx;
      sync();
      if (tid == 0) {
        float m = 0.0f;
        for (int w = 0; w < (int)(nthr >> 5); ++w) m = fmaxf(m, red[w]);
        int e = 0;
        if (m > 0.0f && isfinite(m)) {
          int ex;
          frexpf(m, &ex);
          e = 15 - ex;
          e = e > 100 ? 100 : (e < -100 ? -100 : e);
        }
        xexp[j] = e;
        xscale[j] = ldexpf(1.0f, -e);
      }
      sync();
    }
  } else {
    if (tid < (int)a.batch) {
      xscale[tid] = 2.0f;
      xexp[tid] = 0;
    }
    sync();
  }

  // One thread per group of 8 consecutive elements (block blk, word jj of each of the four
  // lane columns c): packed conversions, four scattered fragment words per variant, and the
  // block sum for the offset term over the block's four groups (adjacent lanes).
  const uint32_t groups = nblk * 4;
  const uint32_t gpad = (groups + 31) & ~31u;
  for (uint32_t j = 0; j < a.batch; ++j) {
    // Q8: multiply by 2^e (exact for a power of two, e in [-100, 100])
    const float p2 = QT == 8 ? __int_as_float((xexp[j] + 127) << 23) : 1.0f;
    for (uint32_t gi = tid; gi < gpad; gi += nthr) {
      const uint32_t blk = gi >> 2, jj = gi & 3;
      float part = 0.0f;
      if (gi < groups) {
        float v[8];
        if (blk < nb) {
          // x written by an earlier phase of the same kernel is read through L2 (no stale L1)
          const float4 *q4 = reinterpret_cast<const float4 *>(src + (size_t)j * ld + blk * 32 + jj * 8);
          const float4 u0 = src_global ? __ldcg(q4) : q4[0];
          const float4 u1 = src_global ? __ldcg(q4 + 1) : q4[1];
          v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
          v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) v[q] = 0.0f;
        }
        const uint32_t pr = blk >> 1, hb = blk & 1;
        // word jj of uint4 ((variant * 4 + c) * 2 + hb) of pair pr; c steps 8 words
        uint32_t *hi_w = xf + ((((pr * nv + 2 * j) * 4) * 2 + hb) * 4 + jj);
        uint32_t *lo_w = xf + ((((pr * nv + 2 * j + 1) * 4) * 2 + hb) * 4 + jj);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float x0 = v[2 * c] * p2, x1 = v[2 * c + 1] * p2;
          uint32_t hw, lw;
          float h0, h1, l0, l1;
          if (QT == 4) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
            h0 = __low2float(h);
            h1 = __high2float(h);
            const __nv_bfloat162 l = __floats2bfloat162_rn(__fsub_rn(x0, h0), __fsub_rn(x1, h1));
            l0 = __low2float(l);
            l1 = __high2float(l);
            hw = *reinterpret_cast<const uint32_t *>(&h);
            lw = *reinterpret_cast<const uint32_t *>(&l);
          } else {
            const __half2 h = __floats2half2_rn(x0, x1);
            h0 = __low2float(h);
            h1 = __high2float(h);
            const __half2 l = __floats2half2_rn(__fsub_rn(x0, h0), __fsub_rn(x1, h1));
            l0 = __low2float(l);
            l1 = __high2float(l);
            hw = *reinterpret_cast<const uint32_t *>(&h);
            lw = *reinterpret_cast<const uint32_t *>(&l);
          }
          hi_w[c * 8] = hw;
          lo_w[c * 8] = lw;
          part += (h0 + l0) + (h1 + l1);
        }
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      // Q4 value 8 + q / 2 = (q - 8) / 2 + 12; Q8 value 1024 + (q + 128) = q + 1152
      if (gi < groups && jj == 0)
        corr[((blk >> 1) * a.batch + j) * 2 + (blk & 1)] = (QT == 4 ? 12.0f : 1152.0f) * part;
    }
  }
  sync();
}

// ---------------------------------------------------------------------------------------
// Q4 input staging with the fused prologue in one pass, batch 1..8: thread t owns the group of
// 8 consecutive input elements 8 t .. 8 t + 7 of every batch row (block t / 4, word t % 4 of
// the fragment layout built by stage_x), so the normalised values go from registers straight
// into the B fragments (no f32 staging in shared memory), and each of the prologue's two sums
// costs one barrier per pair of rows (separate reduction buffers in the unused f32 staging
// area).  The norm gains do not depend on the producer of x and are loaded before its wait
// (load_gains_q4).  Without a prologue a thread converts up to kStageGroups groups per row
// (K <= 16384 with 512 threads).  Same operation order per element as run_prologue; a row's
// sums of squares add a thread's 8 consecutive elements, then the warp, then the warps in
// order, exactly as for batch 1, so every row of a batch is staged bit-identically to the same
// row alone.
constexpr int kStageGroups = 4;
constexpr int kStageRows = 2;  // rows per prologue round (one barrier per sum per round)
struct GainsQ4 {
  float nw[8], pw[8];
};
SX_HD bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }
SX_HD bool stage_q4_ok(const GemvArgs &a, uint32_t nthr, const Layout &L) {
  const uint32_t groups = 8 * pairs_of(a.k);  // 2 * pairs blocks x 4 groups
  if (a.batch < 1 || a.batch > 8 || a.k % 8 != 0 || !al16(a.x) || (a.batch > 1 && a.ldx % 4 != 0))
    return false;
  if (a.pro == kProNone) return groups <= kStageGroups * nthr;
  const uint32_t rounds = (a.batch + kStageRows - 1) / kStageRows;
  if (groups > nthr || !al16(a.pro_w) || a.pro_norm_out != nullptr ||
      L.xin_bytes < rounds * 2 * kStageRows * kWarps * 4 || nthr != kThreads)
    return false;
  if (a.pro == kProResid)
    return al16(a.pro_mlp) && al16(a.pro_x_out) && (!a.pro_post_w || al16(a.pro_post_w)) &&
           a.pro_mlp_parts <= (uint32_t)kProMaxParts &&
           (a.pro_mlp_parts <= 1 || (a.batch == 1 && a.pro_mlp_ld % 4 == 0));
  return true;
}
SX_DEV void load_gains_q4(const GemvArgs &a, GainsQ4 &gn) {
  const uint32_t e0 = 8 * threadIdx.x;
#pragma unroll
  for (int q = 0; q < 8; ++q) gn.nw[q] = gn.pw[q] = 0.0f;
  if (a.pro == kProNone || e0 >= a.k) return;
  const float4 *w4 = reinterpret_cast<const float4 *>(a.pro_w + e0);
  const float4 u0 = w4[0], u1 = w4[1];
  gn.nw[0] = u0.x; gn.nw[1] = u0.y; gn.nw[2] = u0.z; gn.nw[3] = u0.w;
  gn.nw[4] = u1.x; gn.nw[5] = u1.y; gn.nw[6] = u1.z; gn.nw[7] = u1.w;
  if (a.pro == kProResid && a.pro_post_w) {
    const float4 *p4 = reinterpret_cast<const float4 *>(a.pro_post_w + e0);
    const float4 v0 = p4[0], v1 = p4[1];
    gn.pw[0] = v0.x; gn.pw[1] = v0.y; gn.pw[2] = v0.z; gn.pw[3] = v0.w;
    gn.pw[4] = v1.x; gn.pw[5] = v1.y; gn.pw[6] = v1.z; gn.pw[7] = v1.w;
  }
}
SX_DEV void ld8(const float *p, float (&v)[8]) {
  const float4 u0 = __ldcg(reinterpret_cast<const float4 *>(p));
  const float4 u1 = __ldcg(reinterpret_cast<const float4 *>(p) + 1);
  v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
  v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
}
SX_DEV void zero8(float (&v)[8]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = 0.0f;
}
// R sums over the CTA with one barrier: red holds R x kWarps floats for these sums alone
template <int R>
SX_DEV void cta_sums_1bar(float (&v)[R], float *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    v[r] = warp_sum(v[r]);
    if (lane == 0) red[r * kWarps + w] = v[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float t = lane < kWarps ? red[r * kWarps + lane] : 0.0f;
    v[r] = warp_sum(t);
  }
}

SX_DEV void stage_x_q4(const GemvArgs &a, uint8_t *smem, const Layout &L, const GainsQ4 &gn) {
  uint32_t *xf = reinterpret_cast<uint32_t *>(smem + L.xfrag);
  float *corr = reinterpret_cast<float *>(smem + L.corr);
  float *xscale = reinterpret_cast<float *>(smem + L.misc);
  int *xexp = reinterpret_cast<int *>(smem + L.misc + 32);
  // the f32 staging area is unused on this path: per round, [2 sums][kStageRows][kWarps]
  float *red = reinterpret_cast<float *>(smem + L.xin);
  const uint32_t K = a.k, nb = K / 32, nthr = blockDim.x, tid = threadIdx.x, B = a.batch;
  const uint32_t groups = 8 * pairs_of(K), gpad = (groups + 31) & ~31u, nv = nv_of(B);
  if (tid < B) {
    xscale[tid] = 2.0f;
    xexp[tid] = 0;
  }
  // fragments of group gi of row j: block gi / 4, word gi % 4 of each of the four lane columns
  auto frag = [&](uint32_t gi, uint32_t j, const float (&x)[8]) {
    const uint32_t blk = gi >> 2, jj = gi & 3, pr = blk >> 1, hb = blk & 1;
    float part = 0.0f;
    if (gi < groups) {
      uint32_t *hi_w = xf + ((((pr * nv + 2 * j) * 4) * 2 + hb) * 4 + jj);
      uint32_t *lo_w = xf + ((((pr * nv + 2 * j + 1) * 4) * 2 + hb) * 4 + jj);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float x0 = x[2 * c], x1 = x[2 * c + 1];
        const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
        const float h0 = __low2float(h), h1 = __high2float(h);
        const __nv_bfloat162 l = __floats2bfloat162_rn(__fsub_rn(x0, h0), __fsub_rn(x1, h1));
        hi_w[c * 8] = *reinterpret_cast<const uint32_t *>(&h);
        lo_w[c * 8] = *reinterpret_cast<const uint32_t *>(&l);
        part += (h0 + __low2float(l)) + (h1 + __high2float(l));
      }
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if (gi < groups && jj == 0) corr[(pr * B + j) * 2 + hb] = 12.0f * part;
  };

  if (a.pro == kProNone) {
#pragma unroll 1
    for (uint32_t j = 0; j < B; ++j) {
      const float *xr = a.x + (size_t)j * a.ldx;
      float v[kStageGroups][8];
#pragma unroll
      for (int k = 0; k < kStageGroups; ++k) {
        const uint32_t gi = tid + k * nthr;
        if (gi < groups && (gi >> 2) < nb) ld8(xr + 8 * gi, v[k]);
        else zero8(v[k]);
      }
#pragma unroll
      for (int k = 0; k < kStageGroups; ++k) {
        const uint32_t gi = tid + k * nthr;
        if (gi >= gpad) break;  // warp-uniform: gpad is a multiple of 32
        frag(gi, j, v[k]);
      }
    }
    __syncthreads();
    return;
  }

  // with a prologue: one group per thread and row (K <= 8 * nthr), kStageRows rows per round
  const bool live = tid < groups && (tid >> 2) < nb;
#pragma unroll 1
  for (uint32_t j0 = 0, round = 0; j0 < B; j0 += kStageRows, ++round) {
    float *rr = red + round * 2 * kStageRows * kWarps;
    float xv[kStageRows][8];
#pragma unroll
    for (int r = 0; r < kStageRows; ++r) {
      if (live && j0 + r < B) ld8(a.x + (size_t)(j0 + r) * a.ldx + 8 * tid, xv[r]);
      else zero8(xv[r]);
    }
    if (a.pro == kProResid) {
      float mv[kStageRows][8];
#pragma unroll
      for (int r = 0; r < kStageRows; ++r) {
        if (!live || j0 + r >= B) {
          zero8(mv[r]);
        } else if (a.pro_mlp_parts <= 1) {
          ld8(a.pro_mlp + (size_t)(j0 + r) * a.ldx + 8 * tid, mv[r]);
        } else {
          // batch 1: partial vectors added in part order, four parts' loads in flight at a time
#pragma unroll
          for (int p0 = 0; p0 < kProMaxParts; p0 += 4) {
            float pv[4][8];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              if ((uint32_t)(p0 + p) < a.pro_mlp_parts)
                ld8(a.pro_mlp + (size_t)(p0 + p) * a.pro_mlp_ld + 8 * tid, pv[p]);
              else
                zero8(pv[p]);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float m = p0 == 0 ? pv[0][q] : mv[r][q] + pv[0][q];
#pragma unroll
              for (int p = 1; p < 4; ++p)
                if ((uint32_t)(p0 + p) < a.pro_mlp_parts) m += pv[p][q];
              mv[r][q] = m;
            }
          }
        }
      }
      float rm[kStageRows];
#pragma unroll
      for (int r = 0; r < kStageRows; ++r) rm[r] = 1.0f;
      if (a.pro_post_w) {
        float ss[kStageRows];
#pragma unroll
        for (int r = 0; r < kStageRows; ++r) {
          ss[r] = 0.0f;
#pragma unroll
          for (int q = 0; q < 8; ++q) ss[r] = fmaf(mv[r][q], mv[r][q], ss[r]);
        }
        cta_sums_1bar<kStageRows>(ss, rr);
#pragma unroll
        for (int r = 0; r < kStageRows; ++r) rm[r] = inv_rms(ss[r], K, a.eps);
      }
#pragma unroll
      for (int r = 0; r < kStageRows; ++r) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float m = mv[r][q];
          if (a.pro_post_w) m = __fmul_rn(__fmul_rn(m, rm[r]), gn.pw[q]);
          xv[r][q] = __fmul_rn(__fadd_rn(xv[r][q], m), a.pro_scalar);
        }
        if (blockIdx.x == 0 && live && j0 + r < B) {
          float4 *o4 = reinterpret_cast<float4 *>(a.pro_x_out + (size_t)(j0 + r) * a.ldx + 8 * tid);
          o4[0] = make_float4(xv[r][0], xv[r][1], xv[r][2], xv[r][3]);
          o4[1] = make_float4(xv[r][4], xv[r][5], xv[r][6], xv[r][7]);
        }
      }
    }
    float ss[kStageRows];
#pragma unroll
    for (int r = 0; r < kStageRows; ++r) {
      ss[r] = 0.0f;
#pragma unroll
      for (int q = 0; q < 8; ++q) ss[r] = fmaf(xv[r][q], xv[r][q], ss[r]);
    }
    cta_sums_1bar<kStageRows>(ss, rr + kStageRows * kWarps);
#pragma unroll
    for (int r = 0; r < kStageRows; ++r) {
      const float rs = inv_rms(ss[r], K, a.eps);
#pragma unroll
      for (int q = 0; q < 8; ++q) xv[r][q] = live ? __fmul_rn(__fmul_rn(xv[r][q], rs), gn.nw[q]) : 0.0f;
      if (j0 + r < B && tid < gpad) frag(tid, j0 + r, xv[r]);
    }
  }
  __syncthreads();
}

// One 32-element block of one 16-row tile: two chained m16n8k16 MMAs per column set, the
// offset term enters as the C operand, the block scale is applied to the f32 result.
template <int QT>
SX_DEV void block_mma(const uint32_t (&a0)[4], const uint32_t (&a1)[4], uint4 xb, float cr,
                      float sg, float sg8, float (&acc)[2]) {
  float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (QT == 4) {
    mma_bf16_16816(d, a0, xb.x, xb.y);
    mma_bf16_16816(d, a1, xb.z, xb.w);
  } else {
    mma_f16_16816(d, a0, xb.x, xb.y);
    mma_f16_16816(d, a1, xb.z, xb.w);
  }
  acc[0] = fmaf(sg, (d[0] + d[1]) - cr, acc[0]);
  acc[1] = fmaf(sg8, (d[2] + d[3]) - cr, acc[1]);
}

// worker ranges: worker w owns chunks [N*w/NW, N*(w+1)/NW)
SX_DEV uint32_t wstart(uint32_t N, uint32_t NW, uint32_t w) {
  return (uint32_t)((uint64_t)N * w / NW);
}
SX_DEV uint32_t wowner(uint32_t N, uint32_t NW, uint32_t c) {
  return (uint32_t)(((uint64_t)(c + 1) * NW - 1) / N);
}

struct Best {
  float v;
  uint32_t i;
};
SX_DEV bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// The GEMV of one call by one CTA of kThreads threads.  prefetch: issue the first S - 1
// chunks of this CTA's run (they do not depend on x); run: everything else (x staging, main
// loop, split-tile sums, argmax).  A call split in two passes the same a and smem to both
// halves, with no cp.async group committed in between.  standalone: the CTA is a kernel of its
// own and waits for the producer of x with griddepcontrol.wait.
template <int QT, int NMAT, int NSETS, int S>
SX_DEV void gemv_body(const GemvArgs &a, uint8_t *smem, bool prefetch, bool run,
                          bool standalone) {
  // Q8 GeGLU: the f16 weights 1152 + q get the 1152 taken off exactly (q is an f16 integer)
  // before the MMA.  The offset form carries ~16x the signal through the tensor core's f32
  // accumulation; a GeGLU product turns that rounding, where the gate is near zero and the up
  // value large, into a relative error of the (small) product above the path's tolerance.
  // The Q8 LM head keeps the offset form (one logical op less per two weights).
  constexpr bool EXACT8 = QT == 8 && NMAT == 2;
  constexpr int CB = QTraits<QT>::kChunk;
  constexpr int SO = QTraits<QT>::kScaleOff;
  constexpr bool PRIV = kPrivScales && NSETS == 1;  // lane-private scale copies
  constexpr int KS = PRIV ? QTraits<QT>::kStage : QTraits<QT>::kStageShared;
  constexpr int STAGE = NMAT * KS;
  const bool pro = a.pro != kProNone;
  const Layout L = layout_for(a.k, a.batch, NMAT, QT, S);
  const bool have_xin = L.xin_bytes != 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const uint32_t P = pairs_of(a.k), nv = nv_of(a.batch), batch = a.batch;
  const uint32_t T = a.tiles[0] + a.tiles[1] + a.tiles[2];
  // CTA b owns whole tiles [ct0, ct1) (counts balanced to within one); its warps split the
  // run's chunks evenly, warp w taking [cbase + ncta w / 16, cbase + ncta (w + 1) / 16)
  const uint32_t ct0 = (uint32_t)((uint64_t)T * blockIdx.x / gridDim.x);
  const uint32_t ct1 = (uint32_t)((uint64_t)T * (blockIdx.x + 1) / gridDim.x);
  const uint32_t cbase = ct0 * P, ncta = (ct1 - ct0) * P;
  const uint32_t c0 = cbase + wstart(ncta, kWarps, warp), c1 = cbase + wstart(ncta, kWarps, warp + 1);

  uint8_t *const ring = smem + L.ring + warp * S * STAGE;

  auto seg_of = [&](uint32_t tt, uint32_t &t) {
    int s = 0;
    t = tt;
    if (t >= a.tiles[0]) {
      t -= a.tiles[0];
      s = 1;
      if (t >= a.tiles[1]) {
        t -= a.tiles[1];
        s = 2;
      }
    }
    return s;
  };

  // ---- copies: the chunks of the call form one contiguous stream (the segments of a
  // multi-segment call lie back to back in memory, which the host checks), so chunk i of this
  // worker starts at w[0][m] + (c0 + i) * CB ----
  const uint32_t n = c1 - c0;
  const uint8_t *wsrc[NMAT];
#pragma unroll
  for (int m = 0; m < NMAT; ++m) wsrc[m] = static_cast<const uint8_t *>(a.w[0][m]) + (size_t)c0 * CB;
  // lane (g, c) copies bytes [16 lane, 16 lane + 16) of every 512-B quant sub-record and
  // reads back exactly those.  PRIV: it also copies the 16 B of scales of row group g into its
  // own copy c of the scale record, so no lane waits on another lane's copies; otherwise lanes
  // 0..7 copy the one shared scale record and the warp synchronises once per chunk.
  const uint32_t ring_s = smem_u32(ring);
  const uint32_t q_dst = ring_s + lane * 16;
  const uint32_t s_dst = PRIV ? ring_s + SO + c * 128 + g * 16 : ring_s + SO + lane * 16;
  const uint32_t q_src = lane * 16, s_src = PRIV ? SO + g * 16 : SO + lane * 16;
  const bool s_lane = PRIV || lane < 8;
  // copy chunk i into stage i mod S; one commit group per chunk (empty past the end, so the
  // group count stays uniform)
  const uint64_t pol = l2_evict_first_policy();  // weights are read once per token
  auto issue = [&](uint32_t i) {
    const bool live = i < n;
    const uint32_t stage = (i % S) * STAGE;
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const uint8_t *s = wsrc[m] + (size_t)i * CB;
#pragma unroll
      for (int sub = 0; sub < CB / 512; ++sub)
        cp_async16_if_ef(q_dst + stage + m * KS + sub * 512, s + q_src + sub * 512, live, pol);
      cp_async16_if_ef(s_dst + stage + m * KS, s + s_src, live && s_lane, pol);
    }
    cp_async_commit();
  };

  // 1. the weights do not depend on the producer of x: start streaming them now (chunk
  // S - 1 is issued by the first loop iteration)
  if (prefetch) {
#pragma unroll
    for (int st = 0; st < S - 1; ++st) issue(st);
  }
  if (!run) return;
  // Q4 calls of a kernel of their own stage x in one fused pass (stage_x_q4); the norm gains
  // are weights, loaded before the dependency wait
  const bool fast = QT == 4 && standalone && stage_q4_ok(a, blockDim.x, L);
  GainsQ4 gq;
  if (fast) load_gains_q4(a, gq);
  if (standalone) {
    if (a.pf_slots != nullptr) {
      // the following attention's K/V rows, spread over the CTAs (slot j: thread j / grid of
      // CTA j % grid); the slot list and count are graph inputs, ready before this launch
      const uint32_t S = min(a.pf_step[2], a.pf_max);
      for (uint32_t j = tid * gridDim.x + blockIdx.x; j < S; j += blockDim.x * gridDim.x) {
        const uint32_t sl = a.pf_slots[j];
        if (sl < a.pf_max)
#pragma unroll
          for (int b = 0; b < 2; ++b)
            if (a.pf_base[b] != nullptr)
              prefetch_l2_bulk(static_cast<const uint8_t *>(a.pf_base[b]) + (size_t)sl * a.pf_row_bytes,
                               a.pf_row_bytes);
      }
    }
    pdl_launch_dependents();
    // 2. wait for the producer of x, bring x into shared memory and build the B fragments
    pdl_wait();
    if (gate_closed(a.gate)) {  // recorded behind a closed dispatch record: do nothing
      cp_async_wait<0>();
      return;
    }
  }
  float *xin = reinterpret_cast<float *>(smem + L.xin);
  const float *xsrc = a.x;
  uint32_t xld = a.ldx;
  if (fast) {
    stage_x_q4(a, smem, L, gq);
  } else if (pro) {
    run_prologue(a, xin, reinterpret_cast<float *>(smem + L.misc + 64));
    xsrc = xin;
    xld = a.k;
  } else if (have_xin) {
    // independent 16-byte loads, four in flight per thread, through registers: a cp.async
    // group here would also wait for the weight chunks already in flight
    const uint32_t per_row = a.k / 4, total = batch * per_row;
    constexpr uint32_t U = 4;
    for (uint32_t q0 = tid; q0 < total; q0 += U * blockDim.x) {
      float4 v[U];
#pragma unroll
      for (uint32_t u = 0; u < U; ++u) {
        const uint32_t q = q0 + u * blockDim.x, j = q / per_row, i = q % per_row;
        if (q < total) v[u] = __ldcg(reinterpret_cast<const float4 *>(a.x + (size_t)j * a.ldx) + i);
      }
#pragma unroll
      for (uint32_t u = 0; u < U; ++u) {
        const uint32_t q = q0 + u * blockDim.x, j = q / per_row, i = q % per_row;
        if (q < total) *reinterpret_cast<float4 *>(xin + (size_t)j * a.k + 4 * i) = v[u];
      }
    }
    __syncthreads();
    xsrc = xin;
    xld = a.k;
  }
  if (!fast) stage_x<QT>(a, xsrc, xld, smem, L, xsrc == a.x);

  const uint4 *const xf4 = reinterpret_cast<const uint4 *>(smem + L.xfrag);
  const float *const corr = reinterpret_cast<const float *>(smem + L.corr);
  const float *const xscale = reinterpret_cast<const float *>(smem + L.misc);

  // lane constants: column set s uses B variant 8s + g and batch row 4s + c.  Per pair the
  // fragments are [variant][c][half] uint4 and the offset terms [batch row][half] floats, so a
  // lane's two halves are adjacent.
  uint32_t xoff[NSETS], coff[NSETS];
  bool xvalid[NSETS], cvalid[NSETS];
#pragma unroll
  for (int s = 0; s < NSETS; ++s) {
    xoff[s] = ((8 * s + g) * 4 + c) * 2;
    coff[s] = (4 * s + c) * 2;
    xvalid[s] = (uint32_t)(8 * s + g) < 2 * batch;
    cvalid[s] = (uint32_t)(4 * s + c) < batch;
  }
  const uint32_t xstride = nv * 8, cstride = batch * 2;  // per pair

  Best best[NSETS];
#pragma unroll
  for (int s = 0; s < NSETS; ++s) best[s] = {-INFINITY, 0xFFFFFFFFu};

  // epilogue for one (row, batch) value: apply the factor, GeGLU, write, track the argmax
  auto emit = [&](uint32_t tt, uint32_t row, uint32_t j, const float (&v)[NMAT], int s_idx) {
    uint32_t t;
    int s = seg_of(tt, t);
    uint32_t r = t * 16 + row;
    if (r >= a.rows[s] || j >= batch) return;
    float out = v[0] * xscale[j];
    if (NMAT == 2) out = __fmul_rn(gelu_tanh_dev(out), v[NMAT - 1] * xscale[j]);
    a.y[s][(size_t)j * a.ldy + r] = out;
    if (a.epi == kEpiArgmax) {
      uint32_t gi = a.row_base[s] + r;
      float ov = isnan(out) ? -INFINITY : out;
      if (best[s_idx].i == 0xFFFFFFFFu || better(ov, gi, best[s_idx].v, best[s_idx].i))
        best[s_idx] = {ov, gi};
    }
  };

  float acc[NMAT][NSETS][2];
  // sums of the tiles this warp shares with other warps: slot 0 = the tile holding its first
  // chunk, slot 1 = the tile holding its last chunk
  float part0[NMAT][NSETS][2], part1[NMAT][NSETS][2];
  bool has0 = false, has1 = false;
#pragma unroll
  for (int m = 0; m < NMAT; ++m)
#pragma unroll
    for (int s = 0; s < NSETS; ++s) acc[m][s][0] = acc[m][s][1] = 0.0f;

  // ---- main loop: one 16-row x 64-column chunk per iteration, flushing the accumulators
  // at the end of a tile or of the range ----
  uint32_t tt = c0 / P;
  const uint32_t p0 = c0 % P;
  const uint4 *xp = xf4 + p0 * xstride;
  const float *cp = corr + p0 * cstride;
  uint32_t flush_at = min(P - 1 - p0, n - 1);
  const uint8_t *const q_rd = ring + lane * 16;
  const uint8_t *const s_rd = ring + SO + (PRIV ? c * 128 : 0) + g * 16;
  // B fragments and offset terms of unused columns / batch rows are never loaded: those
  // lanes keep zeros (their D columns are never emitted), with no per-chunk re-zeroing
  uint4 xb[2][NSETS];
  float cr[2][NSETS];
#pragma unroll
  for (int s = 0; s < NSETS; ++s) {
    xb[0][s] = xb[1][s] = make_uint4(0, 0, 0, 0);
    cr[0][s] = cr[1][s] = 0.0f;
  }
  uint32_t i = 0;
  while (i < n) {
#pragma unroll 1
    for (; i <= flush_at; ++i) {
      cp_async_wait<S - 2>();  // this lane's copies of chunk i have landed
      if (!PRIV) __syncwarp();  // ... and every other lane's; all finished chunk i - 1
      issue(i + S - 1);         // refill the stage of chunk i - 1
      const uint32_t st_off = (i % S) * STAGE;
#pragma unroll
      for (int s = 0; s < NSETS; ++s) {
        if (xvalid[s]) {
          xb[0][s] = xp[xoff[s]];
          xb[1][s] = xp[xoff[s] + 1];
        }
        if (cvalid[s]) {
          const float2 c2 = *reinterpret_cast<const float2 *>(cp + coff[s]);
          cr[0][s] = c2.x;
          cr[1][s] = c2.y;
        }
      }
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        const float4 sc = *reinterpret_cast<const float4 *>(s_rd + st_off + m * KS);
        uint4 wq[QT == 4 ? 1 : 2];
        wq[0] = *reinterpret_cast<const uint4 *>(q_rd + st_off + m * KS);
        if (QT == 8) wq[QT == 4 ? 0 : 1] = *reinterpret_cast<const uint4 *>(q_rd + st_off + m * KS + 512);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          uint32_t a0[4], a1[4];
          if (QT == 4) {
            uint32_t rg[4], rg8[4];
            dq4_word(hb ? wq[0].z : wq[0].x, rg);
            dq4_word(hb ? wq[0].w : wq[0].y, rg8);
            a0[0] = rg[0]; a0[1] = rg8[0]; a0[2] = rg[1]; a0[3] = rg8[1];
            a1[0] = rg[2]; a1[1] = rg8[2]; a1[2] = rg[3]; a1[3] = rg8[3];
          } else {
            const uint4 q = wq[QT == 4 ? 0 : hb];
            uint32_t g0l, g0h, g1l, g1h, h0l, h0h, h1l, h1h;
            dq8_word(q.x, g0l, g0h);
            dq8_word(q.y, g1l, g1h);
            dq8_word(q.z, h0l, h0h);
            dq8_word(q.w, h1l, h1h);
            a0[0] = g0l; a0[1] = h0l; a0[2] = g0h; a0[3] = h0h;
            a1[0] = g1l; a1[1] = h1l; a1[2] = g1h; a1[3] = h1h;
            if (EXACT8) {
#pragma unroll
              for (int r = 0; r < 4; ++r) {
                a0[r] = sub_f16x2_1152(a0[r]);
                a1[r] = sub_f16x2_1152(a1[r]);
              }
            }
          }
          const float sg = hb ? sc.z : sc.x, sg8 = hb ? sc.w : sc.y;
#pragma unroll
          for (int s = 0; s < NSETS; ++s)
            block_mma<QT>(a0, a1, xb[hb][s], EXACT8 ? 0.0f : cr[hb][s], sg, sg8, acc[m][s]);
        }
      }
      xp += xstride;
      cp += cstride;
    }

    {
      const uint32_t tb = tt * P, te = tb + P;
      if (tb >= c0 && te <= c1) {
        // the whole tile is ours: write it directly
#pragma unroll
        for (int s = 0; s < NSETS; ++s)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) v[m] = acc[m][s][h];
            emit(tt, g + 8 * h, 4 * s + c, v, s);
          }
      } else if (c0 >= tb) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
          for (int s = 0; s < NSETS; ++s) part0[m][s][0] = acc[m][s][0], part0[m][s][1] = acc[m][s][1];
        has0 = true;
      } else {
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
          for (int s = 0; s < NSETS; ++s) part1[m][s][0] = acc[m][s][0], part1[m][s][1] = acc[m][s][1];
        has1 = true;
      }
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int s = 0; s < NSETS; ++s) acc[m][s][0] = acc[m][s][1] = 0.0f;
      // next tile starts at pair 0
      ++tt;
      xp = xf4;
      cp = corr;
      flush_at = min(flush_at + P, n - 1);
    }
  }
  cp_async_wait<0>();

  // ---- tiles shared by several warps of this CTA: the partial sums meet in shared memory
  // (each warp's own ring, free now) and the warp (t - ct0) mod 16 adds them in warp order ----
  {
    float *own = reinterpret_cast<float *>(ring);  // slot sl at own + sl * NMAT * 128
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int s = 0; s < NSETS; ++s) {
        const uint32_t j = 4 * s + c;
        if (has0) {
          own[m * 128 + g * 8 + j] = part0[m][s][0];
          own[m * 128 + (g + 8) * 8 + j] = part0[m][s][1];
        }
        if (has1) {
          own[(NMAT + m) * 128 + g * 8 + j] = part1[m][s][0];
          own[(NMAT + m) * 128 + (g + 8) * 8 + j] = part1[m][s][1];
        }
      }
  }
  __syncthreads();
  for (uint32_t t = ct0 + warp; t < ct1; t += kWarps) {
    const uint32_t fc = (t - ct0) * P, lc = fc + P - 1;  // relative to cbase
    const uint32_t wlo = wowner(ncta, kWarps, fc), whi = wowner(ncta, kWarps, lc);
    if (wlo == whi) continue;  // one warp held the whole tile and wrote it
    float v[4][NMAT];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int m = 0; m < NMAT; ++m) v[q][m] = 0.0f;
    for (uint32_t w = wlo; w <= whi; ++w) {
      if (wstart(ncta, kWarps, w) == wstart(ncta, kWarps, w + 1)) continue;  // empty range
      // the tile is w's last tile only for the first contributor when it started earlier
      const int sl = (w == wlo && wstart(ncta, kWarps, w) < fc) ? 1 : 0;
      const float *r = reinterpret_cast<const float *>(smem + L.ring + w * S * STAGE) + sl * NMAT * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int m = 0; m < NMAT; ++m) v[q][m] += r[m * 128 + lane + 32 * q];
    }
    // lane owns (row, j) = ((lane + 32 q) / 8, lane % 8)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t idx = lane + 32 * q, row = idx >> 3, j = idx & 7;
      emit(t, row, j, v[q], j >= 4 ? NSETS - 1 : 0);
    }
  }

  if (a.epi == kEpiArgmax) {
    // Per batch row j: lane (g, c) tracked rows of batch row 4s + c in best[s].  Reduce over
    // the warp, then over the CTA's warps in shared memory (the rings are free now), publish
    // one candidate per CTA and let the last CTA to arrive merge the CTAs' candidates.
    // better() is a total order (value, then lower index), so the merge order is immaterial.
    float *cv = reinterpret_cast<float *>(smem + L.ring);  // [warp][8]
    uint32_t *ci = reinterpret_cast<uint32_t *>(cv + kWarps * 8);
    auto merge = [](Best &b, float v, uint32_t ix) {
      if (ix != 0xFFFFFFFFu && (b.i == 0xFFFFFFFFu || better(v, ix, b.v, b.i))) b = {v, ix};
    };
    auto warp_merge = [&](Best &b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b.v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, b.i, o);
        merge(b, ov, oi);
      }
    };
    __syncthreads();  // every warp is done with the split-tile records in the rings
    for (uint32_t j = 0; j < batch; ++j) {
      Best b = {-INFINITY, 0xFFFFFFFFu};
#pragma unroll
      for (int s = 0; s < NSETS; ++s)
        if ((uint32_t)(4 * s + c) == j) b = best[s];
      warp_merge(b);
      if (lane == 0) {
        cv[warp * 8 + j] = b.v;
        ci[warp * 8 + j] = b.i;
      }
    }
    __syncthreads();
    if (warp == 0) {
      for (uint32_t j = 0; j < batch; ++j) {
        Best b = {-INFINITY, 0xFFFFFFFFu};
        if (lane < kWarps) b = {cv[lane * 8 + j], ci[lane * 8 + j]};
        warp_merge(b);
        if (lane == 0) {
          a.best_v[(size_t)blockIdx.x * 8 + j] = b.v;
          a.best_i[(size_t)blockIdx.x * 8 + j] = b.i;
        }
      }
      __threadfence();
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atomicAdd(a.done_cnt, 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old + 1 == gridDim.x) {
        __threadfence();
        for (uint32_t j = 0; j < batch; ++j) {
          Best r = {-INFINITY, 0xFFFFFFFFu};
#pragma unroll 8
          for (uint32_t w = lane; w < gridDim.x; w += 32)
            merge(r, __ldcg(a.best_v + (size_t)w * 8 + j), __ldcg(a.best_i + (size_t)w * 8 + j));
          warp_merge(r);
          if (lane == 0) {
            uint32_t tok = r.i == 0xFFFFFFFFu ? 0u : r.i;
            // the CPU rule starts from logits[0]: a NaN there is never beaten
            const bool nan0 = a.row_base[0] == 0 && isnan(__ldcg(a.y[0] + (size_t)j * a.ldy));
            if (nan0) tok = 0;
            a.token[j] = tok;
            if (a.cand) {
              a.cand[j * 4 + 0] = __float_as_uint(r.v);
              a.cand[j * 4 + 1] = r.i;
              a.cand[j * 4 + 2] = nan0 ? 1u : 0u;
              a.cand[j * 4 + 3] = 0u;
            }
          }
        }
        if (lane == 0) *a.done_cnt = 0;
      }
    }
  }
}

}  // namespace
}  // namespace sx
