// sx_gemv.cu -- Q4_0 / Q8_0 GEMV (batch 1..8) and the fused gate+up GeGLU for sm_100a.
//
// Replaces gemv_q4.wgsl, gemv_q8.wgsl and fused_mlp_q4.wgsl (reference dispatch:
// src/gpu/kernels.zig:80-95).  Semantics: y[r] = sum_b sum_e ((q - 8) * d_b) * x[e] for Q4,
// (q * d_b) * x[e] for Q8; fused: y[r] = gelu_tanh(Wg[r].x) * (Wu[r].x) (kernels.zig:94-115).
//
// Design.  Decode GEMVs are HBM-bound (20 B per 32 weights), so the kernel must spend few
// instructions per weight.  Each warp streams 16-row x 64-column chunks of the packed
// matrix with 128-bit no-L1-allocate loads and dequantises nibbles straight into
// mma.m16n8k16 A fragments with one shift + one LOP3 per two weights (bf16 value 8 + q/2,
// exact).  The activation enters as the B operand split into bf16 hi + lo parts (16-bit
// significand, ~2^-17 relative), one column pair per batch row, so the tensor core does the
// 32-element block dot products; the per-block f32 scale and the constant offset are applied
// on the f32 accumulator:  sum_e (q_e - 8) x_e = 2 * (D - 12 * sum_e x_e).
// Q8 uses f16 values 1024 + (q + 128) (exact) and a per-vector power-of-two prescale of x.
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;

SX_HD uint32_t nv_of(uint32_t batch) {
  return batch <= 1 ? 2u : batch <= 2 ? 4u : batch <= 4 ? 8u : 16u;
}

template <int QT>
struct QTraits;
template <>
struct QTraits<4> {
  static constexpr int kChunk = kQ4ChunkBytes;
  static constexpr int kScaleOff = 512;
  static constexpr float kCorr = 12.0f;
};
template <>
struct QTraits<8> {
  static constexpr int kChunk = kQ8ChunkBytes;
  static constexpr int kScaleOff = 1024;
  static constexpr float kCorr = 1152.0f;
};

struct SmemLayout {
  uint32_t xfrag_bytes, corr_off, red_off, scale_off, total;
};

SX_HD SmemLayout smem_layout(uint32_t k, uint32_t batch, int nmat) {
  SmemLayout L;
  uint32_t nblk = 2 * pairs_of(k);
  L.xfrag_bytes = nblk * nv_of(batch) * 4 * 16;
  L.corr_off = L.xfrag_bytes;
  L.red_off = L.corr_off + nblk * 8 * 4;
  L.scale_off = L.red_off + kGemvWarps * nmat * 16 * 8 * 4;
  L.total = L.scale_off + 8 * 4;
  return L;
}

SX_DEV float gelu_tanh_dev(float x) {
  // kernels.zig:94-97, same operation order
  float x3 = __fmul_rn(__fmul_rn(x, x), x);
  float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// Activation -> B fragments.  Item (blk, j, c, jj) converts elements 32*blk + 8*jj + 2c,+1
// of batch row j into the hi/lo pair words and reduces the block sum for the offset term.
template <int QT>
SX_DEV void stage_x(const GemvArgs &a, uint8_t *smem, const SmemLayout &L) {
  uint32_t *xf = reinterpret_cast<uint32_t *>(smem);
  float *corr = reinterpret_cast<float *>(smem + L.corr_off);
  float *xscale = reinterpret_cast<float *>(smem + L.scale_off);
  int *xexp = reinterpret_cast<int *>(smem + L.red_off);  // red area is free here
  const uint32_t nb = a.k / 32, nblk = 2 * pairs_of(a.k), nv = nv_of(a.batch);
  const int tid = threadIdx.x;

  if (QT == 8) {
    // Per-row power-of-two prescale so that the f16 hi/lo split neither overflows nor
    // loses precision: max |x| * 2^e < 2^15.
    for (uint32_t j = 0; j < a.batch; ++j) {
      float mx = 0.0f;
      for (uint32_t i = tid; i < a.k; i += blockDim.x) mx = fmaxf(mx, fabsf(a.x[j * a.ldx + i]));
      mx = warp_max(mx);
      __syncthreads();
      if ((tid & 31) == 0) xscale[tid >> 5] = mx;
      __syncthreads();
      if (tid == 0) {
        float m = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, xscale[w]);
        int e = 0;
        if (m > 0.0f && isfinite(m)) {
          int ex;
          frexpf(m, &ex);
          e = 15 - ex;
          e = e > 100 ? 100 : (e < -100 ? -100 : e);
        }
        xexp[j] = e;
      }
      __syncthreads();
    }
    if (tid < (int)a.batch) xscale[tid] = ldexpf(1.0f, -xexp[tid]);
  } else {
    if (tid < (int)a.batch) xscale[tid] = 2.0f;
  }

  const uint32_t items = nblk * a.batch * 16;
  const uint32_t items_pad = (items + 31) & ~31u;
  for (uint32_t it = tid; it < items_pad; it += blockDim.x) {
    float part = 0.0f;
    uint32_t c = it & 3, jj = (it >> 2) & 3, rest = it >> 4;
    uint32_t j = rest % a.batch, blk = rest / a.batch;
    if (it < items) {
      uint32_t e0 = blk * 32 + jj * 8 + 2 * c;
      float x0 = 0.0f, x1 = 0.0f;
      if (blk < nb) {
        x0 = a.x[j * a.ldx + e0];
        x1 = a.x[j * a.ldx + e0 + 1];
      }
      uint32_t hw, lw;
      if (QT == 4) {
        __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
        float r0 = __fsub_rn(x0, __bfloat162float(h0)), r1 = __fsub_rn(x1, __bfloat162float(h1));
        __nv_bfloat16 l0 = __float2bfloat16_rn(r0), l1 = __float2bfloat16_rn(r1);
        hw = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        lw = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        part = (__bfloat162float(h0) + __bfloat162float(l0)) +
               (__bfloat162float(h1) + __bfloat162float(l1));
      } else {
        int e = xexp[j];
        x0 = ldexpf(x0, e);
        x1 = ldexpf(x1, e);
        __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
        float r0 = __fsub_rn(x0, __half2float(h0)), r1 = __fsub_rn(x1, __half2float(h1));
        __half l0 = __float2half_rn(r0), l1 = __float2half_rn(r1);
        hw = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        lw = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        part = (__half2float(h0) + __half2float(l0)) + (__half2float(h1) + __half2float(l1));
      }
      // uint4 index (blk * nv + v) * 4 + c, word jj
      xf[(((blk * nv + 2 * j) * 4 + c) << 2) + jj] = hw;
      xf[(((blk * nv + 2 * j + 1) * 4 + c) << 2) + jj] = lw;
    }
    part += __shfl_xor_sync(0xffffffffu, part, 8);
    part += __shfl_xor_sync(0xffffffffu, part, 4);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    if (it < items && (it & 15) == 0) corr[blk * 8 + j] = QTraits<QT>::kCorr * part;
  }
  __syncthreads();
}

// One 32-element block of one 16-row tile against the staged activation.
template <int QT, int NSETS>
SX_DEV void block_mma(const uint32_t (&a0)[4], const uint32_t (&a1)[4], const uint4 *xf4,
                      const float *corr, uint32_t blk, uint32_t nv, uint32_t batch, int g, int c,
                      float sg, float sg8, float (&acc)[NSETS][2]) {
#pragma unroll
  for (int s = 0; s < NSETS; ++s) {
    uint32_t v = 8 * s + g;
    uint4 xb = make_uint4(0, 0, 0, 0);
    if (v < 2 * batch) xb = xf4[(blk * nv + v) * 4 + c];
    uint32_t j = 4 * s + c;
    float cr = j < batch ? corr[blk * 8 + j] : 0.0f;
    float d[4] = {-cr, 0.0f, -cr, 0.0f};
    if (QT == 4) {
      mma_bf16_16816(d, a0, xb.x, xb.y);
      mma_bf16_16816(d, a1, xb.z, xb.w);
    } else {
      mma_f16_16816(d, a0, xb.x, xb.y);
      mma_f16_16816(d, a1, xb.z, xb.w);
    }
    acc[s][0] = fmaf(sg, d[0] + d[1], acc[s][0]);
    acc[s][1] = fmaf(sg8, d[2] + d[3], acc[s][1]);
  }
}

template <int QT, int NMAT, int NSETS>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const SmemLayout L = smem_layout(a.k, a.batch, NMAT);
  stage_x<QT>(a, smem, L);

  const uint4 *xf4 = reinterpret_cast<const uint4 *>(smem);
  const float *corr = reinterpret_cast<const float *>(smem + L.corr_off);
  float *red = reinterpret_cast<float *>(smem + L.red_off);
  const float *xscale = reinterpret_cast<const float *>(smem + L.scale_off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const uint32_t T = tiles_of(a.m), P = pairs_of(a.k), nv = nv_of(a.batch);
  constexpr int CB = QTraits<QT>::kChunk;
  constexpr int SO = QTraits<QT>::kScaleOff;
  constexpr int U = NMAT == 1 ? 4 : 2;
  const uint8_t *wbase[2] = {static_cast<const uint8_t *>(a.w0),
                             static_cast<const uint8_t *>(NMAT == 2 ? a.w1 : a.w0)};

  for (uint32_t t = blockIdx.x; t < T; t += gridDim.x) {
    float acc[NMAT][NSETS][2];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int s = 0; s < NSETS; ++s) acc[m][s][0] = acc[m][s][1] = 0.0f;

    for (uint32_t p0 = warp; p0 < P; p0 += kGemvWarps * U) {
      uint4 wq[U][NMAT][QT == 4 ? 1 : 2];
      float4 sc[U][NMAT];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        uint32_t p = p0 + u * kGemvWarps;
        if (p < P) {
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const uint8_t *ch = wbase[m] + ((size_t)t * P + p) * CB;
            wq[u][m][0] = ldg_stream(ch + lane * 16);
            if (QT == 8) wq[u][m][QT == 4 ? 0 : 1] = ldg_stream(ch + 512 + lane * 16);
            sc[u][m] = __ldg(reinterpret_cast<const float4 *>(ch + SO + g * 16));
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        uint32_t p = p0 + u * kGemvWarps;
        if (p >= P) break;
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            uint32_t a0[4], a1[4];
            if (QT == 4) {
              uint32_t rg[4], rg8[4];
              dq4_word(hb ? wq[u][m][0].z : wq[u][m][0].x, rg);
              dq4_word(hb ? wq[u][m][0].w : wq[u][m][0].y, rg8);
              a0[0] = rg[0]; a0[1] = rg8[0]; a0[2] = rg[1]; a0[3] = rg8[1];
              a1[0] = rg[2]; a1[1] = rg8[2]; a1[2] = rg[3]; a1[3] = rg8[3];
            } else {
              const uint4 q = wq[u][m][QT == 4 ? 0 : hb];
              uint32_t g0l, g0h, g1l, g1h, h0l, h0h, h1l, h1h;
              dq8_word(q.x, g0l, g0h);
              dq8_word(q.y, g1l, g1h);
              dq8_word(q.z, h0l, h0h);
              dq8_word(q.w, h1l, h1h);
              a0[0] = g0l; a0[1] = h0l; a0[2] = g0h; a0[3] = h0h;
              a1[0] = g1l; a1[1] = h1l; a1[2] = g1h; a1[3] = h1h;
            }
            float sg = hb ? sc[u][m].z : sc[u][m].x;
            float sg8 = hb ? sc[u][m].w : sc[u][m].y;
            block_mma<QT, NSETS>(a0, a1, xf4, corr, 2 * p + hb, nv, a.batch, g, c, sg, sg8,
                                 acc[m]);
          }
        }
      }
    }

    // cross-warp reduction: red[warp][m][row][batch]
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int s = 0; s < NSETS; ++s) {
        uint32_t j = 4 * s + c;
        if (j < a.batch) {
          red[((warp * NMAT + m) * 16 + g) * 8 + j] = acc[m][s][0];
          red[((warp * NMAT + m) * 16 + g + 8) * 8 + j] = acc[m][s][1];
        }
      }
    __syncthreads();
    for (uint32_t i = tid; i < 16 * a.batch; i += blockDim.x) {
      uint32_t row = i & 15, j = i >> 4;
      float v[NMAT];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) {
        float s = 0.0f;
        for (int w = 0; w < kGemvWarps; ++w) s += red[((w * NMAT + m) * 16 + row) * 8 + j];
        v[m] = s * xscale[j];
      }
      uint32_t r = t * 16 + row;
      if (r < a.m) {
        float out = v[0];
        if (NMAT == 2) out = __fmul_rn(gelu_tanh_dev(v[0]), v[NMAT - 1]);
        a.y[(size_t)j * a.ldy + r] = out;
      }
    }
    __syncthreads();
  }
}

template <int QT, int NMAT, int NSETS>
cudaError_t launch_t(const GemvArgs &a, int num_sms, cudaStream_t s) {
  const SmemLayout L = smem_layout(a.k, a.batch, NMAT);
  auto kern = gemv_kernel<QT, NMAT, NSETS>;
  uint32_t T = tiles_of(a.m);
  uint32_t cap = (uint32_t)num_sms * 8;
  uint32_t grid = T < cap ? T : cap;
  kern<<<grid, kGemvThreads, L.total, s>>>(a);
  return cudaGetLastError();
}

template <int QT, int NMAT, int NSETS>
cudaError_t prepare_t() {
  return cudaFuncSetAttribute(gemv_kernel<QT, NMAT, NSETS>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

}  // namespace

cudaError_t prepare_gemv_kernels() {
  cudaError_t e = cudaSuccess;
  cudaError_t r[8] = {prepare_t<4, 1, 1>(), prepare_t<4, 1, 2>(), prepare_t<4, 2, 1>(),
                      prepare_t<4, 2, 2>(), prepare_t<8, 1, 1>(), prepare_t<8, 1, 2>(),
                      prepare_t<8, 2, 1>(), prepare_t<8, 2, 2>()};
  for (cudaError_t x : r)
    if (x != cudaSuccess) e = x;
  return e;
}

size_t gemv_smem_bytes(int qt, uint32_t k, uint32_t batch) {
  (void)qt;
  return smem_layout(k, batch, 2).total;
}

cudaError_t launch_gemv(int qt, bool geglu, const GemvArgs &a, int num_sms, cudaStream_t s) {
  bool two = a.batch > 4;
  if (qt == 4) {
    if (geglu) return two ? launch_t<4, 2, 2>(a, num_sms, s) : launch_t<4, 2, 1>(a, num_sms, s);
    return two ? launch_t<4, 1, 2>(a, num_sms, s) : launch_t<4, 1, 1>(a, num_sms, s);
  }
  if (geglu) return two ? launch_t<8, 2, 2>(a, num_sms, s) : launch_t<8, 2, 1>(a, num_sms, s);
  return two ? launch_t<8, 1, 2>(a, num_sms, s) : launch_t<8, 1, 1>(a, num_sms, s);
}

}  // namespace sx
