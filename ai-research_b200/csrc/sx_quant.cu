// sx_quant.cu -- weight ingest: reference Q4_0/Q8_0 block layout -> packed MMA layout,
// a debug unpack for the bit-exact dequant check, and the synthetic-input generators.
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {

namespace {

// Reference Q4_0 block (quant.zig:53-90): word 0 = f32 scale, words 1..4 = nibbles, nibble n
// of word w is element w*8+n.  Packed word for (row, block, lane-column c): nibble j holds
// element 8j+2c and nibble j+4 holds element 8j+2c+1, i.e. byte c of reference word j split
// into its two nibbles.
SX_DEV uint32_t q4_pack_word(const uint32_t *blk, uint32_t c) {
  uint32_t pk = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t byte = (blk[1 + j] >> (8 * c)) & 0xFFu;
    pk |= (byte & 0xFu) << (4 * j);
    pk |= (byte >> 4) << (4 * (j + 4));
  }
  return pk;
}

// Reference Q8_0 block (quant.zig:18-51): element e is byte e%4 of word 1 + e/4.  Packed
// words: w0 = {q(2c), q(2c+1), q(2c+8), q(2c+9)}, w1 = {q(16+2c), .., q(24+2c), q(25+2c)}.
SX_DEV void q8_pack_words(const uint32_t *blk, uint32_t c, uint32_t &w0, uint32_t &w1) {
  uint32_t sh = 16 * (c & 1), base = 1 + (c >> 1);
  auto half = [&](int word) { return (blk[base + word] >> sh) & 0xFFFFu; };
  w0 = half(0) | (half(2) << 16);
  w1 = half(4) | (half(6) << 16);
}

template <int QT>
__global__ void repack_kernel(const uint32_t *ref, uint8_t *out, uint32_t m, uint32_t k) {
  const uint32_t T = tiles_of(m), P = pairs_of(k), nb = k / 32;
  constexpr uint32_t WPB = QT == 4 ? 5 : 9;
  constexpr int CB = QT == 4 ? kQ4ChunkBytes : kQ8ChunkBytes;
  const uint64_t total = (uint64_t)T * P * 32;
  for (uint64_t it = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; it < total;
       it += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t lane = it & 31;
    uint64_t tp = it >> 5;
    uint32_t t = (uint32_t)(tp / P), p = (uint32_t)(tp % P);
    uint32_t g = lane >> 2, c = lane & 3;
    uint32_t rows[2] = {t * 16 + g, t * 16 + g + 8};
    uint8_t *ch = out + tp * CB;
    float sc[4];
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      uint32_t b = 2 * p + hb;
      uint32_t wv[2][2];
#pragma unroll
      for (int ri = 0; ri < 2; ++ri) {
        wv[ri][0] = wv[ri][1] = 0;
        float s = 0.0f;
        if (rows[ri] < m && b < nb) {
          const uint32_t *blk = ref + ((size_t)rows[ri] * nb + b) * WPB;
          s = u2f(blk[0]);
          if (QT == 4)
            wv[ri][0] = q4_pack_word(blk, c);
          else
            q8_pack_words(blk, c, wv[ri][0], wv[ri][1]);
        }
        sc[hb * 2 + ri] = s;
      }
      if (QT == 4) {
        uint32_t *dst = reinterpret_cast<uint32_t *>(ch + lane * 16);
        dst[hb * 2 + 0] = wv[0][0];
        dst[hb * 2 + 1] = wv[1][0];
      } else {
        uint4 v = make_uint4(wv[0][0], wv[0][1], wv[1][0], wv[1][1]);
        *reinterpret_cast<uint4 *>(ch + hb * 512 + lane * 16) = v;
      }
    }
    if (c == 0) {
      float4 s4 = make_float4(sc[0], sc[1], sc[2], sc[3]);
      *reinterpret_cast<float4 *>(ch + (QT == 4 ? 512 : 1024) + g * 16) = s4;
    }
  }
}

// Inverse of the Q4 packing, producing dequantised f32 (nib - 8) * d in reference element
// order; used only to prove the packed layout loses nothing.
__global__ void unpack_q4_kernel(const uint8_t *packed, float *out, uint32_t m, uint32_t k) {
  const uint32_t T = tiles_of(m), P = pairs_of(k), nb = k / 32;
  const uint64_t total = (uint64_t)T * P * 32;
  for (uint64_t it = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; it < total;
       it += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t lane = it & 31;
    uint64_t tp = it >> 5;
    uint32_t t = (uint32_t)(tp / P), p = (uint32_t)(tp % P);
    uint32_t g = lane >> 2, c = lane & 3;
    const uint8_t *ch = packed + tp * kQ4ChunkBytes;
    const uint32_t *wd = reinterpret_cast<const uint32_t *>(ch + lane * 16);
    const float *sc = reinterpret_cast<const float *>(ch + 512 + g * 16);
#pragma unroll
    for (int hb = 0; hb < 2; ++hb)
#pragma unroll
      for (int ri = 0; ri < 2; ++ri) {
        uint32_t row = t * 16 + g + 8 * ri, b = 2 * p + hb;
        if (row >= m || b >= nb) continue;
        uint32_t w = wd[hb * 2 + ri];
        float d = sc[hb * 2 + ri];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t nib = (w >> (4 * (j + 4 * h))) & 0xFu;
            uint32_t e = 8 * j + 2 * c + h;
            out[(size_t)row * k + b * 32 + e] = __fmul_rn((float)nib - 8.0f, d);
          }
      }
  }
}

// Reference-layout synthetic blocks (BASELINE distributions; identical bits to the CPU
// checker's generator).
template <int QT>
__global__ void synth_ref_kernel(uint32_t *ref, uint32_t row0, uint32_t rows, uint32_t k,
                                 uint64_t seed, uint64_t stream, uint32_t blk0, uint32_t nbg) {
  const uint32_t nb = k / 32;
  constexpr uint32_t WPB = QT == 4 ? 5 : 9;
  constexpr uint32_t STRIDE = QT == 4 ? 8 : 16;
  const uint64_t total = (uint64_t)rows * nb;
  for (uint64_t it = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; it < total;
       it += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = it / nb, b = it % nb;
    uint64_t idx = (row0 + r) * nbg + blk0 + b;
    uint32_t *blk = ref + it * WPB;
    blk[0] = f2u(synth_scale(seed, stream, idx * STRIDE));
#pragma unroll
    for (uint32_t j = 1; j < WPB; ++j) blk[j] = (uint32_t)hash3(seed, stream, idx * STRIDE + j);
  }
}

__global__ void synth_gain_kernel(float *dst, uint32_t n, uint64_t seed, uint64_t stream) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[i] = bf16_bits_to_f32(bf16_bits_rne(fmaf(0.1f, synth_normal(seed, stream, i), 1.0f)));
}

// Synthetic past K/V rows (one thread per [slot][kv_head] row); sequential fmaf chain so the
// unit-RMS normalisation of V matches the CPU generator bit for bit.
__global__ void fill_kv_kernel(void *k_cache, void *v_cache, int kv_bf16, uint32_t rows,
                               uint32_t D, float eps, uint64_t seed, uint32_t layer,
                               uint32_t heads, uint32_t head0, uint32_t heads_global) {
  const uint64_t ks = 0x10000ull + 2ull * layer, vs = ks + 1;
  for (uint32_t lrow = blockIdx.x * blockDim.x + threadIdx.x; lrow < rows;
       lrow += gridDim.x * blockDim.x) {
    // values of row (slot, head0 + h) of the whole cache, stored at local row lrow
    const uint64_t row = (uint64_t)(lrow / heads) * heads_global + head0 + lrow % heads;
    float ss = 0.0f;
    for (uint32_t d = 0; d < D; ++d) {
      float vz = synth_normal(seed, vs, (uint64_t)row * D + d);
      ss = fmaf(vz, vz, ss);
    }
    float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
    for (uint32_t d = 0; d < D; ++d) {
      const uint64_t i = row * D + d, o = (uint64_t)lrow * D + d;
      float kz = bf16_bits_to_f32(bf16_bits_rne(synth_normal(seed, ks, i)));
      float vz = bf16_bits_to_f32(bf16_bits_rne(__fmul_rn(synth_normal(seed, vs, i), r)));
      if (kv_bf16) {
        reinterpret_cast<uint16_t *>(k_cache)[o] = bf16_bits_rne(kz);
        reinterpret_cast<uint16_t *>(v_cache)[o] = bf16_bits_rne(vz);
      } else {
        reinterpret_cast<float *>(k_cache)[o] = kz;
        reinterpret_cast<float *>(v_cache)[o] = vz;
      }
    }
  }
}

// quantizeRowQ4_0 / quantizeRowQ8_0 (quant.zig:18-90) on the device, one thread per 32-value
// block of a row-major bf16 matrix, the reference block layout out: f32 d = amax / 7 (Q8:
// amax / 127), then q = round_half_away(v * (7 / amax)) clamped to [-8, 7] and stored as
// nibble n = q + 8 of word w for element 8 w + n (Q8: clamp [-128, 127], byte k of word w for
// element 4 w + k).  IEEE-rounded division and product, C roundf: the words equal the CPU
// quantiser's bit for bit.
template <int QT>
__global__ void quantize_kernel(const uint16_t *src, uint32_t *dst, uint64_t nblocks) {
  constexpr float kMax = QT == 4 ? 7.0f : 127.0f;
  constexpr int kWords = QT == 4 ? 5 : 9;
  for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks;
       b += (uint64_t)gridDim.x * blockDim.x) {
    const uint4 *s4 = reinterpret_cast<const uint4 *>(src + b * 32);
    float v[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = s4[i];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
        v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float a = fabsf(v[i]);
      if (a > amax) amax = a;
    }
    const float id = amax > 0.0f ? __fdiv_rn(kMax, amax) : 0.0f;
    uint32_t out[kWords];
    out[0] = __float_as_uint(__fdiv_rn(amax, kMax));
#pragma unroll
    for (int w = 0; w < kWords - 1; ++w) {
      uint32_t word = 0;
#pragma unroll
      for (int k = 0; k < (QT == 4 ? 8 : 4); ++k) {
        int q = (int)roundf(__fmul_rn(v[w * (QT == 4 ? 8 : 4) + k], id));
        if (QT == 4) {
          q = q < -8 ? -8 : (q > 7 ? 7 : q);
          word |= (uint32_t)(q + 8) << (4 * k);
        } else {
          q = q < -128 ? -128 : (q > 127 ? 127 : q);
          word |= (uint32_t)(uint8_t)(int8_t)q << (8 * k);
        }
      }
      out[1 + w] = word;
    }
    uint32_t *o = dst + b * kWords;
#pragma unroll
    for (int w = 0; w < kWords; ++w) o[w] = out[w];
  }
}

uint32_t grid_for(uint64_t items, uint32_t threads) {
  uint64_t g = (items + threads - 1) / threads;
  if (g > 65535u * 16) g = 65535u * 16;
  return g ? (uint32_t)g : 1u;
}

}  // namespace

cudaError_t launch_repack(int qt, const uint32_t *ref, void *packed, uint32_t m, uint32_t k,
                          cudaStream_t s) {
  uint64_t items = (uint64_t)tiles_of(m) * pairs_of(k) * 32;
  if (qt == 4)
    repack_kernel<4><<<grid_for(items, 256), 256, 0, s>>>(ref, (uint8_t *)packed, m, k);
  else
    repack_kernel<8><<<grid_for(items, 256), 256, 0, s>>>(ref, (uint8_t *)packed, m, k);
  return cudaGetLastError();
}

cudaError_t launch_unpack_q4(const void *packed, float *out, uint32_t m, uint32_t k,
                             cudaStream_t s) {
  uint64_t items = (uint64_t)tiles_of(m) * pairs_of(k) * 32;
  unpack_q4_kernel<<<grid_for(items, 256), 256, 0, s>>>((const uint8_t *)packed, out, m, k);
  return cudaGetLastError();
}

cudaError_t launch_synth_ref(int qt, uint32_t *ref, uint32_t row0, uint32_t rows, uint32_t k,
                             uint64_t seed, uint64_t stream_id, cudaStream_t s, uint32_t blk0,
                             uint32_t nb_global) {
  uint64_t items = (uint64_t)rows * (k / 32);
  const uint32_t nbg = nb_global ? nb_global : k / 32;
  if (qt == 4)
    synth_ref_kernel<4><<<grid_for(items, 256), 256, 0, s>>>(ref, row0, rows, k, seed, stream_id,
                                                             blk0, nbg);
  else
    synth_ref_kernel<8><<<grid_for(items, 256), 256, 0, s>>>(ref, row0, rows, k, seed, stream_id,
                                                             blk0, nbg);
  return cudaGetLastError();
}

cudaError_t launch_synth_gain(float *dst, uint32_t n, uint64_t seed, uint64_t stream_id,
                              cudaStream_t s) {
  synth_gain_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, n, seed, stream_id);
  return cudaGetLastError();
}

cudaError_t launch_fill_kv(void *k_cache, void *v_cache, int kv_bf16, uint32_t rows,
                           uint32_t head_dim, float eps, uint64_t seed, uint32_t layer,
                           cudaStream_t s, uint32_t heads, uint32_t head0,
                           uint32_t heads_global) {
  fill_kv_kernel<<<grid_for(rows, 128), 128, 0, s>>>(k_cache, v_cache, kv_bf16, rows, head_dim,
                                                     eps, seed, layer, heads, head0, heads_global);
  return cudaGetLastError();
}

cudaError_t launch_quantize(int qt, const void *bf16, uint32_t *ref, uint64_t nblocks,
                            cudaStream_t s) {
  if (nblocks == 0) return cudaSuccess;
  if (qt == 4)
    quantize_kernel<4><<<grid_for(nblocks, 256), 256, 0, s>>>(static_cast<const uint16_t *>(bf16),
                                                               ref, nblocks);
  else
    quantize_kernel<8><<<grid_for(nblocks, 256), 256, 0, s>>>(static_cast<const uint16_t *>(bf16),
                                                               ref, nblocks);
  return cudaGetLastError();
}

}  // namespace sx
