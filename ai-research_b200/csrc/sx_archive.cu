// sx_archive.cu -- the recall tier on the device: DiffArchive (src/memory.zig:19-151) and the
// per-token integrateMemory (src/model/memory_inject.zig:17-46) as kernels over the model's
// own KV caches.
//
// The reference keeps the archive on the CPU and copies K/V between it and the CPU ring
// (copyKVFromRing / copyKVToRing, memory.zig:70-89); its GPU decode never sees those rows (the
// device caches are separate).  Here the archive lives in device memory next to the caches:
//   1. delta:   diff.zig computeDelta / cosineSimilarity between the token's final normed state
//               and the previous one; below 0.98 similarity the state is appended (unit
//               vector, timestamp, salience = |delta|) -- one CTA;
//   2. capture: the token's K/V rows of every layer copied into the new entry (cache format);
//   3. score:   alpha * dot(query, v_i) + beta * exp(-lambda * (now -| ts_i)) + gamma * sal_i,
//               one warp per entry;
//   4. select:  the reference's selection sort with swaps, min(num_recall, count) rounds, in
//               shared memory (first position of the maximum wins, as its strict `>`), then the
//               access metadata of the selected entries -- one CTA;
//   5. inject:  the selected entries' K/V rows into recall slots A + W + rank of every layer.
// Device state words: {count, write_head, appended, append_index}.
#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {
namespace {

constexpr int kArchThreads = 1024;

SX_DEV float block_sum_1024(float v, float *red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = (threadIdx.x & 31) < (blockDim.x >> 5) ? red[threadIdx.x & 31] : 0.0f;
  return warp_sum(t);
}

__global__ void __launch_bounds__(kArchThreads) archive_delta_kernel(ArchiveArgs a) {
  __shared__ float red[32];
  const float *cur = a.normed;
  float dd = 0.0f, dot = 0.0f, na = 0.0f, nb = 0.0f;
  for (uint32_t i = threadIdx.x; i < a.dim; i += blockDim.x) {
    const float c = cur[i], p = a.prev[i];
    const float d = __fsub_rn(c, p);
    dd = __fadd_rn(dd, __fmul_rn(d, d));
    dot = __fadd_rn(dot, __fmul_rn(p, c));
    na = __fadd_rn(na, __fmul_rn(p, p));
    nb = __fadd_rn(nb, __fmul_rn(c, c));
  }
  dd = block_sum_1024(dd, red);
  dot = block_sum_1024(dot, red);
  na = block_sum_1024(na, red);
  nb = block_sum_1024(nb, red);
  const float denom = __fmul_rn(__fsqrt_rn(na), __fsqrt_rn(nb));
  const float sim = denom < 1e-12f ? 0.0f : __fdiv_rn(dot, denom);
  const bool append = sim < 0.98f;  // memory_inject.zig:10 LANDMARK_SIMILARITY_THRESHOLD
  const uint32_t idx = a.state[1];
  __syncthreads();
  if (append) {
    // appendWithMeta (memory.zig:91-111): the unit-normalised state and its metadata
    const float inv = nb > 1e-12f ? __fdiv_rn(1.0f, __fsqrt_rn(nb)) : 0.0f;
    for (uint32_t i = threadIdx.x; i < a.dim; i += blockDim.x)
      a.vectors[(size_t)idx * a.dim + i] = __fmul_rn(cur[i], inv);
    if (threadIdx.x == 0) {
      a.timestamp[idx] = a.clock;
      a.last_accessed[idx] = a.clock;
      a.access_count[idx] = 0;
      a.salience[idx] = __fsqrt_rn(dd);
      a.state[1] = (idx + 1) % a.capacity;
      if (a.state[0] < a.capacity) a.state[0] += 1;
    }
  }
  if (threadIdx.x == 0) {
    a.state[2] = append ? 1u : 0u;
    a.state[3] = idx;
  }
  // scratch.prev_normed_x = normed_x (after every CTA thread has read prev)
  for (uint32_t i = threadIdx.x; i < a.dim; i += blockDim.x) a.prev[i] = cur[i];
}

// the token's K/V rows (slot a.slot) of layer blockIdx.y into entry state[3] (when appended);
// rows are zero-padded to max_kv like the reference's max_kv_dim rows
__global__ void archive_capture_kernel(ArchiveArgs a) {
  if (a.state[2] == 0) return;
  const uint32_t l = blockIdx.y, idx = a.state[3];
  const ArchiveLayer L = a.layers[l];
  const size_t eb = a.kv_bf16 ? 2 : 4;
  uint8_t *dst = static_cast<uint8_t *>(a.kv) + (((size_t)idx * a.num_layers + l) * 2) * a.max_kv * eb;
  const uint8_t *ks = static_cast<const uint8_t *>(L.k_cache) + (size_t)a.slot * L.kv_dim * eb;
  const uint8_t *vs = static_cast<const uint8_t *>(L.v_cache) + (size_t)a.slot * L.kv_dim * eb;
  const uint32_t row = a.max_kv * (uint32_t)eb;
  for (uint32_t b = blockIdx.x * blockDim.x + threadIdx.x; b < 2 * row; b += gridDim.x * blockDim.x) {
    const uint32_t part = b / row, off = b % row;
    uint8_t v = 0;
    if (off < L.kv_dim * eb) v = part ? vs[off] : ks[off];
    dst[b] = v;
  }
}

// memory.zig:145-151 score, one warp per entry
__global__ void archive_score_kernel(ArchiveArgs a) {
  const uint32_t n = a.state[0];
  const uint32_t lane = threadIdx.x & 31;
  for (uint32_t i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n;
       i += (gridDim.x * blockDim.x) >> 5) {
    const float *row = a.vectors + (size_t)i * a.dim;
    float dot = 0.0f;
    for (uint32_t k = lane; k < a.dim; k += 32) dot = fmaf(a.normed[k], row[k], dot);
    dot = warp_sum(dot);
    if (lane == 0) {
      const uint64_t ts = a.timestamp[i];
      const uint64_t dt = a.clock > ts ? a.clock - ts : 0;  // now -| timestamp
      const float recency = expf(__fmul_rn(-a.lambda, (float)dt));
      a.scores[i] = __fadd_rn(__fadd_rn(__fmul_rn(a.alpha, dot), __fmul_rn(a.beta, recency)),
                              __fmul_rn(a.gamma, a.salience[i]));
    }
  }
}

// memory.zig:113-143 scan: k rounds of "first position of the maximum among [slot, n), swap it
// into slot" over (score, index) pairs in shared memory, then the access metadata
__global__ void __launch_bounds__(kArchThreads) archive_select_kernel(ArchiveArgs a) {
  extern __shared__ uint8_t smem[];
  float *sc = reinterpret_cast<float *>(smem);
  uint32_t *ix = reinterpret_cast<uint32_t *>(sc + a.capacity);
  __shared__ float wv[32];
  __shared__ uint32_t wp[32];
  __shared__ uint32_t win;
  const uint32_t n = a.state[0];
  const uint32_t k = min(a.num_recall, n);
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    sc[i] = a.scores[i];
    ix[i] = i;
  }
  __syncthreads();
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // The reference's round: best = slot, then best = j for every later j with
  // scores[j] > scores[best].  Equivalently: slot itself when its score is NaN (nothing beats
  // a NaN), else the first position of the maximum over the non-NaN scores of [slot, n).
  auto take = [](float &bv, uint32_t &bp, float v, uint32_t p) {
    if (p != 0xFFFFFFFFu && (bp == 0xFFFFFFFFu || v > bv || (v == bv && p < bp))) {
      bv = v;
      bp = p;
    }
  };
  for (uint32_t slot = 0; slot < k; ++slot) {
    float bv = -INFINITY;
    uint32_t bp = 0xFFFFFFFFu;
    for (uint32_t j = slot + threadIdx.x; j < n; j += blockDim.x) {
      const float v = sc[j];
      if (!isnan(v)) take(bv, bp, v, j);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const uint32_t op = __shfl_xor_sync(0xffffffffu, bp, o);
      take(bv, bp, ov, op);
    }
    if (lane == 0) {
      wv[warp] = bv;
      wp[warp] = bp;
    }
    __syncthreads();
    if (warp == 0) {
      bv = -INFINITY;
      bp = 0xFFFFFFFFu;
      if (lane < (blockDim.x >> 5)) take(bv, bp, wv[lane], wp[lane]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t op = __shfl_xor_sync(0xffffffffu, bp, o);
        take(bv, bp, ov, op);
      }
      if (lane == 0) {
        const uint32_t b = (isnan(sc[slot]) || bp == 0xFFFFFFFFu) ? slot : bp;
        const float ts = sc[slot];
        sc[slot] = sc[b];
        sc[b] = ts;
        const uint32_t ti = ix[slot];
        ix[slot] = ix[b];
        ix[b] = ti;
        win = ix[slot];
        a.selected[slot] = win;
        a.sel_ts[slot] = a.timestamp[win];
      }
    }
    __syncthreads();
  }
  if (threadIdx.x < k) {
    const uint32_t m = a.selected[threadIdx.x];
    a.last_accessed[m] = a.clock;
    a.access_count[m] += 1;
  }
  if (threadIdx.x == 0) a.state[4] = k;
}

// copyKVToRing (memory.zig:81-89): entry selected[rank] -> recall slot A + W + rank, layer y
__global__ void archive_inject_kernel(ArchiveArgs a) {
  const uint32_t rank = blockIdx.x, l = blockIdx.y;
  if (rank >= a.state[4]) return;
  const uint32_t m = a.selected[rank];
  const ArchiveLayer L = a.layers[l];
  const size_t eb = a.kv_bf16 ? 2 : 4;
  const uint8_t *src = static_cast<const uint8_t *>(a.kv) + (((size_t)m * a.num_layers + l) * 2) * a.max_kv * eb;
  const uint32_t slot = a.recall_start + rank;
  uint8_t *kd = static_cast<uint8_t *>(L.k_cache) + (size_t)slot * L.kv_dim * eb;
  uint8_t *vd = static_cast<uint8_t *>(L.v_cache) + (size_t)slot * L.kv_dim * eb;
  const uint32_t row = L.kv_dim * (uint32_t)eb;
  for (uint32_t b = threadIdx.x; b < row; b += blockDim.x) {
    kd[b] = src[b];
    vd[b] = src[(size_t)a.max_kv * eb + b];
  }
}

}  // namespace

size_t archive_select_smem(uint32_t capacity) { return (size_t)capacity * 8; }

cudaError_t prepare_archive_kernels() {
  return cudaFuncSetAttribute(archive_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)archive_select_smem(kArchiveMaxCapacity));
}

cudaError_t launch_archive_integrate(const ArchiveArgs &a, cudaStream_t s) {
  archive_delta_kernel<<<1, kArchThreads, 0, s>>>(a);
  archive_capture_kernel<<<dim3(4, a.num_layers), 256, 0, s>>>(a);
  archive_score_kernel<<<148 * 2, 256, 0, s>>>(a);
  archive_select_kernel<<<1, kArchThreads, archive_select_smem(a.capacity), s>>>(a);
  if (a.num_recall > 0) archive_inject_kernel<<<dim3(a.num_recall, a.num_layers), 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace sx
