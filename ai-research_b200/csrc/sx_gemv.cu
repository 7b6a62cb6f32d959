// sx_gemv.cu -- kernels and host launchers of the Q4_0 / Q8_0 GEMV (batch 1..8), fused
// gate+up GeGLU, fused input norms and fused argmax (device code: sx_gemv_dev.cuh).
//
// Replaces gemv_q4.wgsl, gemv_q8.wgsl, fused_mlp_q4.wgsl and argmax.wgsl (reference dispatch:
// src/gpu/kernels.zig:80-95,139-142).
#include "sx_gemv_dev.cuh"

namespace sx {

namespace {

template <int QT, int NMAT, int NSETS, int S>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  gemv_body<QT, NMAT, NSETS, S>(a, smem, true, true, true);
}

template <int QT, int NMAT, int NSETS, int S>
cudaError_t launch_s(const GemvArgs &a, int num_sms, cudaStream_t s, bool pdl) {
  const Layout L = layout_for(a.k, a.batch, NMAT, QT, S);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<QT, NMAT, NSETS, S>, a);
}

template <int QT, int NMAT, int NSETS>
cudaError_t launch_t(const GemvArgs &a, int num_sms, cudaStream_t s, bool pdl) {
  switch (stages_for(a.k, a.batch, NMAT, QT, a.pro != kProNone)) {
    case 8: return launch_s<QT, NMAT, NSETS, 8>(a, num_sms, s, pdl);
    case 6: return launch_s<QT, NMAT, NSETS, 6>(a, num_sms, s, pdl);
    case 4: return launch_s<QT, NMAT, NSETS, 4>(a, num_sms, s, pdl);
    case 2: return launch_s<QT, NMAT, NSETS, 2>(a, num_sms, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int QT, int NMAT, int NSETS>
cudaError_t prepare_t() {
  cudaError_t e[4] = {allow_max_dynamic_smem(gemv_kernel<QT, NMAT, NSETS, 8>),
                      allow_max_dynamic_smem(gemv_kernel<QT, NMAT, NSETS, 6>),
                      allow_max_dynamic_smem(gemv_kernel<QT, NMAT, NSETS, 4>),
                      allow_max_dynamic_smem(gemv_kernel<QT, NMAT, NSETS, 2>)};
  for (cudaError_t x : e)
    if (x != cudaSuccess) return x;
  return cudaSuccess;
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

size_t gemv_smem_bytes(int qt, uint32_t k, uint32_t batch, bool geglu, bool prologue) {
  int st = stages_for(k, batch, geglu ? 2 : 1, qt, prologue);
  return st ? layout_for(k, batch, geglu ? 2 : 1, qt, st).total : (size_t)-1;
}

bool gemv_segments_contiguous(const GemvArgs &a, int qt, int nmat) {
  const uint64_t chunk = qt == 8 ? kQ8ChunkBytes : kQ4ChunkBytes;
  const uint64_t per_tile = (uint64_t)pairs_of(a.k) * chunk;
  for (int m = 0; m < nmat; ++m) {
    uint64_t off = 0;
    for (int s = 0; s < 3; ++s) {
      if (a.tiles[s] == 0) continue;
      if (reinterpret_cast<uintptr_t>(a.w[s][m]) != reinterpret_cast<uintptr_t>(a.w[0][m]) + off)
        return false;
      off += a.tiles[s] * per_tile;
    }
  }
  return true;
}

size_t gemv_part_bytes(int num_sms) { return (size_t)num_sms * kWarps * 2 * 2 * 128 * 4; }
size_t gemv_workers(int num_sms) { return (size_t)num_sms * kWarps; }

cudaError_t launch_gemv(int qt, bool geglu, const GemvArgs &a, int num_sms, cudaStream_t s,
                        bool pdl) {
  bool two = a.batch > 4;
  if (qt == 4) {
    if (geglu)
      return two ? launch_t<4, 2, 2>(a, num_sms, s, pdl) : launch_t<4, 2, 1>(a, num_sms, s, pdl);
    return two ? launch_t<4, 1, 2>(a, num_sms, s, pdl) : launch_t<4, 1, 1>(a, num_sms, s, pdl);
  }
  if (geglu)
    return two ? launch_t<8, 2, 2>(a, num_sms, s, pdl) : launch_t<8, 2, 1>(a, num_sms, s, pdl);
  return two ? launch_t<8, 1, 2>(a, num_sms, s, pdl) : launch_t<8, 1, 1>(a, num_sms, s, pdl);
}

}  // namespace sx
