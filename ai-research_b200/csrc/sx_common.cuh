// sx_common.cuh -- shared device helpers for the sm_100a decode kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SX_DEV __device__ __forceinline__
#define SX_HD __host__ __device__ __forceinline__

namespace sx {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// Device error word.  Every bounded wait in a kernel writes a nonzero code here
// instead of hanging; the host reads it back after a submit.
enum DeviceError : uint32_t {
  kDevOk = 0,
  kDevWaitTimeout = 1,
  kDevBadParams = 2,
  kDevBadSlot = 3,
  kDevBarrierTimeout = 4,
};

SX_DEV void raise_error(uint32_t *err, uint32_t code) {
  if (err) atomicCAS(err, 0u, code);
}

// ---------------------------------------------------------------------------
// bit casts
SX_HD float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}
SX_HD uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
  return u;
#endif
}

// bf16 round-to-nearest-even exactly as tensor.zig:7-13 (integer formulation).
SX_HD uint16_t bf16_bits_rne(float v) {
  uint32_t u = f2u(v);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
SX_HD float bf16_bits_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

// ---------------------------------------------------------------------------
// Synthetic-input generator.  Integer-only mixing so that host, device and the CPU
// checker produce identical bits (splitmix64 finaliser; Irwin-Hall(4) normal).
SX_HD uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
SX_HD uint64_t hash3(uint64_t seed, uint64_t stream, uint64_t idx) {
  return mix64(mix64(seed ^ (stream * 0xD1B54A32D192ED03ull)) + idx);
}
SX_HD float synth_normal(uint64_t seed, uint64_t stream, uint64_t idx) {
  uint64_t h = hash3(seed, stream, idx);
  int32_t s = (int32_t)((h & 0xFFFFu) + ((h >> 16) & 0xFFFFu) + ((h >> 32) & 0xFFFFu) +
                        ((h >> 48) & 0xFFFFu)) -
              131070;
#ifdef __CUDA_ARCH__
  return __fdiv_rn((float)s, 37837.23f);
#else
  return (float)s / 37837.23f;
#endif
}
// f32 -> f16 -> f32 round trip, round to nearest even, subnormals kept.
SX_HD float f16_round(float v) {
  uint32_t x = f2u(v);
  uint32_t sign = x & 0x80000000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return v;
  if (ax >= 0x477FF000u) return u2f(sign | 0x7F800000u);
  if (ax < 0x38800000u) {
#ifdef __CUDA_ARCH__
    float a = __fmul_rn(u2f(ax), 16777216.0f);
    float r = __fmul_rn(rintf(a), 1.0f / 16777216.0f);
#else
    float a = u2f(ax) * 16777216.0f;
    float r = __builtin_rintf(a) * (1.0f / 16777216.0f);
#endif
    return u2f(sign | f2u(r));
  }
  uint32_t lsb = (ax >> 13) & 1u;
  ax = (ax + 0xFFFu + lsb) & ~0x1FFFu;
  return u2f(sign | ax);
}
SX_HD float synth_scale(uint64_t seed, uint64_t stream, uint64_t idx) {
  float z = synth_normal(seed, stream, idx);
#ifdef __CUDA_ARCH__
  return f16_round(__fmul_rn(fabsf(z), 0.02f));
#else
  return f16_round((z < 0 ? -z : z) * 0.02f);
#endif
}

// ---------------------------------------------------------------------------
// Packed weight formats (device layout produced by the repack kernels).
//
// A matrix of M rows x K columns is cut into row tiles of 16 and K block pairs of 64
// (two 32-element quant blocks).  Chunk (tile t, pair p) is one contiguous record:
//   Q4: 512 B nibbles + 128 B scales = 640 B   (= 2 blocks x 16 rows x 20 B)
//   Q8: 2 x 512 B int8 + 128 B scales = 1152 B (= 2 blocks x 16 rows x 36 B)
// Lane l = 4g + c of a warp owns the 16-byte piece l of each 512-byte sub-record; it
// holds exactly the mma.m16n8k16 A-fragment bytes of rows g and g+8 for k-slots
// {2c, 2c+1, 2c+8, 2c+9} of both 16-wide halves of a block.  Scales: g-th 16 B =
// {s(g, 2p), s(g+8, 2p), s(g, 2p+1), s(g+8, 2p+1)}.  The repack is a permutation of the
// reference's nibbles/bytes and f32 scales: dequantised values are bit-identical.
constexpr int kTileRows = 16;
constexpr int kQ4ChunkBytes = 640;
constexpr int kQ8ChunkBytes = 1152;

SX_HD uint32_t tiles_of(uint32_t m) { return (m + kTileRows - 1) / kTileRows; }
SX_HD uint32_t pairs_of(uint32_t k) { return (k / 32 + 1) / 2; }

// ---------------------------------------------------------------------------
// mma.sync m16n8k16 (f32 accumulate).  Used as a 16-row dot-product engine for the
// batch-1..8 GEMV: the weights dequantise straight into A fragments.
SX_DEV void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
SX_DEV void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

SX_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// (a & b) | c in one LOP3 (truth table 0xEA); b and c are registers, so a constant mask and
// magic number are materialised once instead of costing a second logic op per use
SX_DEV uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// Q4: the eight nibbles of one packed word -> four bf16x2 A-fragment registers holding
// 8 + q/2 (exact): register j holds nibble slot j (low half) and slot j + 4 (high half) in
// mantissa bits 3..6; one shift and one LOP3 per register.
SX_DEV void dq4_word(uint32_t u, uint32_t (&r)[4]) {
  const uint32_t m = 0x00780078u, e = 0x41004100u;
  r[0] = and_or(u << 3, m, e);
  r[1] = and_or(u >> 1, m, e);
  r[2] = and_or(u >> 5, m, e);
  r[3] = and_or(u >> 9, m, e);
}
// Q8: four int8 of one packed word -> two f16x2 holding 1024 + (q + 128) (exact).
SX_DEV void dq8_word(uint32_t u, uint32_t &lo, uint32_t &hi) {
  uint32_t v = u ^ 0x80808080u;
  lo = prmt(v, 0x64646464u, 0x4140u);  // bytes 0,1 -> (1024+b0, 1024+b1)
  hi = prmt(v, 0x64646464u, 0x4342u);  // bytes 2,3
}

// f16x2 (1152 + q0, 1152 + q1) -> (q0, q1), exact (both are f16 integers)
SX_DEV uint32_t sub_f16x2_1152(uint32_t v) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(v), "r"(0x64806480u));
  return r;
}

// ---------------------------------------------------------------------------
// loads
SX_DEV uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

SX_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
SX_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` must hold >= 32 floats.  All threads get the result.
SX_DEV float block_sum(float v, float *red) {
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  t = warp_sum(t);
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, non-tensor form).  Waits are bounded: a wait that does
// not complete within ~1 s of SM clock returns false instead of spinning forever.
SX_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
SX_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
SX_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
// cp.async.bulk.prefetch.L2: bring [p, p + bytes) into L2 without a destination (16-byte
// aligned address, size a multiple of 16)
SX_DEV void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}
SX_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
SX_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
SX_DEV bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(phase)
      : "memory");
  return ok != 0;
}
constexpr long long kWaitCycles = 2000000000ll;  // ~1 s at 1.9 GHz
SX_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, phase))
    if (clock64() - t0 > kWaitCycles) return false;
  return true;
}
// global -> shared bulk copy completing on an mbarrier (16-B aligned, size % 16 == 0)
SX_DEV void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Ampere-style asynchronous 16-byte copies (LDGSTS), L1-bypassing, grouped per thread.
SX_DEV void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
// predicated form: no copy (and no read of src) when p is false
SX_DEV void cp_async16_if(uint32_t dst, const void *src, bool p) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.b32 q, %2, 0;\n"
      " @q cp.async.cg.shared.global [%0], [%1], 16;\n}\n" ::"r"(dst),
      "l"(src), "r"((uint32_t)p)
      : "memory");
}
// L2 eviction priority for data read once per token (weights, past K/V rows): such lines are
// replaced first, so the streams do not push activations, norm gains and code out of L2.
SX_DEV uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
SX_DEV void cp_async16_if_ef(uint32_t dst, const void *src, bool p, uint64_t pol) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.b32 q, %2, 0;\n"
      " @q cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %3;\n}\n" ::"r"(dst),
      "l"(src), "r"((uint32_t)p), "l"(pol)
      : "memory");
}
SX_DEV void bulk_g2s_ef(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
      "[%3], %4;\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
SX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
SX_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Allow a kernel the device's opt-in shared memory maximum minus its static shared memory.
template <typename K>
inline cudaError_t allow_max_dynamic_smem(K kernel) {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              optin - (int)fa.sharedSizeBytes);
}

// Indirect dispatch (record*Indirect, kernels.zig:84-134): an op recorded behind a device-side
// dispatch record {x, y, z} does nothing when any of the three is zero (the quiescence gate
// wrote zeros).  Read after the dependency wait.
SX_DEV bool gate_closed(const uint32_t *gate) {
  return gate != nullptr && (gate[0] == 0u || gate[1] == 0u || gate[2] == 0u);
}

// Programmatic dependent launch: wait for the producer grid's memory before reading it.
SX_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
SX_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::); }

}  // namespace sx
