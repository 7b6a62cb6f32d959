// sx_prefill.cu -- batch-prefill projection GEMM with Q4_0 weights on the sm_100a tensor cores.
//
//   Y[T x N] (f32) = X[T x K] (bf16) . deq(W)[N x K]^T,   deq(W)[n][k] = bf16_rne((q - 8) * d)
//
// A new capability of the B200 build: the reference prefills by running forwardToken once per
// token (src/model/forward.zig:19-75, gemv_q4.wgsl per projection); batching the tokens of
// many sessions turns each projection into one GEMM.  The dequantised weight equals the
// checker's (f32)(q - 8) * d rounded to bf16 (round to nearest even), bit for bit.
//
// CTA tile: 256 tokens x 256 weight rows, K in steps of 64, 3 shared-memory stages (74 KB
// each: X 32 KB, dequantised W 32 KB, raw Q4 10 KB); each weight is dequantised once and used
// by 256 tokens, each X tile by 256 weight rows.
//   warp 0, lane 0   loads: one TMA box of X (256 x 64 bf16, 128-byte swizzle) and one TMA box
//                    of the 16 raw 640-byte Q4 chunks of the stage's 256 rows (the packed
//                    weights seen as a u32 tensor [tiles][pairs x 160]), both completing on the
//                    stage's `full` barrier;
//   warps 4..19      dequantise one chunk each into the stage's B tile, written in the UMMA
//                    K-major 128-byte-swizzle layout, fence the async proxy and arrive on `ready`;
//   warp 1, lane 0   issues tcgen05.mma (M 128, N 256, K 16, bf16 x bf16 -> f32) for the two
//                    token halves into two TMEM accumulators (all 512 columns) and commits each
//                    stage to `empty`;
//   warps 4..19      then read the accumulators back (tcgen05.ld 32x32b), stage them in shared
//                    memory and store Y with TMA.
// Every mbarrier wait is bounded; a wait that runs out records kDevWaitTimeout, the CTA stops
// issuing, drains what it already issued and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "sx_common.cuh"
#include "sx_host.h"
#include "sx_internal.h"

namespace sx {

namespace {

constexpr int kBM = 256, kBN = 256, kBK = 64, kStages = 3;
constexpr int kDqWarps = 16;                            // one raw chunk per warp and stage
constexpr int kPThreads = (4 + kDqWarps) * 32;          // 20 warps
constexpr uint32_t kATile = kBM * kBK * 2;              // 32 KB of X per stage
constexpr uint32_t kBTile = kBN * kBK * 2;              // 32 KB of dequantised W per stage
constexpr uint32_t kRaw = (kBN / 16) * kQ4ChunkBytes;   // 16 raw chunks = 10 KB per stage
constexpr uint32_t kStageBytes = kATile + kBTile + ((kRaw + 1023) & ~1023u);
constexpr uint32_t kPrefillSmem = kStages * kStageBytes + 2048;  // + alignment, barriers
constexpr uint32_t kTmemCols = 512;                     // two 128 x 256 f32 accumulators
static_assert(kDqWarps * 8192 <= kStages * kStageBytes, "epilogue staging reuses the stages");

// ---- tcgen05 / TMA wrappers (PTX ISA 8.7, sm_100a) ----
SX_DEV void tmem_alloc(uint32_t dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst_smem),
               "r"(cols)
               : "memory");
}
SX_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
SX_DEV void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(cols)
               : "memory");
}
SX_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
SX_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// D[tmem] (+)= A[smem desc] . B[smem desc]^T, kind::f16 (bf16 operands per the instruction
// descriptor); accumulate = false overwrites D.
SX_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                     bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}
// arrive once on the mbarrier when every tcgen05 operation this thread issued has completed
SX_DEV void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   bar)
               : "memory");
}
SX_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
SX_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// 2-D tiled TMA load of box (x = k, y = token row) into this CTA's own shared memory
SX_DEV void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
      "[%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 2-D tiled TMA store of a shared-memory box to global memory (rows/columns past the tensor's
// extent are not written), tracked by the issuing thread's bulk async-group
SX_DEV void tma_store_2d(const CUtensorMap *map, int32_t x, int32_t y, uint32_t src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(src)
      : "memory");
}
SX_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// the shared-memory source of all but the newest N committed groups has been read
template <int N>
SX_DEV void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
SX_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

// UMMA shared-memory descriptor of a K-major tile in the 128-byte swizzle layout: rows of 128 B
// (64 bf16), 8-row groups 1024 B apart (stride byte offset), version 1, layout type 2.
SX_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: D f32, A and B bf16, both K-major, N >> 3, M >> 4.
constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// fma.rn.f32x2: two independent single-precision FMAs (sm_100), each rounded once
SX_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 pa, pb, pc, pd;\n"
      "mov.b64 pa, {%2, %3};\nmov.b64 pb, {%4, %5};\nmov.b64 pc, {%6, %7};\n"
      "fma.rn.f32x2 pd, pa, pb, pc;\nmov.b64 {%0, %1}, pd;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Nibble at bits [p, p + 4) of v -> the float 2^(23 - p) + q: the nibble becomes the top of the
// mantissa under exponent 23 - p, one LOP3 (p = 8: magic 2^15, p = 12: magic 2^11).
SX_DEV float nib_p8(uint32_t v) { return __uint_as_float(and_or(v, 0x00000F00u, 0x47000000u)); }
SX_DEV float nib_p12(uint32_t v) { return __uint_as_float(and_or(v, 0x0000F000u, 0x45000000u)); }

// Dequantise one raw 640-byte chunk (16 weight rows x 64 columns of the packed Q4_0 layout) into
// rows [row0, row0 + 16) of a K-major 128-byte-swizzled bf16 tile: row n is 128 B long, 8-row
// groups are 1024 B apart and 16-byte column chunk j of row n sits at chunk j ^ (n mod 8).
// Lane l = 4 g + c holds the words of rows g and g + 8 for the pair's two 32-column blocks;
// nibble slot s of a word is column 8 s + 2 c and slot s + 4 column 8 s + 2 c + 1 (sx_quant.cu).
//
// Exactness: with m = 2^(23-p) + q (exact) and C = 2^(23-p) + 8, fma(m, d, -C d) evaluates
// m d - C d = (q - 8) d exactly and rounds once, so it equals the checker's f32 product
// (q - 8) * d whenever -C d is itself exact: d is an f16 scale (11 significant bits) and
// C = 2^15 + 8 = 8 * 4097 (13 bits) or 2^11 + 8 = 8 * 257 (9 bits) keeps C d within 24 bits.
// Slots 0, 1 and 4, 5 are moved to bit positions 8 and 12 by shifts, slots 2, 3 and 6, 7 are
// there already (in v and v >> 16), so every value needs one LOP3 and half a paired FMA.
SX_DEV void dequant_chunk_sw128(const uint8_t *raw, uint32_t btile, uint32_t row0, int lane) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 wq = *reinterpret_cast<const uint4 *>(raw + lane * 16);
  const float4 sc = *reinterpret_cast<const float4 *>(raw + 512 + g * 16);
  const uint32_t w[4] = {wq.x, wq.y, wq.z, wq.w};
  const float s[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    const uint32_t row = row0 + g + (wi & 1) * 8, hb = wi >> 1, rsw = row & 7;
    const uint32_t rbase = btile + (row >> 3) * 1024 + rsw * 128 + 4 * c;
    const uint32_t u = w[wi], ua = u << 8, ub = u >> 8, uc = u >> 16;
    const float2 d2 = make_float2(s[wi], s[wi]);
    const float c8 = -32776.0f * s[wi], c12 = -2056.0f * s[wi];
    const float2 n8 = make_float2(c8, c8), n12 = make_float2(c12, c12);
    // (slot sl, slot sl + 4) = columns (8 sl + 2 c, 8 sl + 2 c + 1)
    const float2 v[4] = {ffma2(make_float2(nib_p8(ua), nib_p8(ub)), d2, n8),
                         ffma2(make_float2(nib_p12(ua), nib_p12(ub)), d2, n12),
                         ffma2(make_float2(nib_p8(u), nib_p8(uc)), d2, n8),
                         ffma2(make_float2(nib_p12(u), nib_p12(uc)), d2, n12)};
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) {
      const __nv_bfloat162 p = __floats2bfloat162_rn(v[sl].x, v[sl].y);
      const uint32_t j = hb * 4 + sl;
      asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(rbase + ((j ^ rsw) << 4)),
                   "r"(*reinterpret_cast<const uint32_t *>(&p))
                   : "memory");
    }
  }
}

struct PrefillArgs {
  const uint8_t *w;  // packed Q4_0, N x K
  float *y;          // T x N f32, row stride ldy
  uint32_t t, n, k, ldy;
  uint32_t *err;
};

SX_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

__global__ void __launch_bounds__(kPThreads, 1)
    prefill_q4_kernel(const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap wmap,
                      const __grid_constant__ CUtensorMap ymap, PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // stage s: [X tile 32 KB | B tile 32 KB | raw chunks 10 KB], 1024-byte aligned (swizzle atoms)
  const uint32_t base = (smem_u32(smem_raw) + 1023) & ~1023u;
  uint8_t *const gbase = smem_raw + (base - smem_u32(smem_raw));
  auto a_tile = [&](int s) { return base + s * kStageBytes; };
  auto b_tile = [&](int s) { return base + s * kStageBytes + kATile; };
  auto raw_off = [&](int s) { return s * kStageBytes + kATile + kBTile; };
  const uint32_t bars = base + kStages * kStageBytes;
  auto full = [&](int s) { return bars + 8 * s; };           // X + raw chunks landed
  auto ready = [&](int s) { return bars + 32 + 8 * s; };     // B tile dequantised
  auto empty = [&](int s) { return bars + 64 + 8 * s; };     // MMAs of the stage done
  const uint32_t acc_bar = bars + 96;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kStages * kStageBytes + 104);
  volatile uint32_t *abort_flag = reinterpret_cast<uint32_t *>(gbase + kStages * kStageBytes + 108);

  const uint32_t m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
  const uint32_t nk = a.k / kBK, ntiles = tiles_of(a.n), tile0 = n0 / 16;
  const uint32_t nvalid = min((uint32_t)(kBN / 16), ntiles - tile0);  // raw chunks that exist

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(ready(s), kPThreads / 32 - 4);
      mbar_init(empty(s), 1);
    }
    mbar_init(acc_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&]() {
    *abort_flag = 1;
    raise_error(a.err, kDevWaitTimeout);
  };

  uint32_t last_round[kStages];  // loads issuer: last round issued per stage (for the drain)
#pragma unroll
  for (int s = 0; s < kStages; ++s) last_round[s] = 0xFFFFFFFFu;

  if (warp == 0 && lane == 0) {
    // ---- loads: X by TMA, the raw Q4 chunks by bulk copies, one `full` barrier per stage
    for (uint32_t i = 0; i < nk && !*abort_flag; ++i) {
      const int s = i % kStages;
      const uint32_t round = i / kStages;
      if (round > 0 && !mbar_wait_bounded(empty(s), (round - 1) & 1)) {
        fail();
        break;
      }
      mbar_arrive_expect_tx(full(s), kATile + kRaw);  // out-of-range boxes are zero-filled
      tma_load_2d(a_tile(s), &xmap, (int32_t)(i * kBK), (int32_t)m0, full(s));
      tma_load_2d(base + raw_off(s), &wmap, (int32_t)(i * (kQ4ChunkBytes / 4)), (int32_t)tile0,
                  full(s));
      last_round[s] = round;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issue: two M-128 halves share the stage's B tile
    constexpr uint32_t idesc = umma_idesc_bf16(128, kBN);
    for (uint32_t i = 0; i < nk; ++i) {
      const int s = i % kStages;
      const uint32_t ph = (i / kStages) & 1;
      if (*abort_flag || !mbar_wait_bounded(full(s), ph) || !mbar_wait_bounded(ready(s), ph)) {
        if (!*abort_flag) fail();
        break;
      }
      tc_fence_after();
      const uint64_t a0 = umma_desc_sw128(a_tile(s)), a1 = umma_desc_sw128(a_tile(s) + kATile / 2);
      const uint64_t b = umma_desc_sw128(b_tile(s));
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {  // +32 B of the swizzled row per K step of 16
        const bool acc = i > 0 || kk > 0;
        umma_f16(tmem, a0 + 2 * kk, b + 2 * kk, idesc, acc);
        umma_f16(tmem + kBN, a1 + 2 * kk, b + 2 * kk, idesc, acc);
      }
      umma_commit(empty(s));
    }
    umma_commit(acc_bar);  // completes once every issued MMA has
  } else if (warp >= 4) {
    // ---- dequantisation: warp 4 + d owns the stage's raw chunk d (16 weight rows)
    const uint32_t dw = warp - 4;
    for (uint32_t i = 0; i < nk && !*abort_flag; ++i) {
      const int s = i % kStages;
      if (!mbar_wait_bounded(full(s), (i / kStages) & 1)) {
        fail();
        break;
      }
      if (dw < nvalid)
        dequant_chunk_sw128(gbase + raw_off(s) + dw * kQ4ChunkBytes, b_tile(s), dw * 16, lane);
      fence_proxy_async();  // generic-proxy stores -> the tensor core's async-proxy reads
      __syncwarp();
      if (lane == 0) mbar_arrive(ready(s));
    }
  }

  if (warp >= 4) {
    // ---- epilogue (the dequantisation warps, once the accumulators are final): the pipeline's
    // shared memory is free by then (every MMA, hence every load and dequantisation, is done),
    // so each warp stages 32 x 32 f32 boxes in the 128-byte-swizzle layout, two buffers deep,
    // and stores them with TMA.  Warp 4 + 4 gi + q reads TMEM lanes 32 q .. 32 q + 31 (its
    // lane quarter) and owns boxes (half h, column block cb) = item gi, gi + 4, gi + 8, gi + 12.
    const uint32_t q = warp & 3, gi = (warp - 4) >> 2;
    const bool ok = mbar_wait_bounded(acc_bar, 0);
    tc_fence_after();
    if (!ok) fail();
    if (ok && !*abort_flag) {
      const uint32_t stage_buf = base + (warp - 4) * 8192;
#pragma unroll 1
      for (uint32_t m = 0; m < 4; ++m) {
        const uint32_t item = gi + 4 * m, h = item >> 3, cb = item & 7;
        const uint32_t buf = stage_buf + (m & 1) * 4096;
        if (m >= 2) {
          if (lane == 0) bulk_wait_read<1>();  // the store issued from this buffer has read it
          __syncwarp();
        }
        uint32_t r[32];
        tmem_ld32(tmem + ((32 * q) << 16) + h * kBN + cb * 32, r);
        tmem_wait_ld();
        const uint32_t row = buf + lane * 128, sw = lane & 7;
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(row + ((c ^ sw) << 4)),
                       "r"(r[4 * c]), "r"(r[4 * c + 1]), "r"(r[4 * c + 2]), "r"(r[4 * c + 3])
                       : "memory");
        fence_proxy_async();  // generic-proxy writes -> the TMA engine's reads
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&ymap, (int32_t)(n0 + cb * 32), (int32_t)(m0 + h * 128 + 32 * q), buf);
          bulk_commit();
        }
      }
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // a stopped CTA waits (bounded) for the copies it issued before its shared memory goes away
    for (int s = 0; s < kStages; ++s)
      if (last_round[s] != 0xFFFFFFFFu) mbar_wait_bounded(full(s), last_round[s] & 1);
  }
  __syncwarp();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

cudaError_t prepare_prefill_kernel() {
  return cudaFuncSetAttribute(prefill_q4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kPrefillSmem);
}

cudaError_t launch_prefill_q4(const void *w, const void *x, float *y, uint32_t t, uint32_t n,
                              uint32_t k, uint32_t ldy, uint32_t *err, cudaStream_t s) {
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {k, t};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  const cuuint32_t box[2] = {kBK, kBM};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // packed Q4_0 as u32 [tiles][pairs * 160]: box = the 16 chunks (160 words each) of one pair
  CUtensorMap wmap;
  const uint32_t pairs = k / 64;
  const cuuint64_t wdims[2] = {(cuuint64_t)pairs * (kQ4ChunkBytes / 4), tiles_of(n)};
  const cuuint64_t wstrides[1] = {(cuuint64_t)pairs * kQ4ChunkBytes};
  const cuuint32_t wbox[2] = {kQ4ChunkBytes / 4, kBN / 16};
  r = encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(w), wdims, wstrides,
             wbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // Y as f32 [t][ldy], stored in 32 x 32 boxes from the 128-byte-swizzled staging buffers
  CUtensorMap ymap;
  const cuuint64_t ydims[2] = {n, t};
  const cuuint64_t ystrides[1] = {(cuuint64_t)ldy * 4};
  const cuuint32_t ybox[2] = {32, 32};
  r = encode(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, y, ydims, ystrides, ybox, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  PrefillArgs a{static_cast<const uint8_t *>(w), y, t, n, k, ldy, err};
  dim3 grid((t + kBM - 1) / kBM, (n + kBN - 1) / kBN);
  prefill_q4_kernel<<<grid, kPThreads, kPrefillSmem, s>>>(map, wmap, ymap, a);
  return cudaGetLastError();
}

double prefill_flops(uint32_t t, uint32_t n, uint32_t k) { return 2.0 * t * n * k; }

}  // namespace sx
