// sx_persist.cu -- the persistent decode kernel.
//
// One cooperative launch per token runs the whole fused decode graph (per layer: q|k|v GEMV
// with the residual + input-norm prologue, fused q/k norm + RoPE + attention, o GEMV, gate+up
// GeGLU with the residual + pre-FFN norm prologue, down GEMV; then the LM head with the final
// norm prologue and the argmax epilogue, model_dispatch.zig:10-43 / gpu.zig:200-263) as a
// table of phases on one 512-thread CTA per SM.  Consecutive phases are separated by a grid
// barrier; kernel launches, their ramps and drains disappear, and the weights of the next
// GEMV phase are streamed into the CTAs' rings *before* each barrier, so HBM keeps reading
// while the CTAs wait, stage x or run the latency-bound attention.
//
// Shared memory: GEMV phases use [0, layout end) (x fragments, offset terms, staging, rings);
// the two attention work items of a CTA live at the top of the arena, above the layout of any
// GEMV phase whose copies are issued before an attention phase.
//
// The grid barrier is a monotonically counted arrival word (zeroed before every launch): CTA
// thread 0 releases the CTA's writes and adds 1, then polls with ld.acquire until the count
// reaches the barrier's target.  The poll is bounded; on timeout it records
// kDevBarrierTimeout in the device error word and proceeds, so a fault elsewhere cannot hang
// the GPU.  Activations written in one phase and read in a later one go through L2 (.cg
// loads, cp.async.cg), never a possibly stale L1 line.
#include "sx_attn_dev.cuh"
#include "sx_gemv_dev.cuh"

namespace sx {

namespace {

constexpr uint32_t kBarrierSpinLimit = 1u << 21;  // x >= 64 ns per poll: > 0.1 s

SX_DEV uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// bar[0]: arrival count; bar[1]: abort word, set by the first barrier that times out so that
// every later barrier returns at once (the token is invalid and the kernel only has to finish).
// Both live in device memory: the host-mapped error word is written on timeout, never polled.
SX_DEV void grid_sync(uint32_t *bar, uint32_t target, uint32_t *err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    uint32_t spins = 0;
    while (ld_acquire_gpu(bar) < target) {
      if (*reinterpret_cast<volatile uint32_t *>(bar + 1) != 0) break;
      if (++spins > kBarrierSpinLimit) {
        atomicExch(bar + 1, 1u);
        raise_error(err, kDevBarrierTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// ---- GEMV phases: (qt, nmat, ring depth) instantiations, batch <= 4 ----
constexpr int kStageOpts[3] = {8, 6, 4};

SX_HD uint32_t gemv_variant_code(int qt, int nmat, int s_index) {
  return (qt == 8 ? 16u : 0u) + (uint32_t)(nmat - 1) * 8u + (uint32_t)s_index;
}

// Inlined into the kernel (a call boundary costs the loop registers and reloads); ring depths
// 8, 6 and 4 only, to bound the kernel's size.
template <int QT, int NMAT, int S>
SX_DEV void gemv_phase(const GemvArgs &a, uint8_t *smem, bool prefetch, bool run) {
  gemv_body<QT, NMAT, 1, S>(a, smem, prefetch, run, false);
}

template <int QT, int NMAT>
SX_DEV void gemv_dispatch_s(const GemvArgs &a, uint32_t s_index, uint8_t *smem, bool prefetch,
                            bool run) {
  switch (s_index) {
    case 0: gemv_phase<QT, NMAT, 8>(a, smem, prefetch, run); break;
    case 1: gemv_phase<QT, NMAT, 6>(a, smem, prefetch, run); break;
    default: gemv_phase<QT, NMAT, 4>(a, smem, prefetch, run); break;
  }
}

SX_DEV void gemv_dispatch(const Phase &ph, uint8_t *smem, bool prefetch, bool run) {
  const uint32_t v = ph.variant, si = v & 7;
  if (v >= 16) gemv_dispatch_s<8, 1>(ph.g, si, smem, prefetch, run);
  else if (v >= 8) gemv_dispatch_s<4, 2>(ph.g, si, smem, prefetch, run);
  else gemv_dispatch_s<4, 1>(ph.g, si, smem, prefetch, run);
}

// ---- attention phases: two work items per CTA (one per 256-thread half, named barriers 1
// and 2), round r covering items [2 r G, 2 (r + 1) G) for a grid of G CTAs; the first round
// waits for the q|k|v phase inside the item, after its K/V rows were fetched ----
SX_HD uint32_t attn_nchunks(const AttnFusedArgs &a) {
  return (a.total_slots + kAttnChunk - 1) / kAttnChunk;
}

template <int DPL, int G, bool BF16>
__device__ __noinline__ void attn_phase(const AttnFusedArgs &a, float *top, uint32_t *flags,
                                        uint32_t *bar, uint32_t target, uint32_t *err) {
  const uint32_t nchunks = attn_nchunks(a), items = a.num_kv * nchunks;
  const uint32_t per_item = (attn_item_floats(G, 32 * DPL, nchunks) + 31) & ~31u;
  const int half = threadIdx.x >> 8, t = threadIdx.x & 255;
  float *sh = top + half * per_item;
  const uint32_t rounds = (items + 2 * gridDim.x - 1) / (2 * gridDim.x);
  for (uint32_t r = 0; r < rounds; ++r) {
    const uint32_t item = blockIdx.x + (2 * r + half) * gridDim.x;
    const bool active = item < items;
    const uint32_t kvh = active ? item / nchunks : 0, chunk = active ? item % nchunks : 0;
    if (r == 0)
      attn_item<DPL, G, BF16>(a, kvh, chunk, nchunks, sh, flags + half, t, 1 + half, active,
                              [&] { grid_sync(bar, target, err); });
    else if (active)
      attn_item<DPL, G, BF16>(a, kvh, chunk, nchunks, sh, flags + half, t, 1 + half, true,
                              [] {});
    __syncthreads();  // the halves reuse their shared memory in the next round
  }
}

template <int DPL, int G>
SX_DEV void attn_dispatch_b(const AttnFusedArgs &a, bool bf16, float *top, uint32_t *flags,
                            uint32_t *bar, uint32_t target, uint32_t *err) {
  if (bf16) attn_phase<DPL, G, true>(a, top, flags, bar, target, err);
  else attn_phase<DPL, G, false>(a, top, flags, bar, target, err);
}

template <int DPL>
SX_DEV void attn_dispatch_g(const AttnFusedArgs &a, uint32_t gi, bool bf16, float *top,
                            uint32_t *flags, uint32_t *bar, uint32_t target, uint32_t *err) {
  switch (gi) {
    case 0: attn_dispatch_b<DPL, 1>(a, bf16, top, flags, bar, target, err); break;
    case 1: attn_dispatch_b<DPL, 2>(a, bf16, top, flags, bar, target, err); break;
    case 2: attn_dispatch_b<DPL, 4>(a, bf16, top, flags, bar, target, err); break;
    default: attn_dispatch_b<DPL, 8>(a, bf16, top, flags, bar, target, err); break;
  }
}

// variant = dpl_index * 8 + g_index * 2 + bf16
SX_DEV void attn_dispatch(const Phase &ph, float *top, uint32_t *flags, uint32_t *bar,
                          uint32_t target, uint32_t *err) {
  const uint32_t v = ph.variant, gi = (v >> 1) & 3;
  const bool bf16 = v & 1;
  switch (v >> 3) {
    case 0: attn_dispatch_g<2>(ph.at, gi, bf16, top, flags, bar, target, err); break;
    case 1: attn_dispatch_g<4>(ph.at, gi, bf16, top, flags, bar, target, err); break;
    case 2: attn_dispatch_g<8>(ph.at, gi, bf16, top, flags, bar, target, err); break;
    default: attn_dispatch_g<16>(ph.at, gi, bf16, top, flags, bar, target, err); break;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    persist_kernel(const Phase *__restrict__ ph, uint32_t n, uint32_t *bar, uint32_t *err) {
  extern __shared__ __align__(128) uint8_t smem[];
  // the attention items' completion flags sit in the top 16 bytes (no static shared memory:
  // the dynamic arena is the whole opt-in size); GEMV layouts may cover them between uses
  uint32_t *flags = reinterpret_cast<uint32_t *>(smem + kSmemLimit - 16);
  uint32_t target = 0;
  for (uint32_t q = 0; q < n; ++q)
    if (ph[q].kind == kPhaseGemv && ph[q].prefetch_after == kNoPhase)
      gemv_dispatch(ph[q], smem, true, false);
  for (uint32_t p = 0; p < n; ++p) {
    const Phase &cur = ph[p];
    target += gridDim.x;
    if (cur.kind == kPhaseGemv) {
      if (p > 0) grid_sync(bar, target, err);
      else target -= gridDim.x;  // the first phase waits for nothing
      gemv_dispatch(cur, smem, false, true);
    } else {
      // the barrier is taken inside the work item, after its K/V fetch
      attn_dispatch(cur, reinterpret_cast<float *>(smem + cur.smem_off), flags, bar, target,
                    err);
    }
    __syncthreads();  // every warp is done with phase p's shared memory
    for (uint32_t q = p + 1; q < n && q <= p + 2; ++q)
      if (ph[q].kind == kPhaseGemv && ph[q].prefetch_after == p)
        gemv_dispatch(ph[q], smem, true, false);
  }
}

}  // namespace

uint32_t persist_smem_bytes() { return kSmemLimit; }

uint32_t persist_attn_offset(const AttnFusedArgs &a) {
  const uint32_t nchunks = attn_nchunks(a);
  const uint32_t g = a.num_q / a.num_kv;
  const uint32_t per_item = (attn_item_floats((int)g, a.head_dim, nchunks) + 31) & ~31u;
  const uint32_t bytes = 2 * per_item * 4 + 16;  // + the completion flags
  return bytes >= kSmemLimit ? 0 : (kSmemLimit - bytes) & ~127u;
}

bool persist_gemv_variant(int qt, bool geglu, const GemvArgs &a, uint32_t smem_limit,
                          uint32_t *variant, uint32_t *smem_end) {
  if (a.batch > 4 || (qt == 8 && geglu)) return false;
  const int nmat = geglu ? 2 : 1;
  for (int si = 0; si < 3; ++si) {
    const Layout L = layout_for(a.k, a.batch, nmat, qt, kStageOpts[si]);
    if (L.total > smem_limit) continue;
    if (a.pro != kProNone && L.xin_bytes == 0) continue;
    *variant = gemv_variant_code(qt, nmat, si);
    *smem_end = L.total;
    return true;
  }
  return false;
}

bool persist_attn_variant(const AttnFusedArgs &a, uint32_t *variant) {
  if (a.num_kv == 0 || a.num_q % a.num_kv) return false;
  const uint32_t g = a.num_q / a.num_kv;
  int gi = g == 1 ? 0 : g == 2 ? 1 : g == 4 ? 2 : g == 8 ? 3 : -1;
  int di = a.head_dim == 64 ? 0 : a.head_dim == 128 ? 1 : a.head_dim == 256 ? 2
         : a.head_dim == 512 ? 3 : -1;
  if (gi < 0 || di < 0 || persist_attn_offset(a) == 0) return false;
  *variant = (uint32_t)di * 8 + (uint32_t)gi * 2 + (a.kv_bf16 ? 1u : 0u);
  return true;
}

cudaError_t prepare_persist_kernel() { return allow_max_dynamic_smem(persist_kernel); }

cudaError_t launch_persist(const Phase *phases, uint32_t n, uint32_t *bar, uint32_t *err,
                           int num_sms, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemLimit;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, persist_kernel, phases, n, bar, err);
}

}  // namespace sx
