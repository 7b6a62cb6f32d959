// sx_stream.cu -- the streaming decode kernel (graph mode 3).
//
// One cooperative launch per token runs the fused decode graph (per layer: q|k|v GEMV with the
// residual + input-norm prologue, fused q/k norm + RoPE + cache write + attention, o GEMV,
// gate+up GeGLU with the residual + pre-FFN norm prologue, down GEMV; then the Q8 LM head with
// the final-norm prologue and the argmax epilogue; model_dispatch.zig:10-43) as a table of
// phases, on one CTA per SM.  The CTA is warp-specialised:
//
//   * one producer warp streams every weight chunk this CTA will consume, phase after phase,
//     into a ring of shared-memory stages with bulk asynchronous copies (cp.async.bulk, one
//     mbarrier per stage for "full" and one for "empty").  Weights do not depend on the token,
//     so the producer never waits for a phase to finish -- only for a free stage.  While the
//     consumers stand at a phase boundary (waiting for every CTA to finish the previous phase,
//     normalising the next input, running the latency-bound attention), HBM keeps filling the
//     ring with the next phases' weights;
//   * sixteen consumer warps take the chunks of each stage round-robin (chunk w and w + 16 of
//     a stage go to warp w), dequantise them into mma.m16n8k16 fragments exactly like the GEMV
//     kernels (sx_gemv_dev.cuh) and accumulate per 16-row tile.  A tile's chunks are spread over
//     all sixteen warps, so each warp deposits its partial tile sums in a shared-memory slot and
//     the last warp to deposit adds the sixteen partials in warp order (deterministic) and
//     writes the rows.
//
// Phases are ordered by per-phase completion counters in device memory (zeroed before every
// launch): a CTA that finished phase p adds 1 to ctr[p] (release); a phase that reads what
// phase p wrote waits until ctr[p] equals the grid size (acquire).  Activations written by
// other CTAs are read through L2 (.cg loads).  Every wait is bounded: a wait that runs out
// records kDevBarrierTimeout, sets the abort word ctr[n], and from then on every wait of every
// warp returns at once, so the kernel runs through its remaining phases without work and
// exits -- no hang, and the token is reported as failed.  All consumer threads take the same
// named barriers in the same order whatever happens, so no barrier can be left waiting.
#include "sx_attn_dev.cuh"
#include "sx_gemv_dev.cuh"

namespace sx {

namespace {

constexpr int kSW = 16;                         // consumer warps
constexpr uint32_t kSConsumers = kSW * 32;      // consumer threads (warps 0..15)
constexpr int kSThreads = kSConsumers + 32;     // + the producer warp (warp 16)
constexpr int kSStages = 7;
constexpr uint32_t kSStageBytes = 20480;        // 32 Q4 chunks, 16 GeGLU pairs, 16 Q8 chunks
constexpr uint32_t kSGroupTiles = 8;  // tiles whose partial sums are reduced together
constexpr uint32_t kSTileFloats = kSW * 16 * 2;  // warps x tile rows x (up to 2) matrices
constexpr uint32_t kSSmem = 227 * 1024;
constexpr uint32_t kSRingOff = kSSmem - kSStages * kSStageBytes;
constexpr uint32_t kSRedOff = kSRingOff - kSGroupTiles * kSTileFloats * 4;
constexpr uint32_t kSMetaOff = kSRedOff - 256;
constexpr uint32_t kSPhaseArea = kSMetaOff;     // x fragments / attention work items
constexpr long long kSWaitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

static_assert(kSRingOff % 128 == 0 && kSRedOff % 128 == 0 && kSMetaOff % 128 == 0,
              "shared-memory regions must stay aligned");

SX_DEV uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SX_DEV void red_release_add(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
SX_DEV bool aborted(const uint32_t *abort_w) {
  return *reinterpret_cast<const volatile uint32_t *>(abort_w) != 0;
}
SX_DEV void set_abort(uint32_t *abort_w, uint32_t *err) {
  atomicExch(abort_w, 1u);
  raise_error(err, kDevBarrierTimeout);
}
SX_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
// bounded mbarrier wait that also gives up once the kernel is aborting
SX_DEV bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, uint32_t *abort_w, uint32_t *err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 255) == 0) {
      if (aborted(abort_w)) return false;
      if (clock64() - t0 > kSWaitCycles) {
        set_abort(abort_w, err);
        return false;
      }
    }
  }
  return true;
}

// consumer-wide named barrier (the producer warp never takes part)
SX_DEV void csync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kSConsumers) : "memory"); }
struct ConsumerSync {
  SX_DEV void operator()() const { csync(); }
  SX_DEV uint32_t threads() const { return kSConsumers; }
};

// Wait (thread 0 of the calling group polls, the group then synchronises through `sync`) until
// every CTA has finished phase p; false when the kernel is aborting.  `flag` is a shared word
// the poller uses to tell the group the outcome.
template <typename Sync>
SX_DEV bool wait_phase(const uint32_t *ctr, uint32_t p, uint32_t *abort_w, uint32_t *err,
                       bool leader, volatile uint32_t *flag, Sync sync) {
  if (leader) {
    uint32_t ok = aborted(abort_w) ? 0u : 1u;
    if (ok && ld_acquire(ctr + p) < gridDim.x) {
      const long long t0 = clock64();
      while (ld_acquire(ctr + p) < gridDim.x) {
        if (aborted(abort_w)) {
          ok = 0;
          break;
        }
        if (clock64() - t0 > kSWaitCycles) {
          set_abort(abort_w, err);
          ok = 0;
          break;
        }
        __nanosleep(32);
      }
    }
    __threadfence();
    *flag = ok;
  }
  sync();
  return *flag != 0;
}

// named barrier of one 256-thread half of the consumers (ids 2 and 3)
struct HalfSync {
  int bar;
  SX_DEV void operator()() const { group_sync(bar); }
  SX_DEV uint32_t threads() const { return 256; }
};

struct SMeta {
  uint64_t full[kSStages];
  uint64_t empty[kSStages];
  uint32_t flag[4];       // [0]: phase-wait outcome for the consumers; [2], [3]: attention halves
  uint32_t item_last[2];  // attention: "this item merges its head" per half
};
static_assert(sizeof(SMeta) <= 256, "meta block");

SX_HD uint32_t chunks_per_warp(int qt, int nmat) { return (qt == 4 && nmat == 1) ? 2u : 1u; }

// This CTA's whole tiles [ct0, ct1) of a GEMV phase.
SX_DEV void cta_tiles(const GemvArgs &a, uint32_t &ct0, uint32_t &ct1) {
  const uint32_t T = a.tiles[0] + a.tiles[1] + a.tiles[2];
  ct0 = (uint32_t)((uint64_t)T * blockIdx.x / gridDim.x);
  ct1 = (uint32_t)((uint64_t)T * (blockIdx.x + 1) / gridDim.x);
}

// ------------------------------------------------------------------------------------------
// Producer warp: every GEMV phase's chunks of this CTA, in phase order, one stage at a time.
SX_DEV void stream_producer(const Phase *__restrict__ ph, uint32_t n, SMeta *meta, uint8_t *ring,
                            uint32_t *abort_w, uint32_t *err) {
  const int lane = threadIdx.x & 31;
  uint32_t st = 0;
  for (uint32_t p = 0; p < n; ++p) {
    const uint32_t kind = ph[p].kind;
    if (kind != kPhaseGemv) continue;
    const GemvArgs &a = ph[p].g;
    const int qt = ph[p].variant >= 2 ? 8 : 4, nmat = (ph[p].variant & 1) ? 2 : 1;
    const uint32_t cb = qt == 4 ? kQ4ChunkBytes : kQ8ChunkBytes;
    const uint32_t spc = kSW * chunks_per_warp(qt, nmat);
    uint32_t ct0, ct1;
    cta_tiles(a, ct0, ct1);
    const uint32_t P = pairs_of(a.k), c0 = ct0 * P, nch = (ct1 - ct0) * P;
    // the K/V rows the following attention reads: into L2 now (the slot list and step record
    // are inputs of the token, ready before the launch), spread over the CTAs and lanes
    if (a.pf_slots != nullptr) {
      const uint32_t S = min(a.pf_step[2], a.pf_max);
      for (uint32_t j = lane * gridDim.x + blockIdx.x; j < S; j += 32 * gridDim.x) {
        const uint32_t sl = a.pf_slots[j];
        if (sl < a.pf_max)
          for (int b = 0; b < 2; ++b)
            if (a.pf_base[b] != nullptr)
              prefetch_l2_bulk(static_cast<const uint8_t *>(a.pf_base[b]) + (size_t)sl * a.pf_row_bytes,
                               a.pf_row_bytes);
      }
    }
    // stage j carries chunks [c0 + j spc, c0 + (j + 1) spc) of each matrix, one bulk copy
    // each (matrix m at + m spc cb)
    for (uint32_t base = 0; base < nch; base += spc, ++st) {
      const uint32_t s = st % kSStages, use = st / kSStages;
      const uint32_t full = smem_u32(&meta->full[s]), empty = smem_u32(&meta->empty[s]);
      bool ok = true;
      if (use > 0) ok = mbar_wait_or_abort(empty, (use - 1) & 1, abort_w, err);
      if (!ok) return;  // aborting: the consumers skip their waits from now on
      const uint32_t cnt = min(spc, nch - base);
      if (lane == 0) {
        mbar_arrive_expect_tx(full, cnt * cb * nmat);
        const uint32_t dst = smem_u32(ring + s * kSStageBytes);
        for (int m = 0; m < nmat; ++m)
          bulk_g2s(dst + m * spc * cb,
                   static_cast<const uint8_t *>(a.w[0][m]) + (size_t)(c0 + base) * cb, cnt * cb,
                   full);
      }
      __syncwarp();
    }
  }
}

// ------------------------------------------------------------------------------------------
// Consumer side of a GEMV phase (batch 1).
struct Emit {
  float bv;
  uint32_t bi;
};

template <int QT, int NMAT>
__device__ __noinline__ void stream_gemv(const GemvArgs &a, uint8_t *smem, SMeta *meta,
                                         uint8_t *ring, float *red, uint32_t &st, bool ok,
                                         const uint32_t *ctr, uint32_t wait_p,
                                         uint32_t *abort_w, uint32_t *err) {
  constexpr int CB = QTraits<QT>::kChunk;
  constexpr int SO = QTraits<QT>::kScaleOff;
  constexpr uint32_t U = (QT == 4 && NMAT == 1) ? 2 : 1;
  constexpr uint32_t SPC = kSW * U;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const bool pro = a.pro != kProNone;
  const Layout L = layout_of(a.k, 1, NMAT, QT, pro, 1);
  const uint32_t P = pairs_of(a.k);
  uint32_t ct0, ct1;
  cta_tiles(a, ct0, ct1);
  const uint32_t nch = (ct1 - ct0) * P;
  ConsumerSync sync;

  // the norm gains do not depend on the previous phase: load them, then wait for it
  ProGains gn;
  if (pro) load_prologue_gains(a, kSConsumers, gn);
  if (wait_p != kNoPhase)
    ok = wait_phase(ctr, wait_p, abort_w, err, threadIdx.x == 0, &meta->flag[0], sync) && ok;
  // input: residual / norm prologue, then the B fragments (x is read through L2)
  float *xin = reinterpret_cast<float *>(smem + L.xin);
  if (pro) {
    run_prologue_gains(a, xin, reinterpret_cast<float *>(smem + L.misc + 64), sync, gn);
    stage_x<QT>(a, xin, a.k, smem, L, false, sync);
  } else {
    stage_x<QT>(a, a.x, a.ldx, smem, L, true, sync);
  }
  const uint4 *const xf4 = reinterpret_cast<const uint4 *>(smem + L.xfrag);
  const float *const corr = reinterpret_cast<const float *>(smem + L.corr);
  const float xs = reinterpret_cast<const float *>(smem + L.misc)[0];
  const uint32_t xoff = (g * 4 + c) * 2, xstride = nv_of(1) * 8;
  const bool xvalid = g < 2, cvalid = c == 0;

  Emit best = {-INFINITY, 0xFFFFFFFFu};
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
  // one row of tile tt: scale, GeGLU, write, track the argmax
  auto emit = [&](uint32_t tt, uint32_t row, const float (&v)[NMAT]) {
    uint32_t tl;
    const int s = seg_of(tt, tl);
    const uint32_t r = tl * 16 + row;
    if (r >= a.rows[s]) return;
    float out = v[0] * xs;
    if (NMAT == 2) out = __fmul_rn(gelu_tanh_dev(out), v[NMAT - 1] * xs);
    a.y[s][r] = out;
    if (a.epi == kEpiArgmax) {
      const uint32_t gi = a.row_base[s] + r;
      const float ov = isnan(out) ? -INFINITY : out;
      if (best.bi == 0xFFFFFFFFu || better(ov, gi, best.bv, best.bi)) best = {ov, gi};
    }
  };
  // A tile's chunks are spread over all sixteen warps (chunk offset o goes to warp o mod 16):
  // each warp stores its partial sums of a tile (plain shared stores), and after every group of
  // kSGroupTiles tiles all consumer threads add the sixteen partials of each row in warp order.
  const uint32_t ntiles = ct1 - ct0;
  auto deposit = [&](uint32_t rt, const float (&acc)[NMAT][2]) {
    if (!cvalid) return;
    float *r = red + ((rt % kSGroupTiles) * kSW + warp) * 16 * NMAT;  // [row][m]
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      r[g * NMAT + m] = acc[m][0];
      r[(g + 8) * NMAT + m] = acc[m][1];
    }
  };
  auto flush = [&](uint32_t grp) {
    csync();  // every warp has deposited every tile of the group
    const uint32_t rt = grp * kSGroupTiles + tid / 16, row = tid % 16;
    if (tid < kSGroupTiles * 16 && rt < ntiles && ok) {
      float v[NMAT];
#pragma unroll
      for (int m = 0; m < NMAT; ++m) v[m] = 0.0f;
      const float *b = red + (rt % kSGroupTiles) * kSW * 16 * NMAT + row * NMAT;
#pragma unroll 4
      for (int w = 0; w < kSW; ++w)
#pragma unroll
        for (int m = 0; m < NMAT; ++m) v[m] += b[w * 16 * NMAT + m];
      emit(ct0 + rt, row, v);
    }
    csync();  // the group's buffer is free again
  };

  float acc[NMAT][2];
#pragma unroll
  for (int m = 0; m < NMAT; ++m) acc[m][0] = acc[m][1] = 0.0f;
  uint4 xb[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  float cr[2] = {0.0f, 0.0f};
  // this warp's next chunk: offset o = base + u * 16 + warp in the CTA's run; its tile / pair
  // (every warp has a chunk in every tile: P >= 16)
  uint32_t tile = ct0 + warp / P, pair = warp % P, cur = tile;
  for (uint32_t base = 0; base < nch; base += SPC, ++st) {
    const uint32_t s = st % kSStages, par = (st / kSStages) & 1;
    if (ok) ok = mbar_wait_or_abort(smem_u32(&meta->full[s]), par, abort_w, err);
    const uint8_t *stage = ring + s * kSStageBytes;
#pragma unroll
    for (uint32_t u = 0; u < U; ++u) {
      const uint32_t o = base + u * kSW + warp;
      if (o < nch) {
        if (tile != cur) {  // the previous tile is done for this warp
          deposit(cur - ct0, acc);
#pragma unroll
          for (int m = 0; m < NMAT; ++m) acc[m][0] = acc[m][1] = 0.0f;
          cur = tile;
          if ((tile - ct0) % kSGroupTiles == 0) flush((tile - ct0) / kSGroupTiles - 1);
        }
        if (ok) {
          const uint8_t *ch = stage + (u * kSW + warp) * CB;
          if (xvalid) {
            xb[0] = xf4[pair * xstride + xoff];
            xb[1] = xf4[pair * xstride + xoff + 1];
          }
          if (cvalid) {
            const float2 c2 = *reinterpret_cast<const float2 *>(corr + pair * 2);
            cr[0] = c2.x;
            cr[1] = c2.y;
          }
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const uint8_t *cm = ch + m * SPC * CB;
            const float4 sc = *reinterpret_cast<const float4 *>(cm + SO + g * 16);
            uint4 wq[QT == 4 ? 1 : 2];
            wq[0] = *reinterpret_cast<const uint4 *>(cm + lane * 16);
            if (QT == 8) wq[QT == 4 ? 0 : 1] = *reinterpret_cast<const uint4 *>(cm + lane * 16 + 512);
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
              }
              const float sg = hb ? sc.z : sc.x, sg8 = hb ? sc.w : sc.y;
              block_mma<QT>(a0, a1, xb[hb], cr[hb], sg, sg8, acc[m]);
            }
          }
        }
        pair += kSW;  // this warp's next chunk is 16 further on
        if (pair >= P) {
          pair -= P;
          ++tile;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&meta->empty[s]));
  }
  if (ntiles > 0) {
    deposit(cur - ct0, acc);
    flush((ntiles - 1) / kSGroupTiles);
  }

  if (a.epi == kEpiArgmax) {
    // warp -> CTA (shared memory) -> grid (one candidate per CTA; the last CTA merges)
    float *cv = reinterpret_cast<float *>(smem + L.misc + 64);  // [16] (after the block sums)
    uint32_t *ci = reinterpret_cast<uint32_t *>(cv + kSW);
    auto merge = [](Emit &b, float v, uint32_t ix) {
      if (ix != 0xFFFFFFFFu && (b.bi == 0xFFFFFFFFu || better(v, ix, b.bv, b.bi))) b = {v, ix};
    };
    auto warp_merge = [&](Emit &b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b.bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, b.bi, o);
        merge(b, ov, oi);
      }
    };
    csync();  // the block-sum scratch is free
    warp_merge(best);
    if (lane == 0) {
      cv[warp] = best.bv;
      ci[warp] = best.bi;
    }
    csync();
    if (warp == 0) {
      Emit b = {-INFINITY, 0xFFFFFFFFu};
      if (lane < kSW) b = {cv[lane], ci[lane]};
      warp_merge(b);
      if (lane == 0) {
        a.best_v[(size_t)blockIdx.x * 8] = b.bv;
        a.best_i[(size_t)blockIdx.x * 8] = b.bi;
      }
      __threadfence();
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atomicAdd(a.done_cnt, 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old + 1 == gridDim.x) {
        __threadfence();
        Emit r = {-INFINITY, 0xFFFFFFFFu};
        for (uint32_t w = lane; w < gridDim.x; w += 32)
          merge(r, __ldcg(a.best_v + (size_t)w * 8), __ldcg(a.best_i + (size_t)w * 8));
        warp_merge(r);
        if (lane == 0) {
          uint32_t tok = r.bi == 0xFFFFFFFFu ? 0u : r.bi;
          const bool nan0 = a.row_base[0] == 0 && isnan(__ldcg(a.y[0]));
          if (nan0) tok = 0;
          a.token[0] = tok;
          if (a.cand) {
            a.cand[0] = __float_as_uint(r.bv);
            a.cand[1] = r.bi;
            a.cand[2] = nan0 ? 1u : 0u;
            a.cand[3] = 0u;
          }
          *a.done_cnt = 0;
        }
      }
    }
  }
}

// ------------------------------------------------------------------------------------------
// Attention phase: work items (kv head, 32-slot chunk) on the two 256-thread halves of the
// consumers (named barriers 2 and 3), or on the first half alone when two items do not fit the
// phase area; the first round's items fetch their K/V rows before waiting for the q|k|v phase.
SX_HD uint32_t stream_item_floats(const AttnFusedArgs &a) {
  const uint32_t nchunks = (a.total_slots + kAttnChunk - 1) / kAttnChunk;
  return (attn_item_floats((int)(a.num_q / a.num_kv), a.head_dim, nchunks) + 31) & ~31u;
}
SX_HD uint32_t stream_item_groups(const AttnFusedArgs &a) {
  const uint32_t per = stream_item_floats(a) * 4;
  return 2 * per <= kSPhaseArea ? 2u : per <= kSPhaseArea ? 1u : 0u;
}

template <int DPL, int G, bool BF16>
__device__ __noinline__ void stream_attn(const AttnFusedArgs &a, uint8_t *smem, SMeta *meta,
                                         const uint32_t *ctr, uint32_t wait_p, bool ok,
                                         uint32_t *abort_w, uint32_t *err) {
  const uint32_t nchunks = (a.total_slots + kAttnChunk - 1) / kAttnChunk, items = a.num_kv * nchunks;
  const uint32_t per = stream_item_floats(a), groups = stream_item_groups(a);
  const int half = threadIdx.x >> 8, t = threadIdx.x & 255;
  float *sh = reinterpret_cast<float *>(smem) + half * per;
  const uint32_t rounds = (items + groups * gridDim.x - 1) / (groups * gridDim.x);
  const bool in_group = (uint32_t)half < groups;
  for (uint32_t r = 0; r < rounds; ++r) {
    const uint32_t item = blockIdx.x + (groups * r + half) * gridDim.x;
    const bool active = ok && in_group && item < items;
    const uint32_t kvh = active ? item / nchunks : 0, chunk = active ? item % nchunks : 0;
    if (r == 0) {
      // every group waits for the q|k|v phase (its leader polls) before it reads q, k, v
      auto wait = [&] {
        ok = wait_phase(ctr, wait_p, abort_w, err, t == 0, &meta->flag[2 + half],
                        HalfSync{2 + half}) && ok;
      };
      if (in_group)
        attn_item<DPL, G, BF16>(a, kvh, chunk, nchunks, sh, &meta->item_last[half], t, 2 + half,
                                active, wait);
    } else if (active) {
      attn_item<DPL, G, BF16>(a, kvh, chunk, nchunks, sh, &meta->item_last[half], t, 2 + half,
                              true, [] {});
    }
    csync();  // the halves reuse their shared memory in the next round
  }
}

template <int DPL>
SX_DEV void stream_attn_g(const AttnFusedArgs &a, uint32_t gi, bool bf16, uint8_t *smem,
                          SMeta *meta, const uint32_t *ctr, uint32_t wait_p, bool ok,
                          uint32_t *abort_w, uint32_t *err) {
#define SX_STREAM_ATTN(G)                                                                   \
  (bf16 ? stream_attn<DPL, G, true>(a, smem, meta, ctr, wait_p, ok, abort_w, err)           \
        : stream_attn<DPL, G, false>(a, smem, meta, ctr, wait_p, ok, abort_w, err))
  switch (gi) {
    case 0: SX_STREAM_ATTN(1); break;
    case 1: SX_STREAM_ATTN(2); break;
    case 2: SX_STREAM_ATTN(4); break;
    default: SX_STREAM_ATTN(8); break;
  }
#undef SX_STREAM_ATTN
}

__global__ void __launch_bounds__(kSThreads, 1)
    stream_kernel(const Phase *__restrict__ ph, uint32_t n, uint32_t *ctr, uint32_t *err) {
  extern __shared__ __align__(1024) uint8_t smem[];
  SMeta *meta = reinterpret_cast<SMeta *>(smem + kSMetaOff);
  float *red = reinterpret_cast<float *>(smem + kSRedOff);
  uint8_t *ring = smem + kSRingOff;
  uint32_t *abort_w = ctr + n;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSStages; ++s) {
      mbar_init(smem_u32(&meta->full[s]), 1);
      mbar_init(smem_u32(&meta->empty[s]), kSW);
    }
    fence_mbar_init();
  }
  __syncthreads();  // the only CTA-wide barrier: the roles split here
  if (threadIdx.x >= kSConsumers) {
    stream_producer(ph, n, meta, ring, abort_w, err);
    return;
  }
  uint32_t st = 0;
  bool ok = true;
  for (uint32_t p = 0; p < n; ++p) {
    const Phase &cur = ph[p];
    if (cur.kind == kPhaseGemv) {
      const uint32_t wp = p > 0 ? p - 1 : kNoPhase;
      switch (cur.variant) {
        case 0: stream_gemv<4, 1>(cur.g, smem, meta, ring, red, st, ok, ctr, wp, abort_w, err); break;
        case 1: stream_gemv<4, 2>(cur.g, smem, meta, ring, red, st, ok, ctr, wp, abort_w, err); break;
        default: stream_gemv<8, 1>(cur.g, smem, meta, ring, red, st, ok, ctr, wp, abort_w, err); break;
      }
    } else {
      const uint32_t v = cur.variant, gi = (v >> 1) & 3;
      const bool bf16 = v & 1;
      switch (v >> 3) {
        case 0: stream_attn_g<2>(cur.at, gi, bf16, smem, meta, ctr, p - 1, ok, abort_w, err); break;
        case 1: stream_attn_g<4>(cur.at, gi, bf16, smem, meta, ctr, p - 1, ok, abort_w, err); break;
        default: stream_attn_g<8>(cur.at, gi, bf16, smem, meta, ctr, p - 1, ok, abort_w, err); break;
      }
    }
    ok = ok && !aborted(abort_w);
    csync();  // every consumer is done with phase p (outputs written, shared memory free)
    if (threadIdx.x == 0) {
      __threadfence();
      red_release_add(ctr + p, 1u);
    }
  }
}

}  // namespace

uint32_t stream_smem_bytes() { return kSSmem; }
uint32_t stream_threads() { return kSThreads; }

// false when the call has no streaming form: batch > 1, k not a whole number of >= 16 block
// pairs, an input layout larger than the phase area, or a tile split across CTAs
bool stream_gemv_variant(int qt, bool geglu, const GemvArgs &a, int num_sms, uint32_t *variant) {
  if (a.batch != 1 || (qt == 8 && geglu) || a.k % 64 != 0 || pairs_of(a.k) < (uint32_t)kSW)
    return false;
  const int nmat = geglu ? 2 : 1;
  const Layout L = layout_of(a.k, 1, nmat, qt, a.pro != kProNone, 1);
  if (L.xin + L.xin_bytes > kSPhaseArea || L.misc + 64 + 4 * 48 > kSPhaseArea) return false;
  (void)num_sms;
  *variant = qt == 8 ? 2u : (geglu ? 1u : 0u);
  return true;
}

bool stream_attn_variant(const AttnFusedArgs &a, uint32_t *variant) {
  if (a.num_kv == 0 || a.num_q % a.num_kv || a.sessions > 1) return false;
  const uint32_t g = a.num_q / a.num_kv;
  const int gi = g == 1 ? 0 : g == 2 ? 1 : g == 4 ? 2 : g == 8 ? 3 : -1;
  const int di = a.head_dim == 64 ? 0 : a.head_dim == 128 ? 1 : a.head_dim == 256 ? 2 : -1;
  if (gi < 0 || di < 0 || stream_item_groups(a) == 0) return false;
  *variant = (uint32_t)di * 8 + (uint32_t)gi * 2 + (a.kv_bf16 ? 1u : 0u);
  return true;
}

cudaError_t prepare_stream_kernel() {
  cudaError_t e = cudaFuncSetAttribute(stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSSmem);
  return e;
}

cudaError_t launch_stream(const Phase *phases, uint32_t n, uint32_t *ctr, uint32_t *err,
                          int num_sms, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = kSSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, stream_kernel, phases, n, ctr, err);
}

}  // namespace sx
