// sx_attn_block.cu -- the decode layer's attention block as one kernel: the q|k|v projection
// (with the residual + input RMSNorm prologue), q/k RMSNorm + partial RoPE + cache write,
// GQA attention over the ring's active-slot list, and the o projection.
//
// Replaces, for one layer of the one-session Q4_0 graph, the launches of gemv_q4.wgsl (q, k,
// v), qkv_rope.wgsl, decode_attn.wgsl and gemv_q4.wgsl (o) that recordLayerDirect issues
// (src/gpu/model_dispatch.zig:10-43); semantics as those shaders (kernels.zig:46-174).
//
// Work split.  The grid is num_kv groups of C CTAs (C = SMs / num_kv, one 512-thread CTA per
// SM); group h owns kv head h and the G = num_q / num_kv q heads that read it:
//   A. q|k|v rows of group h (G q heads, k head h, v head h: (G + 2) * head_dim rows) as
//      whole 16-row tiles split over the group's CTAs, streamed through per-warp cp.async
//      rings exactly as the GEMV kernel does (sx_gemv_dev.cuh); the rows go to global memory
//      and the CTA adds 1 to the group's first counter;
//   B. after the group's C arrivals every CTA normalises and rotates the group's q heads and
//      the new k, v (CTA 0 also stores k, v at the current slot), and runs the online softmax
//      over its share of the active slots, whose K/V rows were bulk-copied into shared memory
//      at kernel start; its (M, L, O) records go to global memory and it adds 1 to the
//      group's second counter;
//   C. after the group's second C arrivals every CTA merges the C records of each q head (in
//      record order) into the group's G x head_dim attention output and multiplies it with its
//      share of the o projection's columns of group h (rows split by tiles over the group's
//      CTAs; those weights were bulk-copied into shared memory at kernel start).  The result is
//      the o projection restricted to the group's columns: opart[h][row].  The consumer (the
//      gate+up GEMV's residual prologue) adds the num_kv partial rows in group order.
// Only the x-dependent work waits: the ring's first chunks, the K/V rows of the CTA's slots,
// its o-projection weights and the norm gains / RoPE table are in flight before the
// programmatic-launch wait.  Counter waits poll with ld.acquire and a time limit; a timeout
// records kDevBarrierTimeout.  The last CTA to leave clears the layer's counters.
#include "sx_attn_dev.cuh"
#include "sx_gemv_dev.cuh"

namespace sx {

namespace {

constexpr int kAbStages = 6;     // phase A ring depth
constexpr int kAbPerWarp = 4;    // slots per warp in phase B (<= 64 slots per CTA)
constexpr uint32_t kAbMaxSlotsPerCta = kWarps * kAbPerWarp;

SX_DEV uint32_t ab_ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SX_DEV uint64_t ab_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Thread 0 polls *p until it reaches target (bounded by wait_ns of GPU time); every thread of
// the CTA leaves together.  Returns false on timeout (recorded in the error word).
SX_DEV bool ab_wait_count(const uint32_t *p, uint32_t target, uint64_t wait_ns, uint32_t *err,
                          uint32_t *flag) {
  if (threadIdx.x == 0) {
    bool ok = true;
    if (ab_ld_acquire(p) < target) {
      const uint64_t t0 = ab_globaltimer();
      while (ab_ld_acquire(p) < target) {
        if (ab_globaltimer() - t0 > wait_ns) {
          ok = false;
          raise_error(err, kDevBarrierTimeout);
          break;
        }
        __nanosleep(32);
      }
    }
    __threadfence();
    *flag = ok ? 1u : 0u;
  }
  __syncthreads();
  return *flag != 0;
}

// A lane's DPL elements of a cached row in shared memory (bf16 pairs or f32) as floats; the
// row slice is DPL * (2 or 4) bytes at a multiple of its own size.
template <int DPL, bool BF16>
SX_DEV void ab_ld_row(const uint8_t *row, float (&v)[DPL]) {
  if constexpr (!BF16) {
    ld_vec<DPL>(reinterpret_cast<const float *>(row), v);
  } else {
    uint32_t w[DPL / 2];
    if constexpr (DPL == 2) {
      w[0] = *reinterpret_cast<const uint32_t *>(row);
    } else if constexpr (DPL == 4) {
      const uint2 u = *reinterpret_cast<const uint2 *>(row);
      w[0] = u.x; w[1] = u.y;
    } else {
#pragma unroll
      for (int i = 0; i < DPL / 8; ++i) {
        const uint4 u = *reinterpret_cast<const uint4 *>(row + 16 * i);
        w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
      }
    }
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) {
      v[2 * i] = u2f(w[i] << 16);
      v[2 * i + 1] = u2f(w[i] & 0xFFFF0000u);
    }
  }
}

// Every thread has made its global writes; publish them with one arrival on *p.
SX_DEV void ab_arrive(uint32_t *p) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(p, 1u);
}

}  // namespace

// Shared-memory plan of one CTA, identical on host and device.
struct AbLayout {
  Layout g;             // phase A GEMV layout (x fragments, x staging, ring) at offset 0
  uint32_t wbuf_end;    // the ring region, reused in phase B for the warp records
  uint32_t kv, kv_bytes;
  uint32_t wo, wo_bytes;
  uint32_t gain;        // q gains [D], k gains [D], sin [D / 2], cos [D / 2]
  uint32_t vec;         // qs [G][D], kn [D], vn [D]
  uint32_t mrg;         // xo [G][D] (16-byte aligned rows), fw [G][C], fl [G][C], ls [G]
  uint32_t ofrag;       // phase C x fragments (layout of a GEMV with k = G * D)
  Layout o;
  uint32_t slots;       // slot indices of this CTA [kAbMaxSlotsPerCta]
  uint32_t bar;         // mbarrier of the bulk copies
  uint32_t total;
};

SX_HD uint32_t ab_align(uint32_t x) { return (x + 127u) & ~127u; }

SX_HD AbLayout ab_layout(uint32_t hidden, uint32_t g, uint32_t d, uint32_t ctas,
                         uint32_t max_slots, uint32_t o_tiles, bool bf16) {
  AbLayout L;
  L.g = layout_of(hidden, 1, 1, 4, true, kAbStages);
  const uint32_t warp_rec = kWarps * g * d * 4 + 2 * kWarps * g * 4;
  L.wbuf_end = L.g.total > L.g.ring + warp_rec ? L.g.total : L.g.ring + warp_rec;
  L.kv = ab_align(L.wbuf_end);
  L.kv_bytes = max_slots * 2 * d * (bf16 ? 2 : 4);
  const uint32_t gp = g * d / 64;
  L.wo = ab_align(L.kv + L.kv_bytes);
  L.wo_bytes = o_tiles * gp * kQ4ChunkBytes;
  L.gain = ab_align(L.wo + L.wo_bytes);
  L.vec = ab_align(L.gain + 3 * d * 4);
  L.mrg = ab_align(L.vec + (g + 2) * d * 4);
  L.ofrag = ab_align(L.mrg + (2 * g * ctas + g + g * d) * 4);
  L.o = layout_of(g * d, 1, 1, 4, false, 0);
  L.slots = ab_align(L.ofrag + L.o.total);
  L.bar = ab_align(L.slots + kAbMaxSlotsPerCta * 4);
  L.total = L.bar + 16;
  return L;
}

namespace {

template <int DPL, int G, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) attn_block_kernel(AttnBlockArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t flag;
  constexpr uint32_t D = 32 * DPL;
  constexpr int S = kAbStages;
  constexpr int CB = kQ4ChunkBytes;
  constexpr uint32_t ESZ = BF16 ? 2 : 4;
  constexpr uint32_t GP = G * D / 64;  // o-projection column pairs of the group
  const GemvArgs &ga = a.g;
  const AttnFusedArgs &at = a.at;
  const uint32_t C = a.ctas, grp = blockIdx.x / C, cta = blockIdx.x % C;
  const uint32_t H = ga.k, P = pairs_of(H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const AbLayout Lb = ab_layout(H, G, D, C, a.max_slots, a.o_tiles, BF16);
  const Layout &L = Lb.g;
  uint32_t *const cnt = a.cnt;
  const uint32_t nkv = at.num_kv;

  // ---- phase 0: everything that does not depend on the producer of x ----
  // active slots of this CTA and its o-projection tiles
  const uint32_t slot = at.step[1];
  uint32_t nS = at.step[2];
  const bool bad_step = nS > at.total_slots || slot >= at.total_slots;
  nS = nS > at.total_slots ? at.total_slots : nS;
  const uint32_t s0 = (uint32_t)((uint64_t)nS * cta / C), s1 = (uint32_t)((uint64_t)nS * (cta + 1) / C);
  const uint32_t ns = min(s1 - s0, kAbMaxSlotsPerCta);
  const uint32_t otiles = a.o_rows / 16;
  const uint32_t ot0 = (uint32_t)((uint64_t)otiles * cta / C), ot1 = (uint32_t)((uint64_t)otiles * (cta + 1) / C);
  const uint32_t no = min(ot1 - ot0, a.o_tiles);
  uint32_t *const slot_s = reinterpret_cast<uint32_t *>(smem + Lb.slots);
  const uint64_t pol = l2_evict_first_policy();  // weights and past K/V: read once per token
  const uint32_t bar = smem_u32(smem + Lb.bar);
  if (warp == 0) {
    if (lane == 0) mbar_init(bar, 32);
    fence_mbar_init();
    __syncwarp();
    // lane l: slots l and l + 32 (K and V rows), o tiles l, l + 32, ...
    uint32_t bytes = 0;
    uint32_t sl_l[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t li = lane + 32 * r;
      sl_l[r] = 0xFFFFFFFFu;
      if (li < ns) {
        sl_l[r] = __ldcg(at.slots + s0 + li);
        slot_s[li] = sl_l[r];
        if (sl_l[r] < at.total_slots) bytes += 2 * D * ESZ;
      }
    }
    for (uint32_t t = lane; t < no; t += 32) bytes += GP * CB;
    mbar_arrive_expect_tx(bar, bytes);
    const uint32_t kv_s = smem_u32(smem + Lb.kv), wo_s = smem_u32(smem + Lb.wo);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t li = lane + 32 * r;
      if (sl_l[r] < at.total_slots) {
        const size_t off = ((size_t)sl_l[r] * at.kv_dim + (size_t)grp * D) * ESZ;
        bulk_g2s_ef(kv_s + (2 * li) * D * ESZ, static_cast<const uint8_t *>(at.k_cache) + off, D * ESZ, bar, pol);
        bulk_g2s_ef(kv_s + (2 * li + 1) * D * ESZ, static_cast<const uint8_t *>(at.v_cache) + off, D * ESZ, bar, pol);
      }
    }
    for (uint32_t t = lane; t < no; t += 32)
      bulk_g2s_ef(wo_s + t * GP * CB,
               static_cast<const uint8_t *>(a.wo) + ((size_t)(ot0 + t) * pairs_of(at.num_q * D) + grp * GP) * CB,
               GP * CB, bar, pol);
  } else if (warp == 1) {
    // q / k norm gains and the RoPE table of this clock (weights and a graph input)
    float *gq = reinterpret_cast<float *>(smem + Lb.gain);
    float *gk = gq + D, *sn = gk + D, *cs = sn + D / 2;
    const uint32_t half = at.rotary_dim / 2;
    const float fclock = (float)at.step[0];
    for (uint32_t i = lane; i < D; i += 32) {
      gq[i] = at.q_norm_w[i];
      gk[i] = at.k_norm_w[i];
    }
    for (uint32_t i = lane; i < D / 2; i += 32) {
      float s = 0.0f, co = 1.0f;
      if (i < half) sincosf(__fmul_rn(fclock, at.inv_freq[i]), &s, &co);
      sn[i] = s;
      cs[i] = co;
    }
  }

  // phase A tile range: the group's virtual tiles are its q heads' tiles, then k's, then v's
  const uint32_t nq_t = G * D / 16, nk_t = D / 16, nt = nq_t + 2 * nk_t;
  const uint32_t vt0 = nt * cta / C, vt1 = nt * (cta + 1) / C;
  const uint32_t cbase = vt0 * P, ncta = (vt1 - vt0) * P;
  const uint32_t c0 = cbase + wstart(ncta, kWarps, warp), c1 = cbase + wstart(ncta, kWarps, warp + 1);
  const uint32_t n = c1 - c0;
  // virtual tile -> (segment, tile of that matrix)
  auto vtile = [&](uint32_t vt, uint32_t &tile) -> int {
    if (vt < nq_t) {
      tile = grp * nq_t + vt;
      return 0;
    }
    if (vt < nq_t + nk_t) {
      tile = grp * nk_t + vt - nq_t;
      return 1;
    }
    tile = grp * nk_t + vt - nq_t - nk_t;
    return 2;
  };
  const uint8_t *const wseg0 = static_cast<const uint8_t *>(ga.w[0][0]);
  const uint8_t *const wseg1 = static_cast<const uint8_t *>(ga.w[1][0]);
  const uint8_t *const wseg2 = static_cast<const uint8_t *>(ga.w[2][0]);
  float *const yseg0 = ga.y[0], *const yseg1 = ga.y[1], *const yseg2 = ga.y[2];
  auto chunk_src = [&](uint32_t vt, uint32_t pair) -> const uint8_t * {
    uint32_t tile;
    const int s = vtile(vt, tile);
    const uint8_t *w = s == 0 ? wseg0 : (s == 1 ? wseg1 : wseg2);
    return w + ((size_t)tile * P + pair) * CB;
  };
  uint8_t *const ring = smem + L.ring + warp * S * QTraits<4>::kStageShared;
  constexpr int KS = QTraits<4>::kStageShared, SO = QTraits<4>::kScaleOff;
  const uint32_t ring_s = smem_u32(ring);
  const uint32_t q_dst = ring_s + lane * 16, s_dst = ring_s + SO + lane * 16;
  const bool s_lane = lane < 8;
  // the issue cursor walks the warp's chunks in order
  uint32_t iv_t = c0 / P, iv_p = c0 % P;
  const uint8_t *iv_src = n > 0 ? chunk_src(iv_t, iv_p) : nullptr;
  uint32_t issued = 0;
  auto issue = [&]() {
    const bool live = issued < n;
    const uint32_t stage = (issued % S) * KS;
    cp_async16_if_ef(q_dst + stage, iv_src + lane * 16, live, pol);
    cp_async16_if_ef(s_dst + stage, iv_src + SO + lane * 16, live && s_lane, pol);
    cp_async_commit();
    ++issued;
    if (live && issued < n) {
      if (++iv_p == P) {
        iv_p = 0;
        iv_src = chunk_src(++iv_t, 0);
      } else {
        iv_src += CB;
      }
    }
  };
#pragma unroll
  for (int st = 0; st < S - 1; ++st) issue();

  const bool gfast = stage_q4_ok(ga, blockDim.x, L);
  GainsQ4 gains_a;
  if (gfast) load_gains_q4(ga, gains_a);
  pdl_launch_dependents();
  pdl_wait();

  // ---- phase A: q | k | v rows of the group ----
  if (gfast) {
    stage_x_q4(ga, smem, L, gains_a);
  } else {
    float *xin = reinterpret_cast<float *>(smem + L.xin);
    run_prologue(ga, xin, reinterpret_cast<float *>(smem + L.misc + 64));
    stage_x<4>(ga, xin, H, smem, L, false);
  }
  {
    const uint4 *const xf4 = reinterpret_cast<const uint4 *>(smem + L.xfrag);
    const float *const corr = reinterpret_cast<const float *>(smem + L.corr);
    const float xs = reinterpret_cast<const float *>(smem + L.misc)[0];
    const uint32_t xoff = (g * 4 + c) * 2, coff = c * 2, xstride = 16, cstride = 2;
    const bool xvalid = g < 2, cvalid = c < 1;
    auto emit = [&](uint32_t vt, uint32_t row, float v) {
      uint32_t tile;
      const int s = vtile(vt, tile);
      float *y = s == 0 ? yseg0 : (s == 1 ? yseg1 : yseg2);
      y[tile * 16 + row] = v * xs;
    };
    float acc[2] = {0.0f, 0.0f}, part0[2] = {0.0f, 0.0f}, part1[2] = {0.0f, 0.0f};
    bool has0 = false, has1 = false;
    uint32_t tt = c0 / P;
    const uint32_t p0 = c0 % P;
    const uint4 *xp = xf4 + p0 * xstride;
    const float *cp = corr + p0 * cstride;
    uint32_t flush_at = n > 0 ? min(P - 1 - p0, n - 1) : 0;
    const uint8_t *const q_rd = ring + lane * 16;
    const uint8_t *const s_rd = ring + SO + g * 16;
    uint4 xb[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    float cr[2] = {0.0f, 0.0f};
    uint32_t i = 0;
    while (i < n) {
#pragma unroll 1
      for (; i <= flush_at; ++i) {
        cp_async_wait<S - 2>();
        __syncwarp();
        issue();
        const uint32_t st_off = (i % S) * KS;
        if (xvalid) {
          xb[0] = xp[xoff];
          xb[1] = xp[xoff + 1];
        }
        if (cvalid) {
          const float2 c2 = *reinterpret_cast<const float2 *>(cp + coff);
          cr[0] = c2.x;
          cr[1] = c2.y;
        }
        const float4 sc = *reinterpret_cast<const float4 *>(s_rd + st_off);
        const uint4 wq = *reinterpret_cast<const uint4 *>(q_rd + st_off);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          uint32_t a0[4], a1[4], rg[4], rg8[4];
          dq4_word(hb ? wq.z : wq.x, rg);
          dq4_word(hb ? wq.w : wq.y, rg8);
          a0[0] = rg[0]; a0[1] = rg8[0]; a0[2] = rg[1]; a0[3] = rg8[1];
          a1[0] = rg[2]; a1[1] = rg8[2]; a1[2] = rg[3]; a1[3] = rg8[3];
          block_mma<4>(a0, a1, xb[hb], cr[hb], hb ? sc.z : sc.x, hb ? sc.w : sc.y, acc);
        }
        xp += xstride;
        cp += cstride;
      }
      const uint32_t tb = tt * P, te = tb + P;
      if (tb >= c0 && te <= c1) {
        if (c == 0) {
          emit(tt, g, acc[0]);
          emit(tt, g + 8, acc[1]);
        }
      } else if (c0 >= tb) {
        part0[0] = acc[0], part0[1] = acc[1];
        has0 = true;
      } else {
        part1[0] = acc[0], part1[1] = acc[1];
        has1 = true;
      }
      acc[0] = acc[1] = 0.0f;
      ++tt;
      xp = xf4;
      cp = corr;
      flush_at = min(flush_at + P, n - 1);
    }
    cp_async_wait<0>();
    // tiles shared by several warps: partial sums meet in the warps' rings, added in warp order
    {
      float *own = reinterpret_cast<float *>(ring);
      if (c == 0) {
        if (has0) {
          own[g] = part0[0];
          own[g + 8] = part0[1];
        }
        if (has1) {
          own[16 + g] = part1[0];
          own[16 + g + 8] = part1[1];
        }
      }
    }
    __syncthreads();
    for (uint32_t t = vt0 + warp; t < vt1; t += kWarps) {
      const uint32_t fc = (t - vt0) * P, lc = fc + P - 1;
      const uint32_t wlo = wowner(ncta, kWarps, fc), whi = wowner(ncta, kWarps, lc);
      if (wlo == whi) continue;
      float v = 0.0f;
      for (uint32_t w = wlo; w <= whi; ++w) {
        if (wstart(ncta, kWarps, w) == wstart(ncta, kWarps, w + 1)) continue;
        const int sl = (w == wlo && wstart(ncta, kWarps, w) < fc) ? 1 : 0;
        const float *r = reinterpret_cast<const float *>(smem + L.ring + w * S * KS) + sl * 16;
        if (lane < 16) v += r[lane];
      }
      if (lane < 16) emit(t, lane, v);
    }
  }
  ab_arrive(cnt + grp);

  // ---- phase B: norm + RoPE of the group's vectors, attention over this CTA's slots ----
  const bool ok_a = ab_wait_count(cnt + grp, C, a.wait_ns, at.err, &flag);
  const bool ok_kv = mbar_wait_bounded(bar, 0);
  if (!ok_kv) {
    if (tid == 0) raise_error(at.err, kDevBarrierTimeout);
    mbar_wait_bounded(bar, 0);  // the copies still in flight land before the CTA leaves
  }
  if (bad_step && tid == 0 && blockIdx.x == 0) raise_error(at.err, kDevBadParams);
  float *const gq = reinterpret_cast<float *>(smem + Lb.gain);
  float *const gk = gq + D, *const sn = gk + D, *const cs = sn + D / 2;
  float *const qs = reinterpret_cast<float *>(smem + Lb.vec);
  float *const kn = qs + G * D, *const vn = kn + D;
  if (ok_a && ok_kv && warp < G + 2) {
    const int vi = warp;
    const float *src = vi < G ? yseg0 + (size_t)(grp * G + vi) * D
                              : (vi == G ? yseg1 : yseg2) + (size_t)grp * D;
    float *buf = vi < G ? qs + vi * D : (vi == G ? kn : vn);
    float x[DPL];
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < DPL; ++q) {
      x[q] = __ldcg(src + lane * DPL + q);
      ss = fmaf(x[q], x[q], ss);
    }
    ss = warp_sum(ss);
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), at.eps)));
#pragma unroll
    for (int q = 0; q < DPL; ++q) {
      const uint32_t e = lane * DPL + q;
      buf[e] = vi <= G ? __fmul_rn(__fmul_rn(x[q], rs), vi < G ? gq[e] : gk[e]) : __fmul_rn(x[q], rs);
    }
    __syncwarp();
    const uint32_t half = at.rotary_dim / 2;
    if (vi <= G) {
      for (uint32_t e = lane; e < half; e += 32) {
        const float v0 = buf[e], v1 = buf[e + half];
        buf[e] = __fsub_rn(__fmul_rn(v0, cs[e]), __fmul_rn(v1, sn[e]));
        buf[e + half] = __fadd_rn(__fmul_rn(v0, sn[e]), __fmul_rn(v1, cs[e]));
      }
      __syncwarp();
    }
    if (vi >= G) {
      void *cache = vi == G ? at.k_cache : at.v_cache;
      const size_t new_off = (size_t)slot * at.kv_dim + (size_t)grp * D;
      const bool wr = cta == 0 && slot < at.total_slots;
      for (uint32_t e = lane; e < D; e += 32) {
        if (BF16) {
          const uint16_t b = bf16_bits_rne(buf[e]);
          buf[e] = bf16_bits_to_f32(b);
          if (wr) reinterpret_cast<uint16_t *>(cache)[new_off + e] = b;
        } else if (wr) {
          reinterpret_cast<float *>(cache)[new_off + e] = buf[e];
        }
      }
    }
  }
  __syncthreads();
  float *const wm = reinterpret_cast<float *>(smem + L.ring);  // [16][G]
  float *const wl = wm + kWarps * G;                          // [16][G]
  float *const wo = wl + kWarps * G;                          // [16][G][D]
  {
    const uint8_t *const kv_sm = smem + Lb.kv;
    float q[G][DPL];
#pragma unroll
    for (int h = 0; h < G; ++h) ld_vec<DPL>(qs + h * D + lane * DPL, q[h]);
    bool live[kAbPerWarp], cur[kAbPerWarp];
    float sc[kAbPerWarp][G];
#pragma unroll
    for (int j = 0; j < kAbPerWarp; ++j) {
      const uint32_t li = warp + kWarps * j;
      const uint32_t sl = li < ns ? slot_s[li] : 0xFFFFFFFFu;
      live[j] = sl < at.total_slots && ok_a && ok_kv;
      cur[j] = sl == slot;
      if (li < ns && sl >= at.total_slots && lane == 0) raise_error(at.err, kDevBadSlot);
      float kv[DPL];
      if (cur[j]) {
        ld_vec<DPL>(kn + lane * DPL, kv);
      } else if (live[j]) {
        ab_ld_row<DPL, BF16>(kv_sm + (2 * li) * D * ESZ + lane * DPL * ESZ, kv);
      } else {
#pragma unroll
        for (int q0 = 0; q0 < DPL; ++q0) kv[q0] = 0.0f;
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        sc[j][h] = 0.0f;
#pragma unroll
        for (int q0 = 0; q0 < DPL; ++q0) sc[j][h] = fmaf(q[h][q0], kv[q0], sc[j][h]);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int j = 0; j < kAbPerWarp; ++j)
#pragma unroll
        for (int h = 0; h < G; ++h) sc[j][h] += __shfl_xor_sync(0xffffffffu, sc[j][h], off);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float mn = -INFINITY;
#pragma unroll
      for (int j = 0; j < kAbPerWarp; ++j) {
        sc[j][h] = live[j] ? sc[j][h] * at.scale : -INFINITY;
        mn = fmaxf(mn, sc[j][h]);
      }
      float p[kAbPerWarp], ps = 0.0f;
#pragma unroll
      for (int j = 0; j < kAbPerWarp; ++j) {
        p[j] = (live[j] && mn != -INFINITY) ? expf(sc[j][h] - mn) : 0.0f;
        ps += p[j];
      }
      float o[DPL];
#pragma unroll
      for (int q0 = 0; q0 < DPL; ++q0) o[q0] = 0.0f;
#pragma unroll
      for (int j = 0; j < kAbPerWarp; ++j) {
        if (p[j] == 0.0f) continue;
        const uint32_t li = warp + kWarps * j;
        float vv[DPL];
        if (cur[j]) {
          ld_vec<DPL>(vn + lane * DPL, vv);
        } else {
          ab_ld_row<DPL, BF16>(kv_sm + (2 * li + 1) * D * ESZ + lane * DPL * ESZ, vv);
        }
#pragma unroll
        for (int q0 = 0; q0 < DPL; ++q0) o[q0] = fmaf(p[j], vv[q0], o[q0]);
      }
      if (lane == 0) {
        wm[warp * G + h] = mn;
        wl[warp * G + h] = ps;
      }
      st_vec<DPL>(wo + (warp * G + h) * D + lane * DPL, o);
    }
  }
  __syncthreads();
  float *const rec_base = a.rec + (size_t)grp * C * G * (D + 2);
  attn_cta_merge<DPL, G, kWarps>(tid, wm, wl, wo, [&](uint32_t h, uint32_t d, float M, float Ls, float O) {
    float *r = rec_base + ((size_t)cta * G + h) * (D + 2);
    r[2 + d] = O;
    if (d == 0) {
      r[0] = M;
      r[1] = Ls;
    }
  });
  ab_arrive(cnt + nkv + grp);

  // ---- phase C: merge the group's records, o projection of the group's columns ----
  const bool ok_b = ab_wait_count(cnt + nkv + grp, C, a.wait_ns, at.err, &flag);
  float *const xo = reinterpret_cast<float *>(smem + Lb.mrg);  // [G][D] attention output
  float *const fw = xo + G * D;                                // [G][C] record maxima -> weights
  float *const fl = fw + G * C;                                // [G][C] record sums
  float *const ls = fl + G * C;                                // [G]
  if (ok_b) {
    for (uint32_t i = tid; i < G * C; i += kThreads) {
      const uint32_t h = i / C, r = i % C;
      const float *rr = rec_base + ((size_t)r * G + h) * (D + 2);
      fw[i] = __ldcg(rr);
      fl[i] = __ldcg(rr + 1);
    }
  }
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (uint32_t r = 0; r < C; ++r) M = fmaxf(M, fw[tid * C + r]);
    float Ls = 0.0f;
    for (uint32_t r = 0; r < C; ++r) {
      const float f = M == -INFINITY ? 0.0f : expf(fw[tid * C + r] - M);
      Ls = fmaf(fl[tid * C + r], f, Ls);
      fw[tid * C + r] = f;
    }
    ls[tid] = Ls;
  }
  __syncthreads();
  for (uint32_t idx = tid; idx < G * D; idx += kThreads) {
    const uint32_t h = idx / D, d = idx % D;
    const float *base = rec_base + (size_t)h * (D + 2) + 2 + d;
    const float *f = fw + h * C;
    float O = 0.0f;
    // up to 32 records' loads in flight, then the weighted sum in record order
    for (uint32_t r0 = 0; r0 < C; r0 += 32) {
      float rv[32];
#pragma unroll
      for (int r = 0; r < 32; ++r)
        rv[r] = r0 + r < C ? __ldcg(base + (size_t)(r0 + r) * G * (D + 2)) : 0.0f;
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (r0 + r < C) O = fmaf(rv[r], f[r0 + r], O);
    }
    const float Ls = ls[h];
    xo[idx] = (ok_b && Ls > 0.0f) ? O / Ls : 0.0f;
  }
  __syncthreads();
  {
    GemvArgs go = ga;
    go.k = G * D;
    go.batch = 1;
    stage_x<4>(go, xo, G * D, smem + Lb.ofrag, Lb.o, false);
    const uint8_t *const osm = smem + Lb.ofrag;
    const uint4 *const xf4 = reinterpret_cast<const uint4 *>(osm + Lb.o.xfrag);
    const float *const corr = reinterpret_cast<const float *>(osm + Lb.o.corr);
    const float xs = reinterpret_cast<const float *>(osm + Lb.o.misc)[0];
    const uint8_t *const wsm = smem + Lb.wo;
    const uint32_t xoff = (g * 4 + c) * 2, coff = c * 2;
    float *const out = a.opart + (size_t)grp * a.o_rows;
    for (uint32_t lt = warp; lt < no; lt += kWarps) {
      float acc[2] = {0.0f, 0.0f};
      uint4 xb[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      float cr[2] = {0.0f, 0.0f};
#pragma unroll 2
      for (uint32_t p = 0; p < GP; ++p) {
        const uint8_t *ch = wsm + ((size_t)lt * GP + p) * CB;
        if (g < 2) {
          xb[0] = xf4[p * 16 + xoff];
          xb[1] = xf4[p * 16 + xoff + 1];
        }
        if (c == 0) {
          const float2 c2 = *reinterpret_cast<const float2 *>(corr + p * 2 + coff);
          cr[0] = c2.x;
          cr[1] = c2.y;
        }
        const float4 sc = *reinterpret_cast<const float4 *>(ch + SO + g * 16);
        const uint4 wq = *reinterpret_cast<const uint4 *>(ch + lane * 16);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          uint32_t a0[4], a1[4], rg[4], rg8[4];
          dq4_word(hb ? wq.z : wq.x, rg);
          dq4_word(hb ? wq.w : wq.y, rg8);
          a0[0] = rg[0]; a0[1] = rg8[0]; a0[2] = rg[1]; a0[3] = rg8[1];
          a1[0] = rg[2]; a1[1] = rg8[2]; a1[2] = rg[3]; a1[3] = rg8[3];
          block_mma<4>(a0, a1, xb[hb], cr[hb], hb ? sc.z : sc.x, hb ? sc.w : sc.y, acc);
        }
      }
      if (c == 0) {
        out[(ot0 + lt) * 16 + g] = acc[0] * xs;
        out[(ot0 + lt) * 16 + g + 8] = acc[1] * xs;
      }
    }
  }

  // ---- the last CTA to leave clears the layer's counters (every wait has been passed) ----
  __syncthreads();
  if (tid == 0) {
    const uint32_t total = C * nkv;
    if (atomicAdd(cnt + 2 * nkv, 1u) + 1 == total) {
      for (uint32_t i = 0; i < 2 * nkv; ++i) cnt[i] = 0;
      __threadfence();
      cnt[2 * nkv] = 0;
    }
  }
}

template <int DPL, int G, bool BF16>
cudaError_t launch_ab_t(const AttnBlockArgs &a, cudaStream_t s) {
  const AbLayout L = ab_layout(a.g.k, G, 32 * DPL, a.ctas, a.max_slots, a.o_tiles, BF16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.ctas * a.at.num_kv);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_block_kernel<DPL, G, BF16>, a);
}

template <int DPL, int G>
cudaError_t launch_ab_g(const AttnBlockArgs &a, cudaStream_t s) {
  return a.at.kv_bf16 ? launch_ab_t<DPL, G, true>(a, s) : launch_ab_t<DPL, G, false>(a, s);
}

template <int DPL>
cudaError_t launch_ab_d(const AttnBlockArgs &a, cudaStream_t s) {
  switch (a.at.num_q / a.at.num_kv) {
    case 1: return launch_ab_g<DPL, 1>(a, s);
    case 2: return launch_ab_g<DPL, 2>(a, s);
    case 4: return launch_ab_g<DPL, 4>(a, s);
    case 8: return launch_ab_g<DPL, 8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

template <int DPL, int G>
cudaError_t prepare_ab_g() {
  cudaError_t e = allow_max_dynamic_smem(attn_block_kernel<DPL, G, true>);
  return e != cudaSuccess ? e : allow_max_dynamic_smem(attn_block_kernel<DPL, G, false>);
}
template <int DPL>
cudaError_t prepare_ab_d() {
  cudaError_t r[4] = {prepare_ab_g<DPL, 1>(), prepare_ab_g<DPL, 2>(), prepare_ab_g<DPL, 4>(),
                      prepare_ab_g<DPL, 8>()};
  for (cudaError_t x : r)
    if (x != cudaSuccess) return x;
  return cudaSuccess;
}

}  // namespace

bool attn_block_plan(uint32_t hidden, uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
                     uint32_t total_slots, bool kv_bf16, int num_sms, uint32_t smem_limit,
                     AttnBlockPlan *plan) {
  if (num_kv == 0 || num_kv > (uint32_t)kProMaxParts || num_q % num_kv != 0) return false;
  const uint32_t G = num_q / num_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return false;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return false;
  if (hidden % 64 != 0 || hidden > kGemvPrologueMaxK || (G * head_dim) % 64 != 0) return false;
  const uint32_t ctas = (uint32_t)num_sms / num_kv;
  if (ctas == 0) return false;
  const uint32_t max_slots = (total_slots + ctas - 1) / ctas;
  if (max_slots > kAbMaxSlotsPerCta) return false;
  const uint32_t o_tiles = (hidden / 16 + ctas - 1) / ctas;
  const AbLayout L = ab_layout(hidden, G, head_dim, ctas, max_slots, o_tiles, kv_bf16);
  if (L.total > smem_limit) return false;
  plan->ctas = ctas;
  plan->max_slots = max_slots;
  plan->o_tiles = o_tiles;
  plan->smem = L.total;
  return true;
}

cudaError_t launch_attn_block(const AttnBlockArgs &a, cudaStream_t s) {
  switch (a.at.head_dim) {
    case 64: return launch_ab_d<2>(a, s);
    case 128: return launch_ab_d<4>(a, s);
    case 256: return launch_ab_d<8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prepare_attn_block_kernels() {
  cudaError_t r[3] = {prepare_ab_d<2>(), prepare_ab_d<4>(), prepare_ab_d<8>()};
  for (cudaError_t x : r)
    if (x != cudaSuccess) return x;
  return cudaSuccess;
}

}  // namespace sx
