// sx_attn_dev.cuh -- device code of the fused decode attention work item, shared by its own
// kernel (sx_ops.cu) and the persistent decode kernel (sx_persist.cu).
#pragma once
#include <cooperative_groups.h>

#include "sx_common.cuh"
#include "sx_internal.h"

namespace sx {
namespace {

constexpr int kAttnChunk = 32;  // ring slots per work item / partial record

// Fused decode attention: qkv_rope + decode_attn (+ the combine) as one work item per (kv head
// h, 32-slot chunk), run by a group of 256 threads (8 warps of 4 slots each) that synchronises
// on its own named barrier:
//   1. before waiting for the QKV projection (the wait hook: griddepcontrol.wait in a kernel of
//      its own, a grid barrier in the persistent decode kernel), every warp reads its 4 slot
//      indices and fetches their K/V rows into registers.  The step word, the slot list and
//      every cache row but the current slot's were written before the token started (host
//      copies, earlier tokens), so the fetch overlaps the end of the projection;
//   2. one warp per vector normalises and rotates the GQA group's q heads and the new k, v of
//      head h (qkv_rope.wgsl semantics, identical rounding to the cache); chunk 0 stores the
//      new K/V at the current slot, whose row every CTA takes from shared memory;
//   3. each warp folds its 4 slots into an online softmax in one step, the CTA merges its
//      warps, and the last CTA of the head merges the chunk partials in chunk order.
constexpr int kFusedWarps = 8;
constexpr int kFusedPerWarp = 4;
static_assert(kFusedWarps * kFusedPerWarp == kAttnChunk, "fused chunk must match the scratch");

// One cache row slice of a lane in its storage format (bf16 pairs or f32 words).
template <int DPL, bool BF16>
struct RawRow {
  static constexpr int kWords = BF16 ? DPL / 2 : DPL;
  uint32_t w[kWords];
};

template <int DPL, bool BF16>
SX_DEV void load_raw(const void *cache, size_t off, int lane, RawRow<DPL, BF16> &r) {
  constexpr int kBytes = RawRow<DPL, BF16>::kWords * 4;
  const char *p = reinterpret_cast<const char *>(cache) + (off + (size_t)lane * DPL) * (BF16 ? 2 : 4);
  if constexpr (kBytes % 16 == 0) {
#pragma unroll
    for (int i = 0; i < kBytes / 16; ++i) {
      uint4 u = __ldcg(reinterpret_cast<const uint4 *>(p) + i);
      r.w[4 * i] = u.x; r.w[4 * i + 1] = u.y; r.w[4 * i + 2] = u.z; r.w[4 * i + 3] = u.w;
    }
  } else if constexpr (kBytes == 8) {
    uint2 u = __ldcg(reinterpret_cast<const uint2 *>(p));
    r.w[0] = u.x; r.w[1] = u.y;
  } else {
    static_assert(kBytes == 4, "head_dim must be 64, 128, 256 or 512");
    r.w[0] = __ldcg(reinterpret_cast<const uint32_t *>(p));
  }
}

template <int DPL, bool BF16>
SX_DEV float raw_at(const RawRow<DPL, BF16> &r, int i) {
  if (BF16) return u2f((i & 1) ? (r.w[i >> 1] & 0xFFFF0000u) : (r.w[i >> 1] << 16));
  return u2f(r.w[i]);
}

// named barrier of one 256-thread work group (id 0 is the whole CTA's barrier)
SX_DEV void group_sync(int bar) { asm volatile("bar.sync %0, 256;\n" ::"r"(bar) : "memory"); }

// Shared memory of one global-merge work item, in floats.
SX_HD uint32_t attn_item_floats(int g, uint32_t d, uint32_t nchunks) {
  return g * d + 2 * d + 2 * kFusedWarps * g + kFusedWarps * g * d + g * nchunks + g;
}

// Everything a warp can fetch or compute before the q|k|v projection is ready: the slot list
// entries and K/V rows of its P slots, this lane's q/k norm gains and the RoPE sin/cos of the
// rotary pairs i = lane + 32 k (they depend only on the clock).
template <int DPL, bool BF16, int P>
struct AttnPre {
  static constexpr int KR = DPL / 2 > 0 ? DPL / 2 : 1;  // rotary pairs per lane (half <= D/2)
  uint32_t sl[P];
  RawRow<DPL, BF16> kr[P], vr[P];
  float qg[DPL], kg[DPL], sn[KR], cs[KR];
};

// v[0..DPL) = p[0..DPL) for 8- or 16-byte aligned p (shared or global)
template <int DPL>
SX_DEV void ld_vec(const float *p, float (&v)[DPL]) {
  if constexpr (DPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < DPL; i += 4) {
      const float4 u = *reinterpret_cast<const float4 *>(p + i);
      v[i] = u.x; v[i + 1] = u.y; v[i + 2] = u.z; v[i + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < DPL; i += 2) {
      const float2 u = *reinterpret_cast<const float2 *>(p + i);
      v[i] = u.x; v[i + 1] = u.y;
    }
  }
}
template <int DPL>
SX_DEV void st_vec(float *p, const float (&v)[DPL]) {
  if constexpr (DPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < DPL; i += 4)
      *reinterpret_cast<float4 *>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < DPL; i += 2) *reinterpret_cast<float2 *>(p + i) = make_float2(v[i], v[i + 1]);
  }
}

// Warp `warp` (of W) of the item owning slots [s0, s1): slots s0 + warp + j W, j < P.
template <int DPL, bool BF16, int P, int W>
SX_DEV void attn_fetch(const AttnFusedArgs &a, uint32_t kvh, uint32_t s0, uint32_t s1,
                       uint32_t slot, int warp, int lane, AttnPre<DPL, BF16, P> &R) {
  constexpr uint32_t D = 32 * DPL;
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const uint32_t si = s0 + warp + j * W;
    R.sl[j] = si < s1 ? __ldcg(a.slots + si) : 0xFFFFFFFFu;
  }
#pragma unroll
  for (int j = 0; j < P; ++j) {
    if (R.sl[j] < a.total_slots && R.sl[j] != slot) {
      const size_t off = (size_t)R.sl[j] * a.kv_dim + (size_t)kvh * D;
      load_raw<DPL, BF16>(a.k_cache, off, lane, R.kr[j]);
      load_raw<DPL, BF16>(a.v_cache, off, lane, R.vr[j]);
    } else {
#pragma unroll
      for (int i = 0; i < RawRow<DPL, BF16>::kWords; ++i) R.kr[j].w[i] = R.vr[j].w[i] = 0u;
    }
  }
  ld_vec<DPL>(a.q_norm_w + lane * DPL, R.qg);
  ld_vec<DPL>(a.k_norm_w + lane * DPL, R.kg);
  const uint32_t half = a.rotary_dim / 2;
  const float fclock = (float)a.step[0];
#pragma unroll
  for (int k = 0; k < AttnPre<DPL, BF16, P>::KR; ++k) {
    const uint32_t i = lane + 32 * k;
    R.sn[k] = 0.0f;
    R.cs[k] = 1.0f;
    if (i < half) sincosf(__fmul_rn(fclock, a.inv_freq[i]), &R.sn[k], &R.cs[k]);
  }
}

// One warp per vector: the G q heads of kv head kvh and its new k, v are RMS-normalised
// (q/k with their gains, v without), q and k rotated over the first rotary_dim elements
// (qkv_rope.wgsl semantics, same rounding as the cache), k and v rounded to the cache
// precision; the item that writes_cache stores them at the current slot.
template <int DPL, int G, bool BF16, int P, int W>
SX_DEV void attn_norm_rope(const AttnFusedArgs &a, uint32_t kvh, bool writes_cache,
                           uint32_t slot, int warp, int lane, const AttnPre<DPL, BF16, P> &R,
                           float *qs, float *kn, float *vn) {
  constexpr uint32_t D = 32 * DPL;
  const uint32_t half = a.rotary_dim / 2;
  const bool slot_ok = slot < a.total_slots;
  for (int vi = warp; vi < G + 2; vi += W) {
    const float *src = vi < G ? a.q + (size_t)(kvh * G + vi) * D
                              : (vi == G || a.k_eq_v ? a.k : a.v) + (size_t)kvh * D;
    float *buf = vi < G ? qs + vi * D : (vi == G ? kn : vn);
    float x[DPL];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      x[i] = __ldcg(src + lane * DPL + i);
      ss = fmaf(x[i], x[i], ss);
    }
    ss = warp_sum(ss);
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps)));
    float y[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const float g = vi < G ? R.qg[i] : R.kg[i];
      y[i] = vi <= G ? __fmul_rn(__fmul_rn(x[i], rs), g) : __fmul_rn(x[i], rs);
    }
    st_vec<DPL>(buf + lane * DPL, y);
    __syncwarp();
    if (vi <= G) {
#pragma unroll
      for (int k = 0; k < AttnPre<DPL, BF16, P>::KR; ++k) {
        const uint32_t i = lane + 32 * k;
        if (i < half) {
          const float v0 = buf[i], v1 = buf[i + half];
          buf[i] = __fsub_rn(__fmul_rn(v0, R.cs[k]), __fmul_rn(v1, R.sn[k]));
          buf[i + half] = __fadd_rn(__fmul_rn(v0, R.sn[k]), __fmul_rn(v1, R.cs[k]));
        }
      }
      __syncwarp();
    }
    if (vi >= G) {
      void *cache = vi == G ? a.k_cache : a.v_cache;
      const size_t new_off = ((size_t)slot * a.num_kv + kvh) * D;
      for (uint32_t d = lane; d < D; d += 32) {
        if (BF16) {
          const uint16_t b = bf16_bits_rne(buf[d]);
          buf[d] = bf16_bits_to_f32(b);
          if (writes_cache && slot_ok) reinterpret_cast<uint16_t *>(cache)[new_off + d] = b;
        } else if (writes_cache && slot_ok) {
          reinterpret_cast<float *>(cache)[new_off + d] = buf[d];
        }
      }
    }
  }
}

// Online softmax of the warp's P slots, folded in one step, for the G q heads; the warp's
// (m, l, o) go to wm / wl / wo.  The current slot's K/V come from kn / vn (it is being written
// in this very step), every other row from the registers fetched before the wait.
template <int DPL, int G, bool BF16, int P>
SX_DEV void attn_softmax(const AttnFusedArgs &a, uint32_t slot, int warp, int lane,
                         const AttnPre<DPL, BF16, P> &R, const float *qs, const float *kn,
                         const float *vn, float *wm, float *wl, float *wo) {
  constexpr uint32_t D = 32 * DPL;
  float q[G][DPL];
#pragma unroll
  for (int h = 0; h < G; ++h) ld_vec<DPL>(qs + h * D + lane * DPL, q[h]);
  bool live[P], cur[P];
  float sc[P][G];
#pragma unroll
  for (int j = 0; j < P; ++j) {
    live[j] = R.sl[j] < a.total_slots;
    cur[j] = R.sl[j] == slot;
    if (!live[j] && R.sl[j] != 0xFFFFFFFFu && lane == 0) raise_error(a.err, kDevBadSlot);
    float kv[DPL];
    if (cur[j]) {
      ld_vec<DPL>(kn + lane * DPL, kv);
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) kv[i] = raw_at<DPL, BF16>(R.kr[j], i);
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      sc[j][h] = 0.0f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) sc[j][h] = fmaf(q[h][i], kv[i], sc[j][h]);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int j = 0; j < P; ++j)
#pragma unroll
      for (int h = 0; h < G; ++h) sc[j][h] += __shfl_xor_sync(0xffffffffu, sc[j][h], off);
  float vcur[DPL];
  ld_vec<DPL>(vn + lane * DPL, vcur);
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float mn = -INFINITY;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      sc[j][h] = live[j] ? sc[j][h] * a.scale : -INFINITY;
      mn = fmaxf(mn, sc[j][h]);
    }
    float p[P], ps = 0.0f;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      p[j] = (live[j] && mn != -INFINITY) ? expf(sc[j][h] - mn) : 0.0f;
      ps += p[j];
    }
    float o[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < P; ++j) acc = fmaf(p[j], cur[j] ? vcur[i] : raw_at<DPL, BF16>(R.vr[j], i), acc);
      o[i] = acc;
    }
    if (lane == 0) {
      wm[warp * G + h] = mn;
      wl[warp * G + h] = ps;
    }
    st_vec<DPL>(wo + (warp * G + h) * D + lane * DPL, o);
  }
}

// Merge of the W warps' (m, l, o) into one (M, L, O[d]) per q head; emit(h, d, M, L, O).
template <int DPL, int G, int W, typename Emit>
SX_DEV void attn_cta_merge(int t, const float *wm, const float *wl, const float *wo, Emit emit) {
  constexpr uint32_t D = 32 * DPL;
  for (uint32_t idx = t; idx < G * D; idx += W * 32) {
    const uint32_t h = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, wm[w * G + h]);
    float Lsum = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float f = M == -INFINITY ? 0.0f : expf(wm[w * G + h] - M);
      Lsum = fmaf(wl[w * G + h], f, Lsum);
      O = fmaf(wo[(w * G + h) * D + d], f, O);
    }
    emit(h, d, M, Lsum, O);
  }
}

// Work item (kvh, chunk) of nchunks for the thread t in [0, 256) of its group, merged through
// global memory: each item publishes one record per q head and the last item of the head to
// arrive merges the chunk records in chunk order.  active = false: the group only takes part
// in wait() (which may be a CTA-wide barrier).
template <int DPL, int G, bool BF16, typename Wait>
SX_DEV void attn_item(const AttnFusedArgs &a, uint32_t kvh, uint32_t chunk, uint32_t nchunks,
                      float *sh, uint32_t *last_flag, int t, int bar, bool active, Wait wait) {
  if (!active) {
    wait();
    return;
  }
  constexpr int W = kFusedWarps, P = kFusedPerWarp;
  constexpr uint32_t D = 32 * DPL;
  const int warp = t >> 5, lane = t & 31;
  float *qs = sh;                  // [G][D] normalised, rotated q
  float *kn = qs + G * D;          // [D] new K (cache precision)
  float *vn = kn + D;              // [D] new V (cache precision)
  float *wm = vn + D;              // [W][G]
  float *wl = wm + W * G;          // [W][G]
  float *wo = wl + W * G;          // [W][G][D]
  float *cf = wo + W * G * D;      // [G][nchunks] combine weights, then [G] sums

  const uint32_t slot = a.step[1];
  uint32_t S = a.step[2];
  const bool bad_step = S > a.total_slots || slot >= a.total_slots;
  S = S > a.total_slots ? a.total_slots : S;

  AttnPre<DPL, BF16, P> R;
  const uint32_t s0 = chunk * kAttnChunk, s1 = min(S, s0 + kAttnChunk);
  attn_fetch<DPL, BF16, P, W>(a, kvh, s0, s1, slot, warp, lane, R);
  wait();
  if (bad_step && t == 0 && chunk == 0 && kvh == 0) raise_error(a.err, kDevBadParams);
  attn_norm_rope<DPL, G, BF16, P, W>(a, kvh, chunk == 0, slot, warp, lane, R, qs, kn, vn);
  group_sync(bar);
  attn_softmax<DPL, G, BF16, P>(a, slot, warp, lane, R, qs, kn, vn, wm, wl, wo);
  group_sync(bar);
  attn_cta_merge<DPL, G, W>(t, wm, wl, wo, [&](uint32_t h, uint32_t d, float M, float L, float O) {
    float *rec = a.part + ((size_t)(kvh * G + h) * nchunks + chunk) * (D + 2);
    rec[2 + d] = O;
    if (d == 0) {
      rec[0] = M;
      rec[1] = L;
    }
  });

  // last CTA of this kv head merges the chunks
  __threadfence();
  group_sync(bar);
  if (t == 0) *last_flag = (atomicAdd(&a.cnt[kvh], 1u) + 1 == nchunks) ? 1u : 0u;
  group_sync(bar);
  if (!*last_flag) return;
  __threadfence();
  float *csum = cf + G * nchunks;
  for (int h = warp; h < G; h += W) {
    const float *base = a.part + (size_t)(kvh * G + h) * nchunks * (D + 2);
    float M = -INFINITY;
    for (uint32_t c = lane; c < nchunks; c += 32) M = fmaxf(M, __ldcg(base + (size_t)c * (D + 2)));
    M = warp_max(M);
    float L = 0.0f;
    for (uint32_t c = lane; c < nchunks; c += 32) {
      const float *rec = base + (size_t)c * (D + 2);
      const float f = M == -INFINITY ? 0.0f : expf(__ldcg(rec) - M);
      cf[h * nchunks + c] = f;
      L = fmaf(__ldcg(rec + 1), f, L);
    }
    L = warp_sum(L);
    if (lane == 0) csum[h] = L;
  }
  group_sync(bar);
  for (uint32_t idx = t; idx < G * D; idx += W * 32) {
    const uint32_t h = idx / D, d = idx % D;
    const float *base = a.part + (size_t)(kvh * G + h) * nchunks * (D + 2) + 2 + d;
    const float *f = cf + h * nchunks;
    float O = 0.0f;
#pragma unroll 8
    for (uint32_t c = 0; c < nchunks; ++c) O = fmaf(__ldcg(base + (size_t)c * (D + 2)), f[c], O);
    const float L = csum[h];
    a.out[(size_t)(kvh * G + h) * D + d] = L > 0.0f ? O / L : 0.0f;
  }
  if (t == 0) a.cnt[kvh] = 0;
}

// ---------------------------------------------------------------------------------------
// Cluster form: the CL CTAs of kv head kvh form one thread-block cluster, CTA `rank` owning
// slots [rank * 64, rank * 64 + 64) (8 warps x 8 slots).  After the CTA merge each CTA keeps
// its (M, L, O[D]) per q head in its own shared memory; the cluster synchronises and CTA r
// merges the slice r of the G x D outputs from all CL records over distributed shared memory,
// in rank order.  No global scratch, fences or atomics.
constexpr int kClusterPerWarp = 8;
constexpr int kClusterSlots = kFusedWarps * kClusterPerWarp;  // 64
constexpr int kClusterMax = 16;                               // non-portable cluster size

SX_HD uint32_t attn_cluster_floats(int g, uint32_t d, uint32_t cl) {
  // qs, kn, vn, wm, wl, wo, rec [G][D + 2], weights [G][CL], sums [G], record sums [G][CL]
  return g * d + 2 * d + 2 * kFusedWarps * g + kFusedWarps * g * d + g * (d + 2) + g * cl + g +
         g * cl;
}

// The cluster merge of attn_cluster_item: every CTA holds its (M, L, O[D]) per q head in
// rec [G][D + 2]; after the cluster barrier CTA r merges slice r of the G x D outputs from all
// CL records over distributed shared memory, in rank order.
template <int G, uint32_t D, int W>
SX_DEV void attn_cluster_merge(const AttnFusedArgs &a, uint32_t kvh, float *rec, float *fw,
                               float *ls, float *fl, int t) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const uint32_t rank = cl.block_rank(), ncl = cl.num_blocks();
  cl.sync();
  // weights of the CL records per head: every CTA reads all CL x G (M, L) pairs at once
  // (independent remote reads), then one thread per head folds them locally in record order
  for (uint32_t i = t; i < G * ncl; i += W * 32) {
    const uint32_t h = i / ncl, r = i % ncl;
    const float *rr = cl.map_shared_rank(rec, r) + h * (D + 2);
    fw[i] = rr[0];
    fl[i] = rr[1];
  }
  __syncthreads();
  if (t < G) {
    float M = -INFINITY;
    for (uint32_t r = 0; r < ncl; ++r) M = fmaxf(M, fw[t * ncl + r]);
    float L = 0.0f;
    for (uint32_t r = 0; r < ncl; ++r) {
      const float f = M == -INFINITY ? 0.0f : expf(fw[t * ncl + r] - M);
      L = fmaf(fl[t * ncl + r], f, L);
      fw[t * ncl + r] = f;
    }
    ls[t] = L;
  }
  __syncthreads();
  // this CTA's slice of the G x D outputs: the CL remote values of an output are loaded
  // together, then summed in record order
  const uint32_t per = (G * D + ncl - 1) / ncl, lo = rank * per, hi = min(G * D, lo + per);
  for (uint32_t idx = lo + t; idx < hi; idx += W * 32) {
    const uint32_t h = idx / D, d = idx % D;
    float v[kClusterMax];
#pragma unroll
    for (uint32_t r = 0; r < (uint32_t)kClusterMax; ++r)
      v[r] = r < ncl ? cl.map_shared_rank(rec, r)[h * (D + 2) + 2 + d] : 0.0f;
    float O = 0.0f;
#pragma unroll
    for (uint32_t r = 0; r < (uint32_t)kClusterMax; ++r)
      if (r < ncl) O = fmaf(v[r], fw[h * ncl + r], O);
    const float L = ls[h];
    a.out[(size_t)(kvh * G + h) * D + d] = L > 0.0f ? O / L : 0.0f;
  }
  cl.sync();  // the records stay readable until every CTA of the cluster is done
}

// CP: ring slots per warp (the CTA owns kFusedWarps * CP slots; the cluster kernel uses
// kClusterPerWarp, the attention + o kernel fewer for more CTAs per kv head)
template <int DPL, int G, bool BF16, typename Wait, int CP = kClusterPerWarp>
SX_DEV void attn_cluster_item(const AttnFusedArgs &a, uint32_t kvh, float *sh, Wait wait) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  constexpr int W = kFusedWarps, P = CP;
  constexpr uint32_t D = 32 * DPL;
  const uint32_t rank = cl.block_rank(), ncl = cl.num_blocks();
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  float *qs = sh;
  float *kn = qs + G * D;
  float *vn = kn + D;
  float *wm = vn + D;
  float *wl = wm + W * G;
  float *wo = wl + W * G;
  float *rec = wo + W * G * D;      // [G][D + 2]: M, L, O[D]
  float *fw = rec + G * (D + 2);    // [G][CL]
  float *ls = fw + G * ncl;         // [G]
  float *fl = ls + G;               // [G][CL]: the records' L

  const uint32_t slot = a.step[1];
  uint32_t S = a.step[2];
  const bool bad_step = S > a.total_slots || slot >= a.total_slots;
  S = S > a.total_slots ? a.total_slots : S;

  AttnPre<DPL, BF16, P> R;
  const uint32_t s0 = rank * (W * P), s1 = min(S, s0 + W * P);
  attn_fetch<DPL, BF16, P, W>(a, kvh, s0, s1, slot, warp, lane, R);
  wait();
  if (bad_step && t == 0 && rank == 0 && kvh == 0) raise_error(a.err, kDevBadParams);
  attn_norm_rope<DPL, G, BF16, P, W>(a, kvh, rank == 0, slot, warp, lane, R, qs, kn, vn);
  __syncthreads();
  attn_softmax<DPL, G, BF16, P>(a, slot, warp, lane, R, qs, kn, vn, wm, wl, wo);
  __syncthreads();
  attn_cta_merge<DPL, G, W>(t, wm, wl, wo, [&](uint32_t h, uint32_t d, float M, float L, float O) {
    rec[h * (D + 2) + 2 + d] = O;
    if (d == 0) {
      rec[h * (D + 2)] = M;
      rec[h * (D + 2) + 1] = L;
    }
  });
  attn_cluster_merge<G, D, W>(a, kvh, rec, fw, ls, fl, t);
}

// ---------------------------------------------------------------------------------------
// Tensor-core form of the cluster work item for 8 q heads per kv head, head_dim 256 and a
// bf16 cache (the shape of configs 3 and 5), run by the same 256 threads and cluster merge.
// Before the dependency wait the CTA gathers its 64 slots' K and V rows into padded shared
// rows with cp.async and stages the norm gains and the RoPE table; after it, one warp per
// vector normalises and rotates the 8 q heads and the new k / v (qkv_rope.wgsl semantics, as
// attn_norm_rope), q goes to shared memory as bf16 hi + lo rows 0..7 of a 16-row tile (rows
// 8..15 zero), the current slot's row takes the new k / v, and
//   S = Q K^T: warp w forms keys 8w..8w+7 for all 16 rows (mma.m16n8k16, bf16, f32 acc);
//   the CTA's per-head maximum and sum over its 64 keys meet in shared memory;
//   O = P V: warp w forms head_dim columns 32w..32w+31 (P split hi + lo, V by ldmatrix.trans);
// and the CTA's (M, L, O) per head goes to the cluster merge.
constexpr uint32_t kTcaStride = 528;  // bytes per shared row: 256 bf16 + 16 pad
struct TcaLayout {
  static constexpr uint32_t kt = 0, vt = kt + 64 * kTcaStride, qh = vt + 64 * kTcaStride,
                            ql = qh + 16 * kTcaStride, qs = ql + 16 * kTcaStride,
                            kn = qs + 8 * 256 * 4, vn = kn + 256 * 4, qg = vn + 256 * 4,
                            kg = qg + 256 * 4, sn = kg + 256 * 4, cs = sn + 128 * 4,
                            sp = cs + 128 * 4, wmax = sp + 8 * 64 * 4, wsum = wmax + 8 * 8 * 4,
                            rec = wsum + 8 * 8 * 4, fw = rec + 8 * 258 * 4,
                            fl = fw + 8 * kClusterMax * 4, ls = fl + 8 * kClusterMax * 4,
                            slots = ls + 8 * 4, misc = slots + 64 * 4, total = misc + 16;
};
SX_DEV void tca_ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                              uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
SX_DEV void tca_split(float x0, float x1, uint32_t &hi, uint32_t &lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  hi = *reinterpret_cast<const uint32_t *>(&h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(__fsub_rn(x0, __low2float(h)), __fsub_rn(x1, __high2float(h)));
  lo = *reinterpret_cast<const uint32_t *>(&l);
}

template <typename Wait>
SX_DEV void attn_cluster_item_tc(const AttnFusedArgs &a, uint32_t kvh, float *sh, Wait wait) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  constexpr int G = 8, W = kFusedWarps;
  constexpr uint32_t D = 256;
  using TL = TcaLayout;
  uint8_t *const sm = reinterpret_cast<uint8_t *>(sh);
  const uint32_t rank = cl.block_rank();
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, g = lane >> 2, c = lane & 3;
  uint32_t *const slot_s = reinterpret_cast<uint32_t *>(sm + TL::slots);
  uint32_t *const cur_s = reinterpret_cast<uint32_t *>(sm + TL::misc);
  float *const qs = reinterpret_cast<float *>(sm + TL::qs);
  float *const kn = reinterpret_cast<float *>(sm + TL::kn);
  float *const vn = reinterpret_cast<float *>(sm + TL::vn);
  float *const qg = reinterpret_cast<float *>(sm + TL::qg);
  float *const kg = reinterpret_cast<float *>(sm + TL::kg);
  float *const sn = reinterpret_cast<float *>(sm + TL::sn);
  float *const cs = reinterpret_cast<float *>(sm + TL::cs);
  float *const sp = reinterpret_cast<float *>(sm + TL::sp);
  float *const wmax = reinterpret_cast<float *>(sm + TL::wmax);
  float *const wsum = reinterpret_cast<float *>(sm + TL::wsum);
  float *const rec = reinterpret_cast<float *>(sm + TL::rec);

  const uint32_t slot = a.step[1];
  uint32_t S = a.step[2];
  const bool bad_step = S > a.total_slots || slot >= a.total_slots;
  S = S > a.total_slots ? a.total_slots : S;
  const uint32_t s0 = rank * kClusterSlots, s1 = min(S, s0 + kClusterSlots);
  const uint32_t ns = s1 > s0 ? s1 - s0 : 0;

  // 1. slot indices, K / V rows, norm gains and the RoPE table (none depends on q|k|v)
  if (t == 0) *cur_s = 0xFFFFFFFFu;
  __syncthreads();
  if (t < kClusterSlots) {
    const uint32_t sl = (uint32_t)t < ns ? __ldcg(a.slots + s0 + t) : 0xFFFFFFFFu;
    slot_s[t] = sl;
    if (sl == slot) *cur_s = (uint32_t)t;
  }
  __syncthreads();
  for (uint32_t q = t; q < kClusterSlots * 32; q += W * 32) {
    const uint32_t li = q >> 5, ch = q & 31, sl = slot_s[li];
    uint8_t *kd = sm + TL::kt + li * kTcaStride + ch * 16;
    uint8_t *vd = sm + TL::vt + li * kTcaStride + ch * 16;
    if (sl < a.total_slots && sl != slot) {
      const size_t off = ((size_t)sl * a.kv_dim + (size_t)kvh * D) * 2 + ch * 16;
      cp_async16(smem_u32(kd), static_cast<const uint8_t *>(a.k_cache) + off);
      cp_async16(smem_u32(vd), static_cast<const uint8_t *>(a.v_cache) + off);
    } else {
      *reinterpret_cast<uint4 *>(kd) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4 *>(vd) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
  const uint32_t half = a.rotary_dim / 2;
  const float fclock = (float)a.step[0];
  for (uint32_t i = t; i < D; i += W * 32) {
    qg[i] = a.q_norm_w[i];
    kg[i] = a.k_norm_w[i];
  }
  for (uint32_t i = t; i < D / 2; i += W * 32) {
    float sv = 0.0f, cv = 1.0f;
    if (i < half) sincosf(__fmul_rn(fclock, a.inv_freq[i]), &sv, &cv);
    sn[i] = sv;
    cs[i] = cv;
  }
  wait();
  if (bad_step && t == 0 && rank == 0 && kvh == 0) raise_error(a.err, kDevBadParams);
  __syncthreads();
  // 2. q / k norm + RoPE, k / v in the cache precision; rank 0 stores the new k / v
  const bool slot_ok = slot < a.total_slots;
  for (int vi = warp; vi < G + 2; vi += W) {
    const float *src = vi < G ? a.q + (size_t)(kvh * G + vi) * D
                              : (vi == G || a.k_eq_v ? a.k : a.v) + (size_t)kvh * D;
    float *buf = vi < G ? qs + vi * D : (vi == G ? kn : vn);
    float x[8];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = __ldcg(src + lane * 8 + i);
      ss = fmaf(x[i], x[i], ss);
    }
    ss = warp_sum(ss);
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps)));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t e = lane * 8 + i;
      buf[e] = vi <= G ? __fmul_rn(__fmul_rn(x[i], rs), vi < G ? qg[e] : kg[e]) : __fmul_rn(x[i], rs);
    }
    __syncwarp();
    if (vi <= G) {
      for (uint32_t e = lane; e < half; e += 32) {
        const float v0 = buf[e], v1 = buf[e + half];
        buf[e] = __fsub_rn(__fmul_rn(v0, cs[e]), __fmul_rn(v1, sn[e]));
        buf[e + half] = __fadd_rn(__fmul_rn(v0, sn[e]), __fmul_rn(v1, cs[e]));
      }
      __syncwarp();
    }
    if (vi >= G) {
      void *cache = vi == G ? a.k_cache : a.v_cache;
      const size_t new_off = (size_t)slot * a.kv_dim + (size_t)kvh * D;
      for (uint32_t d = lane; d < D; d += 32) {
        const uint16_t b = bf16_bits_rne(buf[d]);
        buf[d] = bf16_bits_to_f32(b);
        if (rank == 0 && slot_ok) reinterpret_cast<uint16_t *>(cache)[new_off + d] = b;
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  // 3. q as bf16 hi / lo rows (8..15 zero); the current slot's row takes the new k / v
  const uint32_t cur = *cur_s;
  for (uint32_t p = t; p < 16 * (D / 2); p += W * 32) {
    const uint32_t row = p / (D / 2), dp = p % (D / 2);
    float x0 = 0.0f, x1 = 0.0f;
    if (row < (uint32_t)G) {
      x0 = qs[row * D + 2 * dp];
      x1 = qs[row * D + 2 * dp + 1];
    }
    uint32_t hi, lo;
    tca_split(x0, x1, hi, lo);
    *reinterpret_cast<uint32_t *>(sm + TL::qh + row * kTcaStride + dp * 4) = hi;
    *reinterpret_cast<uint32_t *>(sm + TL::ql + row * kTcaStride + dp * 4) = lo;
    if (cur < (uint32_t)kClusterSlots && row == 0) {
      uint32_t kh, kl, vh, vl;
      tca_split(kn[2 * dp], kn[2 * dp + 1], kh, kl);  // bf16-exact: the lo half is zero
      tca_split(vn[2 * dp], vn[2 * dp + 1], vh, vl);
      *reinterpret_cast<uint32_t *>(sm + TL::kt + cur * kTcaStride + dp * 4) = kh;
      *reinterpret_cast<uint32_t *>(sm + TL::vt + cur * kTcaStride + dp * 4) = vh;
    }
  }
  __syncthreads();
  // 4. S = Q K^T: warp w, keys 8w .. 8w + 7
  float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  {
    const uint8_t *q0 = sm + TL::qh + g * kTcaStride + 4 * c, *q1 = q0 + 8 * kTcaStride;
    const uint8_t *l0 = sm + TL::ql + g * kTcaStride + 4 * c, *l1 = l0 + 8 * kTcaStride;
    const uint8_t *kr = sm + TL::kt + (8 * warp + g) * kTcaStride + 4 * c;
#pragma unroll 4
    for (int kk = 0; kk < 16; ++kk) {
      const uint32_t off = kk * 32;
      uint32_t ah[4], al[4];
      ah[0] = *reinterpret_cast<const uint32_t *>(q0 + off);
      ah[1] = *reinterpret_cast<const uint32_t *>(q1 + off);
      ah[2] = *reinterpret_cast<const uint32_t *>(q0 + off + 16);
      ah[3] = *reinterpret_cast<const uint32_t *>(q1 + off + 16);
      al[0] = *reinterpret_cast<const uint32_t *>(l0 + off);
      al[1] = *reinterpret_cast<const uint32_t *>(l1 + off);
      al[2] = *reinterpret_cast<const uint32_t *>(l0 + off + 16);
      al[3] = *reinterpret_cast<const uint32_t *>(l1 + off + 16);
      const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kr + off);
      const uint32_t b1 = *reinterpret_cast<const uint32_t *>(kr + off + 16);
      mma_bf16_16816(sc, ah, b0, b1);
      mma_bf16_16816(sc, al, b0, b1);
    }
  }
  // rows g (a head) of keys 8w + 2c, + 1; invalid keys and padding rows take no weight
  float p[2];
  {
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const uint32_t li = 8 * warp + 2 * c + e, sl = slot_s[li];
      const bool live = li < ns && sl < a.total_slots;
      if (li < ns && sl >= a.total_slots) raise_error(a.err, kDevBadSlot);
      p[e] = live ? sc[e] * a.scale : -INFINITY;
      m = fmaxf(m, p[e]);
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    if (c == 0) wmax[warp * G + g] = m;
  }
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < W; ++w) M = fmaxf(M, wmax[w * G + g]);
  {
    float ps = 0.0f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      p[e] = p[e] == -INFINITY ? 0.0f : expf(p[e] - M);
      ps += p[e];
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    if (c == 0) wsum[warp * G + g] = ps;
    *reinterpret_cast<float2 *>(sp + g * 64 + 8 * warp + 2 * c) = make_float2(p[0], p[1]);
  }
  __syncthreads();
  // 5. O = P V: warp w, head_dim columns 32w .. 32w + 31 (4 tiles of 8)
  float o[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  const uint32_t vbase = smem_u32(sm + TL::vt) + (lane & 7) * kTcaStride +
                         ((lane >> 3) & 1) * 8 * kTcaStride + (32 * warp + (lane >> 4) * 8) * 2;
#pragma unroll
  for (int s2 = 0; s2 < 4; ++s2) {
    const float2 pa = *reinterpret_cast<const float2 *>(sp + g * 64 + 16 * s2 + 2 * c);
    const float2 pb = *reinterpret_cast<const float2 *>(sp + g * 64 + 16 * s2 + 8 + 2 * c);
    uint32_t ph[4], pl[4];
    tca_split(pa.x, pa.y, ph[0], pl[0]);
    tca_split(pb.x, pb.y, ph[2], pl[2]);
    ph[1] = ph[3] = pl[1] = pl[3] = 0u;  // rows 8..15: padding
#pragma unroll
    for (int jd = 0; jd < 4; jd += 2) {
      uint32_t b00, b01, b10, b11;
      tca_ldsm_x4_trans(vbase + s2 * 16 * kTcaStride + jd * 16, b00, b01, b10, b11);
      mma_bf16_16816(o[jd], ph, b00, b01);
      mma_bf16_16816(o[jd], pl, b00, b01);
      mma_bf16_16816(o[jd + 1], ph, b10, b11);
      mma_bf16_16816(o[jd + 1], pl, b10, b11);
    }
  }
  // 6. this CTA's record per head: (M, L, O[D]) for row g
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t d = 32 * warp + 8 * j + 2 * c;
    rec[g * (D + 2) + 2 + d] = o[j][0];
    rec[g * (D + 2) + 2 + d + 1] = o[j][1];
  }
  if (warp == 0 && c == 0) {
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) L += wsum[w * G + g];
    rec[g * (D + 2)] = M;
    rec[g * (D + 2) + 1] = L;
  }
  __syncthreads();
  attn_cluster_merge<G, D, W>(a, kvh, rec, reinterpret_cast<float *>(sm + TL::fw),
                              reinterpret_cast<float *>(sm + TL::ls),
                              reinterpret_cast<float *>(sm + TL::fl), t);
}

}  // namespace
}  // namespace sx
