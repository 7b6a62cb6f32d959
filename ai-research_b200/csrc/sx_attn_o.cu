// sx_attn_o.cu -- the decode graph's fused attention (q/k norm + RoPE + cache write + GQA
// attention over the ring's active slots, one thread-block cluster per kv head) with the o
// projection of that kv head's q heads folded into its tail.
//
// Replaces, for one session on one GPU with Q4_0 layers, the decode_attn.wgsl + gemv_q4.wgsl (o)
// pair of recordLayerDirect (src/gpu/model_dispatch.zig:10-43).  The o projection is split by
// columns: the CL CTAs of kv head h hold, after the cluster merge (sx_attn_dev.cuh,
// attn_cluster_item), the G x head_dim attention output of h's q heads, which meets exactly the
// columns [h G head_dim, (h + 1) G head_dim) of W_o.  Each CTA multiplies those columns of its
// share of W_o's 16-row tiles and writes opart[h][row]; the consumer (the gate+up GEMV's
// residual prologue, stage_x_q4) adds the num_kv partial vectors in kv-head order.  The W_o
// slice (head_dim G / 64 chunks per tile, contiguous in the packed layout) is bulk-copied into
// shared memory when the CTA starts, before the dependency wait, so the projection itself runs
// from shared memory after the attention.
#include "sx_attn_dev.cuh"
#include "sx_gemv_dev.cuh"

namespace sx {

namespace {

// shared memory after the attention work item: W_o slice | o fragments (layout of a GEMV with
// k = G D) | the G D attention output | mbarrier
struct AoLayout {
  uint32_t wo, ofrag, xo, bar, total;
  Layout o;
};
SX_HD AoLayout ao_layout(int g, uint32_t d, uint32_t cl, uint32_t o_tiles) {
  AoLayout L;
  const uint32_t att = (uint32_t)sizeof(float) * attn_cluster_floats(g, d, cl);
  L.wo = (att + 127u) & ~127u;
  L.ofrag = (L.wo + o_tiles * (g * d / 64) * kQ4ChunkBytes + 127u) & ~127u;
  L.o = layout_of(g * d, 1, 1, 4, false, 0);
  L.xo = (L.ofrag + L.o.total + 127u) & ~127u;
  L.bar = (L.xo + g * d * 4 + 127u) & ~127u;
  L.total = L.bar + 16;
  return L;
}

template <int DPL, int G, bool BF16, int CP>
__global__ void __launch_bounds__(kFusedWarps * 32) attn_o_kernel(AttnOArgs a) {
  extern __shared__ __align__(128) float sh[];
  uint8_t *const smem = reinterpret_cast<uint8_t *>(sh);
  constexpr uint32_t D = 32 * DPL, GD = G * D, GP = GD / 64;
  constexpr int CB = kQ4ChunkBytes, SO = QTraits<4>::kScaleOff;
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const uint32_t rank = cl.block_rank(), ncl = cl.num_blocks(), kvh = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const AoLayout L = ao_layout(G, D, ncl, a.o_tiles);
  const uint32_t otiles = a.o_rows / 16;
  const uint32_t ot0 = otiles * rank / ncl, ot1 = otiles * (rank + 1) / ncl;
  const uint32_t no = min(ot1 - ot0, a.o_tiles);
  const uint32_t bar = smem_u32(smem + L.bar);
  // the W_o slice: tile t's chunks of pairs [kvh GP, kvh GP + GP) lie back to back
  if (warp == 0) {
    if (lane == 0) mbar_init(bar, 32);
    fence_mbar_init();
    __syncwarp();
    uint32_t bytes = 0;
    for (uint32_t t = lane; t < no; t += 32) bytes += GP * CB;
    mbar_arrive_expect_tx(bar, bytes);
    const uint64_t pol = l2_evict_first_policy();
    const uint32_t po = pairs_of(a.at.num_q * D);
    for (uint32_t t = lane; t < no; t += 32)
      bulk_g2s_ef(smem_u32(smem + L.wo) + t * GP * CB,
                  static_cast<const uint8_t *>(a.wo) + ((size_t)(ot0 + t) * po + kvh * GP) * CB,
                  GP * CB, bar, pol);
  }
  pdl_launch_dependents();
  auto wait = [] { pdl_wait(); };
  attn_cluster_item<DPL, G, BF16, decltype(wait), CP>(a.at, kvh, sh, wait);
  // every CTA of the cluster wrote its slice of the G x D output before the cluster barrier
  // that ends the work item: read all of it back (through L2) and stage it as B fragments
  float *const xo = reinterpret_cast<float *>(smem + L.xo);
  for (uint32_t i = tid; i < GD; i += blockDim.x) xo[i] = __ldcg(a.at.out + (size_t)kvh * GD + i);
  __syncthreads();
  GemvArgs go{};
  go.k = GD;
  go.batch = 1;
  stage_x<4>(go, xo, GD, smem + L.ofrag, L.o, false);
  bool ok = mbar_wait_bounded(bar, 0);
  if (!ok) {
    if (tid == 0) raise_error(a.at.err, kDevBarrierTimeout);
    mbar_wait_bounded(bar, 0);  // the copies still in flight land before the CTA leaves
  }
  const uint8_t *const osm = smem + L.ofrag;
  const uint4 *const xf4 = reinterpret_cast<const uint4 *>(osm + L.o.xfrag);
  const float *const corr = reinterpret_cast<const float *>(osm + L.o.corr);
  const float xs = reinterpret_cast<const float *>(osm + L.o.misc)[0];
  const uint8_t *const wsm = smem + L.wo;
  const uint32_t xoff = (g * 4 + c) * 2;
  float *const out = a.opart + (size_t)kvh * a.o_rows;
  for (uint32_t lt = warp; ok && lt < no; lt += kFusedWarps) {
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
        const float2 c2 = *reinterpret_cast<const float2 *>(corr + p * 2);
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

template <int DPL, int G>
cudaError_t launch_ao_t(const AttnOArgs &a, cudaStream_t s) {
  if (a.cta_slots != 40 && a.cta_slots != 64) return cudaErrorInvalidValue;
  const uint32_t ncl = (a.at.total_slots + a.cta_slots - 1) / a.cta_slots;
  if (ncl > (uint32_t)kClusterMax) return cudaErrorInvalidValue;
  const AoLayout L = ao_layout(G, 32 * DPL, ncl, a.o_tiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.at.num_kv, ncl, 1);
  cfg.blockDim = dim3(kFusedWarps * 32);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = ncl;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (a.cta_slots == 40)
    return a.at.kv_bf16 ? cudaLaunchKernelEx(&cfg, attn_o_kernel<DPL, G, true, 5>, a)
                        : cudaLaunchKernelEx(&cfg, attn_o_kernel<DPL, G, false, 5>, a);
  return a.at.kv_bf16 ? cudaLaunchKernelEx(&cfg, attn_o_kernel<DPL, G, true, 8>, a)
                      : cudaLaunchKernelEx(&cfg, attn_o_kernel<DPL, G, false, 8>, a);
}

template <int DPL>
cudaError_t launch_ao_d(const AttnOArgs &a, cudaStream_t s) {
  switch (a.at.num_q / a.at.num_kv) {
    case 1: return launch_ao_t<DPL, 1>(a, s);
    case 2: return launch_ao_t<DPL, 2>(a, s);
    case 4: return launch_ao_t<DPL, 4>(a, s);
    case 8: return launch_ao_t<DPL, 8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

template <int DPL>
cudaError_t prepare_ao_d() {
  for (auto k : {attn_o_kernel<DPL, 1, true, 5>, attn_o_kernel<DPL, 1, false, 5>,
                 attn_o_kernel<DPL, 2, true, 5>, attn_o_kernel<DPL, 2, false, 5>,
                 attn_o_kernel<DPL, 4, true, 5>, attn_o_kernel<DPL, 4, false, 5>,
                 attn_o_kernel<DPL, 8, true, 5>, attn_o_kernel<DPL, 8, false, 5>,
                 attn_o_kernel<DPL, 1, true, 8>, attn_o_kernel<DPL, 1, false, 8>,
                 attn_o_kernel<DPL, 2, true, 8>, attn_o_kernel<DPL, 2, false, 8>,
                 attn_o_kernel<DPL, 4, true, 8>, attn_o_kernel<DPL, 4, false, 8>,
                 attn_o_kernel<DPL, 8, true, 8>, attn_o_kernel<DPL, 8, false, 8>}) {
    cudaError_t e = allow_max_dynamic_smem(k);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

bool attn_o_plan(uint32_t o_rows, uint32_t num_q, uint32_t num_kv, uint32_t head_dim,
                 uint32_t total_slots, uint32_t smem_limit, uint32_t *o_tiles,
                 uint32_t *cta_slots) {
  if (num_kv == 0 || num_q % num_kv != 0 || num_kv > (uint32_t)kProMaxParts) return false;
  const uint32_t g = num_q / num_kv;
  if (g != 1 && g != 2 && g != 4 && g != 8) return false;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return false;
  if (o_rows % 16 != 0 || (g * head_dim) % 64 != 0 || total_slots == 0 ||
      total_slots > kAttnClusterMaxSlots)
    return false;
  // 40 slots per CTA (5 per warp) while the cluster stays within 16 CTAs: more CTAs share
  // the attention and the o projection's tiles; 64 for longer rings
  const uint32_t cs = total_slots <= 40u * kClusterMax ? 40u : (uint32_t)kClusterSlots;
  const uint32_t ncl = (total_slots + cs - 1) / cs;
  const uint32_t tiles = (o_rows / 16 + ncl - 1) / ncl;
  if (ao_layout(g, head_dim, ncl, tiles).total > smem_limit) return false;
  *o_tiles = tiles;
  *cta_slots = cs;
  return true;
}

cudaError_t launch_attn_o(const AttnOArgs &a, cudaStream_t s) {
  if (a.at.sessions > 1) return cudaErrorInvalidValue;
  switch (a.at.head_dim) {
    case 64: return launch_ao_d<2>(a, s);
    case 128: return launch_ao_d<4>(a, s);
    case 256: return launch_ao_d<8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prepare_attn_o_kernels() {
  cudaError_t r[3] = {prepare_ao_d<2>(), prepare_ao_d<4>(), prepare_ao_d<8>()};
  for (cudaError_t x : r)
    if (x != cudaSuccess) return x;
  return cudaSuccess;
}

}  // namespace sx
