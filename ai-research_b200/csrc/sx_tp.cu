// sx_tp.cu -- tensor-parallel decode support: the shard plan, the communicator (NCCL plus a
// one-shot peer-to-peer all-reduce over NVLink), and the on-device merge of the ranks' LM-head
// argmax candidates.
//
// NCCL is opened at run time (dlopen "libnccl.so.2"), only when a communicator is made: a
// process that already loaded torch's NCCL reuses that library, and a single-GPU process never
// loads one.  The per-token collectives are captured into the model's CUDA graph.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "sx_common.cuh"
#include "sx_host.h"
#include "sx_internal.h"

namespace sx {
// One-shot peer all-reduce workspace, one per rank, opened by every peer through CUDA IPC:
// [flags: 8 u32, padded to 256 B][data: 2 parities x 8 source ranks x kP2pMaxCount f32].
constexpr uint32_t kP2pMaxRanks = 8;
constexpr uint32_t kP2pMaxCount = 16384;  // floats per all-reduce (hidden sizes up to 16384)
constexpr size_t kP2pFlagBytes = 256;
constexpr size_t kP2pBytes = kP2pFlagBytes + sizeof(float) * 2ull * kP2pMaxRanks * kP2pMaxCount;
constexpr uint64_t kP2pDefaultWaitNs = 2000000000ull;  // 2 s for the peers' flags
struct P2pArgs {
  uint8_t *ws[kP2pMaxRanks];  // every rank's workspace, mapped into this process (own: local)
  uint32_t nranks, rank;
  uint32_t *gen;              // this rank's call counter (device), equal on all ranks
  uint32_t *err;
  uint64_t wait_ns;           // how long a call waits for the other ranks' flags
};
}  // namespace sx

struct sx_comm {
  sx_engine *e = nullptr;
  ncclComm_t comm = nullptr;
  uint32_t nranks = 1, rank = 0;
  bool p2p = false;  // all-reduce with the peer kernel (else NCCL)
  sx::P2pArgs pa{};
  uint8_t *ws = nullptr;
};

namespace {

struct NcclApi {
  void *lib = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                             ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;

// Loads libnccl.so.2 once; false (with the error set) when it is missing.
bool nccl_api(NcclApi *out) {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (!g_nccl.lib) {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      sx_host_set_error("tensor parallel: libnccl.so.2 could not be loaded (%s)", dlerror());
      return false;
    }
    NcclApi a;
    a.lib = h;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.all_reduce ||
        !a.all_gather || !a.error_string) {
      sx_host_set_error("tensor parallel: libnccl.so.2 lacks an entry point");
      return false;
    }
    g_nccl = a;
  }
  *out = g_nccl;
  return true;
}

sx_status nccl_status(const NcclApi &api, ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return SX_OK;
  sx_host_set_error("%s: %s", what, api.error_string(r));
  return SX_ERR_PEER;
}

// Candidates {value bits, global index, logits[0]-is-NaN, 0} of n ranks -> token.  The order is
// the one-GPU argmax's: a NaN at logits[0] wins, then the larger value, then the lower index.
__global__ void tp_argmax_merge_kernel(const uint32_t *cand, uint32_t n, uint32_t *token) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  bool nan0 = false;
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t r = 0; r < n; ++r) {
    const float v = __uint_as_float(cand[r * 4]);
    const uint32_t i = cand[r * 4 + 1];
    nan0 = nan0 || cand[r * 4 + 2] != 0;
    if (i == 0xFFFFFFFFu) continue;
    if (bi == 0xFFFFFFFFu || v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  *token = (nan0 || bi == 0xFFFFFFFFu) ? 0u : bi;
}

}  // namespace

// ---------------------------------------------------------------------------------------
// shard plan
SX_API sx_status sx_tp_shard_plan(const sx_model_config *cfg, sx_tp_shard *out) {
  if (!cfg || !out) {
    sx_host_set_error("tp plan: null argument");
    return SX_ERR_INVALID;
  }
  const uint32_t n = cfg->tp_size > 1 ? cfg->tp_size : 1;
  const uint32_t r = n > 1 ? cfg->tp_rank : 0;
  const uint32_t gkv = cfg->full_every ? cfg->num_global_kv_heads : n;
  if (r >= n || cfg->num_q_heads % n || cfg->num_kv_heads % n || gkv % n ||
      (cfg->intermediate_size / 32) % n || cfg->intermediate_size % 32 || cfg->vocab_size % n) {
    sx_host_set_error("tp plan: %u ranks do not divide the q heads (%u), kv heads (%u/%u), "
                      "intermediate blocks (%u) and vocabulary (%u) evenly (rank %u)",
                      n, cfg->num_q_heads, cfg->num_kv_heads, cfg->num_global_kv_heads,
                      cfg->intermediate_size / 32, cfg->vocab_size, r);
    return SX_ERR_INVALID;
  }
  sx_tp_shard p{};
  p.q_heads = cfg->num_q_heads / n;
  p.q_head0 = r * p.q_heads;
  p.kv_heads = cfg->num_kv_heads / n;
  p.kv_head0 = r * p.kv_heads;
  p.global_kv_heads = cfg->full_every ? cfg->num_global_kv_heads / n : 0;
  p.global_kv_head0 = r * p.global_kv_heads;
  p.inter = cfg->intermediate_size / n;
  p.inter0 = r * p.inter;
  p.vocab = cfg->vocab_size / n;
  p.vocab0 = r * p.vocab;
  *out = p;
  return SX_OK;
}

// ---------------------------------------------------------------------------------------
namespace {

// One-shot all-reduce over peer memory (one CTA per rank; the vector is a hidden state of at
// most kP2pMaxCount floats, so the exchange is latency-bound and one CTA keeps every rank's
// order of operations simple).  Call g (a counter kept on each device; every rank makes the
// same calls in the same order) uses data parity g & 1:
//   1. store this rank's vector into data[parity][rank] of every rank's workspace (peer stores
//      over NVLink), fence system-wide, then release flags[rank] = g on every rank;
//   2. wait (bounded) until this rank's flags[r] >= g for all r;
//   3. out = sum over r = 0..n-1 of data[parity][r], in rank order -- the same bits on every rank.
// Two parities suffice: a rank can only start call g + 2 after every rank has released g + 1,
// i.e. has finished reading the data of call g.  A wait that runs out records
// kDevWaitTimeout and the kernel finishes with what it has (no hang).
SX_DEV void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
SX_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
SX_DEV uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(512) p2p_allreduce_kernel(float *buf, uint32_t count,
                                                            sx::P2pArgs a) {
  __shared__ uint32_t g_s, late;
  const uint32_t tid = threadIdx.x;
  // programmatic dependent launch: the next kernel may become resident (and stream its first
  // weight chunks) while this one exchanges; it waits for our completion before reading buf
  sx::pdl_launch_dependents();
  sx::pdl_wait();  // the producer of buf is complete
  if (tid == 0) {
    g_s = *a.gen + 1;
    *a.gen = g_s;
    late = 0;
  }
  __syncthreads();
  const uint32_t g = g_s, par = g & 1;
  auto data = [&](uint8_t *ws, uint32_t src) {
    return reinterpret_cast<float *>(ws + sx::kP2pFlagBytes) +
           ((size_t)par * sx::kP2pMaxRanks + src) * sx::kP2pMaxCount;
  };
  auto flags = [&](uint8_t *ws) { return reinterpret_cast<uint32_t *>(ws); };
  // 1. push
  const uint32_t n4 = count / 4;
  for (uint32_t r = 0; r < a.nranks; ++r) {
    float *dst = data(a.ws[r], a.rank);
    const float4 *src = reinterpret_cast<const float4 *>(buf);
    for (uint32_t i = tid; i < n4; i += blockDim.x) reinterpret_cast<float4 *>(dst)[i] = src[i];
    for (uint32_t i = 4 * n4 + tid; i < count; i += blockDim.x) dst[i] = buf[i];
  }
  __threadfence_system();
  __syncthreads();
  if (tid < a.nranks) st_release_sys(flags(a.ws[tid]) + a.rank, g);
  // 2. wait for every rank's data of call g, at most a.wait_ns of global time: a rank that
  // never comes makes the call record kDevWaitTimeout and finish, not hang
  if (tid < a.nranks) {
    const uint32_t *f = flags(a.ws[a.rank]) + tid;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(f) - g) < 0) {
      if (globaltimer_ns() - t0 > a.wait_ns) {
        atomicOr(&late, 1u);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (late && tid == 0) raise_error(a.err, sx::kDevWaitTimeout);
  // 3. sum in rank order
  const float *mine = data(a.ws[a.rank], 0);
  for (uint32_t i = tid; i < count; i += blockDim.x) {
    float s = 0.0f;
    for (uint32_t r = 0; r < a.nranks; ++r) s += mine[(size_t)r * sx::kP2pMaxCount + i];
    buf[i] = s;
  }
}

// Maps every rank's workspace into this process.  Every rank takes the same collective steps
// whatever happens locally -- one NCCL all-gather of {IPC handle, ok} records, then one NCCL
// min-reduce of "everything worked here" -- so all ranks reach the same verdict: either every
// rank has every peer mapped, or none keeps the peer path (and each unmaps what it opened).
// The exchange buffer is allocated before the communicator exists (sx_comm_create), so a rank
// that cannot take part returns before any collective.
struct HandleRec {
  cudaIpcMemHandle_t h;
  uint32_t ok;
  uint32_t pad[3];
};

sx_status p2p_setup(const NcclApi &api, sx_comm *c, void *xbuf) {
  cudaStream_t s = c->e->stream;
  uint32_t ok = c->nranks <= sx::kP2pMaxRanks ? 1u : 0u;
  void *ws = nullptr, *gen = nullptr;
  if (ok && cudaMalloc(&ws, sx::kP2pBytes) != cudaSuccess) ok = 0;
  if (ok && cudaMemset(ws, 0, sx::kP2pBytes) != cudaSuccess) ok = 0;
  if (ok && cudaMalloc(&gen, 256) != cudaSuccess) ok = 0;
  if (ok && cudaMemset(gen, 0, 256) != cudaSuccess) ok = 0;
  HandleRec mine{};
  c->ws = static_cast<uint8_t *>(ws);  // freed by p2p_teardown on any failure below
  c->pa.gen = static_cast<uint32_t *>(gen);
  if (ok && cudaIpcGetMemHandle(&mine.h, ws) != cudaSuccess) ok = 0;
  mine.ok = ok;
  cudaGetLastError();  // a local failure is reported through the agreement, not as sticky state
  // 1. the all-gather runs on every rank, whatever `ok` is
  HandleRec *recs = static_cast<HandleRec *>(xbuf);
  uint32_t *vote = reinterpret_cast<uint32_t *>(recs + c->nranks);
  sx_status st = sx_host_cuda_status(cudaMemcpy(recs + c->rank, &mine, sizeof(mine),
                                                cudaMemcpyHostToDevice),
                                     "ipc handle upload");
  if (st != SX_OK) return st;  // the exchange buffer itself is unusable: nothing can agree
  st = nccl_status(api,
                   api.all_gather(recs + c->rank, recs, sizeof(HandleRec), ncclUint8, c->comm, s),
                   "ncclAllGather (ipc handles)");
  std::vector<HandleRec> all(c->nranks);
  if (st == SX_OK) st = sx_host_cuda_status(cudaStreamSynchronize(s), "ipc handle exchange");
  if (st == SX_OK)
    st = sx_host_cuda_status(cudaMemcpy(all.data(), recs, sizeof(HandleRec) * c->nranks,
                                        cudaMemcpyDeviceToHost),
                             "ipc handle download");
  if (st != SX_OK) return st;
  for (uint32_t r = 0; r < c->nranks && r < sx::kP2pMaxRanks; ++r) {
    ok = ok && all[r].ok;
    if (!ok) break;
    if (r == c->rank) {
      c->pa.ws[r] = static_cast<uint8_t *>(ws);
      continue;
    }
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    }
    c->pa.ws[r] = static_cast<uint8_t *>(p);
  }
  // 2. agree: the peer path stays only if it worked on every rank
  st = sx_host_cuda_status(cudaMemcpy(vote, &ok, 4, cudaMemcpyHostToDevice), "peer vote upload");
  if (st == SX_OK)
    st = nccl_status(api, api.all_reduce(vote, vote, 1, ncclUint32, ncclMin, c->comm, s),
                     "ncclAllReduce (peer vote)");
  uint32_t agreed = 0;
  if (st == SX_OK) st = sx_host_cuda_status(cudaStreamSynchronize(s), "peer vote");
  if (st == SX_OK)
    st = sx_host_cuda_status(cudaMemcpy(&agreed, vote, 4, cudaMemcpyDeviceToHost), "peer vote");
  c->pa.nranks = c->nranks;
  c->pa.rank = c->rank;
  c->pa.err = c->e->err_dev;
  c->pa.wait_ns = sx::kP2pDefaultWaitNs;
  if (st != SX_OK) return st;
  return agreed ? SX_OK : SX_ERR_UNSUPPORTED;
}

void p2p_teardown(sx_comm *c) {
  for (uint32_t r = 0; r < c->nranks && r < sx::kP2pMaxRanks; ++r)
    if (r != c->rank && c->pa.ws[r]) cudaIpcCloseMemHandle(c->pa.ws[r]);
  if (c->ws) cudaFree(c->ws);
  if (c->pa.gen) cudaFree(c->pa.gen);
  c->ws = nullptr;
  c->pa = sx::P2pArgs{};
  c->p2p = false;
}

}  // namespace

// communicator
SX_API sx_status sx_comm_unique_id(uint8_t id[128]) {
  if (!id) {
    sx_host_set_error("comm: null id");
    return SX_ERR_INVALID;
  }
  NcclApi api;
  if (!nccl_api(&api)) return SX_ERR_UNSUPPORTED;
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
  ncclUniqueId u;
  sx_status st = nccl_status(api, api.get_unique_id(&u), "ncclGetUniqueId");
  if (st == SX_OK) memcpy(id, &u, 128);
  return st;
}

SX_API sx_status sx_comm_create(sx_engine *e, const uint8_t id[128], uint32_t nranks,
                                uint32_t rank, sx_comm **out) {
  if (!e || !id || !out || nranks < 1 || rank >= nranks) {
    sx_host_set_error("comm: bad arguments (nranks %u, rank %u)", nranks, rank);
    return SX_ERR_INVALID;
  }
  NcclApi api;
  if (!nccl_api(&api)) return SX_ERR_UNSUPPORTED;
  sx_status st = sx_host_cuda_status(cudaSetDevice(e->device), "cudaSetDevice");
  if (st != SX_OK) return st;
  ncclUniqueId u;
  memcpy(&u, id, 128);
  // the handle-exchange buffer, before any collective (a rank that cannot allocate it leaves
  // before ncclCommInitRank, like any other rank that fails to join)
  void *xbuf = nullptr;
  st = sx_host_cuda_status(cudaMalloc(&xbuf, sizeof(HandleRec) * (nranks + 1)),
                           "ipc handle exchange buffer");
  if (st != SX_OK) return st;
  sx_comm *c = new sx_comm();
  c->e = e;
  c->nranks = nranks;
  c->rank = rank;
  st = nccl_status(api, api.comm_init_rank(&c->comm, (int)nranks, u, (int)rank),
                   "ncclCommInitRank");
  if (st != SX_OK) {
    cudaFree(xbuf);
    delete c;
    return st;
  }
  // map the peer all-reduce's workspaces (collective: every rank does it here and all ranks
  // agree on the outcome); NCCL stays the all-reduce until sx_comm_set_allreduce(c, 0)
  // selects the peer kernel, which then succeeds on every rank or on none
  if (nranks > 1) {
    st = p2p_setup(api, c, xbuf);
    if (st != SX_OK) p2p_teardown(c);
    if (st == SX_ERR_UNSUPPORTED) st = SX_OK;  // agreed: NCCL only, on every rank
  }
  cudaFree(xbuf);
  if (st != SX_OK) {
    if (c->comm) api.comm_destroy(c->comm);
    delete c;
    return st;
  }
  *out = c;
  return SX_OK;
}

SX_API sx_status sx_comm_set_allreduce(sx_comm *c, int use_nccl) {
  if (!c) {
    sx_host_set_error("comm: null");
    return SX_ERR_INVALID;
  }
  if (!use_nccl && !c->ws && c->nranks > 1) {
    sx_host_set_error("comm: the peer all-reduce is unavailable (its workspace could not be "
                      "mapped on every rank)");
    return SX_ERR_UNSUPPORTED;
  }
  c->p2p = !use_nccl && c->nranks > 1;
  return SX_OK;
}

SX_API int sx_comm_allreduce_is_nccl(const sx_comm *c) { return c && c->p2p ? 0 : 1; }

SX_API sx_status sx_comm_set_wait_ns(sx_comm *c, uint64_t wait_ns) {
  if (!c || wait_ns == 0) {
    sx_host_set_error("comm: null communicator or zero wait");
    return SX_ERR_INVALID;
  }
  c->pa.wait_ns = wait_ns;
  return SX_OK;
}

SX_API sx_status sx_comm_allreduce(sx_comm *c, float *buf, uint32_t count) {
  if (!c || !buf || count == 0) {
    sx_host_set_error("comm allreduce: bad arguments");
    return SX_ERR_INVALID;
  }
  sx_status st = sx_host_cuda_status(cudaSetDevice(c->e->device), "cudaSetDevice");
  if (st == SX_OK) st = sx_host_allreduce(c, buf, count, c->e->stream);
  return st;
}

SX_API void sx_comm_destroy(sx_comm *c) {
  if (!c) return;
  NcclApi api;
  cudaSetDevice(c->e->device);
  cudaStreamSynchronize(c->e->stream);
  p2p_teardown(c);
  if (c->comm && nccl_api(&api)) api.comm_destroy(c->comm);
  delete c;
}

// ---------------------------------------------------------------------------------------
// ops of the per-token graph
uint32_t sx_host_comm_ranks(const sx_comm *c) { return c ? c->nranks : 1; }
uint32_t sx_host_comm_rank(const sx_comm *c) { return c ? c->rank : 0; }

sx_status sx_host_allreduce(sx_comm *c, float *buf, size_t count, cudaStream_t s) {
  if (c && c->p2p) {
    // never fall back to NCCL for one call: the other ranks would be in the peer kernel
    if (count > sx::kP2pMaxCount || ((uintptr_t)buf & 15) != 0) {
      sx_host_set_error("peer all-reduce: %zu floats at %p (at most %u, 16-byte aligned)", count,
                        (void *)buf, sx::kP2pMaxCount);
      return SX_ERR_UNSUPPORTED;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(512);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return sx_host_cuda_status(
        cudaLaunchKernelEx(&cfg, p2p_allreduce_kernel, buf, (uint32_t)count, c->pa),
        "peer all-reduce");
  }
  NcclApi api;
  if (!c || !nccl_api(&api)) {
    if (!c) sx_host_set_error("all-reduce: no communicator");
    return SX_ERR_PEER;
  }
  return nccl_status(api, api.all_reduce(buf, buf, count, ncclFloat32, ncclSum, c->comm, s),
                     "ncclAllReduce");
}

sx_status sx_host_allgather(sx_comm *c, const uint32_t *src, uint32_t *dst, size_t words,
                            cudaStream_t s) {
  NcclApi api;
  if (!c || !nccl_api(&api)) {
    if (!c) sx_host_set_error("all-gather: no communicator");
    return SX_ERR_PEER;
  }
  return nccl_status(api, api.all_gather(src, dst, words, ncclUint32, c->comm, s),
                     "ncclAllGather");
}

sx_status sx_host_tp_argmax(const uint32_t *cand, uint32_t n, uint32_t *token, cudaStream_t s) {
  tp_argmax_merge_kernel<<<1, 32, 0, s>>>(cand, n, token);
  return sx_host_cuda_status(cudaGetLastError(), "tp argmax merge");
}
