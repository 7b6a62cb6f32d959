// sx_tp.cu -- tensor-parallel decode support: the shard plan, the NCCL communicator and the
// on-device merge of the ranks' LM-head argmax candidates.
//
// NCCL is opened at run time (dlopen "libnccl.so.2"), only when a communicator is made: a
// process that already loaded torch's NCCL reuses that library, and a single-GPU process never
// loads one.  The per-token collectives are captured into the model's CUDA graph.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "sx_common.cuh"
#include "sx_host.h"
#include "sx_internal.h"

struct sx_comm {
  sx_engine *e = nullptr;
  ncclComm_t comm = nullptr;
  uint32_t nranks = 1, rank = 0;
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
  sx_comm *c = new sx_comm();
  c->e = e;
  c->nranks = nranks;
  c->rank = rank;
  st = nccl_status(api, api.comm_init_rank(&c->comm, (int)nranks, u, (int)rank),
                   "ncclCommInitRank");
  if (st != SX_OK) {
    delete c;
    return st;
  }
  *out = c;
  return SX_OK;
}

SX_API void sx_comm_destroy(sx_comm *c) {
  if (!c) return;
  NcclApi api;
  if (c->comm && nccl_api(&api)) {
    cudaSetDevice(c->e->device);
    api.comm_destroy(c->comm);
  }
  delete c;
}

// ---------------------------------------------------------------------------------------
// ops of the per-token graph
uint32_t sx_host_comm_ranks(const sx_comm *c) { return c ? c->nranks : 1; }
uint32_t sx_host_comm_rank(const sx_comm *c) { return c ? c->rank : 0; }

sx_status sx_host_allreduce(sx_comm *c, float *buf, size_t count, cudaStream_t s) {
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
