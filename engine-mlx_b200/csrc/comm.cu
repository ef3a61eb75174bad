// comm.cu — NCCL communicator for the tensor-parallel (dense) and
// expert-parallel (MoE) decode paths.  The reference has no distributed
// component; this is the collective the sharded configs need: a sum
// all-reduce over NVLink after the row-split o_proj / down_proj and after the
// local experts' combine.
//
// NCCL is resolved with dlopen("libnccl.so.2") so the library shares whatever
// NCCL the host process already loaded (e.g. torch's) instead of binding a
// second copy at link time.
#include <dlfcn.h>
#include <mutex>
#include <vector>
#include <nccl.h>

#include "comm.cuh"
#include "ctx.cuh"
#include "qgemv.cuh"

namespace emx {

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(dlsym(h, "ncclAllReduce"));
    a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    a.AllGather = reinterpret_cast<decltype(a.AllGather)>(dlsym(h, "ncclAllGather"));
    a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.AllReduce && a.GetErrorString && a.AllGather;
  });
  return a;
}

constexpr size_t kRegionBytes = kPeerHeader + 2 * (size_t)kPeerMaxRanks * kPeerSlotFloats * 4;

void peer_release(emx_comm* c) {
  for (int r = 0; r < 8; ++r)
    if (c->mapped[r]) {
      cudaIpcCloseMemHandle(c->mapped[r]);
      c->mapped[r] = nullptr;
    }
  if (c->region) cudaFree(c->region);
  if (c->d_peer) cudaFree(c->d_peer);
  if (c->d_words) cudaFree(c->d_words);
  c->region = nullptr;
  c->d_peer = nullptr;
  c->d_words = nullptr;
}

struct PeerRec {
  cudaIpcMemHandle_t h;
  int device;
  int ok;
};
// Exchange buffers of the set-up collectives (static: every rank can always
// take part, whatever it failed to allocate)
__device__ PeerRec g_peer_recs[kPeerMaxRanks];
__device__ int g_peer_ok;

// The peer-memory exchange: every rank allocates a zeroed region, the IPC
// handles and device ordinals travel by an NCCL all-gather, each rank opens
// the others' regions, and an all-reduce (min) of the outcome makes every
// rank take the same decision.  Any failure (a peer that this GPU cannot
// reach, IPC refused, more than kPeerMaxRanks ranks) leaves the sums on NCCL.
// Every rank runs both collectives whatever happens locally.
void peer_setup(emx_comm* c) {
  NcclApi& a = api();
  const int W = c->nranks;
  if (W < 2 || W > kPeerMaxRanks) return;  // the same on every rank
  cudaStream_t st = c->ctx->stream;
  ncclComm_t comm = static_cast<ncclComm_t>(c->nccl);
  PeerRec* d_recs = nullptr;
  int* d_ok = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&d_recs), g_peer_recs) != cudaSuccess ||
      cudaGetSymbolAddress(reinterpret_cast<void**>(&d_ok), g_peer_ok) != cudaSuccess) {
    cudaGetLastError();
    return;  // cannot happen once the module is loaded; no collective was entered
  }
  PeerRec mine = {};
  mine.device = c->ctx->device;
  mine.ok = cudaMalloc(&c->region, kRegionBytes) == cudaSuccess &&
            cudaMemset(c->region, 0, kRegionBytes) == cudaSuccess &&
            cudaIpcGetMemHandle(&mine.h, c->region) == cudaSuccess;
  cudaGetLastError();
  std::vector<PeerRec> recs(W);
  bool ok = cudaMemcpy(d_recs + c->rank, &mine, sizeof(PeerRec), cudaMemcpyHostToDevice) == cudaSuccess;
  const bool gathered = a.AllGather(d_recs + c->rank, d_recs, sizeof(PeerRec), ncclChar, comm, st) == ncclSuccess &&
                        cudaStreamSynchronize(st) == cudaSuccess &&
                        cudaMemcpy(recs.data(), d_recs, sizeof(PeerRec) * W, cudaMemcpyDeviceToHost) == cudaSuccess;
  ok = ok && gathered && mine.ok;
  for (int r = 0; ok && r < W; ++r) {
    if (!recs[r].ok) ok = false;
    if (r == c->rank || !ok) continue;
    int can = 0;
    if (cudaDeviceCanAccessPeer(&can, c->ctx->device, recs[r].device) != cudaSuccess || !can) ok = false;
  }
  PeerX px = {};
  px.world = W;
  px.rank = c->rank;
  for (int r = 0; ok && r < W; ++r) {
    if (r == c->rank) {
      px.base[r] = static_cast<unsigned char*>(c->region);
      continue;
    }
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, recs[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) ok = false;
    c->mapped[r] = p;
    px.base[r] = static_cast<unsigned char*>(p);
  }
  ok = ok && cudaMalloc(&c->d_words, 2 * sizeof(unsigned)) == cudaSuccess &&
       cudaMemset(c->d_words, 0, 2 * sizeof(unsigned)) == cudaSuccess &&
       cudaMalloc(&c->d_peer, sizeof(PeerX)) == cudaSuccess;
  if (ok) {
    px.epoch = c->d_words;
    px.ticket = c->d_words + 1;
    ok = cudaMemcpy(c->d_peer, &px, sizeof(PeerX), cudaMemcpyHostToDevice) == cudaSuccess;
  }
  cudaGetLastError();
  // one decision for all ranks
  int all = ok ? 1 : 0;
  const bool agreed = cudaMemcpy(d_ok, &all, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
                      a.AllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, comm, st) == ncclSuccess &&
                      cudaStreamSynchronize(st) == cudaSuccess &&
                      cudaMemcpy(&all, d_ok, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess;
  if (!agreed || all != 1) {
    cudaGetLastError();
    peer_release(c);
  }
}

}  // namespace

const PeerX* comm_peer(emx_comm* c) { return c ? c->d_peer : nullptr; }

int comm_all_reduce(emx_comm* c, void* buf, size_t count, emx_dtype dt, cudaStream_t st) {
  NcclApi& a = api();
  if (!a.ok) return fail(EMX_ERR_NCCL, "NCCL is not available");
  const ncclDataType_t t = dt == EMX_F32 ? ncclFloat32 : ncclBfloat16;
  ncclResult_t r = a.AllReduce(buf, buf, count, t, ncclSum, static_cast<ncclComm_t>(c->nccl), st);
  if (r != ncclSuccess) return fail(EMX_ERR_NCCL, "ncclAllReduce: %s", a.GetErrorString(r));
  return EMX_OK;
}

}  // namespace emx

using namespace emx;

extern "C" {

int emx_comm_unique_id(void* id_out) {
  if (!id_out) return fail(EMX_ERR_INVALID, "emx_comm_unique_id: null argument");
  NcclApi& a = api();
  if (!a.ok) return fail(EMX_ERR_NCCL, "emx_comm_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = a.GetUniqueId(&id);
  if (r != ncclSuccess) return fail(EMX_ERR_NCCL, "ncclGetUniqueId: %s", a.GetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == EMX_UNIQUE_ID_BYTES, "unique id size");
  memcpy(id_out, &id, sizeof(id));
  return EMX_OK;
}

int emx_comm_init(emx_ctx* ctx, const void* unique_id, int nranks, int rank, emx_comm** out) {
  if (!ctx || !unique_id || !out) return fail(EMX_ERR_INVALID, "emx_comm_init: null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fail(EMX_ERR_INVALID, "emx_comm_init: rank %d of %d", rank, nranks);
  NcclApi& a = api();
  if (!a.ok) return fail(EMX_ERR_NCCL, "emx_comm_init: libnccl.so.2 could not be loaded");
  cudaSetDevice(ctx->device);
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  ncclResult_t r = a.CommInitRank(&comm, nranks, id, rank);
  if (r != ncclSuccess) return fail(EMX_ERR_NCCL, "ncclCommInitRank: %s", a.GetErrorString(r));
  emx_comm* c = new emx_comm();
  c->ctx = ctx;
  c->nranks = nranks;
  c->rank = rank;
  c->nccl = comm;
  peer_setup(c);
  *out = c;
  return EMX_OK;
}

int emx_comm_destroy(emx_comm* c) {
  if (!c) return EMX_OK;
  NcclApi& a = api();
  peer_release(c);
  if (a.ok && c->nccl) a.CommDestroy(static_cast<ncclComm_t>(c->nccl));
  delete c;
  return EMX_OK;
}

int emx_all_reduce_sum(emx_comm* c, void* buf, size_t count, emx_dtype dt) {
  if (!c || !buf) return fail(EMX_ERR_INVALID, "emx_all_reduce_sum: null argument");
  if (dt != EMX_F32 && dt != EMX_BF16) return fail(EMX_ERR_INVALID, "emx_all_reduce_sum: f32 or bf16 only");
  return comm_all_reduce(c, buf, count, dt, c->ctx->stream);
}

}  // extern "C"
