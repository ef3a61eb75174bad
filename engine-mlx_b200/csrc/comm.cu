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
#include <nccl.h>

#include "comm.cuh"
#include "ctx.cuh"

namespace emx {

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
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
    a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.AllReduce && a.GetErrorString;
  });
  return a;
}

}  // namespace

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
  *out = c;
  return EMX_OK;
}

int emx_comm_destroy(emx_comm* c) {
  if (!c) return EMX_OK;
  NcclApi& a = api();
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
