// comm.cuh — internal communicator definition.
#pragma once
#include <cuda_runtime.h>

#include "../../include/emx.h"

struct emx_comm {
  emx_ctx* ctx = nullptr;
  int nranks = 1, rank = 0;
  void* nccl = nullptr;  // ncclComm_t
};

namespace emx {
// In-place sum all-reduce on `st` (enqueued; graph-capturable).
int comm_all_reduce(emx_comm* c, void* buf, size_t count, emx_dtype dt, cudaStream_t st);
}  // namespace emx
