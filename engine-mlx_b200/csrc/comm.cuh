// comm.cuh — internal communicator definition.
#pragma once
#include <cuda_runtime.h>

#include "../../include/emx.h"

namespace emx {
struct PeerX;
}

struct emx_comm {
  emx_ctx* ctx = nullptr;
  int nranks = 1, rank = 0;
  void* nccl = nullptr;  // ncclComm_t
  // decode sums through peer memory (null when a peer is not reachable)
  void* region = nullptr;               // this rank's exchange region
  void* mapped[8] = {};                 // the peers' regions opened here
  emx::PeerX* d_peer = nullptr;         // device copy of the region table
  unsigned* d_words = nullptr;          // epoch + ticket
};

namespace emx {
// In-place sum all-reduce on `st` (enqueued; graph-capturable).
int comm_all_reduce(emx_comm* c, void* buf, size_t count, emx_dtype dt, cudaStream_t st);
// The peer-memory exchange of the decode sums, or nullptr (then NCCL).
const PeerX* comm_peer(emx_comm* c);
}  // namespace emx
