// peer.cuh — the NVLink peer-memory sum behind tensor- and expert-parallel
// decode (set up by comm.cu; producers and consumers in pgemv_dev.cuh and
// misc.cu).
#pragma once
#include "common.cuh"

namespace emx {

// Decode tensor-parallel sum through NVLink peer memory (comm.cu sets it
// up).  Each rank owns a region [flags (u32 per source rank) | pad to
// kPeerHeader | two buffers of kPeerMaxRanks fp32 slots], mapped into every
// rank.  The producing GEMV (kEpiF32 with `peer`) stores its partial into
// slot [rank] of buffer (e+1) & 1 of every rank's region (peer stores over
// NVLink, e = reductions so far), and its last CTA then sets flag [rank] = e+1
// in every region; the consuming prologue (kProAddNorm with `peer`) waits on
// its own region's flags and sums the local slots in rank order, so every
// rank computes the same bits and the partials cross NVLink once.
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerSlotFloats = 16384;
constexpr int kPeerHeader = 256;
struct PeerX {
  unsigned char* base[kPeerMaxRanks];  // each rank's region in this process (base[rank] is local)
  int world, rank;
  unsigned* epoch;   // local: reductions produced so far
  unsigned* ticket;  // local: CTAs through the producing GEMV
};

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// In rank `dst`'s region: the slot holding rank `src`'s partial of reduction e.
__device__ __forceinline__ float* peer_slot(const PeerX& P, int dst, unsigned e, int src) {
  return reinterpret_cast<float*>(P.base[dst] + kPeerHeader +
                                  ((size_t)(e & 1u) * kPeerMaxRanks + src) * kPeerSlotFloats * 4);
}

// In rank `dst`'s region: rank `src`'s flag (the last reduction it stored there).
__device__ __forceinline__ unsigned* peer_flag(const PeerX& P, int dst, int src) {
  return reinterpret_cast<unsigned*>(P.base[dst]) + src;
}

// After a producer's stores of its partial into the ranks' slots (every
// thread of every CTA): the CTA barrier orders its threads' slot stores
// before thread 0's system-scope fence (fences are cumulative), which
// precedes the CTA's ticket; the last CTA through the ticket advances the
// epoch and sets this rank's flag in every region.
template <class Sync>
__device__ __forceinline__ void peer_publish(const PeerX& P, int tid, unsigned* flag_last) {
  Sync::sync();
  if (tid == 0) {
    __threadfence_system();
    *flag_last = (atomicAdd(P.ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
    if (*flag_last) {
      __threadfence();
      *P.ticket = 0u;
      const unsigned e = *P.epoch + 1u;
      *P.epoch = e;
      __threadfence_system();
      for (int d = 0; d < P.world; ++d) st_release_sys_u32(peer_flag(P, d, P.rank), e);
    }
  }
}

}  // namespace emx
