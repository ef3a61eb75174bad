// moe_route.cuh — the MoE router's softmax top-k for one token by one warp.
//
// Restates crates/ops/src/moe.rs:112-128 (softmax over the router logits,
// stable top-k, optional renormalisation of the k weights):
// p_e = bf16(exp(l_e - max) / sum_e exp(l_e - max)), then k rounds of an
// argmax over p (the largest value, the lowest index among equal ones, each
// taken entry removed; with nothing left to take, index 0), with
// `normalize` the k weights divided by their sum; only experts in
// [e_base, e_base + e_local) are kept (expert parallelism), renumbered from
// 0, in selection order.
//
// Up to 32 * EPL experts, everything in registers: lane l holds experts l,
// l + 32, ...  The softmax sum follows the order of misc.cu's 256-thread
// routing kernel (a butterfly over each group of 32 experts, then a
// butterfly over the eight group sums), so both give the same bits.
#pragma once
#include "common.cuh"

namespace emx {

// All 32 lanes of one warp call it.  `l2` reads the logits through L2 (for
// logits written by other CTAs of the calling kernel).
template <int EPL>
__device__ __forceinline__ void route_warp(const bf16* logits, bool l2, int E, int k, int normalize, int e_base,
                                           int e_local, int* idx, float* w, int* n) {
  const int lane = threadIdx.x & 31;
  float lg[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    float v = -INFINITY;
    if (i < E) {
      const unsigned short raw =
          l2 ? __ldcg(reinterpret_cast<const unsigned short*>(logits) + i) : reinterpret_cast<const unsigned short*>(logits)[i];
      v = __uint_as_float((uint32_t)raw << 16);
    }
    lg[j] = v;
    m = fmaxf(m, lg[j]);
  }
  m = warp_max(m);
  float part = 0.f;  // lane j: the sum of group j
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const float e = lane + 32 * j < E ? expf(lg[j] - m) : 0.f;
    const float t = warp_sum(e);
    if (lane == j) part = t;
  }
  const float s = warp_sum(part);
  float pr[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j)
    pr[j] = lane + 32 * j < E ? bfround(__fdiv_rn(expf(lg[j] - m), s)) : -INFINITY;
  int sel[64];
  float sw[64];
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = E;  // none yet
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int i = lane + 32 * j;
      if (i < E && (pr[j] > bv || (bi == E && pr[j] == bv))) {
        bv = pr[j];
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi >= E) {  // nothing to take: index 0 and its value
      bi = 0;
      bv = __shfl_sync(0xffffffffu, pr[0], 0);
    }
    sel[r] = bi;
    sw[r] = bv;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (lane + 32 * j == bi) pr[j] = -INFINITY;
  }
  if (lane == 0) {
    if (normalize) {
      float sum = 0.f;
      for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, sw[r]);
      if (sum > 1e-20f)
        for (int r = 0; r < k; ++r) sw[r] = __fdiv_rn(sw[r], sum);
    }
    int j = 0;
    for (int r = 0; r < k; ++r) {
      if (sel[r] >= e_base && sel[r] < e_base + e_local) {
        idx[j] = sel[r] - e_base;
        w[j] = sw[r];
        ++j;
      }
    }
    *n = j;
  }
}

}  // namespace emx
