// Warp-level softmax over the experts + descending top-k (ties to the lowest
// expert index), shared by the router kernels.
// Semantics: components/moe/moe_ffn_block.mlir:72-128, oracles/moe.py:90-105.
#pragma once

#include "common.cuh"

namespace frank_topk {

constexpr int kMaxE = 256;  // experts handled by the router
constexpr int kMaxK = 32;   // top-k bound

// One warp: softmax over E logits held in shared memory (stride 1), then k
// rounds of arg-max.  Ties resolve to the lowest expert index.  Lane l owns
// experts l, l+32, ...  MaxE: a compile-time bound on E (a multiple of 32)
// that sizes the per-lane arrays.
template <int MaxE = kMaxE>
__device__ inline void warp_softmax_topk(const float* lg, int E, int k, int normalize,
                                  float* w_out, int32_t* id_out, int64_t T, int64_t t) {
  static_assert(MaxE % 32 == 0 && MaxE <= kMaxE, "MaxE: a multiple of 32, at most kMaxE");
  const int lane = threadIdx.x & 31;
  constexpr int kPer = MaxE / 32;
  float p[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    int e = lane + 32 * i;
    p[i] = (e < E) ? lg[e] : -INFINITY;
    mx = fmaxf(mx, p[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    int e = lane + 32 * i;
    p[i] = (e < E) ? expf(p[i] - mx) : 0.f;
    sum += p[i];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    int e = lane + 32 * i;
    p[i] = (e < E) ? p[i] / sum : -1.f;  // probabilities are >= 0; -1 marks "absent"
  }
  float chosen[kMaxK];
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    // lane-local best (lowest index on ties: scan ascending, strict >)
    float bv = -2.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (p[i] > bv) { bv = p[i]; bi = lane + 32 * i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    // remove the winner from its owner lane
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == bi) p[i] = -2.f;
    chosen[j] = bv;
    wsum += bv;  // ascending j, as numpy's sum over a short axis
    if (lane == 0) id_out[(int64_t)j * T + t] = bi;
  }
  if (lane == 0) {
    for (int j = 0; j < k; ++j)
      w_out[(int64_t)j * T + t] = normalize ? chosen[j] / wsum : chosen[j];
  }
}


}  // namespace frank_topk
