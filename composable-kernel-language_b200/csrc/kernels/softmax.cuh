// Online-softmax state of flash decoding: running maximum, normaliser and the weighted sum of
// four value lanes, with the merge of two partial states over disjoint key sets.
#pragma once

#include "common.cuh"

namespace ckl::kernels {

struct SoftmaxState {
  float m, l;
  float4 acc;
};

__device__ __forceinline__ void mergeState(SoftmaxState &a, const SoftmaxState &b) {
  const float M = fmaxf(a.m, b.m);
  if (M == -CUDART_INF_F)
    return; // both empty
  const float ca = a.m == -CUDART_INF_F ? 0.f : expf(a.m - M);
  const float cb = b.m == -CUDART_INF_F ? 0.f : expf(b.m - M);
  a.l = a.l * ca + b.l * cb;
  a.acc.x = a.acc.x * ca + b.acc.x * cb;
  a.acc.y = a.acc.y * ca + b.acc.y * cb;
  a.acc.z = a.acc.z * ca + b.acc.z * cb;
  a.acc.w = a.acc.w * ca + b.acc.w * cb;
  a.m = M;
}

__device__ __forceinline__ SoftmaxState shuffleState(const SoftmaxState &s, int offset) {
  SoftmaxState o;
  o.m = __shfl_xor_sync(0xffffffffu, s.m, offset);
  o.l = __shfl_xor_sync(0xffffffffu, s.l, offset);
  o.acc.x = __shfl_xor_sync(0xffffffffu, s.acc.x, offset);
  o.acc.y = __shfl_xor_sync(0xffffffffu, s.acc.y, offset);
  o.acc.z = __shfl_xor_sync(0xffffffffu, s.acc.z, offset);
  o.acc.w = __shfl_xor_sync(0xffffffffu, s.acc.w, offset);
  return o;
}

} // namespace ckl::kernels
