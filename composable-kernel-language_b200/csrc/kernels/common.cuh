// Shared device helpers and specialization structs of the sm_100a kernel library.
//
// Every specialization struct is a sequence of int64 fields so that the host compiler (Python)
// packs it as "<Nq" with no padding questions.  Field meaning is documented per struct.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "../library.hpp"

namespace ckl::kernels {

constexpr int kWarp = 32;

__device__ __forceinline__ float warpSum(float v) {
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warpMax(float v) {
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Argmax pair reduction with first-index tie-breaking: `b` replaces `a` when it is strictly
// larger, or equal with a smaller index (the greedy kernel's strict ">" scan keeps the first
// maximum).
__device__ __forceinline__ void argmaxMerge(float &value, int &index, float otherValue,
                                            int otherIndex) {
  if (otherValue > value || (otherValue == value && otherIndex < index)) {
    value = otherValue;
    index = otherIndex;
  }
}

__device__ __forceinline__ bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

inline unsigned ceilDiv(int64_t a, int64_t b) { return unsigned((a + b - 1) / b); }

// 16-byte asynchronous copy global -> shared (both addresses 16-byte aligned), its commit, and
// the wait for all of this thread's copies (a wait on its own loads, which always complete;
// a CTA barrier after it publishes every thread's copies).
__device__ __forceinline__ void copyAsync16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<unsigned>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void copyAsyncCommit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void copyAsyncWaitAll() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Programmatic dependent launch: wait until every kernel this one depends on has completed and
// its memory is visible, then allow the kernels that depend on this one to be scheduled (they
// wait in turn).  Both are no-ops for a kernel launched without a programmatic dependency.
// Library kernels registered as dependent-launch aware call this before any global access.
__device__ __forceinline__ void dependentLaunchEntry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// The same for a long multi-wave kernel: wait at entry, and let the dependents be scheduled
// only as this CTA finishes (dependentLaunchExit), so they do not compete with this kernel's
// later waves for SM slots.
__device__ __forceinline__ void dependentLaunchWait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void dependentLaunchExit() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename Spec> const Spec &specOf(const void *spec) {
  return *static_cast<const Spec *>(spec);
}

// ---- specializations ------------------------------------------------------------------
// Elementwise pointwise kernels over a 1-D vector: n elements, `count` = elements the
// original launch covers (min(n, grid.x * block.x)).
struct PointwiseSpec {
  int64_t n, count;
};
// Fused chain of scalar pointwise ops: op codes 0 = add scalar, 1 = multiply scalar.
struct ChainSpec {
  int64_t n, count, steps, op[4];
};
struct EmbeddingSpec {
  int64_t B, C, V;
};
struct RowsSpec {
  int64_t B, C;
};
struct RmsApplySpec {
  int64_t B, C, L, layer;
};
// dst[B, O] = x[B, I] @ W[layer, I, O] with W holding `W` layers.
struct LinearSpec {
  int64_t B, I, O, W, layer;
};
struct RopeSpec {
  int64_t B, C, A, R, T;
};
// Cache shape [L, B, A, T, D]; hidden C = A * D.
struct CacheSpec {
  int64_t B, C, L, A, T, D, layer;
};
struct SoftmaxSpec {
  int64_t B, A, T;
};
struct GreedySpec {
  int64_t B, V, T;
};

// Fused projection: out = epilogue(prologue(x) @ W[layer]).
//   M rows (requests), K inner, N outputs; W holds `layers` matrices [K, N].
//   Cache-writing epilogues address cache[L=layers, M, A, T, D] at position[0].
//   `tiles` is the number of column tiles of the argmax epilogue (partials per row).
//   `cache` is the request count of the cache's batch dimension (M when 0): a projection over
//   a slice of the requests passes the cache pointer offset to its first request.
struct GemmSpec {
  int64_t M, K, N, layers, layer, A, D, T, tiles, config, cache;
};
// Flash-decoding attention over cache[L, B, A, T, D] at positions 0..position[0].
// `panel` 1 writes the context as a split tensor-core operand (panel.cuh) instead of [B, A*D].
// `rows` requests (B when 0) are processed, starting at the request the q, cache and context
// pointers point to; B is the cache's batch dimension.  `grid` caps the CTAs (0: one per
// request and head), which then loop over (request, head) pairs.
struct AttentionSpec {
  int64_t B, A, T, D, L, layer, splits, chunk, panel, rows, grid;
};
// Batched prefill: row m of a chunk is request m % B at prompt position position[0] + m / B.
//   PrefillRowsSpec: M rows, embedding [V, C], prompts [T, B].
//   PrefillAttentionSpec: cache [L, B, A, T, D]; P positions per chunk (M = P * B rows).
//   PrefillHistorySpec: argmax partials [M, tiles], history [T, B].
struct PrefillRowsSpec {
  int64_t M, B, C, V, T;
};
struct PrefillAttentionSpec {
  int64_t B, A, T, D, L, layer, P;
};
struct PrefillHistorySpec {
  int64_t M, B, tiles, T;
};
struct PositionAddSpec {
  int64_t delta;
};
// Greedy combine of per-tile argmax partials [B, tiles] of (value, index).
struct CombineSpec {
  int64_t B, tiles, T, V;
};
// Whole decode step in one launch (small decoders): B requests, hidden C = A x D, FFN width F,
// vocabulary V, L layers (weights of layers 0..L-1 of arrays holding `weightLayers`), cache
// capacity T, norm/head layer indices of the final norm and LM head, G requests per cluster.
struct DecodeStepSpec {
  int64_t B, C, A, D, F, V, L, T, weightLayers, normLayers, finalLayer, headLayer, G, clusters;
};

} // namespace ckl::kernels
