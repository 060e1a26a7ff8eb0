// Split-operand panel: the activation operand of a tensor-core projection, converted once.
//
// A projection on the tensor cores computes in 3xTF32: each FP32 input x is split into a TF32
// high part and a TF32 low part (x = hi + lo, both rounded to nearest).  The activation
// operand [M, K] is shared by every column tile of the output, so it is split once, by the
// kernel that produces it (RMSNorm, attention, SwiGLU), into a panel laid out exactly as the
// tensor cores read it from shared memory:
//
//   block (row tile mt = m / 128, slice kt = k / 32) of 2 x 128 x 32 floats (32 KB):
//     hi part, then lo part, each K-major without swizzle: element (r = m % 128, k' = k % 32)
//     at float ((k' / 4) * 128 + r) * 4 + k' % 4, i.e. 8-row x 16-byte core matrices,
//     K-adjacent core matrices 2 KB apart, 8-row groups 128 bytes apart.
//   blocks ordered (mt, kt), so a tile's slices are consecutive and one bulk copy moves a
//   block straight into a pipeline stage.
//
// Rows m >= M of the last row tile are never written (their products land in accumulator rows
// that no epilogue stores); columns K <= k < 32 * ceil(K / 32) of valid rows are written as
// zeros by producers whose K is not a multiple of 8 (the consumer issues no MMA k-step that
// lies wholly beyond K).
#pragma once

#include "common.cuh"

namespace ckl::kernels::panel {

constexpr int kRows = 128;                      // rows per tile (MMA M)
constexpr int kSlice = 32;                      // K per block
constexpr int kPart = kRows * kSlice;           // floats in the hi (or lo) part of a block
constexpr int kBlock = 2 * kPart;               // floats per block

__host__ __device__ constexpr int64_t slices(int64_t K) { return (K + kSlice - 1) / kSlice; }

__host__ __device__ constexpr int64_t floats(int64_t M, int64_t K) {
  return ((M + kRows - 1) / kRows) * slices(K) * kBlock;
}

// Offset of the hi value of element (m, k); the lo value is kPart floats further.  Four
// consecutive k starting at a multiple of 4 are contiguous (one 16-byte store per part).
__device__ __forceinline__ int64_t offset(int64_t m, int64_t k, int64_t K) {
  return ((m / kRows) * slices(K) + k / kSlice) * kBlock +
         (((k % kSlice) / 4) * kRows + m % kRows) * 4 + k % 4;
}

// Round to the nearest TF32 value (10 explicit mantissa bits), ties away from zero, with
// integer operations.
__device__ __forceinline__ float toTf32(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ void split(float x, float &hi, float &lo) {
  hi = toTf32(x);
  lo = toTf32(x - hi);
}

__device__ __forceinline__ void split4(const float4 &v, float4 &hi, float4 &lo) {
  split(v.x, hi.x, lo.x);
  split(v.y, hi.y, lo.y);
  split(v.z, hi.z, lo.z);
  split(v.w, hi.w, lo.w);
}

// Store four consecutive values (k a multiple of 4) of row m.
__device__ __forceinline__ void store4(float *panel, int64_t m, int64_t k, int64_t K,
                                       const float4 &v) {
  float4 hi, lo;
  split4(v, hi, lo);
  float *at = panel + offset(m, k, K);
  *reinterpret_cast<float4 *>(at) = hi;
  *reinterpret_cast<float4 *>(at + kPart) = lo;
}

} // namespace ckl::kernels::panel
