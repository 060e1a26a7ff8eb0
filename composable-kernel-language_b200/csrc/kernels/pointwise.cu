// Pointwise vector kernels: the vector pipeline's `update` and fused scalar-op chains.
//
// `update` (examples/vector_pipeline.py:9-14) computes dst[i] = src[i] + bias for every i the
// launch covers.  The fused chain applies a short sequence of scalar ops to each element with
// one rounding per op (no contraction into FMA), which is what two materialized launches
// compute (tests/Runtime/test_pointwise_fusion.py:105-118).  Both stream 16-byte vectors
// when the pointers allow it; grids are sized to a multiple of the SM count.
#include "common.cuh"

namespace ckl::kernels {
namespace {

constexpr int kPointwiseThreads = 256;

__device__ __forceinline__ float applyOp(float x, int64_t op, float s) {
  return op == 0 ? __fadd_rn(x, s) : __fmul_rn(x, s);
}

template <int Steps>
__device__ __forceinline__ float chain(float x, const ChainSpec &spec, const float *scalars) {
#pragma unroll
  for (int k = 0; k < Steps; ++k)
    x = applyOp(x, spec.op[k], scalars[k]);
  return x;
}

template <int Steps>
__device__ void chainBody(const float *__restrict__ src, float *__restrict__ dst,
                          const float *scalars, const ChainSpec &spec) {
  const int64_t count = spec.count;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (aligned16(src) && aligned16(dst)) {
    const int64_t vectors = count / 4;
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    int64_t v = i;
    for (; v + 7 * stride < vectors; v += 8 * stride) { // eight independent loads in flight
      float4 x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        x[u] = __ldcs(s4 + v + u * stride);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        x[u].x = chain<Steps>(x[u].x, spec, scalars);
        x[u].y = chain<Steps>(x[u].y, spec, scalars);
        x[u].z = chain<Steps>(x[u].z, spec, scalars);
        x[u].w = chain<Steps>(x[u].w, spec, scalars);
        __stcs(d4 + v + u * stride, x[u]);
      }
    }
    for (; v < vectors; v += stride) {
      float4 x = __ldcs(s4 + v);
      x.x = chain<Steps>(x.x, spec, scalars);
      x.y = chain<Steps>(x.y, spec, scalars);
      x.z = chain<Steps>(x.z, spec, scalars);
      x.w = chain<Steps>(x.w, spec, scalars);
      __stcs(d4 + v, x);
    }
    for (int64_t e = vectors * 4 + i; e < count; e += stride)
      dst[e] = chain<Steps>(src[e], spec, scalars);
  } else {
    for (int64_t e = i; e < count; e += stride)
      dst[e] = chain<Steps>(src[e], spec, scalars);
  }
}

__global__ void __launch_bounds__(kPointwiseThreads)
    updateKernel(const float *src, float *dst, float bias, PointwiseSpec spec) {
  ChainSpec chainSpec{spec.n, spec.count, 1, {0, 0, 0, 0}};
  const float scalars[1] = {bias};
  chainBody<1>(src, dst, scalars, chainSpec);
}

__global__ void __launch_bounds__(kPointwiseThreads)
    scaleKernel(const float *src, float *dst, float factor, PointwiseSpec spec) {
  ChainSpec chainSpec{spec.n, spec.count, 1, {1, 0, 0, 0}};
  const float scalars[1] = {factor};
  chainBody<1>(src, dst, scalars, chainSpec);
}

__global__ void __launch_bounds__(kPointwiseThreads)
    fillKernel(float *dst, float value, PointwiseSpec spec) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < spec.count; e += stride)
    dst[e] = value;
}

__global__ void __launch_bounds__(kPointwiseThreads)
    copyKernel(const float *src, float *dst, PointwiseSpec spec) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < spec.count; e += stride)
    dst[e] = src[e];
}

__global__ void __launch_bounds__(kPointwiseThreads)
    chain2Kernel(const float *src, float *dst, float s0, float s1, ChainSpec spec) {
  const float scalars[2] = {s0, s1};
  chainBody<2>(src, dst, scalars, spec);
}

__global__ void __launch_bounds__(kPointwiseThreads)
    chain3Kernel(const float *src, float *dst, float s0, float s1, float s2, ChainSpec spec) {
  const float scalars[3] = {s0, s1, s2};
  chainBody<3>(src, dst, scalars, spec);
}

__global__ void __launch_bounds__(kPointwiseThreads)
    chain4Kernel(const float *src, float *dst, float s0, float s1, float s2, float s3,
                 ChainSpec spec) {
  const float scalars[4] = {s0, s1, s2, s3};
  chainBody<4>(src, dst, scalars, spec);
}

// Streaming grid: enough CTAs to cover the data once with 4 vectors per thread, capped at a
// whole number of waves of 148 SMs x 8 resident CTAs.
unsigned streamingGrid(int64_t count) {
  const int64_t perCta = int64_t(kPointwiseThreads) * 4 * 4;
  const int64_t wanted = (count + perCta - 1) / perCta;
  const int64_t cap = 148 * 8 * 4;
  return unsigned(wanted < 1 ? 1 : (wanted > cap ? cap : wanted));
}

bool pointwiseGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<PointwiseSpec>(spec);
  if (s.count < 0 || s.count > s.n)
    return false;
  g->grid[0] = streamingGrid(s.count);
  g->block[0] = kPointwiseThreads;
  return true;
}

bool chainGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<ChainSpec>(spec);
  if (s.count < 0 || s.count > s.n || s.steps < 1 || s.steps > 4)
    return false;
  for (int k = 0; k < s.steps; ++k)
    if (s.op[k] != 0 && s.op[k] != 1)
      return false;
  g->grid[0] = streamingGrid(s.count);
  g->block[0] = kPointwiseThreads;
  return true;
}

} // namespace

CKL_REGISTER_KERNEL("ckl.pointwise.add_scalar", reinterpret_cast<const void *>(&updateKernel),
                    "PPFS", sizeof(PointwiseSpec), pointwiseGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.pointwise.mul_scalar", reinterpret_cast<const void *>(&scaleKernel),
                    "PPFS", sizeof(PointwiseSpec), pointwiseGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.pointwise.fill", reinterpret_cast<const void *>(&fillKernel), "PFS",
                    sizeof(PointwiseSpec), pointwiseGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.pointwise.copy", reinterpret_cast<const void *>(&copyKernel), "PPS",
                    sizeof(PointwiseSpec), pointwiseGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.pointwise.chain2", reinterpret_cast<const void *>(&chain2Kernel),
                    "PPFFS", sizeof(ChainSpec), chainGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.pointwise.chain3", reinterpret_cast<const void *>(&chain3Kernel),
                    "PPFFFS", sizeof(ChainSpec), chainGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.pointwise.chain4", reinterpret_cast<const void *>(&chain4Kernel),
                    "PPFFFFS", sizeof(ChainSpec), chainGeometry, nullptr);

} // namespace ckl::kernels
