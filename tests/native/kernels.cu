// Test kernels for the plan-building callback tests, loaded as a CUBIN through ckl_begin.
// `join` mixes two inputs with fixed weights; `field` iterates a damped update.  They stand
// in for JIT-compiled program kernels (tests/Runtime/kernels.cu in the reference).
#include <cuda_runtime.h>

extern "C" __global__ void join(const float *first, const float *second, float *output, int size) {
  const int i = int(blockIdx.x * blockDim.x + threadIdx.x);
  if (i < size)
    output[i] = first[i] * 0.625f + second[i] * 0.375f;
}

extern "C" __global__ void field(const float *input, float *output, int size, float bias) {
  const int i = int(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= size)
    return;
  float value = input[i];
  for (int k = 0; k < 64; ++k)
    value = value * 0.9990234375f + bias;
  output[i] = value;
}
