// Greedy LM head that allocates nothing: for callers that cannot allocate device memory.
//
// The decoder's head (RMSNorm -> x @ lm -> first-index argmax -> tokens, history, position+1)
// needs scratch beyond its inputs and outputs: per-tile argmax partials and a completion
// counter.  Through the regular entry points that scratch comes from the bind-time heap
// (cudaMalloc).  Some callers cannot allocate at the point they run the head: code inside a
// memory budget fixed by another allocator, code running while an allocator is locked, or a
// host that must not call cudaMalloc (it synchronizes the device) on a latency-critical
// path.  This entry point keeps its scratch in one fixed-size array in the library's own
// device memory instead, so a call performs no allocation of any kind.
//
// Limits and sharing:
//   * the array holds kMaxPartials argmax partials: batch * ceil(vocab / tile width) must not
//     exceed it (the call rejects larger sizes with CKL_INVALID_ARGUMENT);
//   * every GPU that loads the library holds the array (kScratchBytes) until process exit;
//   * all calls on a device share the array and it keeps the last call's contents: calls
//     whose executions overlap on the GPU race on it, so serialize them (one stream, or
//     events between streams);
//   * the first call on each device resolves the array's device address with
//     cudaGetSymbolAddress (this may load the module); make that first call before any
//     stream capture on that device.  The address is cached per device ordinal for the
//     life of the process, so calls after a cudaDeviceReset or under a context other than the
//     device's primary context are not supported.
#include "ckl_b200.h"
#include "../errors.hpp"
#include "common.cuh"
#include "gemm.cuh"

#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

namespace ckl::kernels {
namespace {

constexpr std::size_t kCounterBytes = 256;                  // counter word, padded
constexpr std::size_t kMaxPartials = std::size_t(1) << 19;  // 524288 (value, index) pairs
constexpr std::size_t kScratchBytes = kCounterBytes + kMaxPartials * sizeof(float2); // 4 MiB + 256

// The scratch array: completion counter at offset 0, argmax partials from kCounterBytes.
static __device__ __align__(256) unsigned char g_headScratch[kScratchBytes];

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    headArgmaxKernel(const float *x, const float *gain, const float *w, float *logits,
                     float2 *partials, float eps, GemmSpec s) {
  gemm::Params p;
  p.a = x, p.gain = gain, p.w = w, p.out = logits, p.partials = partials, p.eps = eps, p.s = s;
  gemm::body<Cfg, gemm::kRms, gemm::kArgmax>(p);
}

constexpr int kCombineWarps = 8;

// Per request: merge the tile partials (first index wins ties), write the token and the
// history row at position[0]; the last CTA to finish advances position and re-arms the
// counter.
__global__ void __launch_bounds__(kCombineWarps *kWarp)
    headCombineKernel(const float2 *partials, const float *logits, int *tokens, int *history,
                      int *position, unsigned *counter, CombineSpec s) {
  const int p = position[0];
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  const int64_t row = int64_t(blockIdx.x) * kCombineWarps + warp;
  if (row < s.B) {
    float best = -CUDART_INF_F;
    int index = 0x7fffffff;
    for (int64_t t = lane; t < s.tiles; t += kWarp) {
      const float2 v = partials[row * s.tiles + t];
      argmaxMerge(best, index, v.x, __float_as_int(v.y));
    }
#pragma unroll
    for (int o = kWarp / 2; o > 0; o >>= 1)
      argmaxMerge(best, index, __shfl_xor_sync(0xffffffffu, best, o),
                  __shfl_xor_sync(0xffffffffu, index, o));
    if (lane == 0) {
      const float first = logits[row * s.V];
      if (first != first || index == 0x7fffffff)
        index = 0;
      tokens[row] = index;
      if (p >= 0 && p < s.T)
        history[int64_t(p) * s.B + row] = index;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {
      position[0] = p + 1;
      atomicExch(counter, 0u);
      __threadfence();
    }
  }
}

// Device address of g_headScratch per device, resolved once with that device current.
std::mutex g_setupMutex;
unsigned char *g_scratchAddress[64] = {};

unsigned char *scratchFor(int device) {
  std::lock_guard<std::mutex> lock(g_setupMutex);
  if (device < 0 || device >= 64)
    throw std::invalid_argument("device ordinal out of range");
  if (!g_scratchAddress[device]) {
    void *address = nullptr;
    const cudaError_t status = cudaGetSymbolAddress(&address, g_headScratch);
    if (status != cudaSuccess) {
      cudaGetLastError();
      throw std::runtime_error(std::string("cudaGetSymbolAddress(head scratch) failed: ") +
                               cudaGetErrorString(status));
    }
    g_scratchAddress[device] = static_cast<unsigned char *>(address);
  }
  return g_scratchAddress[device];
}

template <class Cfg>
void launchHead(const float *x, const float *gain, const float *lm, float eps, const GemmSpec &s,
                float *logits, float2 *partials, cudaStream_t stream) {
  const dim3 grid(ceilDiv(s.N, Cfg::BN), ceilDiv(s.M, Cfg::BM));
  headArgmaxKernel<Cfg><<<grid, Cfg::kThreads, 0, stream>>>(x, gain, lm, logits, partials, eps, s);
}

} // namespace
} // namespace ckl::kernels

extern "C" int ckl_greedy_head_noalloc(const float *x, const float *gain, const float *lm,
                                       float eps, int64_t batch, int64_t hidden, int64_t vocab,
                                       int64_t capacity, float *logits, int32_t *tokens,
                                       int32_t *history, int32_t *position, void *stream) {
  using namespace ckl::kernels;
  try {
    if (!x || !gain || !lm || !logits || !tokens || !history || !position)
      throw std::invalid_argument("greedy head: null input or output pointer");
    if (batch <= 0 || hidden <= 0 || vocab <= 0 || capacity <= 0)
      throw std::invalid_argument("greedy head: sizes must be positive");
    GemmSpec s{batch, hidden, vocab, 1, 0, 0, 0, 0, 0, 0};
    // Tiles of the shared FFMA kernel: 16x64 up to 16 rows, otherwise the shape-based choice.
    const int config = batch <= 16 ? 0 : gemm::chooseConfig(s);
    const int width = config == 0 ? gemm::Small::BN : config == 1 ? gemm::Medium::BN
                                                                  : gemm::Large::BN;
    const int64_t tiles = (vocab + width - 1) / width;
    if (batch > int64_t(kMaxPartials) / tiles)
      throw std::invalid_argument(
          "greedy head: batch x vocabulary tiles = " + std::to_string(batch * tiles) +
          " argmax partials exceed the fixed scratch of " + std::to_string(kMaxPartials));
    if ((batch + gemm::Small::BM - 1) / gemm::Small::BM > 65535)
      throw std::invalid_argument("greedy head: batch exceeds the launch grid");
    s.tiles = tiles;
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess)
      throw std::runtime_error(std::string("cudaGetDevice failed: ") + cudaGetErrorString(status));
    unsigned char *scratch = scratchFor(device);
    auto *counter = reinterpret_cast<unsigned *>(scratch);
    auto *partials = reinterpret_cast<float2 *>(scratch + kCounterBytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    status = cudaMemsetAsync(counter, 0, sizeof(unsigned), st);
    if (status != cudaSuccess)
      throw std::runtime_error(std::string("cudaMemsetAsync failed: ") + cudaGetErrorString(status));
    switch (config) {
    case 0: launchHead<gemm::Small>(x, gain, lm, eps, s, logits, partials, st); break;
    case 1: launchHead<gemm::Medium>(x, gain, lm, eps, s, logits, partials, st); break;
    default: launchHead<gemm::Large>(x, gain, lm, eps, s, logits, partials, st); break;
    }
    const CombineSpec c{batch, tiles, capacity, vocab};
    headCombineKernel<<<ceilDiv(batch, kCombineWarps), kCombineWarps * kWarp, 0, st>>>(
        partials, logits, tokens, history, position, counter, c);
    status = cudaGetLastError();
    if (status != cudaSuccess)
      throw std::runtime_error(std::string("greedy head launch failed: ") +
                               cudaGetErrorString(status));
    return CKL_OK;
  } catch (const std::invalid_argument &e) {
    ckl::setLastError(e.what());
    return CKL_INVALID_ARGUMENT;
  } catch (const std::exception &e) {
    ckl::setLastError(e.what());
    return CKL_RUNTIME_ERROR;
  }
}
