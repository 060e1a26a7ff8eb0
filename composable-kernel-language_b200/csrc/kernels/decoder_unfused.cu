// One sm_100a kernel per decoder kernel of the reference program
// (benchmarks/decoder/workloads.py:33-188).  Each computes exactly the effect of its
// reference kernel over the whole index space the reference launch covers; the fused
// decoder path (decoder_fused.cu) is used when the program matches the decoder, these when
// a program composes the kernels differently or when bindings overlap.
//
// Reductions use warp shuffles instead of the reference's one-thread serial loops, so the
// float32 summation order differs (results agree within the decoder's tolerances).
#include "common.cuh"

namespace ckl::kernels {
namespace {

// ---- embedding (workloads.py:33-39) ---------------------------------------------------
// Rows whose token lies outside the table are left unwritten (the reference reads out of
// bounds there).
__global__ void embeddingKernel(const int *tokens, const float *table, float *dst,
                                EmbeddingSpec s) {
  dependentLaunchEntry();
  const int64_t total = s.B * s.C;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = e / s.C, c = e % s.C;
    const int token = tokens[b];
    if (token >= 0 && token < s.V)
      dst[e] = table[int64_t(token) * s.C + c];
  }
}

bool elementGeometry(int64_t total, library::Geometry *g) {
  if (total <= 0)
    return false;
  g->block[0] = 256;
  g->grid[0] = ceilDiv(total, 256) > 148 * 16 ? 148 * 16 : ceilDiv(total, 256);
  return true;
}

bool embeddingGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<EmbeddingSpec>(spec);
  return elementGeometry(s.B * s.C, g);
}

// ---- rms_stats (workloads.py:42-49): inv[b] = rsqrt(sum_c x^2 / C + eps) ---------------
__global__ void rmsStatsKernel(const float *x, float *inv, float eps, RowsSpec s) {
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x / kWarp) + warp;
  if (row >= s.B)
    return;
  float total = 0.f;
  for (int64_t c = lane; c < s.C; c += kWarp) {
    const float v = x[row * s.C + c];
    total += v * v;
  }
  total = warpSum(total);
  if (lane == 0)
    inv[row] = rsqrtf(total / float(s.C) + eps);
}

bool rowsGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<RowsSpec>(spec);
  if (s.B <= 0 || s.C <= 0)
    return false;
  g->block[0] = 256;
  g->grid[0] = ceilDiv(s.B, 8);
  return true;
}

// ---- rms_apply (workloads.py:52-58): dst = x * inv[b] * gain[layer, c] -------------------
__global__ void rmsApplyKernel(const float *x, const float *inv, const float *gain, float *dst,
                               RmsApplySpec s) {
  const int64_t total = s.B * s.C;
  const float *g = gain + s.layer * s.C;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = e / s.C, c = e % s.C;
    dst[e] = __fmul_rn(__fmul_rn(x[e], inv[b]), g[c]);
  }
}

bool rmsApplyGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<RmsApplySpec>(spec);
  return s.layer >= 0 && s.layer < s.L && elementGeometry(s.B * s.C, g);
}

// ---- rope (workloads.py:72-85) ----------------------------------------------------------
__global__ void ropeKernel(const float *src, const float *table, const int *position, float *dst,
                           RopeSpec s) {
  const int p = position[0];
  if (p < 0 || p >= s.T)
    return;
  const int64_t pairs = s.B * s.A * s.R;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < pairs;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e % s.R, h = (e / s.R) % s.A, b = e / (s.R * s.A);
    const int64_t c = b * s.C + h * 2 * s.R + 2 * r;
    const float first = src[c], second = src[c + 1];
    const float cosine = table[(int64_t(p) * s.R + r) * 2], sine = table[(int64_t(p) * s.R + r) * 2 + 1];
    dst[c] = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
    dst[c + 1] = __fadd_rn(__fmul_rn(first, sine), __fmul_rn(second, cosine));
  }
}

bool ropeGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<RopeSpec>(spec);
  return s.C == 2 * s.R * s.A && elementGeometry(s.B * s.A * s.R, g);
}

// ---- append_kv (workloads.py:88-97) -----------------------------------------------------
__global__ void appendKernel(const float *k, const float *v, float *kc, float *vc,
                             const int *position, CacheSpec s) {
  const int p = position[0];
  if (p < 0 || p >= s.T)
    return;
  const int64_t total = s.B * s.A * s.D;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t d = e % s.D, h = (e / s.D) % s.A, b = e / (s.D * s.A);
    const int64_t slot = (((s.layer * s.B + b) * s.A + h) * s.T + p) * s.D + d;
    kc[slot] = k[b * s.C + h * s.D + d];
    vc[slot] = v[b * s.C + h * s.D + d];
  }
}

bool cacheGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<CacheSpec>(spec);
  return s.C == s.A * s.D && s.layer >= 0 && s.layer < s.L && elementGeometry(s.B * s.A * s.D, g);
}

// ---- attention_scores (workloads.py:100-111) -----------------------------------------------
// One warp per (b, h, t) row chunk: lanes split the head dimension.
__global__ void scoresKernel(const float *q, const float *kc, const int *position, float *scores,
                             float scale, CacheSpec s) {
  const int64_t end = int64_t(position[0]) + 1;
  const int64_t limit = end < s.T ? end : s.T;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t rows = s.B * s.A * limit;
  for (int64_t w = int64_t(blockIdx.x) * (blockDim.x / kWarp) + warp; w < rows;
       w += int64_t(gridDim.x) * (blockDim.x / kWarp)) {
    const int64_t t = w % limit, h = (w / limit) % s.A, b = w / (limit * s.A);
    const float *key = kc + (((s.layer * s.B + b) * s.A + h) * s.T + t) * s.D;
    const float *query = q + b * s.C + h * s.D;
    float total = 0.f;
    for (int64_t d = lane; d < s.D; d += kWarp)
      total += query[d] * key[d];
    total = warpSum(total);
    if (lane == 0)
      scores[(b * s.A + h) * s.T + t] = total * scale;
  }
}

bool scoresGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<CacheSpec>(spec);
  if (s.C != s.A * s.D || s.layer < 0 || s.layer >= s.L)
    return false;
  g->block[0] = 256;
  const int64_t rows = s.B * s.A * s.T;
  g->grid[0] = ceilDiv(rows, 8) > 148 * 16 ? 148 * 16 : ceilDiv(rows, 8);
  return true;
}

// ---- softmax (workloads.py:114-128): one block per (b, h) --------------------------------
__global__ void softmaxKernel(const float *scores, const int *position, float *probs,
                              SoftmaxSpec s) {
  __shared__ float partial[32];
  const int64_t end = int64_t(position[0]) + 1;
  const int64_t limit = end < s.T ? end : s.T;
  const int64_t row = blockIdx.x;
  if (row >= s.B * s.A || limit <= 0)
    return;
  const float *in = scores + row * s.T;
  float *out = probs + row * s.T;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp, warps = blockDim.x / kWarp;
  float m = -CUDART_INF_F;
  for (int64_t t = threadIdx.x; t < limit; t += blockDim.x)
    m = fmaxf(m, in[t]);
  m = warpMax(m);
  if (lane == 0)
    partial[warp] = m;
  __syncthreads();
  m = lane < warps ? partial[lane] : -CUDART_INF_F;
  m = warpMax(m);
  __syncthreads();
  float sum = 0.f;
  for (int64_t t = threadIdx.x; t < limit; t += blockDim.x)
    sum += expf(in[t] - m);
  sum = warpSum(sum);
  if (lane == 0)
    partial[warp] = sum;
  __syncthreads();
  sum = lane < warps ? partial[lane] : 0.f;
  sum = warpSum(sum);
  for (int64_t t = threadIdx.x; t < limit; t += blockDim.x)
    out[t] = expf(in[t] - m) / sum;
}

bool softmaxGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<SoftmaxSpec>(spec);
  if (s.B * s.A <= 0)
    return false;
  g->grid[0] = unsigned(s.B * s.A);
  g->block[0] = 128;
  return true;
}

// ---- attention_values (workloads.py:131-142) ------------------------------------------------
__global__ void valuesKernel(const float *probs, const float *vc, const int *position, float *dst,
                             CacheSpec s) {
  const int64_t end = int64_t(position[0]) + 1;
  const int64_t limit = end < s.T ? end : s.T;
  const int64_t total = s.B * s.A * s.D;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t d = e % s.D, h = (e / s.D) % s.A, b = e / (s.D * s.A);
    const float *p = probs + (b * s.A + h) * s.T;
    const float *value = vc + (((s.layer * s.B + b) * s.A + h) * s.T) * s.D + d;
    float total_ = 0.f;
    for (int64_t t = 0; t < limit; ++t)
      total_ += p[t] * value[t * s.D];
    dst[b * s.C + h * s.D + d] = total_;
  }
}

// ---- add / silu / multiply (workloads.py:145-167) ----------------------------------------------
__global__ void addKernel(const float *x, const float *y, float *dst, RowsSpec s) {
  const int64_t total = s.B * s.C;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x)
    dst[e] = __fadd_rn(x[e], y[e]);
}

__global__ void multiplyKernel(const float *x, const float *y, float *dst, RowsSpec s) {
  const int64_t total = s.B * s.C;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x)
    dst[e] = __fmul_rn(x[e], y[e]);
}

__global__ void siluKernel(const float *src, float *dst, RowsSpec s) {
  const int64_t total = s.B * s.C;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const float v = src[e];
    dst[e] = v / (1.0f + expf(-v));
  }
}

bool rowsElementGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<RowsSpec>(spec);
  return elementGeometry(s.B * s.C, g);
}

// ---- greedy (workloads.py:170-183): first-index argmax per row ---------------------------
__global__ void greedyKernel(const float *logits, int *tokens, int *history, const int *position,
                             GreedySpec s) {
  __shared__ float bestValue[32];
  __shared__ int bestIndex[32];
  const int64_t row = blockIdx.x;
  if (row >= s.B)
    return;
  const float *in = logits + row * s.V;
  // The reference scan starts from element 0 and replaces only on a strictly larger score,
  // so NaN never wins and a NaN at element 0 wins outright.
  float value = in[0];
  int index = 0;
  if (value == value) {
    for (int64_t v = threadIdx.x; v < s.V; v += blockDim.x) {
      const float x = in[v];
      if (x > value || (x == value && int(v) < index))
        value = x, index = int(v);
    }
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
#pragma unroll
    for (int o = kWarp / 2; o > 0; o >>= 1)
      argmaxMerge(value, index, __shfl_xor_sync(0xffffffffu, value, o),
                  __shfl_xor_sync(0xffffffffu, index, o));
    if (lane == 0) {
      bestValue[warp] = value;
      bestIndex[warp] = index;
    }
    __syncthreads();
    if (warp == 0) {
      const int warps = blockDim.x / kWarp;
      value = lane < warps ? bestValue[lane] : -CUDART_INF_F;
      index = lane < warps ? bestIndex[lane] : 0x7fffffff;
#pragma unroll
      for (int o = kWarp / 2; o > 0; o >>= 1)
        argmaxMerge(value, index, __shfl_xor_sync(0xffffffffu, value, o),
                    __shfl_xor_sync(0xffffffffu, index, o));
    }
  }
  if (threadIdx.x == 0) {
    const int p = position[0];
    tokens[row] = index;
    if (p >= 0 && p < s.T)
      history[int64_t(p) * s.B + row] = index;
  }
}

bool greedyGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GreedySpec>(spec);
  if (s.B <= 0 || s.V <= 0)
    return false;
  g->grid[0] = unsigned(s.B);
  g->block[0] = 256;
  return true;
}

// ---- advance (workloads.py:186-188) ------------------------------------------------------
__global__ void advanceKernel(int *position) { position[0] = position[0] + 1; }

bool singleThreadGeometry(const void *, std::size_t, library::Geometry *g) { return true; }

} // namespace

CKL_REGISTER_KERNEL("ckl.decoder.embedding", reinterpret_cast<const void *>(&embeddingKernel),
                    "PPPS", sizeof(EmbeddingSpec), embeddingGeometry, nullptr,
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.decoder.rms_stats", reinterpret_cast<const void *>(&rmsStatsKernel),
                    "PPFS", sizeof(RowsSpec), rowsGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.rms_apply", reinterpret_cast<const void *>(&rmsApplyKernel),
                    "PPPPS", sizeof(RmsApplySpec), rmsApplyGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.rope", reinterpret_cast<const void *>(&ropeKernel), "PPPPS",
                    sizeof(RopeSpec), ropeGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.append_kv", reinterpret_cast<const void *>(&appendKernel),
                    "PPPPPS", sizeof(CacheSpec), cacheGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.attention_scores", reinterpret_cast<const void *>(&scoresKernel),
                    "PPPPFS", sizeof(CacheSpec), scoresGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.softmax", reinterpret_cast<const void *>(&softmaxKernel), "PPPS",
                    sizeof(SoftmaxSpec), softmaxGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.attention_values", reinterpret_cast<const void *>(&valuesKernel),
                    "PPPPS", sizeof(CacheSpec), cacheGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.add", reinterpret_cast<const void *>(&addKernel), "PPPS",
                    sizeof(RowsSpec), rowsElementGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.multiply", reinterpret_cast<const void *>(&multiplyKernel), "PPPS",
                    sizeof(RowsSpec), rowsElementGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.silu", reinterpret_cast<const void *>(&siluKernel), "PPS",
                    sizeof(RowsSpec), rowsElementGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.greedy", reinterpret_cast<const void *>(&greedyKernel), "PPPPS",
                    sizeof(GreedySpec), greedyGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.decoder.advance", reinterpret_cast<const void *>(&advanceKernel), "P", 0,
                    singleThreadGeometry, nullptr);

} // namespace ckl::kernels
