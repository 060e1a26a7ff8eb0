// Fused decode-step kernels for the decoder program (benchmarks/decoder/workloads.py:191-254).
//
// One layer of the reference runs 21 dependent launches.  With FFMA projections (up to 16
// requests, or with tensor cores switched off) it is eight graph nodes in five dependency levels:
//   q: RMSNorm -> x @ wq -> RoPE                       (norm_linear_rope)
//   k: RMSNorm -> x @ wk -> RoPE -> append to kc at p  (norm_linear_rope_append)
//   v: RMSNorm -> x @ wv -> append to vc at p          (norm_linear_append)
//   attention over kc/vc[0..p] (flash decoding; scores and probabilities never stored)
//   residual = x + context @ wo                        (linear_residual)
//   gate, up: RMSNorm -> x @ wg / wu                   (norm_linear, two concurrent nodes)
//   next_x = residual + (silu(gate) * up) @ wd         (swiglu_linear_residual)
// and the head is RMSNorm -> x @ lm with per-tile argmax partials, followed by a combine
// that writes tokens and history and advances the position.  Batches of 17 or more requests
// run the projections on the tensor cores instead (decoder_tc.cu); attention then writes its
// context as a split operand panel (AttentionSpec::panel).
#include "ckl_b200.h"
#include "common.cuh"
#include "gemm.cuh"
#include "panel.cuh"
#include "softmax.cuh"

namespace ckl::kernels {
namespace {

using gemm::Large;
using gemm::Medium;
using gemm::Params;
using gemm::Small;

// ---- projection wrappers ---------------------------------------------------------------
template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    linearKernel(const float *x, const float *w, float *dst, GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = x, p.w = w, p.out = dst, p.s = s;
  gemm::dispatch<Cfg, gemm::kPlain, gemm::kStore>(p);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    normLinearKernel(const float *x, const float *gain, const float *w, float *dst, float eps,
                     GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = x, p.gain = gain, p.w = w, p.out = dst, p.eps = eps, p.s = s;
  gemm::dispatch<Cfg, gemm::kRms, gemm::kStore>(p);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    normLinearRopeKernel(const float *x, const float *gain, const float *w, const float *table,
                         const int *position, float *dst, float eps, GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = x, p.gain = gain, p.w = w, p.table = table, p.position = position, p.out = dst;
  p.eps = eps, p.s = s;
  gemm::dispatch<Cfg, gemm::kRms, gemm::kRope>(p);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    normLinearRopeAppendKernel(const float *x, const float *gain, const float *w,
                               const float *table, const int *position, float *cache, float eps,
                               GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = x, p.gain = gain, p.w = w, p.table = table, p.position = position, p.out = cache;
  p.eps = eps, p.s = s;
  gemm::dispatch<Cfg, gemm::kRms, gemm::kRopeAppend>(p);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    normLinearAppendKernel(const float *x, const float *gain, const float *w, const int *position,
                           float *cache, float eps, GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = x, p.gain = gain, p.w = w, p.position = position, p.out = cache, p.eps = eps, p.s = s;
  gemm::dispatch<Cfg, gemm::kRms, gemm::kAppend>(p);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    linearResidualKernel(const float *x, const float *w, const float *residual, float *dst,
                         GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = x, p.w = w, p.residual = residual, p.out = dst, p.s = s;
  gemm::dispatch<Cfg, gemm::kPlain, gemm::kResidual>(p);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    swigluLinearResidualKernel(const float *gate, const float *up, const float *w,
                               const float *residual, float *dst, GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = gate, p.a2 = up, p.w = w, p.residual = residual, p.out = dst, p.s = s;
  gemm::dispatch<Cfg, gemm::kSwiGlu, gemm::kResidual>(p);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads)
    normLinearArgmaxKernel(const float *x, const float *gain, const float *w, float *logits,
                           float2 *partials, float eps, GemmSpec s) {
  dependentLaunchEntry();
  Params p;
  p.a = x, p.gain = gain, p.w = w, p.out = logits, p.partials = partials, p.eps = eps, p.s = s;
  gemm::dispatch<Cfg, gemm::kRms, gemm::kArgmax>(p);
}

bool gemmGeometry(const void *spec, std::size_t, library::Geometry *g) {
  return gemm::geometry(specOf<GemmSpec>(spec), g);
}

bool ropeGemmGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GemmSpec>(spec);
  if (s.D <= 0 || s.D % 2 || s.N % s.D || s.T <= 0)
    return false;
  return gemm::geometry(s, g);
}

bool appendGemmGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GemmSpec>(spec);
  if (s.D <= 0 || s.D % 2 || s.N != s.A * s.D || s.T <= 0)
    return false;
  return gemm::geometry(s, g);
}

#define CKL_GEMM_SELECT(fn)                                                                    \
  [](const void *spec) -> const void * {                                                       \
    switch (gemm::chooseConfig(specOf<GemmSpec>(spec))) {                                      \
    case 0: return reinterpret_cast<const void *>(&fn<Small>);                                 \
    case 1: return reinterpret_cast<const void *>(&fn<Medium>);                                \
    case 2: return reinterpret_cast<const void *>(&fn<Large>);                                 \
    case 6: return reinterpret_cast<const void *>(&fn<gemm::Rows1>);                           \
    case 7: return reinterpret_cast<const void *>(&fn<gemm::Rows4>);                           \
    case 8: return reinterpret_cast<const void *>(&fn<gemm::Rows16>);                          \
    case 9: return reinterpret_cast<const void *>(&fn<gemm::Streamed1>);                       \
    case 10: return reinterpret_cast<const void *>(&fn<gemm::Streamed4>);                      \
    case 11: return reinterpret_cast<const void *>(&fn<gemm::Streamed1Wide>);                  \
    case 12: return reinterpret_cast<const void *>(&fn<gemm::Streamed4Wide>);                  \
    case 13: return reinterpret_cast<const void *>(&fn<gemm::Streamed8>);                      \
    case 14: return reinterpret_cast<const void *>(&fn<gemm::Streamed8Wide>);                  \
    case 15: return reinterpret_cast<const void *>(&fn<gemm::Streamed1Deep>);                  \
    case 16: return reinterpret_cast<const void *>(&fn<gemm::Streamed4Deep>);                  \
    case 17: return reinterpret_cast<const void *>(&fn<gemm::Streamed8Deep>);                  \
    case 18: return reinterpret_cast<const void *>(&fn<gemm::Streamed8Deep16>);                \
    default: return nullptr;                                                                   \
    }                                                                                          \
  }

// ---- attention (flash decoding) ---------------------------------------------------------
// One CTA per (request, head): WARPS warps stream the K and V rows 0..p of the cache with
// 16-byte loads, D/4 lanes per row; each lane group keeps an online softmax state
// (running max, normaliser, weighted V) and the states merge across groups and warps.
// Eight warps of four-row-deep loads: at the cfg5 shard (8192 request-heads, 2048 rows of 256
// bytes) 7.40 TB/s against 7.18-7.19 with four warps per CTA and the same unroll (two, three or
// eight rows deep, 6, 12 or 16 warps, and 1-D bulk copies through shared memory all measured no
// faster).  The split kernel, which runs few CTAs, keeps four warps.
constexpr int kAttentionWarps = 8;
constexpr int kSplitWarps = 4;
constexpr int kAttentionUnroll = 4;

// Attention is registered without dependent launch: started early behind its q/k/v
// producers, its many waiting CTAs cost ~15 % of its own run time on B200.  It still lets its
// dependents (the o projection) be scheduled as its CTAs finish.
template <int D>
__global__ void __launch_bounds__(kAttentionWarps *kWarp)
    attentionKernel(const float *q, const float *kc, const float *vc, const int *position,
                    float *ctx, float scale, AttentionSpec s) {
  dependentLaunchWait();
  constexpr int LPR = D / 4;             // lanes per cache row
  constexpr int RPW = kWarp / LPR;       // rows per warp per iteration
  constexpr int STEP = kAttentionWarps * RPW;
  __shared__ SoftmaxState warpState[kAttentionWarps][LPR];

  const int64_t rows = s.rows > 0 ? s.rows : s.B;
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  const int group = lane / LPR, sub = lane % LPR;
  const int64_t C = s.A * D;
  const int p = position[0];
  const int64_t end = int64_t(p) + 1;
  const int64_t n = end < 0 ? 0 : (end < s.T ? end : s.T);
  constexpr int ROW4 = D / 4; // float4 per row

  for (int64_t bh = blockIdx.x; bh < rows * s.A; bh += gridDim.x) {
    const int64_t h = bh % s.A, b = bh / s.A;
    const float4 qv = *reinterpret_cast<const float4 *>(q + b * C + h * D + 4 * sub);
    const int64_t base = (((s.layer * s.B + b) * s.A + h) * s.T) * D + 4 * sub;
    const float4 *kRows = reinterpret_cast<const float4 *>(kc + base);
    const float4 *vRows = reinterpret_cast<const float4 *>(vc + base);

    SoftmaxState st{-CUDART_INF_F, 0.f, make_float4(0.f, 0.f, 0.f, 0.f)};
    for (int64_t t0 = int64_t(warp) * RPW; t0 < n; t0 += int64_t(STEP) * kAttentionUnroll) {
      float4 kv[kAttentionUnroll], vv[kAttentionUnroll];
      bool valid[kAttentionUnroll];
#pragma unroll
      for (int u = 0; u < kAttentionUnroll; ++u) {
        const int64_t t = t0 + int64_t(u) * STEP + group;
        valid[u] = t < n;
        if (valid[u]) {
          kv[u] = __ldcs(kRows + t * ROW4);
          vv[u] = __ldcs(vRows + t * ROW4);
        } else {
          kv[u] = vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < kAttentionUnroll; ++u) {
        float dot = qv.x * kv[u].x + qv.y * kv[u].y + qv.z * kv[u].z + qv.w * kv[u].w;
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1)
          dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (valid[u]) {
          const float score = dot * scale;
          const float M = fmaxf(st.m, score);
          const float c = st.m == -CUDART_INF_F ? 0.f : expf(st.m - M);
          const float e = expf(score - M);
          st.l = st.l * c + e;
          st.acc.x = st.acc.x * c + e * vv[u].x;
          st.acc.y = st.acc.y * c + e * vv[u].y;
          st.acc.z = st.acc.z * c + e * vv[u].z;
          st.acc.w = st.acc.w * c + e * vv[u].w;
          st.m = M;
        }
      }
    }
    // Merge the lane groups of the warp (same `sub`, different rows).
#pragma unroll
    for (int o = LPR; o < kWarp; o <<= 1) {
      const SoftmaxState other = shuffleState(st, o);
      mergeState(st, other);
    }
    if (group == 0)
      warpState[warp][sub] = st;
    __syncthreads();
    if (warp == 0 && group == 0) {
      SoftmaxState total = warpState[0][sub];
#pragma unroll
      for (int w = 1; w < kAttentionWarps; ++w)
        mergeState(total, warpState[w][sub]);
      float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
      if (total.l > 0.f) {
        out.x = total.acc.x / total.l;
        out.y = total.acc.y / total.l;
        out.z = total.acc.z / total.l;
        out.w = total.acc.w / total.l;
      }
      if (s.panel)
        panel::store4(ctx, b, h * D + 4 * sub, C, out); // split operand of the o projection
      else
        *reinterpret_cast<float4 *>(ctx + b * C + h * D + 4 * sub) = out;
    }
    __syncthreads(); // warpState is reused by the next (request, head)
  }
  dependentLaunchExit();
}

constexpr int kMaxAttentionSplits = 32;

// Split-K flash decoding, for few (request, head) pairs and long caches: the cache rows
// 0..p of every pair are divided into s.splits contiguous ranges of equal length, one CTA per
// (pair, range), so a small batch still puts hundreds of CTAs on the GPU.  Each CTA streams its
// range exactly like attentionKernel and writes its softmax state (maximum, normaliser,
// weighted V sum) to `partials`; the last CTA of a pair to finish (an arrival counter per
// pair, re-armed to zero by that CTA, so nothing ever waits) merges the states of all ranges in
// range order - a fixed order, so results do not depend on which CTA finished last - and
// writes the context row.  Ranges past the last cache row contribute empty states.
template <int D>
__global__ void __launch_bounds__(kSplitWarps *kWarp)
    attentionSplitKernel(const float *q, const float *kc, const float *vc, const int *position,
                         float *ctx, float *partials, unsigned *arrivals, float scale,
                         AttentionSpec s) {
  dependentLaunchWait();
  constexpr int LPR = D / 4;
  constexpr int RPW = kWarp / LPR;
  constexpr int STEP = kSplitWarps * RPW;
  constexpr int ROW4 = D / 4;
  constexpr int SLOT = D + 4; // m, l, two pad words, acc[D]: acc stays 16-byte aligned
  __shared__ SoftmaxState warpState[kSplitWarps][LPR];
  __shared__ int lastArrival;
  // The last arriver's copy of its pair's range states, loaded by all threads at once.
  __shared__ __align__(16) float gathered[kMaxAttentionSplits * SLOT];

  const int64_t rows = s.rows > 0 ? s.rows : s.B;
  const int64_t splits = s.splits;
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  const int group = lane / LPR, sub = lane % LPR;
  const int64_t C = s.A * D;
  const int p = position[0];
  const int64_t end = int64_t(p) + 1;
  const int64_t n = end < 0 ? 0 : (end < s.T ? end : s.T);
  const int64_t span = (n + splits - 1) / splits; // rows per range

  for (int64_t item = blockIdx.x; item < rows * s.A * splits; item += gridDim.x) {
    const int64_t range = item % splits, bh = item / splits;
    const int64_t h = bh % s.A, b = bh / s.A;
    const float4 qv = *reinterpret_cast<const float4 *>(q + b * C + h * D + 4 * sub);
    const int64_t base = (((s.layer * s.B + b) * s.A + h) * s.T) * D + 4 * sub;
    const float4 *kRows = reinterpret_cast<const float4 *>(kc + base);
    const float4 *vRows = reinterpret_cast<const float4 *>(vc + base);
    const int64_t first = range * span;
    const int64_t last = first + span < n ? first + span : n;
    SoftmaxState st{-CUDART_INF_F, 0.f, make_float4(0.f, 0.f, 0.f, 0.f)};
    for (int64_t t0 = first + int64_t(warp) * RPW; t0 < last;
         t0 += int64_t(STEP) * kAttentionUnroll) {
      float4 kv[kAttentionUnroll], vv[kAttentionUnroll];
      bool valid[kAttentionUnroll];
#pragma unroll
      for (int u = 0; u < kAttentionUnroll; ++u) {
        const int64_t t = t0 + int64_t(u) * STEP + group;
        valid[u] = t < last;
        if (valid[u]) {
          kv[u] = __ldcs(kRows + t * ROW4);
          vv[u] = __ldcs(vRows + t * ROW4);
        } else {
          kv[u] = vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < kAttentionUnroll; ++u) {
        float dot = qv.x * kv[u].x + qv.y * kv[u].y + qv.z * kv[u].z + qv.w * kv[u].w;
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1)
          dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (valid[u]) {
          const float score = dot * scale;
          const float M = fmaxf(st.m, score);
          const float c = st.m == -CUDART_INF_F ? 0.f : expf(st.m - M);
          const float e = expf(score - M);
          st.l = st.l * c + e;
          st.acc.x = st.acc.x * c + e * vv[u].x;
          st.acc.y = st.acc.y * c + e * vv[u].y;
          st.acc.z = st.acc.z * c + e * vv[u].z;
          st.acc.w = st.acc.w * c + e * vv[u].w;
          st.m = M;
        }
      }
    }
#pragma unroll
    for (int o = LPR; o < kWarp; o <<= 1) {
      const SoftmaxState other = shuffleState(st, o);
      mergeState(st, other);
    }
    if (group == 0)
      warpState[warp][sub] = st;
    __syncthreads();
    if (warp == 0 && group == 0) {
      SoftmaxState total = warpState[0][sub];
#pragma unroll
      for (int w = 1; w < kSplitWarps; ++w)
        mergeState(total, warpState[w][sub]);
      float *slot = partials + (bh * splits + range) * SLOT;
      if (sub == 0) {
        slot[0] = total.m;
        slot[1] = total.l;
      }
      reinterpret_cast<float4 *>(slot + 4)[sub] = total.acc;
      __threadfence(); // the state is visible device-wide before this CTA's arrival counts
    }
    __syncthreads();
    if (threadIdx.x == 0)
      lastArrival = atomicAdd(&arrivals[bh], 1u) == unsigned(splits - 1);
    __syncthreads();
    if (lastArrival) {
      __threadfence();
      // Every thread loads a share of the pair's states (L2, not L1: other CTAs wrote them
      // during this launch), so the merge below waits for one round of loads, not `splits`.
      const float4 *states = reinterpret_cast<const float4 *>(partials + bh * splits * SLOT);
      for (int64_t i = threadIdx.x; i < splits * (SLOT / 4); i += blockDim.x)
        reinterpret_cast<float4 *>(gathered)[i] = __ldcg(states + i);
      __syncthreads();
      if (warp == 0 && group == 0) {
        SoftmaxState total{-CUDART_INF_F, 0.f, make_float4(0.f, 0.f, 0.f, 0.f)};
        for (int64_t r = 0; r < splits; ++r) {
          const float *slot = gathered + r * SLOT;
          const SoftmaxState part{slot[0], slot[1], reinterpret_cast<const float4 *>(slot + 4)[sub]};
          if (r == 0)
            total = part;
          else
            mergeState(total, part);
        }
        float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
        if (total.l > 0.f) {
          out.x = total.acc.x / total.l;
          out.y = total.acc.y / total.l;
          out.z = total.acc.z / total.l;
          out.w = total.acc.w / total.l;
        }
        if (s.panel)
          panel::store4(ctx, b, h * D + 4 * sub, C, out);
        else
          *reinterpret_cast<float4 *>(ctx + b * C + h * D + 4 * sub) = out;
      }
      if (threadIdx.x == 0)
        arrivals[bh] = 0; // every range of this pair has arrived: re-arm for the next launch
    }
    __syncthreads(); // warpState and lastArrival are reused by the next item
  }
  dependentLaunchExit();
}

bool attentionSplitGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<AttentionSpec>(spec);
  if (s.B <= 0 || s.A <= 0 || s.T <= 0 || s.layer < 0 || s.layer >= s.L || s.splits < 2 ||
      s.splits > kMaxAttentionSplits)
    return false;
  if (s.D != 16 && s.D != 32 && s.D != 64 && s.D != 128)
    return false;
  const int64_t rows = s.rows > 0 ? s.rows : s.B;
  if (s.rows < 0 || rows > s.B || s.grid < 0 || rows * s.A * s.splits >= (int64_t(1) << 31))
    return false;
  const int64_t items = rows * s.A * s.splits;
  g->grid[0] = unsigned(s.grid > 0 && s.grid < items ? s.grid : items);
  g->block[0] = kSplitWarps * kWarp;
  return true;
}

const void *attentionSplitSelect(const void *spec) {
  switch (specOf<AttentionSpec>(spec).D) {
  case 16: return reinterpret_cast<const void *>(&attentionSplitKernel<16>);
  case 32: return reinterpret_cast<const void *>(&attentionSplitKernel<32>);
  case 64: return reinterpret_cast<const void *>(&attentionSplitKernel<64>);
  case 128: return reinterpret_cast<const void *>(&attentionSplitKernel<128>);
  default: return nullptr;
  }
}

bool attentionGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<AttentionSpec>(spec);
  if (s.B <= 0 || s.A <= 0 || s.T <= 0 || s.layer < 0 || s.layer >= s.L || s.splits != 1)
    return false;
  if (s.D != 16 && s.D != 32 && s.D != 64 && s.D != 128)
    return false;
  const int64_t rows = s.rows > 0 ? s.rows : s.B;
  if (s.rows < 0 || rows > s.B || s.grid < 0 || rows * s.A >= (int64_t(1) << 31))
    return false;
  const int64_t pairs = rows * s.A;
  g->grid[0] = unsigned(s.grid > 0 && s.grid < pairs ? s.grid : pairs);
  g->block[0] = kAttentionWarps * kWarp;
  return true;
}

const void *attentionSelect(const void *spec) {
  switch (specOf<AttentionSpec>(spec).D) {
  case 16: return reinterpret_cast<const void *>(&attentionKernel<16>);
  case 32: return reinterpret_cast<const void *>(&attentionKernel<32>);
  case 64: return reinterpret_cast<const void *>(&attentionKernel<64>);
  case 128: return reinterpret_cast<const void *>(&attentionKernel<128>);
  default: return nullptr;
  }
}

// ---- greedy combine -----------------------------------------------------------------
// One warp per request merges its [tiles] argmax partials (first index wins ties), writes
// tokens[b] and history[p, b]; the last CTA to finish advances position.  `counter` is a
// zero-initialised word that the last CTA returns to zero, so replays need no reset.
constexpr int kCombineWarps = 8;

__global__ void __launch_bounds__(kCombineWarps *kWarp)
    greedyCombineKernel(const float2 *partials, const float *logits, int *tokens, int *history,
                        int *position, unsigned *counter, CombineSpec s) {
  dependentLaunchEntry();
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
        index = 0; // a NaN first score wins the reference's strict scan outright
      tokens[row] = index;
      if (p >= 0 && p < s.T)
        history[int64_t(p) * s.B + row] = index;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(counter, 1u);
    if (done == gridDim.x - 1) {
      position[0] = p + 1;
      atomicExch(counter, 0u);
      __threadfence();
    }
  }
}

bool combineGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<CombineSpec>(spec);
  if (s.B <= 0 || s.tiles <= 0 || s.V <= 0)
    return false;
  g->grid[0] = ceilDiv(s.B, kCombineWarps);
  g->block[0] = kCombineWarps * kWarp;
  return true;
}

} // namespace

CKL_REGISTER_KERNEL("ckl.decoder.linear", reinterpret_cast<const void *>(&linearKernel<Medium>),
                    "PPPS", sizeof(GemmSpec), gemmGeometry, CKL_GEMM_SELECT(linearKernel));
CKL_REGISTER_KERNEL("ckl.fused.norm_linear", reinterpret_cast<const void *>(&normLinearKernel<Medium>),
                    "PPPPFS", sizeof(GemmSpec), gemmGeometry,
                    CKL_GEMM_SELECT(normLinearKernel),
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.norm_linear_rope",
                    reinterpret_cast<const void *>(&normLinearRopeKernel<Medium>), "PPPPPPFS",
                    sizeof(GemmSpec), ropeGemmGeometry,
                    CKL_GEMM_SELECT(normLinearRopeKernel),
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.norm_linear_rope_append",
                    reinterpret_cast<const void *>(&normLinearRopeAppendKernel<Medium>), "PPPPPPFS",
                    sizeof(GemmSpec), appendGemmGeometry,
                    CKL_GEMM_SELECT(normLinearRopeAppendKernel),
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.norm_linear_append",
                    reinterpret_cast<const void *>(&normLinearAppendKernel<Medium>), "PPPPPFS",
                    sizeof(GemmSpec), appendGemmGeometry,
                    CKL_GEMM_SELECT(normLinearAppendKernel),
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.linear_residual",
                    reinterpret_cast<const void *>(&linearResidualKernel<Medium>), "PPPPS",
                    sizeof(GemmSpec), gemmGeometry,
                    CKL_GEMM_SELECT(linearResidualKernel),
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.swiglu_linear_residual",
                    reinterpret_cast<const void *>(&swigluLinearResidualKernel<Medium>), "PPPPPS",
                    sizeof(GemmSpec), gemmGeometry, CKL_GEMM_SELECT(swigluLinearResidualKernel),
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.norm_linear_argmax",
                    reinterpret_cast<const void *>(&normLinearArgmaxKernel<Medium>), "PPPPPFS",
                    sizeof(GemmSpec), gemmGeometry,
                    CKL_GEMM_SELECT(normLinearArgmaxKernel),
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.attention", reinterpret_cast<const void *>(&attentionKernel<64>),
                    "PPPPPFS", sizeof(AttentionSpec), attentionGeometry, attentionSelect,
                    nullptr, 0, false);
CKL_REGISTER_KERNEL("ckl.fused.attention_split",
                    reinterpret_cast<const void *>(&attentionSplitKernel<64>), "PPPPPPPFS",
                    sizeof(AttentionSpec), attentionSplitGeometry, attentionSplitSelect,
                    nullptr, 0, false);
CKL_REGISTER_KERNEL("ckl.fused.greedy_combine",
                    reinterpret_cast<const void *>(&greedyCombineKernel), "PPPPPPS",
                    sizeof(CombineSpec), combineGeometry, nullptr,
                    nullptr, 0, true);

} // namespace ckl::kernels
