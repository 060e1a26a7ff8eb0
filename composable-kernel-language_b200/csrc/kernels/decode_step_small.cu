// Whole decode step of a small decoder, one CTA per group of up to eight requests.
//
// For decoders whose weights are a few MB at most (one request, hidden 64,
// two layers; config 4: 256 requests, hidden 64, eight layers) the cluster kernel of
// decode_step.cu spends most of a step in cluster barriers and distributed-shared-memory
// exchanges, which exist to spread each projection's weights over eight SMs.  Here every CTA
// of 1024 threads runs the whole step for its own requests and reads all weights itself (from
// L2, where they stay), with nothing but CTA barriers; CTAs never wait for one another and the
// last one to finish advances the position (an arrival counter it re-arms):
//   * every projection puts one thread on each (output column, K slice) pair: all of its
//     weight loads are independent and go out at once (one L2 round trip per projection),
//     each load serving every request of the step (one accumulator per request); the K slices'
//     partial sums then add up in slice order through shared memory (deterministic);
//   * q, k and v are one pass over the three weight matrices side by side, gate and up another;
//   * attention gives each (request, head) pair one or more warps: lanes in groups of D / 4 own
//     one cache row at a time (16-byte loads) with an online softmax, merged across the groups
//     of a warp by shuffles and across the pair's warps through shared memory in warp order;
//   * the residual stream, normalized rows, queries, attention outputs and the SwiGLU product
//     stay in shared memory; only cache rows, logits, tokens, history and position are written.
// Same arguments as the cluster kernel (DecodeStepSpec::G requests per CTA, ::clusters CTAs).
// Same arithmetic conventions (RMSNorm with rsqrtf, RoPE and SwiGLU rounded
// as the other decoder kernels, expf softmax, first-index argmax with the NaN-at-zero rule).
#include "ckl_b200.h"
#include "common.cuh"
#include "softmax.cuh"

namespace ckl::kernels {
namespace {

constexpr int kSmallThreads = 1024;
constexpr int kSmallWarps = kSmallThreads / kWarp;
constexpr int kSmallRows = 8;          // requests per CTA
constexpr int kSmallMaxHidden = 256;
constexpr int kSmallMaxFfn = 1024;
constexpr int kSmallMaxCache = 4096;
constexpr std::size_t kSmallMaxShared = 227 * 1024;

// Shared memory of the step, in floats, each region rounded up to 16 bytes: x, act, q, ctx
// [B][C]; h [B][F]; tile [B][max(3C, 2F)]; partial sums [kSmallThreads][kSmallRows]; softmax
// states (32 bytes each) [kSmallWarps][kWarp]; argmax partials [kSmallWarps][kSmallRows] x 2.
__host__ __device__ inline int64_t pad4(int64_t floats) { return (floats + 3) / 4 * 4; }
__host__ __device__ inline int64_t smallTileColumns(const DecodeStepSpec &s) {
  return 3 * s.C > 2 * s.F ? 3 * s.C : 2 * s.F;
}
struct SmallLayout {
  int64_t act, q, ctx, h, tile, partial, states, bestValue, bestIndex, total;
};
__host__ __device__ inline SmallLayout smallLayout(const DecodeStepSpec &s) {
  SmallLayout o;
  o.act = pad4(s.G * s.C);
  o.q = o.act + pad4(s.G * s.C);
  o.ctx = o.q + pad4(s.G * s.C);
  o.h = o.ctx + pad4(s.G * s.C);
  o.tile = o.h + pad4(s.G * s.F);
  o.partial = o.tile + pad4(s.G * smallTileColumns(s));
  o.states = o.partial + int64_t(kSmallThreads) * kSmallRows;
  o.bestValue = o.states + int64_t(kSmallWarps) * kWarp * 8;
  o.bestIndex = o.bestValue + kSmallWarps * kSmallRows;
  o.total = o.bestIndex + kSmallWarps * kSmallRows;
  return o;
}

// acc[r] += in[r * ldIn + k] * column[k * width] for k in [k0, k1), in k order, with the weight
// loads issued BATCH at a time before their multiply-adds (independent loads in flight).
template <int BATCH>
__device__ __forceinline__ void accumulate(const float *in, int ldIn, int rows,
                                           const float *column, int width, int k0, int k1,
                                           float (&acc)[kSmallRows]) {
  for (int k = k0; k < k1; k += BATCH) {
    float weight[BATCH];
#pragma unroll
    for (int j = 0; j < BATCH; ++j)
      weight[j] = k + j < k1 ? __ldg(column + int64_t(k + j) * width) : 0.f;
#pragma unroll
    for (int j = 0; j < BATCH; ++j)
      if (k + j < k1)
#pragma unroll
        for (int r = 0; r < kSmallRows; ++r)
          if (r < rows)
            acc[r] = fmaf(in[r * ldIn + k + j], weight[j], acc[r]);
  }
}

// out[r * ldOut + n] = sum_k in[r * ldIn + k] * W(n)[k] for n < count * width and r < rows,
// where W(n) is column n % width of matrix n / width (row-major [K][width]).  Below
// kSmallThreads columns, thread t takes column t % N and K slice t / N; above, columns stride
// over the threads with the whole K.  Ends with a barrier.
__device__ void smallProject(const float *in, int ldIn, int rows, int K, const float *const *w,
                             int count, int width, float *partial, float *out, int64_t ldOut) {
  const int N = count * width, tid = threadIdx.x;
  if (N >= kSmallThreads) {
    for (int n = tid; n < N; n += kSmallThreads) {
      const float *column = w[n / width] + n % width;
      float acc[kSmallRows];
#pragma unroll
      for (int r = 0; r < kSmallRows; ++r)
        acc[r] = 0.f;
      accumulate<16>(in, ldIn, rows, column, width, 0, K, acc);
#pragma unroll
      for (int r = 0; r < kSmallRows; ++r)
        if (r < rows)
          out[r * ldOut + n] = acc[r];
    }
    __syncthreads();
    return;
  }
  int slices = kSmallThreads / N;
  if (slices > K)
    slices = K;
  const int n = tid % N, slice = tid / N;
  if (slice < slices) {
    const int k0 = int(int64_t(slice) * K / slices), k1 = int(int64_t(slice + 1) * K / slices);
    const float *column = w[n / width] + n % width;
    float acc[kSmallRows];
#pragma unroll
    for (int r = 0; r < kSmallRows; ++r)
      acc[r] = 0.f;
    accumulate<8>(in, ldIn, rows, column, width, k0, k1, acc);
#pragma unroll
    for (int r = 0; r < kSmallRows; ++r)
      partial[(slice * N + n) * kSmallRows + r] = acc[r];
  }
  __syncthreads();
  for (int e = tid; e < N * rows; e += kSmallThreads) {
    const int column = e % N, r = e / N;
    float v = partial[column * kSmallRows + r];
    for (int j = 1; j < slices; ++j)
      v += partial[(j * N + column) * kSmallRows + r];
    out[r * ldOut + column] = v;
  }
  __syncthreads();
}

// act[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * gain, one warp per row.  Ends with a barrier.
__device__ void smallNorm(const float *x, const float *gain, float *act, int rows, int C,
                          float eps) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  if (warp < rows) {
    float total = 0.f;
    for (int c = lane; c < C; c += kWarp)
      total += x[warp * C + c] * x[warp * C + c];
    total = warpSum(total);
    const float inv = rsqrtf(total / float(C) + eps);
    for (int c = lane; c < C; c += kWarp)
      act[warp * C + c] = __fmul_rn(__fmul_rn(x[warp * C + c], inv), gain[c]);
  }
  __syncthreads();
}

template <int D>
__device__ void smallAttention(const float *q, const float *kc, const float *vc, float *ctx,
                               SoftmaxState *states, int rows, int64_t r0, int64_t B, int A,
                               int64_t T, int64_t layer, int64_t n, float scale) {
  constexpr int LPR = D / 4, RPW = kWarp / LPR;
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  const int group = lane / LPR, sub = lane % LPR;
  const int C = A * D, pairs = rows * A;
  int wp = 1; // warps per (request, head)
  while (wp < kSmallWarps && pairs * wp * 2 <= kSmallWarps)
    wp *= 2;
  const int member = warp % wp, perRound = kSmallWarps / wp;
  for (int base = 0; base < pairs; base += perRound) {
    const int pair = base + warp / wp;
    SoftmaxState st{-CUDART_INF_F, 0.f, make_float4(0.f, 0.f, 0.f, 0.f)};
    if (pair < pairs) {
      const int b = pair / A, h = pair % A;
      const float4 qv = *reinterpret_cast<const float4 *>(q + b * C + h * D + 4 * sub);
      const int64_t rowsBase = (((layer * B + r0 + b) * A + h) * T) * D + 4 * sub;
      const float4 *kRows = reinterpret_cast<const float4 *>(kc + rowsBase);
      const float4 *vRows = reinterpret_cast<const float4 *>(vc + rowsBase);
      for (int64_t t0 = int64_t(member) * RPW; t0 < n; t0 += int64_t(wp) * RPW * 2) {
        float4 kv[2], vv[2];
        bool valid[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int64_t t = t0 + int64_t(u) * wp * RPW + group;
          valid[u] = t < n;
          kv[u] = valid[u] ? __ldcg(kRows + t * (D / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
          vv[u] = valid[u] ? __ldcg(vRows + t * (D / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
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
      for (int o = LPR; o < kWarp; o <<= 1)
        mergeState(st, shuffleState(st, o));
    }
    if (group == 0)
      states[warp * kWarp + sub] = st;
    __syncthreads();
    if (pair < pairs && member == 0 && group == 0) {
      const int b = pair / A, h = pair % A;
      SoftmaxState total = states[warp * kWarp + sub];
      for (int j = 1; j < wp; ++j)
        mergeState(total, states[(warp + j) * kWarp + sub]);
      float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
      if (total.l > 0.f)
        out = make_float4(total.acc.x / total.l, total.acc.y / total.l, total.acc.z / total.l,
                          total.acc.w / total.l);
      *reinterpret_cast<float4 *>(ctx + b * C + h * D + 4 * sub) = out;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kSmallThreads, 1)
    decodeStepSmallKernel(int *tokens, int *position, int *history, const float *emb,
                          const float *norm1, const float *norm2, const float *finalNorm,
                          const float *wq, const float *wk, const float *wv, const float *wo,
                          const float *wg, const float *wu, const float *wd, const float *lm,
                          const float *sincos, float *kc, float *vc, float *logits,
                          unsigned *counter, float eps, float scale, DecodeStepSpec s) {
  const int tid = threadIdx.x, lane = tid % kWarp, warp = tid / kWarp;
  const int C = int(s.C), A = int(s.A), D = int(s.D), F = int(s.F);
  const int64_t B = s.B, V = s.V, T = s.T;
  const int64_t r0 = int64_t(blockIdx.x) * s.G;
  const int rows = int(s.G < B - r0 ? s.G : B - r0); // this CTA's requests r0 .. r0 + rows
  extern __shared__ float4 smallShared[];
  const SmallLayout at = smallLayout(s);
  float *x = reinterpret_cast<float *>(smallShared);
  float *act = x + at.act, *q = x + at.q, *ctx = x + at.ctx, *h = x + at.h, *tile = x + at.tile;
  float *partial = x + at.partial;
  auto *states = reinterpret_cast<SoftmaxState *>(x + at.states);
  float *bestValue = x + at.bestValue;
  int *bestIndex = reinterpret_cast<int *>(x + at.bestIndex);

  const int p = position[0];
  if (p >= 0 && p < T) {
    for (int e = tid; e < rows * C; e += kSmallThreads) {
      const int token = tokens[r0 + e / C];
      x[e] = token >= 0 && token < V ? emb[int64_t(token) * C + e % C] : 0.f;
    }
    __syncthreads();
    const float *cs = sincos + int64_t(p) * (D / 2) * 2;
    const int ldQkv = 3 * C;
    for (int64_t l = 0; l < s.L; ++l) {
      smallNorm(x, norm1 + l * C, act, rows, C, eps);
      const float *qkv[3] = {wq + l * C * C, wk + l * C * C, wv + l * C * C};
      smallProject(act, C, rows, C, qkv, 3, C, partial, tile, ldQkv);
      // RoPE on q and k, append k and v at position p.
      for (int e = tid; e < rows * C / 2; e += kSmallThreads) {
        const int b = e / (C / 2), c = 2 * (e % (C / 2)), hh = c / D, d = c % D;
        const float cosine = cs[(d / 2) * 2], sine = cs[(d / 2) * 2 + 1];
        const float *row = tile + b * ldQkv;
        auto rotate = [&](float first, float second, float &outFirst, float &outSecond) {
          outFirst = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
          outSecond = __fadd_rn(__fmul_rn(first, sine), __fmul_rn(second, cosine));
        };
        rotate(row[c], row[c + 1], q[b * C + c], q[b * C + c + 1]);
        const int64_t slot = (((l * B + r0 + b) * A + hh) * T + p) * D + d;
        rotate(row[C + c], row[C + c + 1], kc[slot], kc[slot + 1]);
        vc[slot] = row[2 * C + c];
        vc[slot + 1] = row[2 * C + c + 1];
      }
      __syncthreads();
      const int64_t n = int64_t(p) + 1;
      switch (D) {
      case 16: smallAttention<16>(q, kc, vc, ctx, states, rows, r0, B, A, T, l, n, scale); break;
      case 32: smallAttention<32>(q, kc, vc, ctx, states, rows, r0, B, A, T, l, n, scale); break;
      case 64: smallAttention<64>(q, kc, vc, ctx, states, rows, r0, B, A, T, l, n, scale); break;
      default: smallAttention<128>(q, kc, vc, ctx, states, rows, r0, B, A, T, l, n, scale); break;
      }
      const float *o[1] = {wo + l * C * C};
      smallProject(ctx, C, rows, C, o, 1, C, partial, tile, C);
      for (int e = tid; e < rows * C; e += kSmallThreads)
        x[e] = __fadd_rn(x[e], tile[e]);
      __syncthreads();
      smallNorm(x, norm2 + l * C, act, rows, C, eps);
      const float *gateUp[2] = {wg + l * C * F, wu + l * C * F};
      smallProject(act, C, rows, C, gateUp, 2, F, partial, tile, 2 * F);
      for (int e = tid; e < rows * F; e += kSmallThreads) {
        const int b = e / F, f = e % F;
        const float g = tile[b * 2 * F + f], u = tile[b * 2 * F + F + f];
        h[e] = __fmul_rn(g / (1.0f + expf(-g)), u);
      }
      __syncthreads();
      const float *down[1] = {wd + l * F * C};
      smallProject(h, F, rows, F, down, 1, C, partial, tile, C);
      for (int e = tid; e < rows * C; e += kSmallThreads)
        x[e] = __fadd_rn(x[e], tile[e]);
      __syncthreads();
    }
    // Head: final norm, logits straight to global memory, first-index argmax per request.
    smallNorm(x, finalNorm + s.finalLayer * C, act, rows, C, eps);
    const float *head[1] = {lm + s.headLayer * C * V};
    float *rowLogits = logits + r0 * V;
    smallProject(act, C, rows, C, head, 1, int(V), partial, rowLogits, V);
    for (int b = 0; b < rows; ++b) {
      float best = -CUDART_INF_F;
      int index = 0x7fffffff;
      for (int64_t j = tid; j < V; j += kSmallThreads)
        argmaxMerge(best, index, rowLogits[b * V + j], int(j));
#pragma unroll
      for (int o = kWarp / 2; o > 0; o >>= 1)
        argmaxMerge(best, index, __shfl_xor_sync(0xffffffffu, best, o),
                    __shfl_xor_sync(0xffffffffu, index, o));
      if (lane == 0) {
        bestValue[warp * kSmallRows + b] = best;
        bestIndex[warp * kSmallRows + b] = index;
      }
    }
    __syncthreads();
    if (tid < rows) {
      float best = -CUDART_INF_F;
      int index = 0x7fffffff;
      for (int w = 0; w < kSmallWarps; ++w)
        argmaxMerge(best, index, bestValue[w * kSmallRows + tid], bestIndex[w * kSmallRows + tid]);
      const float first = rowLogits[int64_t(tid) * V];
      if (first != first || index == 0x7fffffff)
        index = 0; // a NaN first score wins the reference's strict scan outright
      tokens[r0 + tid] = index;
      history[int64_t(p) * B + r0 + tid] = index;
    }
  }
  // The last CTA to finish advances the position (every CTA read it before arriving).
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(counter, 1u) == unsigned(s.clusters) - 1) {
      position[0] = p + 1;
      atomicExch(counter, 0u);
      __threadfence();
    }
  }
}

bool decodeStepSmallGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<DecodeStepSpec>(spec);
  if (s.B <= 0 || s.G <= 0 || s.G > kSmallRows || s.clusters <= 0 ||
      s.clusters * s.G < s.B || (s.clusters - 1) * s.G >= s.B || s.clusters >= (int64_t(1) << 31) ||
      s.L <= 0 ||
      s.A <= 0 || (s.D != 16 && s.D != 32 && s.D != 64 && s.D != 128) || s.A * s.D != s.C ||
      s.C > kSmallMaxHidden || s.F <= 0 || s.F > kSmallMaxFfn || s.V <= 0 ||
      s.V >= (int64_t(1) << 31) || s.T <= 0 || s.T > kSmallMaxCache)
    return false;
  if (s.L > s.weightLayers || s.L > s.normLayers || s.finalLayer < 0 || s.headLayer < 0)
    return false;
  const std::size_t bytes = std::size_t(smallLayout(s).total) * sizeof(float);
  if (bytes > kSmallMaxShared)
    return false;
  g->grid[0] = unsigned(s.clusters);
  g->block[0] = kSmallThreads;
  g->sharedBytes = unsigned(bytes);
  return true;
}

} // namespace

CKL_REGISTER_KERNEL("ckl.fused.decode_step_small",
                    reinterpret_cast<const void *>(&decodeStepSmallKernel),
                    "PPPPPPPPPPPPPPPPPPPPFFS", sizeof(DecodeStepSpec), decodeStepSmallGeometry,
                    nullptr, nullptr, 0, false);

} // namespace ckl::kernels
