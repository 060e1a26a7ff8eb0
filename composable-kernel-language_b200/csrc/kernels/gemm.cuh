// FP32 SIMT projection kernel with fused prologues and epilogues.
//
// out = epilogue(prologue(A) @ W[layer]), A row-major [M, K], W row-major [K, N] per layer.
// The decoder's projections must agree with an FP32 reference within 1e-4 relative, so they
// run on FFMA (no TF32).  A CTA computes a BM x BN tile with a TM x TN register tile per
// thread; K advances in BK-wide slices staged in double-buffered shared memory, loaded with
// 16-byte vectors when shapes and pointers allow (register prefetch of the next slice
// overlaps the FMAs of the current one).
//
// Prologues: plain; RMSNorm (row scale rsqrt(mean(x^2)+eps) times the layer gain, computed
// by the CTA for its rows before the K loop); SwiGLU (silu(gate) * up from two inputs).
// Epilogues: store; residual add; RoPE at position[0]; RoPE + KV-cache append; KV-cache
// append; store + per-row argmax partials for the greedy head.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace ckl::kernels::gemm {

enum Prologue : int { kPlain = 0, kRms = 1, kSwiGlu = 2 };
// kSwiGluPanel (tensor-core path only): the tile's columns are gate and up projections of the
// same outputs; the epilogue writes silu(gate) * up as a split operand panel.
enum Epilogue : int {
  kStore = 0, kResidual = 1, kRope = 2, kRopeAppend = 3, kAppend = 4, kArgmax = 5, kSwiGluPanel = 6,
  // q, k and v in one launch (tensor-core pair kernel only): column tiles of q take kRope into
  // out, of k kRopeAppend into out2, of v kAppend into out3.
  kQkv = 7
};

struct Params {
  const float *a = nullptr;        // [M, K]
  const float *a2 = nullptr;       // [M, K] up projection (SwiGLU)
  const float *gain = nullptr;     // [layers, K] (RMSNorm)
  const float *w = nullptr;        // [layers, K, N]
  const float *w2 = nullptr;       // [layers, K, N] up projection (kSwiGluPanel), k (kQkv)
  const float *w3 = nullptr;       // [layers, K, N] v (kQkv)
  const float *residual = nullptr; // [M, N]
  const float *table = nullptr;    // [T, D/2, 2]
  const int *position = nullptr;   // [1]
  float *out = nullptr;            // [M, N] or cache [layers, M, A, T, D]
  float *out2 = nullptr, *out3 = nullptr; // k and v caches (kQkv)
  float2 *partials = nullptr;      // [M, tiles] (value, index bits)
  float eps = 0.f;
  GemmSpec s{};
};

template <int BM_, int BN_, int BK_, int TM_, int TN_> struct Config {
  static constexpr int BM = BM_, BN = BN_, BK = BK_, TM = TM_, TN = TN_;
  static constexpr int kColThreads = BN / TN;
  static constexpr int kThreads = (BM / TM) * kColThreads;
  static constexpr int kALoads = (BM * BK / 4 + kThreads - 1) / kThreads; // float4 per thread
  static constexpr int kBLoads = (BK * BN / 4 + kThreads - 1) / kThreads;
  static_assert(BK % 4 == 0 && BN % 4 == 0 && TN % 2 == 0, "tile shape");
};

using Small = Config<16, 64, 16, 2, 4>;    // 128 threads, M <= 16
using Medium = Config<64, 64, 16, 4, 4>;   // 256 threads
using Large = Config<128, 128, 8, 8, 8>;   // 256 threads, M >= 256 and wide N

// The streamed few-row kernel (below) takes 1 to 16 rows (more than 8 as groups of 8 rows,
// grid.y) of a projection with 1 MB or more of weights whose K rows of A fit its
// shared-memory staging.
inline bool streamedFits(const GemmSpec &s) {
  return s.M <= 16 && s.N % 4 == 0 && s.K % 4 == 0 && s.K <= 4096 &&
         s.K * s.N >= (int64_t(1) << 18);
}

// Rows, CTA columns and threads of a streamed configuration (9-18).
inline int streamedRows(int config) {
  switch (config) {
  case 9: case 11: case 15: return 1;
  case 10: case 12: case 16: return 4;
  default: return 8;
  }
}
inline bool streamedWide(int config) { return config == 11 || config == 12 || config == 14; }
inline int streamedThreads(int config) { return config >= 15 ? 512 : 256; }
inline int streamedColumns(int config) {
  return streamedWide(config) ? 64 : config >= 15 && config <= 17 ? 8 : 16;
}

// Shared-memory floats of the streamed kernel: [the CTA's weight block, K x COLS, when staged],
// A [K][R], gains [K], the k-slots' sums [SLOTS][R x COLS + 4], the tile [R][COLS], row scales.
__host__ __device__ inline int64_t streamedFloats(int64_t K, int R, int COLS, int threads,
                                                  bool staged) {
  const int64_t slots = threads / (COLS / 4);
  return (staged ? K * COLS : 0) + K * R + K + slots * (R * COLS + 4) + R * COLS + 4;
}

// Whether the weight block is staged in shared memory (one round of cp.async for all of it):
// single-row launches whose layout fits a CTA and whose grid still runs in one wave at the
// resulting occupancy (two 256-thread CTAs per SM by registers, one of 512).  Measured at cfg5
// dimensions (same box, alternating builds): one request 0.234 -> 0.225 ms per step, four
// requests 0.299 -> 0.310 ms with staging, so it is kept for one row only.
constexpr int64_t kStreamedSms = 148;
constexpr int64_t kStreamedSharedLimit = 227 * 1024, kStreamedSmShared = 228 * 1024;
inline bool streamedStaged(const GemmSpec &s, int config, int64_t ctas) {
  if (streamedRows(config) != 1)
    return false;
  const int threads = streamedThreads(config);
  const int64_t bytes =
      4 * streamedFloats(s.K, streamedRows(config), streamedColumns(config), threads, true);
  if (bytes > kStreamedSharedLimit)
    return false;
  int64_t perSm = kStreamedSmShared / (bytes + 1024); // 1 KB reserved per CTA
  const int64_t byRegisters = threads == 512 ? 1 : 2;
  perSm = perSm < byRegisters ? perSm : byRegisters;
  return ctas <= kStreamedSms * perSm;
}

// Tile configuration for a specialization: 0 small, 1 medium, 2 large, 6/7/8 the few-row
// kernel for 1 / 4 / 16 rows, 9/10/13 the streamed few-row kernel for 1 / 4 / 8 rows with
// 16-column CTAs, 11/12/14 with 64-column CTAs (outputs of 16384 columns or more), 15/16/17
// with 8-column CTAs of 512 threads (K of 2048 or more: twice the CTAs of a narrow output) and
// 18 with 16-column CTAs of 512 threads (K of 2048 or more, 9 to 16 rows: two row groups of
// 8-column CTAs, each filling an SM's shared memory, would run in two waves).
// `config` 1-3 forces a tile; 0 (automatic) and 5 (FFMA only) choose by shape.
inline int chooseConfig(const GemmSpec &s) {
  if (s.config > 0 && s.config <= 3)
    return int(s.config - 1);
  if (streamedFits(s)) {
    const int rows = s.M <= 1 ? 0 : s.M <= 4 ? 1 : 2;
    if (s.N >= 16384)
      return rows == 2 ? 14 : 11 + rows;
    if (s.K >= 2048)
      return s.M > 8 ? 18 : 15 + rows;
    return rows == 2 ? 13 : 9 + rows;
  }
  if (s.M <= 1)
    return 6;
  if (s.M <= 4)
    return 7;
  if (s.M <= 16)
    return 8;
  if (s.M >= 256 && s.N >= 2048)
    return 2;
  return 1;
}

template <class Cfg> inline void tileGrid(const GemmSpec &s, library::Geometry *g) {
  g->grid[0] = ceilDiv(s.N, Cfg::BN);
  g->grid[1] = ceilDiv(s.M, Cfg::BM);
  g->block[0] = Cfg::kThreads;
}

inline bool geometry(const GemmSpec &s, library::Geometry *g) {
  if (s.M <= 0 || s.K <= 0 || s.N <= 0 || s.layers <= 0 || s.layer < 0 || s.layer >= s.layers)
    return false;
  switch (chooseConfig(s)) {
  case 0: tileGrid<Small>(s, g); break;
  case 1: tileGrid<Medium>(s, g); break;
  case 2: tileGrid<Large>(s, g); break;
  case 6:
  case 7:
  case 8:
    g->grid[0] = ceilDiv(s.N, 32);
    g->grid[1] = 1;
    g->block[0] = 256;
    break;
  case 9:
  case 10:
  case 11:
  case 12:
  case 13:
  case 14:
  case 15:
  case 16:
  case 17:
  case 18: {
    const int config = chooseConfig(s);
    const int threads = streamedThreads(config);
    g->grid[0] = ceilDiv(s.N, streamedColumns(config));
    g->grid[1] = ceilDiv(s.M, streamedRows(config));
    g->block[0] = unsigned(threads);
    const bool staged = streamedStaged(s, config, int64_t(g->grid[0]) * g->grid[1]);
    g->sharedBytes = unsigned(4 * streamedFloats(s.K, streamedRows(config),
                                                 streamedColumns(config), threads, staged));
    break;
  }
  default: return false;
  }
  return g->grid[1] <= 65535;
}

template <int PRO>
__device__ __forceinline__ float prologue(const Params &p, float v, int64_t m, int64_t k,
                                          const float *rowInv, int localRow) {
  if constexpr (PRO == kRms) {
    return __fmul_rn(__fmul_rn(v, rowInv[localRow]), p.gain[p.s.layer * p.s.K + k]);
  } else if constexpr (PRO == kSwiGlu) {
    const float up = p.a2[m * p.s.K + k];
    return __fmul_rn(v / (1.0f + expf(-v)), up);
  } else {
    return v;
  }
}

template <class Cfg, int PRO, int EPI> __device__ void body(const Params &p) {
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, TM = Cfg::TM, TN = Cfg::TN;
  constexpr int T = Cfg::kThreads;
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN];
  __shared__ float rowInv[BM];

  const GemmSpec &s = p.s;
  const int tid = threadIdx.x;
  const int tx = tid % Cfg::kColThreads, ty = tid / Cfg::kColThreads;
  const int64_t m0 = int64_t(blockIdx.y) * BM, n0 = int64_t(blockIdx.x) * BN;
  const int64_t M = s.M, K = s.K, N = s.N;
  const float *A = p.a;
  const float *W = p.w + s.layer * K * N;

  int position = 0;
  if constexpr (EPI == kRope || EPI == kRopeAppend || EPI == kAppend) {
    position = p.position[0];
    if (position < 0 || position >= s.T)
      return; // outside cache capacity: the step writes nothing
  }

  if constexpr (PRO == kRms) {
    const int warp = tid / kWarp, lane = tid % kWarp;
    for (int r = warp; r < BM; r += T / kWarp) {
      const int64_t m = m0 + r;
      float total = 0.f;
      if (m < M)
        for (int64_t k = lane; k < K; k += kWarp) {
          const float v = A[m * K + k];
          total += v * v;
        }
      total = warpSum(total);
      if (lane == 0)
        rowInv[r] = rsqrtf(total / float(K) + p.eps);
    }
    __syncthreads();
  }

  const bool vec = (K % 4 == 0) && (N % 4 == 0) && aligned16(A) && aligned16(W) &&
                   (PRO != kSwiGlu || aligned16(p.a2));
  float4 aReg[Cfg::kALoads], bReg[Cfg::kBLoads];

  auto loadA = [&](int64_t k0) {
#pragma unroll
    for (int l = 0; l < Cfg::kALoads; ++l) {
      const int e = tid + l * T; // float4 index within the BM x BK/4 tile
      const int r = e / (BK / 4), c = (e % (BK / 4)) * 4;
      const int64_t m = m0 + r, k = k0 + c;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < BM * BK / 4 && m < M) {
        if (vec && k + 3 < K) {
          v = *reinterpret_cast<const float4 *>(A + m * K + k);
        } else {
          v.x = k < K ? A[m * K + k] : 0.f;
          v.y = k + 1 < K ? A[m * K + k + 1] : 0.f;
          v.z = k + 2 < K ? A[m * K + k + 2] : 0.f;
          v.w = k + 3 < K ? A[m * K + k + 3] : 0.f;
        }
        if constexpr (PRO != kPlain) {
          if (k < K) v.x = prologue<PRO>(p, v.x, m, k, rowInv, r);
          if (k + 1 < K) v.y = prologue<PRO>(p, v.y, m, k + 1, rowInv, r);
          if (k + 2 < K) v.z = prologue<PRO>(p, v.z, m, k + 2, rowInv, r);
          if (k + 3 < K) v.w = prologue<PRO>(p, v.w, m, k + 3, rowInv, r);
        }
      }
      aReg[l] = v;
    }
  };
  auto storeA = [&](int stage) {
#pragma unroll
    for (int l = 0; l < Cfg::kALoads; ++l) {
      const int e = tid + l * T;
      if (e < BM * BK / 4) {
        const int r = e / (BK / 4), c = (e % (BK / 4)) * 4;
        As[stage][c][r] = aReg[l].x;
        As[stage][c + 1][r] = aReg[l].y;
        As[stage][c + 2][r] = aReg[l].z;
        As[stage][c + 3][r] = aReg[l].w;
      }
    }
  };
  auto loadB = [&](int64_t k0) {
#pragma unroll
    for (int l = 0; l < Cfg::kBLoads; ++l) {
      const int e = tid + l * T;
      const int r = e / (BN / 4), c = (e % (BN / 4)) * 4;
      const int64_t k = k0 + r, n = n0 + c;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < BK * BN / 4 && k < K) {
        const float *row = W + k * N;
        if (vec && n + 3 < N) {
          v = __ldg(reinterpret_cast<const float4 *>(row + n));
        } else {
          v.x = n < N ? row[n] : 0.f;
          v.y = n + 1 < N ? row[n + 1] : 0.f;
          v.z = n + 2 < N ? row[n + 2] : 0.f;
          v.w = n + 3 < N ? row[n + 3] : 0.f;
        }
      }
      bReg[l] = v;
    }
  };
  auto storeB = [&](int stage) {
#pragma unroll
    for (int l = 0; l < Cfg::kBLoads; ++l) {
      const int e = tid + l * T;
      if (e < BK * BN / 4) {
        const int r = e / (BN / 4), c = (e % (BN / 4)) * 4;
        *reinterpret_cast<float4 *>(&Bs[stage][r][c]) = bReg[l];
      }
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j)
      acc[i][j] = 0.f;

  loadA(0);
  loadB(0);
  storeA(0);
  storeB(0);
  __syncthreads();
  int stage = 0;
  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    const bool more = k0 + BK < K;
    if (more) {
      loadA(k0 + BK);
      loadB(k0 + BK);
    }
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i)
        a[i] = As[stage][kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; j += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(&Bs[stage][kk][tx * TN + j]);
        b[j] = v.x;
        if (j + 1 < TN) b[j + 1] = v.y;
        if (j + 2 < TN) b[j + 2] = v.z;
        if (j + 3 < TN) b[j + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j)
          acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) {
      storeA(stage ^ 1);
      storeB(stage ^ 1);
    }
    __syncthreads();
    stage ^= 1;
  }

  // ---- epilogue ----------------------------------------------------------------------
  const int64_t nBase = n0 + tx * TN;
  if constexpr (EPI == kArgmax) {
    // Store logits and reduce each row's maximum over this CTA's columns.
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t m = m0 + ty * TM + i;
      float best = -CUDART_INF_F;
      int bestIndex = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t n = nBase + j;
        if (m < M && n < N) {
          p.out[m * N + n] = acc[i][j];
          argmaxMerge(best, bestIndex, acc[i][j], int(n));
        }
      }
#pragma unroll
      for (int o = Cfg::kColThreads / 2; o > 0; o >>= 1)
        argmaxMerge(best, bestIndex, __shfl_xor_sync(0xffffffffu, best, o),
                    __shfl_xor_sync(0xffffffffu, bestIndex, o));
      if (tx == 0 && m < M)
        p.partials[m * s.tiles + blockIdx.x] = make_float2(best, __int_as_float(bestIndex));
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t m = m0 + ty * TM + i;
    if (m >= M)
      continue;
    if constexpr (EPI == kStore || EPI == kResidual) {
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t n = nBase + j;
        if (n < N) {
          float v = acc[i][j];
          if constexpr (EPI == kResidual)
            v = __fadd_rn(p.residual[m * N + n], v);
          p.out[m * N + n] = v;
        }
      }
    } else {
      const int64_t D = s.D, R = s.D / 2;
#pragma unroll
      for (int j = 0; j < TN; j += 2) {
        const int64_t n = nBase + j;
        if (n >= N)
          continue;
        float first = acc[i][j], second = acc[i][j + 1];
        const int64_t h = n / D, d = n % D;
        if constexpr (EPI == kRope || EPI == kRopeAppend) {
          const float *cs = p.table + (int64_t(position) * R + d / 2) * 2;
          const float cosine = cs[0], sine = cs[1];
          const float x = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
          const float y = __fadd_rn(__fmul_rn(first, sine), __fmul_rn(second, cosine));
          first = x;
          second = y;
        }
        if constexpr (EPI == kRope) {
          p.out[m * N + n] = first;
          p.out[m * N + n + 1] = second;
        } else {
          float *slot = p.out + (((s.layer * M + m) * s.A + h) * s.T + position) * D + d;
          slot[0] = first;
          slot[1] = second;
        }
      }
    }
  }
}

// ---- few-row projections (decode with up to 16 requests) -------------------------------
// The batch-1 decode GEMVs: a CTA owns 32 output columns (one per lane) for all rows; its 8
// warps split K.  Rows of A go through the prologue once per CTA into shared memory, a chunk
// of K at a time (k-major, read as broadcasts); each thread keeps one accumulator per row for
// its column and its K range, reading the weights as coalesced 128-byte rows; the warps'
// partial sums are added in warp order (deterministic) before the fused epilogue.
template <int ROWS> struct Rows {
  static constexpr int kRows = ROWS, kThreads = 256, kWarps = 8, kCols = 32, kChunk = 256;
};
using Rows1 = Rows<1>;
using Rows4 = Rows<4>;
using Rows16 = Rows<16>;

template <class Cfg> struct IsRows : std::false_type {};
template <int R> struct IsRows<Rows<R>> : std::true_type {};

template <class Cfg, int PRO, int EPI> __device__ void rowsBody(const Params &p) {
  constexpr int R = Cfg::kRows, KC = Cfg::kChunk, WARPS = Cfg::kWarps;
  constexpr int SLAB = KC / WARPS; // k per warp per chunk
  __shared__ float As[KC][R + 1];
  __shared__ float partial[WARPS][R][kWarp];
  __shared__ float rowInv[R];

  const GemmSpec &s = p.s;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int64_t M = s.M, K = s.K, N = s.N;
  const int64_t n = int64_t(blockIdx.x) * Cfg::kCols + lane;
  const float *A = p.a;
  const float *W = p.w + s.layer * K * N;

  int position = 0;
  if constexpr (EPI == kRope || EPI == kRopeAppend || EPI == kAppend) {
    position = p.position[0];
    if (position < 0 || position >= s.T)
      return; // outside cache capacity: the step writes nothing
  }
  if constexpr (PRO == kRms) {
    for (int m = warp; m < R; m += WARPS) {
      float total = 0.f;
      if (m < M)
        for (int64_t k = lane; k < K; k += kWarp) {
          const float v = A[m * K + k];
          total += v * v;
        }
      total = warpSum(total);
      if (lane == 0)
        rowInv[m] = rsqrtf(total / float(K) + p.eps);
    }
    __syncthreads();
  }

  float acc[R];
#pragma unroll
  for (int m = 0; m < R; ++m)
    acc[m] = 0.f;
  for (int64_t k0 = 0; k0 < K; k0 += KC) {
    for (int e = tid; e < KC * R; e += Cfg::kThreads) {
      const int m = e / KC, kk = e % KC;
      const int64_t k = k0 + kk;
      As[kk][m] = (m < M && k < K) ? prologue<PRO>(p, A[m * K + k], m, k, rowInv, m) : 0.f;
    }
    __syncthreads();
    const int64_t kEnd = K - k0 < KC ? K - k0 : KC;
#pragma unroll 8
    for (int kk = warp * SLAB; kk < (warp + 1) * SLAB; ++kk) {
      if (kk >= kEnd)
        break;
      const float w = n < N ? __ldg(W + (k0 + kk) * N + n) : 0.f;
#pragma unroll
      for (int m = 0; m < R; ++m)
        acc[m] = fmaf(As[kk][m], w, acc[m]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int m = 0; m < R; ++m)
    partial[warp][m][lane] = acc[m];
  __syncthreads();

  // One warp per row: lane = column.
  for (int m = warp; m < R && m < M; m += WARPS) {
    float v = partial[0][m][lane];
#pragma unroll
    for (int w = 1; w < WARPS; ++w)
      v = __fadd_rn(v, partial[w][m][lane]);
    if constexpr (EPI == kStore || EPI == kResidual || EPI == kArgmax) {
      if (n < N) {
        float out = v;
        if constexpr (EPI == kResidual)
          out = __fadd_rn(p.residual[m * N + n], v);
        p.out[m * N + n] = out;
      }
      if constexpr (EPI == kArgmax) {
        float best = n < N ? v : -CUDART_INF_F;
        int bestIndex = n < N ? int(n) : 0x7fffffff;
#pragma unroll
        for (int o = kWarp / 2; o > 0; o >>= 1)
          argmaxMerge(best, bestIndex, __shfl_xor_sync(0xffffffffu, best, o),
                      __shfl_xor_sync(0xffffffffu, bestIndex, o));
        if (lane == 0)
          p.partials[m * s.tiles + blockIdx.x] = make_float2(best, __int_as_float(bestIndex));
      }
    } else {
      // Adjacent columns (even n, n + 1) pair up across neighbouring lanes.
      const float other = __shfl_xor_sync(0xffffffffu, v, 1);
      if (lane % 2 == 0 && n < N) {
        float first = v, second = other;
        const int64_t D = s.D, R2 = s.D / 2, h = n / D, d = n % D;
        if constexpr (EPI == kRope || EPI == kRopeAppend) {
          const float *cs = p.table + (int64_t(position) * R2 + d / 2) * 2;
          const float cosine = cs[0], sine = cs[1];
          const float x = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
          const float y = __fadd_rn(__fmul_rn(first, sine), __fmul_rn(second, cosine));
          first = x;
          second = y;
        }
        if constexpr (EPI == kRope) {
          p.out[m * N + n] = first;
          p.out[m * N + n + 1] = second;
        } else {
          float *slot = p.out + (((s.layer * M + m) * s.A + h) * s.T + position) * D + d;
          slot[0] = first;
          slot[1] = second;
        }
      }
    }
  }
}

// ---- few-row projections streaming large weights (1 to 16 requests) ---------------------
// The kernel above gives a 1024-wide output 32 CTAs whose threads each keep eight 4-byte loads
// in flight, ~8 KB per CTA: far less than HBM needs to stream the weights of the decoder's
// larger projections (4-131 MB).  Here a CTA owns QUADS float4 columns and its 256 threads are
// QUADS quads x SLOTS k-slots: thread (q, j) reads the 16-byte quad q of k rows j, j + SLOTS,
// ..., kDepth loads in flight and the next kDepth issued before the current ones are used (a
// 1024-wide output runs on 64 CTAs of 16 columns, the LM head on 500 of 64).  The rows of A
// (all of K, at most eight rows: larger batches run as groups of eight rows, one per
// blockIdx.y, which stream the same weights together) go through the prologue into shared memory once, k-major and
// read as broadcasts, while the first loads are in flight.  Each thread keeps one float4
// accumulator per row over its k rows in increasing order; the k-slots' sums are added in slot
// order (deterministic) and the fused epilogue runs per (row, quad).
template <int ROWS, int QUADS, int THREADS = 256> struct Streamed {
  static constexpr int kRows = ROWS, kQuads = QUADS, kThreads = THREADS;
  static constexpr int kSlots = kThreads / QUADS, kCols = 4 * QUADS, kDepth = 8;
};
using Streamed1 = Streamed<1, 4>;
using Streamed4 = Streamed<4, 4>;
using Streamed1Wide = Streamed<1, 16>;
using Streamed4Wide = Streamed<4, 16>;
using Streamed8 = Streamed<8, 4>;
using Streamed8Wide = Streamed<8, 16>;
// 512 threads for deep K (2048 rows or more): twice the loads in flight per CTA, for grids
// of fewer CTAs than SMs or CTAs that fill an SM's shared memory alone; 8 columns per CTA up
// to eight rows (a 1024-wide output on 128 CTAs), 16 for two row groups.
using Streamed1Deep = Streamed<1, 2, 512>;
using Streamed4Deep = Streamed<4, 2, 512>;
using Streamed8Deep = Streamed<8, 2, 512>;
using Streamed8Deep16 = Streamed<8, 4, 512>;

template <class Cfg> struct IsStreamed : std::false_type {};
template <int R, int Q, int T> struct IsStreamed<Streamed<R, Q, T>> : std::true_type {};

// Dynamic shared memory (geometry, config 9-18): A [K][ROWS], the gains [K], the k-slots'
// sums [SLOTS][ROWS x COLS + 4], the reduced tile [ROWS][COLS] and the row scales.
template <class Cfg, int PRO, int EPI> __device__ void streamedBody(const Params &p) {
  constexpr int R = Cfg::kRows, Q = Cfg::kQuads, SLOTS = Cfg::kSlots, DEPTH = Cfg::kDepth;
  constexpr int COLS = Cfg::kCols, kThreads = Cfg::kThreads;
  extern __shared__ __align__(16) float dynamicShared[];
  const GemmSpec &s = p.s;
  const int64_t M = s.M, K = s.K, N = s.N;
  // Row group of this CTA (blockIdx.y): rows m0 .. m0 + rows - 1 of A and of the outputs.
  const int64_t m0 = int64_t(blockIdx.y) * R;
  const int64_t rows = M - m0 < R ? M - m0 : R;
  // The weight block [K][COLS] leads the layout when geometry allocated it (streamedStaged);
  // it is used when the weights also admit 16-byte copies.
  unsigned dynamicBytes;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dynamicBytes));
  const bool stagedLayout =
      int64_t(dynamicBytes) >= 4 * streamedFloats(K, R, COLS, kThreads, true);
  float *Ws = dynamicShared;                               // [K][COLS] (staged)
  float *As = dynamicShared + (stagedLayout ? K * COLS : 0); // [K][R]
  float *gainS = As + K * R;                 // [K] (RMSNorm)
  // k-slot j's sums at partial + j * SP: [R][COLS] plus 4 floats, so that the slots of a warp
  // start in different banks.
  constexpr int SP = R * COLS + 4;
  float *partial = gainS + K;                // [SLOTS][SP]
  float *tile = partial + SLOTS * SP;        // [R][COLS]
  float *rowInv = tile + R * COLS;           // [R]
  const int tid = threadIdx.x, q = tid % Q, slot = tid / Q;
  const int64_t n0 = int64_t(blockIdx.x) * COLS, n = n0 + 4 * q;
  const bool live = n < N; // N % 4 == 0 (geometry): a quad is inside or outside as a whole
  const float *W = p.w + s.layer * K * N + n;
  const bool vec = aligned16(p.w) && N % 4 == 0; // CTA-uniform

  int position = 0;
  if constexpr (EPI == kRope || EPI == kRopeAppend || EPI == kAppend) {
    position = p.position[0];
    if (position < 0 || position >= s.T)
      return; // outside cache capacity: the step writes nothing
  }
  auto load = [&](int64_t k) {
    if (!live || k >= K)
      return make_float4(0.f, 0.f, 0.f, 0.f);
    const float *row = W + k * N;
    return vec ? __ldg(reinterpret_cast<const float4 *>(row))
               : make_float4(__ldg(row), __ldg(row + 1), __ldg(row + 2), __ldg(row + 3));
  };
  const bool staged = stagedLayout && vec; // CTA-uniform
  float4 w[DEPTH];
  if (staged) {
    // The CTA's whole weight block in one round: row k's COLS columns, quads of 16 bytes.
    const float *block = p.w + s.layer * K * N + n0;
    for (int64_t e = tid; e < K * Q; e += kThreads) {
      const int64_t k = e / Q;
      const int qq = int(e % Q);
      float *dst = Ws + k * COLS + 4 * qq;
      if (n0 + 4 * qq < N)
        copyAsync16(dst, block + k * N + 4 * qq);
      else
        *reinterpret_cast<float4 *>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    copyAsyncCommit();
  } else {
#pragma unroll
    for (int d = 0; d < DEPTH; ++d)
      w[d] = load(slot + int64_t(d) * SLOTS);
  }

  // Rows of A into As [K][R] (k-major): every thread's float4s of the rows are loaded eight at
  // a time with all loads in flight (SwiGLU: silu(gate) * up as stored); for RMSNorm the raw
  // rows and the layer's gains are staged first, the rows' sums of squares reduced over the CTA
  // (fixed order) and the rows then scaled in place, x * inv * gain rounded as the reference.
  const int64_t K4 = K / 4; // K % 4 == 0 (streamedFits)
  const bool avec = aligned16(p.a) && (PRO != kSwiGlu || aligned16(p.a2)) &&
                    (PRO != kRms || aligned16(p.gain));
  auto load4 = [&](const float *at) {
    return avec ? *reinterpret_cast<const float4 *>(at)
                : make_float4(at[0], at[1], at[2], at[3]);
  };
  // Float4 f of the staging is row f % R, columns 4 (f / R) .. + 3: the lanes of a warp write
  // consecutive rows of the same k (few bank conflicts), and as kThreads % R == 0 every float4
  // of a thread is in row tid % R.
  static_assert(kThreads % R == 0, "rows per thread");
  float sumSquares = 0.f;
  for (int64_t f0 = tid; f0 < R * K4; f0 += 8 * kThreads) {
    float4 a[8], b[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t f = f0 + int64_t(u) * kThreads, m = f % R, k = 4 * (f / R);
      a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (f < R * K4 && m < rows) {
        a[u] = load4(p.a + (m0 + m) * K + k);
        if constexpr (PRO == kSwiGlu)
          b[u] = load4(p.a2 + (m0 + m) * K + k);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t f = f0 + int64_t(u) * kThreads, m = f % R, k = 4 * (f / R);
      if (f >= R * K4)
        continue;
      float4 v = a[u];
      if constexpr (PRO == kSwiGlu) {
        v = make_float4(__fmul_rn(a[u].x / (1.0f + expf(-a[u].x)), b[u].x),
                        __fmul_rn(a[u].y / (1.0f + expf(-a[u].y)), b[u].y),
                        __fmul_rn(a[u].z / (1.0f + expf(-a[u].z)), b[u].z),
                        __fmul_rn(a[u].w / (1.0f + expf(-a[u].w)), b[u].w));
      }
      if constexpr (PRO == kRms)
        sumSquares += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      As[(k + 0) * R + m] = v.x;
      As[(k + 1) * R + m] = v.y;
      As[(k + 2) * R + m] = v.z;
      As[(k + 3) * R + m] = v.w;
    }
  }
  if constexpr (PRO == kRms) {
    // The layer's gains beside A.
    for (int64_t k4 = tid; k4 < K4; k4 += kThreads)
      *reinterpret_cast<float4 *>(gainS + 4 * k4) = load4(p.gain + s.layer * K + 4 * k4);
    // Row sums: the lanes of one row (lane % R) by shuffles, then the warps in order.
    const int warp = tid / kWarp, lane = tid % kWarp;
    float *warpSums = partial; // [warps][R], free until the k-slots' sums
#pragma unroll
    for (int o = kWarp / 2; o >= R; o >>= 1)
      sumSquares += __shfl_xor_sync(0xffffffffu, sumSquares, o);
    if (lane < R)
      warpSums[warp * R + lane] = sumSquares;
    __syncthreads();
    if (tid < R) {
      float total = warpSums[tid];
      for (int w = 1; w < kThreads / kWarp; ++w)
        total += warpSums[w * R + tid];
      rowInv[tid] = rsqrtf(total / float(K) + p.eps);
    }
    __syncthreads();
    for (int64_t e = tid; e < K * R; e += kThreads) {
      const int m = int(e % R);
      As[e] = m < rows ? __fmul_rn(__fmul_rn(As[e], rowInv[m]), gainS[e / R]) : 0.f;
    }
  }
  if (staged)
    copyAsyncWaitAll(); // this thread's copies of the block; the barrier publishes everyone's
  __syncthreads();

  float4 acc[R];
#pragma unroll
  for (int m = 0; m < R; ++m)
    acc[m] = make_float4(0.f, 0.f, 0.f, 0.f);
  // This k row of every row of A (16-byte reads when R % 4 == 0).
  auto rowOfA = [&](int64_t k, float (&a)[R]) {
    if constexpr (R % 4 == 0) {
#pragma unroll
      for (int m = 0; m < R; m += 4) {
        const float4 four = *reinterpret_cast<const float4 *>(&As[k * R + m]);
        a[m] = four.x, a[m + 1] = four.y, a[m + 2] = four.z, a[m + 3] = four.w;
      }
    } else {
#pragma unroll
      for (int m = 0; m < R; ++m)
        a[m] = As[k * R + m];
    }
  };
  if (staged) {
#pragma unroll 4
    for (int64_t k = slot; k < K; k += SLOTS) {
      const float4 wk = *reinterpret_cast<const float4 *>(&Ws[k * COLS + 4 * q]);
      float a[R];
      rowOfA(k, a);
#pragma unroll
      for (int m = 0; m < R; ++m) {
        acc[m].x = fmaf(a[m], wk.x, acc[m].x);
        acc[m].y = fmaf(a[m], wk.y, acc[m].y);
        acc[m].z = fmaf(a[m], wk.z, acc[m].z);
        acc[m].w = fmaf(a[m], wk.w, acc[m].w);
      }
    }
  }
  for (int64_t base = slot; !staged && base < K; base += int64_t(DEPTH) * SLOTS) {
    float4 next[DEPTH];
#pragma unroll
    for (int d = 0; d < DEPTH; ++d)
      next[d] = load(base + int64_t(DEPTH + d) * SLOTS);
#pragma unroll
    for (int d = 0; d < DEPTH; ++d) {
      const int64_t k = base + int64_t(d) * SLOTS;
      if (k < K) {
        float a[R];
        rowOfA(k, a);
#pragma unroll
        for (int m = 0; m < R; ++m) {
          acc[m].x = fmaf(a[m], w[d].x, acc[m].x);
          acc[m].y = fmaf(a[m], w[d].y, acc[m].y);
          acc[m].z = fmaf(a[m], w[d].z, acc[m].z);
          acc[m].w = fmaf(a[m], w[d].w, acc[m].w);
        }
      }
    }
#pragma unroll
    for (int d = 0; d < DEPTH; ++d)
      w[d] = next[d];
  }
#pragma unroll
  for (int m = 0; m < R; ++m)
    *reinterpret_cast<float4 *>(&partial[slot * SP + m * COLS + 4 * q]) = acc[m];
  __syncthreads();
  // Sum of the k-slots of every (row, column), in slot order.
  for (int o = tid; o < R * COLS; o += kThreads) {
    float v = partial[o];
#pragma unroll 16
    for (int j = 1; j < SLOTS; ++j)
      v = __fadd_rn(v, partial[j * SP + o]);
    tile[o] = v;
  }
  __syncthreads();

  if constexpr (EPI == kArgmax) {
    // One warp per row: the row's logits over the CTA's columns, then its argmax partial.
    const int warp = tid / kWarp, lane = tid % kWarp;
    for (int m = warp; m < R && m < rows; m += kThreads / kWarp) {
      float best = -CUDART_INF_F;
      int bestIndex = 0x7fffffff;
      for (int c = lane; c < COLS; c += kWarp) {
        const int64_t col = n0 + c;
        if (col < N) {
          const float v = tile[m * COLS + c];
          p.out[(m0 + m) * N + col] = v;
          argmaxMerge(best, bestIndex, v, int(col));
        }
      }
#pragma unroll
      for (int o = kWarp / 2; o > 0; o >>= 1)
        argmaxMerge(best, bestIndex, __shfl_xor_sync(0xffffffffu, best, o),
                    __shfl_xor_sync(0xffffffffu, bestIndex, o));
      if (lane == 0)
        p.partials[(m0 + m) * s.tiles + blockIdx.x] =
            make_float2(best, __int_as_float(bestIndex));
    }
    return;
  }
  // One thread per (row, quad) of the tile.
  if (tid >= R * Q)
    return;
  const int m = tid / Q, qq = tid % Q;
  const int64_t c = n0 + 4 * qq;
  if (m >= rows || c >= N)
    return;
  float4 v = *reinterpret_cast<const float4 *>(&tile[m * COLS + 4 * qq]);
  if constexpr (EPI == kStore || EPI == kResidual) {
    float *lanes = &v.x;
    if constexpr (EPI == kResidual) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        lanes[j] = __fadd_rn(p.residual[(m0 + m) * N + c + j], lanes[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      p.out[(m0 + m) * N + c + j] = lanes[j];
  } else {
    // Pairs (c, c + 1) and (c + 2, c + 3): c is a multiple of 4 and D is even, so a pair never
    // straddles two heads.
    const float *lanes = &v.x;
    const int64_t D = s.D, R2 = s.D / 2;
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const int64_t col = c + j, h = col / D, d = col % D;
      float first = lanes[j], second = lanes[j + 1];
      if constexpr (EPI == kRope || EPI == kRopeAppend) {
        const float *cs = p.table + (int64_t(position) * R2 + d / 2) * 2;
        const float cosine = cs[0], sine = cs[1];
        const float x = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
        const float y = __fadd_rn(__fmul_rn(first, sine), __fmul_rn(second, cosine));
        first = x;
        second = y;
      }
      if constexpr (EPI == kRope) {
        p.out[(m0 + m) * N + col] = first;
        p.out[(m0 + m) * N + col + 1] = second;
      } else {
        float *at = p.out + (((s.layer * M + m0 + m) * s.A + h) * s.T + position) * D + d;
        at[0] = first;
        at[1] = second;
      }
    }
  }
}

// The projection body of a tile configuration.
template <class Cfg, int PRO, int EPI> __device__ __forceinline__ void dispatch(const Params &p) {
  if constexpr (IsRows<Cfg>::value)
    rowsBody<Cfg, PRO, EPI>(p);
  else if constexpr (IsStreamed<Cfg>::value)
    streamedBody<Cfg, PRO, EPI>(p);
  else
    body<Cfg, PRO, EPI>(p);
}

} // namespace ckl::kernels::gemm
