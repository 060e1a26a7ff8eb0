// Tensor-core path of the decoder's batched projections (benchmarks/decoder/workloads.py:191-254
// with 17 or more requests).
//
// Each projection's activation operand is split into a TF32 hi/lo panel once, by the kernel
// that produces it, and every projection then runs the tcgen05 3xTF32 kernel (tcgemm.cuh) on
// that panel with the layer's FP32 weights:
//   rms_panel:    panel = split(RMSNorm(x) * gain)        (feeds q/k/v, gate/up, lm head)
//   attention writes its context rows as a panel           (feeds the o projection)
//   panel_gate_up: panel = split(silu(a @ wg) * (a @ wu))  (feeds the down projection)
//   panel_linear{,_rope,_rope_append,_append,_residual,_argmax}: the projections with the same
//   fused epilogues as the FFMA kernels.
// The normalised values are rounded exactly as in the FFMA kernels (x * rsqrt(mean(x^2) + eps)
// * gain); silu(g) * u uses the fast division (within 2 ulp of the FFMA kernels' value) before
// the split.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ckl_b200.h"
#include "common.cuh"
#include "gemm.cuh"
#include "panel.cuh"
#include "tcgemm.cuh"
#include "tcpair.cuh"

namespace ckl::kernels {
namespace {

using gemm::Params;

// ---- panel producers -----------------------------------------------------------------------
constexpr int kPanelWarps = 4;

// One warp per row: sum of squares, then the normalised row split into the panel.  Columns
// between K and the next multiple of 32 are written as zeros.  Rows of up to 1024 columns are
// held in registers between the two passes.
constexpr int kRmsHeld = 8; // float4 per lane

__device__ __forceinline__ float4 rmsScale(const float4 &a, float inv, const float4 &g) {
  return make_float4(__fmul_rn(__fmul_rn(a.x, inv), g.x), __fmul_rn(__fmul_rn(a.y, inv), g.y),
                     __fmul_rn(__fmul_rn(a.z, inv), g.z), __fmul_rn(__fmul_rn(a.w, inv), g.w));
}

// Rows of up to 1024 columns (the decoder's common case) take the staged path: the CTA's
// eight normalised rows go to shared memory, then eight consecutive threads store one 8-row x
// 16-byte core matrix of the panel (128 contiguous bytes) instead of each lane storing 16 bytes
// 2 KB apart along its own row.  The arithmetic is the same on both paths.
constexpr int kStagedColumns = 4 * kWarp * kRmsHeld; // 1024

__global__ void __launch_bounds__(kPanelWarps *kWarp)
    rmsPanelKernel(const float *x, const float *gain, float *out, float eps, RmsApplySpec s) {
  dependentLaunchEntry();
  __shared__ __align__(16) float staged[kPanelWarps][kStagedColumns + 4]; // +4: no bank conflicts
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t m = int64_t(blockIdx.x) * kPanelWarps + warp;
  const int64_t K = s.C;
  const float *g = gain + s.layer * K;
  const bool vec = K % 4 == 0 && aligned16(x) && aligned16(g);
  const int64_t padded = panel::slices(K) * panel::kSlice;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  if (vec && padded <= kStagedColumns) { // uniform over the CTA
    if (m < s.B) {
      const float4 *row4 = reinterpret_cast<const float4 *>(x + m * K);
      float4 held[kRmsHeld];
      float total = 0.f;
#pragma unroll
      for (int i = 0; i < kRmsHeld; ++i) {
        const int64_t q = lane + i * kWarp;
        held[i] = q < K / 4 ? row4[q] : zero;
        total += held[i].x * held[i].x + held[i].y * held[i].y + held[i].z * held[i].z +
                 held[i].w * held[i].w;
      }
      total = warpSum(total);
      const float inv = rsqrtf(total / float(K) + eps);
#pragma unroll
      for (int i = 0; i < kRmsHeld; ++i) {
        const int64_t k = 4 * (lane + int64_t(i) * kWarp);
        if (k < padded)
          *reinterpret_cast<float4 *>(&staged[warp][k]) =
              k < K ? rmsScale(held[i], inv, reinterpret_cast<const float4 *>(g)[k / 4]) : zero;
      }
    }
    __syncthreads();
    const int64_t m0 = int64_t(blockIdx.x) * kPanelWarps;
    for (int64_t i = threadIdx.x; i < kPanelWarps * (padded / 4); i += kPanelWarps * kWarp) {
      const int r = int(i % kPanelWarps);
      const int64_t k = 4 * (i / kPanelWarps);
      if (m0 + r < s.B)
        panel::store4(out, m0 + r, k, K, *reinterpret_cast<const float4 *>(&staged[r][k]));
    }
    return;
  }
  if (m >= s.B)
    return;
  const float *row = x + m * K;
  float total = 0.f;
  if (vec) {
    for (int64_t q = lane; q < K / 4; q += kWarp) {
      const float4 v = reinterpret_cast<const float4 *>(row)[q];
      total += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  } else {
    for (int64_t k = lane; k < K; k += kWarp)
      total += row[k] * row[k];
  }
  total = warpSum(total);
  const float inv = rsqrtf(total / float(K) + eps);
  for (int64_t k = 4 * int64_t(lane); k < padded; k += 4 * kWarp) {
    float4 v;
    if (vec && k < K) {
      v = rmsScale(reinterpret_cast<const float4 *>(row)[k / 4], inv,
                   reinterpret_cast<const float4 *>(g)[k / 4]);
    } else {
      float *lanes = &v.x;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        lanes[j] = k + j < K ? __fmul_rn(__fmul_rn(row[k + j], inv), g[k + j]) : 0.f;
    }
    panel::store4(out, m, k, K, v);
  }
}

bool rmsPanelGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<RmsApplySpec>(spec);
  if (s.B <= 0 || s.C <= 0 || s.layer < 0 || s.layer >= s.L)
    return false;
  g->grid[0] = ceilDiv(s.B, kPanelWarps);
  g->block[0] = kPanelWarps * kWarp;
  return true;
}

// ---- projections on a panel ------------------------------------------------------------------
// Every projection takes the panel of A, the weights [layers, K, N], its outputs, the
// specialization and (last, added at bind time) the weights' tensor map.  SPLITS > 1 splits
// K over a cluster of that many CTAs per output tile.
#define CKL_PANEL_KERNEL(fn, EPI, params, assign)                                               \
  template <int BN, int SPLITS, int MT>                                                        \
  __global__ void __cluster_dims__(1, 1, SPLITS) __launch_bounds__(tc::kThreads)               \
      fn(const float *a, const float *w, CKL_UNPACK params, GemmSpec s,                         \
         const __grid_constant__ tc::WeightMap weights) {                                      \
    dependentLaunchEntry();                                                                    \
    Params p;                                                                                  \
    p.a = a, p.w = w, p.s = s;                                                                 \
    CKL_UNPACK assign;                                                                         \
    tc::body<BN, EPI, SPLITS, MT>(p, weights);                                                 \
  }
#define CKL_UNPACK(...) __VA_ARGS__

CKL_PANEL_KERNEL(panelLinearTc, gemm::kStore, (float *dst), (p.out = dst))
CKL_PANEL_KERNEL(panelLinearRopeTc, gemm::kRope,
                 (const float *table, const int *position, float *dst),
                 (p.table = table, p.position = position, p.out = dst))
CKL_PANEL_KERNEL(panelLinearRopeAppendTc, gemm::kRopeAppend,
                 (const float *table, const int *position, float *cache),
                 (p.table = table, p.position = position, p.out = cache))
CKL_PANEL_KERNEL(panelLinearAppendTc, gemm::kAppend, (const int *position, float *cache),
                 (p.position = position, p.out = cache))
CKL_PANEL_KERNEL(panelLinearResidualTc, gemm::kResidual, (const float *residual, float *dst),
                 (p.residual = residual, p.out = dst))
CKL_PANEL_KERNEL(panelLinearArgmaxTc, gemm::kArgmax, (float *logits, float2 *partials),
                 (p.out = logits, p.partials = partials))
// Argmax partials only, no logits (the batched prefill's heads: only the greedy tokens of the
// prompt positions are kept, as history).
CKL_PANEL_KERNEL(panelArgmaxTc, gemm::kArgmax, (float2 *partials),
                 (p.out = nullptr, p.partials = partials))

// Fused gate/up/SwiGLU: out is the panel of silu(a @ wg) * (a @ wu) [M, N].
template <int MT>
__global__ void __launch_bounds__(tc::kThreads)
    panelGateUpTc(const float *a, const float *wg, const float *wu, float *out, GemmSpec s,
                  const __grid_constant__ tc::WeightMapPair maps) {
  dependentLaunchEntry();
  Params p;
  p.a = a, p.w = wg, p.w2 = wu, p.out = out, p.s = s;
  tc::body<128, gemm::kSwiGluPanel, 1, MT>(p, maps.gate, &maps.up);
}

// ---- 2-SM pair kernels (tcpair.cuh) for the wide projections --------------------------------
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc::kThreads, 1)
    panelLinearArgmaxPairTc(const float *a, const float *w, float *logits, float2 *partials,
                            GemmSpec s, const __grid_constant__ tc::WeightMap weights) {
  dependentLaunchEntry();
  Params p;
  p.a = a, p.w = w, p.out = logits, p.partials = partials, p.s = s;
  tc::pair::body<gemm::kArgmax, 1, tc::pair::kWide>(p, weights);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc::kThreads, 1)
    panelArgmaxPairTc(const float *a, const float *w, float2 *partials, GemmSpec s,
                      const __grid_constant__ tc::WeightMap weights) {
  dependentLaunchEntry();
  Params p;
  p.a = a, p.w = w, p.out = nullptr, p.partials = partials, p.s = s;
  tc::pair::body<gemm::kArgmax, 1, tc::pair::kWide>(p, weights);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(tc::kThreads, 1)
    panelGateUpPairTc(const float *a, const float *wg, const float *wu, float *out, GemmSpec s,
                      const __grid_constant__ tc::WeightMapPair maps) {
  dependentLaunchEntry();
  Params p;
  p.a = a, p.w = wg, p.w2 = wu, p.out = out, p.s = s;
  tc::pair::body<gemm::kSwiGluPanel, 1, tc::pair::kWide>(p, maps.gate, &maps.up);
}

// The projections with store / RoPE / KV-append / residual epilogues on CTA pairs, K split
// over SPLITS pairs of one cluster (2 x 1 x SPLITS).
#define CKL_PAIR_KERNEL(fn, EPI, params, assign)                                                \
  template <int SPLITS, int BN>                                                                \
  __global__ void __cluster_dims__(2, 1, SPLITS) __launch_bounds__(tc::kThreads, 1)            \
      fn(const float *a, const float *w, CKL_UNPACK params, GemmSpec s,                         \
         const __grid_constant__ tc::WeightMap weights) {                                      \
    dependentLaunchEntry();                                                                    \
    Params p;                                                                                  \
    p.a = a, p.w = w, p.s = s;                                                                 \
    CKL_UNPACK assign;                                                                         \
    tc::pair::body<EPI, SPLITS, BN>(p, weights);                                               \
  }

CKL_PAIR_KERNEL(panelLinearPairTc, gemm::kStore, (float *dst), (p.out = dst))
CKL_PAIR_KERNEL(panelLinearRopePairTc, gemm::kRope,
                (const float *table, const int *position, float *dst),
                (p.table = table, p.position = position, p.out = dst))
CKL_PAIR_KERNEL(panelLinearRopeAppendPairTc, gemm::kRopeAppend,
                (const float *table, const int *position, float *cache),
                (p.table = table, p.position = position, p.out = cache))
CKL_PAIR_KERNEL(panelLinearAppendPairTc, gemm::kAppend, (const int *position, float *cache),
                (p.position = position, p.out = cache))
CKL_PAIR_KERNEL(panelLinearResidualPairTc, gemm::kResidual, (const float *residual, float *dst),
                (p.residual = residual, p.out = dst))

// q, k and v in one launch on pairs: the panel of the normalised rows times wq | wk | wv, each
// 256-column tile with its projection's epilogue (RoPE into q; RoPE and cache append into kc;
// cache append into vc).
template <int SPLITS>
__global__ void __cluster_dims__(2, 1, SPLITS) __launch_bounds__(tc::kThreads, 1)
    panelQkvPairTc(const float *a, const float *wq, const float *wk, const float *wv,
                   const float *table, const int *position, float *q, float *kc, float *vc,
                   GemmSpec s, const __grid_constant__ tc::WeightMapTriple maps) {
  dependentLaunchEntry();
  Params p;
  p.a = a, p.w = wq, p.w2 = wk, p.w3 = wv, p.table = table, p.position = position;
  p.out = q, p.out2 = kc, p.out3 = vc, p.s = s;
  tc::pair::body<gemm::kQkv, SPLITS, tc::pair::kWide>(p, maps.q, &maps.k, &maps.v);
}

// Pair kernels run a projection when its output spans at least two row tiles, one tile width
// of columns, and pair tiles for at least 96 CTAs (about two thirds of the SMs); otherwise the
// single-CTA kernel with its row-tile sharing and K splits fills the GPU better.
// CKL_B200_TC_PAIRS (read when a program is compiled and again when it is bound; keep it
// unchanged between the two, or the bound kernel may not match the planned grid): 0 keeps the
// single-CTA kernel everywhere, 2 takes pairs whenever there are two row tiles (tests of small
// shapes).
bool usePairs(const GemmSpec &s, int64_t tileColumns) {
  const char *mode = std::getenv("CKL_B200_TC_PAIRS");
  if ((mode && mode[0] == '0') || s.N < tileColumns || s.K <= 0)
    return false;
  const int64_t rowTiles = (s.M + tc::BM - 1) / tc::BM;
  if (rowTiles < 2)
    return false;
  if (mode && mode[0] == '2')
    return true;
  const int64_t pairTiles = ((rowTiles + 1) / 2) * ((s.N + tileColumns - 1) / tileColumns);
  return 2 * pairTiles >= 96;
}

bool argmaxPairs(const GemmSpec &s) { return usePairs(s, tc::pair::kWide); }
bool gateUpPairs(const GemmSpec &s) { return usePairs(s, tc::pair::kWide / 2); }

// CTAs of a pair grid without K splits.
int64_t pairCtas(const GemmSpec &s, int64_t tileColumns) {
  const int64_t rowTiles = (s.M + tc::BM - 1) / tc::BM;
  return 2 * ((rowTiles + 1) / 2) * ((s.N + tileColumns - 1) / tileColumns);
}

// K splits on pairs: doubled while the grid stays within one CTA per SM and every split keeps
// at least two slices; at most 4 (portable 8-CTA clusters) for 128-wide tiles, 8 (16-CTA
// clusters) for 256-wide ones.
int pairSplits(const GemmSpec &s, int width) {
  const int64_t ctas = pairCtas(s, width), slices = panel::slices(s.K);
  const int most = width == tc::pair::kWide ? 8 : 4;
  int splits = 1;
  while (splits < most && ctas * splits * 2 <= tc::kTargetCtas && slices >= int64_t(splits) * 4)
    splits *= 2;
  return splits;
}

// Pair tile width of the linear family (q/k/v/o/down and the prefill projections), 0 for the
// single-CTA kernel: 256-wide tiles when they give at least 96 CTAs without K splits (the
// batched prefill).  The 1024-wide decode projections at 512 rows keep the single-CTA
// kernel's 128 CTAs: on 256-wide pairs split over 4-pair clusters they get 64 CTAs and
// measured slower (27 vs 24.5 us for q), and on 128-wide pairs (each CTA holding 64 weight
// columns, 32 pair CTAs x 4 splits = 128 CTAs) slower still (q ~37 us, o/down shares
// 5.2 -> 7.5 % of the step): with eight 32-deep slices per CTA the pair's start-up, split
// reduction and cluster barriers outweigh the halved operand traffic.
// 256-wide pairs with an eight-way K split on 16-CTA clusters (128 CTAs for the o and down
// projections at the cfg5 shard) measured slower too: o/down 5.5 -> 6.2 % of the step, 5.60
// -> 5.66 ms per step in one call; forced pairs still take them where the grid is small.
// CKL_B200_TC_PAIRS=2 / 3 force 256- / 128-wide pairs wherever there are two row tiles (the
// tests run every tensor-core shape both ways), =0 disables pairs.
int linearPairWidth(const GemmSpec &s) {
  const char *mode = std::getenv("CKL_B200_TC_PAIRS");
  const int64_t rowTiles = (s.M + tc::BM - 1) / tc::BM;
  if ((mode && mode[0] == '0') || s.K <= 0 || rowTiles < 2)
    return 0;
  if (mode && mode[0] == '2')
    return s.N >= tc::pair::kWide ? tc::pair::kWide : 0;
  if (mode && mode[0] == '3')
    return s.N >= tc::pair::kNarrow ? tc::pair::kNarrow : 0;
  return usePairs(s, tc::pair::kWide) ? tc::pair::kWide : 0;
}

// The fused q/k/v node applies when each projection is a whole number of 256-wide tiles, there
// are two row tiles, and the 3N-wide pair grid with its K splits gives at least 96 CTAs (the
// cfg5 shard: 12 column tiles x 2 row pairs x 2 splits); otherwise the planner keeps three
// nodes.  CKL_B200_TC_PAIRS=0 (or CKL_B200_TC_QKV=0) disables it, CKL_B200_TC_PAIRS=2 / 3 take
// it whenever the shape allows.
bool qkvPairs(const GemmSpec &s, GemmSpec *wide = nullptr) {
  const char *mode = std::getenv("CKL_B200_TC_PAIRS");
  const char *fused = std::getenv("CKL_B200_TC_QKV");
  const int64_t rowTiles = (s.M + tc::BM - 1) / tc::BM;
  if ((mode && mode[0] == '0') || (fused && fused[0] == '0') || s.K <= 0 || s.N <= 0 || s.N % tc::pair::kWide != 0 ||
      rowTiles < 2)
    return false;
  GemmSpec all = s;
  all.N = 3 * s.N;
  if (wide)
    *wide = all;
  if (mode && (mode[0] == '2' || mode[0] == '3'))
    return true;
  return pairCtas(all, tc::pair::kWide) * pairSplits(all, tc::pair::kWide) >= 96;
}

void pairGeometry(const GemmSpec &s, int64_t tileColumns, library::Geometry *g,
                  int splits = 1, int width = tc::pair::kWide) {
  const int64_t rowTiles = (s.M + tc::BM - 1) / tc::BM;
  g->grid[0] = 2 * ceilDiv(s.N, tileColumns);
  g->grid[1] = unsigned((rowTiles + 1) / 2);
  g->grid[2] = unsigned(splits);
  g->block[0] = tc::kThreads;
  g->sharedBytes = unsigned(tc::pair::sharedBytes(width));
}

// Row tiles per CTA of the gate/up kernel (full-width tiles of 64 gate + 64 up columns): two
// when single-tile CTAs would already fill the SMs.
int gateUpRowTiles(const GemmSpec &s) {
  const int64_t tiles = int64_t(ceilDiv(s.M, tc::BM)) * ceilDiv(s.N, tc::BM / 2);
  return s.M > tc::BM && tiles >= tc::kTargetCtas ? 2 : 1;
}

bool gateUpGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GemmSpec>(spec);
  if (s.M <= 0 || s.K <= 0 || s.N <= 0 || s.layers <= 0 || s.layer < 0 || s.layer >= s.layers)
    return false;
  if (gateUpPairs(s)) {
    pairGeometry(s, tc::pair::kWide / 2, g);
    return g->grid[1] <= 65535;
  }
  const int mt = gateUpRowTiles(s);
  g->grid[0] = ceilDiv(s.N, tc::BM / 2);
  g->grid[1] = ceilDiv(ceilDiv(s.M, tc::BM), mt);
  g->block[0] = tc::kThreads;
  g->sharedBytes = unsigned(tc::sharedBytes(128, mt));
  return g->grid[1] <= 65535;
}

const void *gateUpSelect(const void *spec) {
  if (gateUpPairs(specOf<GemmSpec>(spec)))
    return reinterpret_cast<const void *>(&panelGateUpPairTc);
  return gateUpRowTiles(specOf<GemmSpec>(spec)) == 2
             ? reinterpret_cast<const void *>(&panelGateUpTc<2>)
             : reinterpret_cast<const void *>(&panelGateUpTc<1>);
}

// Tensor map of the weights [layers, K, N] for the kernel's column width, built once per bound
// node from the resolved weight pointer (slot 1 of every panel projection).  Weights whose
// shape or address admit no map get valid == 0 and are read with plain loads.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encodeTiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *entry = nullptr;
    cudaDriverEntryPointQueryResult found{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &entry, cudaEnableDefault, &found) ==
            cudaSuccess &&
        found == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(entry);
    else
      cudaGetLastError();
  });
  return fn;
}

// Map of the weights at `address` with a box of `width` columns x 32 rows x 1 layer.
tc::WeightMap weightMap(uint64_t address, const GemmSpec &s, int width) {
  tc::WeightMap local;
  std::memset(&local, 0, sizeof(local));
  const EncodeTiledFn encode = encodeTiled();
  if (encode != nullptr && s.N % 4 == 0 && address % 16 == 0 && s.K > 0 && s.N > 0 &&
      s.layers > 0) {
    const cuuint64_t dims[3] = {cuuint64_t(s.N), cuuint64_t(s.K), cuuint64_t(s.layers)};
    const cuuint64_t strides[2] = {cuuint64_t(s.N) * 4, cuuint64_t(s.K) * cuuint64_t(s.N) * 4};
    const cuuint32_t box[3] = {cuuint32_t(width), cuuint32_t(tc::BK), 1};
    const cuuint32_t unit[3] = {1, 1, 1};
    const CUresult status =
        encode(&local.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, reinterpret_cast<void *>(address),
               dims, strides, box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    local.valid = status == CUDA_SUCCESS ? 1 : 0;
  }
  return local;
}

uint64_t pointerSlot(const void *const *arguments, std::size_t index) {
  uint64_t address = 0;
  std::memcpy(&address, arguments[index], sizeof(address));
  return address;
}

// Box width: half a pair tile of the linear family, or the single-CTA kernel's tile width.
bool prepareWeights(const void *spec, const void *const *arguments, std::size_t count,
                    void *extra) {
  if (spec == nullptr || count < 2)
    return false;
  const GemmSpec &s = specOf<GemmSpec>(spec);
  const int pairWidth = linearPairWidth(s);
  const int width = pairWidth ? pairWidth / 2 : tc::chooseWidth(s);
  const tc::WeightMap map = weightMap(pointerSlot(arguments, 1), s, width);
  std::memcpy(extra, &map, sizeof(map));
  return true;
}

// The argmax heads: their pair tiles (256 wide, N >= 256) and the single-CTA kernel's tiles
// (128 wide for N > 64) both take boxes of chooseWidth(s) columns.
bool prepareArgmaxWeights(const void *spec, const void *const *arguments, std::size_t count,
                          void *extra) {
  if (spec == nullptr || count < 2)
    return false;
  const GemmSpec &s = specOf<GemmSpec>(spec);
  const tc::WeightMap map = weightMap(pointerSlot(arguments, 1), s, tc::chooseWidth(s));
  std::memcpy(extra, &map, sizeof(map));
  return true;
}

// Gate weights in slot 1, up weights in slot 2; boxes of half a tile each (the pair kernel's
// tile: 128 gate columns in the leader, 128 up columns in its peer).
bool prepareGateUp(const void *spec, const void *const *arguments, std::size_t count,
                   void *extra) {
  if (spec == nullptr || count < 3)
    return false;
  const GemmSpec &s = specOf<GemmSpec>(spec);
  const int width = gateUpPairs(s) ? tc::pair::kWide / 2 : tc::BM / 2;
  tc::WeightMapPair maps;
  maps.gate = weightMap(pointerSlot(arguments, 1), s, width);
  maps.up = weightMap(pointerSlot(arguments, 2), s, width);
  std::memcpy(extra, &maps, sizeof(maps));
  return true;
}

// Weights of q, k and v in slots 1-3; 128-column boxes (half of a 256-wide pair tile).
bool prepareQkv(const void *spec, const void *const *arguments, std::size_t count,
                void *extra) {
  if (spec == nullptr || count < 4)
    return false;
  const GemmSpec &s = specOf<GemmSpec>(spec);
  tc::WeightMapTriple maps;
  maps.q = weightMap(pointerSlot(arguments, 1), s, tc::pair::kWide / 2);
  maps.k = weightMap(pointerSlot(arguments, 2), s, tc::pair::kWide / 2);
  maps.v = weightMap(pointerSlot(arguments, 3), s, tc::pair::kWide / 2);
  std::memcpy(extra, &maps, sizeof(maps));
  return true;
}

bool qkvGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GemmSpec>(spec);
  GemmSpec all;
  if (s.M <= 0 || s.layers <= 0 || s.layer < 0 || s.layer >= s.layers || s.D <= 0 ||
      s.D % 2 || s.N != s.A * s.D || s.T <= 0 || !qkvPairs(s, &all))
    return false;
  const int splits = pairSplits(all, tc::pair::kWide);
  pairGeometry(all, tc::pair::kWide, g, splits, tc::pair::kWide);
  return g->grid[1] <= 65535;
}

const void *qkvSelect(const void *spec) {
  GemmSpec all;
  if (!qkvPairs(specOf<GemmSpec>(spec), &all))
    return nullptr;
  switch (pairSplits(all, tc::pair::kWide)) {
  case 8: return reinterpret_cast<const void *>(&panelQkvPairTc<8>);
  case 4: return reinterpret_cast<const void *>(&panelQkvPairTc<4>);
  case 2: return reinterpret_cast<const void *>(&panelQkvPairTc<2>);
  default: return reinterpret_cast<const void *>(&panelQkvPairTc<1>);
  }
}

bool panelGeometry(const GemmSpec &s, library::Geometry *g, bool pairsAllowed = true) {
  if (s.M <= 0 || s.K <= 0 || s.N <= 0 || s.layers <= 0 || s.layer < 0 || s.layer >= s.layers)
    return false;
  if (const int width = pairsAllowed ? linearPairWidth(s) : 0) {
    pairGeometry(s, width, g, pairSplits(s, width), width);
    return g->grid[1] <= 65535;
  }
  const int width = tc::chooseWidth(s), mt = tc::chooseRowTiles(s);
  g->grid[0] = ceilDiv(s.N, width);
  g->grid[1] = ceilDiv(ceilDiv(s.M, tc::BM), mt);
  g->grid[2] = unsigned(tc::chooseSplits(s));
  g->block[0] = tc::kThreads;
  g->sharedBytes = unsigned(tc::sharedBytes(width, mt));
  return g->grid[1] <= 65535;
}

bool panelGemmGeometry(const void *spec, std::size_t, library::Geometry *g) {
  return panelGeometry(specOf<GemmSpec>(spec), g);
}

// The argmax heads (LM head, prefill heads) take the pair kernel's 256-column tiles when
// argmaxPairs holds; their partials hold grid.x entries per row (the pair kernel: two per
// column tile, one of them empty).
bool panelArgmaxGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GemmSpec>(spec);
  if (argmaxPairs(s)) {
    if (s.M <= 0 || s.layers <= 0 || s.layer < 0 || s.layer >= s.layers)
      return false;
    pairGeometry(s, tc::pair::kWide, g);
    return g->grid[1] <= 65535;
  }
  return panelGeometry(s, g, false);
}

bool panelRopeGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GemmSpec>(spec);
  if (s.D <= 0 || s.D % 2 || s.N % s.D || s.T <= 0)
    return false;
  return panelGeometry(s, g);
}

bool panelAppendGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<GemmSpec>(spec);
  if (s.D <= 0 || s.D % 2 || s.N != s.A * s.D || s.T <= 0)
    return false;
  return panelGeometry(s, g);
}

#define CKL_PANEL_PAIR_SELECT(fn, pairFn)                                                      \
  [](const void *spec) -> const void * {                                                       \
    const GemmSpec &s = specOf<GemmSpec>(spec);                                                \
    if (const int width = linearPairWidth(s)) {                                                \
      const int splits = pairSplits(s, width);                                                 \
      if (width == tc::pair::kWide)                                                            \
        return splits == 8   ? reinterpret_cast<const void *>(&pairFn<8, tc::pair::kWide>)     \
               : splits == 4 ? reinterpret_cast<const void *>(&pairFn<4, tc::pair::kWide>)     \
               : splits == 2 ? reinterpret_cast<const void *>(&pairFn<2, tc::pair::kWide>)     \
                             : reinterpret_cast<const void *>(&pairFn<1, tc::pair::kWide>);    \
      return splits == 4   ? reinterpret_cast<const void *>(&pairFn<4, tc::pair::kNarrow>)     \
             : splits == 2 ? reinterpret_cast<const void *>(&pairFn<2, tc::pair::kNarrow>)     \
                           : reinterpret_cast<const void *>(&pairFn<1, tc::pair::kNarrow>);    \
    }                                                                                          \
    return CKL_PANEL_SELECT(fn)(spec);                                                         \
  }

#define CKL_PANEL_SELECT(fn)                                                                   \
  [](const void *spec) -> const void * {                                                       \
    const GemmSpec &s = specOf<GemmSpec>(spec);                                                \
    switch (tc::chooseWidth(s)) {                                                              \
    case 128:                                                                                  \
      if (tc::chooseRowTiles(s) == 2)                                                          \
        switch (tc::chooseSplits(s)) {                                                         \
        case 8: return reinterpret_cast<const void *>(&fn<128, 8, 2>);                         \
        case 4: return reinterpret_cast<const void *>(&fn<128, 4, 2>);                         \
        case 2: return reinterpret_cast<const void *>(&fn<128, 2, 2>);                         \
        default: return reinterpret_cast<const void *>(&fn<128, 1, 2>);                        \
        }                                                                                      \
      switch (tc::chooseSplits(s)) {                                                           \
      case 8: return reinterpret_cast<const void *>(&fn<128, 8, 1>);                           \
      case 4: return reinterpret_cast<const void *>(&fn<128, 4, 1>);                           \
      case 2: return reinterpret_cast<const void *>(&fn<128, 2, 1>);                           \
      default: return reinterpret_cast<const void *>(&fn<128, 1, 1>);                          \
      }                                                                                        \
    case 64: return reinterpret_cast<const void *>(&fn<64, 1, 1>);                             \
    default: return reinterpret_cast<const void *>(&fn<32, 1, 1>);                             \
    }                                                                                          \
  }

const void *linearArgmaxSelect(const void *spec) {
  if (argmaxPairs(specOf<GemmSpec>(spec)))
    return reinterpret_cast<const void *>(&panelLinearArgmaxPairTc);
  return CKL_PANEL_SELECT(panelLinearArgmaxTc)(spec);
}

const void *argmaxSelect(const void *spec) {
  if (argmaxPairs(specOf<GemmSpec>(spec)))
    return reinterpret_cast<const void *>(&panelArgmaxPairTc);
  return CKL_PANEL_SELECT(panelArgmaxTc)(spec);
}

} // namespace

CKL_REGISTER_KERNEL("ckl.fused.rms_panel", reinterpret_cast<const void *>(&rmsPanelKernel),
                    "PPPFS", sizeof(RmsApplySpec), rmsPanelGeometry, nullptr,
                    nullptr, 0, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_gate_up", reinterpret_cast<const void *>(&panelGateUpTc<1>),
                    "PPPPS", sizeof(GemmSpec), gateUpGeometry, gateUpSelect, prepareGateUp,
                    sizeof(tc::WeightMapPair), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_qkv", reinterpret_cast<const void *>(&panelQkvPairTc<1>),
                    "PPPPPPPPPS", sizeof(GemmSpec), qkvGeometry, qkvSelect, prepareQkv,
                    sizeof(tc::WeightMapTriple), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_linear", reinterpret_cast<const void *>(&panelLinearTc<32, 1, 1>),
                    "PPPS", sizeof(GemmSpec), panelGemmGeometry, CKL_PANEL_PAIR_SELECT(panelLinearTc, panelLinearPairTc),
                    prepareWeights, sizeof(tc::WeightMap), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_linear_rope", reinterpret_cast<const void *>(&panelLinearRopeTc<32, 1, 1>),
                    "PPPPPS", sizeof(GemmSpec), panelRopeGeometry, CKL_PANEL_PAIR_SELECT(panelLinearRopeTc, panelLinearRopePairTc),
                    prepareWeights, sizeof(tc::WeightMap), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_linear_rope_append", reinterpret_cast<const void *>(&panelLinearRopeAppendTc<32, 1, 1>),
                    "PPPPPS", sizeof(GemmSpec), panelAppendGeometry, CKL_PANEL_PAIR_SELECT(panelLinearRopeAppendTc, panelLinearRopeAppendPairTc),
                    prepareWeights, sizeof(tc::WeightMap), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_linear_append", reinterpret_cast<const void *>(&panelLinearAppendTc<32, 1, 1>),
                    "PPPPS", sizeof(GemmSpec), panelAppendGeometry, CKL_PANEL_PAIR_SELECT(panelLinearAppendTc, panelLinearAppendPairTc),
                    prepareWeights, sizeof(tc::WeightMap), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_linear_residual", reinterpret_cast<const void *>(&panelLinearResidualTc<32, 1, 1>),
                    "PPPPS", sizeof(GemmSpec), panelGemmGeometry, CKL_PANEL_PAIR_SELECT(panelLinearResidualTc, panelLinearResidualPairTc),
                    prepareWeights, sizeof(tc::WeightMap), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_linear_argmax", reinterpret_cast<const void *>(&panelLinearArgmaxTc<32, 1, 1>),
                    "PPPPS", sizeof(GemmSpec), panelArgmaxGeometry, linearArgmaxSelect,
                    prepareArgmaxWeights, sizeof(tc::WeightMap), true, true);
CKL_REGISTER_KERNEL("ckl.fused.panel_argmax", reinterpret_cast<const void *>(&panelArgmaxTc<32, 1, 1>),
                    "PPPS", sizeof(GemmSpec), panelArgmaxGeometry, argmaxSelect,
                    prepareArgmaxWeights, sizeof(tc::WeightMap), true, true);

} // namespace ckl::kernels

// Fault word of the tensor-core kernels: bit 0 a bounded wait expired, bit 1 a panel operand or
// the shared-memory ring was misaligned.  `reset` clears it after reading.
extern "C" int ckl_library_faults(uint32_t *out, int reset) {
  unsigned value = 0;
  cudaError_t status = cudaMemcpyFromSymbol(&value, ckl::kernels::tc::g_libraryFaults, sizeof(value));
  if (status == cudaSuccess && reset) {
    const unsigned zero = 0;
    status = cudaMemcpyToSymbol(ckl::kernels::tc::g_libraryFaults, &zero, sizeof(zero));
  }
  if (status != cudaSuccess) {
    cudaGetLastError();
    return CKL_RUNTIME_ERROR;
  }
  if (out)
    *out = value;
  return CKL_OK;
}

namespace {
int setSymbolOnDevice(int device, const void *symbol, const void *value, std::size_t bytes) {
  int previous = 0;
  cudaError_t status = cudaGetDevice(&previous);
  if (status == cudaSuccess)
    status = cudaSetDevice(device);
  if (status == cudaSuccess)
    status = cudaMemcpyToSymbol(symbol, value, bytes);
  const cudaError_t restored = cudaSetDevice(previous);
  if (status == cudaSuccess)
    status = restored;
  if (status != cudaSuccess) {
    cudaGetLastError();
    return CKL_RUNTIME_ERROR;
  }
  return CKL_OK;
}
} // namespace

// Limit of the tensor-core kernels' pipeline waits on `device` for launches made after the
// call (the default is 2 s); the waits that drain a CTA's own copies keep their fixed limit.
extern "C" int ckl_set_wait_limit(int device, uint64_t nanoseconds) {
  const unsigned long long value = nanoseconds;
  return setSymbolOnDevice(device, &ckl::kernels::tc::g_waitLimitNs, &value, sizeof(value));
}

// Test hook: while enabled, every tensor-core kernel CTA launched on `device` first waits on an
// mbarrier that nothing signals; the wait expires after the wait limit, records fault bit 0 and
// takes the abort path (no work done, tensor memory freed, no copy left in flight).
extern "C" int ckl_inject_unsignalled_wait(int device, int enable) {
  const int value = enable ? 1 : 0;
  return setSymbolOnDevice(device, &ckl::kernels::tc::g_injectUnsignalledWait, &value,
                           sizeof(value));
}
