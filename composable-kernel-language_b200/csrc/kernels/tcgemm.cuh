// Tensor-core (tcgen05) projection kernel with FP32-level accuracy (3xTF32).
//
// out = epilogue(A @ W[layer]) for batched decode (17 or more requests), A given as a split
// panel (panel.cuh: TF32 hi/lo parts in the tensor cores' shared-memory layout, produced
// once by the kernel that computes A), W the FP32 weights [K, N] of one layer, read as stored.
// hi*hi accumulates in one FP32 tensor-memory accumulator and the correction products
// hi*lo + lo*hi in a second one, summed in FP32 by the epilogue (the dropped lo*lo term is
// ~2^-22 relative).  This keeps the decoder's 1e-4 relative tolerance and greedy-token parity
// that plain TF32 breaks.
//
// CTA: one 128 x BN output tile, K in slices of 32, ten warps with fixed roles:
//   warp 0 (producer): per slice one 32 KB bulk copy of the panel block (hi + lo) and one TMA
//     tensor copy of the 32 x BN weight box (zero-filled beyond K and N; the tensor map is
//     built at bind time and passed as a __grid_constant__ parameter) into a ring of S
//     stages, completing on the stage's `full` mbarrier; a stage is refilled after the MMAs
//     that read it completed;
//   warp 1 (MMA): allocates 2*BN tensor-memory columns; per slice, once the panel block has
//     landed and the weight slice is converted, one thread issues up to 4 k-steps x 3
//     `tcgen05.mma.cta_group::1.kind::tf32` (M=128, N=BN, K=8) and commits them to the
//     stage's `empty` and the weight buffer's `bEmpty` mbarriers;
//   warps 2-9 (converters, then epilogue): split each landed weight slice into TF32 hi/lo in
//     K-major no-swizzle layout (two buffers), then read the accumulators with
//     `tcgen05.ld.32x32b` (warp w reads TMEM lanes 32 (w % 4).., one output row per thread,
//     half of the columns each) and apply the fused epilogue.
// A tf32 MMA costs about the same at N = 32 as at N = 128, so tiles are 128 columns wide
// (narrower only for narrow outputs) and the K loop is split over gridDim.z CTAs when the
// output has too few tiles to fill the GPU.  The splits of a tile form a thread-block
// cluster: each stages its summed accumulators in shared memory, and after a cluster barrier
// each reduces a slice of the tile's rows by reading its peers' staging through distributed
// shared memory in rank order (deterministic), then applies the fused epilogue.
// Weights whose rows or pointer do not allow a tensor map (N % 4 != 0, unaligned base) are read
// by the converters straight from global memory instead.
//
// Every mbarrier wait is bounded by time.  A wait that expires records a fault bit
// (ckl_library_faults) and raises a CTA-wide abort flag that ends the other roles' waits; the
// CTA then waits (again bounded) for its in-flight copies and MMAs, frees its tensor memory
// and returns.  No wait spins without a limit.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gemm.cuh"
#include "panel.cuh"

namespace ckl::kernels::tc {

constexpr int BM = panel::kRows;
constexpr int BK = panel::kSlice;
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kConverterWarps = 8; // warps 2..9; also the epilogue (two warps per TMEM lane quarter)
constexpr int kConverterThreads = kConverterWarps * kWarp;
constexpr int kThreads = (2 + kConverterWarps) * kWarp;
// Default limit of a pipeline wait; ckl_set_wait_limit changes it per device (tests).
constexpr unsigned long long kWaitLimitNs = 2000000000ull; // 2 s
// Limit of the waits that drain a CTA's own copies and MMAs before it frees its tensor memory
// and exits; fixed, so that no setting can let a CTA leave with an operation in flight.
constexpr unsigned long long kDrainLimitNs = 2000000000ull; // 2 s
constexpr std::size_t kMaxDynamicSmem = 227 * 1024;

// TMA tensor map of a weight buffer [layers, K, N] with a box of BN x 32 x 1 (N innermost),
// or valid == 0 when the buffer does not admit one.
struct WeightMap {
  CUtensorMap map;
  int valid;
};

// Gate and up weights of the fused gate/up/SwiGLU projection, each with a box of BN/2 columns.
struct WeightMapPair {
  WeightMap gate, up;
};

// q, k and v weights of the fused q/k/v projection.
struct WeightMapTriple {
  WeightMap q, k, v;
};

// Output columns of one tile: the gate/up tile holds BN/2 gate and BN/2 up columns of the same
// BN/2 outputs.
template <int BN, int EPI> constexpr int tileColumns() {
  return EPI == gemm::kSwiGluPanel ? BN / 2 : BN;
}

// silu(g) * u for the tensor-core gate/up epilogues.  The quotient uses the fast division
// (at most 2 ulp from the IEEE-rounded one), which has no slow path: the IEEE division's slow
// path (taken for instance for a zero dividend) made the pair gate/up epilogue 2.5x longer
// (27.0 k against 10.7 k cycles per CTA in a development trace with zero activations).  The
// value then goes into a TF32 hi/lo split whose products carry ~2^-21 relative error anyway.
__device__ __forceinline__ float swigluValue(float g, float u) {
  return __fmul_rn(__fdividef(g, 1.0f + expf(-g)), u);
}

// Fault word of the library (bit 0: a tensor-core wait expired).  One translation unit
// instantiates these kernels and reports the word (ckl_library_faults).
static __device__ unsigned g_libraryFaults = 0;
// Limit of the pipeline waits (those that an abort can end) on this device, in nanoseconds.
static __device__ unsigned long long g_waitLimitNs = kWaitLimitNs;
// Nonzero: the MMA warp first waits on an mbarrier that nothing signals, so its bounded wait
// expires and the CTA takes the abort path (ckl_inject_unsignalled_wait; tests only).
static __device__ int g_injectUnsignalledWait = 0;

__device__ __forceinline__ unsigned smemAddress(const void *p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long matrixDescriptor(const void *start, unsigned lbo,
                                                               unsigned sbo) {
  const unsigned address = smemAddress(start);
  unsigned long long d = 0;
  d |= static_cast<unsigned long long>((address >> 4) & 0x3FFFu);
  d |= static_cast<unsigned long long>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<unsigned long long>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46; // descriptor version for sm_100; base offset 0, no swizzle
  return d;
}

// kind::tf32 instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = BN.
template <int BN> __host__ __device__ constexpr unsigned instructionDescriptor() {
  return (1u << 4) | (2u << 7) | (2u << 10) | (unsigned(BN >> 3) << 17) | (unsigned(BM >> 4) << 24);
}

__device__ __forceinline__ void mbarrierInit(unsigned long long *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemAddress(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbarrierArrive(unsigned long long *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smemAddress(bar))
               : "memory");
}

__device__ __forceinline__ void mbarrierArriveExpectTx(unsigned long long *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               ::"r"(smemAddress(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbarrierTryWait(unsigned long long *bar, unsigned phase) {
  unsigned done;
  asm volatile("{\n\t.reg .pred P;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
               "selp.b32 %0, 1, 0, P;\n\t}"
               : "=r"(done)
               : "r"(smemAddress(bar)), "r"(phase)
               : "memory");
  return done != 0;
}

__device__ __forceinline__ unsigned long long globalTimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for an mbarrier phase.  Gives up when `abort` is raised by another thread, or
// raises it (and the fault bit) when the time limit expires.  Pipeline waits (with an abort
// flag) use the device's settable limit, drain waits (abort == nullptr) the fixed one.
__device__ __forceinline__ bool waitPhase(unsigned long long *bar, unsigned phase,
                                          volatile int *abort) {
  if (mbarrierTryWait(bar, phase))
    return true;
  const unsigned long long start = globalTimer();
  const unsigned long long limit = abort != nullptr ? g_waitLimitNs : kDrainLimitNs;
  while (true) {
    if (mbarrierTryWait(bar, phase))
      return true;
    if (abort != nullptr && *abort)
      return false;
    if (globalTimer() - start > limit) {
      atomicOr(&g_libraryFaults, 1u);
      if (abort != nullptr)
        *abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void bulkCopy(void *dst, const void *src, unsigned bytes,
                                         unsigned long long *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
               "[%0], [%1], %2, [%3];" ::"r"(smemAddress(dst)),
               "l"(src), "r"(bytes), "r"(smemAddress(bar))
               : "memory");
}

// TMA copy of the weight box at (n0, k0, layer) into shared memory.
__device__ __forceinline__ void tensorCopy(void *dst, const CUtensorMap *map, int n0, int k0,
                                           int layer, unsigned long long *bar) {
  asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
               "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smemAddress(dst)),
               "l"(reinterpret_cast<unsigned long long>(map)), "r"(n0), "r"(k0), "r"(layer),
               "r"(smemAddress(bar))
               : "memory");
}

__device__ __forceinline__ void fenceAsyncShared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mma(unsigned tmem, unsigned long long a, unsigned long long b,
                                    unsigned idesc, unsigned accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\t"
               "setp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
               ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
               : "memory");
}

__device__ __forceinline__ void commit(unsigned long long *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smemAddress(bar))
               : "memory");
}

template <int N> __device__ __forceinline__ void tmemAlloc(unsigned *slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smemAddress(slot)), "r"(N)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

template <int N> __device__ __forceinline__ void tmemFree(unsigned base) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(N)
               : "memory");
}

__device__ __forceinline__ void fenceBeforeSync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fenceAfterSync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 16 consecutive accumulator columns of this thread's row.
__device__ __forceinline__ void tmemLoad16(unsigned address, float (&v)[16]) {
  unsigned r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
               "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                 "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(address));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i)
    v[i] = __uint_as_float(r[i]);
}

// Column width of the tile for a specialization.
inline int chooseWidth(const GemmSpec &s) { return s.N <= 32 ? 32 : (s.N <= 64 ? 64 : 128); }

constexpr int64_t kTargetCtas = 148; // one CTA per SM

// K splits (1, 2, 4 or 8; the CTAs of one tile form a cluster): about one wave of CTAs over
// the SMs, at least two slices per split, full-width tiles only.  A split whose slice range
// is empty contributes zeros.
// Row tiles per CTA: when single-tile CTAs would already fill the SMs, full-width tiles go two
// per CTA and share every converted weight slice (half the weight conversion and copy traffic
// per row tile; a wide projection's tiles fit in fewer waves).  Narrower grids keep one row
// tile per CTA and split K instead.
inline int chooseRowTiles(const GemmSpec &s) {
  if (chooseWidth(s) != 128 || s.M <= BM)
    return 1;
  const int64_t tiles = ((s.M + BM - 1) / BM) * ((s.N + 127) / 128);
  return tiles >= kTargetCtas ? 2 : 1;
}

inline int chooseSplits(const GemmSpec &s) {
  const int width = chooseWidth(s);
  if (width != 128)
    return 1;
  const int64_t rowGroups = ((s.M + BM - 1) / BM + chooseRowTiles(s) - 1) / chooseRowTiles(s);
  const int64_t tiles = rowGroups * ((s.N + width - 1) / width);
  const int64_t slices = panel::slices(s.K);
  int64_t wanted = kTargetCtas / (tiles > 0 ? tiles : 1);
  if (wanted > slices / 2)
    wanted = slices / 2;
  int splits = 1;
  while (splits * 2 <= wanted && splits < 8)
    splits *= 2;
  return splits;
}

template <int BN, int S, int MT = 1> struct Smem {
  float a[S][MT][2][BK / 4][BM][4]; // panel blocks (MT row tiles x hi, lo) as copied
  float bHi[2][BK / 4][BN][4];  // converted weight slices, K-major
  float bLo[2][BK / 4][BN][4];
  float rawB[S][BK][BN];        // weight box as copied (128-byte aligned)
  unsigned long long full[S], empty[S], bFull[2], bEmpty[2], accDone;
  unsigned long long unsignalled; // never arrived on (injected expiring wait)
  unsigned tmemBase;
  int abort;
};

// Deepest ring (at most 6 stages) that fits the shared-memory budget.
template <int BN, int MT = 1, int S = 6> constexpr int stages() {
  if constexpr (S <= 2 || sizeof(Smem<BN, S, MT>) <= kMaxDynamicSmem)
    return S;
  else
    return stages<BN, MT, S - 1>();
}
static_assert(sizeof(Smem<128, stages<128>()>) <= kMaxDynamicSmem, "shared memory budget");
static_assert(sizeof(Smem<128, stages<128, 2>(), 2>) <= kMaxDynamicSmem, "shared memory budget");

// Dynamic shared memory of the kernel at a column width and row tiles per CTA.
inline std::size_t sharedBytes(int width, int rowTiles = 1) {
  switch (width) {
  case 128:
    return rowTiles == 2 ? sizeof(Smem<128, stages<128, 2>(), 2>)
                         : sizeof(Smem<128, stages<128>()>);
  case 64: return sizeof(Smem<64, stages<64>()>);
  default: return sizeof(Smem<32, stages<32>()>);
  }
}

// Fused epilogue of four consecutive output values v of row m starting at column n (a multiple
// of 4); columns at or beyond N are skipped.
template <int EPI>
__device__ __forceinline__ void storeQuad(const gemm::Params &p, int64_t m, int64_t n, float4 v,
                                          int position, bool vec4, float &best, int &bestIndex) {
  const GemmSpec &s = p.s;
  const int64_t M = s.M, N = s.N;
  float *lanes = &v.x;
  if constexpr (EPI == gemm::kStore || EPI == gemm::kResidual || EPI == gemm::kArgmax) {
    if constexpr (EPI == gemm::kArgmax) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n + j < N)
          argmaxMerge(best, bestIndex, lanes[j], int(n + j));
    }
    if (EPI == gemm::kArgmax && p.out == nullptr)
      return; // argmax partials only (batched prefill heads)
    if (vec4 && n + 4 <= N) {
      if constexpr (EPI == gemm::kResidual) {
        const float4 r = *reinterpret_cast<const float4 *>(p.residual + m * N + n);
        v = make_float4(__fadd_rn(r.x, v.x), __fadd_rn(r.y, v.y), __fadd_rn(r.z, v.z),
                        __fadd_rn(r.w, v.w));
      }
      *reinterpret_cast<float4 *>(p.out + m * N + n) = v;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (n + j >= N)
          continue;
        float value = lanes[j];
        if constexpr (EPI == gemm::kResidual)
          value = __fadd_rn(p.residual[m * N + n + j], value);
        p.out[m * N + n + j] = value;
      }
    }
  } else {
    // Row m is request m % cache at position position[0] + m / cache (decode: M == cache, so
    // every row is at position[0]; batched prefill: several positions per launch).
    // Row, column and head indices fit in 32 bits: their divisions by the runtime row count and
    // head dimension use 32-bit unsigned arithmetic (64-bit division is a long software
    // sequence, and this runs for every output quad); only the cache offset is 64-bit.
    const int64_t D = s.D, R = s.D / 2;
    const unsigned rows = unsigned(s.cache > 0 ? s.cache : M);
    const unsigned wave = unsigned(m) / rows;
    const int64_t request = int64_t(unsigned(m) - wave * rows), at = position + int64_t(wave);
    if (at >= s.T)
      return;
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const int64_t c = n + j;
      if (c >= N)
        continue;
      float first = lanes[j], second = lanes[j + 1];
      const unsigned head = unsigned(c) / unsigned(D);
      const int64_t h = head, d = int64_t(unsigned(c) - head * unsigned(D));
      if constexpr (EPI == gemm::kRope || EPI == gemm::kRopeAppend) {
        const float *cs = p.table + (at * R + d / 2) * 2;
        const float cosine = cs[0], sine = cs[1];
        const float x = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
        const float y = __fadd_rn(__fmul_rn(first, sine), __fmul_rn(second, cosine));
        first = x;
        second = y;
      }
      if constexpr (EPI == gemm::kRope) {
        p.out[m * N + c] = first;
        p.out[m * N + c + 1] = second;
      } else {
        float *slot = p.out + (((s.layer * rows + request) * s.A + h) * s.T + at) * D + d;
        slot[0] = first;
        slot[1] = second;
      }
    }
  }
}

// Named barrier over the epilogue warps that also ANDs a predicate across them.
__device__ __forceinline__ bool epilogueAll(bool value) {
  unsigned out;
  asm volatile("{\n\t.reg .pred p, q;\n\t"
               "setp.ne.u32 p, %1, 0;\n\t"
               "barrier.cta.red.and.pred q, 1, %2, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}"
               : "=r"(out)
               : "r"(unsigned(value)), "n"(kConverterThreads)
               : "memory");
  return out != 0;
}

// Barrier over every thread of every CTA of the cluster (the K splits of one tile).
__device__ __forceinline__ void clusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Four floats at the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ float4 loadCluster(const float *local, unsigned rank) {
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smemAddress(local)), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// Accumulators staged in shared memory, one padded row per output row (conflict-free row-wise
// writes and column-wise reads); aliases the idle panel ring after the main loop.
template <int BN> using Staging = float[BM][BN + 4];

// Output rows [rank * 128 / SPLITS, (rank + 1) * 128 / SPLITS) of the tile: each epilogue warp
// takes a row at a time, each lane four consecutive columns, summing the K splits' staged
// partials in rank order (deterministic), and stores them through the fused epilogue (the
// gate/up tile, whose output is a panel, and the unsplit argmax scan go one row per lane).
template <int BN, int EPI, int SPLITS>
__device__ __forceinline__ void reduceAndStore(const gemm::Params &p, Staging<BN> &stage,
                                               int64_t m0, int64_t nt, int position) {
  const GemmSpec &s = p.s;
  const int64_t M = s.M, N = s.N, n0 = nt * tileColumns<BN, EPI>();
  const int warp = threadIdx.x / kWarp - 2, lane = threadIdx.x % kWarp;
  const unsigned rank = blockIdx.z;
  constexpr int kRows = BM / SPLITS;
  if constexpr (EPI == gemm::kSwiGluPanel) {
    // One row per lane: the gate and up values of an output quad sit in the same staged row
    // (columns c and c + 64), and a warp's panel store of one quad then covers 32 consecutive
    // rows (512 contiguous bytes of the K-major panel) instead of 16 scattered quads of a row.
    // Warps split the tile into four groups of 32 rows x two halves of the 16 output quads.
    static_assert(SPLITS == 1 && BN == 4 * kWarp, "gate/up tiles");
    const int row = (warp % 4) * kWarp + lane;
    const int64_t m = m0 + row, padded = panel::slices(N) * panel::kSlice;
    if (m >= M)
      return;
    for (int q = (warp / 4) * (BN / 16); q < (warp / 4 + 1) * (BN / 16); ++q) {
      const int64_t k = n0 + 4 * q; // output column (the panel's K)
      if (k >= padded)
        break;
      const float4 gate = *reinterpret_cast<const float4 *>(&stage[row][4 * q]);
      const float4 up = *reinterpret_cast<const float4 *>(&stage[row][BN / 2 + 4 * q]);
      const float *g = &gate.x, *u = &up.x;
      float4 v;
      float *out = &v.x;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        out[j] = k + j < N ? swigluValue(g[j], u[j]) : 0.f;
      panel::store4(p.out, m, k, N, v);
    }
    return;
  }
  const bool vec4 = N % 4 == 0 && aligned16(p.out) &&
                    (EPI != gemm::kResidual || aligned16(p.residual));
  if constexpr (EPI == gemm::kArgmax && SPLITS == 1) {
    // Logits row by row (coalesced stores), then the argmax partial of each row scanned by one
    // lane over the staged row in column order: the same (largest value, smallest index) as a
    // shuffle reduction, without five dependent shuffle rounds per row.
    if (p.out != nullptr) {
      const int c = 4 * lane;
      for (int r = warp; r < BM && m0 + r < M; r += kConverterWarps) {
        if (c >= BN || n0 + c >= N)
          continue;
        const int64_t m = m0 + r;
        const float4 v = *reinterpret_cast<const float4 *>(&stage[r][c]);
        if (vec4 && n0 + c + 4 <= N) {
          *reinterpret_cast<float4 *>(p.out + m * N + n0 + c) = v;
        } else {
          const float *lanes = &v.x;
          for (int j = 0; j < 4 && n0 + c + j < N; ++j)
            p.out[m * N + n0 + c + j] = lanes[j];
        }
      }
    }
    const int row = warp * kWarp + lane;
    if (row < BM && m0 + row < M) {
      float best = -CUDART_INF_F;
      int bestIndex = 0x7fffffff;
      for (int c = 0; c < BN && n0 + c < N; c += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(&stage[row][c]);
        const float *lanes = &v.x;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n0 + c + j < N)
            argmaxMerge(best, bestIndex, lanes[j], int(n0 + c + j));
      }
      p.partials[(m0 + row) * s.tiles + nt] = make_float2(best, __int_as_float(bestIndex));
    }
    return;
  }
  if constexpr ((EPI == gemm::kResidual || EPI == gemm::kStore) && BN == 4 * kWarp &&
                kRows % kConverterWarps == 0) {
    if (vec4) {
      // One quad per lane; a warp's rows in batches of up to four, every load of a batch (the
      // splits' staged partials through distributed shared memory, the residual from global
      // memory) issued before any is used: one round trip per batch instead of per row (the
      // per-row loop spent ~4,300 of a ~24,000-cycle o-projection CTA here).  The sums and the
      // residual add are the per-row loop's, in the same order.
      constexpr int kPerWarp = kRows / kConverterWarps;
      constexpr int kBatch = kPerWarp < 4 ? kPerWarp : 4;
      const int c = 4 * lane;
      for (int b0 = 0; b0 < kPerWarp; b0 += kBatch) {
        float4 part[kBatch][SPLITS], res[kBatch];
        bool use[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          const int row = int(rank) * kRows + warp + (b0 + i) * kConverterWarps;
          const int64_t m = m0 + row;
          use[i] = m < M && n0 + c < N;
          if constexpr (SPLITS == 1) {
            part[i][0] = *reinterpret_cast<const float4 *>(&stage[row][c]);
          } else {
#pragma unroll
            for (unsigned q = 0; q < SPLITS; ++q)
              part[i][q] = loadCluster(&stage[row][c], q);
          }
          if constexpr (EPI == gemm::kResidual)
            if (use[i])
              res[i] = *reinterpret_cast<const float4 *>(p.residual + m * N + n0 + c);
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          if (!use[i])
            continue;
          const int64_t m = m0 + int(rank) * kRows + warp + (b0 + i) * kConverterWarps;
          float4 v = part[i][0];
#pragma unroll
          for (int q = 1; q < SPLITS; ++q)
            v = make_float4(__fadd_rn(v.x, part[i][q].x), __fadd_rn(v.y, part[i][q].y),
                            __fadd_rn(v.z, part[i][q].z), __fadd_rn(v.w, part[i][q].w));
          if constexpr (EPI == gemm::kResidual)
            v = make_float4(__fadd_rn(res[i].x, v.x), __fadd_rn(res[i].y, v.y),
                            __fadd_rn(res[i].z, v.z), __fadd_rn(res[i].w, v.w));
          *reinterpret_cast<float4 *>(p.out + m * N + n0 + c) = v;
        }
      }
      return;
    }
  }
  for (int r = warp; r < kRows; r += kConverterWarps) {
    const int row = int(rank) * kRows + r;
    const int64_t m = m0 + row;
    if (m >= M)
      break; // rows increase with r
    float best = -CUDART_INF_F;
    int bestIndex = 0x7fffffff;
    for (int c = 4 * lane; c < BN; c += 4 * kWarp) {
      float4 sum;
      if constexpr (SPLITS == 1) {
        sum = *reinterpret_cast<const float4 *>(&stage[row][c]);
      } else {
        sum = loadCluster(&stage[row][c], 0);
#pragma unroll
        for (unsigned q = 1; q < SPLITS; ++q) {
          const float4 part = loadCluster(&stage[row][c], q);
          sum = make_float4(__fadd_rn(sum.x, part.x), __fadd_rn(sum.y, part.y),
                            __fadd_rn(sum.z, part.z), __fadd_rn(sum.w, part.w));
        }
      }
      if constexpr (EPI != gemm::kSwiGluPanel) // handled above
        if (n0 + c < N)
          storeQuad<EPI>(p, m, n0 + c, sum, position, vec4, best, bestIndex);
    }
    if constexpr (EPI == gemm::kArgmax && SPLITS > 1) {
#pragma unroll
      for (int o = kWarp / 2; o > 0; o >>= 1) {
        const float otherBest = __shfl_xor_sync(0xffffffffu, best, o);
        const int otherIndex = __shfl_xor_sync(0xffffffffu, bestIndex, o);
        argmaxMerge(best, bestIndex, otherBest, otherIndex);
      }
      if (lane == 0)
        p.partials[m * s.tiles + nt] = make_float2(best, __int_as_float(bestIndex));
    }
  }
}

// MT x 128 rows by BN columns (MT row tiles sharing every converted weight slice).  p.a is the
// panel of A [M, K]; p.w the weights [layers, K, N].
template <int BN, int EPI, int SPLITS, int MT = 1>
__device__ void body(const gemm::Params &p, const WeightMap &weights,
                     const WeightMap *upWeights = nullptr) {
  static_assert(EPI != gemm::kSwiGluPanel || (SPLITS == 1 && BN == 128), "gate/up tiles");
  static_assert(SPLITS == 1 || BN == 128, "K splits use full-width tiles");
  static_assert(MT == 1 || BN == 128, "two row tiles use full-width tiles");
  constexpr int S = stages<BN, MT>();
  using Layout = Smem<BN, S, MT>;
  static_assert(sizeof(Staging<BN>) <= sizeof(Layout::a), "staging fits the ring");
  extern __shared__ __align__(1024) unsigned char raw[];
  Layout &sm = *reinterpret_cast<Layout *>(raw);
  const GemmSpec &s = p.s;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t K = s.K, N = s.N;
  // Tiles in launch order with the row group varying fastest: the CTAs that share a weight
  // tile run together and read it from HBM once.
  const int64_t rowGroups = gridDim.y;
  const int64_t tile = int64_t(blockIdx.y) * gridDim.x + blockIdx.x;
  const int64_t group = tile % rowGroups, nt = tile / rowGroups;
  const int64_t rowTiles = (s.M + BM - 1) / BM;
  const int tiles = int(rowTiles - group * MT < MT ? rowTiles - group * MT : MT); // >= 1
  const int64_t n0 = nt * tileColumns<BN, EPI>();
  // This split's K slices [kBegin, kEnd).
  const int64_t allSlices = panel::slices(K);
  const int64_t perSplit = (allSlices + SPLITS - 1) / SPLITS;
  const int64_t kBegin = perSplit * blockIdx.z;
  const int64_t kEnd = kBegin + perSplit < allSlices ? kBegin + perSplit : allSlices;
  const int64_t slices = kEnd > kBegin ? kEnd - kBegin : 0;
  const bool hasWork = slices > 0;
  const float *W = p.w + s.layer * K * N;

  int position = 0;
  if constexpr (EPI == gemm::kRope || EPI == gemm::kRopeAppend || EPI == gemm::kAppend) {
    position = p.position[0];
    if (position < 0 || position >= s.T)
      return; // outside cache capacity: the step writes nothing
  }
  if (!aligned16(p.a) || smemAddress(raw) % 128 != 0) {
    if (threadIdx.x == 0)
      atomicOr(&g_libraryFaults, 2u); // panels and the shared ring are aligned by construction
    return;
  }
  // Weight boxes by TMA when the buffer admits a tensor map.
  const bool copyRows =
      weights.valid != 0 && (EPI != gemm::kSwiGluPanel || upWeights->valid != 0);
  const float *W2 = EPI == gemm::kSwiGluPanel ? p.w2 + s.layer * K * N : nullptr;

  if (warp == kMmaWarp)
    tmemAlloc<2 * BN * MT>(&sm.tmemBase);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbarrierInit(&sm.full[i], 1);
      mbarrierInit(&sm.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbarrierInit(&sm.bFull[i], kConverterWarps);
      mbarrierInit(&sm.bEmpty[i], 1);
    }
    mbarrierInit(&sm.accDone, 1);
    mbarrierInit(&sm.unsignalled, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fenceBeforeSync();
  __syncthreads();
  fenceAfterSync();
  const unsigned tmem = sm.tmemBase;
  volatile int *abort = &sm.abort;
  bool valid = false; // converter warps: every issued MMA completed, nothing aborted

  if (warp == kProducerWarp) {
    const unsigned boxBytes = copyRows ? unsigned(BK * BN * 4) : 0u; // full box, OOB zero-filled
    const unsigned blockBytes = unsigned(2 * panel::kPart * 4);
    int64_t issued = 0;
    if (lane == 0 && copyRows) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&weights.map))
                   : "memory");
      if constexpr (EPI == gemm::kSwiGluPanel)
        asm volatile("prefetch.tensormap [%0];"
                     ::"l"(reinterpret_cast<unsigned long long>(&upWeights->map))
                     : "memory");
    }
    for (int64_t kt = 0; kt < slices; ++kt) {
      const int slot = int(kt % S);
      bool ok = true;
      if (lane == 0 && kt >= S)
        ok = waitPhase(&sm.empty[slot], unsigned((kt / S - 1) & 1), abort);
      if (!__shfl_sync(0xffffffffu, ok, 0))
        break;
      if (lane == 0) {
        mbarrierArriveExpectTx(&sm.full[slot], blockBytes * unsigned(tiles) + boxBytes);
        for (int j = 0; j < tiles; ++j)
          bulkCopy(&sm.a[slot][j][0][0][0][0],
                   p.a + ((group * MT + j) * allSlices + kBegin + kt) * panel::kBlock, blockBytes,
                   &sm.full[slot]);
        if (copyRows) {
          const int k0 = int((kBegin + kt) * BK);
          if constexpr (EPI == gemm::kSwiGluPanel) {
            // Gate box, then up box: [2][BK][BN / 2] in the stage.
            tensorCopy(&sm.rawB[slot][0][0], &weights.map, int(n0), k0, int(s.layer),
                       &sm.full[slot]);
            tensorCopy(&sm.rawB[slot][0][0] + BK * (BN / 2), &upWeights->map, int(n0), k0,
                       int(s.layer), &sm.full[slot]);
          } else {
            tensorCopy(&sm.rawB[slot][0][0], &weights.map, int(n0), k0, int(s.layer),
                       &sm.full[slot]);
          }
        }
      }
      issued = kt + 1;
    }
    // Leave no copy in flight: wait (bounded, regardless of abort) for the last use of each
    // stage.  In a completed pipeline these phases are long done.
    if (lane == 0)
      for (int64_t kt = issued > S ? issued - S : 0; kt < issued; ++kt)
        waitPhase(&sm.full[kt % S], unsigned((kt / S) & 1), nullptr);
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr unsigned idesc = instructionDescriptor<BN>();
      // Injected fault: a wait on a barrier nothing signals expires and aborts the CTA.
      const bool injected =
          g_injectUnsignalledWait != 0 && !waitPhase(&sm.unsignalled, 0, abort);
      for (int64_t kt = 0; kt < slices && !injected; ++kt) {
        const int slot = int(kt % S), buffer = int(kt & 1);
        if (!waitPhase(&sm.full[slot], unsigned((kt / S) & 1), abort) ||
            !waitPhase(&sm.bFull[buffer], unsigned((kt / 2) & 1), abort))
          break;
        fenceAfterSync();
        const int64_t remaining = K - (kBegin + kt) * BK;
        const int steps = int(remaining >= BK ? BK / 8 : (remaining + 7) / 8);
        for (int ks = 0; ks < steps; ++ks) {
          const unsigned long long bHi = matrixDescriptor(sm.bHi[buffer][2 * ks], BN * 16, 128);
          const unsigned long long bLo = matrixDescriptor(sm.bLo[buffer][2 * ks], BN * 16, 128);
          const unsigned first = (kt == 0 && ks == 0) ? 0u : 1u;
          for (int j = 0; j < tiles; ++j) {
            const unsigned long long aHi =
                matrixDescriptor(sm.a[slot][j][0][2 * ks], BM * 16, 128);
            const unsigned long long aLo =
                matrixDescriptor(sm.a[slot][j][1][2 * ks], BM * 16, 128);
            const unsigned d = tmem + unsigned(j * 2 * BN);
            mma(d, aHi, bHi, idesc, first);
            mma(d + BN, aHi, bLo, idesc, first);
            mma(d + BN, aLo, bHi, idesc, 1u);
          }
        }
        commit(&sm.empty[slot]);
        commit(&sm.bEmpty[buffer]);
      }
      // Tracks every MMA issued above, on success and on abort alike.
      commit(&sm.accDone);
    }
    __syncwarp();
  } else {
    const int t = threadIdx.x - 2 * kWarp;
    for (int64_t kt = 0; kt < slices; ++kt) {
      const int slot = int(kt % S), buffer = int(kt & 1);
      bool ok = !copyRows || waitPhase(&sm.full[slot], unsigned((kt / S) & 1), abort);
      if (ok && kt >= 2)
        ok = waitPhase(&sm.bEmpty[buffer], unsigned((kt / 2 - 1) & 1), abort);
      if (!__all_sync(0xffffffffu, ok))
        break;
      const int64_t k0 = (kBegin + kt) * BK;
      // Group i: four consecutive k (chunk c) of column n.  Full slices of copied boxes need no
      // bounds checks (the box is zero-filled beyond N).
      if (copyRows && k0 + BK <= K) {
#pragma unroll
        for (int g = 0; g < (BK / 4) * BN / kConverterThreads; ++g) {
          const int i = t + g * kConverterThreads;
          const int c = i / BN, n = i % BN;
          float4 v;
          if constexpr (EPI == gemm::kSwiGluPanel) {
            const float *box = &sm.rawB[slot][0][0] + (n / (BN / 2)) * BK * (BN / 2) + n % (BN / 2);
            v = make_float4(box[(4 * c) * (BN / 2)], box[(4 * c + 1) * (BN / 2)],
                            box[(4 * c + 2) * (BN / 2)], box[(4 * c + 3) * (BN / 2)]);
          } else {
            v = make_float4(sm.rawB[slot][4 * c][n], sm.rawB[slot][4 * c + 1][n],
                            sm.rawB[slot][4 * c + 2][n], sm.rawB[slot][4 * c + 3][n]);
          }
          float4 hi, lo;
          panel::split4(v, hi, lo);
          *reinterpret_cast<float4 *>(sm.bHi[buffer][c][n]) = hi;
          *reinterpret_cast<float4 *>(sm.bLo[buffer][c][n]) = lo;
        }
      } else {
#pragma unroll
      for (int g = 0; g < (BK / 4) * BN / kConverterThreads; ++g) {
        const int i = t + g * kConverterThreads;
        const int c = i / BN, n = i % BN;
        float4 v;
        float *lanes = &v.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t k = k0 + 4 * c + j;
          float value = 0.f;
          if (k < K) {
            if constexpr (EPI == gemm::kSwiGluPanel) {
              const int half = n / (BN / 2), col = n % (BN / 2);
              if (copyRows)
                value = (&sm.rawB[slot][0][0])[(half * BK + 4 * c + j) * (BN / 2) + col];
              else if (n0 + col < N)
                value = (half ? W2 : W)[k * N + n0 + col];
            } else {
              if (copyRows)
                value = sm.rawB[slot][4 * c + j][n];
              else if (n0 + n < N)
                value = W[k * N + n0 + n];
            }
          }
          lanes[j] = value;
        }
        float4 hi, lo;
        panel::split4(v, hi, lo);
        *reinterpret_cast<float4 *>(sm.bHi[buffer][c][n]) = hi;
        *reinterpret_cast<float4 *>(sm.bLo[buffer][c][n]) = lo;
      }
      }
      fenceAsyncShared();
      __syncwarp();
      if (lane == 0)
        mbarrierArrive(&sm.bFull[buffer]);
    }
    // Wait (bounded) for every issued MMA.
    const bool done = waitPhase(&sm.accDone, 0, nullptr);
    fenceAfterSync();
    valid = epilogueAll(done && !*abort) && hasWork; // uniform over these warps
  }
  // Epilogue, one row tile at a time: stage this warp's TMEM lanes (main + correction, one row
  // per thread, half of the columns) in shared memory over the idle ring, then reduce the K
  // splits and store.  Every thread of every split CTA takes part in the same barriers.
  Staging<BN> &stage = *reinterpret_cast<Staging<BN> *>(&sm.a[0][0][0][0][0][0]);
  for (int j = 0; j < MT; ++j) {
    if (warp >= 2) {
      const int row = (warp % 4) * 32 + lane;
      const unsigned rowAddress = tmem + unsigned(j * 2 * BN) + (unsigned((warp % 4) * 32) << 16);
      const int half = (warp - 2) / 4;
      const bool use = valid && j < tiles;
#pragma unroll 1
      for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
        float v[16], correction[16];
        if (use) {
          tmemLoad16(rowAddress + unsigned(c0), v);
          tmemLoad16(rowAddress + unsigned(BN + c0), correction);
        }
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4 *>(&stage[row][c0 + q]) =
              use ? make_float4(__fadd_rn(v[q], correction[q]),
                                __fadd_rn(v[q + 1], correction[q + 1]),
                                __fadd_rn(v[q + 2], correction[q + 2]),
                                __fadd_rn(v[q + 3], correction[q + 3]))
                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if constexpr (SPLITS > 1)
      clusterSync();
    else
      __syncthreads();
    if (warp >= 2 && j < tiles && __all_sync(0xffffffffu, !*abort))
      reduceAndStore<BN, EPI, SPLITS>(p, stage, (group * MT + j) * BM, nt, position);
    fenceBeforeSync();
    if constexpr (SPLITS > 1)
      clusterSync(); // peers read this CTA's staging until here
    else
      __syncthreads();
  }
  if (warp == kMmaWarp)
    tmemFree<2 * BN * MT>(tmem);
}

} // namespace ckl::kernels::tc
