// Tensor-core projections on CTA pairs: 2-SM (cta_group::2) tcgen05 3xTF32 with 256 x 256
// output tiles (256 x 128 in the narrow build), for the wide projections of batched decode and
// prefill: fused gate/up + SwiGLU, the LM head with its argmax partials, fused q/k/v, and the
// batched prefill's o / down projections.
//
// Why pairs.  The single-CTA kernel (tcgemm.cuh) is bound by shared-memory bandwidth: an
// M=128, N=128, K=8 tf32 MMA reads 8 KB of operands for 65 cycles of tensor work, about the
// 128 bytes per cycle that shared memory delivers, before the TMA fills and the weight
// conversion are counted.  A pair of CTAs on two SMs issues M=256, N=256 MMAs: each SM holds
// its own 128 rows of A and half (128 columns) of B, and computes its 128 rows x 256 columns,
// so one MMA costs each SM 4 KB of A + 4 KB of B for twice the work, and each SM converts only
// its half of the weight box.  Per 32-deep slice and 128 x 256 outputs an SM moves ~192 KB
// through shared memory (12 MMAs x 8 KB, 48 KB of copies, 48 KB of conversion) against ~1550
// cycles of tensor work: about balanced, instead of ~2.5x over.
//
// Pair protocol (the pair's two CTAs adjacent along cluster x, the dimension CTA pairs are
// formed on; the even cluster rank is the leader; K splits of a tile, if any, along cluster z):
//   * both CTAs' warp 1 allocate 2 x BN tensor-memory columns with `tcgen05.alloc.cta_group::2`
//     (hi*hi accumulator in columns 0..BN-1, the hi*lo + lo*hi correction in BN..2BN-1: all 512
//     columns for 256-wide tiles);
//   * each CTA's producer (warp 0) copies its own panel block (its 128 rows, hi + lo) and its
//     half of the weight box into its own ring, completing on its own `full` barrier: no copy
//     signals the other CTA;
//   * each CTA's converter warps (2-9) wait for `full`, split the weight half into TF32 hi/lo
//     (K-major), fence their writes for the tensor cores' (async) proxy, meet at a named
//     barrier, and one thread arrives on the LEADER's `ready` barrier (2 arrivals: one per
//     CTA), which certifies both the panel block and the converted weights of that CTA (a
//     cluster-scope release per warp and slice measured as the kernel's top stall);
//   * the leader's MMA thread waits on `ready`, issues per 8-deep
//     k-step three `tcgen05.mma.cta_group::2.kind::tf32` (M=256, N=BN), and commits with
//     `.multicast::cluster` to both CTAs' `empty` (ring stage) and `bEmpty` (conversion
//     buffer) barriers, and finally to both CTAs' `accDone`;
//   * each CTA's epilogue reads its own tensor memory (its 128 rows, all 256 columns);
//   * a cluster barrier precedes `tcgen05.dealloc.cta_group::2` in both CTAs and the exit, so
//     no CTA leaves while its peer may still touch its shared or tensor memory.
// Every mbarrier wait is bounded as in tcgemm.cuh (fault bit, abort flag, drain); every thread
// of both CTAs reaches both cluster barriers on every path (early exits are grid-uniform).
#pragma once

#include "tcgemm.cuh"

namespace ckl::kernels::tc::pair {

constexpr int kWide = 256;   // pair tile width of the wide projections (the MMA's N)
constexpr int kNarrow = 128; // pair tile width of the 1024-wide decode projections
constexpr int S = 3;         // ring stages
constexpr int kReadyArrivals = 2; // one per CTA of the pair
constexpr int kConverterBarrier = 2; // named barrier of the converter warps (0: CTA, 1: epilogue)

// Shared memory of a pair CTA for tiles BN columns wide: each CTA holds HB = BN / 2 weight
// columns; NB conversion buffers (two for 256-wide tiles, four for 128-wide ones, whose MMAs
// take half as long, so that conversion runs further ahead of them).
template <int BN_> struct Layout {
  static constexpr int BN = BN_, HB = BN_ / 2, NB = BN_ == kWide ? 2 : 4;
  float a[S][2][BK / 4][BM][4]; // panel block of this CTA's 128 rows (hi, lo) as copied
  float rawB[S][BK][HB];        // this CTA's half of the weight box as copied
  float bHi[NB][BK / 4][HB][4]; // converted weight half, K-major
  float bLo[NB][BK / 4][HB][4];
  unsigned long long full[S], empty[S], ready[NB], bEmpty[NB], accDone;
  unsigned long long unsignalled; // never arrived on (injected expiring wait)
  float2 halves[2][BM];           // argmax partials of each row's two column halves
  unsigned tmemBase;
  int abort;
};
static_assert(sizeof(Layout<kWide>) <= kMaxDynamicSmem, "shared memory budget");
static_assert(sizeof(Layout<kNarrow>) <= kMaxDynamicSmem, "shared memory budget");
// Accumulators staged row by row (logits, split-K partials); aliases the idle ring after the
// main loop.
template <int BN> using Staging = float[BM][BN + 4];
static_assert(sizeof(Staging<kWide>) <= sizeof(Layout<kWide>::a) + sizeof(Layout<kWide>::rawB),
              "staging fits the ring");
static_assert(sizeof(Staging<kNarrow>) <= sizeof(Layout<kNarrow>::a), "staging fits the ring");

inline std::size_t sharedBytes(int width) {
  return width == kWide ? sizeof(Layout<kWide>) : sizeof(Layout<kNarrow>);
}

// Output columns of one pair tile: the gate/up tile holds BN / 2 gate and BN / 2 up columns of
// the same outputs (gate in the leader's weight half, up in the peer's).
template <int EPI, int BN> constexpr int tileColumns() {
  return EPI == gemm::kSwiGluPanel ? BN / 2 : BN;
}

// kind::tf32, D f32, both operands K-major, M = 256 (over the pair), N = BN.
template <int BN> constexpr unsigned instruction() {
  return (1u << 4) | (2u << 7) | (2u << 10) | (unsigned(BN >> 3) << 17) |
         (unsigned(256 >> 4) << 24);
}

__device__ __forceinline__ unsigned clusterRank() {
  unsigned rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  return rank;
}

// Both CTAs' same warp allocate (and later free) `Columns` tensor-memory columns as a pair.
template <int Columns> __device__ __forceinline__ void tmemAllocPair(unsigned *slot) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smemAddress(slot)), "n"(Columns)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int Columns> __device__ __forceinline__ void tmemFreePair(unsigned base) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "n"(Columns)
               : "memory");
}

template <int BN>
__device__ __forceinline__ void mmaPair(unsigned tmem, unsigned long long a, unsigned long long b,
                                        unsigned accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\t"
               "setp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
               ::"r"(tmem), "l"(a), "l"(b), "n"(instruction<BN>()), "r"(accumulate)
               : "memory");
}

// Arrive (once, when the MMAs issued so far complete) on the barrier at the same offset in
// both CTAs of the pair whose leader has cluster rank `leader`.
__device__ __forceinline__ void commitPair(unsigned long long *bar, unsigned leader) {
  const unsigned short mask = static_cast<unsigned short>(0x3u << leader);
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::"
               "cluster.b64 [%0], %1;" ::"r"(smemAddress(bar)),
               "h"(mask)
               : "memory");
}

// Arrive on the barrier at the same offset in CTA `rank` of the cluster.  The data it
// announces is this CTA's own shared memory, read by this SM's tensor core as part of the
// pair's MMA; the writers fenced it for the async proxy and met at a CTA barrier first.
__device__ __forceinline__ void arriveRemote(unsigned long long *bar, unsigned rank) {
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smemAddress(bar)), "r"(rank));
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

__device__ __forceinline__ void converterSync() {
  asm volatile("bar.sync %0, %1;" ::"n"(kConverterBarrier), "n"(kConverterThreads) : "memory");
}

// Named barrier over the converter warps that also ANDs a predicate across them, so that they
// leave the main loop together (none is left waiting at converterSync).
__device__ __forceinline__ bool converterAll(bool value) {
  unsigned out;
  asm volatile("{\n\t.reg .pred p, q;\n\t"
               "setp.ne.u32 p, %1, 0;\n\t"
               "barrier.cta.red.and.pred q, %2, %3, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}"
               : "=r"(out)
               : "r"(unsigned(value)), "n"(kConverterBarrier), "n"(kConverterThreads)
               : "memory");
  return out != 0;
}

// 16 consecutive accumulator columns of this thread's row, without waiting for them.
__device__ __forceinline__ void tmemLoad16Async(unsigned address, unsigned (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
               "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                 "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(address));
}

__device__ __forceinline__ void tmemWaitLoads() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Rows [128 * (2 * group + rank), +128) of A times a 256-column tile of W (gate/up: 128 gate
// and 128 up columns).  Grid: x = 2 x column tiles (the pair's two CTAs adjacent in x), y = row
// pairs, z = SPLITS contiguous ranges of K slices (cluster 2 x 1 x SPLITS: the pairs of one
// tile's K splits reduce their partial tiles through distributed shared memory, in split
// order).  The argmax head (SPLITS == 1) writes two partial slots per row and column tile
// (slots 2 nt and 2 nt + 1, so that the slot count is grid.x): the row's partial and an empty
// one.
//
// EPI == kQkv: q, k and v (each [K, N] with N a multiple of 256) as one 3N-wide output; each
// column tile lies in one projection, whose weight map (weights, upWeights, vWeights), RoPE /
// cache-append epilogue and output it takes.
template <int EPI, int SPLITS = 1, int BN = kWide>
__device__ void body(const gemm::Params &p, const WeightMap &weights,
                     const WeightMap *upWeights = nullptr, const WeightMap *vWeights = nullptr) {
  using Smem = Layout<BN>;
  constexpr int HB = Smem::HB, NB = Smem::NB;
  static_assert(EPI != gemm::kQkv || BN == kWide, "q/k/v tiles are 256 wide");
  static_assert(SPLITS == 1 || (EPI != gemm::kSwiGluPanel && EPI != gemm::kArgmax),
                "gate/up and the argmax heads are not split");
  // Clusters of up to 16 CTAs: more than 8 is a non-portable size, allowed per kernel by the
  // runtime (cudaFuncAttributeNonPortableClusterSizeAllowed) when it selects the kernel.
  static_assert(2 * SPLITS <= 16 && (BN == kWide || 2 * SPLITS <= 8), "cluster size");
  extern __shared__ __align__(1024) unsigned char raw[];
  Smem &sm = *reinterpret_cast<Smem *>(raw);
  const GemmSpec &s = p.s;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const unsigned clusterRankValue = clusterRank();
  const unsigned rank = clusterRankValue & 1u;     // 0: the pair's leader
  const unsigned leader = clusterRankValue & ~1u;  // the leader's rank in the cluster
  const unsigned split = blockIdx.z;               // == the cluster's z index
  const int64_t K = s.K, N = s.N;
  const int64_t rowTiles = (s.M + BM - 1) / BM;
  const int64_t pairs = gridDim.y, columnTiles = gridDim.x / 2;
  // Tiles in launch order with the row pair varying fastest: the pairs that share a weight
  // tile run together and read it from HBM once.
  const int64_t tile = int64_t(blockIdx.y) * columnTiles + blockIdx.x / 2;
  const int64_t group = tile % pairs, nt = tile / pairs;
  const int64_t rowTile = 2 * group + rank;
  const bool hasRows = rowTile < rowTiles;
  // kQkv: projection (0 q, 1 k, 2 v) of this column tile; n0 is the tile's first column
  // within that projection.
  const int projection = EPI == gemm::kQkv ? int((nt * BN) / N) : 0;
  const int64_t n0 = nt * tileColumns<EPI, BN>() - int64_t(projection) * N;
  const bool upHalf = (EPI == gemm::kSwiGluPanel && rank == 1) || projection == 1;
  const int64_t wn0 = EPI == gemm::kSwiGluPanel ? n0 : n0 + int64_t(rank) * HB;
  const WeightMap &map = projection == 2 ? *vWeights : upHalf ? *upWeights : weights;
  const float *W = (projection == 2 ? p.w3 : upHalf ? p.w2 : p.w) + s.layer * K * N;
  // This split's K slices [kBegin, kEnd); an empty range contributes zeros.
  const int64_t allSlices = panel::slices(K);
  const int64_t perSplit = (allSlices + SPLITS - 1) / SPLITS;
  const int64_t kBegin = perSplit * split;
  const int64_t kEnd = kBegin + perSplit < allSlices ? kBegin + perSplit : allSlices;
  const int64_t slices = kEnd > kBegin ? kEnd - kBegin : 0;

  int position = 0;
  if constexpr (EPI == gemm::kRope || EPI == gemm::kRopeAppend || EPI == gemm::kAppend ||
                EPI == gemm::kQkv) {
    position = p.position[0];
    if (position < 0 || position >= s.T)
      return; // outside cache capacity: the step writes nothing (grid-uniform)
  }
  if (!aligned16(p.a) || smemAddress(raw) % 128 != 0) {
    if (threadIdx.x == 0)
      atomicOr(&g_libraryFaults, 2u); // grid-uniform: every CTA returns here
    return;
  }
  const bool copyRows =
      weights.valid != 0 &&
      (EPI != gemm::kSwiGluPanel || upWeights->valid != 0) &&
      (EPI != gemm::kQkv || (upWeights->valid != 0 && vWeights->valid != 0));

  if (warp == kMmaWarp)
    tmemAllocPair<2 * BN>(&sm.tmemBase);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbarrierInit(&sm.full[i], 1);
      mbarrierInit(&sm.empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbarrierInit(&sm.ready[i], kReadyArrivals);
      mbarrierInit(&sm.bEmpty[i], 1);
    }
    mbarrierInit(&sm.accDone, 1);
    mbarrierInit(&sm.unsignalled, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fenceBeforeSync();
  clusterSync(); // every CTA's barriers initialised before any remote arrival
  fenceAfterSync();
  const unsigned tmem = sm.tmemBase;
  volatile int *abort = &sm.abort;
  bool valid = false; // epilogue warps: every MMA completed, nothing aborted

  if (warp == kProducerWarp) {
    const unsigned boxBytes = copyRows ? unsigned(BK * HB * 4) : 0u;
    const unsigned blockBytes = hasRows ? unsigned(2 * panel::kPart * 4) : 0u;
    int64_t issued = 0;
    if (lane == 0 && copyRows)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&map.map))
                   : "memory");
    for (int64_t kt = 0; kt < slices; ++kt) {
      const int slot = int(kt % S);
      bool ok = true;
      if (lane == 0 && kt >= S)
        ok = waitPhase(&sm.empty[slot], unsigned((kt / S - 1) & 1), abort);
      if (!__shfl_sync(0xffffffffu, ok, 0))
        break;
      if (lane == 0) {
        mbarrierArriveExpectTx(&sm.full[slot], blockBytes + boxBytes);
        if (hasRows)
          bulkCopy(&sm.a[slot][0][0][0][0],
                   p.a + (rowTile * allSlices + kBegin + kt) * panel::kBlock, blockBytes,
                   &sm.full[slot]);
        if (copyRows)
          tensorCopy(&sm.rawB[slot][0][0], &map.map, int(wn0), int((kBegin + kt) * BK),
                     int(s.layer), &sm.full[slot]);
      }
      issued = kt + 1;
    }
    // Leave no copy in flight (bounded, regardless of abort).
    if (lane == 0)
      for (int64_t kt = issued > S ? issued - S : 0; kt < issued; ++kt)
        waitPhase(&sm.full[kt % S], unsigned((kt / S) & 1), nullptr);
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (rank == 0 && lane == 0) {
      const bool injected =
          g_injectUnsignalledWait != 0 && !waitPhase(&sm.unsignalled, 0, abort);
      for (int64_t kt = 0; kt < slices && !injected; ++kt) {
        const int slot = int(kt % S), buffer = int(kt % NB);
        if (!waitPhase(&sm.ready[buffer], unsigned((kt / NB) & 1), abort))
          break;
        fenceAfterSync();
        const int64_t remaining = K - (kBegin + kt) * BK;
        const int steps = int(remaining >= BK ? BK / 8 : (remaining + 7) / 8);
        for (int ks = 0; ks < steps; ++ks) {
          const unsigned long long bHi = matrixDescriptor(sm.bHi[buffer][2 * ks], HB * 16, 128);
          const unsigned long long bLo = matrixDescriptor(sm.bLo[buffer][2 * ks], HB * 16, 128);
          const unsigned long long aHi = matrixDescriptor(sm.a[slot][0][2 * ks], BM * 16, 128);
          const unsigned long long aLo = matrixDescriptor(sm.a[slot][1][2 * ks], BM * 16, 128);
          const unsigned first = (kt == 0 && ks == 0) ? 0u : 1u;
          mmaPair<BN>(tmem, aHi, bHi, first);
          mmaPair<BN>(tmem + BN, aHi, bLo, first);
          mmaPair<BN>(tmem + BN, aLo, bHi, 1u);
        }
        commitPair(&sm.empty[slot], leader);
        commitPair(&sm.bEmpty[buffer], leader);
      }
      // Tracks every MMA issued above, on success and on abort alike.
      commitPair(&sm.accDone, leader);
    }
    __syncwarp();
  } else {
    const int t = threadIdx.x - 2 * kWarp;
    for (int64_t kt = 0; kt < slices; ++kt) {
      const int slot = int(kt % S), buffer = int(kt % NB);
      bool ok = waitPhase(&sm.full[slot], unsigned((kt / S) & 1), abort);
      if (ok && kt >= NB)
        ok = waitPhase(&sm.bEmpty[buffer], unsigned((kt / NB - 1) & 1), abort);
      if (!converterAll(ok)) // uniform over the converter warps
        break;
      const int64_t k0 = (kBegin + kt) * BK;
      if (copyRows) {
        // Rows beyond K and columns beyond N arrive zero-filled.
#pragma unroll
        for (int g = 0; g < (BK / 4) * HB / kConverterThreads; ++g) {
          const int i = t + g * kConverterThreads;
          const int c = i / HB, n = i % HB;
          const float4 v = make_float4(sm.rawB[slot][4 * c][n], sm.rawB[slot][4 * c + 1][n],
                                       sm.rawB[slot][4 * c + 2][n], sm.rawB[slot][4 * c + 3][n]);
          float4 hi, lo;
          panel::split4(v, hi, lo);
          *reinterpret_cast<float4 *>(sm.bHi[buffer][c][n]) = hi;
          *reinterpret_cast<float4 *>(sm.bLo[buffer][c][n]) = lo;
        }
      } else {
#pragma unroll
        for (int g = 0; g < (BK / 4) * HB / kConverterThreads; ++g) {
          const int i = t + g * kConverterThreads;
          const int c = i / HB, n = i % HB;
          float4 v;
          float *lanes = &v.x;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int64_t k = k0 + 4 * c + j;
            lanes[j] = k < K && wn0 + n < N ? W[k * N + wn0 + n] : 0.f;
          }
          float4 hi, lo;
          panel::split4(v, hi, lo);
          *reinterpret_cast<float4 *>(sm.bHi[buffer][c][n]) = hi;
          *reinterpret_cast<float4 *>(sm.bLo[buffer][c][n]) = lo;
        }
      }
      fenceAsyncShared();
      converterSync();
      if (threadIdx.x == 2 * kWarp)
        arriveRemote(&sm.ready[buffer], leader);
    }
    // Wait (bounded) for every MMA the leader issued.
    const bool done = waitPhase(&sm.accDone, 0, nullptr);
    fenceAfterSync();
    valid = epilogueAll(done && !*abort) && slices > 0; // uniform over these warps
  }

  // Epilogue: this CTA's 128 rows from its own tensor memory, one row per thread; the two
  // warps of a lane quarter take half of the columns each.
  const int quarter = warp % 4, half = (warp - 2) / 4;
  const int row = quarter * kWarp + lane;
  const int64_t m = rowTile * BM + row;
  const unsigned rowAddress = tmem + (unsigned(quarter * kWarp) << 16);
  Staging<BN> &stage = *reinterpret_cast<Staging<BN> *>(&sm.a[0][0][0][0][0]);
  if constexpr (EPI == gemm::kSwiGluPanel) {
    // Outputs [half * 64, half * 64 + 64) of the tile: gate in columns c, up in HB + c.  A
    // warp's panel store of one output quad covers 32 consecutive rows (512 contiguous bytes).
    if (warp >= 2 && valid && hasRows) {
      const int64_t padded = panel::slices(N) * panel::kSlice;
#pragma unroll 1
      for (int c0 = half * (HB / 2); c0 < (half + 1) * (HB / 2); c0 += 16) {
        unsigned g[16], gc[16], u[16], uc[16];
        tmemLoad16Async(rowAddress + unsigned(c0), g);
        tmemLoad16Async(rowAddress + unsigned(BN + c0), gc);
        tmemLoad16Async(rowAddress + unsigned(HB + c0), u);
        tmemLoad16Async(rowAddress + unsigned(BN + HB + c0), uc);
        tmemWaitLoads();
        if (m < s.M) {
#pragma unroll
          for (int q = 0; q < 16; q += 4) {
            const int64_t k = n0 + c0 + q; // output column (the down panel's K)
            if (k >= padded)
              break;
            float4 v;
            float *out = &v.x;
#pragma unroll
            for (int j = 0; j < 4; ++j)
              out[j] = k + j < N
                           ? swigluValue(__fadd_rn(__uint_as_float(g[q + j]),
                                                   __uint_as_float(gc[q + j])),
                                         __fadd_rn(__uint_as_float(u[q + j]),
                                                   __uint_as_float(uc[q + j])))
                           : 0.f;
            panel::store4(p.out, m, k, N, v);
          }
        }
      }
    }
  } else if constexpr (EPI == gemm::kArgmax) {
    // Logits staged row by row, the row's argmax over each column half from registers in
    // column order; then halves merged (the lower half first: first index wins ties) and the
    // staged rows stored coalesced.
    if (warp >= 2 && valid && hasRows) {
      float best = -CUDART_INF_F;
      int bestIndex = 0x7fffffff;
#pragma unroll 1
      for (int c0 = half * HB; c0 < (half + 1) * HB; c0 += 16) {
        unsigned main[16], correction[16];
        float v[16];
        tmemLoad16Async(rowAddress + unsigned(c0), main);
        tmemLoad16Async(rowAddress + unsigned(BN + c0), correction);
        tmemWaitLoads();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = __fadd_rn(__uint_as_float(main[j]), __uint_as_float(correction[j]));
          if (n0 + c0 + j < N)
            argmaxMerge(best, bestIndex, v[j], int(n0 + c0 + j));
        }
        if (p.out != nullptr)
#pragma unroll
          for (int q = 0; q < 16; q += 4)
            *reinterpret_cast<float4 *>(&stage[row][c0 + q]) =
                make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      }
      sm.halves[half][row] = make_float2(best, __int_as_float(bestIndex));
    }
    __syncthreads();
    if (warp >= 2 && valid && hasRows) {
      if (half == 0 && m < s.M) {
        const float2 lower = sm.halves[0][row], upper = sm.halves[1][row];
        float best = lower.x;
        int bestIndex = __float_as_int(lower.y);
        argmaxMerge(best, bestIndex, upper.x, __float_as_int(upper.y));
        p.partials[m * s.tiles + 2 * nt] = make_float2(best, __int_as_float(bestIndex));
        p.partials[m * s.tiles + 2 * nt + 1] =
            make_float2(-CUDART_INF_F, __int_as_float(0x7fffffff)); // never wins a merge
      }
      if (p.out != nullptr) {
        const bool vec4 = N % 4 == 0 && aligned16(p.out);
        for (int r = warp - 2; r < BM && rowTile * BM + r < s.M; r += kConverterWarps) {
          const int64_t mr = rowTile * BM + r;
#pragma unroll
          for (int c = 4 * lane; c < BN; c += 4 * kWarp) {
            if (n0 + c >= N)
              break;
            const float4 v = *reinterpret_cast<const float4 *>(&stage[r][c]);
            if (vec4 && n0 + c + 4 <= N) {
              *reinterpret_cast<float4 *>(p.out + mr * N + n0 + c) = v;
            } else {
              const float *lanes = &v.x;
              for (int j = 0; j < 4 && n0 + c + j < N; ++j)
                p.out[mr * N + n0 + c + j] = lanes[j];
            }
          }
        }
      }
    }
  } else {
    // Stage the summed accumulators (zeros for an empty or abandoned split), then each split
    // CTA reduces rows [split * 128 / SPLITS, +128 / SPLITS) of this CTA's 128 rows over the
    // splits in rank order (deterministic) and stores them through the fused epilogue: one warp
    // per row, each lane four consecutive columns (512-byte rows).
    if (warp >= 2) {
#pragma unroll 1
      for (int c0 = half * HB; c0 < (half + 1) * HB; c0 += 16) {
        unsigned main[16], correction[16];
        if (valid) {
          tmemLoad16Async(rowAddress + unsigned(c0), main);
          tmemLoad16Async(rowAddress + unsigned(BN + c0), correction);
          tmemWaitLoads();
        }
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4 *>(&stage[row][c0 + q]) =
              valid ? make_float4(
                          __fadd_rn(__uint_as_float(main[q]), __uint_as_float(correction[q])),
                          __fadd_rn(__uint_as_float(main[q + 1]),
                                    __uint_as_float(correction[q + 1])),
                          __fadd_rn(__uint_as_float(main[q + 2]),
                                    __uint_as_float(correction[q + 2])),
                          __fadd_rn(__uint_as_float(main[q + 3]),
                                    __uint_as_float(correction[q + 3])))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if constexpr (SPLITS > 1)
      clusterSync();
    else
      __syncthreads();
    if (warp >= 2 && hasRows && __all_sync(0xffffffffu, !*abort)) {
      constexpr int kRows = BM / SPLITS;
      const bool vec4 = N % 4 == 0 && aligned16(p.out) &&
                        (EPI != gemm::kResidual || aligned16(p.residual));
      // kQkv: the projection's own epilogue and output.
      gemm::Params own = p;
      if constexpr (EPI == gemm::kQkv)
        own.out = projection == 0 ? p.out : projection == 1 ? p.out2 : p.out3;
      float best = -CUDART_INF_F; // unused by these epilogues
      int bestIndex = 0x7fffffff;
      // A warp's rows in batches: every staged partial of a batch (through distributed shared
      // memory for K splits) is loaded before any is summed, instead of one round trip per row
      // (traced: the row-at-a-time loop took ~15,700 of a ~47,000-cycle fused q/k/v CTA).  The
      // batch keeps at most 8 float4 partials per lane live; sums are in split order as before.
      constexpr int kQuads = BN / (4 * kWarp);
      constexpr int kPerWarp = kRows / kConverterWarps;
      constexpr int kFit = 8 / (kQuads * SPLITS) > 0 ? 8 / (kQuads * SPLITS) : 1;
      constexpr int kBatch = kPerWarp < kFit ? kPerWarp : kFit;
      static_assert(kRows % kConverterWarps == 0, "rows split evenly over the warps");
      const int r0 = int(split) * kRows + (warp - 2);
      for (int b0 = 0; b0 < kPerWarp; b0 += kBatch) {
        float4 part[kBatch][kQuads][SPLITS];
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
#pragma unroll
          for (int qd = 0; qd < kQuads; ++qd) {
            const int r = r0 + (b0 + i) * kConverterWarps, c = 4 * lane + qd * 4 * kWarp;
            if constexpr (SPLITS == 1) {
              part[i][qd][0] = *reinterpret_cast<const float4 *>(&stage[r][c]);
            } else {
#pragma unroll
              for (unsigned q = 0; q < SPLITS; ++q)
                part[i][qd][q] = loadCluster(&stage[r][c], rank + 2 * q);
            }
          }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          const int r = r0 + (b0 + i) * kConverterWarps;
          const int64_t mr = rowTile * BM + r;
          if (mr >= s.M)
            break; // rows increase with i
#pragma unroll
          for (int qd = 0; qd < kQuads; ++qd) {
            const int c = 4 * lane + qd * 4 * kWarp;
            if (n0 + c >= N)
              break;
            float4 sum = part[i][qd][0];
#pragma unroll
            for (int q = 1; q < SPLITS; ++q)
              sum = make_float4(__fadd_rn(sum.x, part[i][qd][q].x),
                                __fadd_rn(sum.y, part[i][qd][q].y),
                                __fadd_rn(sum.z, part[i][qd][q].z),
                                __fadd_rn(sum.w, part[i][qd][q].w));
            if constexpr (EPI == gemm::kQkv) {
              if (projection == 0)
                storeQuad<gemm::kRope>(own, mr, n0 + c, sum, position, vec4, best, bestIndex);
              else if (projection == 1)
                storeQuad<gemm::kRopeAppend>(own, mr, n0 + c, sum, position, vec4, best,
                                             bestIndex);
              else
                storeQuad<gemm::kAppend>(own, mr, n0 + c, sum, position, vec4, best, bestIndex);
            } else {
              storeQuad<EPI>(p, mr, n0 + c, sum, position, vec4, best, bestIndex);
            }
          }
        }
      }
    }
  }
  fenceBeforeSync();
  clusterSync(); // every CTA done with tensor memory and with the others' shared memory
  fenceAfterSync();
  if (warp == kMmaWarp)
    tmemFreePair<2 * BN>(tmem);
}

} // namespace ckl::kernels::tc::pair
