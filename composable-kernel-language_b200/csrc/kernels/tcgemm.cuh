// Tensor-core (tcgen05) projection kernel with FP32-level accuracy (3xTF32).
//
// out = epilogue(A @ W[layer]) for batched decode (M >= 128 requests), A given as a split
// panel (panel.cuh: TF32 hi/lo parts in the tensor cores' shared-memory layout, produced
// once by the kernel that computes A), W the FP32 weights [K, N] of one layer, read as stored.
// hi*hi accumulates in one FP32 tensor-memory accumulator and the correction products
// hi*lo + lo*hi in a second one, summed in FP32 by the epilogue (the dropped lo*lo term is
// ~2^-22 relative).  This keeps the decoder's 1e-4 relative tolerance and greedy-token parity
// that plain TF32 breaks.
//
// CTA: one 128 x BN output tile, K in slices of 32, six warps with fixed roles:
//   warp 0 (producer): per slice one 32 KB bulk copy of the panel block (hi + lo) and one
//     bulk copy per weight row (BN floats) into a ring of S stages, completing on the
//     stage's `full` mbarrier; a stage is refilled after the MMAs that read it completed;
//   warp 1 (MMA): allocates 2*BN tensor-memory columns; per slice, once the panel block has
//     landed and the weight slice is converted, one thread issues up to 4 k-steps x 3
//     `tcgen05.mma.cta_group::1.kind::tf32` (M=128, N=BN, K=8) and commits them to the
//     stage's `empty` and the weight buffer's `bEmpty` mbarriers;
//   warps 2-5 (converters, then epilogue): split each landed weight slice into TF32 hi/lo in
//     K-major no-swizzle layout (two buffers), then read the accumulators with
//     `tcgen05.ld.32x32b` (warp w reads TMEM lanes 32 (w % 4).., one output row per thread)
//     and apply the fused epilogue.
// Weight slices whose rows or pointer do not allow 16-byte copies are read by the converters
// straight from global memory instead.
//
// Every mbarrier wait is bounded by time.  A wait that expires records a fault bit
// (ckl_library_faults) and raises a CTA-wide abort flag that ends the other roles' waits; the
// CTA then waits (again bounded) for its in-flight copies and MMAs, frees its tensor memory
// and returns.  No wait spins without a limit.
#pragma once

#include "common.cuh"
#include "gemm.cuh"
#include "panel.cuh"

namespace ckl::kernels::tc {

constexpr int BM = panel::kRows;
constexpr int BK = panel::kSlice;
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kConverterWarps = 4; // warps 2..5; also the epilogue
constexpr int kConverterThreads = kConverterWarps * kWarp;
constexpr int kThreads = (2 + kConverterWarps) * kWarp;
constexpr unsigned long long kWaitLimitNs = 2000000000ull; // 2 s
constexpr std::size_t kMaxDynamicSmem = 227 * 1024;

// Fault word of the library (bit 0: a tensor-core wait expired).  One translation unit
// instantiates these kernels and reports the word (ckl_library_faults).
static __device__ unsigned g_libraryFaults = 0;

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
// raises it (and the fault bit) when the time limit expires.
__device__ __forceinline__ bool waitPhase(unsigned long long *bar, unsigned phase,
                                          volatile int *abort) {
  if (mbarrierTryWait(bar, phase))
    return true;
  const unsigned long long start = globalTimer();
  while (true) {
    if (mbarrierTryWait(bar, phase))
      return true;
    if (abort != nullptr && *abort)
      return false;
    if (globalTimer() - start > kWaitLimitNs) {
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

// Column width of the tile for a specialization: enough CTAs to fill the GPU when possible.
inline int chooseWidth(const GemmSpec &s) {
  const int64_t rowTiles = (s.M + BM - 1) / BM;
  for (int width : {128, 64})
    if (rowTiles * ((s.N + width - 1) / width) >= 120)
      return width;
  return 32;
}

template <int BN, int S> struct Smem {
  float a[S][2][BK / 4][BM][4]; // panel blocks (hi, lo) as copied
  float bHi[2][BK / 4][BN][4];  // converted weight slices, K-major
  float bLo[2][BK / 4][BN][4];
  float rawB[S][BK][BN];        // weight rows as copied
  unsigned long long full[S], empty[S], bFull[2], bEmpty[2], accDone;
  unsigned tmemBase;
  int abort;
};

template <int BN> constexpr int stages() {
  return sizeof(Smem<BN, 4>) <= kMaxDynamicSmem ? 4 : (sizeof(Smem<BN, 3>) <= kMaxDynamicSmem ? 3 : 2);
}
static_assert(sizeof(Smem<128, stages<128>()>) <= kMaxDynamicSmem, "shared memory budget");

// Dynamic shared memory of the kernel at a column width.
inline std::size_t sharedBytes(int width) {
  switch (width) {
  case 128: return sizeof(Smem<128, stages<128>()>);
  case 64: return sizeof(Smem<64, stages<64>()>);
  default: return sizeof(Smem<32, stages<32>()>);
  }
}

// Epilogue of one output row (this thread's) over the tile's BN columns: main + correction
// accumulators summed in FP32, then the fused epilogue.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue(const gemm::Params &p, unsigned rowAddress, int64_t m,
                                         int64_t n0, int position) {
  const GemmSpec &s = p.s;
  const int64_t M = s.M, N = s.N;
  const bool vec4 = N % 4 == 0 && aligned16(p.out) &&
                    (EPI != gemm::kResidual || aligned16(p.residual));
  float best = -CUDART_INF_F;
  int bestIndex = 0x7fffffff;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 16) {
    float v[16], correction[16];
    tmemLoad16(rowAddress + unsigned(c0), v);
    tmemLoad16(rowAddress + unsigned(BN + c0), correction);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      v[j] = __fadd_rn(v[j], correction[j]);
    const int64_t nBase = n0 + c0;
    if (m >= M || nBase >= N)
      continue;
    if constexpr (EPI == gemm::kStore || EPI == gemm::kResidual || EPI == gemm::kArgmax) {
      if (vec4 && nBase + 16 <= N) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          float4 value = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          if constexpr (EPI == gemm::kResidual) {
            const float4 r = *reinterpret_cast<const float4 *>(p.residual + m * N + nBase + j);
            value = make_float4(__fadd_rn(r.x, value.x), __fadd_rn(r.y, value.y),
                                __fadd_rn(r.z, value.z), __fadd_rn(r.w, value.w));
          }
          *reinterpret_cast<float4 *>(p.out + m * N + nBase + j) = value;
        }
        if constexpr (EPI == gemm::kArgmax) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            argmaxMerge(best, bestIndex, v[j], int(nBase + j));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int64_t n = nBase + j;
          if (n < N) {
            float value = v[j];
            if constexpr (EPI == gemm::kResidual)
              value = __fadd_rn(p.residual[m * N + n], value);
            p.out[m * N + n] = value;
            if constexpr (EPI == gemm::kArgmax)
              argmaxMerge(best, bestIndex, v[j], int(n));
          }
        }
      }
    } else {
      const int64_t D = s.D, R = s.D / 2;
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const int64_t n = nBase + j;
        if (n >= N)
          continue;
        float first = v[j], second = v[j + 1];
        const int64_t h = n / D, d = n % D;
        if constexpr (EPI == gemm::kRope || EPI == gemm::kRopeAppend) {
          const float *cs = p.table + (int64_t(position) * R + d / 2) * 2;
          const float cosine = cs[0], sine = cs[1];
          const float x = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
          const float y = __fadd_rn(__fmul_rn(first, sine), __fmul_rn(second, cosine));
          first = x;
          second = y;
        }
        if constexpr (EPI == gemm::kRope) {
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
  if constexpr (EPI == gemm::kArgmax) {
    if (m < M)
      p.partials[m * s.tiles + blockIdx.x] = make_float2(best, __int_as_float(bestIndex));
  }
}

// One 128 x BN tile.  p.a is the panel of A [M, K]; p.w the weights [layers, K, N].
template <int BN, int EPI> __device__ void body(const gemm::Params &p) {
  constexpr int S = stages<BN>();
  using Layout = Smem<BN, S>;
  extern __shared__ __align__(1024) unsigned char raw[];
  Layout &sm = *reinterpret_cast<Layout *>(raw);
  const GemmSpec &s = p.s;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t M = s.M, K = s.K, N = s.N;
  const int64_t m0 = int64_t(blockIdx.y) * BM, n0 = int64_t(blockIdx.x) * BN;
  const int64_t slices = panel::slices(K);
  const float *W = p.w + s.layer * K * N;
  const float *blocks = p.a + int64_t(blockIdx.y) * slices * panel::kBlock;

  int position = 0;
  if constexpr (EPI == gemm::kRope || EPI == gemm::kRopeAppend || EPI == gemm::kAppend) {
    position = p.position[0];
    if (position < 0 || position >= s.T)
      return; // outside cache capacity: the step writes nothing
  }
  if (!aligned16(p.a)) {
    if (threadIdx.x == 0)
      atomicOr(&g_libraryFaults, 2u); // panel operands are 16-byte aligned by construction
    return;
  }
  // Weight rows by bulk copy when every row slice is a 16-byte multiple at a 16-byte address.
  const bool copyRows = N % 4 == 0 && aligned16(W);

  if (warp == kMmaWarp)
    tmemAlloc<2 * BN>(&sm.tmemBase);
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
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fenceBeforeSync();
  __syncthreads();
  fenceAfterSync();
  const unsigned tmem = sm.tmemBase;
  volatile int *abort = &sm.abort;

  if (warp == kProducerWarp) {
    const unsigned rowBytes = unsigned((N - n0 < BN ? N - n0 : BN) * 4);
    int64_t issued = 0;
    for (int64_t kt = 0; kt < slices; ++kt) {
      const int slot = int(kt % S);
      bool ok = true;
      if (lane == 0 && kt >= S)
        ok = waitPhase(&sm.empty[slot], unsigned((kt / S - 1) & 1), abort);
      if (!__shfl_sync(0xffffffffu, ok, 0))
        break;
      const int64_t k0 = kt * BK;
      const int rows = int(K - k0 < BK ? K - k0 : BK);
      if (lane == 0)
        mbarrierArriveExpectTx(&sm.full[slot],
                               unsigned(2 * panel::kPart * 4) + (copyRows ? rows * rowBytes : 0u));
      __syncwarp();
      if (lane == 0)
        bulkCopy(&sm.a[slot][0][0][0][0], blocks + kt * panel::kBlock,
                 unsigned(2 * panel::kPart * 4), &sm.full[slot]);
      if (copyRows && lane < rows)
        bulkCopy(&sm.rawB[slot][lane][0], W + (k0 + lane) * N + n0, rowBytes, &sm.full[slot]);
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
      for (int64_t kt = 0; kt < slices; ++kt) {
        const int slot = int(kt % S), buffer = int(kt & 1);
        if (!waitPhase(&sm.full[slot], unsigned((kt / S) & 1), abort) ||
            !waitPhase(&sm.bFull[buffer], unsigned((kt / 2) & 1), abort))
          break;
        fenceAfterSync();
        const int64_t remaining = K - kt * BK;
        const int steps = int(remaining >= BK ? BK / 8 : (remaining + 7) / 8);
        for (int ks = 0; ks < steps; ++ks) {
          const unsigned long long aHi = matrixDescriptor(sm.a[slot][0][2 * ks], BM * 16, 128);
          const unsigned long long aLo = matrixDescriptor(sm.a[slot][1][2 * ks], BM * 16, 128);
          const unsigned long long bHi = matrixDescriptor(sm.bHi[buffer][2 * ks], BN * 16, 128);
          const unsigned long long bLo = matrixDescriptor(sm.bLo[buffer][2 * ks], BN * 16, 128);
          const unsigned first = (kt == 0 && ks == 0) ? 0u : 1u;
          mma(tmem, aHi, bHi, idesc, first);
          mma(tmem + BN, aHi, bLo, idesc, first);
          mma(tmem + BN, aLo, bHi, idesc, 1u);
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
      const int64_t k0 = kt * BK;
      // Group i: four consecutive k (chunk c) of column n.
      for (int i = t; i < (BK / 4) * BN; i += kConverterThreads) {
        const int c = i / BN, n = i % BN;
        float4 v;
        float *lanes = &v.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t k = k0 + 4 * c + j;
          float value = 0.f;
          if (k < K) {
            if (copyRows)
              value = sm.rawB[slot][4 * c + j][n];
            else if (n0 + n < N)
              value = W[k * N + n0 + n];
          }
          lanes[j] = value;
        }
        float4 hi, lo;
        panel::split4(v, hi, lo);
        *reinterpret_cast<float4 *>(sm.bHi[buffer][c][n]) = hi;
        *reinterpret_cast<float4 *>(sm.bLo[buffer][c][n]) = lo;
      }
      fenceAsyncShared();
      __syncwarp();
      if (lane == 0)
        mbarrierArrive(&sm.bFull[buffer]);
    }
    // Epilogue: wait (bounded) for every issued MMA, then read this warp's TMEM lanes.
    const bool done = waitPhase(&sm.accDone, 0, nullptr);
    fenceAfterSync();
    if (__all_sync(0xffffffffu, done && !*abort)) { // warp-uniform: tcgen05.ld is .aligned
      const int quarter = warp % 4;
      epilogue<BN, EPI>(p, tmem + (unsigned(quarter * 32) << 16), m0 + quarter * 32 + lane, n0,
                        position);
    }
  }
  fenceBeforeSync();
  __syncthreads();
  if (warp == kMmaWarp)
    tmemFree<2 * BN>(tmem);
}

} // namespace ckl::kernels::tc
