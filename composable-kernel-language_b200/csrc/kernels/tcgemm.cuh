// Tensor-core (tcgen05) projection kernel with FP32-level accuracy (3xTF32).
//
// out = epilogue(prologue(A) @ W[layer]) for batched decode (M >= 128 requests), where a
// projection is a true dense contraction.  Each FP32 operand is split into a TF32 high part
// and a TF32 low part (x = hi + lo, both rounded to nearest); hi*hi accumulates in one FP32
// tensor-memory accumulator and the two correction products hi*lo + lo*hi in a second one,
// summed in FP32 by the epilogue (the dropped lo*lo term is ~2^-22 relative).  This keeps
// the decoder's 1e-4 relative tolerance and greedy-token parity that plain TF32 breaks.
//
// CTA: 256 threads (8 warps), tile 128 rows x BN columns, K in slices of 32.
//   * raw FP32 slices of A, W (and the RMSNorm gain) stream from global memory into a ring
//     of S shared-memory stages with 16-byte cp.async copies, S-1 slices ahead (when shapes
//     and pointers allow; otherwise each slice is loaded synchronously into stage 0);
//   * all threads convert a landed slice into one of two canonical stages: prologue (RMSNorm
//     gain; the row scale is applied in the epilogue from sums of squares accumulated here),
//     TF32 hi/lo split by integer rounding, K-major no-swizzle layout: element (row, k) at
//     byte ((k / 4) * rows + row) * 16 + (k % 4) * 4 (8-row x 16-byte core matrices, K-chunks
//     `rows * 16` bytes apart = LBO, 8-row groups 128 bytes apart = SBO);
//   * one thread issues 4 k-steps x 3 `tcgen05.mma.cta_group::1.kind::tf32` (M=128, N=BN,
//     K=8) per slice and commits them to the stage's mbarrier; a canonical stage is reused
//     only after those MMAs completed;
//   * the epilogue reads the accumulators with `tcgen05.ld.32x32b` (warps w and w+4 share
//     TMEM lanes 32(w%4).., one row per thread, half the columns each).
// Every mbarrier wait is bounded by time: on expiry the kernel records a fault bit
// (ckl_library_faults), waits (again bounded) for its in-flight MMAs, frees its tensor memory
// and returns; it never spins without a limit.
#pragma once

#include "common.cuh"
#include "gemm.cuh"

namespace ckl::kernels::tc {

constexpr int BM = 128;
constexpr int BK = 32;
constexpr int kThreads = 256; // 8 warps: two per accumulator lane quarter
constexpr unsigned long long kWaitLimitNs = 2000000000ull; // 2 s

// Fault word of the library (bit 0: a tensor-core wait expired).  One translation unit
// (decoder_fused.cu) instantiates these kernels and reports the word (ckl_library_faults).
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

// Round to the nearest TF32 value (10 explicit mantissa bits) with integer operations
// (ties away from zero, as cvt.rna); keeps the conversion off the transcendental pipe.
__device__ __forceinline__ float toTf32(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ void split(float x, float &hi, float &lo) {
  hi = toTf32(x);
  lo = toTf32(x - hi);
}

__device__ __forceinline__ void mbarrierInit(unsigned long long *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemAddress(bar)), "r"(count)
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

// Bounded wait for an mbarrier phase; false when the time limit expired.
__device__ __forceinline__ bool mbarrierWait(unsigned long long *bar, unsigned phase) {
  if (mbarrierTryWait(bar, phase))
    return true;
  const unsigned long long start = globalTimer();
  while (true) {
    if (mbarrierTryWait(bar, phase))
      return true;
    if (globalTimer() - start > kWaitLimitNs)
      return false;
  }
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

constexpr std::size_t kMaxDynamicSmem = 227 * 1024;

template <int BN, int S> struct Smem {
  float aHi[2][BK / 4][BM][4];
  float aLo[2][BK / 4][BM][4];
  float bHi[2][BK / 4][BN][4];
  float bLo[2][BK / 4][BN][4];
  float rawA[S][BM][BK + 4]; // padded rows: conflict-free 16-byte reads per row
  float rawB[S][BK][BN + 4];
  float rawG[S][BK];         // RMSNorm gain slice
  float squares[2][BM];      // per-row partial sums of squares (RMSNorm)
  unsigned long long mmaDone[2];
  unsigned long long accDone;
  unsigned tmemBase;
};

template <int BN, int S = 8> constexpr int stages() {
  if constexpr (S < 2)
    return 1;
  else if constexpr (sizeof(Smem<BN, S>) + 1024 <= kMaxDynamicSmem)
    return S;
  else
    return stages<BN, S - 1>();
}

// Dynamic shared memory of the asynchronous pipeline at a column width (the synchronous one
// needs less).
inline std::size_t sharedBytes(int width) {
  switch (width) {
  case 128: return sizeof(Smem<128, stages<128>()>);
  case 64: return sizeof(Smem<64, stages<64>()>);
  default: return sizeof(Smem<32, stages<32>()>);
  }
}

__device__ __forceinline__ void cpAsync16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smemAddress(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cpAsyncCommit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N> __device__ __forceinline__ void cpAsyncWait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int BN, class Layout>
__device__ __forceinline__ void issueSlice(Layout &sm, int stage, unsigned tmem, bool first) {
  constexpr unsigned idesc = instructionDescriptor<BN>();
#pragma unroll
  for (int ks = 0; ks < BK / 8; ++ks) {
    const unsigned long long aHi = matrixDescriptor(sm.aHi[stage][2 * ks], BM * 16, 128);
    const unsigned long long aLo = matrixDescriptor(sm.aLo[stage][2 * ks], BM * 16, 128);
    const unsigned long long bHi = matrixDescriptor(sm.bHi[stage][2 * ks], BN * 16, 128);
    const unsigned long long bLo = matrixDescriptor(sm.bLo[stage][2 * ks], BN * 16, 128);
    // Main products and correction products accumulate separately: the corrections are
    // ~2^-11 of the main term and keep their precision in their own accumulator.
    mma(tmem, aHi, bHi, idesc, (first && ks == 0) ? 0u : 1u);
    mma(tmem + BN, aHi, bLo, idesc, (first && ks == 0) ? 0u : 1u);
    mma(tmem + BN, aLo, bHi, idesc, 1u);
  }
}

// Epilogue: warps w and w+4 read TMEM lanes 32(w%4).. (one row per thread), columns
// [half*BN/2, (half+1)*BN/2); main + correction accumulators summed in FP32, optional row
// scale (RMSNorm), then the fused epilogue.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue(const gemm::Params &p, unsigned tmem, int64_t m0,
                                         int64_t n0, int position, float rowScale,
                                         float2 *rowBest) {
  const GemmSpec &s = p.s;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int quarter = warp % 4, half = warp / 4;
  const int64_t M = s.M, N = s.N;
  const int64_t m = m0 + quarter * 32 + lane;
  const unsigned rowAddress = tmem + (unsigned(quarter * 32) << 16);
  float best = -CUDART_INF_F;
  int bestIndex = 0x7fffffff;
#pragma unroll 1
  for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
    float v[16], correction[16];
    tmemLoad16(rowAddress + unsigned(c0), v);
    tmemLoad16(rowAddress + unsigned(BN + c0), correction);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      v[j] = __fmul_rn(v[j] + correction[j], rowScale);
    if (m >= M)
      continue;
    const int64_t nBase = n0 + c0;
    if constexpr (EPI == gemm::kStore || EPI == gemm::kResidual || EPI == gemm::kArgmax) {
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
    // The two column halves of a row meet in shared memory; the lower index wins ties.
    rowBest[half * BM + quarter * 32 + lane] = make_float2(best, __int_as_float(bestIndex));
    __syncthreads();
    if (half == 0 && m < M) {
      const float2 other = rowBest[BM + quarter * 32 + lane];
      argmaxMerge(best, bestIndex, other.x, __float_as_int(other.y));
      p.partials[m * s.tiles + blockIdx.x] = make_float2(best, __int_as_float(bestIndex));
    }
  }
}

template <int BN, int PRO, int EPI, bool ASYNC> __device__ void body(const gemm::Params &p) {
  static_assert(PRO != gemm::kSwiGlu, "the tensor-core path takes a materialised SwiGLU input");
  constexpr int S = ASYNC ? stages<BN>() : 1;
  using Layout = Smem<BN, S>;
  extern __shared__ __align__(1024) unsigned char raw[];
  Layout &sm = *reinterpret_cast<Layout *>(raw);
  const GemmSpec &s = p.s;
  const int tid = threadIdx.x, warp = tid / kWarp;
  const int64_t m0 = int64_t(blockIdx.y) * BM, n0 = int64_t(blockIdx.x) * BN;
  const int64_t M = s.M, K = s.K, N = s.N;
  const float *W = p.w + s.layer * K * N;
  const float *gain = p.gain + s.layer * K;

  int position = 0;
  if constexpr (EPI == gemm::kRope || EPI == gemm::kRopeAppend || EPI == gemm::kAppend) {
    position = p.position[0];
    if (position < 0 || position >= s.T)
      return;
  }
  const int64_t slices = (K + BK - 1) / BK;

  // Raw slice kt -> ring slot kt % S.
  auto fetch = [&](int64_t kt) {
    const int slot = int(kt % S);
    const int64_t k0 = kt * BK;
    for (int e = tid; e < BM * (BK / 4); e += kThreads) {
      const int r = e / (BK / 4), c = e % (BK / 4);
      const int64_t m = m0 + r, k = k0 + 4 * c;
      float *dst = &sm.rawA[slot][r][4 * c];
      if constexpr (ASYNC) {
        const bool valid = m < M && k < K;
        cpAsync16(dst, valid ? p.a + m * K + k : p.a, valid);
      } else {
        for (int i = 0; i < 4; ++i)
          dst[i] = (m < M && k + i < K) ? p.a[m * K + k + i] : 0.f;
      }
    }
    for (int e = tid; e < BK * (BN / 4); e += kThreads) {
      const int r = e / (BN / 4), c = e % (BN / 4);
      const int64_t k = k0 + r, n = n0 + 4 * c;
      float *dst = &sm.rawB[slot][r][4 * c];
      if constexpr (ASYNC) {
        const bool valid = k < K && n < N;
        cpAsync16(dst, valid ? W + k * N + n : W, valid);
      } else {
        for (int i = 0; i < 4; ++i)
          dst[i] = (k < K && n + i < N) ? W[k * N + n + i] : 0.f;
      }
    }
    if constexpr (PRO == gemm::kRms) {
      if (tid < BK / 4) {
        const int64_t k = k0 + 4 * tid;
        float *dst = &sm.rawG[slot][4 * tid];
        if constexpr (ASYNC) {
          cpAsync16(dst, k < K ? gain + k : gain, k < K);
        } else {
          for (int i = 0; i < 4; ++i)
            dst[i] = k + i < K ? gain[k + i] : 0.f;
        }
      }
    }
  };

  if constexpr (ASYNC) {
    for (int64_t i = 0; i < S - 1; ++i) {
      if (i < slices)
        fetch(i);
      cpAsyncCommit();
    }
  }
  if (warp == 0)
    tmemAlloc<2 * BN>(&sm.tmemBase);
  if (tid == 0) {
    mbarrierInit(&sm.mmaDone[0], 1);
    mbarrierInit(&sm.mmaDone[1], 1);
    mbarrierInit(&sm.accDone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fenceBeforeSync();
  __syncthreads();
  fenceAfterSync();
  const unsigned tmem = sm.tmemBase;

  // Conversion: thread tid takes A row tid % 128, chunks of its half, and a run of one B
  // column.  The RMSNorm row statistic accumulates here from the raw values.
  const int row = tid % BM, half = tid / BM;
  float squares = 0.f;
  auto convert = [&](int slot, int stage) {
#pragma unroll
    for (int cc = 0; cc < BK / 8; ++cc) {
      const int c = half * (BK / 8) + cc;
      float4 v = *reinterpret_cast<const float4 *>(&sm.rawA[slot][row][4 * c]);
      if constexpr (PRO == gemm::kRms) {
        squares += v.x * v.x;
        squares += v.y * v.y;
        squares += v.z * v.z;
        squares += v.w * v.w;
        const float4 g = *reinterpret_cast<const float4 *>(&sm.rawG[slot][4 * c]);
        v.x = __fmul_rn(v.x, g.x);
        v.y = __fmul_rn(v.y, g.y);
        v.z = __fmul_rn(v.z, g.z);
        v.w = __fmul_rn(v.w, g.w);
      }
      float4 hi, lo;
      split(v.x, hi.x, lo.x);
      split(v.y, hi.y, lo.y);
      split(v.z, hi.z, lo.z);
      split(v.w, hi.w, lo.w);
      *reinterpret_cast<float4 *>(sm.aHi[stage][c][row]) = hi;
      *reinterpret_cast<float4 *>(sm.aLo[stage][c][row]) = lo;
    }
    constexpr int kPerThread = BK * BN / kThreads; // k values of one column per thread
    const int col = tid % BN, kb = (tid / BN) * kPerThread;
#pragma unroll
    for (int j = 0; j < kPerThread; j += 4) {
      float4 hi, lo;
      split(sm.rawB[slot][kb + j][col], hi.x, lo.x);
      split(sm.rawB[slot][kb + j + 1][col], hi.y, lo.y);
      split(sm.rawB[slot][kb + j + 2][col], hi.z, lo.z);
      split(sm.rawB[slot][kb + j + 3][col], hi.w, lo.w);
      *reinterpret_cast<float4 *>(sm.bHi[stage][(kb + j) / 4][col]) = hi;
      *reinterpret_cast<float4 *>(sm.bLo[stage][(kb + j) / 4][col]) = lo;
    }
  };

  bool ok = true;
  unsigned phase[2] = {0, 0};
  for (int64_t kt = 0; kt < slices && ok; ++kt) {
    if constexpr (ASYNC) {
      if (kt + S - 1 < slices)
        fetch(kt + S - 1);
      cpAsyncCommit();
      cpAsyncWait<S - 1>(); // this thread's copies of slice kt have landed
    } else {
      fetch(kt);
    }
    const int stage = int(kt & 1);
    if (kt >= 2) {
      ok = mbarrierWait(&sm.mmaDone[stage], phase[stage]);
      phase[stage] ^= 1;
    }
    __syncthreads(); // slice kt visible to every thread
    if (ok) {
      convert(int(kt % S), stage);
      fenceAsyncShared();
    }
    ok = __syncthreads_and(ok);
    if (ok && tid == 0) {
      fenceAfterSync();
      issueSlice<BN, Layout>(sm, stage, tmem, kt == 0);
      commit(&sm.mmaDone[stage]);
    }
  }
  if constexpr (ASYNC)
    cpAsyncWait<0>();
  if (tid == 0)
    commit(&sm.accDone);
  bool done = mbarrierWait(&sm.accDone, 0);
  if constexpr (PRO == gemm::kRms)
    sm.squares[half][row] = squares;
  done = __syncthreads_and(done);
  if (!ok || !done) {
    if (tid == 0)
      atomicOr(&g_libraryFaults, 1u);
    fenceBeforeSync();
    __syncthreads();
    if (warp == 0)
      tmemFree<2 * BN>(tmem);
    return;
  }
  fenceAfterSync();
  float rowScale = 1.f;
  if constexpr (PRO == gemm::kRms) {
    const int r = (warp % 4) * 32 + tid % kWarp;
    rowScale = rsqrtf((sm.squares[0][r] + sm.squares[1][r]) / float(K) + p.eps);
  }
  // The argmax epilogue reuses the (now idle) raw A ring to merge column halves.
  epilogue<BN, EPI>(p, tmem, m0, n0, position, rowScale,
                    reinterpret_cast<float2 *>(&sm.rawA[0][0][0]));
  fenceBeforeSync();
  __syncthreads();
  if (warp == 0)
    tmemFree<2 * BN>(tmem);
}

// Entry used by the kernel wrappers: the asynchronous pipeline when shapes and pointers
// allow 16-byte copies, the synchronous one otherwise.
template <int BN, int PRO, int EPI> __device__ void run(const gemm::Params &p) {
  const GemmSpec &s = p.s;
  const float *W = p.w + s.layer * s.K * s.N;
  const bool vec = s.K % 4 == 0 && s.N % 4 == 0 && aligned16(p.a) && aligned16(W) &&
                   (PRO != gemm::kRms || aligned16(p.gain + s.layer * s.K));
  if (vec)
    body<BN, PRO, EPI, true>(p);
  else
    body<BN, PRO, EPI, false>(p);
}

} // namespace ckl::kernels::tc
