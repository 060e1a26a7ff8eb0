// Whole decode step of a small decoder in one launch.
//
// For decoders whose weights stay resident in L2 (a few MB: the latency-bound configurations),
// a step of 19-76 dependent graph nodes costs mostly launch and drain latency.  This kernel runs
// the entire step (embedding, every layer, final norm, LM head, greedy selection and the
// position advance) as one launch of 8-CTA thread-block clusters:
//   * requests are partitioned across clusters (G rows each); clusters never wait for one
//     another: the last cluster to finish advances `position` (a last-arriver counter);
//   * inside a cluster every CTA keeps a full copy of its rows' residual stream in shared
//     memory; the heads are partitioned over the 8 CTAs (by row group when there are fewer
//     than 8), and a CTA computes q/k/v of its heads, appends them to the cache, runs their
//     attention and multiplies the result by its rows of Wo, all in its own shared memory;
//   * the o projection and the down projection (K split by CTA: its heads' columns, its FFN
//     columns) leave partial sums [rows][C] in each CTA; after one cluster barrier
//     (barrier.cluster arrive/wait, release/acquire at cluster scope) every CTA adds all
//     partials, read through distributed shared memory in rank order, to its own copy, so a
//     layer needs two cluster barriers; gate/up split their output columns over the CTAs;
//   * projections read their weights straight from L2 (they stay resident there), each thread
//     reusing every weight load for the requests of a row block (two or four) held in registers;
//   * RMSNorm statistics are recomputed by every CTA from its own copy (no exchange);
//   * attention gives each (request, head) of a CTA one or more of its warps, which split the
//     cache rows: scores, softmax in shared memory, then the weighted value sums.
// FFMA throughout; per output the K range is split over threads and reduced in a fixed order.
#include "ckl_b200.h"
#include "common.cuh"

#include <cooperative_groups.h>

namespace ckl::kernels {
namespace {

namespace cg = cooperative_groups;

constexpr int kStepCtas = 8;      // CTAs per cluster
constexpr int kStepThreads = 256; // threads per CTA
constexpr int kStepWarps = kStepThreads / kWarp;
constexpr int kMaxRows = 16;      // rows (requests) per cluster
constexpr int kRowBlock = 4;              // rows per single projection pass (accumulators)
constexpr int kFusedRowBlock = 2;         // rows per pass of fused q/k/v or gate/up
// Partials of one pass plus the segment sums: a pass holds at most 256 x COUNT x RB float4
// partials (threads x slices x rows of a row block), the larger of the fused three-slice pass
// and the single-slice pass, and at most 256 float4 segment sums.
constexpr int kPassPartials =
    kStepThreads * (3 * kFusedRowBlock > kRowBlock ? 3 * kFusedRowBlock : kRowBlock);
constexpr int kReduceFloats = 4 * (kPassPartials + kStepThreads);
constexpr int kMaxCacheRows = 1024;
constexpr std::size_t kMaxSharedPerCta = 113 * 1024; // two CTAs per SM
constexpr int kMaxLayers = 32;
constexpr int kProjections = 7;           // q, k, v, o, gate, up, down per layer
constexpr int kMaxSlices = kMaxLayers * kProjections + 1;

__device__ __forceinline__ float4 f4(float a, float b, float c, float d) {
  return make_float4(a, b, c, d);
}

__device__ __forceinline__ void fma4(float4 &acc, float a, const float4 &w) {
  acc.x = fmaf(a, w.x, acc.x);
  acc.y = fmaf(a, w.y, acc.y);
  acc.z = fmaf(a, w.z, acc.z);
  acc.w = fmaf(a, w.w, acc.w);
}

__device__ __forceinline__ float4 add4(const float4 &a, const float4 &b) {
  return f4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// ---- the projections ---------------------------------------------------------------------------
// One projection of the step as this CTA sees it: its column slice [o0, o0 + width) of a
// K x O row-major matrix.
struct Slice {
  const float *w;
  int K, O, o0, width;
};

// The step's slices in order (per layer q, k, v, o, gate, up, down; then the LM head).
struct StreamTable {
  Slice slices[kMaxSlices];
};

struct Cursor {
  int slice = 0;
};

__device__ Slice makeSlice(const float *w, int64_t K, int64_t O, int64_t o0, int64_t width) {
  Slice s;
  s.w = w;
  s.K = int(K);
  s.O = int(O);
  s.o0 = int(o0);
  s.width = int(width);
  return s;
}

// The next COUNT slices of the table (same K and width: q/k/v, or gate/up) applied to the same
// input: tile[c][r][4q .. 4q+3] = sum_k in[r][k] * W_c[k][o0 + 4q ..] for slice c < COUNT,
// r < rows and the quads q of the slices (slab of rows * width floats per slice).  Rows are
// taken in blocks of RB, each thread holding a float4 accumulator per (slice, row of its block)
// so that every weight load (straight from L2) serves all rows of the block; threads split the
// quads, the K rows and the row blocks, and the K partials reduce through shared memory in
// fixed-order levels.  For nq >= 256 a thread owns whole quads.  One out-of-line copy per
// COUNT serves every projection.
template <int COUNT, int RB>
__device__ __noinline__ void project(const StreamTable &t, Cursor &cur, const float *in, int ldIn,
                                     int rows, float *red, float *tile) {
  const int tid = threadIdx.x;
  const float4 *w0[COUNT];
  int nq = 0, K = 0;
  int64_t O4 = 0;
#pragma unroll
  for (int c = 0; c < COUNT; ++c) {
    const Slice sl = t.slices[cur.slice++];
    w0[c] = reinterpret_cast<const float4 *>(sl.w + sl.o0);
    nq = sl.width / 4;
    K = sl.K;
    O4 = sl.O / 4;
  }
  if (rows <= 0) // a CTA without rows in this projection (CTA-uniform)
    return;
  const int slab = rows * nq * 4;
  if (nq >= kStepThreads) {
    for (int rb = 0; rb < rows; rb += RB) {
      const int rr = rows - rb < RB ? rows - rb : RB;
      const float *x = in + rb * ldIn;
      for (int q = tid; q < nq; q += kStepThreads) {
        float4 acc[COUNT][RB];
#pragma unroll
        for (int c = 0; c < COUNT; ++c)
#pragma unroll
          for (int r = 0; r < RB; ++r)
            acc[c][r] = f4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
        for (int k = 0; k < K; ++k) {
#pragma unroll
          for (int c = 0; c < COUNT; ++c) {
            const float4 wk = __ldg(w0[c] + k * O4 + q);
#pragma unroll
            for (int r = 0; r < RB; ++r)
              if (r < rr)
                fma4(acc[c][r], x[r * ldIn + k], wk);
          }
        }
#pragma unroll
        for (int c = 0; c < COUNT; ++c)
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < rr)
              *reinterpret_cast<float4 *>(tile + c * slab + ((rb + r) * nq + q) * 4) = acc[c][r];
      }
    }
    __syncthreads();
    return;
  }
  // Row blocks of RB rows are handled side by side (`together` per pass, as many as keep at
  // least four K slices per output), and K is split kparts ways with at least two K rows per
  // slice (fewer partials to reduce).  Thread t owns quad t % nq, K slice (t / nq) % kparts and
  // row block t / (nq * kparts) of the pass.
  const int blocks = (rows + RB - 1) / RB;
  int together = blocks;
  while (together > 1 && nq * together * 4 > kStepThreads)
    --together;
  int kparts = kStepThreads / (nq * together);
  while (kparts > 1 && kparts * 2 > K)
    kparts >>= 1;
  const int q = tid % nq, kp = (tid / nq) % kparts, blk = tid / (nq * kparts);
  for (int rb = 0; rb < rows; rb += RB * together) {
    const int passRows = rows - rb < RB * together ? rows - rb : RB * together;
    const int first = blk * RB;
    const int rr = passRows - first < RB ? passRows - first : RB;
    const bool busy = blk < together && rr > 0;
    const float *x = in + (rb + first) * ldIn;
    float4 acc[COUNT][RB];
#pragma unroll
    for (int c = 0; c < COUNT; ++c)
#pragma unroll
      for (int r = 0; r < RB; ++r)
        acc[c][r] = f4(0.f, 0.f, 0.f, 0.f);
    // Long K ranges per thread (a CTA's slice of 64 KB or more, e.g. gate/up at hidden 256)
    // issue their weight loads in batches of BATCH K rows before any FMA of the batch: eight
    // loads in flight for single and fused pairs of slices instead of four.  The K rows still
    // accumulate in increasing order, so the sums are those of the short form.
    constexpr int BATCH = COUNT == 1 ? 8 : COUNT == 2 ? 4 : 2;
    const bool deep = (K + kparts - 1) / kparts >= 4 * BATCH; // CTA-uniform
    if (busy && deep) {
      int k = kp;
      for (; k + (BATCH - 1) * kparts < K; k += BATCH * kparts) {
        float4 wv[BATCH][COUNT];
#pragma unroll
        for (int u = 0; u < BATCH; ++u)
#pragma unroll
          for (int c = 0; c < COUNT; ++c)
            wv[u][c] = __ldg(w0[c] + (k + u * kparts) * O4 + q);
#pragma unroll
        for (int u = 0; u < BATCH; ++u)
#pragma unroll
          for (int c = 0; c < COUNT; ++c)
#pragma unroll
            for (int r = 0; r < RB; ++r)
              if (r < rr)
                fma4(acc[c][r], x[r * ldIn + k + u * kparts], wv[u][c]);
      }
      for (; k < K; k += kparts) {
#pragma unroll
        for (int c = 0; c < COUNT; ++c) {
          const float4 wk = __ldg(w0[c] + k * O4 + q);
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < rr)
              fma4(acc[c][r], x[r * ldIn + k], wk);
        }
      }
    } else if (busy) {
      // Loads in flight per thread: four K rows for a single slice, two for the fused passes.
#pragma unroll(COUNT == 1 ? 4 : 2)
      for (int k = kp; k < K; k += kparts) {
#pragma unroll
        for (int c = 0; c < COUNT; ++c) {
          const float4 wk = __ldg(w0[c] + k * O4 + q);
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < rr)
              fma4(acc[c][r], x[r * ldIn + k], wk);
        }
      }
    }
    // Partials of every (K slice, output) to shared memory, then a fixed-order sum: one level
    // for a few K slices per output, else segments of K slices and then the segments (no warp
    // shuffles: the shuffle pipe is the scarcer resource here).
    const int per = passRows * nq, outputs = COUNT * per;
    float4 *partial = reinterpret_cast<float4 *>(red);
    if (busy)
#pragma unroll
      for (int c = 0; c < COUNT; ++c)
#pragma unroll
        for (int r = 0; r < RB; ++r)
          if (r < rr)
            partial[kp * outputs + c * per + (first + r) * nq + q] = acc[c][r];
    __syncthreads();
    int segments = 1; // about sqrt(kparts): both levels sum a few terms each
    while (outputs * segments * 2 <= kStepThreads && segments * segments < kparts)
      segments *= 2;
    const int span = (kparts + segments - 1) / segments; // K slices per segment (last: fewer)
    float4 *level = partial + kparts * outputs;
    if (segments > 1) {
      if (tid < outputs * segments) {
        const int o = tid % outputs, seg = tid / outputs;
        const int lo = seg * span, hi = lo + span < kparts ? lo + span : kparts;
        float4 v = f4(0.f, 0.f, 0.f, 0.f);
        if (lo < hi) {
          v = partial[lo * outputs + o];
          for (int j = lo + 1; j < hi; ++j)
            v = add4(v, partial[j * outputs + o]);
        }
        level[seg * outputs + o] = v;
      }
      __syncthreads();
    }
    const float4 *terms = segments > 1 ? level : partial;
    const int count = segments > 1 ? segments : kparts;
    for (int e = tid; e < outputs; e += kStepThreads) {
      float4 v = terms[e];
      for (int g = 1; g < count; ++g)
        v = add4(v, terms[g * outputs + e]);
      const int c = e / per, o = e % per;
      *reinterpret_cast<float4 *>(tile + c * slab + (rb * nq + o) * 4) = v;
    }
    __syncthreads();
  }
}

// fn(r, column, value) for every (row, quad) of a projection tile.
template <class Fn>
__device__ __forceinline__ void eachQuad(int rows, int nq, int o0, const float *tile, Fn fn) {
  for (int e = threadIdx.x; e < rows * nq; e += kStepThreads)
    fn(e / nq, o0 + 4 * (e % nq), *reinterpret_cast<const float4 *>(tile + e * 4));
}

// act[g][:] = x[g][:] * rsqrt(mean(x[g]^2) + eps) * gain, one warp per row (row stride ld).
__device__ void rmsRows(const float *x, const float *gain, float *act, int rows, int C, int ld,
                        float eps) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  for (int g = warp; g < rows; g += kStepWarps) {
    float total = 0.f;
    for (int c = lane; c < C; c += kWarp) {
      const float v = x[g * ld + c];
      total += v * v;
    }
    total = warpSum(total);
    const float inv = rsqrtf(total / float(C) + eps);
    for (int c = lane; c < C; c += kWarp)
      act[g * ld + c] = __fmul_rn(__fmul_rn(x[g * ld + c], inv), gain[c]);
  }
  __syncthreads();
}

// Activation rows are padded by four floats so that the rows read together in a projection
// start in different shared-memory banks (and stay 16-byte aligned).
__host__ __device__ constexpr int64_t rowStride(int64_t columns) { return columns + 4; }

// Heads are partitioned over the cluster's CTAs: with A >= 8 heads CTA r owns the A / 8
// consecutive heads from r * A / 8 for every row; with fewer, CTA r owns head r % A for the rows
// of row group r / A (8 / A contiguous groups).  A CTA computes q, k and v of its heads, their
// attention and their part of the o projection without leaving its shared memory.
__host__ __device__ inline int64_t headsPerCta(const DecodeStepSpec &s) {
  return s.A >= kStepCtas ? s.A / kStepCtas : 1;
}
__host__ __device__ inline int64_t rowGroups(const DecodeStepSpec &s) {
  return s.A >= kStepCtas ? 1 : kStepCtas / s.A;
}
__host__ __device__ inline int64_t ownColumns(const DecodeStepSpec &s) {
  return headsPerCta(s) * s.D;
}

// Columns of one CTA's widest column-split projection output (fused q/k/v of its heads, fused
// gate/up, or the LM head).
__host__ __device__ inline int64_t tileColumns(const DecodeStepSpec &s) {
  int64_t widest = 3 * ownColumns(s);
  widest = widest > 2 * s.F / kStepCtas ? widest : 2 * s.F / kStepCtas;
  return widest > s.V / kStepCtas ? widest : s.V / kStepCtas;
}

constexpr std::size_t kTableBytes = (sizeof(StreamTable) + 15) / 16 * 16;

// x / act: the rows' residual stream and its normalization (full copies in every CTA);
// q / ctx: queries and attention outputs of the CTA's heads; h: the SwiGLU product of its FFN
// columns; partO / partD: its partial o and down projections [rows][C], which every CTA of the
// cluster reads (distributed shared memory) after the cluster barrier that follows them.
// operands: the RMSNorm gains of every layer and of the head, [norm1: L][norm2: L][final] x C,
// and the RoPE row of position p (D floats), copied in at the start of the step when they fit
// (operandsStaged).
struct StepBuffers {
  StreamTable *table;
  float *x, *act, *q, *ctx, *h, *partO, *partD, *red, *probs, *tile, *partValue, *first;
  int *partIndex;
  float *operands;
};

__device__ StepBuffers carve(unsigned char *base, const DecodeStepSpec &s) {
  StepBuffers b;
  const int64_t G = s.G, C = s.C;
  b.table = reinterpret_cast<StreamTable *>(base);
  b.x = reinterpret_cast<float *>(base + kTableBytes);
  b.act = b.x + G * rowStride(C);
  b.q = b.act + G * rowStride(C);
  b.ctx = b.q + G * rowStride(ownColumns(s));
  b.h = b.ctx + G * rowStride(ownColumns(s));
  b.partO = b.h + G * rowStride(s.F / kStepCtas);
  b.partD = b.partO + G * C;
  b.red = b.partD + G * C;
  b.probs = b.red + kReduceFloats;
  b.tile = b.probs + kStepWarps * s.T;
  b.partValue = b.tile + G * tileColumns(s);
  b.partIndex = reinterpret_cast<int *>(b.partValue + kStepCtas * kMaxRows);
  b.first = reinterpret_cast<float *>(b.partIndex + kStepCtas * kMaxRows);
  b.operands = b.first + kStepCtas * kMaxRows; // every region above is a multiple of 4 floats
  return b;
}

__host__ __device__ inline std::size_t baseSharedBytes(const DecodeStepSpec &s) {
  const int64_t floats = 2 * s.G * rowStride(s.C) + 2 * s.G * rowStride(ownColumns(s)) +
                         s.G * rowStride(s.F / kStepCtas) + 2 * s.G * s.C + kReduceFloats +
                         kStepWarps * s.T +
                         s.G * tileColumns(s) + 3 * kStepCtas * kMaxRows;
  return kTableBytes + std::size_t(floats) * sizeof(float);
}

// The step's gains and RoPE row in shared memory: each phase that uses them (the RMSNorms, the
// RoPE of q and k) then reads shared memory instead of making an L2 round trip; staged when
// they are at most 16 KB and fit the per-CTA budget.
__host__ __device__ inline int64_t operandFloats(const DecodeStepSpec &s) {
  return (2 * s.L + 1) * s.C + s.D;
}
__host__ __device__ inline bool operandsStaged(const DecodeStepSpec &s) {
  const std::size_t bytes = std::size_t(operandFloats(s)) * sizeof(float);
  return bytes <= 16 * 1024 && baseSharedBytes(s) + bytes <= kMaxSharedPerCta;
}

std::size_t stepSharedBytes(const DecodeStepSpec &s) {
  return baseSharedBytes(s) +
         (operandsStaged(s) ? std::size_t(operandFloats(s)) * sizeof(float) : 0);
}

// OCC CTAs per SM.  Two (at most 128 registers a thread and half of an SM's shared memory each)
// for wide grids: with one CTA per SM only about 15 eight-CTA clusters fit on the GPU at once,
// with two 33, so grids of up to 32 clusters run in one wave.  One (up to 255 registers, no
// spills) for grids of a few clusters, which are co-resident either way.
template <int OCC>
__global__ void __cluster_dims__(kStepCtas, 1, 1) __launch_bounds__(kStepThreads, OCC)
    decodeStepKernel(int *tokens, int *position, int *history, const float *emb,
                     const float *norm1, const float *norm2, const float *finalNorm,
                     const float *wq, const float *wk, const float *wv, const float *wo,
                     const float *wg, const float *wu, const float *wd, const float *lm,
                     const float *sincos, float *kc, float *vc, float *logits, unsigned *counter,
                     float eps, float scale, DecodeStepSpec s) {
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = int(cluster.block_rank());
  const int tid = threadIdx.x, lane = tid % kWarp, warp = tid / kWarp;
  extern __shared__ float4 sharedRaw[];
  const StepBuffers sb = carve(reinterpret_cast<unsigned char *>(sharedRaw), s);
  StreamTable &table = *sb.table;
  const int64_t B = s.B, C = s.C, A = s.A, D = s.D, F = s.F, V = s.V, T = s.T;
  const int64_t r0 = int64_t(blockIdx.x / kStepCtas) * s.G;
  const int rows = int(s.G < B - r0 ? s.G : B - r0);
  const int64_t own = ownColumns(s), hpc = headsPerCta(s);
  const int head0 = int(A >= kStepCtas ? rank * hpc : rank % A);
  const int64_t hc0 = head0 * D; // first column of the CTA's heads
  const int groupRows = int((rows + rowGroups(s) - 1) / rowGroups(s));
  const int group = int(A >= kStepCtas ? 0 : rank / A);
  const int gFirst = group * groupRows < rows ? group * groupRows : rows;
  const int gCount = rows - gFirst < groupRows ? rows - gFirst : groupRows;
  const int ldC = int(rowStride(C)), ldO = int(rowStride(own)), ldH = int(rowStride(F / kStepCtas));
  const int p = position[0];
  const bool inside = p >= 0 && p < T;
  // Every CTA of the cluster has read the position before any of them can finish (and so
  // before the last cluster can advance it).
  cluster.sync();

  Cursor cur;
  if (inside) {
    // The step's weight slices in consumption order: per layer q, k, v (the columns of the
    // CTA's heads), o (the rows of its heads, all columns), gate, up (its FFN columns), down
    // (the rows of its FFN columns, all columns); then the LM head (its vocabulary columns).
    const int count = int(s.L) * kProjections + 1;
    for (int i = tid; i < count; i += kStepThreads) {
      const int64_t l = i / kProjections, fr = F / kStepCtas;
      Slice sl;
      switch (i == count - 1 ? -1 : i % kProjections) {
      case 0: sl = makeSlice(wq + l * C * C, C, C, hc0, own); break;
      case 1: sl = makeSlice(wk + l * C * C, C, C, hc0, own); break;
      case 2: sl = makeSlice(wv + l * C * C, C, C, hc0, own); break;
      case 3: sl = makeSlice(wo + l * C * C + hc0 * C, own, C, 0, C); break;
      case 4: sl = makeSlice(wg + l * C * F, C, F, rank * fr, fr); break;
      case 5: sl = makeSlice(wu + l * C * F, C, F, rank * fr, fr); break;
      case 6: sl = makeSlice(wd + l * F * C + rank * fr * C, fr, C, 0, C); break;
      default:
        sl = makeSlice(lm + s.headLayer * C * V, C, V, rank * (V / kStepCtas), V / kStepCtas);
        break;
      }
      table.slices[i] = sl;
    }
    __syncthreads();

    // Gains and the RoPE row copied in behind the embedding gather (C, D multiples of 4; the
    // fused plan's buffers are 16-byte aligned).
    const bool staged = operandsStaged(s);
    float *op = sb.operands;
    if (staged) {
      const int64_t LC4 = s.L * C / 4;
      for (int64_t e = tid; e < LC4; e += kStepThreads) {
        copyAsync16(op + 4 * e, norm1 + 4 * e);
        copyAsync16(op + s.L * C + 4 * e, norm2 + 4 * e);
      }
      for (int64_t e = tid; e < C / 4; e += kStepThreads)
        copyAsync16(op + 2 * s.L * C + 4 * e, finalNorm + s.finalLayer * C + 4 * e);
      for (int64_t e = tid; e < D / 4; e += kStepThreads)
        copyAsync16(op + (2 * s.L + 1) * C + 4 * e, sincos + int64_t(p) * D + 4 * e);
      copyAsyncCommit();
    }

    for (int64_t e = tid; e < rows * C; e += kStepThreads) {
      const int64_t g = e / C, c = e % C;
      const int token = tokens[r0 + g];
      sb.x[g * ldC + c] = token >= 0 && token < V ? emb[int64_t(token) * C + c] : 0.f;
    }
    if (staged)
      copyAsyncWaitAll(); // this thread's copies; the barrier publishes everyone's
    __syncthreads();

    const int nqO = int(own / 4), nqF = int(F / kStepCtas / 4);
    const int oF = rank * int(F / kStepCtas);
    const int64_t R = D / 2;
    const float *cs = staged ? op + (2 * s.L + 1) * C : sincos + int64_t(p) * R * 2;
    auto rope = [&](int col, float4 v) {
      const int d = int(col % D);
      const float c0 = cs[(d / 2) * 2], s0 = cs[(d / 2) * 2 + 1];
      const float c1 = cs[(d / 2 + 1) * 2], s1 = cs[(d / 2 + 1) * 2 + 1];
      return f4(__fsub_rn(__fmul_rn(v.x, c0), __fmul_rn(v.y, s0)),
                __fadd_rn(__fmul_rn(v.x, s0), __fmul_rn(v.y, c0)),
                __fsub_rn(__fmul_rn(v.z, c1), __fmul_rn(v.w, s1)),
                __fadd_rn(__fmul_rn(v.z, s1), __fmul_rn(v.w, c1)));
    };
    // After the cluster barrier that follows a partial projection: x[r] += the sum of the
    // partials [row][C] of the CTAs holding row r, in rank order (every CTA computes the same
    // sums for all rows, so the copies stay identical).  `byHead`: the o projection, whose
    // partials come from the CTAs of the row's group when heads are split by row group.
    auto gather = [&](float *part, bool byHead) {
      const int c4n = int(C / 4);
      for (int e = tid; e < rows * c4n; e += kStepThreads) {
        const int r = e / c4n, c = 4 * (e % c4n);
        int first = 0, ctas = kStepCtas, local = r;
        if (byHead && A < kStepCtas) {
          const int gr = r / groupRows;
          first = gr * int(A);
          ctas = int(A);
          local = r - gr * groupRows;
        }
        float *at = part + int64_t(local) * C + c;
        float4 sum = *reinterpret_cast<const float4 *>(cluster.map_shared_rank(at, first));
        for (int j = 1; j < ctas; ++j)
          sum = add4(sum, *reinterpret_cast<const float4 *>(cluster.map_shared_rank(at, first + j)));
        float4 *x = reinterpret_cast<float4 *>(sb.x + r * ldC + c);
        const float4 old = *x;
        *x = f4(__fadd_rn(old.x, sum.x), __fadd_rn(old.y, sum.y), __fadd_rn(old.z, sum.z),
                __fadd_rn(old.w, sum.w));
      }
      __syncthreads();
    };
    for (int64_t l = 0; l < s.L; ++l) {
      auto cacheSlot = [&](float *cache, int r, int col) {
        const int64_t b = r0 + r, h = col / D, d = col % D;
        return reinterpret_cast<float4 *>(cache + (((l * B + b) * A + h) * T + p) * D + d);
      };
      // Attention block of the CTA's heads over its row group: norm, q/k/v in one pass (tile
      // slabs q | k | v), RoPE, cache append; no exchange with the other CTAs.
      rmsRows(sb.x + gFirst * ldC, staged ? op + l * C : norm1 + l * C, sb.act + gFirst * ldC,
              gCount, int(C), ldC, eps);
      project<3, kFusedRowBlock>(table, cur, sb.act + gFirst * ldC, ldC, gCount, sb.red, sb.tile);
      const int slabO = gCount * nqO * 4;
      eachQuad(gCount, nqO, int(hc0), sb.tile, [&](int r, int col, float4 v) {
        *reinterpret_cast<float4 *>(sb.q + (gFirst + r) * ldO + (col - hc0)) = rope(col, v);
      });
      eachQuad(gCount, nqO, int(hc0), sb.tile + slabO, [&](int r, int col, float4 v) {
        *cacheSlot(kc, gFirst + r, col) = rope(col, v);
      });
      eachQuad(gCount, nqO, int(hc0), sb.tile + 2 * slabO,
               [&](int r, int col, float4 v) { *cacheSlot(vc, gFirst + r, col) = v; });
      __syncthreads(); // this CTA's cache rows at p and queries are in place

      // Attention: every (row, head) pair of the CTA gets `wp` warps, which split its cache
      // rows 0..p into contiguous chunks; the chunks' maxima combine before the exponentials,
      // their sums and value sums after, in warp order (shared memory).
      {
        const int64_t n = int64_t(p) + 1;
        const int pairs = gCount * int(hpc);
        int wp = 1;
        while (wp < kStepWarps && pairs * wp * 2 <= kStepWarps)
          wp *= 2;
        const int lead = warp - warp % wp, member = warp % wp;
        const int perRound = kStepWarps / wp;
        const int64_t chunk = (n + wp - 1) / wp;
        const int64_t lo = member * chunk, hi = lo + chunk < n ? lo + chunk : n;
        const int quads = int(D / 4), subs = kWarp / quads;
        const int dq = lane % quads, sub = lane / quads;
        float *probs = sb.probs + warp * T;
        float *stats = sb.red;                  // per warp: chunk maximum, chunk sum
        float *values = sb.red + 2 * kStepWarps; // per warp: D partial value sums
        // Uniform trip count over the CTA (its barriers are reached by every warp).
        for (int base = 0; base < pairs; base += perRound) {
          const int pair = base + warp / wp;
          const bool active = pair < pairs;
          const int g = active ? gFirst + pair / int(hpc) : 0;
          const int hh = active ? pair % int(hpc) : 0;
          const int64_t cacheBase = ((l * B + r0 + g) * A + head0 + hh) * T * D;
          if (active) {
            // Scores: `quads` lanes per cache row (one float4 each), `subs` rows at a time.
            const float4 q4 = *reinterpret_cast<const float4 *>(sb.q + g * ldO + hh * D + 4 * dq);
            float best = -CUDART_INF_F;
            const float4 *krows = reinterpret_cast<const float4 *>(kc + cacheBase) + dq;
            for (int64_t t0 = lo + sub; t0 - sub < hi; t0 += 4 * subs) {
              float4 kv[4]; // four rows' loads in flight per lane
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int64_t t = t0 + u * subs;
                kv[u] = t < hi ? __ldcg(krows + t * quads) : f4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int64_t t = t0 + u * subs;
                float dot = 0.f;
                dot = fmaf(q4.x, kv[u].x, dot);
                dot = fmaf(q4.y, kv[u].y, dot);
                dot = fmaf(q4.z, kv[u].z, dot);
                dot = fmaf(q4.w, kv[u].w, dot);
                for (int o = 1; o < quads; o <<= 1)
                  dot += __shfl_xor_sync(0xffffffffu, dot, o);
                if (t < hi) {
                  const float score = dot * scale;
                  if (dq == 0)
                    probs[t] = score;
                  best = fmaxf(best, score);
                }
              }
            }
            best = warpMax(best);
            if (lane == 0)
              stats[2 * warp] = best;
          }
          __syncthreads();
          if (active) {
            float top = stats[2 * lead];
            for (int j = 1; j < wp; ++j)
              top = fmaxf(top, stats[2 * (lead + j)]);
            float total = 0.f;
            for (int64_t t = lo + lane; t < hi; t += kWarp) {
              const float e = expf(probs[t] - top);
              probs[t] = e;
              total += e;
            }
            total = warpSum(total);
            __syncwarp();
            // Value sums: lane (dq, sub) accumulates quad dq over rows sub, sub + subs, ...
            float4 acc = f4(0.f, 0.f, 0.f, 0.f);
            const float4 *vrows = reinterpret_cast<const float4 *>(vc + cacheBase) + dq;
            for (int64_t t0 = lo + sub; t0 - sub < hi; t0 += 4 * subs) {
              float4 v[4]; // four rows' loads in flight per lane
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int64_t t = t0 + u * subs;
                v[u] = t < hi ? __ldcg(vrows + t * quads) : f4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < 4; ++u)
                if (t0 + u * subs < hi)
                  fma4(acc, probs[t0 + u * subs], v[u]);
            }
            for (int o = quads; o < kWarp; o <<= 1) {
              acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
              acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
              acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
              acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
            }
            if (sub == 0)
              *reinterpret_cast<float4 *>(values + warp * D + 4 * dq) = acc;
            if (lane == 0)
              stats[2 * warp + 1] = total;
          }
          __syncthreads();
          if (active) {
            float total = stats[2 * lead + 1];
            for (int j = 1; j < wp; ++j)
              total += stats[2 * (lead + j) + 1];
            for (int64_t d = member * kWarp + lane; d < D; d += wp * kWarp) {
              float v = values[lead * D + d];
              for (int j = 1; j < wp; ++j)
                v += values[(lead + j) * D + d];
              sb.ctx[g * ldO + hh * D + d] = v / total;
            }
          }
          __syncthreads();
        }
      }

      // o projection of the CTA's heads (K = their columns, all C outputs) as a partial sum;
      // then every CTA adds the partials of all heads to its copy of the residual stream.
      project<1, kRowBlock>(table, cur, sb.ctx + gFirst * ldO, ldO, gCount, sb.red, sb.partO);
      cluster.sync();
      gather(sb.partO, true);

      // MLP: gate and up of the CTA's FFN columns in one pass with the SwiGLU product, then
      // the down projection of those columns (K = F / 8, all C outputs) as a partial sum.
      rmsRows(sb.x, staged ? op + (s.L + l) * C : norm2 + l * C, sb.act, rows, int(C), ldC, eps);
      project<2, kFusedRowBlock>(table, cur, sb.act, ldC, rows, sb.red, sb.tile);
      const int slabF = rows * nqF * 4;
      eachQuad(rows, nqF, oF, sb.tile, [&](int r, int col, float4 gate) {
        const float4 up = *reinterpret_cast<const float4 *>(sb.tile + slabF + (r * nqF + (col - oF) / 4) * 4);
        auto act = [](float gv, float uv) { return __fmul_rn(gv / (1.0f + expf(-gv)), uv); };
        *reinterpret_cast<float4 *>(sb.h + r * ldH + (col - oF)) =
            f4(act(gate.x, up.x), act(gate.y, up.y), act(gate.z, up.z), act(gate.w, up.w));
      });
      __syncthreads();
      project<1, kRowBlock>(table, cur, sb.h, ldH, rows, sb.red, sb.partD);
      cluster.sync();
      gather(sb.partD, false);
    }

    // Head: final norm, logits of this CTA's vocabulary columns and their per-row maximum.
    rmsRows(sb.x, staged ? op + 2 * s.L * C : finalNorm + s.finalLayer * C, sb.act, rows, int(C),
            ldC, eps);
    const int64_t Wv = V / kStepCtas;
    const int oV = rank * int(Wv);
    project<1, kRowBlock>(table, cur, sb.act, ldC, rows, sb.red, sb.tile);
    eachQuad(rows, int(Wv / 4), oV, sb.tile, [&](int r, int col, float4 v) {
      *reinterpret_cast<float4 *>(logits + (r0 + r) * V + col) = v;
    });
    for (int r = warp; r < rows; r += kStepWarps) {
      float best = -CUDART_INF_F;
      int index = 0x7fffffff;
      for (int64_t j = lane; j < Wv; j += kWarp)
        argmaxMerge(best, index, sb.tile[r * Wv + j], int(oV + j));
#pragma unroll
      for (int o = kWarp / 2; o > 0; o >>= 1)
        argmaxMerge(best, index, __shfl_xor_sync(0xffffffffu, best, o),
                    __shfl_xor_sync(0xffffffffu, index, o));
      if (lane == 0) {
        *cluster.map_shared_rank(sb.partValue + rank * kMaxRows + r, 0) = best;
        *cluster.map_shared_rank(sb.partIndex + rank * kMaxRows + r, 0) = index;
        if (rank == 0)
          sb.first[r] = sb.tile[r * Wv];
      }
    }
    cluster.sync();
    if (rank == 0) {
      for (int g = tid; g < rows; g += kStepThreads) {
        float best = -CUDART_INF_F;
        int index = 0x7fffffff;
        for (int k = 0; k < kStepCtas; ++k)
          argmaxMerge(best, index, sb.partValue[k * kMaxRows + g], sb.partIndex[k * kMaxRows + g]);
        const float first = sb.first[g];
        if (first != first || index == 0x7fffffff)
          index = 0; // a NaN first score wins the reference's strict scan outright
        tokens[r0 + g] = index;
        history[int64_t(p) * B + r0 + g] = index;
      }
    }
  }
  // The last cluster to finish advances the position (clusters never wait for each other).
  if (rank == 0) {
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const unsigned done = atomicAdd(counter, 1u);
      if (done == unsigned(s.clusters) - 1) {
        position[0] = p + 1;
        atomicExch(counter, 0u);
        __threadfence();
      }
    }
  }
}

bool decodeStepGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<DecodeStepSpec>(spec);
  // Column quads per CTA: below 256 (threads split K) or a multiple of 256 (whole quads per
  // thread).
  auto quadsOk = [](int64_t columns) {
    if (columns <= 0 || columns % (kStepCtas * 4))
      return false;
    const int64_t nq = columns / (kStepCtas * 4);
    return nq < kStepThreads || nq % kStepThreads == 0;
  };
  // Head dimension: a power of two up to 128 (one float4 per lane across a cache row); head
  // count: a power of two (the heads split evenly over the 8 CTAs, or the CTAs over the heads).
  if (s.B <= 0 || s.L <= 0 || s.L > kMaxLayers || s.A <= 0 || (s.A & (s.A - 1)) || s.D < 4 ||
      s.D > 128 || (s.D & (s.D - 1)) || s.A * s.D != s.C)
    return false;
  if (!quadsOk(s.C) || !quadsOk(s.F) || !quadsOk(s.V) || s.T <= 0 || s.T > kMaxCacheRows)
    return false;
  if (s.G <= 0 || s.G > kMaxRows || s.clusters <= 0 || s.clusters * s.G < s.B ||
      (s.clusters - 1) * s.G >= s.B)
    return false;
  if (s.L > s.weightLayers || s.L > s.normLayers || s.finalLayer < 0 || s.headLayer < 0)
    return false;
  const std::size_t bytes = stepSharedBytes(s);
  if (bytes > kMaxSharedPerCta)
    return false;
  g->grid[0] = unsigned(s.clusters * kStepCtas);
  g->block[0] = kStepThreads;
  g->sharedBytes = unsigned(bytes);
  return true;
}

// Grids of up to this many clusters run the one-CTA-per-SM build (measured at one request,
// C = 64, two layers: 41 us per step against 45 us for the two-CTA build).
constexpr int64_t kWideRegisterClusters = 12;

const void *decodeStepSelect(const void *spec) {
  return specOf<DecodeStepSpec>(spec).clusters <= kWideRegisterClusters
             ? reinterpret_cast<const void *>(&decodeStepKernel<1>)
             : reinterpret_cast<const void *>(&decodeStepKernel<2>);
}

} // namespace

CKL_REGISTER_KERNEL("ckl.fused.decode_step", reinterpret_cast<const void *>(&decodeStepKernel<2>),
                    "PPPPPPPPPPPPPPPPPPPPFFS", sizeof(DecodeStepSpec), decodeStepGeometry,
                    decodeStepSelect, nullptr, 0, false);


} // namespace ckl::kernels
