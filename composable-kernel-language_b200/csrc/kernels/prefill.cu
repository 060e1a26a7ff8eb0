// Batched prompt prefill for the decoder (the reference prefills by replaying the decode step
// once per prompt token with the next prompt token forced, benchmarks/decoder/reference.py:98-108).
//
// A prefill chunk processes P prompt positions of all B requests at once: row m of every
// chunk-sized activation is request m % B at position position[0] + m / B.  The projections are
// the tensor-core panel kernels (their RoPE / KV-append epilogues place each row at its own
// position, and an argmax-only head produces the greedy token of every row); the kernels here
// are the rest of the chunk:
//   prefill.embedding: rows from the prompts buffer [T, B];
//   prefill.attention: causal flash attention of the chunk's queries over the KV cache rows
//     0..position (earlier chunks and this chunk's appends), written as the o projection's panel;
//   prefill.history:   the greedy token of each row into history[position, request];
//   prefill.advance:   position[0] += P once the chunk is done.
#include "ckl_b200.h"
#include "common.cuh"
#include "panel.cuh"

namespace ckl::kernels {
namespace {

// ---- embedding -----------------------------------------------------------------------------
// Rows whose prompt token lies outside the table are left unwritten, like the decode step's.
__global__ void prefillEmbeddingKernel(const int *prompts, const int *position, const float *table,
                                       float *dst, PrefillRowsSpec s) {
  const int64_t p0 = position[0];
  const int64_t total = s.M * s.C;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = e / s.C, c = e % s.C;
    const int64_t at = p0 + m / s.B;
    if (at < 0 || at >= s.T)
      continue;
    const int token = prompts[at * s.B + m % s.B];
    if (token >= 0 && token < s.V)
      dst[e] = table[int64_t(token) * s.C + c];
  }
}

bool prefillEmbeddingGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<PrefillRowsSpec>(spec);
  if (s.M <= 0 || s.B <= 0 || s.C <= 0 || s.V <= 0 || s.T <= 0)
    return false;
  const int64_t wanted = ceilDiv(s.M * s.C, 256 * 4);
  g->grid[0] = unsigned(wanted < 148 * 16 ? wanted : 148 * 16);
  g->block[0] = 256;
  return true;
}

// ---- causal attention over the cache ---------------------------------------------------------
// One CTA of 128 threads per (request, head, block of QB chunk positions).  Keys stream through
// shared memory KB rows at a time from 0 to the block's last position.  Thread (quad, lane)
// owns queries 4 quad .. 4 quad + 3.  Scores: it accumulates those 4 queries x keys lane,
// lane + 16, lane + 32, lane + 48 over the head dimension in float4 steps (rows padded to D + 4
// floats, so a warp's 16-byte key loads hit distinct banks and its query loads broadcast); each
// query row keeps an online softmax (running maximum and normaliser, shared by the 16 threads
// of the row's quad through shuffles) with keys after the query's own position masked.  The
// probabilities go to shared memory key-major, so the value pass reads a query quad's four with
// one 16-byte load; there the thread owns the same 4 queries x float4 groups lane, lane + 16 ..
// of the head dimension.  FFMA throughout.
constexpr int kPrefillQueries = 32;
constexpr int kPrefillKeys = 64;
constexpr int kPrefillThreads = 128;
constexpr int kPrefillGroup = 16; // threads sharing a query quad

template <int D> struct PrefillSmem {
  float q[kPrefillQueries][D + 4];
  float k[kPrefillKeys][D + 4];
  float4 v[kPrefillKeys][D / 4];
  float p[kPrefillKeys][kPrefillQueries + 4]; // probabilities, key-major
};

// 16-byte asynchronous copy global -> shared that zero-fills the destination instead when
// `valid` is false (no bytes are read then), and waits for all but the newest `N` groups.
__device__ __forceinline__ void copyAsync16OrZero(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<unsigned>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(valid ? 16u : 0u)
               : "memory");
}
template <int N> __device__ __forceinline__ void copyAsyncWaitAllBut() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kPrefillThreads)
    prefillAttentionKernel(const float *q, const float *kc, const float *vc, const int *position,
                           float *ctx, float scale, PrefillAttentionSpec s) {
  constexpr int QB = kPrefillQueries, KB = kPrefillKeys, TG = kPrefillGroup;
  constexpr int G = D / 4;               // float4 groups of a row
  constexpr int KPT = KB / TG;           // keys per thread (4), 16 apart
  constexpr int GPT = (G + TG - 1) / TG; // value groups per thread
  extern __shared__ __align__(16) unsigned char raw[];
  auto &sm = *reinterpret_cast<PrefillSmem<D> *>(raw);

  const int64_t blocks = (s.P + QB - 1) / QB;
  const int64_t qb = blockIdx.x % blocks, bh = blockIdx.x / blocks;
  const int64_t h = bh % s.A, b = bh / s.A;
  const int64_t C = s.A * D, i0 = qb * QB;
  const int64_t p0 = position[0];
  const int tid = threadIdx.x, quad = tid / TG, lane16 = tid % TG;

  for (int e = tid; e < QB * G; e += kPrefillThreads) {
    const int i = e / G, g = e % G;
    float4 value = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i0 + i < s.P) {
      const float *src = q + ((i0 + i) * s.B + b) * C + h * D + 4 * g;
      value = make_float4(src[0], src[1], src[2], src[3]);
    }
    *reinterpret_cast<float4 *>(&sm.q[i][4 * g]) = value;
  }
  bool live[4];
  int64_t mine[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    live[a] = i0 + 4 * quad + a < s.P;
    mine[a] = p0 + i0 + 4 * quad + a;
  }
  const int64_t lastLocal = (i0 + QB < s.P ? i0 + QB : s.P) - 1;
  int64_t last = p0 + lastLocal;
  if (last >= s.T)
    last = s.T - 1;
  const int64_t base = (((s.layer * s.B + b) * s.A + h) * s.T) * D;

  float m[4], l[4];
  float4 acc[4][GPT];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    m[a] = -CUDART_INF_F;
    l[a] = 0.f;
#pragma unroll
    for (int j = 0; j < GPT; ++j)
      acc[a][j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  // Keys and values stream through the same shared buffers with cp.async when the cache rows
  // start on 16-byte boundaries: the next block's keys are requested as soon as every thread
  // has read this block's keys (they load under the softmax and the value pass), the next
  // block's values as soon as the value pass is done (they load under the next score pass).
  // No second buffer (which would halve the CTAs per SM) and no registers hold them.
  const bool streamed = last >= 0 && aligned16(kc + base) && aligned16(vc + base);
  auto copyKeys = [&](int64_t from) {
    for (int e = tid; e < KB * G; e += kPrefillThreads) {
      const int r = e / G, g = e % G;
      const int64_t t = from + r;
      const bool valid = t <= last;
      copyAsync16OrZero(&sm.k[r][4 * g], kc + base + (valid ? t * D + 4 * g : 0), valid);
    }
  };
  auto copyValues = [&](int64_t from) {
    for (int e = tid; e < KB * G; e += kPrefillThreads) {
      const int r = e / G, g = e % G;
      const int64_t t = from + r;
      const bool valid = t <= last;
      copyAsync16OrZero(&sm.v[r][g], vc + base + (valid ? t * D + 4 * g : 0), valid);
    }
  };
  if (streamed) {
    copyKeys(0);
    copyValues(0);
    copyAsyncCommit();
  }

  for (int64_t t0 = 0; t0 <= last; t0 += KB) {
    const bool more = t0 + KB <= last; // uniform over the CTA
    if (streamed) {
      // This block's keys (group committed after the previous score pass, or the first group
      // with the first values) have landed; the newest group (values) may still be in flight.
      if (t0 == 0)
        copyAsyncWaitAllBut<0>();
      else
        copyAsyncWaitAllBut<1>();
      __syncthreads(); // every thread's copies visible (and the queries staged)
    } else {
    __syncthreads(); // previous block's keys and probabilities consumed (queries staged)
    for (int e = tid; e < KB * G; e += kPrefillThreads) {
      const int r = e / G, g = e % G;
      const int64_t t = t0 + r;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (t <= last) {
        const float *kr = kc + base + t * D + 4 * g, *vr = vc + base + t * D + 4 * g;
        if (aligned16(kr) && aligned16(vr)) {
          kv = *reinterpret_cast<const float4 *>(kr);
          vv = *reinterpret_cast<const float4 *>(vr);
        } else {
          kv = make_float4(kr[0], kr[1], kr[2], kr[3]);
          vv = make_float4(vr[0], vr[1], vr[2], vr[3]);
        }
      }
      *reinterpret_cast<float4 *>(&sm.k[r][4 * g]) = kv;
      sm.v[r][g] = vv;
    }
    __syncthreads();
    }
    float score[4][KPT];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int u = 0; u < KPT; ++u)
        score[a][u] = 0.f;
#pragma unroll 2
    for (int g = 0; g < G; ++g) {
      float4 qv[4], kv[KPT];
#pragma unroll
      for (int a = 0; a < 4; ++a)
        qv[a] = *reinterpret_cast<const float4 *>(&sm.q[4 * quad + a][4 * g]);
#pragma unroll
      for (int u = 0; u < KPT; ++u)
        kv[u] = *reinterpret_cast<const float4 *>(&sm.k[lane16 + TG * u][4 * g]);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int u = 0; u < KPT; ++u) {
          score[a][u] = fmaf(qv[a].x, kv[u].x, score[a][u]);
          score[a][u] = fmaf(qv[a].y, kv[u].y, score[a][u]);
          score[a][u] = fmaf(qv[a].z, kv[u].z, score[a][u]);
          score[a][u] = fmaf(qv[a].w, kv[u].w, score[a][u]);
        }
    }
    if (streamed) {
      __syncthreads(); // every thread has read this block's keys
      if (more) {
        copyKeys(t0 + KB);
        copyAsyncCommit();
      }
    }
    float correction[4], e[4][KPT];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float blockMax = -CUDART_INF_F;
#pragma unroll
      for (int u = 0; u < KPT; ++u) {
        const int64_t t = t0 + lane16 + TG * u;
        score[a][u] = live[a] && t <= mine[a] && t <= last ? score[a][u] * scale : -CUDART_INF_F;
        blockMax = fmaxf(blockMax, score[a][u]);
      }
#pragma unroll
      for (int o = 1; o < TG; o <<= 1)
        blockMax = fmaxf(blockMax, __shfl_xor_sync(0xffffffffu, blockMax, o));
      const float next = fmaxf(m[a], blockMax);
      correction[a] = m[a] == -CUDART_INF_F ? 0.f : expf(m[a] - next);
      float sum = 0.f;
#pragma unroll
      for (int u = 0; u < KPT; ++u) {
        e[a][u] = score[a][u] == -CUDART_INF_F ? 0.f : expf(score[a][u] - next);
        sum += e[a][u];
      }
#pragma unroll
      for (int o = 1; o < TG; o <<= 1)
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l[a] = l[a] * correction[a] + sum;
      m[a] = next;
    }
#pragma unroll
    for (int u = 0; u < KPT; ++u)
      *reinterpret_cast<float4 *>(&sm.p[lane16 + TG * u][4 * quad]) =
          make_float4(e[0][u], e[1][u], e[2][u], e[3][u]);
    __syncwarp(); // a quad's probabilities come from the 16 threads of this half-warp
    if (streamed) {
      // This block's values: all but the newest group (the next keys, if requested).
      if (more)
        copyAsyncWaitAllBut<1>();
      else
        copyAsyncWaitAllBut<0>();
      __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < GPT; ++j) {
      const int g = lane16 + TG * j;
      if (g >= G)
        continue;
      float4 r[4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
        r[a] = make_float4(acc[a][j].x * correction[a], acc[a][j].y * correction[a],
                           acc[a][j].z * correction[a], acc[a][j].w * correction[a]);
#pragma unroll 4
      for (int kj = 0; kj < KB; ++kj) {
        const float4 w = *reinterpret_cast<const float4 *>(&sm.p[kj][4 * quad]);
        const float4 v = sm.v[kj][g];
        const float ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          r[a].x = fmaf(ws[a], v.x, r[a].x);
          r[a].y = fmaf(ws[a], v.y, r[a].y);
          r[a].z = fmaf(ws[a], v.z, r[a].z);
          r[a].w = fmaf(ws[a], v.w, r[a].w);
        }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
        acc[a][j] = r[a];
    }
    if (streamed) {
      __syncthreads(); // every thread has read this block's values and probabilities
      if (more) {
        copyValues(t0 + KB);
        copyAsyncCommit();
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    if (!live[a] || mine[a] >= s.T)
      continue;
#pragma unroll
    for (int j = 0; j < GPT; ++j) {
      const int g = lane16 + TG * j;
      if (g >= G)
        continue;
      float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
      if (l[a] > 0.f)
        out = make_float4(acc[a][j].x / l[a], acc[a][j].y / l[a], acc[a][j].z / l[a],
                          acc[a][j].w / l[a]);
      panel::store4(ctx, (i0 + 4 * quad + a) * s.B + b, h * D + 4 * g, C, out);
    }
  }
}

bool prefillAttentionGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<PrefillAttentionSpec>(spec);
  if (s.B <= 0 || s.A <= 0 || s.T <= 0 || s.P <= 0 || s.layer < 0 || s.layer >= s.L)
    return false;
  std::size_t bytes = 0;
  switch (s.D) {
  case 16: bytes = sizeof(PrefillSmem<16>); break;
  case 32: bytes = sizeof(PrefillSmem<32>); break;
  case 64: bytes = sizeof(PrefillSmem<64>); break;
  case 128: bytes = sizeof(PrefillSmem<128>); break;
  default: return false;
  }
  const int64_t ctas = s.B * s.A * ((s.P + kPrefillQueries - 1) / kPrefillQueries);
  if (ctas >= (int64_t(1) << 31))
    return false;
  g->grid[0] = unsigned(ctas);
  g->block[0] = kPrefillThreads;
  g->sharedBytes = unsigned(bytes);
  return true;
}

const void *prefillAttentionSelect(const void *spec) {
  switch (specOf<PrefillAttentionSpec>(spec).D) {
  case 16: return reinterpret_cast<const void *>(&prefillAttentionKernel<16>);
  case 32: return reinterpret_cast<const void *>(&prefillAttentionKernel<32>);
  case 64: return reinterpret_cast<const void *>(&prefillAttentionKernel<64>);
  case 128: return reinterpret_cast<const void *>(&prefillAttentionKernel<128>);
  default: return nullptr;
  }
}

// ---- greedy tokens of the prompt positions --------------------------------------------------
// One warp per row: the first index of the row's maximum over its tiles' partials (the decode
// step's greedy rule) goes to history[position, request].
constexpr int kHistoryWarps = 8;

__global__ void __launch_bounds__(kHistoryWarps *kWarp)
    prefillHistoryKernel(const float2 *partials, const int *position, int *history,
                         PrefillHistorySpec s) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  const int64_t m = int64_t(blockIdx.x) * kHistoryWarps + warp;
  if (m >= s.M)
    return;
  float best = -CUDART_INF_F;
  int index = 0x7fffffff;
  for (int64_t t = lane; t < s.tiles; t += kWarp) {
    const float2 candidate = partials[m * s.tiles + t];
    argmaxMerge(best, index, candidate.x, __float_as_int(candidate.y));
  }
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1)
    argmaxMerge(best, index, __shfl_xor_sync(0xffffffffu, best, o),
                __shfl_xor_sync(0xffffffffu, index, o));
  const int64_t at = int64_t(position[0]) + m / s.B;
  if (lane == 0 && at >= 0 && at < s.T)
    history[at * s.B + m % s.B] = index;
}

bool prefillHistoryGeometry(const void *spec, std::size_t, library::Geometry *g) {
  const auto &s = specOf<PrefillHistorySpec>(spec);
  if (s.M <= 0 || s.B <= 0 || s.tiles <= 0 || s.T <= 0)
    return false;
  g->grid[0] = ceilDiv(s.M, kHistoryWarps);
  g->block[0] = kHistoryWarps * kWarp;
  return true;
}

__global__ void prefillAdvanceKernel(int *position, PositionAddSpec s) {
  position[0] = int(position[0] + s.delta);
}

bool prefillAdvanceGeometry(const void *spec, std::size_t, library::Geometry *g) {
  (void)specOf<PositionAddSpec>(spec);
  g->grid[0] = 1;
  g->block[0] = 1;
  return true;
}

} // namespace

CKL_REGISTER_KERNEL("ckl.prefill.embedding", reinterpret_cast<const void *>(&prefillEmbeddingKernel),
                    "PPPPS", sizeof(PrefillRowsSpec), prefillEmbeddingGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.prefill.attention",
                    reinterpret_cast<const void *>(&prefillAttentionKernel<64>), "PPPPPFS",
                    sizeof(PrefillAttentionSpec), prefillAttentionGeometry, prefillAttentionSelect);
CKL_REGISTER_KERNEL("ckl.prefill.history", reinterpret_cast<const void *>(&prefillHistoryKernel),
                    "PPPS", sizeof(PrefillHistorySpec), prefillHistoryGeometry, nullptr);
CKL_REGISTER_KERNEL("ckl.prefill.advance", reinterpret_cast<const void *>(&prefillAdvanceKernel),
                    "PS", sizeof(PositionAddSpec), prefillAdvanceGeometry, nullptr);

} // namespace ckl::kernels
