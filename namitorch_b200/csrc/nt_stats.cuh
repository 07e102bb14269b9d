// Statistics primitives shared by the gradient-statistics kernels (nt_stats.cu) and the
// fused ZeRO-1 reduce-scatter (nt_zero.cu): the per-block partial record, its workspace,
// the found_inf / norm finalisation and the per-value accumulators.
#pragma once

#include <cmath>

#include "nt_common.cuh"

namespace nt {

constexpr int kStatsThreads = 256;
constexpr int kUnroll = 4;  // 16-byte vectors in flight per thread
constexpr int kStatsMaxBlocks = 1024;
constexpr int kNoAllocChunk = 8192;

struct StatsPartial {
  double sumsq;
  double powsum;
  float maxabs;
  unsigned nonfinite;
  unsigned nan;
  unsigned pad;
};

struct StatsWorkspace {
  unsigned counter;
  unsigned pad[63];
  StatsPartial partials[kStatsMaxBlocks];
};

// Norm and found_inf from the reduced fields; the early returns follow _total_norm
// (namitorch/optim/clip_grad.py:63-79): a NaN / infinite / zero max|g| or p = inf returns
// max|g| itself. For p = 2 the norm is sqrt(sum g^2) (one read of the gradients); any
// other p uses max * (sum (|g|/max)^p)^(1/p) with the reference's log-space fallback.
__device__ inline void stats_finalize(nt_stats* s, double p) {
  s->found_inf = s->nonfinite > 0.0 ? 1.0 : 0.0;
  const double mx = s->maxabs;
  double norm;
  if (s->nan > 0.0) norm = __longlong_as_double(0x7ff8000000000000ll);
  else if (s->nonfinite > 0.0) norm = __longlong_as_double(0x7ff0000000000000ll);
  else if (mx == 0.0) norm = 0.0;
  else if (isinf(p)) norm = mx;
  else if (p == 2.0) norm = sqrt(s->sumsq);
  else {
    const double total = s->powsum;
    norm = mx * pow(total, 1.0 / p);
    if (!isfinite(norm)) norm = exp(log(mx) + log(total) / p);
  }
  s->norm = norm;
}

enum { kScaleNone = 0, kScaleMul = 1, kScaleDiv = 2 };

template <int MODE>
__device__ __forceinline__ float unscale_by(float g, float scale, float inv) {
  if constexpr (MODE == kScaleNone) return g;
  else if constexpr (MODE == kScaleMul) return __fmul_rn(g, inv);
  else return __fdiv_rn(g, scale);
}

struct StatsAcc {
  double ss0, ss1, ps;
  float mx;
  unsigned nf, nn;
};

// One value the slow way: non-finite values are counted, finite ones accumulated.
__device__ __forceinline__ void stats_one(float u, StatsAcc& a) {
  const float m = fabsf(u);
  a.mx = fmaxf(a.mx, m);  // fmaxf skips NaN
  if (m <= 3.402823466e38f) {
    const double d = (double)u;
    a.ss0 = fma(d, d, a.ss0);  // u*u is exact in double
  } else {
    ++a.nf;
    if (u != u) ++a.nn;
  }
}

template <int N>
__device__ __forceinline__ void stats_pass0(const float* u, StatsAcc& a) {
  float m = fabsf(u[0]);
#pragma unroll
  for (int q = 1; q < N; ++q) m = max_nan(m, fabsf(u[q]));
  if (m <= 3.402823466e38f) {  // every value finite (a NaN makes m NaN)
    a.mx = fmaxf(a.mx, m);
#pragma unroll
    for (int q = 0; q < N; ++q) {
      const double d = (double)u[q];  // u*u is exact in double
      if (q & 1) a.ss1 = fma(d, d, a.ss1);
      else a.ss0 = fma(d, d, a.ss0);
    }
  } else {
#pragma unroll
    for (int q = 0; q < N; ++q) stats_one(u[q], a);
  }
}

// Reduces the per-block partials (fixed order) into the pass-0 fields of `st` once every
// block has stored its own; returns true in the block that did it.
template <int THREADS = kStatsThreads>
__device__ __forceinline__ bool stats_reduce_pass0(const StatsAcc& a, StatsWorkspace* ws, nt_stats* st) {
  __shared__ double red_d[THREADS / 32];
  __shared__ float red_f[THREADS / 32];
  __shared__ unsigned red_u[THREADS / 32];
  __shared__ bool last;
  double ss = block_reduce(a.ss0 + a.ss1, red_d, SumOp(), 0.0);
  float mx = block_reduce(a.mx, red_f, MaxOp(), 0.0f);
  unsigned nf = block_reduce(a.nf, red_u, SumOp(), 0u);
  unsigned nn = block_reduce(a.nn, red_u, SumOp(), 0u);
  if (threadIdx.x == 0) {
    StatsPartial& out = ws->partials[blockIdx.x];
    out.sumsq = ss; out.powsum = 0.0; out.maxabs = mx; out.nonfinite = nf; out.nan = nn;
  }
  if (!last_block_ticket(&ws->counter, &last)) return false;
  ss = 0.0; mx = 0.0f;
  double nfd = 0.0, nnd = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    const StatsPartial q = ws->partials[b];
    ss += q.sumsq; mx = fmaxf(mx, q.maxabs); nfd += q.nonfinite; nnd += q.nan;
  }
  ss = block_reduce(ss, red_d, SumOp(), 0.0);
  nfd = block_reduce(nfd, red_d, SumOp(), 0.0);
  nnd = block_reduce(nnd, red_d, SumOp(), 0.0);
  mx = block_reduce(mx, red_f, MaxOp(), 0.0f);
  if (threadIdx.x == 0) {
    st->sumsq = ss; st->nonfinite = nfd; st->nan = nnd; st->maxabs = (double)mx;
    ws->counter = 0u;
  }
  return true;
}

}  // namespace nt
