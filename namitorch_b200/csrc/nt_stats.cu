// Gradient statistics (found_inf + total norm), in-place gradient transforms
// (unscale / clip-by-norm / clip-by-value) and the device-side dynamic loss-scale update.
#include <cuda.h>

#include <mutex>

#include "nt_stats.cuh"

namespace nt {

struct StatsParams {
  const nt_span* spans;
  int nspan;
  int chunk_elems;
  int64_t nchunks;
  const float* scale;
  int pass;
  double p;
  int finalize;
  nt_stats* stats;
  StatsWorkspace* ws;
};

__device__ __forceinline__ void stats_pass1(float u, double p, double maxabs, StatsAcc& a) {
  if (!(fabsf(u) <= 3.402823466e38f)) return;
  const double scaled = __ddiv_rn(fabs((double)u), maxabs);
  a.ps += p == 2.0 ? scaled * scaled : pow(scaled, p);
}

// Pass-0 variants. EXACT follows the reference's per-element float32 unscale and counts
// every non-finite value. SUMSQ serves p = 2 with no scale or a power-of-two scale <= 1:
// it sums g^2 of the stored values in f64 (the scale's square, a power of two, is applied
// once at the end, and g * scale^-1 cannot overflow float32 when scale >= 1), tracks max|g|
// and skips the per-element finiteness test. A sum of squares of finite float32 values
// cannot overflow f64 (at most 1.2e77 * 2^31), so a thread's sum is non-finite exactly when
// one of its values is inf or NaN; that thread then re-reads its own elements with EXACT to
// count them. The f64 square of g * 2^-k differs from the square of the float32 product only
// when that product is an f32 subnormal (|g * 2^-k| < 2^-126), by less than 2^-250 each.
enum { kPassExact = 0, kPassSumsq = 1, kPassPow = 2 };

template <int VARIANT> struct PassShape {   // threads per block and 16-byte vectors in flight per thread
  static constexpr int kThreads = VARIANT == kPassSumsq ? 128 : kStatsThreads;
  static constexpr int kUnrollV = VARIANT == kPassSumsq ? 8 : kUnroll;
};

template <int DT, int MODE, int VARIANT>
__device__ __forceinline__ void stats_vector(const uint4& raw, float scale, float inv, double maxabs, double p,
                                             StatsAcc& a) {
  constexpr int EPV = DT == NT_F32 ? 4 : 8;
  float x[EPV];
  unpack16<DT>(raw, x);
  if constexpr (VARIANT == kPassSumsq) {
#pragma unroll
    for (int q = 0; q < EPV; ++q) {
      a.mx = fmaxf(a.mx, fabsf(x[q]));
      const double d = (double)x[q];
      if (q & 1) a.ss1 = fma(d, d, a.ss1);
      else a.ss0 = fma(d, d, a.ss0);
    }
  } else {
#pragma unroll
    for (int q = 0; q < EPV; ++q) x[q] = unscale_by<MODE>(x[q], scale, inv);
    if constexpr (VARIANT == kPassExact) {
      stats_pass0<EPV>(x, a);
    } else {
#pragma unroll
      for (int q = 0; q < EPV; ++q) stats_pass1(x[q], p, maxabs, a);
    }
  }
}

template <int DT, int MODE, int VARIANT>
__device__ __forceinline__ void stats_scalar(float g, float scale, float inv, double maxabs, double p, StatsAcc& a) {
  if constexpr (VARIANT == kPassSumsq) {
    a.mx = fmaxf(a.mx, fabsf(g));
    const double d = (double)g;
    a.ss0 = fma(d, d, a.ss0);
  } else {
    const float u = unscale_by<MODE>(g, scale, inv);
    if constexpr (VARIANT == kPassExact) stats_one(u, a);
    else stats_pass1(u, p, maxabs, a);
  }
}

// Elements [begin, end) of one span. Thread t takes the vectors whose index is t modulo T,
// U 16-byte vectors' worth in flight (guard-free full rounds, then the remainder): U / 2
// 32-byte vectors when the range starts on a 32-byte boundary, else U 16-byte ones when it
// starts on a 16-byte boundary; then the elements after the last full vector, one by one.
// Every pass over the same range takes the same vectors in the same threads (the choice
// depends only on the range), which the sum-of-squares pass relies on when a thread
// re-reads its own elements.
// T is the block size of the launch (the kernel's shape, whichever path a thread takes).
template <int DT, int MODE, int VARIANT, int T, int U>
__device__ __forceinline__ void stats_range(const StatsParams& P, const nt_span& sp, int64_t begin, int64_t end,
                                            float scale, float inv, double maxabs, StatsAcc& a) {
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  const char* base = static_cast<const char*>(sp.ptr) + begin * ES;
  int64_t e = begin;
  if ((reinterpret_cast<uintptr_t>(base) & 31u) == 0) {
    constexpr int U2 = U > 1 ? U / 2 : 1;   // the same bytes in flight as U 16-byte vectors
    const int64_t nv = (end - begin) / (2 * EPV);
    int64_t v0 = threadIdx.x;
    for (; v0 + (U2 - 1) * T < nv; v0 += U2 * T) {
      uint4 raw[U2][2];
#pragma unroll
      for (int u = 0; u < U2; ++u) load32_cs(base + (v0 + u * T) * 32, raw[u][0], raw[u][1]);
#pragma unroll
      for (int u = 0; u < U2; ++u) {
        stats_vector<DT, MODE, VARIANT>(raw[u][0], scale, inv, maxabs, P.p, a);
        stats_vector<DT, MODE, VARIANT>(raw[u][1], scale, inv, maxabs, P.p, a);
      }
    }
    for (; v0 < nv; v0 += T) {
      uint4 lo, hi;
      load32_cs(base + v0 * 32, lo, hi);
      stats_vector<DT, MODE, VARIANT>(lo, scale, inv, maxabs, P.p, a);
      stats_vector<DT, MODE, VARIANT>(hi, scale, inv, maxabs, P.p, a);
    }
    e = begin + nv * 2 * EPV;
  } else if ((reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
    const uint4* vec = reinterpret_cast<const uint4*>(base);
    const int64_t nv = (end - begin) / EPV;
    int64_t v0 = threadIdx.x;
    for (; v0 + (U - 1) * T < nv; v0 += U * T) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) raw[u] = __ldcs(vec + v0 + u * T);
#pragma unroll
      for (int u = 0; u < U; ++u) stats_vector<DT, MODE, VARIANT>(raw[u], scale, inv, maxabs, P.p, a);
    }
    for (; v0 < nv; v0 += T) stats_vector<DT, MODE, VARIANT>(__ldcs(vec + v0), scale, inv, maxabs, P.p, a);
    e = begin + nv * EPV;
  }
  for (int64_t i = e + threadIdx.x; i < end; i += T)
    stats_scalar<DT, MODE, VARIANT>(load1<DT>(sp.ptr, i), scale, inv, maxabs, P.p, a);
}

// Each block takes a contiguous range of chunks [c0, c1). The chunks of one span inside it
// are contiguous in memory, so the block reads them as one range (one span lookup per
// block; empty spans own no chunk and are stepped over).
template <int DT, int MODE, int VARIANT, int T, int U>
__device__ __forceinline__ void stats_all_chunks(const StatsParams& P, float scale, float inv, double maxabs,
                                                 StatsAcc& a) {
  const int64_t per = (P.nchunks + gridDim.x - 1) / gridDim.x;
  const int64_t c0 = (int64_t)blockIdx.x * per;
  const int64_t c1 = c0 + per < P.nchunks ? c0 + per : P.nchunks;
  if (c0 >= c1) return;
  int s = find_owner([&](int i) { return P.spans[i].chunk_begin; }, P.nspan, c0);
  for (int64_t c = c0; c < c1 && s < P.nspan; ++s) {
    const nt_span sp = P.spans[s];
    const int64_t next_begin = s + 1 < P.nspan ? P.spans[s + 1].chunk_begin : INT64_MAX;
    const int64_t stop = c1 < next_begin ? c1 : next_begin;
    if (stop <= c) continue;
    const int64_t begin = (c - sp.chunk_begin) * (int64_t)P.chunk_elems;
    int64_t end = (stop - sp.chunk_begin) * (int64_t)P.chunk_elems;
    if (end > sp.count) end = sp.count;
    stats_range<DT, MODE, VARIANT, T, U>(P, sp, begin, end, scale, inv, maxabs, a);
    c = stop;
  }
}

// kPassSumsq applies when the launch chose it (p = 2, pass 0) and the device scale allows
// it; the block shape is the same for both, so the choice is per thread at run time.
template <int DT, int VARIANT>
__device__ __forceinline__ void stats_dispatch_scale(const StatsParams& P, const Unscale& un, double maxabs,
                                                     StatsAcc& a) {
  constexpr int T = PassShape<VARIANT>::kThreads;
  constexpr int U = PassShape<VARIANT>::kUnrollV;
  if constexpr (VARIANT == kPassSumsq) {
    if (!un.active || (un.pow2 && un.inv <= 1.0f)) {
      StatsAcc f{0.0, 0.0, 0.0, 0.0f, 0u, 0u};
      stats_all_chunks<DT, kScaleNone, kPassSumsq, T, U>(P, 1.0f, 1.0f, maxabs, f);
      if (isfinite(f.ss0) && isfinite(f.ss1)) {
        const double s2 = un.active ? (double)un.inv * (double)un.inv : 1.0;   // exact: a power of two
        a.ss0 = f.ss0 * s2;
        a.ss1 = f.ss1 * s2;
        a.mx = un.active ? __fmul_rn(f.mx, un.inv) : f.mx;
        return;
      }
    }
  }
  // The exact per-element path (also the re-read of a thread that saw inf / NaN above).
  constexpr int V = VARIANT == kPassPow ? kPassPow : kPassExact;
  constexpr int UE = kUnroll;   // the exact path is rare inside the sumsq kernel: keep its registers low
  if (!un.active) stats_all_chunks<DT, kScaleNone, V, T, UE>(P, 1.0f, 1.0f, maxabs, a);
  else if (un.pow2) stats_all_chunks<DT, kScaleMul, V, T, UE>(P, un.scale, un.inv, maxabs, a);
  else stats_all_chunks<DT, kScaleDiv, V, T, UE>(P, un.scale, un.inv, maxabs, a);
}

template <int DT, int VARIANT>
__global__ void __launch_bounds__(PassShape<VARIANT>::kThreads, 2048 / PassShape<VARIANT>::kThreads / 2)
    grad_stats_kernel(const __grid_constant__ StatsParams P) {
  constexpr int T = PassShape<VARIANT>::kThreads;
  constexpr int PASS = VARIANT == kPassPow ? 1 : 0;
  __shared__ double red_d[T / 32];
  __shared__ float red_f[T / 32];
  __shared__ unsigned red_u[T / 32];
  __shared__ bool last;
  Unscale un;
  un.init(P.scale);
  const double maxabs = PASS == 1 ? P.stats->maxabs : 0.0;
  StatsAcc a{0.0, 0.0, 0.0, 0.0f, 0u, 0u};
  stats_dispatch_scale<DT, VARIANT>(P, un, maxabs, a);

  double ss = block_reduce(a.ss0 + a.ss1, red_d, SumOp(), 0.0);
  double ps = block_reduce(a.ps, red_d, SumOp(), 0.0);
  float mx = block_reduce(a.mx, red_f, MaxOp(), 0.0f);
  unsigned nf = block_reduce(a.nf, red_u, SumOp(), 0u);
  unsigned nn = block_reduce(a.nn, red_u, SumOp(), 0u);
  if (threadIdx.x == 0) {
    StatsPartial& out = P.ws->partials[blockIdx.x];
    out.sumsq = ss; out.powsum = ps; out.maxabs = mx; out.nonfinite = nf; out.nan = nn;
  }
  if (!last_block_ticket(&P.ws->counter, &last)) return;

  // Fixed-order reduction of the block partials.
  ss = 0.0; ps = 0.0; mx = 0.0f;
  double nfd = 0.0, nnd = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    const StatsPartial q = P.ws->partials[b];
    ss += q.sumsq; ps += q.powsum; mx = fmaxf(mx, q.maxabs); nfd += q.nonfinite; nnd += q.nan;
  }
  ss = block_reduce(ss, red_d, SumOp(), 0.0);
  ps = block_reduce(ps, red_d, SumOp(), 0.0);
  nfd = block_reduce(nfd, red_d, SumOp(), 0.0);
  nnd = block_reduce(nnd, red_d, SumOp(), 0.0);
  mx = block_reduce(mx, red_f, MaxOp(), 0.0f);
  if (threadIdx.x == 0) {
    nt_stats* st = P.stats;
    if (PASS == 0) {
      st->sumsq = ss; st->nonfinite = nfd; st->nan = nnd; st->maxabs = (double)mx;
    } else {
      st->powsum = ps;
    }
    if (P.finalize) stats_finalize(st, P.p);
    P.ws->counter = 0u;
  }
}

__global__ void stats_finalize_kernel(nt_stats* s, double p) {
  if (threadIdx.x == 0 && blockIdx.x == 0) stats_finalize(s, p);
}

// ---- in-place transforms ----------------------------------------------------------------
struct TransformParams {
  const nt_span* spans;
  int nspan;
  int chunk_elems;
  int64_t nchunks;
  const float* scale;
  const nt_stats* stats;
  int clip;
  double max_norm;
  int mode;          // 0: unscale / clip-by-norm, 1: clip-by-value
  double clip_value;
};

template <int DT>
__device__ __forceinline__ float transform_one(float x, const TransformParams& P, const Unscale& un,
                                               bool clip, double coef) {
  if (P.mode == 1) {
    const double d = (double)x;
    const double r = d < -P.clip_value ? -P.clip_value : (d > P.clip_value ? P.clip_value : d);
    return __double2float_rn(r);
  }
  float u = un(x);
  if (clip) u = __double2float_rn(__dmul_rn((double)u, coef));
  return u;
}

template <int DT>
__global__ void __launch_bounds__(256) grad_transform_kernel(const __grid_constant__ TransformParams P) {
  Unscale un;
  un.init(P.scale);
  bool clip = false;
  double coef = 1.0;
  if (P.clip && P.stats != nullptr) {
    const double c = P.max_norm / (P.stats->norm + 1e-6);
    if (c < 1.0) { clip = true; coef = c; }
  }
  if (P.mode == 0 && !un.active && !clip) return;
  const int esize = DT == NT_F32 ? 4 : 2;
  for (int64_t chunk = blockIdx.x; chunk < P.nchunks; chunk += gridDim.x) {
    const int s = find_owner([&](int i) { return P.spans[i].chunk_begin; }, P.nspan, chunk);
    const nt_span sp = P.spans[s];
    void* ptr = const_cast<void*>(sp.ptr);
    const int64_t begin = (chunk - sp.chunk_begin) * (int64_t)P.chunk_elems;
    int64_t end = begin + P.chunk_elems;
    if (end > sp.count) end = sp.count;
    int64_t e = begin;
    if (((reinterpret_cast<uintptr_t>(static_cast<char*>(ptr) + begin * esize)) & 15u) == 0) {
      const int64_t body_end = begin + ((end - begin) & ~(int64_t)7);
      for (int64_t i = begin + (int64_t)threadIdx.x * 8; i < body_end; i += (int64_t)blockDim.x * 8) {
        float x[8];
        load8<DT>(ptr, i, x);
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = transform_one<DT>(x[k], P, un, clip, coef);
        store8<DT>(ptr, i, x);
      }
      e = body_end;
    }
    for (int64_t i = e + threadIdx.x; i < end; i += blockDim.x)
      store1<DT>(ptr, i, transform_one<DT>(load1<DT>(ptr, i), P, un, clip, coef));
  }
}

// ---- GradScaler.update ------------------------------------------------------------------
struct ScalerParams {
  float* scale;
  int32_t* tracker;
  const double* found[NT_MAX_FOUND_INF];
  int count;
  double growth;
  double backoff;
  int interval;
};

__global__ void scaler_update_kernel(const __grid_constant__ ScalerParams P) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  bool inf = false;
  for (int i = 0; i < P.count; ++i) inf = inf || (*P.found[i] != 0.0);
  const double tiny = 1.1754943508222875e-38;     // float32 tiny
  const double fmax32 = 3.4028234663852886e+38;   // float32 max
  const double s = (double)*P.scale;
  if (inf) {
    double r = __dmul_rn(s, P.backoff);
    if (r < tiny) r = tiny;
    *P.scale = __double2float_rn(r);
    *P.tracker = 0;
  } else {
    int t = *P.tracker + 1;
    if (t == P.interval) {
      double r = __dmul_rn(s, P.growth);
      if (r > fmax32) r = fmax32;
      *P.scale = __double2float_rn(r);
      t = 0;
    }
    *P.tracker = t;
  }
}

struct ScheduleParams {
  int32_t* step;
  const double* found[NT_MAX_FOUND_INF];
  int count;
};

__global__ void schedule_step_kernel(const __grid_constant__ ScheduleParams P) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  bool inf = false;
  for (int i = 0; i < P.count; ++i) inf = inf || (*P.found[i] != 0.0);
  if (!inf) *P.step += 1;
}

static int check_spans(const nt_span* spans, int32_t num_spans, int32_t chunk_elems, int64_t num_chunks,
                       int32_t dtype, const char* who) {
  if (num_spans < 0 || num_chunks < 0) { set_error("%s: negative sizes", who); return NT_EINVAL; }
  if (num_spans > 0 && num_chunks > 0 && !spans) { set_error("%s: spans is NULL", who); return NT_EINVAL; }
  if (chunk_elems <= 0 || (chunk_elems & 7) != 0) {
    set_error("%s: chunk_elems must be a positive multiple of 8 (got %d)", who, chunk_elems);
    return NT_EINVAL;
  }
  if (dtype_size(dtype) == 0) { set_error("%s: unsupported dtype %d", who, dtype); return NT_EUNSUPPORTED; }
  return NT_OK;
}

template <typename K, typename Params>
static int launch_grid(K kernel, const Params& P, int64_t nchunks, int threads, int per_sm,
                       int64_t max_blocks, cudaStream_t stream, const char* what) {
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  if (grid > max_blocks) grid = max_blocks;
  if (grid > nchunks) grid = nchunks;
  if (grid < 1) grid = 1;
  kernel<<<(unsigned)grid, threads, 0, stream>>>(P);
  return launch_status(what);
}

template <int DT>
static int launch_stats_dt(const StatsParams& P, int64_t nchunks, cudaStream_t s, const char* what) {
  if (P.pass == 1)
    return launch_grid(grad_stats_kernel<DT, kPassPow>, P, nchunks, kStatsThreads, 6, kStatsMaxBlocks, s, what);
  if (P.p == 2.0)
    return launch_grid(grad_stats_kernel<DT, kPassSumsq>, P, nchunks, PassShape<kPassSumsq>::kThreads, 8,
                       kStatsMaxBlocks, s, what);
  return launch_grid(grad_stats_kernel<DT, kPassExact>, P, nchunks, kStatsThreads, 6, kStatsMaxBlocks, s, what);
}

static int launch_stats(const StatsParams& P, int32_t dtype, int64_t nchunks, cudaStream_t s, const char* what) {
  switch (dtype) {
    case NT_F32: return launch_stats_dt<NT_F32>(P, nchunks, s, what);
    case NT_F16: return launch_stats_dt<NT_F16>(P, nchunks, s, what);
    default: return launch_stats_dt<NT_BF16>(P, nchunks, s, what);
  }
}

}  // namespace nt

using namespace nt;

extern "C" {

size_t nt_grad_stats_workspace_size(void) { return sizeof(StatsWorkspace); }

int nt_grad_stats(const nt_grad_stats_args* args, void* stream) {
  nt::TraceRange trace("nt_grad_stats");
  if (!args) { set_error("nt_grad_stats: args is NULL"); return NT_EINVAL; }
  const nt_grad_stats_args& a = *args;
  int rc = check_spans(a.spans, a.num_spans, a.chunk_elems, a.num_chunks, a.dtype, "nt_grad_stats");
  if (rc) return rc;
  if (!a.stats || !a.workspace) { set_error("nt_grad_stats: stats / workspace is NULL"); return NT_EINVAL; }
  if (a.workspace_bytes < sizeof(StatsWorkspace)) {
    set_error("nt_grad_stats: workspace needs %zu bytes (got %zu)", sizeof(StatsWorkspace), a.workspace_bytes);
    return NT_EINVAL;
  }
  if (a.pass != 0 && a.pass != 1) { set_error("nt_grad_stats: pass must be 0 or 1"); return NT_EINVAL; }
  if (!(a.norm_type > 0.0)) { set_error("nt_grad_stats: norm_type must be positive"); return NT_EINVAL; }
  StatsParams P;
  P.spans = a.spans; P.nspan = a.num_spans; P.chunk_elems = a.chunk_elems;
  P.nchunks = (a.num_spans == 0) ? 0 : a.num_chunks;
  P.scale = a.scale; P.pass = a.pass; P.p = a.norm_type; P.finalize = a.finalize;
  P.stats = a.stats; P.ws = static_cast<StatsWorkspace*>(a.workspace);
  cudaStream_t s = as_stream(stream);
  // An empty gradient list still runs one block so the statistics are written.
  const int64_t nchunks = P.nchunks > 0 ? P.nchunks : 1;
  return launch_stats(P, a.dtype, nchunks, s, "nt_grad_stats launch");
}

int nt_schedule_step(int32_t* lr_step, const double* const* found_inf, int32_t count, void* stream) {
  nt::TraceRange trace("nt_schedule_step");
  if (!lr_step) { set_error("nt_schedule_step: lr_step is NULL"); return NT_EINVAL; }
  if (count < 0 || count > NT_MAX_FOUND_INF || (count > 0 && !found_inf)) {
    set_error("nt_schedule_step: count must be in [0, %d] with a pointer array", NT_MAX_FOUND_INF);
    return NT_EINVAL;
  }
  ScheduleParams P;
  P.step = lr_step;
  P.count = count;
  for (int i = 0; i < count; ++i) {
    if (!found_inf[i]) { set_error("nt_schedule_step: found_inf[%d] is NULL", i); return NT_EINVAL; }
    P.found[i] = found_inf[i];
  }
  schedule_step_kernel<<<1, 32, 0, as_stream(stream)>>>(P);
  return launch_status("nt_schedule_step launch");
}

int nt_grad_stats_finalize(nt_stats* stats, double norm_type, void* stream) {
  nt::TraceRange trace("nt_grad_stats_finalize");
  if (!stats) { set_error("nt_grad_stats_finalize: stats is NULL"); return NT_EINVAL; }
  if (!(norm_type > 0.0)) { set_error("nt_grad_stats_finalize: norm_type must be positive"); return NT_EINVAL; }
  stats_finalize_kernel<<<1, 32, 0, as_stream(stream)>>>(stats, norm_type);
  return launch_status("nt_grad_stats_finalize launch");
}

static int transform_common(TransformParams& P, int32_t dtype, cudaStream_t s) {
  if (P.nspan == 0 || P.nchunks == 0) return NT_OK;
  switch (dtype) {
    case NT_F32: return launch_grid(grad_transform_kernel<NT_F32>, P, P.nchunks, 256, 8, 1 << 20, s, "nt_grad_transform launch");
    case NT_F16: return launch_grid(grad_transform_kernel<NT_F16>, P, P.nchunks, 256, 8, 1 << 20, s, "nt_grad_transform launch");
    default: return launch_grid(grad_transform_kernel<NT_BF16>, P, P.nchunks, 256, 8, 1 << 20, s, "nt_grad_transform launch");
  }
}

int nt_grad_transform(const nt_span* spans, int32_t num_spans, int32_t chunk_elems, int64_t num_chunks,
                      int32_t dtype, const float* scale, const nt_stats* stats, int32_t clip,
                      double max_norm, void* stream) {
  nt::TraceRange trace("nt_grad_transform");
  int rc = check_spans(spans, num_spans, chunk_elems, num_chunks, dtype, "nt_grad_transform");
  if (rc) return rc;
  if (clip && !stats) { set_error("nt_grad_transform: clip needs stats"); return NT_EINVAL; }
  TransformParams P;
  P.spans = spans; P.nspan = num_spans; P.chunk_elems = chunk_elems; P.nchunks = num_chunks;
  P.scale = scale; P.stats = stats; P.clip = clip; P.max_norm = max_norm; P.mode = 0; P.clip_value = 0.0;
  return transform_common(P, dtype, as_stream(stream));
}

int nt_grad_clip_value(const nt_span* spans, int32_t num_spans, int32_t chunk_elems, int64_t num_chunks,
                       int32_t dtype, double clip_value, void* stream) {
  nt::TraceRange trace("nt_grad_clip_value");
  int rc = check_spans(spans, num_spans, chunk_elems, num_chunks, dtype, "nt_grad_clip_value");
  if (rc) return rc;
  if (!(clip_value >= 0.0) || !isfinite(clip_value)) {
    set_error("clip_value must be finite and nonnegative.");
    return NT_EINVAL;
  }
  TransformParams P;
  P.spans = spans; P.nspan = num_spans; P.chunk_elems = chunk_elems; P.nchunks = num_chunks;
  P.scale = nullptr; P.stats = nullptr; P.clip = 0; P.max_norm = 0.0; P.mode = 1; P.clip_value = clip_value;
  return transform_common(P, dtype, as_stream(stream));
}

int nt_scaler_update(float* scale, int32_t* growth_tracker, const double* const* found_inf, int32_t count,
                     double growth_factor, double backoff_factor, int32_t growth_interval, void* stream) {
  nt::TraceRange trace("nt_scaler_update");
  if (!scale || !growth_tracker) { set_error("nt_scaler_update: NULL scale / tracker"); return NT_EINVAL; }
  if (count < 1 || count > NT_MAX_FOUND_INF || !found_inf) {
    set_error("nt_scaler_update: count must be in [1, %d]", NT_MAX_FOUND_INF);
    return NT_EINVAL;
  }
  if (!(growth_factor > 1.0) || !isfinite(growth_factor)) { set_error("growth_factor must be greater than 1."); return NT_EINVAL; }
  if (!(backoff_factor > 0.0 && backoff_factor < 1.0)) { set_error("backoff_factor must be between 0 and 1."); return NT_EINVAL; }
  if (growth_interval <= 0) { set_error("growth_interval must be positive."); return NT_EINVAL; }
  ScalerParams P;
  P.scale = scale; P.tracker = growth_tracker; P.count = count;
  for (int i = 0; i < NT_MAX_FOUND_INF; ++i) P.found[i] = i < count ? found_inf[i] : nullptr;
  for (int i = 0; i < count; ++i) {
    if (!P.found[i]) { set_error("nt_scaler_update: found_inf[%d] is NULL", i); return NT_EINVAL; }
  }
  P.growth = growth_factor; P.backoff = backoff_factor; P.interval = growth_interval;
  scaler_update_kernel<<<1, 32, 0, as_stream(stream)>>>(P);
  return launch_status("nt_scaler_update launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Allocation-free gradient statistics.
//
// Some callers cannot allocate device memory themselves: a host that has handed all of
// its device memory to its own pool or arena, a plugin that runs inside another
// runtime's allocator, or a C/FFI caller without access to the CUDA runtime's
// allocation calls. For them, nt_grad_stats_noalloc keeps the cross-block scratch of the
// statistics reduction (the block partials and the last-block ticket) and the span table
// in one file-scope device array. Every GPU that loads this library reserves it
// (kNoAllocScratchBytes) until the process exits.
// ---------------------------------------------------------------------------------------------
namespace nt {

struct NoAllocScratch {
  StatsWorkspace ws;
  nt_span spans[NT_NOALLOC_MAX_SPANS];
};

static __device__ __align__(256) unsigned char g_noalloc_scratch[sizeof(NoAllocScratch)];

struct NoAllocSpans {
  nt_span spans[NT_NOALLOC_MAX_SPANS];
  int count;
};

// Writes this call's span table into the scratch and clears the ticket counter (the
// previous call leaves the array as it was, so nothing is assumed to start at zero).
__global__ void noalloc_prepare_kernel(const __grid_constant__ NoAllocSpans S) {
  NoAllocScratch* scratch = reinterpret_cast<NoAllocScratch*>(g_noalloc_scratch);
  for (int i = threadIdx.x; i < S.count; i += blockDim.x) scratch->spans[i] = S.spans[i];
  if (threadIdx.x == 0) scratch->ws.counter = 0u;
}

// Device address of the scratch array in the CUDA context current on this thread.
//
// The host-side name of a __device__ array is only a stand-in for its device address,
// and that address belongs to a context, not to a device: the primary context that
// cudaDeviceReset destroyed, or a context the caller created with the driver API, each
// load this library's module at their own address. So the address is looked up with
// cudaGetSymbolAddress once per context and cached under the context's unique ID
// (cuCtxGetId; a context handle can be reused by a later context, an ID is not). The
// lookup is serialised by a mutex, so two host threads making the first call at once
// are safe. When no context is current yet, the lookup itself creates the runtime's
// primary context for the current device, and the cache entry is made after it.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct NoAllocContextSlot {
  unsigned long long context_id;
  void* address;
};

constexpr int kNoAllocContextSlots = 64;
static std::mutex g_noalloc_lock;
static NoAllocContextSlot g_noalloc_slots[kNoAllocContextSlots];
static int g_noalloc_slots_used = 0;
static CtxGetCurrentFn g_ctx_get_current = nullptr;
static CtxGetIdFn g_ctx_get_id = nullptr;

// Called with g_noalloc_lock held.
static int resolve_context_calls() {
  if (g_ctx_get_current && g_ctx_get_id) return NT_OK;
  void* current = nullptr;
  void* id = nullptr;
  cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e1 = cudaGetDriverEntryPoint("cuCtxGetCurrent", &current, cudaEnableDefault, &q1);
  cudaError_t e2 = cudaGetDriverEntryPoint("cuCtxGetId", &id, cudaEnableDefault, &q2);
  if (e1 != cudaSuccess) return cuda_fail(e1, "cudaGetDriverEntryPoint(cuCtxGetCurrent)");
  if (e2 != cudaSuccess) return cuda_fail(e2, "cudaGetDriverEntryPoint(cuCtxGetId)");
  if (q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || !current || !id) {
    set_error("nt_grad_stats_noalloc: the driver does not provide cuCtxGetCurrent / cuCtxGetId");
    return NT_ECUDA;
  }
  g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(current);
  g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(id);
  return NT_OK;
}

// Called with g_noalloc_lock held. *id = 0 when no context is current.
static int current_context_id(unsigned long long* id) {
  *id = 0;
  CUcontext ctx = nullptr;
  CUresult r = g_ctx_get_current(&ctx);
  if (r != CUDA_SUCCESS) { set_error("nt_grad_stats_noalloc: cuCtxGetCurrent failed (%d)", int(r)); return NT_ECUDA; }
  if (!ctx) return NT_OK;
  r = g_ctx_get_id(ctx, id);
  if (r != CUDA_SUCCESS) { set_error("nt_grad_stats_noalloc: cuCtxGetId failed (%d)", int(r)); return NT_ECUDA; }
  return NT_OK;
}

static int noalloc_scratch_address(void** out) {
  std::lock_guard<std::mutex> guard(g_noalloc_lock);
  int rc = resolve_context_calls();
  if (rc) return rc;
  unsigned long long id = 0;
  rc = current_context_id(&id);
  if (rc) return rc;
  if (id != 0) {
    for (int i = 0; i < g_noalloc_slots_used; ++i) {
      if (g_noalloc_slots[i].context_id == id) { *out = g_noalloc_slots[i].address; return NT_OK; }
    }
  }
  void* ptr = nullptr;
  cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(noalloc scratch)");
  if (id == 0) {   // the lookup above created the primary context: key the entry by it
    rc = current_context_id(&id);
    if (rc) return rc;
  }
  // A process that has used more contexts than the table holds still gets the right
  // address; it is then looked up on every call instead of being cached.
  if (id != 0 && g_noalloc_slots_used < kNoAllocContextSlots) {
    g_noalloc_slots[g_noalloc_slots_used].context_id = id;
    g_noalloc_slots[g_noalloc_slots_used].address = ptr;
    ++g_noalloc_slots_used;
  }
  *out = ptr;
  return NT_OK;
}

}  // namespace nt

extern "C" {

size_t nt_grad_stats_noalloc_scratch_bytes(void) { return sizeof(nt::NoAllocScratch); }

int nt_grad_stats_noalloc(const nt_span* spans, int32_t num_spans, int32_t dtype, const float* scale,
                          double norm_type, nt_stats* stats, void* stream) {
  nt::TraceRange trace("nt_grad_stats_noalloc");
  using namespace nt;
  if (num_spans < 0) { set_error("nt_grad_stats_noalloc: negative span count"); return NT_EINVAL; }
  if (num_spans > NT_NOALLOC_MAX_SPANS) {
    set_error("nt_grad_stats_noalloc: %d spans exceed the maximum of %d (the span table lives in a fixed "
              "%zu-byte static scratch array); merge gradients into fewer contiguous spans or use nt_grad_stats",
              num_spans, NT_NOALLOC_MAX_SPANS, sizeof(NoAllocScratch));
    return NT_EINVAL;
  }
  if (num_spans > 0 && !spans) { set_error("nt_grad_stats_noalloc: spans is NULL"); return NT_EINVAL; }
  if (!stats) { set_error("nt_grad_stats_noalloc: stats is NULL"); return NT_EINVAL; }
  if (dtype_size(dtype) == 0) { set_error("nt_grad_stats_noalloc: unsupported dtype %d", dtype); return NT_EUNSUPPORTED; }
  if (!(norm_type > 0.0)) { set_error("nt_grad_stats_noalloc: norm_type must be positive"); return NT_EINVAL; }
  void* base = nullptr;
  int rc = noalloc_scratch_address(&base);
  if (rc) return rc;
  NoAllocScratch* scratch = static_cast<NoAllocScratch*>(base);

  NoAllocSpans S;
  int64_t chunks = 0;
  int used = 0;
  for (int i = 0; i < num_spans; ++i) {
    if (spans[i].count < 0) { set_error("nt_grad_stats_noalloc: span %d has a negative count", i); return NT_EINVAL; }
    if (spans[i].count == 0) continue;
    if (!spans[i].ptr) { set_error("nt_grad_stats_noalloc: span %d has a NULL pointer", i); return NT_EINVAL; }
    S.spans[used].ptr = spans[i].ptr;
    S.spans[used].count = spans[i].count;
    S.spans[used].chunk_begin = chunks;
    chunks += (spans[i].count + kNoAllocChunk - 1) / kNoAllocChunk;
    ++used;
  }
  S.count = used;
  cudaStream_t s = as_stream(stream);
  noalloc_prepare_kernel<<<1, 64, 0, s>>>(S);
  rc = launch_status("nt_grad_stats_noalloc prepare launch");
  if (rc) return rc;

  StatsParams P;
  P.spans = scratch->spans;
  P.nspan = used;
  P.chunk_elems = kNoAllocChunk;
  P.nchunks = used == 0 ? 0 : chunks;
  P.scale = scale;
  P.p = norm_type;
  P.stats = stats;
  P.ws = &scratch->ws;
  const int64_t grid_chunks = P.nchunks > 0 ? P.nchunks : 1;
  const bool two_pass = !(norm_type == 2.0 || isinf(norm_type));
  for (int pass = 0; pass <= (two_pass ? 1 : 0); ++pass) {
    P.pass = pass;
    P.finalize = pass == (two_pass ? 1 : 0);
    rc = launch_stats(P, dtype, grid_chunks, s, "nt_grad_stats_noalloc launch");
    if (rc) return rc;
  }
  return NT_OK;
}

}  // extern "C"
