// Row softmax family for attention scores (rows of at most 4096 elements): softmax, masked
// and causal softmax and their backward passes, the operations of the reference's
// SoftmaxCUDAKernels (namitorch/backends/cuda/softmax.py:6-88).
//
// A row stays in registers: one read, max and sum reductions with warp shuffles (shared
// memory across the warps of a row), one write: 8 bytes per element for float32 forward,
// 12 for backward. Semantics follow the reference kernel:
//   allowed(c) = (not causal or c <= offset + row % queries) and (no mask or mask[row % mask_rows][c])
//   forward:  m = max over allowed values (NaN propagates); empty = m is -inf, invalid = m is
//             NaN or +inf; y = empty ? 0 : exp(x - m) / sum (NaN everywhere when invalid),
//             with exp on the SFU and the division as a multiply by 1/sum (each within a few
//             float32 ulps of expf and IEEE division)
//   backward: y' = allowed ? y * (g - sum_c g*y) : 0
// Sum orders differ from the reference's shared-memory tree, so results agree to float32
// rounding. Half and bfloat16 rows are computed in float32 and rounded once on store.
#include <cmath>

#include "nt_rows.cuh"

namespace nt {

struct SoftmaxParams {
  const void* x;
  const void* g;
  const uint8_t* mask;
  void* y;
  unsigned long long* summary;   // {empty rows, invalid rows, first bad row, unused} or NULL
  int64_t rows;
  int width;
  int64_t mask_rows;             // 0: one mask row for every row
  int64_t queries;
  int64_t offset;
  int causal;
  int vec;                       // rows start on 16-byte boundaries and width fills whole vectors
};

constexpr int kSoftmaxThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the SFU; results below 2^-126 flush to zero (an entry that far below the row max
// contributes nothing to the sum, and its probability is below 2^-126 of the largest).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16-bit rows of the backward pass on the vector path stay packed in registers (EPV values
// per 16-byte vector) and are unpacked in each of the two passes. That keeps the register
// count low enough for the warps that hide memory latency when a row is only 2 bytes per
// element. (The forward keeps its row in float32 and spreads it over more warps instead:
// repacking it would mean evaluating exp twice.)
template <int DT, int NPL, int WARPS, bool BACKWARD>
__device__ __forceinline__ void packed_row(const SoftmaxParams& P, int64_t row, bool live, int last,
                                           const uint8_t* mrow, int t, float* smem) {
  constexpr int EPV = 8;
  constexpr int NC = NPL / EPV;
  constexpr int T = 32 * WARPS;
  const int width = P.width;
  const int64_t base = (live ? row : 0) * (int64_t)width;
  const uint4* xv = reinterpret_cast<const uint4*>(static_cast<const char*>(P.x) + base * 2);
  uint4 xr[NC], gr[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int k = c * T + t;
    xr[c] = live && k * EPV < width ? __ldcs(xv + k) : make_uint4(0, 0, 0, 0);
  }
  if constexpr (BACKWARD) {
    const uint4* gv = reinterpret_cast<const uint4*>(static_cast<const char*>(P.g) + base * 2);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int k = c * T + t;
      gr[c] = live && k * EPV < width ? __ldcs(gv + k) : make_uint4(0, 0, 0, 0);
    }
  }
  auto ok = [&](int j) { return j <= last && (mrow == nullptr || __ldg(mrow + j) != 0); };
  uint4* yv = reinterpret_cast<uint4*>(static_cast<char*>(P.y) + base * 2);
  if constexpr (BACKWARD) {
    float dot = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float y[EPV], g[EPV];
      unpack16<DT>(xr[c], y);
      unpack16<DT>(gr[c], g);
#pragma unroll
      for (int e = 0; e < EPV; ++e) dot = __fadd_rn(dot, __fmul_rn(g[e], y[e]));
    }
    dot = row_sum<WARPS>(dot, smem);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int k = c * T + t;
      float y[EPV], g[EPV];
      unpack16<DT>(xr[c], y);
      unpack16<DT>(gr[c], g);
#pragma unroll
      for (int e = 0; e < EPV; ++e) y[e] = ok(k * EPV + e) ? __fmul_rn(y[e], __fsub_rn(g[e], dot)) : 0.0f;
      if (live && k * EPV < width) store_vec16<DT>(yv, k, y);
    }
    return;
  }
  float m = -INFINITY;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int k = c * T + t;
    float x[EPV];
    unpack16<DT>(xr[c], x);
#pragma unroll
    for (int e = 0; e < EPV; ++e) m = max_nan(m, ok(k * EPV + e) ? x[e] : -INFINITY);
  }
  m = row_max<WARPS>(m, smem);
  const bool empty = m == -INFINITY;
  const bool invalid = isnan(m) || m == INFINITY;
  if (live && t == 0 && P.summary != nullptr && (empty || invalid)) {
    atomicAdd(&P.summary[empty ? 0 : 1], 1ull);
    atomicMin(&P.summary[2], (unsigned long long)row);
  }
  const bool normal = !empty && !invalid;
  const float ml = normal ? m * kLog2e : 0.0f;
  float s = 0.0f;
  if (normal) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int k = c * T + t;
      float x[EPV];
      unpack16<DT>(xr[c], x);
#pragma unroll
      for (int e = 0; e < EPV; ++e) s += ok(k * EPV + e) ? ex2(fmaf(x[e], kLog2e, -ml)) : 0.0f;
    }
  }
  s = row_sum<WARPS>(s, smem);
  const float inv = __frcp_rn(s);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int k = c * T + t;
    float x[EPV];
    unpack16<DT>(xr[c], x);
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      const float p = ok(k * EPV + e) ? ex2(fmaf(x[e], kLog2e, -ml)) * inv : 0.0f;
      x[e] = normal ? p : (empty ? 0.0f : __int_as_float(0x7fffffff));
    }
    if (live && k * EPV < width) store_vec16<DT>(yv, k, x);
  }
}

// r % n, in 32 bits when both fit (a 64-bit division costs several times more).
__device__ __forceinline__ int64_t row_mod(int64_t r, int64_t n) {
  if ((uint64_t)r <= 0xffffffffull && (uint64_t)n <= 0xffffffffull) return (int64_t)((uint32_t)r % (uint32_t)n);
  return r % n;
}

template <int DT, int NPL, int WARPS, bool BACKWARD, bool VEC>
__global__ void __launch_bounds__(kSoftmaxThreads) row_softmax_kernel(const __grid_constant__ SoftmaxParams P) {
  __shared__ float smem[kSoftmaxThreads / 32];
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  constexpr int T = 32 * WARPS;
  constexpr int GROUPS = kSoftmaxThreads / T;   // rows in flight per block
  const int t = threadIdx.x % T;
  const int group = threadIdx.x / T;
  constexpr bool vec = VEC;
  const int width = P.width;
  const float NEG_INF = -INFINITY;

  // Rows are visited in rounds of GROUPS per block so that every warp of the block reaches
  // the same barriers (a group past the last row computes on an empty row and stores nothing).
  for (int64_t first = (int64_t)blockIdx.x * GROUPS; first < P.rows; first += (int64_t)gridDim.x * GROUPS) {
    const int64_t row = first + group;
    const bool live = row < P.rows;
    const int64_t r = live ? row : 0;
    const int64_t base = r * (int64_t)width;
    // The last allowed column of the row (-1: none): the width, cut by the causal rule.
    int last = live ? width - 1 : -1;
    if (P.causal) {
      const int64_t limit = P.offset + row_mod(r, P.queries);
      if (limit < last) last = (int)limit;
    }
    const uint8_t* mrow = P.mask == nullptr ? nullptr
                          : P.mask + (P.mask_rows == 0 ? 0 : row_mod(r, P.mask_rows) * (int64_t)width);
    if constexpr (ES == 2 && VEC && BACKWARD) {
      packed_row<DT, NPL, WARPS, BACKWARD>(P, row, live, last, mrow, t, smem);
      continue;
    }
    const char* xrow = static_cast<const char*>(P.x) + base * ES;
    char* yrow = static_cast<char*>(P.y) + base * ES;
    float v[NPL];
    // Forward over whole vectors without a mask tensor: the vectors past the last allowed
    // column (half of a causal row on average) are neither read nor exponentiated.
    constexpr bool kUpto = !BACKWARD && VEC;
    const bool upto = kUpto && mrow == nullptr;
    if (live && upto) load_row_upto<DT, NPL, WARPS>(xrow, last, t, v);
    else if (live) load_row<DT, NPL, WARPS>(xrow, width, t, vec, v);
    else {
#pragma unroll
      for (int q = 0; q < NPL; ++q) v[q] = 0.0f;
    }
    if constexpr (BACKWARD) {
      float w[NPL];
      const char* grow = static_cast<const char*>(P.g) + base * ES;
      if (live) load_row<DT, NPL, WARPS>(grow, width, t, vec, w);
      else {
#pragma unroll
        for (int q = 0; q < NPL; ++q) w[q] = 0.0f;
      }
      float dot = 0.0f;
#pragma unroll
      for (int q = 0; q < NPL; ++q) dot = __fadd_rn(dot, __fmul_rn(w[q], v[q]));
      dot = row_sum<WARPS>(dot, smem);
      if (vec && mrow == nullptr) {
        // Whole vectors: per-element checks only where a vector reaches past `last`.
#pragma unroll
        for (int c = 0; c < NPL / EPV; ++c) {
          const int j0 = (c * T + t) * EPV;
          if (j0 + EPV - 1 <= last) {
#pragma unroll
            for (int e = 0; e < EPV; ++e) v[c * EPV + e] = __fmul_rn(v[c * EPV + e], __fsub_rn(w[c * EPV + e], dot));
          } else {
#pragma unroll
            for (int e = 0; e < EPV; ++e)
              v[c * EPV + e] = j0 + e <= last ? __fmul_rn(v[c * EPV + e], __fsub_rn(w[c * EPV + e], dot)) : 0.0f;
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < NPL; ++q) {
          const int j = slot_column<EPV>(q, t, T, vec);
          const bool ok = j <= last && (mrow == nullptr || __ldg(mrow + j) != 0);
          v[q] = ok ? __fmul_rn(v[q], __fsub_rn(w[q], dot)) : 0.0f;
        }
      }
    } else {
      float m = NEG_INF;
      if (vec && mrow == nullptr) {
        // Whole vectors: only a vector that reaches past the last allowed column (the
        // diagonal of a causal row, or a vector past the width) needs per-element masking.
#pragma unroll
        for (int c = 0; c < NPL / EPV; ++c) {
          const int j0 = (c * T + t) * EPV;
          if (j0 + EPV - 1 > last) {
#pragma unroll
            for (int e = 0; e < EPV; ++e)
              if (j0 + e > last) v[c * EPV + e] = NEG_INF;
          }
        }
#pragma unroll
        for (int q = 0; q < NPL; ++q) m = max_nan(m, v[q]);
      } else {
#pragma unroll
        for (int q = 0; q < NPL; ++q) {
          const int j = slot_column<EPV>(q, t, T, vec);
          const bool ok = j <= last && (mrow == nullptr || __ldg(mrow + j) != 0);
          v[q] = ok ? v[q] : NEG_INF;
          m = max_nan(m, v[q]);
        }
      }
      m = row_max<WARPS>(m, smem);
      const bool empty = m == NEG_INF;
      const bool invalid = isnan(m) || m == INFINITY;
      if (live && t == 0 && P.summary != nullptr && (empty || invalid)) {
        atomicAdd(&P.summary[empty ? 0 : 1], 1ull);
        atomicMin(&P.summary[2], (unsigned long long)row);
      }
      // exp(x - m) = 2^(x log2e - m log2e): one FMA and one SFU op per entry (a disallowed
      // entry is -inf and gives 0); one reciprocal of the row sum replaces the divisions.
      float s = 0.0f;
      if (!empty && !invalid) {
        const float ml = m * kLog2e;
        float s2 = 0.0f;   // two partial sums: independent additions
#pragma unroll
        for (int c = 0; c < NPL / EPV; ++c) {
          // A vector that starts past `last` holds only -inf: its exponentials are 0 and add
          // nothing (s + 0 is s), so it is skipped.
          if (upto && (c * T + t) * EPV > last) {
#pragma unroll
            for (int e = 0; e < EPV; ++e) v[c * EPV + e] = 0.0f;
            continue;
          }
#pragma unroll
          for (int e = 0; e < EPV; ++e) {
            const int q = c * EPV + e;
            v[q] = ex2(fmaf(v[q], kLog2e, -ml));
            if (q & 1) s2 += v[q];
            else s += v[q];
          }
        }
        s += s2;
      } else {
#pragma unroll
        for (int q = 0; q < NPL; ++q) v[q] = empty ? 0.0f : __int_as_float(0x7fffffff);
        s = empty ? 0.0f : __int_as_float(0x7fffffff);
      }
      s = row_sum<WARPS>(s, smem);
      if (!empty) {
        const float inv = __frcp_rn(s);
#pragma unroll
        for (int q = 0; q < NPL; ++q) v[q] *= inv;
      }
    }
    if (live) store_row<DT, NPL, WARPS>(yrow, width, t, vec, v);
  }
}

template <int DT, int NPL, int WARPS, bool BACKWARD, bool VEC>
static int launch_variant(const SoftmaxParams& P, cudaStream_t s) {
  static int per_sm = 0;
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, row_softmax_kernel<DT, NPL, WARPS, BACKWARD, VEC>,
                                                      kSoftmaxThreads, 0) != cudaSuccess || per_sm <= 0)
      per_sm = 4;
  }
  constexpr int GROUPS = kSoftmaxThreads / (32 * WARPS);
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  const int64_t need = (P.rows + GROUPS - 1) / GROUPS;
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  row_softmax_kernel<DT, NPL, WARPS, BACKWARD, VEC><<<(unsigned)grid, kSoftmaxThreads, 0, s>>>(P);
  return launch_status("nt_row_softmax launch");
}

template <int DT, int NPL, int WARPS, bool BACKWARD>
static int launch_softmax(const SoftmaxParams& P, cudaStream_t s) {
  return P.vec ? launch_variant<DT, NPL, WARPS, BACKWARD, true>(P, s)
               : launch_variant<DT, NPL, WARPS, BACKWARD, false>(P, s);
}

template <int DT, bool BACKWARD>
static int dispatch_width(const SoftmaxParams& P, cudaStream_t s) {
  if (DT != NT_F32 && !BACKWARD) {   // float32 rows of 16-bit data: 16 values per thread up to 2048
    if (P.width <= 256) return launch_softmax<DT, 8, 1, BACKWARD>(P, s);
    if (P.width <= 512) return launch_softmax<DT, 16, 1, BACKWARD>(P, s);
    if (P.width <= 1024) return launch_softmax<DT, 16, 2, BACKWARD>(P, s);
    if (P.width <= 2048) return launch_softmax<DT, 16, 4, BACKWARD>(P, s);
    return launch_softmax<DT, 32, 4, BACKWARD>(P, s);
  }
  if (P.width <= 256) return launch_softmax<DT, 8, 1, BACKWARD>(P, s);
  if (P.width <= 512) return launch_softmax<DT, 16, 1, BACKWARD>(P, s);
  if (P.width <= 1024) return launch_softmax<DT, 32, 1, BACKWARD>(P, s);
  if (P.width <= 2048) return launch_softmax<DT, 32, 2, BACKWARD>(P, s);
  return launch_softmax<DT, 32, 4, BACKWARD>(P, s);
}

template <bool BACKWARD>
static int dispatch_dtype(const SoftmaxParams& P, int dtype, cudaStream_t s) {
  switch (dtype) {
    case NT_F32: return dispatch_width<NT_F32, BACKWARD>(P, s);
    case NT_F16: return dispatch_width<NT_F16, BACKWARD>(P, s);
    case NT_BF16: return dispatch_width<NT_BF16, BACKWARD>(P, s);
    default:
      set_error("nt_row_softmax: unsupported dtype %d", dtype);
      return NT_EUNSUPPORTED;
  }
}

}  // namespace nt

using namespace nt;

extern "C" {

int nt_row_softmax(const nt_softmax_args* args, void* stream) {
  nt::TraceRange trace("nt_row_softmax");
  if (!args) { set_error("nt_row_softmax: args is NULL"); return NT_EINVAL; }
  const nt_softmax_args& a = *args;
  if (a.op < NT_SOFTMAX || a.op > NT_CAUSAL_SOFTMAX_BACKWARD) {
    set_error("nt_row_softmax: unknown operation %d", a.op);
    return NT_EINVAL;
  }
  const bool backward = a.op >= NT_SOFTMAX_BACKWARD;
  const int kind = backward ? a.op - NT_SOFTMAX_BACKWARD : a.op;   // 0 plain, 1 masked, 2 causal
  if (a.rows < 0 || a.width < 0 || a.width > NT_SOFTMAX_MAX_WIDTH) {
    set_error("nt_row_softmax: width must be in [0, %d] and rows nonnegative", NT_SOFTMAX_MAX_WIDTH);
    return NT_EINVAL;
  }
  if (a.rows == 0 || a.width == 0) return NT_OK;
  if (!a.input || !a.output || (backward && !a.gradient)) {
    set_error("nt_row_softmax: NULL input/output%s", backward ? "/gradient" : "");
    return NT_EINVAL;
  }
  if (kind == 1 && !a.mask) { set_error("nt_row_softmax: masked softmax needs a mask"); return NT_EINVAL; }
  if (kind == 2 && a.queries < 1) { set_error("nt_row_softmax: causal softmax needs queries >= 1"); return NT_EINVAL; }
  if (a.mask_rows < 0 || a.offset < 0) { set_error("nt_row_softmax: negative mask_rows / offset"); return NT_EINVAL; }
  const int es = dtype_size(a.dtype);
  if (es == 0) { set_error("nt_row_softmax: unsupported dtype %d", a.dtype); return NT_EUNSUPPORTED; }
  SoftmaxParams P;
  P.x = a.input; P.g = a.gradient; P.mask = kind == 0 ? nullptr : a.mask; P.y = a.output;
  P.summary = backward ? nullptr : reinterpret_cast<unsigned long long*>(a.summary);
  P.rows = a.rows; P.width = (int)a.width; P.mask_rows = a.mask_rows;
  P.queries = a.queries < 1 ? 1 : a.queries;
  P.offset = a.offset < a.width ? a.offset : a.width;
  P.causal = kind == 2;
  const int epv = 16 / es;
  P.vec = aligned16(a.input) && aligned16(a.output) && (!backward || aligned16(a.gradient)) &&
          (a.width % epv) == 0;
  cudaStream_t s = as_stream(stream);
  return backward ? dispatch_dtype<true>(P, a.dtype, s) : dispatch_dtype<false>(P, a.dtype, s);
}

}  // extern "C"
