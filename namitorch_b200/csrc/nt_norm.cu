// RMS / layer normalization over the last dimension (rows of at most 8192 elements): the
// forward, input-gradient and affine-gradient stages of the reference's
// NormalizationCUDAKernels (namitorch/backends/cuda/normalization.py:58-157).
//
// Forward: a row stays in registers (one read, one write). Layer norm shifts the row by its
// first element (the reference's anchor), takes the mean and the second moment of the
// shifted values in two passes over the registers, and saves (shifted mean, 1/sqrt(var +
// eps)); RMS norm saves (0, 1/sqrt(mean(x^2) + eps)). y = normalized * weight + bias.
// Input gradient: dx = inverse * (g*w - mean(g*w) - normalized * mean(g*w * normalized)),
// without the mean(g*w) term for RMS norm, from the saved statistics.
// Affine gradient: dweight = sum over rows of g * normalized, dbias = sum of g, computed in
// the same pass as the input gradient. A thread keeps the same columns of every row it
// visits, so it sums them in registers; the row groups of a block are combined in shared
// memory and the block writes one partial row per column to the workspace; a second kernel
// sums the blocks' partial rows per column in a fixed order. The grid and the row order are
// fixed for a given shape and device, so the result does not depend on scheduling. (The
// reference splits the rows into tiles for the same reason and re-reads x and g; here x
// and g are read once for both gradients.)
// Half and bfloat16 tensors are computed in float32 (statistics and weight/bias gradients
// are float32).
#include <cmath>
#include <type_traits>

#include "nt_rows.cuh"

namespace nt {

struct NormParams {
  const void* x;
  const void* w;
  const void* b;
  void* y;
  float* stats;
  const void* g;
  void* dx;
  float* part_w;
  float* part_b;
  int64_t rows;
  int width;
  float eps;
};

template <int WARPS> struct NormShape {
  static constexpr int kThreads = WARPS * 32 > 128 ? WARPS * 32 : 128;
};

// Most blocks of the backward pass when the weight or bias gradient is requested: one
// partial row per block in the workspace.
constexpr int64_t kNormMaxSlots = 1024;

template <int DT, int NPL, int WARPS, bool LAYER, bool VEC>
__global__ void __launch_bounds__(NormShape<WARPS>::kThreads) norm_forward_kernel(const __grid_constant__ NormParams P) {
  constexpr int THREADS = NormShape<WARPS>::kThreads;
  __shared__ float smem[THREADS / 32];
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  constexpr int T = 32 * WARPS;
  constexpr int GROUPS = THREADS / T;
  const int t = threadIdx.x % T;
  const int group = threadIdx.x / T;
  const int width = P.width;
  const float fw = (float)width;
  for (int64_t first = (int64_t)blockIdx.x * GROUPS; first < P.rows; first += (int64_t)gridDim.x * GROUPS) {
    const int64_t row = first + group;
    const bool live = row < P.rows;
    const int64_t base = (live ? row : 0) * (int64_t)width;
    const char* xrow = static_cast<const char*>(P.x) + base * ES;
    float v[NPL];
    if (live) load_row<DT, NPL, WARPS>(xrow, width, t, VEC, v);
    else {
#pragma unroll
      for (int q = 0; q < NPL; ++q) v[q] = 0.0f;
    }
    float mean = 0.0f, inv;
    if constexpr (LAYER) {
      const float anchor = live ? load1<DT>(xrow, 0) : 0.0f;
      float sum = 0.0f;
#pragma unroll
      for (int q = 0; q < NPL; ++q) {
        const bool in = slot_column<EPV>(q, t, T, VEC) < width;
        v[q] = in ? __fsub_rn(v[q], anchor) : 0.0f;
        sum = __fadd_rn(sum, v[q]);
      }
      mean = __fdiv_rn(row_sum<WARPS>(sum, smem), fw);
      float m2 = 0.0f;
#pragma unroll
      for (int q = 0; q < NPL; ++q) {
        const float d = slot_column<EPV>(q, t, T, VEC) < width ? __fsub_rn(v[q], mean) : 0.0f;
        m2 = __fadd_rn(m2, __fmul_rn(d, d));
      }
      inv = rsqrtf(__fadd_rn(__fdiv_rn(row_sum<WARPS>(m2, smem), fw), P.eps));
    } else {
      float ss = 0.0f;
#pragma unroll
      for (int q = 0; q < NPL; ++q) ss = __fadd_rn(ss, __fmul_rn(v[q], v[q]));
      inv = rsqrtf(__fadd_rn(__fdiv_rn(row_sum<WARPS>(ss, smem), fw), P.eps));
    }
    if (live && t == 0 && P.stats != nullptr) {
      P.stats[2 * row] = mean;
      P.stats[2 * row + 1] = inv;
    }
#pragma unroll
    for (int c = 0; c < NPL / EPV; ++c) {
      float wv[EPV], bv[EPV];
      if (P.w != nullptr) load_group<DT, NPL, WARPS>(P.w, width, t, VEC, c, wv);
      if (P.b != nullptr) load_group<DT, NPL, WARPS>(P.b, width, t, VEC, c, bv);
#pragma unroll
      for (int e = 0; e < EPV; ++e) {
        const int q = c * EPV + e;
        float y = __fmul_rn(LAYER ? __fsub_rn(v[q], mean) : v[q], inv);
        if (P.w != nullptr) y = __fmul_rn(y, wv[e]);
        if (P.b != nullptr) y = __fadd_rn(y, bv[e]);
        v[q] = y;
      }
    }
    if (live) store_row<DT, NPL, WARPS>(static_cast<char*>(P.y) + base * ES, width, t, VEC, v);
  }
}

// Backward over rows: the input gradient (when P.dx is set) and, with AFFINE, the block's
// partial sums of g * normalized and g per column (when P.part_w / P.part_b are set).
template <int DT, int NPL, int WARPS, bool LAYER, bool VEC, bool AFFINE>
__global__ void __launch_bounds__(NormShape<WARPS>::kThreads) norm_backward_kernel(const __grid_constant__ NormParams P) {
  constexpr int THREADS = NormShape<WARPS>::kThreads;
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  constexpr int T = 32 * WARPS;
  constexpr int GROUPS = THREADS / T;
  constexpr int ACC = AFFINE ? NPL : 1;
  __shared__ float smem[THREADS / 32];
  __shared__ float combine[AFFINE && GROUPS > 1 ? 2 * (GROUPS - 1) * T * NPL : 1];
  const int t = threadIdx.x % T;
  const int group = threadIdx.x / T;
  const int width = P.width;
  const float fw = (float)width;
  const bool want_dx = P.dx != nullptr;
  float aw[ACC], ab[ACC];
#pragma unroll
  for (int q = 0; q < ACC; ++q) aw[q] = ab[q] = 0.0f;
  for (int64_t first = (int64_t)blockIdx.x * GROUPS; first < P.rows; first += (int64_t)gridDim.x * GROUPS) {
    const int64_t row = first + group;
    const bool live = row < P.rows;
    const int64_t r = live ? row : 0;
    const int64_t base = r * (int64_t)width;
    const char* xrow = static_cast<const char*>(P.x) + base * ES;
    float n[NPL], g[NPL];
    if (live) {
      load_row<DT, NPL, WARPS>(xrow, width, t, VEC, n);
      load_row<DT, NPL, WARPS>(static_cast<const char*>(P.g) + base * ES, width, t, VEC, g);
    } else {
#pragma unroll
      for (int q = 0; q < NPL; ++q) n[q] = g[q] = 0.0f;
    }
    const float mean = P.stats[2 * r], inv = P.stats[2 * r + 1];
    const float anchor = LAYER && live ? load1<DT>(xrow, 0) : 0.0f;
#pragma unroll
    for (int q = 0; q < NPL; ++q) {
      const bool in = live && slot_column<EPV>(q, t, T, VEC) < width;
      n[q] = in ? __fmul_rn(LAYER ? __fsub_rn(__fsub_rn(n[q], anchor), mean) : n[q], inv) : 0.0f;
    }
    if constexpr (AFFINE) {
#pragma unroll
      for (int q = 0; q < NPL; ++q) {
        aw[q] = __fadd_rn(aw[q], __fmul_rn(g[q], n[q]));
        ab[q] = __fadd_rn(ab[q], g[q]);
      }
    }
    if (want_dx) {
      if (P.w != nullptr) {
#pragma unroll
        for (int c = 0; c < NPL / EPV; ++c) {
          float wv[EPV];
          load_group<DT, NPL, WARPS>(P.w, width, t, VEC, c, wv);
#pragma unroll
          for (int e = 0; e < EPV; ++e) g[c * EPV + e] = __fmul_rn(g[c * EPV + e], wv[e]);
        }
      }
      float sg = 0.0f, sp = 0.0f;
#pragma unroll
      for (int q = 0; q < NPL; ++q) {
        sg = __fadd_rn(sg, g[q]);
        sp = __fadd_rn(sp, __fmul_rn(g[q], n[q]));
      }
      const float mg = LAYER ? __fdiv_rn(row_sum<WARPS>(sg, smem), fw) : 0.0f;
      const float mp = __fdiv_rn(row_sum<WARPS>(sp, smem), fw);
#pragma unroll
      for (int q = 0; q < NPL; ++q) n[q] = __fmul_rn(inv, __fsub_rn(__fsub_rn(g[q], mg), __fmul_rn(n[q], mp)));
      if (live) store_row<DT, NPL, WARPS>(static_cast<char*>(P.dx) + base * ES, width, t, VEC, n);
    }
  }
  if constexpr (AFFINE) {
    if constexpr (GROUPS > 1) {
      // Row groups 1.. hand their sums to group 0, which adds them in group order.
      if (group > 0) {
        float* slot = combine + (size_t)(group - 1) * 2 * T * NPL;
#pragma unroll
        for (int q = 0; q < NPL; ++q) {
          slot[q * T + t] = aw[q];
          slot[(NPL + q) * T + t] = ab[q];
        }
      }
      __syncthreads();
      if (group > 0) return;
#pragma unroll 1
      for (int k = 0; k < GROUPS - 1; ++k) {
        const float* slot = combine + (size_t)k * 2 * T * NPL;
#pragma unroll
        for (int q = 0; q < NPL; ++q) {
          aw[q] = __fadd_rn(aw[q], slot[q * T + t]);
          ab[q] = __fadd_rn(ab[q], slot[(NPL + q) * T + t]);
        }
      }
    }
    const int64_t row_out = (int64_t)blockIdx.x * width;
#pragma unroll
    for (int q = 0; q < NPL; ++q) {
      const int c = slot_column<EPV>(q, t, T, VEC);
      if (c < width) {
        if (P.part_w != nullptr) P.part_w[row_out + c] = aw[q];
        if (P.part_b != nullptr) P.part_b[row_out + c] = ab[q];
      }
    }
  }
}

constexpr int kReduceColumns = 32;
constexpr int kReduceLanes = 32;

// Column sums of the blocks' partial rows (blockIdx.y: 0 weight, 1 bias). Lane j of a
// column sums partial rows j, j + 32, ... in order; the 32 lane sums are then added in lane
// order.
__global__ void __launch_bounds__(kReduceColumns * kReduceLanes)
norm_affine_reduce_kernel(const float* part_w, const float* part_b, int64_t slots, int width, float* out_w, float* out_b) {
  __shared__ float lanes[kReduceLanes][kReduceColumns];
  const float* part = blockIdx.y == 0 ? part_w : part_b;
  float* out = blockIdx.y == 0 ? out_w : out_b;
  if (part == nullptr) return;
  const int col = threadIdx.x % kReduceColumns;
  const int lane = threadIdx.x / kReduceColumns;
  const int c = blockIdx.x * kReduceColumns + col;
  float s = 0.0f;
  if (c < width)
    for (int64_t k = lane; k < slots; k += kReduceLanes) s = __fadd_rn(s, part[k * width + c]);
  lanes[lane][col] = s;
  __syncthreads();
  if (lane == 0 && c < width) {
#pragma unroll
    for (int j = 1; j < kReduceLanes; ++j) s = __fadd_rn(s, lanes[j][col]);
    out[c] = s;
  }
}

// Grid of a row kernel: every resident block, no more blocks than row groups, and at most
// `cap` blocks. Returns the grid size it launched (0 on error).
template <typename K>
static int64_t launch_rows(K kernel, const NormParams& P, int threads, int groups, int64_t cap, cudaStream_t s) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm <= 0)
    per_sm = 2;
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  const int64_t need = (P.rows + groups - 1) / groups;
  if (grid > need) grid = need;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  kernel<<<(unsigned)grid, threads, 0, s>>>(P);
  return launch_status("nt_norm launch") == NT_OK ? grid : 0;
}

// Forward: returns the grid launched (0 on error).
template <int DT, int NPL, int WARPS, bool LAYER>
static int64_t launch_forward(const NormParams& P, bool vec, cudaStream_t s) {
  constexpr int THREADS = NormShape<WARPS>::kThreads;
  constexpr int GROUPS = THREADS / (32 * WARPS);
  const int64_t cap = INT32_MAX;
  return vec ? launch_rows(norm_forward_kernel<DT, NPL, WARPS, LAYER, true>, P, THREADS, GROUPS, cap, s)
             : launch_rows(norm_forward_kernel<DT, NPL, WARPS, LAYER, false>, P, THREADS, GROUPS, cap, s);
}

// Backward: returns the grid launched, which is the number of partial rows written when
// the affine sums are requested (0 on error).
template <int DT, int NPL, int WARPS, bool LAYER>
static int64_t launch_backward(const NormParams& P, bool vec, cudaStream_t s) {
  constexpr int THREADS = NormShape<WARPS>::kThreads;
  constexpr int GROUPS = THREADS / (32 * WARPS);
  if (P.part_w != nullptr || P.part_b != nullptr)
    return vec ? launch_rows(norm_backward_kernel<DT, NPL, WARPS, LAYER, true, true>, P, THREADS, GROUPS, kNormMaxSlots, s)
               : launch_rows(norm_backward_kernel<DT, NPL, WARPS, LAYER, false, true>, P, THREADS, GROUPS, kNormMaxSlots, s);
  return vec ? launch_rows(norm_backward_kernel<DT, NPL, WARPS, LAYER, true, false>, P, THREADS, GROUPS, INT32_MAX, s)
             : launch_rows(norm_backward_kernel<DT, NPL, WARPS, LAYER, false, false>, P, THREADS, GROUPS, INT32_MAX, s);
}

// Row shapes (values per thread, warps per row) by width: at most 16 values per thread, so
// that the registers leave room for the warps that hide memory latency (at width 2048, 16
// values over 4 warps beat 32 over 2 warps and 8 over 8 warps in both passes, f32 and bf16).
template <int DT, bool LAYER, bool BACKWARD>
static int64_t dispatch_norm_width(const NormParams& P, bool vec, cudaStream_t s) {
  constexpr auto launch = [](const NormParams& p, bool v, cudaStream_t st, auto npl, auto warps) {
    if constexpr (BACKWARD) return launch_backward<DT, decltype(npl)::value, decltype(warps)::value, LAYER>(p, v, st);
    else return launch_forward<DT, decltype(npl)::value, decltype(warps)::value, LAYER>(p, v, st);
  };
  using I8 = std::integral_constant<int, 8>;
  using I16 = std::integral_constant<int, 16>;
  if (P.width <= 256) return launch(P, vec, s, I8{}, std::integral_constant<int, 1>{});
  if (P.width <= 512) return launch(P, vec, s, I16{}, std::integral_constant<int, 1>{});
  if (P.width <= 1024) return launch(P, vec, s, I16{}, std::integral_constant<int, 2>{});
  if (P.width <= 2048) return launch(P, vec, s, I16{}, std::integral_constant<int, 4>{});
  if (P.width <= 4096) return launch(P, vec, s, I16{}, std::integral_constant<int, 8>{});
  return launch(P, vec, s, I16{}, std::integral_constant<int, 16>{});
}

template <bool BACKWARD>
static int64_t dispatch_norm(const NormParams& P, int dtype, bool layer, bool vec, cudaStream_t s) {
  switch (dtype) {
    case NT_F32: return layer ? dispatch_norm_width<NT_F32, true, BACKWARD>(P, vec, s)
                              : dispatch_norm_width<NT_F32, false, BACKWARD>(P, vec, s);
    case NT_F16: return layer ? dispatch_norm_width<NT_F16, true, BACKWARD>(P, vec, s)
                              : dispatch_norm_width<NT_F16, false, BACKWARD>(P, vec, s);
    default: return layer ? dispatch_norm_width<NT_BF16, true, BACKWARD>(P, vec, s)
                          : dispatch_norm_width<NT_BF16, false, BACKWARD>(P, vec, s);
  }
}

static int check_norm(const nt_norm_args& a, const char* who) {
  if (a.op != NT_RMS_NORM && a.op != NT_LAYER_NORM) { set_error("%s: unknown operation %d", who, a.op); return NT_EINVAL; }
  if (a.rows < 0 || a.width < 1 || a.width > NT_NORM_MAX_WIDTH) {
    set_error("%s: width must be in [1, %d] and rows nonnegative", who, NT_NORM_MAX_WIDTH);
    return NT_EINVAL;
  }
  if (dtype_size(a.dtype) == 0) { set_error("%s: unsupported dtype %d", who, a.dtype); return NT_EUNSUPPORTED; }
  if (a.bias && a.op != NT_LAYER_NORM) { set_error("%s: RMS norm takes no bias", who); return NT_EINVAL; }
  return NT_OK;
}

static bool norm_vec(const nt_norm_args& a, std::initializer_list<const void*> ptrs) {
  const int epv = 16 / dtype_size(a.dtype);
  if (a.width % epv) return false;
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return false;
  return true;
}

}  // namespace nt

using namespace nt;

extern "C" {

size_t nt_norm_workspace_size(int64_t rows, int64_t width) {
  if (rows < 1 || width < 1) return 0;
  const int64_t slots = rows < kNormMaxSlots ? rows : kNormMaxSlots;
  return (size_t)slots * (size_t)width * 2 * sizeof(float);
}

int nt_norm_forward(const nt_norm_args* args, void* stream) {
  nt::TraceRange trace("nt_norm_forward");
  if (!args) { set_error("nt_norm_forward: args is NULL"); return NT_EINVAL; }
  const nt_norm_args& a = *args;
  int rc = check_norm(a, "nt_norm_forward");
  if (rc) return rc;
  if (a.rows == 0) return NT_OK;
  if (!a.input || !a.output) { set_error("nt_norm_forward: NULL input/output"); return NT_EINVAL; }
  if (!(a.eps > 0.0f) || !isfinite(a.eps)) { set_error("nt_norm_forward: eps must be positive and finite"); return NT_EINVAL; }
  NormParams P{};
  P.x = a.input; P.w = a.weight; P.b = a.bias; P.y = a.output; P.stats = a.statistics;
  P.rows = a.rows; P.width = (int)a.width; P.eps = a.eps;
  const bool vec = norm_vec(a, {a.input, a.output, a.weight, a.bias});
  return dispatch_norm<false>(P, a.dtype, a.op == NT_LAYER_NORM, vec, as_stream(stream)) > 0 ? NT_OK : NT_ECUDA;
}

int nt_norm_backward(const nt_norm_args* args, void* stream) {
  nt::TraceRange trace("nt_norm_backward");
  if (!args) { set_error("nt_norm_backward: args is NULL"); return NT_EINVAL; }
  const nt_norm_args& a = *args;
  int rc = check_norm(a, "nt_norm_backward");
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  const bool affine = a.grad_weight || a.grad_bias;
  if (a.rows == 0) {
    if (a.grad_weight) { cudaError_t e = cudaMemsetAsync(a.grad_weight, 0, a.width * 4, s); if (e) return cuda_fail(e, "nt_norm_backward"); }
    if (a.grad_bias) { cudaError_t e = cudaMemsetAsync(a.grad_bias, 0, a.width * 4, s); if (e) return cuda_fail(e, "nt_norm_backward"); }
    return NT_OK;
  }
  if (!a.input || !a.gradient || !a.statistics) {
    set_error("nt_norm_backward: NULL input/gradient/statistics");
    return NT_EINVAL;
  }
  if (affine) {
    const size_t need = nt_norm_workspace_size(a.rows, a.width);
    if (!a.workspace || a.workspace_bytes < need) {
      set_error("nt_norm_backward: weight/bias gradients need a workspace of %zu bytes (got %zu)", need, a.workspace_bytes);
      return NT_EINVAL;
    }
  } else if (!a.grad_input) {
    return NT_OK;
  }
  NormParams P{};
  P.x = a.input; P.w = a.weight; P.g = a.gradient; P.dx = a.grad_input; P.stats = a.statistics;
  P.rows = a.rows; P.width = (int)a.width;
  float* part = static_cast<float*>(a.workspace);
  const int64_t slot_cap = a.rows < kNormMaxSlots ? a.rows : kNormMaxSlots;
  P.part_w = a.grad_weight ? part : nullptr;
  P.part_b = a.grad_bias ? part + slot_cap * a.width : nullptr;
  const bool vec = norm_vec(a, {a.input, a.gradient, a.grad_input, a.weight});
  const int64_t slots = dispatch_norm<true>(P, a.dtype, a.op == NT_LAYER_NORM, vec, s);
  if (slots <= 0) return NT_ECUDA;
  if (!affine) return NT_OK;
  const dim3 grid((unsigned)((a.width + kReduceColumns - 1) / kReduceColumns), 2);
  norm_affine_reduce_kernel<<<grid, kReduceColumns * kReduceLanes, 0, s>>>(P.part_w, P.part_b, slots, P.width,
                                                                           a.grad_weight, a.grad_bias);
  return launch_status("nt_norm_backward (reduce) launch");
}

}  // extern "C"
