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
// Affine gradient: dweight = sum over rows of g * normalized, dbias = sum of g. Each block
// owns a tile of rows and a tile of columns (a thread per column, coalesced across the
// warp), writes per-tile partial sums to the workspace, and a second kernel sums the tiles
// per column in a fixed order, so the result does not depend on scheduling.
// Half and bfloat16 tensors are computed in float32 (statistics and weight/bias gradients
// are float32).
#include <cmath>

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
  int64_t tile_rows;
  int64_t row_tiles;
};

template <int WARPS> struct NormShape {
  static constexpr int kThreads = WARPS * 32 > 128 ? WARPS * 32 : 128;
};

// Tiles of rows of the affine-gradient stage: enough tiles for every SM, at most 1024.
static int64_t norm_row_tiles(int64_t rows, int64_t width) {
  const int64_t col_tiles = (width + 255) / 256;
  int64_t tiles = (4 * 148 + col_tiles - 1) / col_tiles;
  if (tiles > rows) tiles = rows;
  if (tiles > 1024) tiles = 1024;
  return tiles < 1 ? 1 : tiles;
}

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
    float wv[NPL], bv[NPL];
    if (P.w != nullptr) load_row<DT, NPL, WARPS>(P.w, width, t, VEC, wv);
    if (P.b != nullptr) load_row<DT, NPL, WARPS>(P.b, width, t, VEC, bv);
#pragma unroll
    for (int q = 0; q < NPL; ++q) {
      float y = __fmul_rn(LAYER ? __fsub_rn(v[q], mean) : v[q], inv);
      if (P.w != nullptr) y = __fmul_rn(y, wv[q]);
      if (P.b != nullptr) y = __fadd_rn(y, bv[q]);
      v[q] = y;
    }
    if (live) store_row<DT, NPL, WARPS>(static_cast<char*>(P.y) + base * ES, width, t, VEC, v);
  }
}

template <int DT, int NPL, int WARPS, bool LAYER, bool VEC>
__global__ void __launch_bounds__(NormShape<WARPS>::kThreads) norm_input_grad_kernel(const __grid_constant__ NormParams P) {
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
    const int64_t r = live ? row : 0;
    const int64_t base = r * (int64_t)width;
    const char* xrow = static_cast<const char*>(P.x) + base * ES;
    float n[NPL], wg[NPL];
    if (live) {
      load_row<DT, NPL, WARPS>(xrow, width, t, VEC, n);
      load_row<DT, NPL, WARPS>(static_cast<const char*>(P.g) + base * ES, width, t, VEC, wg);
    } else {
#pragma unroll
      for (int q = 0; q < NPL; ++q) n[q] = wg[q] = 0.0f;
    }
    const float mean = P.stats[2 * r], inv = P.stats[2 * r + 1];
    const float anchor = LAYER && live ? load1<DT>(xrow, 0) : 0.0f;
    if (P.w != nullptr) {
      float wv[NPL];
      load_row<DT, NPL, WARPS>(P.w, width, t, VEC, wv);
#pragma unroll
      for (int q = 0; q < NPL; ++q) wg[q] = __fmul_rn(wg[q], wv[q]);
    }
    float sg = 0.0f, sp = 0.0f;
#pragma unroll
    for (int q = 0; q < NPL; ++q) {
      const bool in = slot_column<EPV>(q, t, T, VEC) < width;
      n[q] = in ? __fmul_rn(LAYER ? __fsub_rn(__fsub_rn(n[q], anchor), mean) : n[q], inv) : 0.0f;
      sg = __fadd_rn(sg, wg[q]);
      sp = __fadd_rn(sp, __fmul_rn(wg[q], n[q]));
    }
    const float mg = LAYER ? __fdiv_rn(row_sum<WARPS>(sg, smem), fw) : 0.0f;
    const float mp = __fdiv_rn(row_sum<WARPS>(sp, smem), fw);
#pragma unroll
    for (int q = 0; q < NPL; ++q) n[q] = __fmul_rn(inv, __fsub_rn(__fsub_rn(wg[q], mg), __fmul_rn(n[q], mp)));
    if (live) store_row<DT, NPL, WARPS>(static_cast<char*>(P.dx) + base * ES, width, t, VEC, n);
  }
}

constexpr int kAffineThreads = 256;

// Block (row tile, column tile): a thread per column sums g * normalized and g over the
// tile's rows (4 rows in flight) and writes the tile's partial sums.
template <int DT, bool LAYER>
__global__ void __launch_bounds__(kAffineThreads) norm_affine_partial_kernel(const __grid_constant__ NormParams P) {
  const int col_tiles = (P.width + kAffineThreads - 1) / kAffineThreads;
  const int64_t tiles = P.row_tiles * col_tiles;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t rt = tile / col_tiles;
    const int c = (int)(tile % col_tiles) * kAffineThreads + threadIdx.x;
    if (c >= P.width) continue;
    const int64_t r0 = rt * P.tile_rows;
    const int64_t r1 = r0 + P.tile_rows < P.rows ? r0 + P.tile_rows : P.rows;
    float sw = 0.0f, sb = 0.0f;
    int64_t r = r0;
    for (; r + 4 <= r1; r += 4) {
      float xg[4], gg[4], an[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t base = (r + u) * (int64_t)P.width;
        xg[u] = load1<DT>(P.x, base + c);
        gg[u] = load1<DT>(P.g, base + c);
        an[u] = LAYER ? load1<DT>(P.x, base) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float mean = P.stats[2 * (r + u)], inv = P.stats[2 * (r + u) + 1];
        const float nrm = __fmul_rn(LAYER ? __fsub_rn(__fsub_rn(xg[u], an[u]), mean) : xg[u], inv);
        sw = __fadd_rn(sw, __fmul_rn(gg[u], nrm));
        sb = __fadd_rn(sb, gg[u]);
      }
    }
    for (; r < r1; ++r) {
      const int64_t base = r * (int64_t)P.width;
      const float mean = P.stats[2 * r], inv = P.stats[2 * r + 1];
      const float gv = load1<DT>(P.g, base + c);
      const float xv = load1<DT>(P.x, base + c);
      const float nrm = __fmul_rn(LAYER ? __fsub_rn(__fsub_rn(xv, load1<DT>(P.x, base)), mean) : xv, inv);
      sw = __fadd_rn(sw, __fmul_rn(gv, nrm));
      sb = __fadd_rn(sb, gv);
    }
    if (P.part_w != nullptr) P.part_w[rt * P.width + c] = sw;
    if (P.part_b != nullptr) P.part_b[rt * P.width + c] = sb;
  }
}

// Column sums of the partial tiles, in tile order.
__global__ void norm_affine_reduce_kernel(const float* part, int64_t tiles, int width, float* out) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < width; c += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int64_t k = 0; k < tiles; ++k) s = __fadd_rn(s, part[k * width + c]);
    out[c] = s;
  }
}

template <typename K>
static int launch_rows(K kernel, const NormParams& P, int threads, int groups, cudaStream_t s) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm <= 0)
    per_sm = 2;
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  const int64_t need = (P.rows + groups - 1) / groups;
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  kernel<<<(unsigned)grid, threads, 0, s>>>(P);
  return launch_status("nt_norm launch");
}

template <int DT, int NPL, int WARPS, bool LAYER, bool BACKWARD>
static int launch_norm(const NormParams& P, bool vec, cudaStream_t s) {
  constexpr int THREADS = NormShape<WARPS>::kThreads;
  constexpr int GROUPS = THREADS / (32 * WARPS);
  if constexpr (BACKWARD) {
    return vec ? launch_rows(norm_input_grad_kernel<DT, NPL, WARPS, LAYER, true>, P, THREADS, GROUPS, s)
               : launch_rows(norm_input_grad_kernel<DT, NPL, WARPS, LAYER, false>, P, THREADS, GROUPS, s);
  } else {
    return vec ? launch_rows(norm_forward_kernel<DT, NPL, WARPS, LAYER, true>, P, THREADS, GROUPS, s)
               : launch_rows(norm_forward_kernel<DT, NPL, WARPS, LAYER, false>, P, THREADS, GROUPS, s);
  }
}

template <int DT, bool LAYER, bool BACKWARD>
static int dispatch_norm_width(const NormParams& P, bool vec, cudaStream_t s) {
  if (P.width <= 256) return launch_norm<DT, 8, 1, LAYER, BACKWARD>(P, vec, s);
  if (P.width <= 512) return launch_norm<DT, 16, 1, LAYER, BACKWARD>(P, vec, s);
  if (P.width <= 1024) return launch_norm<DT, 32, 1, LAYER, BACKWARD>(P, vec, s);
  if (P.width <= 2048) return launch_norm<DT, 32, 2, LAYER, BACKWARD>(P, vec, s);
  if (P.width <= 4096) return launch_norm<DT, 32, 4, LAYER, BACKWARD>(P, vec, s);
  return launch_norm<DT, 32, 8, LAYER, BACKWARD>(P, vec, s);
}

template <bool BACKWARD>
static int dispatch_norm(const NormParams& P, int dtype, bool layer, bool vec, cudaStream_t s) {
  switch (dtype) {
    case NT_F32: return layer ? dispatch_norm_width<NT_F32, true, BACKWARD>(P, vec, s)
                              : dispatch_norm_width<NT_F32, false, BACKWARD>(P, vec, s);
    case NT_F16: return layer ? dispatch_norm_width<NT_F16, true, BACKWARD>(P, vec, s)
                              : dispatch_norm_width<NT_F16, false, BACKWARD>(P, vec, s);
    case NT_BF16: return layer ? dispatch_norm_width<NT_BF16, true, BACKWARD>(P, vec, s)
                               : dispatch_norm_width<NT_BF16, false, BACKWARD>(P, vec, s);
    default:
      set_error("nt_norm: unsupported dtype %d", dtype);
      return NT_EUNSUPPORTED;
  }
}

template <int DT>
static int launch_affine(const NormParams& P, bool layer, cudaStream_t s) {
  const int64_t col_tiles = (P.width + kAffineThreads - 1) / kAffineThreads;
  int64_t grid = P.row_tiles * col_tiles;
  const int64_t cap = (int64_t)current_sm_count() * 8;
  if (grid > cap) grid = cap;
  if (layer) norm_affine_partial_kernel<DT, true><<<(unsigned)grid, kAffineThreads, 0, s>>>(P);
  else norm_affine_partial_kernel<DT, false><<<(unsigned)grid, kAffineThreads, 0, s>>>(P);
  return launch_status("nt_norm_backward (affine) launch");
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
  return (size_t)norm_row_tiles(rows, width) * (size_t)width * 2 * sizeof(float);
}

int nt_norm_forward(const nt_norm_args* args, void* stream) {
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
  return dispatch_norm<false>(P, a.dtype, a.op == NT_LAYER_NORM, vec, as_stream(stream));
}

int nt_norm_backward(const nt_norm_args* args, void* stream) {
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
  NormParams P{};
  P.x = a.input; P.w = a.weight; P.g = a.gradient; P.dx = a.grad_input; P.stats = a.statistics;
  P.rows = a.rows; P.width = (int)a.width;
  if (a.grad_input) {
    const bool vec = norm_vec(a, {a.input, a.gradient, a.grad_input, a.weight});
    rc = dispatch_norm<true>(P, a.dtype, a.op == NT_LAYER_NORM, vec, s);
    if (rc) return rc;
  }
  if (!affine) return NT_OK;
  const size_t need = nt_norm_workspace_size(a.rows, a.width);
  if (!a.workspace || a.workspace_bytes < need) {
    set_error("nt_norm_backward: weight/bias gradients need a workspace of %zu bytes (got %zu)", need, a.workspace_bytes);
    return NT_EINVAL;
  }
  P.row_tiles = norm_row_tiles(a.rows, a.width);
  P.tile_rows = (a.rows + P.row_tiles - 1) / P.row_tiles;
  float* part = static_cast<float*>(a.workspace);
  P.part_w = a.grad_weight ? part : nullptr;
  P.part_b = a.grad_bias ? part + P.row_tiles * a.width : nullptr;
  const bool layer = a.op == NT_LAYER_NORM;
  switch (a.dtype) {
    case NT_F32: rc = launch_affine<NT_F32>(P, layer, s); break;
    case NT_F16: rc = launch_affine<NT_F16>(P, layer, s); break;
    default: rc = launch_affine<NT_BF16>(P, layer, s); break;
  }
  if (rc) return rc;
  const int blocks = (int)((a.width + 255) / 256);
  if (a.grad_weight) norm_affine_reduce_kernel<<<blocks, 256, 0, s>>>(P.part_w, P.row_tiles, P.width, a.grad_weight);
  if (a.grad_bias) norm_affine_reduce_kernel<<<blocks, 256, 0, s>>>(P.part_b, P.row_tiles, P.width, a.grad_bias);
  return launch_status("nt_norm_backward (reduce) launch");
}

}  // extern "C"
