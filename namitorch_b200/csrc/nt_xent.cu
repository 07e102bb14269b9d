// Fused softmax cross-entropy forward + backward.
//
// Math (per row i with target t, logits x, class weights w (1 without), smoothing e, V classes):
//   M = max x,  S = sum exp(x - M),  lse = M + log S,  logp = x - lse,  p = exp(x - M) / S
//   loss_i = (1-e) * (-w_t * logp_t) + e * (-(1/V) * sum_c w_c * logp_c)
//   dloss_i/dx_c = (1-e) * w_t * (p_c - [c==t]) + (e/V) * (p_c * W - w_c),   W = sum_c w_c
// reduced by 'mean' (divide by sum of w_t over non-ignored rows), 'sum' or 'none'
// (namitorch/nn/functional.py:819-863; log_softmax forward namitorch/_backend.py:321-354;
// backward namitorch/autograd.py:538-564, whose rows of all -inf get a zero gradient).
// Non-finite rows follow the reference: a NaN or +inf logit makes the whole row NaN;
// a row of all -inf has loss +inf and zero gradient.
//
// Data movement: each CTA is persistent over rows. A row (V * esize bytes, not 16-byte
// aligned in general) is fetched with one cp.async.bulk from the 16-byte boundary at or
// below its start into shared memory, completion tracked by an mbarrier; the few bytes
// past the last 16-byte boundary of the whole tensor are loaded with plain loads. Three
// passes then run from shared memory (max, sum of exp, gradient), and the gradient is
// written with 16-byte streaming stores at the same alignment offset. HBM traffic is one
// read of the logits and one write of dlogits.
#include <cmath>

#include "nt_bulk.cuh"

namespace nt {

constexpr int kPrepThreads = 1024;

struct XentWorkspace {
  unsigned counter;
  unsigned pad[63];
};

struct XentParams {
  const void* logits;
  void* dl;
  const int64_t* targets;
  const float* weight;
  int64_t rows;
  int64_t classes;
  int64_t ignore;
  float smoothing;
  int reduction;
  float* loss;
  float* row_loss;
  nt_xent_info* info;
  XentWorkspace* ws;
  uintptr_t tensor_end;   // one past the last byte of the logits
  int staged;
  int64_t stage_stride;   // bytes per staged row buffer
};

// 2^x on the SFU. Results below 2^-126 flush to zero: a logit that far below the row max
// contributes nothing to the sum and its gradient is below 2^-126 times the row scale.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;

template <int DT>
__device__ __forceinline__ uint4 pack16(const float* v) {
  uint4 raw;
  if constexpr (DT == NT_BF16) {
    __nv_bfloat162 h[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    raw = *reinterpret_cast<uint4*>(h);
    return raw;
  }
  if constexpr (DT == NT_F32) {
    raw.x = __float_as_uint(v[0]); raw.y = __float_as_uint(v[1]);
    raw.z = __float_as_uint(v[2]); raw.w = __float_as_uint(v[3]);
  } else {
    using T = typename Elem<DT>::T;
    T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] = Elem<DT>::from_f32(v[k]);
  }
  return raw;
}

__global__ void __launch_bounds__(kPrepThreads) xent_prepare_kernel(const __grid_constant__ XentParams P) {
  __shared__ double red[kPrepThreads / 32];
  double valid = 0.0, bad = 0.0, den = 0.0, wsum = 0.0;
  for (int64_t i = threadIdx.x; i < P.rows; i += blockDim.x) {
    const int64_t t = P.targets[i];
    if (t == P.ignore) continue;
    if (t < 0 || t >= P.classes) { bad += 1.0; continue; }
    valid += 1.0;
    den += P.weight ? (double)P.weight[t] : 1.0;
  }
  if (P.weight) {
    for (int64_t c = threadIdx.x; c < P.classes; c += blockDim.x) wsum += (double)P.weight[c];
  }
  valid = block_reduce(valid, red, SumOp(), 0.0);
  bad = block_reduce(bad, red, SumOp(), 0.0);
  den = block_reduce(den, red, SumOp(), 0.0);
  wsum = block_reduce(wsum, red, SumOp(), 0.0);
  if (threadIdx.x == 0) {
    nt_xent_info* info = P.info;
    info->n_valid = valid;
    info->bad_targets = bad;
    info->denominator = den;
    info->weight_sum = P.weight ? wsum : (double)P.classes;
    info->loss_sum = 0.0;
    info->error = 0.0;
    if (P.rows == 0 && P.reduction != NT_REDUCTION_NONE) P.loss[0] = 0.0f;
  }
}

// One 16-byte vector k of the row (EPV elements starting at element j0).
template <int DT, int STAGES>
__device__ __forceinline__ void row_vector(const unsigned char* stage, const void* logits, int64_t row_base,
                                           int k, int j0, int V, float* x) {
  constexpr int EPV = DT == NT_F32 ? 4 : 8;
  if constexpr (STAGES > 0) {
    uint4 raw;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(raw.x), "=r"(raw.y), "=r"(raw.z), "=r"(raw.w)
                 : "r"(smem_u32(stage) + (uint32_t)k * 16u));
    unpack16<DT>(raw, x);
  } else {
#pragma unroll
    for (int q = 0; q < EPV; ++q) {
      const int j = j0 + q;
      x[q] = (j >= 0 && j < V) ? load1<DT>(logits, row_base + j) : -INFINITY;
    }
  }
}

// Issues the bulk copy of `row` into `buf` (thread 0) and loads the bytes between the last
// 16-byte boundary of the tensor and its end with plain loads (all threads). The copy starts
// at the 16-byte boundary at or below the row start; the kernel indexes from the offset.
template <int ES>
__device__ __forceinline__ void stage_row(const XentParams& P, int64_t row, unsigned char* buf, uint64_t* bar) {
  const uintptr_t start = reinterpret_cast<uintptr_t>(P.logits) + (uintptr_t)(row * P.classes * ES);
  const uintptr_t a = start & ~(uintptr_t)15;
  const int span = (int)(start - a) + (int)P.classes * ES;
  int64_t bulk = (int64_t)((span + 15) >> 4) * 16;
  const uintptr_t limit = P.tensor_end & ~(uintptr_t)15;
  if ((int64_t)(limit - a) < bulk) bulk = (int64_t)(limit - a);
  if (threadIdx.x == 0) {
    fence_proxy_async();
    mbar_arrive_expect_tx(bar, (uint32_t)bulk);
    if (bulk > 0) bulk_g2s(buf, reinterpret_cast<const void*>(a), (uint32_t)bulk, bar);
  }
  for (int k = (int)bulk + threadIdx.x; k < span; k += blockDim.x) buf[k] = *reinterpret_cast<const unsigned char*>(a + k);
}

// STAGES = 2: double-buffered rows (the next row's copy is in flight while this one is
// processed); 1: one staged row at a time (rows too large for two buffers); 0: no
// staging (unaligned tensors), values read from global memory.
template <int DT, int STAGES, bool WEIGHTED, int THREADS>
__global__ void __launch_bounds__(THREADS) xent_kernel(const __grid_constant__ XentParams P) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bars[2];
  __shared__ float red_f[THREADS / 32];
  __shared__ float red_pair[THREADS / 32];
  __shared__ double red_d[THREADS / 32];
  __shared__ bool last;
  __shared__ int abort_flag;

  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;  // elements per 16-byte vector
  const int V = (int)P.classes;
  const nt_xent_info* info = P.info;
  const bool mean = P.reduction == NT_REDUCTION_MEAN;
  const double D = mean ? info->denominator : 1.0;
  const bool zero_all = mean && D == 0.0;
  const double W = info->weight_sum;
  const float inv_den = zero_all ? 0.0f : (float)(1.0 / D);
  const float e = P.smoothing;
  const bool smooth = e != 0.0f;

  if (STAGES > 0) {
    if (threadIdx.x == 0) {
      mbar_init(&bars[0], 1);
      mbar_init(&bars[1], 1);
      abort_flag = 0;
      fence_proxy_async();
    }
    __syncthreads();
  }
  uint32_t phase0 = 0, phase1 = 0;
  int64_t row = blockIdx.x;
  if (STAGES > 0 && row < P.rows) stage_row<ES>(P, row, smem, &bars[0]);

  for (int it = 0; row < P.rows; row += gridDim.x, ++it) {
    const int buf = STAGES == 2 ? (it & 1) : 0;
    const unsigned char* stage = smem + (size_t)buf * P.stage_stride;
    const int64_t next = row + gridDim.x;
    if (STAGES == 2 && next < P.rows)
      stage_row<ES>(P, next, smem + (size_t)(buf ^ 1) * P.stage_stride, &bars[buf ^ 1]);
    if (STAGES > 0) {
      if (threadIdx.x == 0 && !wait_stage(&bars[buf], buf ? phase1 : phase0)) abort_flag = 1;
      __syncthreads();
      if (buf) phase1 ^= 1u; else phase0 ^= 1u;
      if (abort_flag) {
        if (threadIdx.x == 0) {
          atomicAdd(&P.info->error, 1.0);
          // Let a copy still in flight into the other buffer land (bounded) before leaving.
          if (STAGES == 2 && next < P.rows) wait_stage(&bars[buf ^ 1], buf ? phase0 : phase1);
        }
        return;
      }
    }

    const int64_t t64 = P.targets[row];
    const bool valid = t64 != P.ignore && t64 >= 0 && t64 < V;
    const int t = valid ? (int)t64 : -1;
    const int64_t row_base = row * (int64_t)V;
    const uintptr_t start = reinterpret_cast<uintptr_t>(P.logits) + (uintptr_t)(row_base * ES);
    const int head = (int)(start & 15u);
    const int span = head + V * ES;           // bytes from the 16-byte boundary to the row end
    const int nvec = (span + 15) >> 4;
    const int full_lo = head ? 1 : 0;         // vectors [full_lo, full_hi) hold only row elements
    const int full_hi = span >> 4;
    const int dj = THREADS * EPV;

    // Pass A: online max / sum of exp per thread. The running max propagates NaN
    // (max.NaN.f32), so one value carries both; label smoothing also needs sum_c w_c x_c.
    // Interior vectors need no bounds checks; the <= 2 edge vectors of the row are
    // masked and taken by the first threads after the interior loop.
    float m = -INFINITY, s = 0.0f;
    double swx = 0.0;
    auto accumulate = [&](const float* x, int j0, bool edge) {
      float vmax = x[0];
#pragma unroll
      for (int q = 1; q < EPV; ++q) vmax = max_nan(vmax, x[q]);
      const float mn = max_nan(m, vmax);
      if (mn != m) {
        s = m > -INFINITY ? s * ex2((m - mn) * kLog2e) : 0.0f;
        m = mn;
      }
      if (m > -INFINITY) {
        const float sh = m * kLog2e;
#pragma unroll
        for (int q = 0; q < EPV; ++q) s += ex2(fmaf(x[q], kLog2e, -sh));
      }
      if (smooth) {
#pragma unroll
        for (int q = 0; q < EPV; ++q) {
          const int j = j0 + q;
          if (!edge || (j >= 0 && j < V)) swx += WEIGHTED ? (double)P.weight[j] * (double)x[q] : (double)x[q];
        }
      }
    };
    {
      int j0 = ((full_lo + (int)threadIdx.x) * 16 - head) / ES;
      for (int k = full_lo + threadIdx.x; k < full_hi; k += THREADS, j0 += dj) {
        float x[EPV];
        row_vector<DT, STAGES>(stage, P.logits, row_base, k, j0, V, x);
        accumulate(x, j0, false);
      }
      // Edge vectors: the head vector when the row starts inside it and the tail vector when the
      // row ends inside it; one vector when the whole row fits in it.
      const int nedge = full_lo + ((full_hi < nvec && full_hi >= full_lo) ? 1 : 0);
      if ((int)threadIdx.x < nedge) {
        const int k = (threadIdx.x == 0 && full_lo) ? 0 : full_hi;
        const int j0e = (k * 16 - head) / ES;
        float x[EPV];
        row_vector<DT, STAGES>(stage, P.logits, row_base, k, j0e, V, x);
#pragma unroll
        for (int q = 0; q < EPV; ++q)
          if (j0e + q < 0 || j0e + q >= V) x[q] = -INFINITY;
        accumulate(x, j0e, true);
      }
    }
    // One block-wide merge of the (max, sum) pairs, in a fixed order.
    {
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        const float mm = max_nan(m, m2);
        s = mm > -INFINITY ? (m > -INFINITY ? s * ex2((m - mm) * kLog2e) : 0.0f) +
                                 (m2 > -INFINITY ? s2 * ex2((m2 - mm) * kLog2e) : 0.0f)
                           : 0.0f;
        m = mm;
      }
      if (lane == 0) { red_f[warp] = m; red_pair[warp] = s; }
      __syncthreads();
      float M0 = -INFINITY;
#pragma unroll 4
      for (int w = 0; w < THREADS / 32; ++w) M0 = max_nan(M0, red_f[w]);
      float S0 = 0.0f;
      if (M0 > -INFINITY) {
#pragma unroll 4
        for (int w = 0; w < THREADS / 32; ++w)
          if (red_f[w] > -INFINITY) S0 += red_pair[w] * ex2((red_f[w] - M0) * kLog2e);
      }
      m = M0;
      s = S0;
    }
    const float M = m;
    const float S = s;
    if (smooth) swx = block_reduce(swx, red_d, SumOp(), 0.0);
    const bool bad_row = M != M || M == INFINITY;
    const bool neg_row = !bad_row && M == -INFINITY;

    // Row loss and the gradient coefficients: d_c = e_c * A - G_c, minus B at c == t.
    const float wt = valid ? (WEIGHTED ? P.weight[t] : 1.0f) : 0.0f;
    int mode = 0;  // 0: zero row, 1: NaN row, 2: regular
    float loss_i = 0.0f, A = 0.0f, B = 0.0f, G = 0.0f;
    if (valid && !zero_all) {
      if (bad_row) {
        mode = 1;
        loss_i = __int_as_float(0x7fc00000);
      } else if (neg_row) {
        loss_i = INFINITY;
      } else {
        mode = 2;
        float xt;
        if constexpr (STAGES > 0) {
          const int off = head + t * ES;
          if constexpr (DT == NT_F32) xt = *reinterpret_cast<const float*>(stage + off);
          else if constexpr (DT == NT_BF16) xt = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(stage + off));
          else xt = __half2float(*reinterpret_cast<const __half*>(stage + off));
        } else {
          xt = load1<DT>(P.logits, row_base + t);
        }
        const float lse = M + logf(S);
        const float base = -wt * (xt - lse);
        if (smooth) {
          const double sm = -(swx - (double)lse * W) / (double)V;
          loss_i = (1.0f - e) * base + e * (float)sm;
        } else {
          loss_i = base;
        }
        const float invS = 1.0f / S;
        const float a_coef = WEIGHTED ? ((1.0f - e) * wt + (float)((double)e * W / (double)V)) * inv_den : inv_den;
        A = a_coef * invS;
        B = (1.0f - e) * wt * inv_den;
        G = smooth ? (float)((double)e / (double)V) * inv_den : 0.0f;
      }
    }
    if (threadIdx.x == 0) P.row_loss[row] = loss_i;

    // Pass B: gradient.
    if (P.dl != nullptr) {
      const uintptr_t out_start = reinterpret_cast<uintptr_t>(P.dl) + (uintptr_t)(row_base * ES);
      const uintptr_t oa = out_start & ~(uintptr_t)15;
      const bool vec_out = STAGES > 0 && (int)(out_start - oa) == head;
      const float shM = M * kLog2e;
      const int kt = valid ? ((head + t * ES) >> 4) : -1;
      const int lane_t = valid ? (((head + t * ES) & 15) / ES) : 0;
      const float nanv = __int_as_float(0x7fc00000);
      auto gradient = [&](int k, int j0, float* d) {
        if (mode == 2) {
          float x[EPV];
          row_vector<DT, STAGES>(stage, P.logits, row_base, k, j0, V, x);
#pragma unroll
          for (int q = 0; q < EPV; ++q) {
            const float g = WEIGHTED ? G * ((j0 + q >= 0 && j0 + q < V) ? P.weight[j0 + q] : 0.0f) : G;
            d[q] = fmaf(ex2(fmaf(x[q], kLog2e, -shM)), A, -g);
          }
          if (k == kt) {
#pragma unroll
            for (int q = 0; q < EPV; ++q)
              if (q == lane_t) d[q] -= B;
          }
        } else {
#pragma unroll
          for (int q = 0; q < EPV; ++q) d[q] = mode == 1 ? nanv : 0.0f;
        }
      };
      auto store_scalar = [&](int j0, const float* d) {
#pragma unroll
        for (int q = 0; q < EPV; ++q) {
          const int j = j0 + q;
          if (j >= 0 && j < V) store1<DT>(P.dl, row_base + j, d[q]);
        }
      };
      int j0 = ((full_lo + (int)threadIdx.x) * 16 - head) / ES;
      for (int k = full_lo + threadIdx.x; k < full_hi; k += THREADS, j0 += dj) {
        float d[EPV];
        gradient(k, j0, d);
        if (vec_out) __stcs(reinterpret_cast<uint4*>(oa + (uintptr_t)k * 16), pack16<DT>(d));
        else store_scalar(j0, d);
      }
      const int nedge = full_lo + ((full_hi < nvec && full_hi >= full_lo) ? 1 : 0);
      if ((int)threadIdx.x < nedge) {
        const int k = (threadIdx.x == 0 && full_lo) ? 0 : full_hi;
        const int j0e = (k * 16 - head) / ES;
        float d[EPV];
        gradient(k, j0e, d);
        store_scalar(j0e, d);
      }
    }
    __syncthreads();  // every thread is done with this row's buffer and reduction scratch
    if (STAGES == 1 && next < P.rows) stage_row<ES>(P, next, smem, &bars[0]);
  }

  // Loss reduction over rows, in a fixed order, by the last block.
  if (P.reduction == NT_REDUCTION_NONE) return;
  if (!last_block_ticket(&P.ws->counter, &last)) return;
  double acc = 0.0;
  for (int64_t r = threadIdx.x; r < P.rows; r += THREADS) acc += (double)P.row_loss[r];
  acc = block_reduce(acc, red_d, SumOp(), 0.0);
  if (threadIdx.x == 0) {
    P.info->loss_sum = acc;
    P.loss[0] = zero_all ? 0.0f : (float)(mean ? acc / D : acc);
    P.ws->counter = 0u;
  }
}

// Upstream-gradient multiply for the autograd backward.
template <int DT>
__global__ void __launch_bounds__(256) xent_scale_kernel(void* dl, int64_t rows, int64_t classes,
                                                         const float* grad, int per_row) {
  if (!per_row && *grad == 1.0f) return;
  const int64_t n = rows * classes;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float g = per_row ? grad[i / classes] : *grad;
    store1<DT>(dl, i, __fmul_rn(load1<DT>(dl, i), g));
  }
}

template <int DT, int STAGES, bool WEIGHTED, int THREADS>
static int launch_variant(const XentParams& P, size_t smem, cudaStream_t stream) {
  auto kernel = xent_kernel<DT, STAGES, WEIGHTED, THREADS>;
  if (smem > 0) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute(xent)");
  }
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, THREADS, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  if (grid > P.rows) grid = P.rows;
  if (grid < 1) grid = 1;
  kernel<<<(unsigned)grid, THREADS, smem, stream>>>(P);
  return launch_status("nt_softmax_xent launch");
}

template <int DT, bool WEIGHTED>
static int launch_xent(const XentParams& P0, cudaStream_t stream) {
  XentParams P = P0;
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  // Row buffer: the row plus up to 15 leading bytes, rounded to 128 bytes.
  const size_t stride = (size_t)((P.classes * ES + 16 + 127) / 128 * 128);
  P.stage_stride = (int64_t)stride;
  int max_optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t budget = (size_t)max_optin > 4096 ? (size_t)max_optin - 4096 : 0;
  // Each CTA stages one row; where two buffers fit on an SM (bf16 / fp16 rows up to
  // ~56K classes) two CTAs share it and one's copy overlaps the other's compute.
  int sm_smem = 0;
  cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  (void)sm_smem;
  if (P.staged && stride <= budget) return launch_variant<DT, 1, WEIGHTED, 512>(P, stride, stream);
  return launch_variant<DT, 0, WEIGHTED, 512>(P, 0, stream);
}

template <int DT>
static int launch_xent_dt(const XentParams& P, cudaStream_t stream) {
  return P.weight ? launch_xent<DT, true>(P, stream) : launch_xent<DT, false>(P, stream);
}

}  // namespace nt

using namespace nt;

extern "C" {

size_t nt_xent_workspace_size(void) { return sizeof(XentWorkspace); }

int nt_softmax_xent(const nt_xent_args* args, void* stream) {
  if (!args) { set_error("nt_softmax_xent: args is NULL"); return NT_EINVAL; }
  const nt_xent_args& a = *args;
  if (a.rows < 0) { set_error("nt_softmax_xent: negative row count"); return NT_EINVAL; }
  if (a.classes <= 0) {
    set_error("Classification loss input must have shape [..., C] with C > 0, got C=%lld.", (long long)a.classes);
    return NT_EINVAL;
  }
  if (dtype_size(a.dtype) == 0) { set_error("nt_softmax_xent: unsupported dtype %d", a.dtype); return NT_EUNSUPPORTED; }
  if (a.classes > (int64_t)(INT32_MAX / 4 - 64)) {
    set_error("nt_softmax_xent: at most %d classes per row", INT32_MAX / 4 - 64);
    return NT_EUNSUPPORTED;
  }
  if (a.reduction < NT_REDUCTION_NONE || a.reduction > NT_REDUCTION_SUM) {
    set_error("nt_softmax_xent: invalid reduction %d", a.reduction);
    return NT_EINVAL;
  }
  if (!(a.label_smoothing >= 0.0f && a.label_smoothing < 1.0f)) {
    set_error("label_smoothing must be in [0, 1).");
    return NT_EINVAL;
  }
  if (!a.info || !a.loss || !a.workspace || (a.rows > 0 && (!a.logits || !a.targets || !a.row_loss))) {
    set_error("nt_softmax_xent: NULL logits/targets/loss/row_loss/info/workspace");
    return NT_EINVAL;
  }
  if (a.workspace_bytes < sizeof(XentWorkspace)) {
    set_error("nt_softmax_xent: workspace needs %zu bytes", sizeof(XentWorkspace));
    return NT_EINVAL;
  }
  XentParams P;
  P.logits = a.logits; P.dl = a.dlogits; P.targets = a.targets; P.weight = a.class_weight;
  P.rows = a.rows; P.classes = a.classes; P.ignore = a.ignore_index; P.smoothing = a.label_smoothing;
  P.reduction = a.reduction; P.loss = a.loss; P.row_loss = a.row_loss; P.info = a.info;
  P.ws = static_cast<XentWorkspace*>(a.workspace);
  const int es = dtype_size(a.dtype);
  P.tensor_end = reinterpret_cast<uintptr_t>(a.logits) + (uintptr_t)(a.rows * a.classes * es);
  P.staged = aligned16(a.logits) && (a.dlogits == nullptr || aligned16(a.dlogits));
  cudaStream_t s = as_stream(stream);
  xent_prepare_kernel<<<1, kPrepThreads, 0, s>>>(P);
  int rc = launch_status("nt_softmax_xent prepare launch");
  if (rc || a.rows == 0) return rc;
  switch (a.dtype) {
    case NT_F32: return launch_xent_dt<NT_F32>(P, s);
    case NT_F16: return launch_xent_dt<NT_F16>(P, s);
    default: return launch_xent_dt<NT_BF16>(P, s);
  }
}

int nt_xent_backward_scale(void* dlogits, int32_t dtype, int64_t rows, int64_t classes, const float* grad_output,
                           int32_t per_row, void* stream) {
  if (rows < 0 || classes < 0) { set_error("nt_xent_backward_scale: negative sizes"); return NT_EINVAL; }
  if (rows == 0 || classes == 0) return NT_OK;
  if (!dlogits || !grad_output) { set_error("nt_xent_backward_scale: NULL pointer"); return NT_EINVAL; }
  int64_t blocks = (rows * classes + 255) / 256;
  const int64_t cap = (int64_t)current_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case NT_F32: xent_scale_kernel<NT_F32><<<(unsigned)blocks, 256, 0, s>>>(dlogits, rows, classes, grad_output, per_row); break;
    case NT_F16: xent_scale_kernel<NT_F16><<<(unsigned)blocks, 256, 0, s>>>(dlogits, rows, classes, grad_output, per_row); break;
    case NT_BF16: xent_scale_kernel<NT_BF16><<<(unsigned)blocks, 256, 0, s>>>(dlogits, rows, classes, grad_output, per_row); break;
    default: set_error("nt_xent_backward_scale: unsupported dtype %d", dtype); return NT_EUNSUPPORTED;
  }
  return launch_status("nt_xent_backward_scale launch");
}

}  // extern "C"
