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
// Data movement: each CTA is persistent over rows and stages one row at a time in shared
// memory. A row (V * esize bytes, not 16-byte aligned in general) is fetched from the 16-byte
// boundary at or below its start by cp.async.bulk (kXentChunks copies, each completing on its
// own mbarrier); the few bytes past the last 16-byte boundary of the whole tensor are loaded
// with plain loads. Three passes run from shared memory: the row max (packed two-lane
// max.NaN for 16-bit types), the sum of exp(x - max), and the gradient. The last warp to
// finish a chunk in the gradient pass refills it with the CTA's next row (a shared-memory
// count per chunk; no warp waits for another). At [8192, 50257] bf16 two CTAs share an SM,
// so one CTA's copy overlaps the other's passes; one chunk per row measured fastest (more
// chunks let a row's copy start earlier but add per-chunk work to every pass, and the
// passes, not the copies, bound the kernel: about 17 instructions per logit). The gradient
// is written with 16-byte streaming stores at the same alignment offset. HBM traffic is one
// read of the logits and one write of dlogits. Tensors that do not start on a 16-byte
// boundary take the same three passes over global memory instead. Without class weights
// each CTA counts the valid targets (the mean's denominator) itself while its first row is
// in flight; with weights a one-block prepare kernel sums the weights first.
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
  int self_count;         // the main kernel counts the targets (no prepare launch)
  int64_t chunk;          // bytes per staged chunk (a multiple of 128)
};

constexpr int kXentChunks = 1;
constexpr int kXentThreads = 512;

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

// Two-lane max of packed 16-bit values; NaN in either operand gives NaN.
template <int DT>
__device__ __forceinline__ uint32_t max_nan_x2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (DT == NT_BF16) asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <int DT>
__device__ __forceinline__ float max_of_pair(uint32_t r) {
  float lo, hi;
  if constexpr (DT == NT_BF16) {
    lo = __uint_as_float(r << 16);
    hi = __uint_as_float(r & 0xffff0000u);
  } else {
    lo = __half2float(__ushort_as_half((unsigned short)(r & 0xffffu)));
    hi = __half2float(__ushort_as_half((unsigned short)(r >> 16)));
  }
  return max_nan(lo, hi);
}

// Vector k of the row: from the staged buffer, or (unstaged) element by element from global
// memory with -inf outside the row. Staged edge vectors hold bytes of the neighbouring rows
// (or past the tensor) in the lanes outside [0, V); callers mask them.
// (Plain loads: the mbarrier waits that precede them clobber memory, so the compiler keeps
// them after the wait.)
template <int DT, bool STAGED>
__device__ __forceinline__ uint4 row_raw(const unsigned char* stage, int k) {
  return reinterpret_cast<const uint4*>(stage)[k];
}

template <int DT, bool STAGED>
__device__ __forceinline__ void row_values(const unsigned char* stage, const void* logits, int64_t row_base, int k,
                                           int j0, int V, bool edge, float* x) {
  constexpr int EPV = DT == NT_F32 ? 4 : 8;
  if constexpr (STAGED) {
    unpack16<DT>(row_raw<DT, true>(stage, k), x);
    if (edge) {
#pragma unroll
      for (int q = 0; q < EPV; ++q)
        if (j0 + q < 0 || j0 + q >= V) x[q] = -INFINITY;
    }
  } else {
#pragma unroll
    for (int q = 0; q < EPV; ++q) {
      const int j = j0 + q;
      x[q] = (j >= 0 && j < V) ? load1<DT>(logits, row_base + j) : -INFINITY;
    }
  }
}

// Stages chunk c of `row` into `buf` (called by one whole warp): bytes [c * chunk,
// (c + 1) * chunk) counted from the 16-byte boundary at or below the row start, by one bulk
// copy issued by lane 0 and completing on `bar` (an empty chunk arrives with no bytes, so
// every chunk's barrier completes once per row). The bytes between the last 16-byte boundary
// of the tensor and its end (fewer than 16, at the end of the last row) are loaded with
// plain loads by the warp before lane 0 arrives; the arrival (release) and the readers' wait
// (acquire) make them visible.
template <int ES>
__device__ __forceinline__ void stage_chunk(const XentParams& P, int64_t row, unsigned char* buf, uint64_t* bar,
                                            int c, int lane) {
  const uintptr_t start = reinterpret_cast<uintptr_t>(P.logits) + (uintptr_t)(row * P.classes * ES);
  const uintptr_t a = start & ~(uintptr_t)15;
  const int span = (int)(start - a) + (int)P.classes * ES;
  int bulk = ((span + 15) >> 4) << 4;
  const uintptr_t limit = P.tensor_end & ~(uintptr_t)15;
  if ((int64_t)(limit - a) < bulk) bulk = (int)(limit - a);
  const int lo = c * (int)P.chunk;
  const int end = lo + (int)P.chunk;
  const int hi = bulk < end ? bulk : end;
  if (bulk < span && bulk >= lo && bulk < end)
    for (int k = bulk + lane; k < span; k += 32) buf[k] = *reinterpret_cast<const unsigned char*>(a + k);
  __syncwarp();
  if (lane == 0) {
    fence_proxy_async();
    const uint32_t bytes = hi > lo ? (uint32_t)(hi - lo) : 0u;
    mbar_arrive_expect_tx(bar, bytes);
    if (bytes) bulk_g2s(buf + lo, reinterpret_cast<const void*>(a + lo), bytes, bar);
  }
}

// STAGED: rows staged in shared memory in chunks (16-byte aligned logits and dlogits);
// otherwise the passes read global memory.
template <int DT, bool STAGED, bool WEIGHTED>
__global__ void __launch_bounds__(kXentThreads) xent_kernel(const __grid_constant__ XentParams P) {
  constexpr int THREADS = kXentThreads;
  constexpr int NCH = kXentChunks;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bars[NCH];
  __shared__ unsigned done[NCH];   // warps finished with a chunk of the current row
  __shared__ float red_f[THREADS / 32];
  __shared__ float red_s[THREADS / 32];
  __shared__ float coef[4];   // A, B, G and the row mode of the current row
  __shared__ double red_d[THREADS / 32];
  __shared__ bool last;
  __shared__ int abort_flag;

  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;  // elements per 16-byte vector
  const int V = (int)P.classes;
  const nt_xent_info* info = P.info;
  const bool mean = P.reduction == NT_REDUCTION_MEAN;
  const float e = P.smoothing;
  const bool smooth = e != 0.0f;
  const int cvec = (int)(P.chunk >> 4);   // vectors per chunk

  const int lane = threadIdx.x & 31;
  if constexpr (STAGED) {
    if (threadIdx.x == 0) {
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        mbar_init(&bars[c], 1);
        done[c] = 0;
      }
      abort_flag = 0;
      fence_proxy_async();
    }
    __syncthreads();
    if (threadIdx.x < 32 && (int64_t)blockIdx.x < P.rows) {
#pragma unroll 1
      for (int c = 0; c < NCH; ++c) stage_chunk<ES>(P, blockIdx.x, smem, &bars[c], c, lane);
    }
  }

  // The mean's denominator. Without class weights every CTA counts the targets itself while
  // its first row's copy is in flight (the same counts as xent_prepare_kernel, which then is
  // not launched), and CTA 0 records them; with weights the prepare kernel has.
  double D = 1.0, W;
  if (!WEIGHTED && P.self_count) {
    double valid = 0.0, bad = 0.0;
    for (int64_t i = threadIdx.x; i < P.rows; i += THREADS) {
      const int64_t t = P.targets[i];
      if (t == P.ignore) continue;
      if (t < 0 || t >= V) bad += 1.0;
      else valid += 1.0;
    }
    valid = block_reduce(valid, red_d, SumOp(), 0.0);
    bad = block_reduce(bad, red_d, SumOp(), 0.0);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      nt_xent_info* out = P.info;
      out->n_valid = valid;
      out->bad_targets = bad;
      out->denominator = valid;
      out->weight_sum = (double)V;
    }
    if (mean) D = valid;
    W = (double)V;
  } else {
    if (mean) D = info->denominator;
    W = info->weight_sum;
  }
  const bool zero_all = mean && D == 0.0;
  const float inv_den = zero_all ? 0.0f : (float)(1.0 / D);

  uint32_t parity = 0;
  // The target of the CTA's next row is loaded one row ahead.
  int64_t t_next = (int64_t)blockIdx.x < P.rows ? P.targets[blockIdx.x] : 0;
  for (int64_t row = blockIdx.x; row < P.rows; row += gridDim.x, parity ^= 1u) {
    const int64_t next = row + gridDim.x;
    const int64_t t64 = t_next;
    if (next < P.rows) t_next = P.targets[next];
    const bool valid = t64 != P.ignore && t64 >= 0 && t64 < V;
    const int t = valid ? (int)t64 : -1;
    const int64_t row_base = row * (int64_t)V;
    const uintptr_t start = reinterpret_cast<uintptr_t>(P.logits) + (uintptr_t)(row_base * ES);
    const int head = STAGED ? (int)(start & 15u) : 0;
    const int span = head + V * ES;           // bytes from the 16-byte boundary to the row end
    const int nvec = (span + 15) >> 4;
    const int full_lo = head ? 1 : 0;         // vectors [full_lo, full_hi) hold only row elements
    const int full_hi = span >> 4;
    auto first_elem = [&](int k) { return (k * 16 - head) / ES; };

    // Vectors [lo, hi) of this thread, two per iteration (independent work for the
    // scheduler to interleave).
    auto for_vectors = [&](int lo, int hi, auto&& body) {
      int k = lo + (int)threadIdx.x;
      for (; k + THREADS < hi; k += 2 * THREADS) {
        body(k);
        body(k + THREADS);
      }
      if (k < hi) body(k);
    };
    // The <= 2 edge vectors (the head vector when the row starts inside it, the tail vector
    // when the row ends inside it; one vector when the whole row fits in it), taken by
    // threads 0 and 1; `in_range(k)` limits them to a chunk.
    const int tail_k = full_hi < nvec && full_hi >= full_lo ? full_hi : -1;
    auto edge_vector = [&](int lo, int hi) {
      int k = -1;
      if (threadIdx.x == 0 && full_lo) k = 0;
      if (threadIdx.x == (full_lo ? 1 : 0)) k = tail_k;
      return k >= lo && k < hi ? k : -1;
    };
    auto interior = [&](int lo, int hi, int& a, int& b) {
      a = lo > full_lo ? lo : full_lo;
      b = hi < full_hi ? hi : full_hi;
    };

    // Pass 1: the row max, chunk by chunk as the chunks land. NaN propagates (max.NaN).
    float m = -INFINITY;
    {
      uint32_t m2 = DT == NT_BF16 ? 0xff80ff80u : 0xfc00fc00u;   // a pair of -inf
#pragma unroll 1
      for (int c = 0; c < (STAGED ? NCH : 1); ++c) {
        int k0 = 0, k1 = nvec;
        if constexpr (STAGED) {
          k0 = c * cvec;
          k1 = k0 + cvec < nvec ? k0 + cvec : nvec;
          if (k0 < k1 && !wait_stage(&bars[c], parity)) abort_flag = 1;
        }
        int a, b;
        interior(k0, k1, a, b);
        for_vectors(a, b, [&](int k) {
          if constexpr (STAGED && DT != NT_F32) {
            const uint4 raw = row_raw<DT, true>(smem, k);
            m2 = max_nan_x2<DT>(m2, max_nan_x2<DT>(max_nan_x2<DT>(raw.x, raw.y), max_nan_x2<DT>(raw.z, raw.w)));
          } else {
            float x[EPV];
            row_values<DT, STAGED>(smem, P.logits, row_base, k, first_elem(k), V, false, x);
#pragma unroll
            for (int q = 0; q < EPV; ++q) m = max_nan(m, x[q]);
          }
        });
      }
      const int k = edge_vector(0, nvec);
      if (k >= 0) {
        float x[EPV];
        row_values<DT, STAGED>(smem, P.logits, row_base, k, first_elem(k), V, true, x);
#pragma unroll
        for (int q = 0; q < EPV; ++q) m = max_nan(m, x[q]);
      }
      if constexpr (DT != NT_F32) m = max_nan(m, max_of_pair<DT>(m2));
    }
    const float M = block_reduce(m, red_f, [](float a, float b) { return max_nan(a, b); }, -INFINITY);
    if (STAGED && abort_flag) {
      // A copy did not land in time: report it, let this row's other copies land (each wait
      // bounded) and leave. No copy of the next row has been issued yet.
      if (threadIdx.x == 0) {
        atomicAdd(&P.info->error, 1.0);
        for (int c = 0; c < NCH; ++c) wait_stage(&bars[c], parity);
      }
      return;
    }
    const bool bad_row = M != M || M == INFINITY;
    const bool neg_row = !bad_row && M == -INFINITY;

    // Pass 2: sum of exp(x - M) (2^(x log2e - M log2e): one FMA and one SFU op per element;
    // masked lanes are -inf and add 0); label smoothing also needs sum_c w_c x_c.
    // One partial sum per vector lane keeps the additions of a vector independent.
    float s = 0.0f;
    double swx = 0.0;
    if (!bad_row && !neg_row) {
      const float sh = M * kLog2e;
      float part[EPV];
#pragma unroll
      for (int q = 0; q < EPV; ++q) part[q] = 0.0f;
      auto add = [&](int k, bool edge) {
        const int j0 = first_elem(k);
        float x[EPV];
        row_values<DT, STAGED>(smem, P.logits, row_base, k, j0, V, edge, x);
#pragma unroll
        for (int q = 0; q < EPV; ++q) part[q] += ex2(fmaf(x[q], kLog2e, -sh));
        if (smooth) {
#pragma unroll
          for (int q = 0; q < EPV; ++q) {
            const int j = j0 + q;
            if (!edge || (j >= 0 && j < V)) swx += WEIGHTED ? (double)P.weight[j] * (double)x[q] : (double)x[q];
          }
        }
      };
      for_vectors(full_lo, full_hi, [&](int k) { add(k, false); });
      const int k = edge_vector(0, nvec);
      if (k >= 0) add(k, true);
#pragma unroll
      for (int q = 0; q < EPV; ++q) s += part[q];
    }
    // Row sum, row loss and the gradient coefficients (d_c = e_c * A - G_c, minus B at
    // c == t): warp partials in shared memory; warp 0 adds them (a fixed shuffle tree),
    // computes the row's scalars once and broadcasts them.
    constexpr int NW = THREADS / 32;
    {
      const float sw = warp_sum(s);
      const double dw = smooth ? warp_sum(swx) : 0.0;
      if (lane == 0) {
        red_s[threadIdx.x >> 5] = sw;
        if (smooth) red_d[threadIdx.x >> 5] = dw;
      }
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const float S = warp_sum(lane < NW ? red_s[lane] : 0.0f);
      const double sx = smooth ? warp_sum(lane < NW ? red_d[lane] : 0.0) : 0.0;
      if (lane == 0) {
        const float wt = valid ? (WEIGHTED ? P.weight[t] : 1.0f) : 0.0f;
        int mode = 0;  // 0: zero row, 1: NaN row, 2: regular
        float loss_i = 0.0f, A = 0.0f, B = 0.0f, G = 0.0f, xt = 0.0f;
        if (valid && !zero_all) {
          if (bad_row) {
            mode = 1;
            loss_i = __int_as_float(0x7fc00000);
          } else if (neg_row) {
            loss_i = INFINITY;
          } else {
            mode = 2;
            if constexpr (STAGED) {
              const int off = head + t * ES;
              if constexpr (DT == NT_F32) xt = *reinterpret_cast<const float*>(smem + off);
              else if constexpr (DT == NT_BF16) xt = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(smem + off));
              else xt = __half2float(*reinterpret_cast<const __half*>(smem + off));
            } else {
              xt = load1<DT>(P.logits, row_base + t);
            }
            const float lse = M + logf(S);
            const float base = -wt * (xt - lse);
            if (smooth) {
              const double sm = -(sx - (double)lse * W) / (double)V;
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
        P.row_loss[row] = loss_i;
        coef[0] = A; coef[1] = B; coef[2] = G; coef[3] = __int_as_float(mode);
      }
    }
    __syncthreads();
    const float A = coef[0], B = coef[1], G = coef[2];
    const int mode = __float_as_int(coef[3]);

    // Pass 3: the gradient, chunk by chunk. The last warp to finish a chunk refills it with
    // the CTA's next row (a shared-memory count per chunk; no warp waits for another).
    const uintptr_t out_start = reinterpret_cast<uintptr_t>(P.dl) + (uintptr_t)(row_base * ES);
    const uintptr_t oa = out_start & ~(uintptr_t)15;
    const bool vec_out = STAGED && (int)(out_start - oa) == head;
    const float shM = M * kLog2e;
    const float fill = mode == 1 ? __int_as_float(0x7fc00000) : 0.0f;
    const int kt = mode == 2 ? ((head + t * ES) >> 4) : -1;
    const int lane_t = mode == 2 ? (((head + t * ES) & 15) / ES) : 0;
    auto grad_vector = [&](int k, float* d) {
      const int j0 = first_elem(k);
      if (mode == 2) {
        float x[EPV];
        row_values<DT, STAGED>(smem, P.logits, row_base, k, j0, V, false, x);
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
        for (int q = 0; q < EPV; ++q) d[q] = fill;
      }
    };
    auto store_scalar = [&](int k, const float* d) {
      const int j0 = first_elem(k);
#pragma unroll
      for (int q = 0; q < EPV; ++q) {
        const int j = j0 + q;
        if (j >= 0 && j < V) store1<DT>(P.dl, row_base + j, d[q]);
      }
    };
#pragma unroll 1
    for (int c = 0; c < (STAGED ? NCH : 1); ++c) {
      int k0 = 0, k1 = nvec;
      if constexpr (STAGED) {
        k0 = c * cvec;
        k1 = k0 + cvec < nvec ? k0 + cvec : nvec;
      }
      if (P.dl != nullptr) {
        int a, b;
        interior(k0, k1, a, b);
        if (vec_out) {
          for_vectors(a, b, [&](int k) {
            float d[EPV];
            grad_vector(k, d);
            __stcs(reinterpret_cast<uint4*>(oa + (uintptr_t)k * 16), pack16<DT>(d));
          });
        } else {
          for_vectors(a, b, [&](int k) {
            float d[EPV];
            grad_vector(k, d);
            store_scalar(k, d);
          });
        }
        const int k = edge_vector(k0, k1);
        if (k >= 0) {
          float d[EPV];
          grad_vector(k, d);
          store_scalar(k, d);
        }
      }
      if constexpr (STAGED) {
        // This warp's reads of chunk c are complete (their values are consumed above).
        __syncwarp();
        unsigned last_warp = 0;
        if (lane == 0) {
          __threadfence_block();
          last_warp = atomicAdd(&done[c], 1u) == THREADS / 32 - 1;
          if (last_warp) done[c] = 0;
        }
        if (__shfl_sync(0xffffffffu, last_warp, 0) && next < P.rows) stage_chunk<ES>(P, next, smem, &bars[c], c, lane);
      }
    }
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

template <int DT, bool STAGED, bool WEIGHTED>
static int launch_variant(const XentParams& P, size_t smem, cudaStream_t stream) {
  auto kernel = xent_kernel<DT, STAGED, WEIGHTED>;
  if (smem > 0) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute(xent)");
  }
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kXentThreads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  if (grid > P.rows) grid = P.rows;
  if (grid < 1) grid = 1;
  kernel<<<(unsigned)grid, kXentThreads, smem, stream>>>(P);
  return launch_status("nt_softmax_xent launch");
}

template <int DT, bool WEIGHTED>
static int launch_xent(const XentParams& P0, cudaStream_t stream) {
  XentParams P = P0;
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  // Row buffer: the row plus up to 15 leading bytes, in kXentChunks chunks of a multiple of
  // 128 bytes. Two CTAs share an SM where two buffers fit (16-bit rows up to ~56K classes).
  const int64_t need = (P.classes * ES + 15 + 15) / 16 * 16;
  const int64_t chunk = (need + kXentChunks - 1) / kXentChunks;
  P.chunk = (chunk + 127) / 128 * 128;
  const size_t buffer = (size_t)P.chunk * kXentChunks;
  int max_optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t budget = (size_t)max_optin > 4096 ? (size_t)max_optin - 4096 : 0;
  if (P.staged && buffer <= budget) return launch_variant<DT, true, WEIGHTED>(P, buffer, stream);
  P.chunk = 16;
  return launch_variant<DT, false, WEIGHTED>(P, 0, stream);
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
  nt::TraceRange trace("nt_softmax_xent");
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
  // Without class weights the main kernel counts the targets itself; the one-block prepare
  // kernel runs for weighted losses and for zero rows (where it writes the zero loss).
  P.self_count = a.class_weight == nullptr && a.rows > 0;
  if (P.self_count) {
    // The record starts from zero (loss_sum stays 0 for reduction NONE; error accumulates).
    const cudaError_t err = cudaMemsetAsync(a.info, 0, sizeof(nt_xent_info), s);
    if (err != cudaSuccess) return cuda_fail(err, "nt_softmax_xent: clearing the info record");
  } else {
    xent_prepare_kernel<<<1, kPrepThreads, 0, s>>>(P);
    const int rc = launch_status("nt_softmax_xent prepare launch");
    if (rc || a.rows == 0) return rc;
  }
  switch (a.dtype) {
    case NT_F32: return launch_xent_dt<NT_F32>(P, s);
    case NT_F16: return launch_xent_dt<NT_F16>(P, s);
    default: return launch_xent_dt<NT_BF16>(P, s);
  }
}

int nt_xent_backward_scale(void* dlogits, int32_t dtype, int64_t rows, int64_t classes, const float* grad_output,
                           int32_t per_row, void* stream) {
  nt::TraceRange trace("nt_xent_backward_scale");
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
