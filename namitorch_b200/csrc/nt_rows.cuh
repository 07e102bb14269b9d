// Row helpers shared by the row-wise kernels (softmax, normalization): a row of at most a
// few thousand elements is spread over WARPS warps, each thread holding NPL values in
// registers; reductions run over warp shuffles and, across the warps of a row, shared memory
// (one float per warp of the block). Every thread of a block must reach the reductions.
#pragma once

#include "nt_common.cuh"

namespace nt {

template <int WARPS>
__device__ __forceinline__ float row_max(float v, float* smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
  if constexpr (WARPS > 1) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, first = warp - warp % WARPS;
    __syncwarp();
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    v = smem[first];
#pragma unroll
    for (int w = 1; w < WARPS; ++w) v = max_nan(v, smem[first + w]);
    __syncthreads();
  }
  return v;
}

template <int WARPS>
__device__ __forceinline__ float row_sum(float v, float* smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if constexpr (WARPS > 1) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, first = warp - warp % WARPS;
    __syncwarp();
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    v = smem[first];
#pragma unroll
    for (int w = 1; w < WARPS; ++w) v += smem[first + w];
    __syncthreads();
  }
  return v;
}

// Column of slot q of thread t (T threads per row): 16-byte vectors of EPV elements dealt
// round-robin on the vector path, single elements round-robin otherwise.
template <int EPV>
__device__ __forceinline__ int slot_column(int q, int t, int T, bool vec) {
  return vec ? ((q / EPV) * T + t) * EPV + q % EPV : q * T + t;
}

// STREAM: the row is read once (evict-first loads); otherwise it is shared by every row of
// the tensor (a weight or a bias) and kept in the caches.
template <int DT, int NPL, int WARPS, bool STREAM = true>
__device__ __forceinline__ void load_row(const void* base, int width, int t, bool vec, float (&v)[NPL]) {
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  constexpr int T = 32 * WARPS;
  if (vec) {
#pragma unroll
    for (int c = 0; c < NPL / EPV; ++c) {
      const int k = c * T + t;
      if (k * EPV < width) {
        const uint4* src = static_cast<const uint4*>(base) + k;
        const uint4 raw = STREAM ? __ldcs(src) : __ldg(src);
        unpack16<DT>(raw, v + c * EPV);
      } else {
#pragma unroll
        for (int e = 0; e < EPV; ++e) v[c * EPV + e] = 0.0f;
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < NPL; ++q) {
      const int j = q * T + t;
      v[q] = j < width ? load1<DT>(base, j) : 0.0f;
    }
  }
}

// load_row on the vector path for the forward of a row whose columns past `last` are masked
// out: a vector that starts past `last` is never read and enters as -inf (the masked part of
// a causal row is not part of the result, whatever it holds).
template <int DT, int NPL, int WARPS>
__device__ __forceinline__ void load_row_upto(const void* base, int last, int t, float (&v)[NPL]) {
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  constexpr int T = 32 * WARPS;
#pragma unroll
  for (int c = 0; c < NPL / EPV; ++c) {
    const int k = c * T + t;
    if (k * EPV <= last) {
      unpack16<DT>(__ldcs(static_cast<const uint4*>(base) + k), v + c * EPV);
    } else {
#pragma unroll
      for (int e = 0; e < EPV; ++e) v[c * EPV + e] = -INFINITY;
    }
  }
}

// The EPV values of slot group c (slots c * EPV .. c * EPV + EPV - 1) of a row shared by every
// row of the tensor (a weight or a bias), cached; 0 past the width. One group at a time keeps
// only EPV of those values in registers.
template <int DT, int NPL, int WARPS>
__device__ __forceinline__ void load_group(const void* base, int width, int t, bool vec, int c, float* out) {
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  constexpr int T = 32 * WARPS;
  if (vec) {
    const int k = c * T + t;
    if (k * EPV < width) {
      unpack16<DT>(__ldg(static_cast<const uint4*>(base) + k), out);
    } else {
#pragma unroll
      for (int e = 0; e < EPV; ++e) out[e] = 0.0f;
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      const int j = (c * EPV + e) * T + t;
      out[e] = j < width ? load1<DT>(base, j) : 0.0f;
    }
  }
}

// One 16-byte vector: EPV values rounded to the storage type (round to nearest even; the
// 16-bit types convert two values per instruction).
template <int DT>
__device__ __forceinline__ void store_vec16(void* base, int k, const float* v) {
  uint4 raw;
  if constexpr (DT == NT_F32) {
    raw = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
  } else if constexpr (DT == NT_BF16) {
    __nv_bfloat162 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    raw = *reinterpret_cast<const uint4*>(h);
  } else {
    __half2 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    raw = *reinterpret_cast<const uint4*>(h);
  }
  __stcs(static_cast<uint4*>(base) + k, raw);
}

template <int DT, int NPL, int WARPS>
__device__ __forceinline__ void store_row(void* base, int width, int t, bool vec, const float (&v)[NPL]) {
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;
  constexpr int T = 32 * WARPS;
  if (vec) {
#pragma unroll
    for (int c = 0; c < NPL / EPV; ++c) {
      const int k = c * T + t;
      if (k * EPV < width) store_vec16<DT>(base, k, v + c * EPV);
    }
  } else {
#pragma unroll
    for (int q = 0; q < NPL; ++q) {
      const int j = q * T + t;
      if (j < width) store1<DT>(base, j, v[q]);
    }
  }
}

}  // namespace nt
