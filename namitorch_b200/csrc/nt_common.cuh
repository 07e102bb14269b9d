// Shared helpers of the sm_100a kernels: error plumbing, dtype loads/stores, chunk lookup
// and block reductions. Everything here is header-only so each .cu file stays standalone.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "namitorch_b200.h"
#include <nvtx3/nvToolsExt.h>

namespace nt {

// An NVTX range around one entry point, named after it: each call shows up as a range in
// Nsight Systems / Compute timelines. Header-only NVTX; a no-op unless a tool is attached.
struct TraceRange {
  explicit TraceRange(const char* name) { nvtxRangePushA(name); }
  ~TraceRange() { nvtxRangePop(); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

// ---- host-side error plumbing (nt_runtime.cu) ----------------------------------------
void set_error(const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* what);
int current_sm_count();

// Checks the launch that was just issued.
inline int launch_status(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, what);
  return NT_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int dtype) {
  switch (dtype) {
    case NT_F32: return 4;
    case NT_F16: return 2;
    case NT_BF16: return 2;
    default: return 0;
  }
}

// ---- device-side value conversion ----------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<NT_F32> {
  using T = float;
  static __device__ __forceinline__ float to_f32(float v) { return v; }
  static __device__ __forceinline__ float from_f32(float v) { return v; }
};
template <> struct Elem<NT_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
};
template <> struct Elem<NT_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
};

// Loads 8 consecutive elements starting at a 16-byte aligned address as fp32
// (streaming: the optimizer touches every byte once per step).
template <int DT>
__device__ __forceinline__ void load8(const void* base, int64_t i, float out[8]) {
  if constexpr (DT == NT_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
    float4 a = __ldcs(p), b = __ldcs(p + 1);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
    using T = typename Elem<DT>::T;
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const T*>(base) + i);
    uint4 raw = __ldcs(p);
    const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) out[k] = Elem<DT>::to_f32(h[k]);
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* base, int64_t i) {
  using T = typename Elem<DT>::T;
  return Elem<DT>::to_f32(static_cast<const T*>(base)[i]);
}

template <int DT>
__device__ __forceinline__ void store8(void* base, int64_t i, const float v[8]) {
  if constexpr (DT == NT_F32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + i);
    __stcs(p, make_float4(v[0], v[1], v[2], v[3]));
    __stcs(p + 1, make_float4(v[4], v[5], v[6], v[7]));
  } else {
    using T = typename Elem<DT>::T;
    uint4 raw;
    T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] = Elem<DT>::from_f32(v[k]);
    __stcs(reinterpret_cast<uint4*>(static_cast<T*>(base) + i), raw);
  }
}

template <int DT>
__device__ __forceinline__ void store1(void* base, int64_t i, float v) {
  using T = typename Elem<DT>::T;
  static_cast<T*>(base)[i] = Elem<DT>::from_f32(v);
}

__device__ __forceinline__ void load8_f32(const float* p, float out[8]) {
  const float4* q = reinterpret_cast<const float4*>(p);
  float4 a = __ldcs(q), b = __ldcs(q + 1);
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

__device__ __forceinline__ void store8_f32(float* p, const float v[8]) {
  float4* q = reinterpret_cast<float4*>(p);
  __stcs(q, make_float4(v[0], v[1], v[2], v[3]));
  __stcs(q + 1, make_float4(v[4], v[5], v[6], v[7]));
}

// The same 8 values as one 32-byte access (sm_100's 256-bit loads and stores); `p` must be
// 32-byte aligned.
__device__ __forceinline__ void load8_f32_v8(const float* p, float out[8]) {
  asm volatile("ld.global.cs.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(out[0]), "=f"(out[1]), "=f"(out[2]), "=f"(out[3]), "=f"(out[4]), "=f"(out[5]),
                 "=f"(out[6]), "=f"(out[7])
               : "l"(p));
}

__device__ __forceinline__ void store8_f32_v8(float* p, const float v[8]) {
  asm volatile("st.global.cs.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]), "f"(v[1]),
               "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

// 32 raw bytes in one streaming access (sm_100), as two 16-byte halves; `p` must be
// 32-byte aligned. Read-only streams and peer reads move more per request than with
// 16-byte loads.
__device__ __forceinline__ void load32_cs(const void* p, uint4& lo, uint4& hi) {
  asm volatile("ld.global.cs.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z), "=r"(hi.w)
               : "l"(p));
}

__device__ __forceinline__ void store32_cs(void* p, const uint4& lo, const uint4& hi) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(lo.x), "r"(lo.y),
               "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
               : "memory");
}

// ---- loss-scale handling -------------------------------------------------------------
// Division by the loss scale, bit-identical to IEEE f32 division. When the scale is a
// normal power of two its reciprocal is exact, and g * 2^-k rounds the same exact real
// number g / 2^k does, so the multiply replaces the divide.
struct Unscale {
  float scale;
  float inv;
  bool active;
  bool pow2;
  __device__ __forceinline__ void init(const float* scale_ptr) {
    active = scale_ptr != nullptr;
    scale = active ? *scale_ptr : 1.0f;
    uint32_t bits = __float_as_uint(scale);
    uint32_t exponent = (bits >> 23) & 0xffu;
    pow2 = active && (bits & 0x007fffffu) == 0 && exponent != 0 && exponent != 0xffu;
    inv = pow2 ? __frcp_rn(scale) : 1.0f;
  }
  __device__ __forceinline__ float operator()(float g) const {
    if (!active) return g;
    return pow2 ? __fmul_rn(g, inv) : __fdiv_rn(g, scale);
  }
};

// NaN-propagating max (the result is NaN if either operand is).
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Unpacks one 16-byte vector into fp32 values (4 for float32, 8 for 16-bit types).
template <int DT>
__device__ __forceinline__ void unpack16(const uint4& raw, float* out) {
  if constexpr (DT == NT_F32) {
    out[0] = __uint_as_float(raw.x); out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z); out[3] = __uint_as_float(raw.w);
  } else if constexpr (DT == NT_BF16) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[2 * k] = __uint_as_float(w[k] << 16);
      out[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  } else {
    const __half* h = reinterpret_cast<const __half*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) out[k] = __half2float(h[k]);
  }
}

// ---- chunk -> span lookup ------------------------------------------------------------
// `begin(i)` is non-decreasing; returns the last index whose begin <= chunk.
template <typename Begin>
__device__ __forceinline__ int find_owner(Begin begin, int n, int64_t chunk) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (begin(mid) <= chunk) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ---- warp / block reductions ---------------------------------------------------------
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ unsigned warp_sum(unsigned v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum / max with a fixed combination order (deterministic for a fixed block
// size). `scratch` needs blockDim.x / 32 slots; every thread receives the result.
template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* scratch, Op op, T identity) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  T r = identity;
  for (int w = 0; w < nwarps; ++w) r = op(r, scratch[w]);
  return r;
}

struct SumOp {
  template <typename T> __device__ __forceinline__ T operator()(T a, T b) const { return a + b; }
};
struct MaxOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); }
};

// "Last block done" ticket: returns true in exactly one block, after every other block
// has finished its global writes (each block fences before taking its ticket).
__device__ __forceinline__ bool last_block_ticket(unsigned* counter, bool* smem_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned ticket = atomicAdd(counter, 1u);
    *smem_flag = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  bool last = *smem_flag;
  if (last) __threadfence();
  return last;
}

}  // namespace nt
