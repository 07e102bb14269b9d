// Fused elementwise activations: the operations of the reference's FusedCUDAKernels
// (namitorch/backends/cuda/fused.py:8-69) — sigmoid, silu and tanh-approximated gelu with
// their backward passes, swiglu, bias + activation (sigmoid, silu, gelu, relu) and clamp.
//
// Each is one streaming pass: 16-byte vectors (4 float32 or 8 16-bit values) when every
// operand is 16-byte aligned and the element count (and, for the bias operations, the row
// width) is a whole number of vectors; one element at a time otherwise. Two vectors per
// thread per iteration keep loads in flight. Bias rows are read through the read-only cache
// (every row of the tensor reads them); the column of a thread's vector advances by the
// grid stride modulo the width instead of a division per vector. Half and bfloat16 operands
// are computed in float32 and rounded once, with the SFU's exp / reciprocal / divide (below).
//
// The arithmetic follows the reference's device helpers, with CUDA's expf:
//   sigmoid(x) = 1 / (1 + e) for x >= 0, e / (1 + e) otherwise, e = exp(-|x|)
//   silu(x) = x * sigmoid(x) (0 at -inf); silu'(x) = s + x * s * (1 - s) (s alone where x is
//   not finite); gelu(x) = 0.5 x (1 + tanh(k (x + 0.044715 x^3))), x itself (or -0) beyond
//   |x| > 20, and its derivative (evaluated through sigmoid, below); relu'(x) = NaN for NaN,
//   else [x > 0].
#include <cmath>

#include "nt_common.cuh"

namespace nt {

struct FusedParams {
  const void* a;
  const void* b;
  const void* c;
  const void* d;
  void* out;
  void* second;
  int64_t count;
  int64_t width;
};

constexpr int kFusedThreads = 256;
constexpr float kGeluScale = 0.7978845608028654f;   // sqrt(2 / pi)
constexpr float kGeluCubic = 0.044715f;
constexpr float kGeluCubic3 = 0.134145f;            // 3 * 0.044715

// FAST (16-bit operands): the SFU's exp and reciprocal (`__expf`, `rcp.approx`,
// `__fdividef`, each within a few float32 ulps) instead of the rounded `expf`, `__frcp_rn`
// and IEEE division; the result is rounded to 8 or 11 significant bits on store, where the
// difference almost never shows (the tests allow one unit of the stored type).
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <bool FAST>
__device__ __forceinline__ float sigmoid_of(float x) {
  const float e = FAST ? __expf(-fabsf(x)) : expf(-fabsf(x));   // in [0, 1]
  if constexpr (FAST) return x >= 0.0f ? rcp_approx(1.0f + e) : __fdividef(e, 1.0f + e);
  return x >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
}
template <bool FAST>
__device__ __forceinline__ float silu_of(float x) {
  return (isinf(x) && x < 0.0f) ? 0.0f : x * sigmoid_of<FAST>(x);
}
template <bool FAST>
__device__ __forceinline__ float silu_grad(float x) {
  const float s = sigmoid_of<FAST>(x);
  return isfinite(x) ? s + x * (s * (1.0f - s)) : s;
}
template <bool FAST>
__device__ __forceinline__ float sigmoid_grad(float x) {
  const float s = sigmoid_of<FAST>(x);
  return s * (1.0f - s);
}
// gelu with the tanh approximation through the identity 0.5 (1 + tanh(u)) = sigmoid(2u):
// gelu(x) = x * sigmoid(2u) and gelu'(x) = s + 2 x s (1 - s) u', s = sigmoid(2u),
// u = sqrt(2/pi) (x + 0.044715 x^3). One SFU exp2 and one reciprocal replace tanhf, with no
// cancellation where tanh(u) is near -1; results agree with the tanh form to a few float32
// ulps. 2^(-2u log2 e) overflows to +inf for very negative u, which gives s = 0.
template <bool FAST>
__device__ __forceinline__ float sigmoid_2u(float x) {
  const float u = kGeluScale * (x + kGeluCubic * x * x * x);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(u * -2.8853900817779268f));   // -2 log2(e) u
  return FAST ? rcp_approx(1.0f + e) : __frcp_rn(1.0f + e);
}
template <bool FAST>
__device__ __forceinline__ float gelu_of(float x) {
  if (fabsf(x) > 20.0f) return x > 0.0f ? x : -0.0f;
  return x * sigmoid_2u<FAST>(x);
}
template <bool FAST>
__device__ __forceinline__ float gelu_grad(float x) {
  if (fabsf(x) > 20.0f) return x > 0.0f ? 1.0f : 0.0f;
  const float s = sigmoid_2u<FAST>(x);
  const float inner = kGeluScale * (1.0f + kGeluCubic3 * x * x);
  return s + 2.0f * x * (s * (1.0f - s)) * inner;
}
__device__ __forceinline__ float relu_of(float x) { return x <= 0.0f ? 0.0f : x; }
__device__ __forceinline__ float relu_grad(float x) { return isnan(x) ? x : (x > 0.0f ? 1.0f : 0.0f); }

// Operands an operation reads: bit 0 a, 1 b, 2 c, 3 d; BIAS: b is a [width] row.
template <int OP> struct FusedOp {
  static constexpr bool kBias = OP >= NT_FUSED_BIAS_SIGMOID && OP <= NT_FUSED_BIAS_RELU_BACKWARD;
  static constexpr bool kClamp = OP == NT_FUSED_CLAMP || OP == NT_FUSED_CLAMP_BACKWARD;
  static constexpr bool kReadB = !kClamp && OP != NT_FUSED_SIGMOID && OP != NT_FUSED_SILU && OP != NT_FUSED_GELU_TANH;
  static constexpr bool kReadC = OP == NT_FUSED_SWIGLU_BACKWARD ||
                                 (kBias && OP >= NT_FUSED_BIAS_SIGMOID_BACKWARD);
  static constexpr bool kReadD = OP == NT_FUSED_CLAMP_BACKWARD;
  static constexpr bool kSecond = OP == NT_FUSED_SWIGLU_BACKWARD;
};

// One element. `lo` / `hi` are the clamp bounds (has_lo / has_hi: present).
template <int OP, bool FAST>
__device__ __forceinline__ float fused_value(float a, float b, float c, float d, float lo, float hi, bool has_lo,
                                             bool has_hi, float& second) {
  switch (OP) {
    case NT_FUSED_SIGMOID: return sigmoid_of<FAST>(a);
    case NT_FUSED_SILU: return silu_of<FAST>(a);
    case NT_FUSED_GELU_TANH: return gelu_of<FAST>(a);
    case NT_FUSED_SIGMOID_BACKWARD: return b * (a * (1.0f - a));
    case NT_FUSED_SILU_BACKWARD: return b * silu_grad<FAST>(a);
    case NT_FUSED_GELU_TANH_BACKWARD: return b * gelu_grad<FAST>(a);
    case NT_FUSED_SWIGLU: return silu_of<FAST>(a) * b;
    case NT_FUSED_SWIGLU_BACKWARD:
      second = c * silu_of<FAST>(a);
      return (c * b) * silu_grad<FAST>(a);
    case NT_FUSED_BIAS_SIGMOID: return sigmoid_of<FAST>(a + b);
    case NT_FUSED_BIAS_SILU: return silu_of<FAST>(a + b);
    case NT_FUSED_BIAS_GELU_TANH: return gelu_of<FAST>(a + b);
    case NT_FUSED_BIAS_RELU: return relu_of(a + b);
    case NT_FUSED_BIAS_SIGMOID_BACKWARD: return c * sigmoid_grad<FAST>(a + b);
    case NT_FUSED_BIAS_SILU_BACKWARD: return c * silu_grad<FAST>(a + b);
    case NT_FUSED_BIAS_GELU_TANH_BACKWARD: return c * gelu_grad<FAST>(a + b);
    case NT_FUSED_BIAS_RELU_BACKWARD: return c * relu_grad(a + b);
    case NT_FUSED_CLAMP: {
      const float l = has_lo ? lo : 0.0f, h = has_hi ? hi : 0.0f;
      if (isnan(a) || isnan(l) || isnan(h)) return a + l + h;
      float x = a;
      if (has_lo && x <= l) x = l;
      if (has_hi && x >= h) x = h;
      return x;
    }
    default: {  // NT_FUSED_CLAMP_BACKWARD
      const float l = has_lo ? lo : 0.0f, h = has_hi ? hi : 0.0f;
      if (isnan(a) || isnan(l) || isnan(h)) return a + l + h;
      return ((!has_lo || a > l) && (!has_hi || a < h)) ? d : 0.0f;
    }
  }
}

template <int DT, int EPV>
__device__ __forceinline__ void load_vec(const void* base, int64_t v, float* x) {
  if constexpr (EPV == 1) {
    x[0] = load1<DT>(base, v);
  } else {
    unpack16<DT>(__ldcs(static_cast<const uint4*>(base) + v), x);
  }
}

template <int DT, int EPV>
__device__ __forceinline__ void store_vec(void* base, int64_t v, const float* x) {
  if constexpr (EPV == 1) {
    store1<DT>(base, v, x[0]);
  } else if constexpr (DT == NT_F32) {
    __stcs(static_cast<uint4*>(base) + v,
           make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3])));
  } else {
    uint4 raw;
    uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (DT == NT_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * k], x[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __half2 h = __floats2half2_rn(x[2 * k], x[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    __stcs(static_cast<uint4*>(base) + v, raw);
  }
}

// EPV > 1: vector v holds elements [v * EPV, v * EPV + EPV); EPV == 1: element v.
template <int DT, int OP, int EPV>
__global__ void __launch_bounds__(kFusedThreads) fused_kernel(const __grid_constant__ FusedParams P) {
  using O = FusedOp<OP>;
  const int64_t n = P.count / EPV;
  const int64_t stride = (int64_t)gridDim.x * kFusedThreads;
  int64_t v = (int64_t)blockIdx.x * kFusedThreads + threadIdx.x;
  float lo = 0.0f, hi = 0.0f;
  const bool has_lo = O::kClamp && P.b != nullptr, has_hi = O::kClamp && P.c != nullptr;
  if (has_lo) lo = load1<DT>(P.b, 0);
  if (has_hi) hi = load1<DT>(P.c, 0);
  // Bias column (in units of EPV) of vectors v and v + stride, advanced by the stride.
  const int64_t wv = O::kBias ? P.width / EPV : 1;
  int64_t col = O::kBias ? v % wv : 0;
  const int64_t step = O::kBias ? stride % wv : 0;
  auto advance = [&](int64_t c) {
    c += step;
    return c >= wv ? c - wv : c;
  };
  auto one = [&](int64_t vi, int64_t ci, float* out, float* sec) {
    float a[EPV], b[EPV], c[EPV], d[EPV];
    load_vec<DT, EPV>(P.a, vi, a);
    if constexpr (O::kBias) {
      if constexpr (EPV == 1) b[0] = load1<DT>(P.b, ci);
      else unpack16<DT>(__ldg(static_cast<const uint4*>(P.b) + ci), b);
    } else if constexpr (O::kReadB) {
      load_vec<DT, EPV>(P.b, vi, b);
    }
    if constexpr (O::kReadC) load_vec<DT, EPV>(P.c, vi, c);
    if constexpr (O::kReadD) load_vec<DT, EPV>(P.d, vi, d);
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      float s = 0.0f;
      out[e] = fused_value<OP, DT != NT_F32>(a[e], O::kReadB || O::kBias ? b[e] : 0.0f, O::kReadC ? c[e] : 0.0f,
                               O::kReadD ? d[e] : 0.0f, lo, hi, has_lo, has_hi, s);
      sec[e] = s;
    }
  };
  // Two vectors per iteration: both sets of loads are issued before either is used.
  for (; v + stride < n; v += 2 * stride) {
    const int64_t c2 = advance(col);
    float o1[EPV], s1[EPV], o2[EPV], s2[EPV];
    one(v, col, o1, s1);
    one(v + stride, c2, o2, s2);
    store_vec<DT, EPV>(P.out, v, o1);
    store_vec<DT, EPV>(P.out, v + stride, o2);
    if constexpr (O::kSecond) {
      store_vec<DT, EPV>(P.second, v, s1);
      store_vec<DT, EPV>(P.second, v + stride, s2);
    }
    col = advance(c2);
  }
  if (v < n) {
    float o[EPV], s[EPV];
    one(v, col, o, s);
    store_vec<DT, EPV>(P.out, v, o);
    if constexpr (O::kSecond) store_vec<DT, EPV>(P.second, v, s);
  }
}

// A persistent grid of exactly the resident blocks: a grid-stride loop over more blocks than
// fit at once would run the excess as a late second wave.
template <int DT, int OP, int EPV>
static int launch_fused(const FusedParams& P, cudaStream_t s) {
  static int per_sm = 0;
  if (per_sm == 0 && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_kernel<DT, OP, EPV>, kFusedThreads, 0) !=
                          cudaSuccess || per_sm < 1))
    per_sm = 4;
  const int64_t n = P.count / EPV;
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  const int64_t need = (n + kFusedThreads - 1) / kFusedThreads;
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  fused_kernel<DT, OP, EPV><<<(unsigned)grid, kFusedThreads, 0, s>>>(P);
  return launch_status("nt_fused_elementwise launch");
}

template <int DT, int OP>
static int dispatch_vec(const FusedParams& P, bool vec, cudaStream_t s) {
  constexpr int EPV = DT == NT_F32 ? 4 : 8;
  return vec ? launch_fused<DT, OP, EPV>(P, s) : launch_fused<DT, OP, 1>(P, s);
}

template <int DT>
static int dispatch_op(const FusedParams& P, int op, bool vec, cudaStream_t s) {
  switch (op) {
    case NT_FUSED_SIGMOID: return dispatch_vec<DT, NT_FUSED_SIGMOID>(P, vec, s);
    case NT_FUSED_SILU: return dispatch_vec<DT, NT_FUSED_SILU>(P, vec, s);
    case NT_FUSED_GELU_TANH: return dispatch_vec<DT, NT_FUSED_GELU_TANH>(P, vec, s);
    case NT_FUSED_SIGMOID_BACKWARD: return dispatch_vec<DT, NT_FUSED_SIGMOID_BACKWARD>(P, vec, s);
    case NT_FUSED_SILU_BACKWARD: return dispatch_vec<DT, NT_FUSED_SILU_BACKWARD>(P, vec, s);
    case NT_FUSED_GELU_TANH_BACKWARD: return dispatch_vec<DT, NT_FUSED_GELU_TANH_BACKWARD>(P, vec, s);
    case NT_FUSED_SWIGLU: return dispatch_vec<DT, NT_FUSED_SWIGLU>(P, vec, s);
    case NT_FUSED_SWIGLU_BACKWARD: return dispatch_vec<DT, NT_FUSED_SWIGLU_BACKWARD>(P, vec, s);
    case NT_FUSED_BIAS_SIGMOID: return dispatch_vec<DT, NT_FUSED_BIAS_SIGMOID>(P, vec, s);
    case NT_FUSED_BIAS_SILU: return dispatch_vec<DT, NT_FUSED_BIAS_SILU>(P, vec, s);
    case NT_FUSED_BIAS_GELU_TANH: return dispatch_vec<DT, NT_FUSED_BIAS_GELU_TANH>(P, vec, s);
    case NT_FUSED_BIAS_RELU: return dispatch_vec<DT, NT_FUSED_BIAS_RELU>(P, vec, s);
    case NT_FUSED_BIAS_SIGMOID_BACKWARD: return dispatch_vec<DT, NT_FUSED_BIAS_SIGMOID_BACKWARD>(P, vec, s);
    case NT_FUSED_BIAS_SILU_BACKWARD: return dispatch_vec<DT, NT_FUSED_BIAS_SILU_BACKWARD>(P, vec, s);
    case NT_FUSED_BIAS_GELU_TANH_BACKWARD: return dispatch_vec<DT, NT_FUSED_BIAS_GELU_TANH_BACKWARD>(P, vec, s);
    case NT_FUSED_BIAS_RELU_BACKWARD: return dispatch_vec<DT, NT_FUSED_BIAS_RELU_BACKWARD>(P, vec, s);
    case NT_FUSED_CLAMP: return dispatch_vec<DT, NT_FUSED_CLAMP>(P, vec, s);
    default: return dispatch_vec<DT, NT_FUSED_CLAMP_BACKWARD>(P, vec, s);
  }
}

// Operands the operation needs (bit 0 a ... bit 3 d; bit 4 second output).
static int fused_operands(int op) {
  switch (op) {
    case NT_FUSED_SIGMOID: case NT_FUSED_SILU: case NT_FUSED_GELU_TANH: return 0x1;
    case NT_FUSED_SIGMOID_BACKWARD: case NT_FUSED_SILU_BACKWARD: case NT_FUSED_GELU_TANH_BACKWARD:
    case NT_FUSED_SWIGLU: return 0x3;
    case NT_FUSED_SWIGLU_BACKWARD: return 0x7 | 0x10;
    case NT_FUSED_BIAS_SIGMOID: case NT_FUSED_BIAS_SILU: case NT_FUSED_BIAS_GELU_TANH: case NT_FUSED_BIAS_RELU:
      return 0x3;
    case NT_FUSED_BIAS_SIGMOID_BACKWARD: case NT_FUSED_BIAS_SILU_BACKWARD: case NT_FUSED_BIAS_GELU_TANH_BACKWARD:
    case NT_FUSED_BIAS_RELU_BACKWARD: return 0x7;
    case NT_FUSED_CLAMP: return 0x1;
    case NT_FUSED_CLAMP_BACKWARD: return 0x9;
    default: return -1;
  }
}

}  // namespace nt

using namespace nt;

extern "C" int nt_fused_elementwise(const nt_fused_args* args, void* stream) {
  nt::TraceRange trace("nt_fused_elementwise");
  if (!args) { set_error("nt_fused_elementwise: args is NULL"); return NT_EINVAL; }
  const nt_fused_args& a = *args;
  const int need = fused_operands(a.op);
  if (need < 0) { set_error("nt_fused_elementwise: unknown operation %d", a.op); return NT_EINVAL; }
  if (dtype_size(a.dtype) == 0) { set_error("nt_fused_elementwise: unsupported dtype %d", a.dtype); return NT_EUNSUPPORTED; }
  if (a.count < 0) { set_error("nt_fused_elementwise: negative count"); return NT_EINVAL; }
  const bool bias = a.op >= NT_FUSED_BIAS_SIGMOID && a.op <= NT_FUSED_BIAS_RELU_BACKWARD;
  const bool clamp = a.op == NT_FUSED_CLAMP || a.op == NT_FUSED_CLAMP_BACKWARD;
  if (bias && (a.width < 1 || a.count % a.width != 0)) {
    set_error("nt_fused_elementwise: bias operations need width >= 1 dividing count");
    return NT_EINVAL;
  }
  if (clamp && !a.b && !a.c) { set_error("nt_fused_elementwise: clamp needs a minimum or a maximum"); return NT_EINVAL; }
  if (a.count == 0) return NT_OK;
  const void* ops[4] = {a.a, a.b, a.c, a.d};
  for (int k = 0; k < 4; ++k)
    if ((need >> k & 1) && !ops[k]) { set_error("nt_fused_elementwise: operand %c is NULL", "abcd"[k]); return NT_EINVAL; }
  if (!a.output || ((need & 0x10) && !a.second)) { set_error("nt_fused_elementwise: NULL output"); return NT_EINVAL; }
  FusedParams P{};
  P.a = a.a; P.b = a.b; P.c = a.c; P.d = a.d; P.out = a.output; P.second = a.second;
  P.count = a.count; P.width = bias ? a.width : 1;
  const int epv = 16 / dtype_size(a.dtype);
  // Element-wise operands and outputs aligned to 16 bytes and a whole number of vectors (and of
  // vectors per bias row): the vector path.
  bool vec = a.count % epv == 0 && aligned16(a.a) && aligned16(a.output) && (!(need & 0x10) || aligned16(a.second));
  if (bias) vec = vec && a.width % epv == 0 && aligned16(a.b) && (!(need & 0x4) || aligned16(a.c));
  else if (!clamp) vec = vec && (!(need & 0x2) || aligned16(a.b)) && (!(need & 0x4) || aligned16(a.c));
  else vec = vec && (!(need & 0x8) || aligned16(a.d));
  cudaStream_t s = as_stream(stream);
  switch (a.dtype) {
    case NT_F32: return dispatch_op<NT_F32>(P, a.op, vec, s);
    case NT_F16: return dispatch_op<NT_F16>(P, a.op, vec, s);
    default: return dispatch_op<NT_BF16>(P, a.op, vec, s);
  }
}
