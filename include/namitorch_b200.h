/*
 * namitorch_b200 — C ABI of the B200 (sm_100a) optimizer-step / mixed-precision hot path.
 *
 * The reference (renderityai/NamiTorch) reaches its CUDA kernels through CuPy RawKernel
 * objects created from source strings (namitorch/backends/cuda/kernels.py:114-130) and
 * launched on CuPy's current stream. This library is what that seam binds instead: plain
 * pointers, element counts and a caller-given cudaStream_t passed as `void*` (NULL = the
 * legacy default stream). No torch, CuPy or Python types cross this boundary.
 *
 * Conventions
 *  - Every entry point returns an nt_status code. On failure, nt_last_error() returns a
 *    message for the calling thread (thread-local, valid until that thread's next call).
 *  - All kernel launches are asynchronous on `stream`; nothing here synchronises the host
 *    except nt_stream_synchronize / nt_memcpy_sync.
 *  - Device pointers are owned by the caller; the library never frees caller memory.
 *  - "Workspace" buffers are caller-allocated device memory that a kernel uses for its
 *    cross-block reduction. They must be zero-filled once after allocation; every call
 *    leaves them zeroed again. Two launches that share one workspace must not overlap.
 *  - Kernels never trap. A spin-wait that gives up, an out-of-range step index or a
 *    malformed table sets a device-side error word that the caller can read.
 */
#ifndef NAMITORCH_B200_H
#define NAMITORCH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NT_ABI_VERSION 8
#define NT_MAX_GROUPS 32      /* coefficient groups per nt_adamw_mt call */
#define NT_MAX_FOUND_INF 16   /* optimizers combined by one nt_scaler_update call */

typedef enum nt_status {
  NT_OK = 0,
  NT_EINVAL = 1,       /* bad argument: maps to ValueError / TypeError in the Python host */
  NT_ECUDA = 2,        /* CUDA runtime error (launch failure, invalid device, ...) */
  NT_ENOMEM = 3,       /* device allocation failed: maps to NamiTorchCUDAOutOfMemoryError */
  NT_EUNSUPPORTED = 4  /* layout or dtype this entry point does not handle */
} nt_status;

typedef enum nt_dtype {
  NT_F32 = 0,
  NT_F16 = 1,
  NT_BF16 = 2
} nt_dtype;

typedef enum nt_reduction {
  NT_REDUCTION_NONE = 0,
  NT_REDUCTION_MEAN = 1,
  NT_REDUCTION_SUM = 2
} nt_reduction;

/* ------------------------------------------------------------------------------------ */
/* Library / runtime                                                                     */
/* ------------------------------------------------------------------------------------ */

int nt_abi_version(void);
/* Message of the last failing call on this thread ("" when none). */
const char* nt_last_error(void);

/* Selects `device` for the calling thread and caches its SM count.
   Replaces CUDABackend.__init__ device selection (namitorch/backends/cuda/__init__.py:24-45). */
int nt_device_init(int device);
/* Number of SMs of the current device (148 on B200). */
int nt_sm_count(int* count);

/* Flat-buffer allocator primitives. Replace the CuPy MemoryPool wrapper
   (namitorch/backends/_cuda_memory.py:24-94); NT_ENOMEM carries the byte counts that
   NamiTorchCUDAOutOfMemoryError reports (_cuda_memory.py:8-21) in nt_last_error(). */
int nt_malloc(void** ptr, size_t bytes);
int nt_free(void* ptr);
int nt_mem_info(size_t* free_bytes, size_t* total_bytes);
int nt_memset_async(void* ptr, int value, size_t bytes, void* stream);
int nt_memcpy_async(void* dst, const void* src, size_t bytes, void* stream);
int nt_memcpy_sync(void* dst, const void* src, size_t bytes);
int nt_stream_synchronize(void* stream);

/* Elementwise dtype conversion (round-to-nearest-even), used to seed and refresh the
   low-precision model copy. Replaces the per-op autocast casts
   (namitorch/nn/functional.py:57-60, namitorch/tensor.py:634-636). */
int nt_cast(void* dst, int dst_dtype, const void* src, int src_dtype, int64_t count, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Per-tensor AdamW — the `backend.adamw` plugin seam                                    */
/* ------------------------------------------------------------------------------------ */

/* One fp32 AdamW step over `count` elements, bit-identical to the NumPy path.
   Replaces AdamWCUDAKernel.run (namitorch/backends/cuda/adamw.py:54-73) and its kernel
   namitorch_adamw_float32 (adamw.py:7-28). `coefficients` are the ten float32 values
   AdamW._update_parameter builds (namitorch/optim/adam.py:82-86):
   lr, beta1, beta2, 1-beta1, 1-beta2, eps, weight_decay, 1-lr*wd, 1-beta1^t, 1-beta2^t. */
int nt_adamw_f32(float* param, const float* grad, float* exp_avg, float* exp_avg_sq,
                 const float coefficients[10], int maximize, int update_parameter,
                 uint64_t count, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Multi-tensor fused AdamW + AMP over flat arenas                                       */
/* ------------------------------------------------------------------------------------ */

/* One parameter (or the part of one that a ZeRO-1 shard owns). */
typedef struct nt_segment {
  const void* grad;      /* gradient storage of the segment, dtype = args.grad_dtype */
  int64_t offset;        /* element offset of the segment in the fp32 arenas and the model copy */
  int64_t count;         /* elements */
  int64_t chunk_begin;   /* first work chunk: prefix sum of ceil(count / chunk_elems) */
  int32_t group;         /* index into args.groups */
  int32_t step_slot;     /* index into args.steps; each slot appears in at most one segment of a
                            call. A negative value -k-1 reads counter k but leaves it for a later
                            call (another piece of the same parameter) to advance. */
} nt_segment;

/* Per param-group coefficients, float32 exactly as the reference computes them
   (_scalar, namitorch/optim/_common.py:39-47; AdamW coefficients adam.py:82-86). */
typedef struct nt_adamw_group {
  float lr, beta1, beta2, one_minus_beta1, one_minus_beta2, eps, weight_decay, decay_factor;
  int32_t maximize;          /* negate the gradient (_common.py:57-62) */
  int32_t decay_mode;        /* NT_DECAY_*: decided from the unrounded weight decay != 0 */
  int32_t update_parameter;  /* 0 when lr == 0: moments and step still advance (adam.py:87) */
  int32_t correction_row;    /* row of this group in the bias-correction table */
  int32_t schedule_column;   /* column of this group in args.lr_schedule (ignored without one) */
  int32_t reserved;
} nt_adamw_group;

/* One learning-rate schedule entry of one parameter group for one scheduler step: the three
   lr-dependent coefficients, computed on the host exactly as the reference computes them
   from the scheduled lr (_scalar(lr), _scalar(1 - lr*wd), lr != 0). */
typedef struct nt_lr_entry {
  float lr;
  float decay_factor;
  int32_t update_parameter;
  int32_t reserved;
} nt_lr_entry;

enum {
  NT_DECAY_NONE = 0,
  NT_DECAY_DECOUPLED = 1,  /* AdamW: p = f32(p * decay_factor) before the update (_common.py:67-73) */
  NT_DECAY_COUPLED = 2     /* Adam: g = g + f32(wd) * p (_common.py:57-64) */
};

/* Device-resident gradient statistics (64 bytes). sumsq/nonfinite/nan are consecutive so
   that a ZeRO-1 process group can sum them with one all-reduce. */
typedef struct nt_stats {
  double sumsq;      /* sum of squared unscaled finite gradients */
  double nonfinite;  /* count of non-finite unscaled gradients */
  double nan;        /* count of NaN unscaled gradients */
  double maxabs;     /* max |g| over non-NaN unscaled gradients */
  double powsum;     /* sum (|g|/maxabs)^p, second pass of a general-p norm */
  double norm;       /* total norm, namitorch/optim/clip_grad.py:63-79 */
  double found_inf;  /* 1.0 when any unscaled gradient is non-finite (namitorch/amp.py:153-167) */
  double error;      /* non-zero when a kernel rejected its input */
} nt_stats;

typedef struct nt_adamw_mt_args {
  float* param;                   /* fp32 master arena */
  float* exp_avg;                 /* fp32 first-moment arena */
  float* exp_avg_sq;              /* fp32 second-moment arena */
  void* model_copy;               /* low-precision copy arena (same offsets) or NULL */
  int32_t model_dtype;            /* NT_F16 / NT_BF16 when model_copy != NULL */
  int32_t grad_dtype;             /* NT_F32 / NT_F16 / NT_BF16 */
  const nt_segment* segments;     /* device array */
  int32_t num_segments;
  int32_t chunk_elems;            /* elements per work chunk, multiple of 8 */
  int64_t num_chunks;             /* total chunks over all segments */
  int32_t* steps;                 /* device step counters, one per slot (state["step"]) */
  const float* corrections;       /* device [rows][capacity][2]: f32(1-beta1^t), f32(1-beta2^t) */
  int32_t correction_capacity;    /* t >= capacity reads row capacity-1, so the caller keeps t below
                                     capacity until that row holds (1.0f, 1.0f) in every group */
  const float* scale;             /* device GradScaler scale or NULL: gradients are divided by it */
  const nt_stats* stats;     /* device stats or NULL */
  int32_t skip_nonfinite;         /* skip the whole step when stats->found_inf != 0 (amp.py:210-217) */
  int32_t clip;                   /* multiply by max_norm/(stats->norm+1e-6) when < 1 (clip_grad.py:106-111) */
  double max_norm;
  void* workspace;                /* nt_adamw_workspace_size() bytes, zero-filled once */
  int32_t* error;                 /* device error word (may be NULL) */
  const nt_adamw_group* groups;   /* host array of num_groups entries */
  int32_t num_groups;             /* 1..NT_MAX_GROUPS */
  /* Optional device-side learning-rate schedule (no host round trip per step): when set, each
     group's lr, decay factor and update flag come from
     lr_schedule[min(*lr_step, rows - 1) * columns + group.schedule_column]. */
  const nt_lr_entry* lr_schedule; /* device [rows][columns] or NULL */
  int32_t lr_schedule_rows;
  int32_t lr_schedule_columns;
  const int32_t* lr_step;         /* device: the scheduler's step (nt_schedule_step advances it) */
} nt_adamw_mt_args;

size_t nt_adamw_workspace_size(void);

/* Fused AMP optimizer step over every segment: unscale by the device loss scale, skip on a
   device found_inf flag, global-norm clip, maximize / coupled or decoupled weight decay, the
   two moment updates, bias correction from the device step counter, the parameter update
   and the cast into the low-precision model copy, in one read-once / write-once pass.
   Replaces the chain GradScaler.unscale_ -> clip_grad_norm_ -> GradScaler.step ->
   _FirstOrderOptimizer.step -> AdamW._update_parameter (namitorch/amp.py:169-217,
   namitorch/optim/clip_grad.py:96-112, namitorch/optim/_common.py:133-167,
   namitorch/optim/adam.py:28-42 and :69-94). Step counters of the updated segments advance
   by one inside the same launch (the last block commits them). */
int nt_adamw_mt(const nt_adamw_mt_args* args, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Gradient statistics, clipping and loss scaling                                        */
/* ------------------------------------------------------------------------------------ */

/* A contiguous run of gradient elements for the statistics / transform kernels. */
typedef struct nt_span {
  const void* ptr;
  int64_t count;
  int64_t chunk_begin;   /* prefix sum of ceil(count / chunk_elems) */
} nt_span;

typedef struct nt_grad_stats_args {
  const nt_span* spans;  /* device array */
  int32_t num_spans;
  int32_t chunk_elems;   /* multiple of 8 */
  int64_t num_chunks;
  int32_t dtype;         /* NT_F32 / NT_F16 / NT_BF16 */
  const float* scale;    /* device loss scale or NULL */
  int32_t pass;          /* 0: sumsq / maxabs / counts; 1: powsum (reads stats->maxabs) */
  double norm_type;      /* p: 2, +inf or any positive value */
  int32_t finalize;      /* 1: the last block also writes norm and found_inf */
  nt_stats* stats;  /* device output */
  void* workspace;       /* nt_grad_stats_workspace_size() bytes, zero-filled once */
  size_t workspace_bytes;
} nt_grad_stats_args;

size_t nt_grad_stats_workspace_size(void);

/* One deterministic two-level reduction over all spans: block partials, then the last
   block reduces them in a fixed order. Replaces GradScaler._finite (namitorch/amp.py:153-167,
   run after unscale_) and _total_norm (namitorch/optim/clip_grad.py:63-79). Pass 0 gives
   found_inf, the max |g| and, for p = 2, the norm in one read; a general p needs pass 1. */
int nt_grad_stats(const nt_grad_stats_args* args, void* stream);

/* Allocation-free variant of nt_grad_stats (no counterpart in the reference). For callers
   that cannot allocate device memory themselves -- a host whose device memory is owned by
   its own pool, a plugin inside another runtime's allocator, a C/FFI caller without the
   CUDA allocation calls -- the block partials, the last-block ticket and the span table
   live in one static device array of nt_grad_stats_noalloc_scratch_bytes() bytes (about
   33 KB) inside this library; every GPU that loads the library holds it until the process
   exits. The caller still passes the gradients (`spans`: a HOST array of at most
   NT_NOALLOC_MAX_SPANS {ptr, count} pairs; chunk_begin is ignored), the device loss scale
   (or NULL) and the device nt_stats output. More spans are rejected with NT_EINVAL.
   Same result as nt_grad_stats with finalize = 1 (two passes for a general p).
   The first call in each CUDA context (normally once per device: the runtime's primary
   context; again after cudaDeviceReset, or in a context the caller created with the driver
   API) looks up the array's device address in that context and caches it under the
   context's ID; make that first call before any stream capture. All calls share the one array,
   so calls that overlap on the GPU (different streams, different host threads) race;
   serialise them. Nothing here calls cudaMalloc, cudaFree or an allocating library. */
#define NT_NOALLOC_MAX_SPANS 64
size_t nt_grad_stats_noalloc_scratch_bytes(void);
int nt_grad_stats_noalloc(const nt_span* spans, int32_t num_spans, int32_t dtype, const float* scale,
                          double norm_type, nt_stats* stats, void* stream);

/* The scheduler step gated on the device: *lr_step += 1 when every found_inf[i] is 0
   (count == 0: unconditionally). Replaces `if updated: scheduler.step()` of the training
   loop (namitorch/training/runner.py:250-254), which needs found_inf on the host.
   `found_inf` is a host array of `count` device pointers (nt_stats.found_inf fields). */
int nt_schedule_step(int32_t* lr_step, const double* const* found_inf, int32_t count, void* stream);

/* Computes norm and found_inf from the reduced fields (after a ZeRO-1 all-reduce). */
int nt_grad_stats_finalize(nt_stats* stats, double norm_type, void* stream);

/* Rewrites gradients in place: g = dtype(f32(g) / scale) when scale != NULL
   (GradScaler.unscale_, namitorch/amp.py:186-191), then g = dtype(f64(g) * coef) with
   coef = max_norm / (stats->norm + 1e-6) when clip != 0 and coef < 1
   (clip_grad_norm_, namitorch/optim/clip_grad.py:106-111). */
int nt_grad_transform(const nt_span* spans, int32_t num_spans, int32_t chunk_elems,
                      int64_t num_chunks, int32_t dtype, const float* scale,
                      const nt_stats* stats, int32_t clip, double max_norm, void* stream);

/* clip_grad_value_ (namitorch/optim/clip_grad.py:115-121): g = dtype(clip(f64(g), -v, v)). */
int nt_grad_clip_value(const nt_span* spans, int32_t num_spans, int32_t chunk_elems,
                       int64_t num_chunks, int32_t dtype, double clip_value, void* stream);

/* Dynamic loss-scale update on the device (GradScaler.update, namitorch/amp.py:219-234):
   any found_inf -> scale = f32(max(tiny, scale*backoff)), tracker = 0; otherwise
   tracker += 1 and, at growth_interval, scale = f32(min(f32max, scale*growth)), tracker = 0.
   `found_inf` is a host array of `count` device pointers (nt_stats.found_inf fields). */
int nt_scaler_update(float* scale, int32_t* growth_tracker, const double* const* found_inf,
                     int32_t count, double growth_factor, double backoff_factor,
                     int32_t growth_interval, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Row softmax family for attention scores                                               */
/* ------------------------------------------------------------------------------------ */

#define NT_SOFTMAX_MAX_WIDTH 4096
enum {
  NT_SOFTMAX = 0,
  NT_MASKED_SOFTMAX = 1,
  NT_CAUSAL_SOFTMAX = 2,
  NT_SOFTMAX_BACKWARD = 3,
  NT_MASKED_SOFTMAX_BACKWARD = 4,
  NT_CAUSAL_SOFTMAX_BACKWARD = 5
};

typedef struct nt_softmax_args {
  int32_t op;            /* NT_SOFTMAX ... NT_CAUSAL_SOFTMAX_BACKWARD */
  int32_t dtype;         /* NT_F32 / NT_F16 / NT_BF16 of input, gradient and output */
  const void* input;     /* [rows, width] scores (forward) or softmax output (backward), contiguous */
  const void* gradient;  /* [rows, width] upstream gradient (backward) or NULL */
  const uint8_t* mask;   /* bool [mask_rows or 1, width] (masked; optional for causal) or NULL */
  void* output;          /* [rows, width] */
  void* summary;         /* forward: NULL or device uint64[4] = {0, 0, UINT64_MAX, 0}, receiving
                            {rows with no allowed key, rows whose max is NaN or +inf, first such row} */
  int64_t rows;
  int64_t width;         /* 0..NT_SOFTMAX_MAX_WIDTH */
  int64_t mask_rows;     /* mask row of `row` is row % mask_rows; 0: one mask row for all */
  int64_t queries;       /* size of the query dimension (causal: allowed column <= offset + row % queries) */
  int64_t offset;        /* query position offset, clamped to width */
} nt_softmax_args;

/* The reference's SoftmaxCUDAKernels operations (namitorch/backends/cuda/softmax.py:6-178):
   softmax over the last dimension with an optional boolean mask and a causal rule, and the
   matching backward y * (g - sum(g * y)) restricted to the allowed entries. Float32 as in
   the reference, plus float16 / bfloat16 rows computed in float32. */
int nt_row_softmax(const nt_softmax_args* args, void* stream);

/* ------------------------------------------------------------------------------------ */
/* RMS / layer normalization                                                             */
/* ------------------------------------------------------------------------------------ */

#define NT_NORM_MAX_WIDTH 8192
enum { NT_RMS_NORM = 0, NT_LAYER_NORM = 1 };

typedef struct nt_norm_args {
  int32_t op;              /* NT_RMS_NORM / NT_LAYER_NORM */
  int32_t dtype;           /* NT_F32 / NT_F16 / NT_BF16 of input, weight, bias, output, gradient, grad_input */
  const void* input;       /* [rows, width] contiguous */
  const void* weight;      /* [width] or NULL */
  const void* bias;        /* [width] or NULL (layer norm only) */
  void* output;            /* forward: [rows, width] */
  float* statistics;       /* [rows, 2] float32 (shifted mean, 1/sqrt(var + eps)): written by the
                              forward (NULL: not saved), read by the backward */
  const void* gradient;    /* backward: [rows, width] upstream gradient */
  void* grad_input;        /* backward: [rows, width] or NULL */
  float* grad_weight;      /* backward: float32 [width] or NULL */
  float* grad_bias;        /* backward: float32 [width] or NULL */
  void* workspace;         /* backward with grad_weight / grad_bias: nt_norm_workspace_size bytes */
  size_t workspace_bytes;
  int64_t rows;
  int64_t width;           /* 1..NT_NORM_MAX_WIDTH */
  float eps;               /* forward: positive, finite */
} nt_norm_args;

/* Bytes of the per-tile partial sums the weight / bias gradients of [rows, width] need. */
size_t nt_norm_workspace_size(int64_t rows, int64_t width);

/* Forward of the reference's NormalizationCUDAKernels (namitorch/backends/cuda/normalization.py:
   58-84, 160-202): y = normalized * weight + bias with the statistics above; layer norm
   centres on the row's first element before the mean, as the reference does. */
int nt_norm_forward(const nt_norm_args* args, void* stream);

/* Backward (normalization.py:86-157, 204-235): grad_input from the saved statistics, and the
   weight / bias gradients as per-tile partial sums reduced per column in a fixed order. */
int nt_norm_backward(const nt_norm_args* args, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Fused elementwise activations                                                         */
/* ------------------------------------------------------------------------------------ */

/* The operations of the reference's FusedCUDAKernels (namitorch/backends/cuda/fused.py:44-69).
   Operand roles per operation (count elements each unless noted):
     NT_FUSED_SIGMOID, _SILU, _GELU_TANH                 output = f(a)
     NT_FUSED_SIGMOID_BACKWARD                           output = b * a * (1 - a)   (a = sigmoid output)
     NT_FUSED_SILU_BACKWARD, _GELU_TANH_BACKWARD         output = b * f'(a)
     NT_FUSED_SWIGLU                                     output = silu(a) * b
     NT_FUSED_SWIGLU_BACKWARD                            output = c * b * silu'(a), second = c * silu(a)
     NT_FUSED_BIAS_<F>        (b: [width])               output = f(a + b[i % width])
     NT_FUSED_BIAS_<F>_BACKWARD (b: [width], c: grad)    output = c * f'(a + b[i % width])
     NT_FUSED_CLAMP           (b, c: one element or NULL) output = clamp(a, b[0], c[0])
     NT_FUSED_CLAMP_BACKWARD  (d: grad)                   output = d where b[0] < a < c[0], else 0
   with the reference's special cases (stable sigmoid, silu(-inf) = 0, gelu beyond |x| > 20,
   NaN propagation in relu' and clamp). */
enum {
  NT_FUSED_SIGMOID = 0,
  NT_FUSED_SILU = 1,
  NT_FUSED_GELU_TANH = 2,
  NT_FUSED_SIGMOID_BACKWARD = 3,
  NT_FUSED_SILU_BACKWARD = 4,
  NT_FUSED_GELU_TANH_BACKWARD = 5,
  NT_FUSED_SWIGLU = 6,
  NT_FUSED_SWIGLU_BACKWARD = 7,
  NT_FUSED_BIAS_SIGMOID = 8,
  NT_FUSED_BIAS_SILU = 9,
  NT_FUSED_BIAS_GELU_TANH = 10,
  NT_FUSED_BIAS_RELU = 11,
  NT_FUSED_BIAS_SIGMOID_BACKWARD = 12,
  NT_FUSED_BIAS_SILU_BACKWARD = 13,
  NT_FUSED_BIAS_GELU_TANH_BACKWARD = 14,
  NT_FUSED_BIAS_RELU_BACKWARD = 15,
  NT_FUSED_CLAMP = 16,
  NT_FUSED_CLAMP_BACKWARD = 17
};

typedef struct nt_fused_args {
  int32_t op;            /* NT_FUSED_* */
  int32_t dtype;         /* NT_F32 / NT_F16 / NT_BF16 of every operand and output */
  const void* a;
  const void* b;         /* second operand, bias [width], or the clamp minimum (NULL: none) */
  const void* c;         /* third operand, or the clamp maximum (NULL: none) */
  const void* d;         /* clamp backward: upstream gradient */
  void* output;
  void* second;          /* swiglu backward: gradient of the second operand */
  int64_t count;         /* elements of `a` */
  int64_t width;         /* bias operations: size of the last dimension (count % width == 0) */
} nt_fused_args;

/* One fused elementwise operation, the kernel bodies of namitorch/backends/cuda/fused.py:
   8-69 (float32 there; float16 / bfloat16 here too, computed in float32 and rounded once). */
int nt_fused_elementwise(const nt_fused_args* args, void* stream);

/* ------------------------------------------------------------------------------------ */
/* ZeRO-1 over peer memory (NVLink / NVSwitch)                                           */
/* ------------------------------------------------------------------------------------ */
/* The reference has no distributed code. These entry points run the two ZeRO-1 exchanges
   inside the kernels that consume or produce the exchanged data, as loads and stores to
   the other GPUs' memory: the gradient reduce-scatter inside the statistics pass, and the
   model-copy all-gather inside the AdamW update. One process drives one GPU. Ordering
   between the ranks (peers' gradients written before they are read, every push landed
   before the copy is read) is the caller's: a stream-ordered barrier collective before
   nt_zero_reduce_scatter_stats and after nt_adamw_mt_push. */
#define NT_MAX_RANKS 8

/* CUDA IPC export of a device buffer that may start inside a larger allocation: the
   allocation's IPC handle and the byte offset of `ptr` inside it. */
int nt_ipc_export(const void* ptr, unsigned char handle[64], uint64_t* offset);

/* Maps an exported buffer of another process into this one, on the current device, with
   peer access enabled lazily; *ptr = mapping + offset. */
int nt_ipc_open(const unsigned char handle[64], uint64_t offset, void** ptr);

/* Unmaps a pointer returned by nt_ipc_open. */
int nt_ipc_close(void* ptr);

/* *ok = 1 when the current device can load from and store to device `peer` directly. */
int nt_can_access_peer(int32_t peer, int32_t* ok);

typedef struct nt_zero_reduce_args {
  const void* sources[NT_MAX_RANKS]; /* rank-ordered: rank q's gradients for this rank's shard
                                        (the local buffer at this rank's index, peer mappings
                                        elsewhere), all 16-byte aligned */
  int32_t num_ranks;                 /* 1..NT_MAX_RANKS */
  int32_t dtype;                     /* NT_F32 / NT_F16 / NT_BF16 */
  int64_t count;                     /* shard elements */
  int32_t average;                   /* 1: the sum is divided by num_ranks */
  void* dest;                        /* reduced shard (same dtype, 16-byte aligned); with count 0
                                        dest and sources may be NULL and only stats is written */
  const float* scale;                /* device loss scale applied to the statistics, or NULL */
  nt_stats* stats;                   /* device: sumsq, nonfinite, nan, maxabs of dest/scale */
  void* workspace;                   /* nt_grad_stats_workspace_size() bytes, zero-filled once */
  size_t workspace_bytes;
} nt_zero_reduce_args;

/* Reduce-scatter fused with the first statistics pass: dest[i] = dtype(sum over q in rank
   order of f32(sources[q][i]), divided by num_ranks when averaging), and, in the same pass,
   the pass-0 fields of nt_grad_stats over dest/scale. The norm and found_inf need the
   other ranks' fields: sum-reduce (sumsq, nonfinite, nan), max-reduce maxabs, then call
   nt_grad_stats_finalize. */
int nt_zero_reduce_scatter_stats(const nt_zero_reduce_args* args, void* stream);

/* nt_adamw_mt whose model-copy stores also go to `num_peers` (0..NT_MAX_RANKS-1) other
   copies: element `offset` of a segment is written at model_copy + offset and at
   peer_copies[k] + offset (same dtype), which fuses the ZeRO-1 all-gather of the model
   copy into the update. `peer_copies` is a host array of device pointers. */
int nt_adamw_mt_push(const nt_adamw_mt_args* args, void* const* peer_copies, int32_t num_peers, void* stream);

/* Cross-GPU ordering of the two ZeRO-1 kernels without NCCL: every rank owns one mailbox in
   its device memory (zero-filled once, exported with nt_ipc_export, mapped by the others);
   ranks write epochs into each other's mailboxes and wait on their own. No counterpart in
   the reference (it has no distributed code). */
#define NT_ZERO_READY 0   /* the rank's gradients are final: its shard may be pulled */
#define NT_ZERO_STATS 1   /* the rank's shard statistics are in stats[rank] */
#define NT_ZERO_DONE 2    /* the rank's pushes have landed and its pulls have ended */
typedef struct nt_zero_mailbox {
  uint64_t flags[3][NT_MAX_RANKS];  /* flags[k][q]: the last epoch at which rank q signalled k */
  double stats[NT_MAX_RANKS][4];    /* rank q's {sum g^2, #non-finite, #NaN, max|g|} of its shard */
} nt_zero_mailbox;

typedef struct nt_zero_sync {
  nt_zero_mailbox* mailboxes[NT_MAX_RANKS]; /* rank-ordered: this rank's own and every peer's */
  int32_t rank;
  int32_t reserved;
  uint64_t epoch;       /* this step's number: above every earlier one, the same on every rank */
  uint64_t timeout_ns;  /* bound of every wait on another rank */
  int32_t* error;       /* device word, sticky: |= 1 when a wait of the reduce-scatter ran out
                           (the statistics then report found_inf, so the update skips), |= 2
                           when the update's final wait ran out */
} nt_zero_sync;

/* nt_zero_reduce_scatter_stats plus the exchanges around it, in the same kernel: every rank
   signals READY and waits for every other rank's READY (all gradients final) before
   pulling; after the pull the last block sends the shard's statistics to every rank, waits
   for everyone's, adds them in rank order and finalizes with `norm_type` (2 or inf): every
   rank then holds the same global found_inf and norm, with no NCCL call. Every wait is
   bounded by sync->timeout_ns. */
int nt_zero_reduce_scatter_exchange(const nt_zero_reduce_args* args, const nt_zero_sync* sync, double norm_type,
                                    void* stream);

/* The exchanges of nt_zero_reduce_scatter_exchange as kernels of their own, for a
   reduce-scatter whose peer reads are copy-engine copies into local staging buffers (which
   keep more of each link busy than SM loads when both directions carry data):
   nt_zero_flag_exchange signals `flag` (NT_ZERO_READY before the copies, NT_ZERO_DONE after
   the last pushes) and waits for every rank's, bounded by sync->timeout_ns; *status (if
   given) becomes 0, or 1 if the wait ran out (also error bit 0 for READY / STATS, bit 1 for
   DONE). nt_zero_stats_exchange adds `count` statistics records in order (the pieces of the
   shard, each reduced by nt_zero_reduce_scatter_stats from the staged copies), exchanges
   the totals and finalizes `out` with `norm_type` (2 or inf) as the fused kernel does; a
   nonzero *ready_status skips the exchange and reports found_inf with a NaN norm. */
int nt_zero_flag_exchange(const nt_zero_sync* sync, int32_t num_ranks, int32_t flag, uint32_t* status, void* stream);
int nt_zero_stats_exchange(const nt_stats* records, int32_t count, const nt_zero_sync* sync, int32_t num_ranks,
                           const uint32_t* ready_status, double norm_type, nt_stats* out, void* stream);

/* nt_adamw_mt_push followed, in the same kernel, by the closing exchange: once every block's
   stores (its own copy and the peers') are complete, the last block signals DONE to every
   rank and waits for everyone's DONE, so when the kernel ends every peer's push into this
   rank's copy has landed and no peer still reads this rank's gradients. Launched even when
   the shard holds no parameter, and when the GradScaler skips the step. */
int nt_adamw_mt_push_exchange(const nt_adamw_mt_args* args, void* const* peer_copies, int32_t num_peers,
                              const nt_zero_sync* sync, void* stream);

/* No counterpart in the reference: copies `count` (1..NT_MAX_RANKS) independent ranges of
   `bytes_each` bytes (a multiple of 16; 16-byte aligned pointers), src[k] -> dst[k], with
   plain SM loads and stores as the two ZeRO-1 kernels above issue them (no copy engine, no
   multicast): 32-byte accesses when every pointer is 32-byte aligned and bytes_each a
   multiple of 32, else 16-byte. With src pointing at peers' memory (nt_ipc_open) it measures the
   inbound peer bandwidth the reduce-scatter pull sees; with dst at peers, the outbound
   bandwidth of the all-gather push. `src` and `dst` are host arrays of device pointers. */
int nt_peer_copy(const void* const* src, void* const* dst, int32_t count, uint64_t bytes_each, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Fused softmax cross-entropy forward + backward                                        */
/* ------------------------------------------------------------------------------------ */

/* Device-resident summary of the targets (filled by nt_softmax_xent). */
typedef struct nt_xent_info {
  double denominator;   /* mean-reduction denominator: valid rows, or sum of their class weights */
  double weight_sum;    /* sum of all class weights (C without weights) */
  double loss_sum;      /* sum of the per-row losses */
  double n_valid;       /* rows whose target != ignore_index */
  double bad_targets;   /* non-ignored targets outside [0, C) (the reference raises IndexError) */
  double error;         /* non-zero when a bounded wait gave up */
  double reserved[2];
} nt_xent_info;

typedef struct nt_xent_args {
  const void* logits;        /* [rows, classes] contiguous */
  int32_t dtype;             /* NT_F32 / NT_F16 / NT_BF16 */
  int64_t rows;
  int64_t classes;
  const int64_t* targets;    /* [rows] */
  int64_t ignore_index;
  const float* class_weight; /* [classes] or NULL */
  float label_smoothing;     /* in [0, 1) */
  int32_t reduction;         /* nt_reduction */
  void* dlogits;             /* [rows, classes] same dtype, or NULL for forward only */
  float* loss;               /* [rows] for NONE, [1] otherwise */
  float* row_loss;           /* scratch [rows] (may alias loss for NONE) */
  nt_xent_info* info;        /* device; the call resets it before use */
  void* workspace;           /* nt_xent_workspace_size() bytes, zero-filled once */
  size_t workspace_bytes;
} nt_xent_args;

size_t nt_xent_workspace_size(void);

/* Cross-entropy of logits against integer targets and, in the same pass, its gradient for
   a unit upstream gradient: mean over non-ignored rows of -log_softmax(x)[t], with class
   weights, label smoothing and ignore_index. Replaces F.cross_entropy
   (namitorch/nn/functional.py:792-863), the log_softmax forward
   (namitorch/_backend.py:321-354) and its backward (namitorch/autograd.py:538-564).
   One HBM read of the logits and one write of dlogits. */
int nt_softmax_xent(const nt_xent_args* args, void* stream);

/* Multiplies dlogits by the upstream gradient read on the device: one scalar (returns
   without touching memory when it is exactly 1) or one value per row (reduction NONE). */
int nt_xent_backward_scale(void* dlogits, int32_t dtype, int64_t rows, int64_t classes,
                           const float* grad_output, int32_t per_row, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NAMITORCH_B200_H */
