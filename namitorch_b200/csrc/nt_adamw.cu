// AdamW kernels.
//
// Arithmetic contract: every float32 operation of the reference NumPy path
// (namitorch/optim/adam.py:28-42, namitorch/optim/_common.py:57-73) is issued as a separately
// rounded IEEE operation (__fmul_rn / __fadd_rn / __fdiv_rn / __fsqrt_rn), in the reference's
// order, so no multiply-add is ever contracted and the results are bit-identical to NumPy:
//   g  = -g if maximize;  g = g + f32(wd)*p for coupled Adam
//   m  = b1*m + (1-b1)*g
//   v  = b2*v + ((1-b2)*g)*g
//   p  = p*decay (AdamW, wd != 0);  p = p - lr*((m/c1) / (sqrt(v/c2) + eps))
// with c1 = f32(1-b1^t), c2 = f32(1-b2^t) computed on the host exactly as the reference.
// A division by a correction that has reached exactly 1.0f is skipped (x / 1 == x).
#include "nt_common.cuh"
#include "nt_peer_sync.cuh"

namespace nt {

constexpr int kNoCopy = -1;

struct Coef {
  float lr, b1, b2, c1, c2, eps, wd, decay, corr1, corr2;
  int decay_mode;
  bool maximize, update;
};

__device__ __forceinline__ void adam_update(float& p, float g, float& m, float& v, const Coef& c) {
  if (c.maximize) g = -g;
  if (c.decay_mode == NT_DECAY_COUPLED) g = __fadd_rn(g, __fmul_rn(c.wd, p));
  m = __fadd_rn(__fmul_rn(c.b1, m), __fmul_rn(c.c1, g));
  v = __fadd_rn(__fmul_rn(c.b2, v), __fmul_rn(__fmul_rn(c.c2, g), g));
  if (c.update) {
    const float fc = c.corr1 == 1.0f ? m : __fdiv_rn(m, c.corr1);
    const float sc = c.corr2 == 1.0f ? v : __fdiv_rn(v, c.corr2);
    const float den = __fadd_rn(__fsqrt_rn(sc), c.eps);
    const float u = __fdiv_rn(fc, den);
    const float base = c.decay_mode == NT_DECAY_DECOUPLED ? __fmul_rn(p, c.decay) : p;
    p = __fsub_rn(base, __fmul_rn(c.lr, u));
  }
}

// ---------------------------------------------------------------------------------------
// Per-tensor kernel: the `backend.adamw` seam (namitorch/backends/cuda/adamw.py:7-28).
// Same operation order as the reference kernel compiled with --fmad=false.
// ---------------------------------------------------------------------------------------
struct SingleArgs {
  float* p;
  const float* g;
  float* m;
  float* v;
  uint64_t count;
  float coef[10];
  int maximize;
  int update;
  int vec;
};

__device__ __forceinline__ void single_elem(float& p, float g, float& m, float& v, const SingleArgs& a) {
  const float lr = a.coef[0], b1 = a.coef[1], b2 = a.coef[2], c1 = a.coef[3], c2 = a.coef[4];
  const float eps = a.coef[5], wd = a.coef[6], decay = a.coef[7], corr1 = a.coef[8], corr2 = a.coef[9];
  if (a.maximize) g = -g;
  m = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(c1, g));
  v = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(c2, g), g));
  if (a.update) {
    float value = p;
    if (wd != 0.0f) value = __fmul_rn(value, decay);
    const float corrected = __fdiv_rn(m, corr1);
    const float den = __fadd_rn(__fsqrt_rn(__fdiv_rn(v, corr2)), eps);
    p = __fsub_rn(value, __fmul_rn(lr, __fdiv_rn(corrected, den)));
  }
}

__global__ void __launch_bounds__(256) adamw_single_kernel(const __grid_constant__ SingleArgs a) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t tail_begin = 0;
  if (a.vec) {
    const uint64_t nvec = a.count / 8;
    for (uint64_t i = t; i < nvec; i += stride) {
      float p[8], g[8], m[8], v[8];
      load8_f32(a.p + i * 8, p);
      load8_f32(a.g + i * 8, g);
      load8_f32(a.m + i * 8, m);
      load8_f32(a.v + i * 8, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) single_elem(p[k], g[k], m[k], v[k], a);
      store8_f32(a.m + i * 8, m);
      store8_f32(a.v + i * 8, v);
      if (a.update) store8_f32(a.p + i * 8, p);
    }
    tail_begin = nvec * 8;
  }
  for (uint64_t i = tail_begin + t; i < a.count; i += stride) {
    float p = a.p[i], m = a.m[i], v = a.v[i];
    single_elem(p, a.g[i], m, v, a);
    a.m[i] = m;
    a.v[i] = v;
    if (a.update) a.p[i] = p;
  }
}

// ---------------------------------------------------------------------------------------
// Multi-tensor fused AMP kernel.
// ---------------------------------------------------------------------------------------
struct MtParams {
  float* p;
  float* m;
  float* v;
  void* copy;
  const nt_segment* segs;
  int nseg;
  int chunk_elems;
  int64_t nchunks;
  int32_t* steps;
  const float2* corr;
  int cap;
  const float* scale;
  const nt_stats* stats;
  int skip_nonfinite;
  int clip;
  double max_norm;
  unsigned* counter;
  int32_t* error;
  int ngroups;
  int npeers;                        // other model copies the update also writes (ZeRO-1)
  void* peers[NT_MAX_RANKS - 1];
  const nt_lr_entry* sched;          // device lr schedule or NULL
  int sched_rows;
  int sched_cols;
  const int32_t* sched_step;
  PeerSync sync;                     // the closing exchange (nt_adamw_mt_push_exchange only)
  int vec32;                         // p, m and v start on 32-byte boundaries: 256-bit accesses
  nt_adamw_group groups[NT_MAX_GROUPS];
};

struct AdamwWorkspace {
  unsigned counter;
  unsigned pad[63];
};

// Stores 8 updated parameters into the model copy and, with PUSH, into every peer's copy
// at the same offset (the ZeRO-1 all-gather, as stores over NVLink).
template <int CDT, bool PUSH>
__device__ __forceinline__ void store_copy8(const MtParams& P, int64_t ai, const float v[8]) {
  using T = typename Elem<CDT>::T;
  uint4 raw;
  T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int k = 0; k < 8; ++k) h[k] = Elem<CDT>::from_f32(v[k]);
  __stcs(reinterpret_cast<uint4*>(static_cast<T*>(P.copy) + ai), raw);
  if constexpr (PUSH) {
#pragma unroll 1
    for (int q = 0; q < P.npeers; ++q) __stcs(reinterpret_cast<uint4*>(static_cast<T*>(P.peers[q]) + ai), raw);
  }
}

template <int CDT, bool PUSH>
__device__ __forceinline__ void store_copy1(const MtParams& P, int64_t ai, float v) {
  store1<CDT>(P.copy, ai, v);
  if constexpr (PUSH) {
    for (int q = 0; q < P.npeers; ++q) store1<CDT>(P.peers[q], ai, v);
  }
}

template <int GDT, int CDT, bool PUSH>
__device__ __forceinline__ void mt_vec8(const MtParams& P, int64_t ai, const void* g, int64_t gi,
                                        const Coef& c, const Unscale& un, bool clip, double coef) {
  float pv[8], mv[8], vv[8], gv[8];
  if (P.vec32) {   // uniform across the grid
    load8_f32_v8(P.p + ai, pv);
    load8_f32_v8(P.m + ai, mv);
    load8_f32_v8(P.v + ai, vv);
  } else {
    load8_f32(P.p + ai, pv);
    load8_f32(P.m + ai, mv);
    load8_f32(P.v + ai, vv);
  }
  load8<GDT>(g, gi, gv);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float gg = un(gv[k]);
    if (clip) gg = __double2float_rn(__dmul_rn((double)gg, coef));
    adam_update(pv[k], gg, mv[k], vv[k], c);
  }
  if (P.vec32) {
    store8_f32_v8(P.m + ai, mv);
    store8_f32_v8(P.v + ai, vv);
  } else {
    store8_f32(P.m + ai, mv);
    store8_f32(P.v + ai, vv);
  }
  if (c.update) {
    if (P.vec32) store8_f32_v8(P.p + ai, pv);
    else store8_f32(P.p + ai, pv);
    if constexpr (CDT != kNoCopy) store_copy8<CDT, PUSH>(P, ai, pv);
  }
}

template <int GDT, int CDT, bool PUSH>
__device__ __forceinline__ void mt_elem(const MtParams& P, int64_t ai, const void* g, int64_t gi,
                                        const Coef& c, const Unscale& un, bool clip, double coef) {
  float p = P.p[ai], m = P.m[ai], v = P.v[ai];
  float gg = un(load1<GDT>(g, gi));
  if (clip) gg = __double2float_rn(__dmul_rn((double)gg, coef));
  adam_update(p, gg, m, v, c);
  P.m[ai] = m;
  P.v[ai] = v;
  if (c.update) {
    P.p[ai] = p;
    if constexpr (CDT != kNoCopy) store_copy1<CDT, PUSH>(P, ai, p);
  }
}

template <int GDT, int CDT, bool PUSH, bool SYNC>
__global__ void __launch_bounds__(256) adamw_mt_kernel(const __grid_constant__ MtParams P) {
  __shared__ bool last;
  const bool skip = P.stats != nullptr && P.skip_nonfinite && P.stats->found_inf != 0.0;   // GradScaler skip
  if (!SYNC && skip) return;   // with SYNC the blocks still reach the closing exchange
  Unscale un;
  un.init(P.scale);
  bool clip = false;
  double coef = 1.0;
  if (P.clip && P.stats != nullptr) {
    const double c = P.max_norm / (P.stats->norm + 1e-6);
    if (c < 1.0) { clip = true; coef = c; }
  }
  const int gsize = GDT == NT_F32 ? 4 : 2;
  int sched_row = 0;
  if (P.sched != nullptr) {
    sched_row = *P.sched_step;
    sched_row = sched_row < 0 ? 0 : (sched_row >= P.sched_rows ? P.sched_rows - 1 : sched_row);
  }

  // Each block takes a contiguous range of chunks: one segment lookup per block, then the
  // segment's record, coefficients and bias corrections are carried in registers until the
  // chunks cross into the next segment.
  const int64_t per = (P.nchunks + gridDim.x - 1) / gridDim.x;
  const int64_t c0 = (int64_t)blockIdx.x * per;
  const int64_t c1 = skip ? c0 : (c0 + per < P.nchunks ? c0 + per : P.nchunks);
  int s = c0 < c1 ? find_owner([&](int i) { return P.segs[i].chunk_begin; }, P.nseg, c0) : 0;
  int64_t next_begin = -1;  // forces a load of segment s at the first chunk
  nt_segment seg{};
  Coef c{};
  bool seg_ok = false;
  for (int64_t chunk = c0; chunk < c1; ++chunk) {
    if (chunk >= next_begin) {
      if (next_begin >= 0) ++s;
      while (s + 1 < P.nseg && P.segs[s + 1].chunk_begin <= chunk) ++s;
      seg = P.segs[s];
      next_begin = s + 1 < P.nseg ? P.segs[s + 1].chunk_begin : INT64_MAX;
      const nt_adamw_group& gr = P.groups[seg.group];
      const int slot = seg.step_slot >= 0 ? seg.step_slot : -seg.step_slot - 1;
      const int t = P.steps[slot] + 1;
      seg_ok = t > 0;
      if (!seg_ok && threadIdx.x == 0 && P.error) atomicOr(P.error, 1);
      // Steps past the table use its last row: the host only lets that happen once every
      // row has saturated at exactly 1.0f, where f32(1 - beta^t) stays for all larger t.
      const int ti = t < P.cap ? t : P.cap - 1;
      const float2 corr = seg_ok ? P.corr[(int64_t)gr.correction_row * P.cap + ti] : make_float2(1.0f, 1.0f);
      c.lr = gr.lr; c.b1 = gr.beta1; c.b2 = gr.beta2; c.c1 = gr.one_minus_beta1; c.c2 = gr.one_minus_beta2;
      c.eps = gr.eps; c.wd = gr.weight_decay; c.decay = gr.decay_factor; c.corr1 = corr.x; c.corr2 = corr.y;
      c.decay_mode = gr.decay_mode; c.maximize = gr.maximize != 0; c.update = gr.update_parameter != 0;
      if (P.sched != nullptr) {   // this step's scheduled lr-dependent coefficients
        const nt_lr_entry e = P.sched[(int64_t)sched_row * P.sched_cols + gr.schedule_column];
        c.lr = e.lr; c.decay = e.decay_factor; c.update = e.update_parameter != 0;
      }
    }
    if (!seg_ok) continue;

    const int64_t begin = (chunk - seg.chunk_begin) * (int64_t)P.chunk_elems;
    int64_t end = begin + P.chunk_elems;
    if (end > seg.count) end = seg.count;
    const int64_t abase = seg.offset;
    const char* gbytes = static_cast<const char*>(seg.grad);
    const bool vec = ((abase + begin) & 7) == 0 &&
                     ((reinterpret_cast<uintptr_t>(gbytes + begin * gsize)) & 15u) == 0;
    int64_t e = begin;
    if (vec) {
      const int64_t body_end = begin + ((end - begin) & ~(int64_t)7);
      for (int64_t i = begin + (int64_t)threadIdx.x * 8; i < body_end; i += (int64_t)blockDim.x * 8)
        mt_vec8<GDT, CDT, PUSH>(P, abase + i, seg.grad, i, c, un, clip, coef);
      e = body_end;
    }
    for (int64_t i = e + threadIdx.x; i < end; i += blockDim.x)
      mt_elem<GDT, CDT, PUSH>(P, abase + i, seg.grad, i, c, un, clip, coef);
  }

  // The last block advances the step counter of every updated segment. With SYNC the ticket
  // is taken at system scope (every block's stores, the pushes to the peers included, are
  // then visible everywhere) and the last block closes the step: DONE to every rank, then
  // a bounded wait for every rank's DONE.
  if (SYNC ? last_block_ticket_sys(P.counter, &last) : last_block_ticket(P.counter, &last)) {
    if (!skip) {
      for (int i = threadIdx.x; i < P.nseg; i += blockDim.x) {
        const int slot = P.segs[i].step_slot;
        if (slot >= 0) P.steps[slot] += 1;  // negative: another launch advances this counter
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      *P.counter = 0u;
      if constexpr (SYNC) {
        signal_all(P.sync, NT_ZERO_DONE);
        if (!wait_all(P.sync, NT_ZERO_DONE)) atomicOr(P.sync.error, 2);
      }
    }
  }
}

// The closing exchange alone, for a rank with nothing to update (an empty shard).
__global__ void zero_done_kernel(const __grid_constant__ PeerSync S) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    signal_all(S, NT_ZERO_DONE);
    if (!wait_all(S, NT_ZERO_DONE)) atomicOr(S.error, 2);
  }
}

template <int GDT, int CDT, bool PUSH, bool SYNC = false>
static int launch_mt(const MtParams& P, cudaStream_t stream) {
  static int per_sm = 0;
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adamw_mt_kernel<GDT, CDT, PUSH, SYNC>, 256, 0) !=
            cudaSuccess ||
        per_sm <= 0)
      per_sm = 2;
  }
  int64_t grid = (int64_t)current_sm_count() * per_sm;
  if (grid > P.nchunks) grid = P.nchunks;
  if (grid < 1) grid = 1;
  adamw_mt_kernel<GDT, CDT, PUSH, SYNC><<<(unsigned)grid, 256, 0, stream>>>(P);
  return launch_status("nt_adamw_mt launch");
}

template <int GDT>
static int dispatch_copy_sync(const MtParams& P, int copy_dtype, cudaStream_t stream) {
  if (copy_dtype == NT_BF16) return launch_mt<GDT, NT_BF16, true, true>(P, stream);
  if (copy_dtype == NT_F16) return launch_mt<GDT, NT_F16, true, true>(P, stream);
  set_error("nt_adamw_mt_push_exchange: model copy dtype must be NT_F16 or NT_BF16 (got %d)", copy_dtype);
  return NT_EUNSUPPORTED;
}

template <int GDT>
static int dispatch_copy(const MtParams& P, int copy_dtype, cudaStream_t stream) {
  const bool push = P.npeers > 0;
  if (P.copy == nullptr) return launch_mt<GDT, kNoCopy, false>(P, stream);
  if (copy_dtype == NT_BF16)
    return push ? launch_mt<GDT, NT_BF16, true>(P, stream) : launch_mt<GDT, NT_BF16, false>(P, stream);
  if (copy_dtype == NT_F16)
    return push ? launch_mt<GDT, NT_F16, true>(P, stream) : launch_mt<GDT, NT_F16, false>(P, stream);
  set_error("nt_adamw_mt: model copy dtype must be NT_F16 or NT_BF16 (got %d)", copy_dtype);
  return NT_EUNSUPPORTED;
}

// Validates the arguments and fills the kernel parameters; NT_OK with P.nchunks == 0 means
// there is nothing to launch.
static int build_mt_params(const nt_adamw_mt_args* args, MtParams& P) {
  if (!args) { set_error("nt_adamw_mt: args is NULL"); return NT_EINVAL; }
  const nt_adamw_mt_args& a = *args;
  if (a.num_segments < 0 || a.num_chunks < 0) { set_error("nt_adamw_mt: negative sizes"); return NT_EINVAL; }
  P.nchunks = 0;
  P.npeers = 0;
  if (a.num_segments == 0 || a.num_chunks == 0) return NT_OK;
  if (!a.param || !a.exp_avg || !a.exp_avg_sq || !a.segments || !a.steps || !a.corrections || !a.workspace) {
    set_error("nt_adamw_mt: NULL param/exp_avg/exp_avg_sq/segments/steps/corrections/workspace");
    return NT_EINVAL;
  }
  if (a.chunk_elems <= 0 || (a.chunk_elems & 7) != 0) {
    set_error("nt_adamw_mt: chunk_elems must be a positive multiple of 8 (got %d)", a.chunk_elems);
    return NT_EINVAL;
  }
  if (a.num_groups < 1 || a.num_groups > NT_MAX_GROUPS || !a.groups) {
    set_error("nt_adamw_mt: num_groups must be in [1, %d] (got %d)", NT_MAX_GROUPS, a.num_groups);
    return NT_EINVAL;
  }
  if (a.correction_capacity < 2) { set_error("nt_adamw_mt: correction_capacity < 2"); return NT_EINVAL; }
  if ((a.skip_nonfinite || a.clip) && !a.stats) {
    set_error("nt_adamw_mt: skip_nonfinite / clip need stats");
    return NT_EINVAL;
  }
  if (!aligned16(a.param) || !aligned16(a.exp_avg) || !aligned16(a.exp_avg_sq) ||
      (a.model_copy && !aligned16(a.model_copy))) {
    set_error("nt_adamw_mt: arenas must be 16-byte aligned");
    return NT_EINVAL;
  }
  for (int i = 0; i < a.num_groups; ++i) {
    const nt_adamw_group& g = a.groups[i];
    if (!(g.eps > 0.0f) || !isfinite(g.lr) || !isfinite(g.beta1) || !isfinite(g.beta2) ||
        !isfinite(g.weight_decay) || !isfinite(g.decay_factor) || g.decay_mode < 0 || g.decay_mode > 2 ||
        g.correction_row < 0) {
      set_error("nt_adamw_mt: group %d has invalid coefficients", i);
      return NT_EINVAL;
    }
  }
  P.p = a.param; P.m = a.exp_avg; P.v = a.exp_avg_sq; P.copy = a.model_copy;
  // The vector path runs at element offsets that are multiples of 8 (32 bytes of fp32), so
  // 32-byte aligned arenas allow one 256-bit access per 8 values.
  P.vec32 = ((reinterpret_cast<uintptr_t>(a.param) | reinterpret_cast<uintptr_t>(a.exp_avg) |
              reinterpret_cast<uintptr_t>(a.exp_avg_sq)) & 31u) == 0;
  P.segs = a.segments; P.nseg = a.num_segments; P.chunk_elems = a.chunk_elems; P.nchunks = a.num_chunks;
  P.steps = a.steps; P.corr = reinterpret_cast<const float2*>(a.corrections); P.cap = a.correction_capacity;
  P.scale = a.scale; P.stats = a.stats; P.skip_nonfinite = a.skip_nonfinite; P.clip = a.clip;
  P.max_norm = a.max_norm;
  P.counter = &static_cast<AdamwWorkspace*>(a.workspace)->counter;
  P.error = a.error;
  P.ngroups = a.num_groups;
  for (int i = 0; i < a.num_groups; ++i) P.groups[i] = a.groups[i];
  P.sched = a.lr_schedule;
  P.sched_rows = a.lr_schedule_rows;
  P.sched_cols = a.lr_schedule_columns;
  P.sched_step = a.lr_step;
  if (a.lr_schedule) {
    if (!a.lr_step || a.lr_schedule_rows < 1 || a.lr_schedule_columns < 1) {
      set_error("nt_adamw_mt: lr_schedule needs lr_step, rows >= 1 and columns >= 1");
      return NT_EINVAL;
    }
    for (int i = 0; i < a.num_groups; ++i) {
      if (a.groups[i].schedule_column < 0 || a.groups[i].schedule_column >= a.lr_schedule_columns) {
        set_error("nt_adamw_mt: group %d schedule_column %d outside [0, %d)", i, a.groups[i].schedule_column,
                  a.lr_schedule_columns);
        return NT_EINVAL;
      }
    }
  }
  return NT_OK;
}

static int dispatch_mt_sync(const MtParams& P, const nt_adamw_mt_args& a, cudaStream_t s) {
  switch (a.grad_dtype) {
    case NT_F32: return dispatch_copy_sync<NT_F32>(P, a.model_dtype, s);
    case NT_F16: return dispatch_copy_sync<NT_F16>(P, a.model_dtype, s);
    case NT_BF16: return dispatch_copy_sync<NT_BF16>(P, a.model_dtype, s);
    default:
      set_error("nt_adamw_mt_push_exchange: unsupported gradient dtype %d", a.grad_dtype);
      return NT_EUNSUPPORTED;
  }
}

// Checks the peer copies of a push and stores them in P.
static int set_push_peers(const nt_adamw_mt_args* args, void* const* peer_copies, int32_t num_peers, MtParams& P,
                          const char* what) {
  if (num_peers < 0 || num_peers > NT_MAX_RANKS - 1 || (num_peers > 0 && !peer_copies)) {
    set_error("%s: num_peers must be in [0, %d] with a peer array (got %d)", what, NT_MAX_RANKS - 1, num_peers);
    return NT_EINVAL;
  }
  if (num_peers > 0 && !args->model_copy) {
    set_error("%s: peer copies need a model copy", what);
    return NT_EINVAL;
  }
  for (int q = 0; q < num_peers; ++q) {
    if (!peer_copies[q] || !aligned16(peer_copies[q])) {
      set_error("%s: peer copy %d is NULL or not 16-byte aligned", what, q);
      return NT_EINVAL;
    }
    P.peers[q] = peer_copies[q];
  }
  P.npeers = num_peers;
  return NT_OK;
}

static int dispatch_mt(const MtParams& P, const nt_adamw_mt_args& a, cudaStream_t s) {
  switch (a.grad_dtype) {
    case NT_F32: return dispatch_copy<NT_F32>(P, a.model_dtype, s);
    case NT_F16: return dispatch_copy<NT_F16>(P, a.model_dtype, s);
    case NT_BF16: return dispatch_copy<NT_BF16>(P, a.model_dtype, s);
    default:
      set_error("nt_adamw_mt: unsupported gradient dtype %d", a.grad_dtype);
      return NT_EUNSUPPORTED;
  }
}

}  // namespace nt

using namespace nt;

extern "C" {

int nt_adamw_f32(float* param, const float* grad, float* exp_avg, float* exp_avg_sq,
                 const float coefficients[10], int maximize, int update_parameter,
                 uint64_t count, void* stream) {
  nt::TraceRange trace("nt_adamw_f32");
  if (!coefficients) { set_error("nt_adamw_f32: coefficients is NULL"); return NT_EINVAL; }
  for (int i = 0; i < 10; ++i) {
    if (!isfinite(coefficients[i])) {
      set_error("Fused AdamW requires ten finite float32 coefficients.");
      return NT_EINVAL;
    }
  }
  if (coefficients[5] <= 0.0f || coefficients[8] <= 0.0f || coefficients[9] <= 0.0f) {
    set_error("Fused AdamW eps and bias corrections must be positive.");
    return NT_EINVAL;
  }
  if (count == 0) return NT_OK;
  if (!param || !grad || !exp_avg || !exp_avg_sq) {
    set_error("nt_adamw_f32: NULL array");
    return NT_EINVAL;
  }
  SingleArgs a;
  a.p = param; a.g = grad; a.m = exp_avg; a.v = exp_avg_sq; a.count = count;
  for (int i = 0; i < 10; ++i) a.coef[i] = coefficients[i];
  a.maximize = maximize != 0;
  a.update = update_parameter != 0;
  a.vec = aligned16(param) && aligned16(grad) && aligned16(exp_avg) && aligned16(exp_avg_sq);
  const uint64_t work = a.vec ? (count + 7) / 8 : count;
  uint64_t grid = (work + 255) / 256;
  const uint64_t cap = (uint64_t)current_sm_count() * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  adamw_single_kernel<<<(unsigned)grid, 256, 0, as_stream(stream)>>>(a);
  return launch_status("nt_adamw_f32 launch");
}

size_t nt_adamw_workspace_size(void) { return sizeof(AdamwWorkspace); }

int nt_adamw_mt(const nt_adamw_mt_args* args, void* stream) {
  nt::TraceRange trace("nt_adamw_mt");
  MtParams P;
  const int rc = build_mt_params(args, P);
  if (rc != NT_OK || P.nchunks == 0) return rc;
  return dispatch_mt(P, *args, as_stream(stream));
}

int nt_adamw_mt_push(const nt_adamw_mt_args* args, void* const* peer_copies, int32_t num_peers, void* stream) {
  nt::TraceRange trace("nt_adamw_mt_push");
  MtParams P;
  int rc = build_mt_params(args, P);
  if (rc != NT_OK || P.nchunks == 0) return rc;
  rc = set_push_peers(args, peer_copies, num_peers, P, "nt_adamw_mt_push");
  if (rc) return rc;
  return dispatch_mt(P, *args, as_stream(stream));
}

int nt_adamw_mt_push_exchange(const nt_adamw_mt_args* args, void* const* peer_copies, int32_t num_peers,
                              const nt_zero_sync* sync, void* stream) {
  nt::TraceRange trace("nt_adamw_mt_push_exchange");
  const char* what = "nt_adamw_mt_push_exchange";
  MtParams P;
  int rc = build_mt_params(args, P);
  if (rc != NT_OK) return rc;
  if (num_peers < 0 || num_peers > NT_MAX_RANKS - 1) {
    set_error("%s: num_peers must be in [0, %d] (got %d)", what, NT_MAX_RANKS - 1, num_peers);
    return NT_EINVAL;
  }
  PeerSync S;
  rc = build_peer_sync(sync, num_peers + 1, S, what);
  if (rc) return rc;
  if (P.nchunks == 0) {   // nothing to update on this rank: the closing exchange only
    zero_done_kernel<<<1, 32, 0, as_stream(stream)>>>(S);
    return launch_status("nt_adamw_mt_push_exchange launch");
  }
  rc = set_push_peers(args, peer_copies, num_peers, P, what);
  if (rc) return rc;
  P.sync = S;
  return dispatch_mt_sync(P, *args, as_stream(stream));
}

}  // extern "C"
