// ZeRO-1 over peer memory: CUDA IPC of the flat buffers and the reduce-scatter fused with
// the first statistics pass.
//
// Each rank owns one contiguous shard of the flat gradient buffer. The reduce-scatter is a
// pull: the owner reads the same shard range from every rank's buffer (its own from HBM,
// the others' over NVLink through IPC mappings), sums the contributions in f32 in rank
// order, rounds once to the gradient dtype and writes its reduced shard. The statistics of
// that shard (sum of squares, non-finite and NaN counts, max |g|, all of g / scale) are
// accumulated from the values just written, so found_inf and the norm cost no extra pass.
// The sum order is fixed, so the result does not depend on the transport's chunking.
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "nt_peer_sync.cuh"
#include "nt_stats.cuh"

namespace nt {

struct ZeroReduceParams {
  const void* src[NT_MAX_RANKS];
  int nranks;
  int64_t count;
  int average;
  float inv_n;      // 1/num_ranks when that is exact (power of two), else 0: divide instead
  float n_f;
  void* dst;
  const float* scale;
  nt_stats* stats;
  StatsWorkspace* ws;
  PeerSync sync;      // used by the exchange variant only
  double norm_type;   // exchange variant: 2 or inf
  int vec32;          // every source and the destination are 32-byte aligned
};

constexpr int kZeroThreads = kStatsThreads;

template <int DT>
__device__ __forceinline__ uint4 pack_vec(const float* x) {
  uint4 raw;
  if constexpr (DT == NT_F32) {
    raw.x = __float_as_uint(x[0]); raw.y = __float_as_uint(x[1]);
    raw.z = __float_as_uint(x[2]); raw.w = __float_as_uint(x[3]);
  } else {
    using T = typename Elem<DT>::T;
    T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] = Elem<DT>::from_f32(x[k]);
  }
  return raw;
}

__device__ __forceinline__ float average(float sum, const ZeroReduceParams& P) {
  if (P.average) sum = P.inv_n != 0.0f ? __fmul_rn(sum, P.inv_n) : __fdiv_rn(sum, P.n_f);
  return sum;
}

// NR > 0: the rank count is a compile-time constant (2, 4, 8); NR == 0: any count up to
// NT_MAX_RANKS, one vector per source in flight. H = 2: each access moves 32 bytes (every
// source and the destination 32-byte aligned); H = 1: 16 bytes. The statistics see exactly
// the values stored in the shard (rounded to the gradient dtype, then unscaled).
template <int DT, int NR, int MODE, int H>
__device__ __forceinline__ void zero_reduce_body(const ZeroReduceParams& P, const Unscale& un, StatsAcc& a) {
  constexpr int ES = DT == NT_F32 ? 4 : 2;
  constexpr int EPV = 16 / ES;                 // elements per 16-byte half
  constexpr int R = NR > 0 ? NR : NT_MAX_RANKS;
  constexpr int U = NR > 0 && NR * H < 8 ? 8 / (NR * H) : 1;   // accesses in flight per source
  const int nr = NR > 0 ? NR : P.nranks;
  const int64_t nv = P.count / (EPV * H);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * U;
  char* dst = static_cast<char*>(P.dst);

  for (int64_t v0 = (int64_t)blockIdx.x * blockDim.x * U + threadIdx.x; v0 < nv; v0 += stride) {
    uint4 raw[U][R][H];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
#pragma unroll
      for (int q = 0; q < R; ++q) {
        if (v < nv && q < nr) {
          const char* src = static_cast<const char*>(P.src[q]) + v * (16 * H);
          if constexpr (H == 2) load32_cs(src, raw[u][q][0], raw[u][q][1]);
          else raw[u][q][0] = __ldcs(reinterpret_cast<const uint4*>(src));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      if (v >= nv) continue;
      uint4 out[H];
#pragma unroll
      for (int h = 0; h < H; ++h) {
        float sum[EPV], x[EPV];
        unpack16<DT>(raw[u][0][h], sum);
#pragma unroll
        for (int q = 1; q < R; ++q) {
          if (q < nr) {
            unpack16<DT>(raw[u][q][h], x);
#pragma unroll
            for (int k = 0; k < EPV; ++k) sum[k] = __fadd_rn(sum[k], x[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < EPV; ++k) sum[k] = average(sum[k], P);
        out[h] = pack_vec<DT>(sum);
        unpack16<DT>(out[h], x);
#pragma unroll
        for (int k = 0; k < EPV; ++k) x[k] = unscale_by<MODE>(x[k], un.scale, un.inv);
        stats_pass0<EPV>(x, a);
      }
      if constexpr (H == 2) store32_cs(dst + v * 32, out[0], out[1]);
      else __stcs(reinterpret_cast<uint4*>(dst) + v, out[0]);
    }
  }
  // Elements past the last full vector (count not a multiple of the vector width).
  for (int64_t i = nv * EPV * H + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < P.count;
       i += (int64_t)gridDim.x * blockDim.x) {
    float sum = load1<DT>(P.src[0], i);
    for (int q = 1; q < nr; ++q) sum = __fadd_rn(sum, load1<DT>(P.src[q], i));
    store1<DT>(P.dst, i, average(sum, P));
    stats_one(unscale_by<MODE>(load1<DT>(P.dst, i), un.scale, un.inv), a);
  }
}

template <int DT, int NR, int MODE>
__device__ __forceinline__ void zero_reduce_width(const ZeroReduceParams& P, const Unscale& un, StatsAcc& a) {
  if (P.vec32) zero_reduce_body<DT, NR, MODE, 2>(P, un, a);
  else zero_reduce_body<DT, NR, MODE, 1>(P, un, a);
}

// One thread: sends this rank's shard totals {sum of squares, non-finite count, NaN count,
// max |g|} to every rank's mailbox, signals STATS, waits for every rank's (bounded), adds the
// N totals in rank order (the same doubles in the same order on every rank, so every rank
// finalizes the same found_inf and norm) and finalizes into `st`. With `ok` false (an
// earlier wait of this step ran out), or when this wait runs out, the record reports
// found_inf with a NaN norm, so the update skips, and bit 0 of the error word is set.
__device__ __forceinline__ void exchange_shard_totals(const PeerSync& S, bool ok, double ss, double nfd, double nnd,
                                                      double mx, double norm_type, nt_stats* st) {
  if (ok) {
    for (int q = 0; q < S.nranks; ++q) {
      double* slot = S.box[q]->stats[S.rank];
      slot[0] = ss; slot[1] = nfd; slot[2] = nnd; slot[3] = mx;
    }
    signal_all(S, NT_ZERO_STATS);   // the release orders the four stores above before it
    ok = wait_all(S, NT_ZERO_STATS);
  }
  if (ok) {
    const volatile nt_zero_mailbox* own = S.box[S.rank];
    double gs = 0.0, gnf = 0.0, gnn = 0.0, gmx = 0.0;
    for (int q = 0; q < S.nranks; ++q) {
      gs += own->stats[q][0]; gnf += own->stats[q][1]; gnn += own->stats[q][2];
      gmx = fmax(gmx, own->stats[q][3]);
    }
    st->sumsq = gs; st->nonfinite = gnf; st->nan = gnn; st->maxabs = gmx;
    stats_finalize(st, norm_type);
  } else {
    atomicOr(S.error, 1);
    const double nan = __longlong_as_double(0x7ff8000000000000ll);
    st->sumsq = nan; st->nonfinite = 1.0; st->nan = 1.0; st->maxabs = nan; st->norm = nan; st->found_inf = 1.0;
  }
}

// The exchange variant's end: the block partials are reduced in a fixed order by the last
// block, which sends the shard's totals to every rank's mailbox, waits for every rank's,
// adds them in rank order (the same doubles in the same order on every rank, so every rank
// finalizes the same found_inf and norm) and finalizes. If any wait ran out (READY in some
// block, STATS here), the record reports found_inf with a NaN norm, so the update skips.
__device__ __forceinline__ void zero_exchange_stats(const StatsAcc& a, const ZeroReduceParams& P) {
  __shared__ double red_d[kZeroThreads / 32];
  __shared__ float red_f[kZeroThreads / 32];
  __shared__ unsigned red_u[kZeroThreads / 32];
  __shared__ bool last;
  double ss = block_reduce(a.ss0 + a.ss1, red_d, SumOp(), 0.0);
  float mx = block_reduce(a.mx, red_f, MaxOp(), 0.0f);
  unsigned nf = block_reduce(a.nf, red_u, SumOp(), 0u);
  unsigned nn = block_reduce(a.nn, red_u, SumOp(), 0u);
  if (threadIdx.x == 0) {
    StatsPartial& out = P.ws->partials[blockIdx.x];
    out.sumsq = ss; out.powsum = 0.0; out.maxabs = mx; out.nonfinite = nf; out.nan = nn;
  }
  if (!last_block_ticket(&P.ws->counter, &last)) return;
  ss = 0.0; mx = 0.0f;
  double nfd = 0.0, nnd = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    const StatsPartial q = P.ws->partials[b];
    ss += q.sumsq; mx = fmaxf(mx, q.maxabs); nfd += q.nonfinite; nnd += q.nan;
  }
  ss = block_reduce(ss, red_d, SumOp(), 0.0);
  nfd = block_reduce(nfd, red_d, SumOp(), 0.0);
  nnd = block_reduce(nnd, red_d, SumOp(), 0.0);
  mx = block_reduce(mx, red_f, MaxOp(), 0.0f);
  if (threadIdx.x != 0) return;
  const bool ready = *reinterpret_cast<volatile unsigned*>(&P.ws->pad[0]) == 0u;   // every block saw every rank READY
  exchange_shard_totals(P.sync, ready, ss, nfd, nnd, (double)mx, P.norm_type, P.stats);
  P.ws->pad[0] = 0u;
  P.ws->counter = 0u;
}

template <int DT, int NR, bool SYNC>
__global__ void __launch_bounds__(kZeroThreads, 2) zero_reduce_stats_kernel(const __grid_constant__ ZeroReduceParams P) {
  bool run = true;
  if constexpr (SYNC) {
    // Any block may run first, so every block signals READY (the same epoch) and waits for
    // every rank's before it pulls. This rank's gradients were written by earlier kernels of
    // its stream, so they are final when any block of this kernel runs.
    __shared__ bool ready;
    if (threadIdx.x == 0) {
      signal_all(P.sync, NT_ZERO_READY);
      ready = wait_all(P.sync, NT_ZERO_READY);
      if (!ready) atomicOr(&P.ws->pad[0], 1u);
    }
    __syncthreads();
    run = ready;
  }
  Unscale un;
  un.init(P.scale);
  StatsAcc a{0.0, 0.0, 0.0, 0.0f, 0u, 0u};
  if (run) {
    if (!un.active) zero_reduce_width<DT, NR, kScaleNone>(P, un, a);
    else if (un.pow2) zero_reduce_width<DT, NR, kScaleMul>(P, un, a);
    else zero_reduce_width<DT, NR, kScaleDiv>(P, un, a);
  }
  if constexpr (SYNC) zero_exchange_stats(a, P);
  else stats_reduce_pass0(a, P.ws, P.stats);
}

// One thread: this rank's `flag` for the epoch into every rank's mailbox, then a bounded
// wait for every rank's. `status` (if given) records 0 (every rank arrived) or 1 (the wait
// ran out, which also sets `error_bit` in the sticky error word).
__global__ void zero_flag_kernel(const PeerSync S, int flag, uint32_t* status, int error_bit) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  signal_all(S, flag);
  const bool ok = wait_all(S, flag);
  if (status) *status = ok ? 0u : 1u;
  if (!ok) atomicOr(S.error, error_bit);
}

// One thread: adds `count` shard statistics records in order (the pieces of this rank's
// shard, reduced one launch each) and runs the statistics exchange on their totals.
__global__ void zero_records_exchange_kernel(const nt_stats* records, int count, const PeerSync S,
                                             const uint32_t* ready_status, double norm_type, nt_stats* out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double ss = 0.0, nfd = 0.0, nnd = 0.0, mx = 0.0;
  for (int k = 0; k < count; ++k) {
    ss += records[k].sumsq; nfd += records[k].nonfinite; nnd += records[k].nan;
    mx = fmax(mx, records[k].maxabs);
  }
  const bool ready = ready_status == nullptr || *reinterpret_cast<const volatile uint32_t*>(ready_status) == 0u;
  exchange_shard_totals(S, ready, ss, nfd, nnd, mx, norm_type, out);
}

template <int DT, int NR, bool SYNC>
static int launch_zero_reduce(const ZeroReduceParams& P, cudaStream_t s) {
  int grid = current_sm_count() * 2;   // two 256-thread blocks per SM, 8 vectors in flight per thread
  if (grid > kStatsMaxBlocks) grid = kStatsMaxBlocks;
  const int64_t epv = DT == NT_F32 ? 4 : 8;
  const int64_t want = (P.count / epv + kZeroThreads - 1) / kZeroThreads;
  if (want < grid) grid = want > 0 ? (int)want : 1;
  zero_reduce_stats_kernel<DT, NR, SYNC><<<grid, kZeroThreads, 0, s>>>(P);
  return launch_status("nt_zero_reduce_scatter_stats launch");
}

template <int DT, bool SYNC>
static int dispatch_ranks(const ZeroReduceParams& P, cudaStream_t s) {
  switch (P.nranks) {
    case 2: return launch_zero_reduce<DT, 2, SYNC>(P, s);
    case 4: return launch_zero_reduce<DT, 4, SYNC>(P, s);
    case 8: return launch_zero_reduce<DT, 8, SYNC>(P, s);
    default: return launch_zero_reduce<DT, 0, SYNC>(P, s);
  }
}

template <bool SYNC>
static int dispatch_dtype(const ZeroReduceParams& P, int dtype, cudaStream_t s, const char* what) {
  switch (dtype) {
    case NT_F32: return dispatch_ranks<NT_F32, SYNC>(P, s);
    case NT_F16: return dispatch_ranks<NT_F16, SYNC>(P, s);
    case NT_BF16: return dispatch_ranks<NT_BF16, SYNC>(P, s);
    default:
      set_error("%s: unsupported dtype %d", what, dtype);
      return NT_EUNSUPPORTED;
  }
}

// Checks an nt_zero_sync and copies it into the kernel's parameters.
int build_peer_sync(const nt_zero_sync* sync, int nranks, PeerSync& S, const char* what) {
  if (!sync) { set_error("%s: sync is NULL", what); return NT_EINVAL; }
  if (sync->rank < 0 || sync->rank >= nranks) {
    set_error("%s: rank %d outside [0, %d)", what, sync->rank, nranks);
    return NT_EINVAL;
  }
  if (sync->epoch == 0 || sync->timeout_ns == 0 || !sync->error) {
    set_error("%s: epoch and timeout_ns must be positive and error non-NULL", what);
    return NT_EINVAL;
  }
  for (int q = 0; q < NT_MAX_RANKS; ++q) {
    if (q < nranks && (!sync->mailboxes[q] || (reinterpret_cast<uintptr_t>(sync->mailboxes[q]) & 7u))) {
      set_error("%s: mailbox %d is NULL or not 8-byte aligned", what, q);
      return NT_EINVAL;
    }
    S.box[q] = q < nranks ? sync->mailboxes[q] : nullptr;
  }
  S.nranks = nranks;
  S.rank = sync->rank;
  S.epoch = sync->epoch;
  S.timeout_ns = sync->timeout_ns;
  S.error = sync->error;
  return NT_OK;
}


// Copies count independent ranges (src[k] -> dst[k], `vectors` 16-byte vectors each) with
// plain SM loads and stores, the access pattern of the ZeRO-1 pull and push: pointing src
// at peers measures the inbound link, dst at peers the outbound one. H = 2: 32-byte
// accesses (every pointer 32-byte aligned and an even vector count, as the reduce-scatter
// takes them); H = 1: 16-byte.
struct PeerCopyParams {
  const char* src[NT_MAX_RANKS];
  char* dst[NT_MAX_RANKS];
  int count;
  int64_t vectors;
};

constexpr int kPeerCopyThreads = 256;
constexpr int kPeerCopyUnroll = 4;

template <int H>
__global__ void __launch_bounds__(kPeerCopyThreads) peer_copy_kernel(const __grid_constant__ PeerCopyParams P) {
  const int k = blockIdx.x % P.count;              // the blocks are dealt round robin to the ranges
  const int64_t block = blockIdx.x / P.count;
  const int64_t blocks = gridDim.x / P.count;
  const char* src = P.src[k];
  char* dst = P.dst[k];
  const int64_t n = P.vectors / H;
  const int64_t step = blocks * kPeerCopyThreads * kPeerCopyUnroll;
  for (int64_t v0 = block * kPeerCopyThreads * kPeerCopyUnroll + threadIdx.x; v0 < n; v0 += step) {
    uint4 r[kPeerCopyUnroll][H];
#pragma unroll
    for (int u = 0; u < kPeerCopyUnroll; ++u) {
      const int64_t v = v0 + (int64_t)u * kPeerCopyThreads;
      if (v < n) {
        if constexpr (H == 2) load32_cs(src + v * 32, r[u][0], r[u][1]);
        else r[u][0] = __ldcs(reinterpret_cast<const uint4*>(src) + v);
      }
    }
#pragma unroll
    for (int u = 0; u < kPeerCopyUnroll; ++u) {
      const int64_t v = v0 + (int64_t)u * kPeerCopyThreads;
      if (v < n) {
        if constexpr (H == 2) store32_cs(dst + v * 32, r[u][0], r[u][1]);
        else __stcs(reinterpret_cast<uint4*>(dst) + v, r[u][0]);
      }
    }
  }
}

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  }
  return fn;
}

// Pointer handed out by nt_ipc_open -> the mapping's base, which cudaIpcCloseMemHandle wants.
static std::mutex g_ipc_lock;
static std::unordered_map<void*, void*> g_ipc_bases;

static int build_zero_reduce(const nt_zero_reduce_args* args, ZeroReduceParams& P, const char* what) {
  if (!args) { set_error("%s: args is NULL", what); return NT_EINVAL; }
  const nt_zero_reduce_args& a = *args;
  if (a.num_ranks < 1 || a.num_ranks > NT_MAX_RANKS) {
    set_error("%s: num_ranks must be in [1, %d] (got %d)", what, NT_MAX_RANKS, a.num_ranks);
    return NT_EINVAL;
  }
  if (a.count < 0) { set_error("%s: negative count", what); return NT_EINVAL; }
  if (!a.stats || !a.workspace || (a.count > 0 && !a.dest)) {
    set_error("%s: NULL dest/stats/workspace", what);
    return NT_EINVAL;
  }
  if (a.workspace_bytes < sizeof(StatsWorkspace)) {
    set_error("%s: workspace needs %zu bytes (got %zu)", what, sizeof(StatsWorkspace), a.workspace_bytes);
    return NT_EINVAL;
  }
  if (!aligned16(a.dest)) { set_error("%s: dest must be 16-byte aligned", what); return NT_EINVAL; }
  for (int q = 0; q < a.num_ranks && a.count > 0; ++q) {   // an empty shard reads nothing
    if (!a.sources[q] || !aligned16(a.sources[q])) {
      set_error("%s: source %d is NULL or not 16-byte aligned", what, q);
      return NT_EINVAL;
    }
  }
  for (int q = 0; q < NT_MAX_RANKS; ++q) P.src[q] = q < a.num_ranks ? a.sources[q] : a.sources[0];
  P.nranks = a.num_ranks;
  P.count = a.count;
  P.average = a.average != 0;
  P.n_f = (float)a.num_ranks;
  P.inv_n = (a.num_ranks & (a.num_ranks - 1)) == 0 ? 1.0f / (float)a.num_ranks : 0.0f;
  P.dst = a.dest;
  P.scale = a.scale;
  P.stats = a.stats;
  P.ws = static_cast<StatsWorkspace*>(a.workspace);
  P.norm_type = 2.0;
  memset(&P.sync, 0, sizeof(P.sync));
  bool a32 = (reinterpret_cast<uintptr_t>(a.dest) & 31u) == 0;
  for (int q = 0; q < a.num_ranks && a.count > 0; ++q) a32 = a32 && (reinterpret_cast<uintptr_t>(a.sources[q]) & 31u) == 0;
  P.vec32 = a32 ? 1 : 0;
  return NT_OK;
}

}  // namespace nt

using namespace nt;

extern "C" {

int nt_ipc_export(const void* ptr, unsigned char handle[64], uint64_t* offset) {
  if (!ptr || !handle || !offset) { set_error("nt_ipc_export: NULL argument"); return NT_EINVAL; }
  GetAddressRangeFn range = address_range_fn();
  if (!range) { set_error("nt_ipc_export: cuMemGetAddressRange is unavailable"); return NT_ECUDA; }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("nt_ipc_export: %p is not device memory of this process", ptr);
    return NT_EINVAL;
  }
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return cuda_fail(err, "nt_ipc_export (cudaIpcGetMemHandle)");
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  memcpy(handle, &h, 64);
  *offset = reinterpret_cast<uint64_t>(ptr) - static_cast<uint64_t>(base);
  return NT_OK;
}

int nt_ipc_open(const unsigned char handle[64], uint64_t offset, void** ptr) {
  if (!handle || !ptr) { set_error("nt_ipc_open: NULL argument"); return NT_EINVAL; }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, 64);
  void* base = nullptr;
  cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_fail(err, "nt_ipc_open (cudaIpcOpenMemHandle)");
  *ptr = static_cast<char*>(base) + offset;
  std::lock_guard<std::mutex> lock(g_ipc_lock);
  g_ipc_bases[*ptr] = base;
  return NT_OK;
}

int nt_ipc_close(void* ptr) {
  if (!ptr) return NT_OK;
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_ipc_lock);
    auto it = g_ipc_bases.find(ptr);
    if (it == g_ipc_bases.end()) {
      set_error("nt_ipc_close: %p was not returned by nt_ipc_open", ptr);
      return NT_EINVAL;
    }
    base = it->second;
    g_ipc_bases.erase(it);
  }
  cudaError_t err = cudaIpcCloseMemHandle(base);
  if (err != cudaSuccess) return cuda_fail(err, "nt_ipc_close (cudaIpcCloseMemHandle)");
  return NT_OK;
}

int nt_can_access_peer(int32_t peer, int32_t* ok) {
  if (!ok) { set_error("nt_can_access_peer: NULL argument"); return NT_EINVAL; }
  int dev = 0, can = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "nt_can_access_peer (cudaGetDevice)");
  if (peer == dev) { *ok = 1; return NT_OK; }
  err = cudaDeviceCanAccessPeer(&can, dev, peer);
  if (err != cudaSuccess) return cuda_fail(err, "nt_can_access_peer");
  *ok = can ? 1 : 0;
  return NT_OK;
}

int nt_zero_reduce_scatter_stats(const nt_zero_reduce_args* args, void* stream) {
  nt::TraceRange trace("nt_zero_reduce_scatter_stats");
  ZeroReduceParams P;
  int rc = build_zero_reduce(args, P, "nt_zero_reduce_scatter_stats");
  if (rc) return rc;
  return dispatch_dtype<false>(P, args->dtype, as_stream(stream), "nt_zero_reduce_scatter_stats");
}

int nt_zero_reduce_scatter_exchange(const nt_zero_reduce_args* args, const nt_zero_sync* sync, double norm_type,
                                    void* stream) {
  nt::TraceRange trace("nt_zero_reduce_scatter_exchange");
  const char* what = "nt_zero_reduce_scatter_exchange";
  ZeroReduceParams P;
  int rc = build_zero_reduce(args, P, what);
  if (rc) return rc;
  if (!(norm_type == 2.0 || isinf(norm_type))) {
    set_error("%s: norm_type must be 2 or inf (another norm needs a second pass)", what);
    return NT_EINVAL;
  }
  rc = build_peer_sync(sync, args->num_ranks, P.sync, what);
  if (rc) return rc;
  P.norm_type = norm_type;
  return dispatch_dtype<true>(P, args->dtype, as_stream(stream), what);
}

int nt_zero_flag_exchange(const nt_zero_sync* sync, int32_t num_ranks, int32_t flag, uint32_t* status, void* stream) {
  nt::TraceRange trace("nt_zero_flag_exchange");
  const char* what = "nt_zero_flag_exchange";
  if (num_ranks < 1 || num_ranks > NT_MAX_RANKS) {
    set_error("%s: num_ranks must be in [1, %d] (got %d)", what, NT_MAX_RANKS, num_ranks);
    return NT_EINVAL;
  }
  if (flag < NT_ZERO_READY || flag > NT_ZERO_DONE) {
    set_error("%s: flag must be NT_ZERO_READY, NT_ZERO_STATS or NT_ZERO_DONE (got %d)", what, flag);
    return NT_EINVAL;
  }
  PeerSync S;
  int rc = build_peer_sync(sync, num_ranks, S, what);
  if (rc) return rc;
  zero_flag_kernel<<<1, 32, 0, as_stream(stream)>>>(S, flag, status, flag == NT_ZERO_DONE ? 2 : 1);
  return launch_status("nt_zero_flag_exchange launch");
}

int nt_zero_stats_exchange(const nt_stats* records, int32_t count, const nt_zero_sync* sync, int32_t num_ranks,
                           const uint32_t* ready_status, double norm_type, nt_stats* out, void* stream) {
  nt::TraceRange trace("nt_zero_stats_exchange");
  const char* what = "nt_zero_stats_exchange";
  if (num_ranks < 1 || num_ranks > NT_MAX_RANKS) {
    set_error("%s: num_ranks must be in [1, %d] (got %d)", what, NT_MAX_RANKS, num_ranks);
    return NT_EINVAL;
  }
  if (count < 1 || !records || !out) {
    set_error("%s: needs at least one record and an output record", what);
    return NT_EINVAL;
  }
  if (!(norm_type == 2.0 || isinf(norm_type))) {
    set_error("%s: norm_type must be 2 or inf (another norm needs a second pass)", what);
    return NT_EINVAL;
  }
  PeerSync S;
  int rc = build_peer_sync(sync, num_ranks, S, what);
  if (rc) return rc;
  zero_records_exchange_kernel<<<1, 32, 0, as_stream(stream)>>>(records, count, S, ready_status, norm_type, out);
  return launch_status("nt_zero_stats_exchange launch");
}

int nt_peer_copy(const void* const* src, void* const* dst, int32_t count, uint64_t bytes_each, void* stream) {
  nt::TraceRange trace("nt_peer_copy");
  if (count < 1 || count > NT_MAX_RANKS) {
    set_error("nt_peer_copy: count must be in [1, %d] (got %d)", NT_MAX_RANKS, count);
    return NT_EINVAL;
  }
  if (!src || !dst) { set_error("nt_peer_copy: NULL pointer array"); return NT_EINVAL; }
  if (bytes_each % 16 != 0) { set_error("nt_peer_copy: bytes_each must be a multiple of 16"); return NT_EINVAL; }
  PeerCopyParams P;
  for (int k = 0; k < NT_MAX_RANKS; ++k) { P.src[k] = nullptr; P.dst[k] = nullptr; }
  for (int k = 0; k < count; ++k) {
    if (bytes_each > 0 && (!src[k] || !dst[k] || !aligned16(src[k]) || !aligned16(dst[k]))) {
      set_error("nt_peer_copy: range %d has a NULL or not 16-byte aligned pointer", k);
      return NT_EINVAL;
    }
    P.src[k] = static_cast<const char*>(src[k]);
    P.dst[k] = static_cast<char*>(dst[k]);
  }
  P.count = count;
  P.vectors = (int64_t)(bytes_each / 16);
  if (P.vectors == 0) return NT_OK;
  bool wide = bytes_each % 32 == 0;
  for (int k = 0; k < count; ++k)
    wide = wide && ((reinterpret_cast<uintptr_t>(src[k]) | reinterpret_cast<uintptr_t>(dst[k])) & 31u) == 0;
  const int H = wide ? 2 : 1;
  int per = current_sm_count() * 4 / count;   // four 256-thread blocks per SM in all
  if (per < 1) per = 1;
  const int64_t want = (P.vectors / H + kPeerCopyThreads * kPeerCopyUnroll - 1) / (kPeerCopyThreads * kPeerCopyUnroll);
  if (want < per) per = (int)want;
  if (wide) peer_copy_kernel<2><<<per * count, kPeerCopyThreads, 0, as_stream(stream)>>>(P);
  else peer_copy_kernel<1><<<per * count, kPeerCopyThreads, 0, as_stream(stream)>>>(P);
  return launch_status("nt_peer_copy launch");
}

}  // extern "C"
