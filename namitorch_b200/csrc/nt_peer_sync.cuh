// Cross-GPU flags of the ZeRO-1 kernels: epochs written into other ranks' mailboxes with
// system-scope release stores, and bounded waits with system-scope acquire loads on this
// rank's own mailbox (nt_zero_mailbox, include/namitorch_b200.h). A wait that runs past its
// bound returns false; the caller records the failure in the sync error word and carries on,
// so no kernel ever waits without limit on another GPU.
#pragma once

#include "nt_common.cuh"

namespace nt {

struct PeerSync {
  nt_zero_mailbox* box[NT_MAX_RANKS];
  int nranks;
  int rank;
  uint64_t epoch;
  uint64_t timeout_ns;
  int32_t* error;
};

// Checks an nt_zero_sync for `nranks` ranks and copies it into `S` (host side, nt_zero.cu).
int build_peer_sync(const nt_zero_sync* sync, int nranks, PeerSync& S, const char* what);

__device__ __forceinline__ uint64_t peer_clock_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t load_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// This rank's `flag` becomes the epoch in every rank's mailbox (its own included). The release
// orders every earlier memory operation of the calling thread before it, at system scope.
__device__ __forceinline__ void signal_all(const PeerSync& S, int flag) {
  for (int q = 0; q < S.nranks; ++q) store_release_sys(&S.box[q]->flags[flag][S.rank], S.epoch);
}

// Waits until every rank has signalled `flag` for this epoch in this rank's mailbox; false if
// the bound ran out first.
__device__ __forceinline__ bool wait_all(const PeerSync& S, int flag) {
  const nt_zero_mailbox* own = S.box[S.rank];
  const uint64_t t0 = peer_clock_ns();
  for (int q = 0; q < S.nranks; ++q) {
    while (load_acquire_sys(&own->flags[flag][q]) < S.epoch) {
      if (peer_clock_ns() - t0 > S.timeout_ns) return false;
      __nanosleep(256);
    }
  }
  return true;
}

// last_block_ticket at system scope: every block's earlier stores, to this GPU and to peers,
// are visible system-wide before the last block goes on.
__device__ __forceinline__ bool last_block_ticket_sys(unsigned* counter, bool* smem_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned ticket = atomicAdd(counter, 1u);
    *smem_flag = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  const bool last = *smem_flag;
  if (last) __threadfence_system();
  return last;
}

}  // namespace nt
