// Flag exchange between the GPUs of one node through peer-mapped memory (CUDA IPC
// mappings of each rank's signal block in every other rank), for collective kernels
// whose ranks each run on their own GPU. Every wait is bounded by %globaltimer.
//
// A rank's signal block:
//   entry[r]   the call (epoch) rank r has started: everything rank r's stream did
//              before that call, including reads of its output buffer, is complete
//   exit[r]    the call whose stores into this rank's memory rank r has performed
//   arrivals   CTAs of this rank's current call that are done (the last one resets it)
// Epochs count the calls made with one registered buffer (the same on every rank)
// and are compared modulo 2^32.
#pragma once

#include "kernel_configs.h"
#include "sm100.cuh"

namespace tb {

struct SignalBlock {
  uint32_t entry[TB_MAX_RANKS];
  uint32_t exit[TB_MAX_RANKS];
  uint32_t arrivals;
  uint32_t pad[15];
};
static_assert(sizeof(SignalBlock) == TB_SIGNAL_BLOCK_BYTES, "signal block layout");

// Signal block of every rank, mapped in this process (index = rank).
struct RankSignals {
  SignalBlock* block[TB_MAX_RANKS];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Writes `epoch` into slot `self` of field `entry` (exit = false) or `exit` of every
// other rank's block.
__device__ __forceinline__ void signal_peers(const RankSignals& s, int ranks, int self, uint32_t epoch, bool exit) {
  for (int d = 0; d < ranks; ++d) {
    if (d == self) continue;
    SignalBlock* b = s.block[d];
    st_release_sys(exit ? &b->exit[self] : &b->entry[self], epoch);
  }
}

// Waits until every other rank's slot of this rank's `entry` / `exit` field has reached
// `epoch`; false after ~1 s.
__device__ __forceinline__ bool wait_peers(const RankSignals& s, int ranks, int self, uint32_t epoch, bool exit) {
  const SignalBlock* mine = s.block[self];
  const uint64_t start = global_timer_ns();
  for (int d = 0; d < ranks; ++d) {
    if (d == self) continue;
    const uint32_t* slot = exit ? &mine->exit[d] : &mine->entry[d];
    while (static_cast<int32_t>(ld_acquire_sys(slot) - epoch) < 0) {
      if (global_timer_ns() - start > kWaitLimitNs) return false;
    }
  }
  return true;
}

// Entry of call `epoch` of a fused kernel, for every CTA: CTA 0 announces the epoch in
// every peer's signal block; each CTA's thread 0 waits until every peer has announced
// it (so every peer is done with its previous output). Returns, to all threads of the
// CTA, whether the wait succeeded (a failure records `fail_code`). Contains a
// __syncthreads.
__device__ __forceinline__ bool call_entry(const RankSignals& sig, int ranks, int self, uint32_t epoch,
                                           uint32_t* status, uint32_t fail_code) {
  __shared__ int entered;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) signal_peers(sig, ranks, self, epoch, false);
    entered = wait_peers(sig, ranks, self, epoch, false) ? 1 : 0;
    if (!entered) report_status(status, fail_code);
  }
  __syncthreads();
  return entered != 0;
}

// Exit, called by every thread of every CTA after all of the CTA's threads have fenced
// their peer stores system-wide and met at a barrier: thread 0 counts the CTA in, and
// the last CTA of the grid tells every peer that this rank's stores have landed and
// waits until every peer has said the same (a failure records `fail_code`), so the
// kernel ends only when this rank's output is whole.
__device__ __forceinline__ void call_exit(const RankSignals& sig, int ranks, int self, uint32_t epoch, bool entered,
                                          uint32_t* status, uint32_t fail_code) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  SignalBlock* mine = sig.block[self];
  if (atomicAdd(&mine->arrivals, 1u) == gridDim.x - 1) {
    mine->arrivals = 0;  // the next call starts after this kernel (stream order)
    if (entered) {
      signal_peers(sig, ranks, self, epoch, true);
      if (!wait_peers(sig, ranks, self, epoch, true)) report_status(status, fail_code);
    }
  }
}

}  // namespace tb
