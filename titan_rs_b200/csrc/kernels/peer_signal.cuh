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

}  // namespace tb
