// ep_sync.cuh - step flags between the ranks of an expert-parallel group (peer memory).
//
// Each rank owns two flag arrays in its exchange region, in_flag[world] and done_flag[world];
// rank p writes the number of the step it reached into slot p of every rank's arrays. Flags
// only grow (step numbers, compared wrap-safe), so a rank that is one step ahead never
// confuses a waiter. A signal is a system-scope release after a system fence; a wait is a
// system-scope acquire poll with a time bound, after which the caller records
// kStatusTimeout and skips the work that needed the data (the launch always completes).
#pragma once

#include "moe_kernels.cuh"

namespace ftb {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread: every write this rank made before (earlier launches on the stream included)
// becomes visible to a rank that observes `epoch` in its slot.
__device__ inline void ep_signal(uint32_t* const* sig, int world, uint32_t epoch) {
  __threadfence_system();
  for (int p = 0; p < world; ++p) st_release_sys(sig[p], epoch);
}

// One thread: wait until *flag has reached `epoch`. Gives up after wait_ns nanoseconds of
// global time (or 2^26 polls, whichever comes first) and returns false.
__device__ inline bool ep_wait(const uint32_t* flag, uint32_t epoch, int64_t wait_ns) {
  if ((int32_t)(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0; it < (1u << 26); ++it) {
    __nanosleep(128);
    if ((int32_t)(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if ((int64_t)(globaltimer_ns() - t0) > wait_ns) return false;
  }
  return false;
}

}  // namespace ftb
