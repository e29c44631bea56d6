// Device helpers of the sequence-split exchange over peer memory (internal header).
#pragma once
#include <cstdint>

#include "lbq_kernels.h"
#include "lbq_ptx.cuh"

namespace lbq {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Heap base of rank p as mapped in this process.
__device__ __forceinline__ char* heap(const uint64_t* peers, int p) {
  return reinterpret_cast<char*>(static_cast<uintptr_t>(peers[p]));
}
// Waits until counter `flag` reaches `target` (modular u32 order); false after `timeout_ns`.
__device__ __forceinline__ bool wait_counter(const uint32_t* flag, uint32_t target, uint64_t timeout_ns) {
  if (int32_t(ld_acquire_sys(flag) - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < LBQ_SPIN_LIMIT; ++i) {
    __nanosleep(64);
    if (int32_t(ld_acquire_sys(flag) - target) >= 0) return true;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > timeout_ns) break;
  }
  return false;
}
// End of a push kernel: every CTA fences its (remote) stores at system scope and counts itself done
// in this rank's exchange area (`done_off`); the last CTA resets the count and raises every other
// rank's data counter for this rank by one (release, system scope). Causality through the count makes
// every CTA's stores visible to a receiver that observes the raised counter.
__device__ __forceinline__ void signal_after_last_cta(const uint64_t* peers, int nranks, int rank, int64_t xchg_off,
                                                      int64_t done_off) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence_system();
  uint32_t* done = reinterpret_cast<uint32_t*>(heap(peers, rank) + xchg_off + done_off);
  const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
  if (atomicAdd(done, 1u) != total - 1) return;
  *done = 0;
  __threadfence_system();
  for (int q = 1; q < nranks; ++q) {
    char* dst = heap(peers, (rank + q) % nranks) + xchg_off;
    red_release_sys_add(reinterpret_cast<uint32_t*>(dst + xchg::kFlagsData) + rank, 1u);
  }
}

}  // namespace lbq
