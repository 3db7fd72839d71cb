// Flag words shared between GPUs of one node (symmetric memory over NVLink): system-scope
// release stores, acquire loads and a bounded wait that records kErrWaitTimeout in the
// device error word and returns false instead of spinning forever.
#pragma once

#include "common.cuh"

namespace nsw {
namespace peer {

constexpr unsigned long long kWaitNs = 4000000000ull;  // 4 s

__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// wait until *p >= v (wrap-safe comparison of epoch counters); false on timeout
static __device__ __noinline__ bool wait_geq(const uint32_t* p, uint32_t v, int* err) {
  if ((int)(ld_acquire(p) - v) >= 0) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t spin = 0;; ++spin) {
    if ((int)(ld_acquire(p) - v) >= 0) return true;
    if ((spin & 63u) == 63u) {
      __nanosleep(200);
      if (now_ns() - t0 > kWaitNs) {
        record_error(err, kErrWaitTimeout);
        return false;
      }
    }
  }
}

}  // namespace peer
}  // namespace nsw
