// System-scope flag primitives shared by the peer-memory collectives (comm.cu, nvls.cu).
#pragma once
#include "ptx.cuh"

namespace rf {

constexpr uint64_t kCommWaitNs = 10000000000ull;   // 10 s

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spin (bounded by limit_ns of wall time, kCommWaitNs by default) until *flag == value; records kErrTimeoutPeer
// and returns false on expiry.
__device__ __forceinline__ bool wait_value(const int* flag, int value, int* err, uint64_t limit_ns = kCommWaitNs) {
  if (ld_acquire_sys(flag) == value) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (ld_acquire_sys(flag) == value) return true;
    if ((++spins & 63u) == 0u) {
      if (global_timer_ns() - t0 > limit_ns) {
        record_error(err, kErrTimeoutPeer);
        return false;
      }
      __nanosleep(200);
    }
  }
}

}  // namespace rf
