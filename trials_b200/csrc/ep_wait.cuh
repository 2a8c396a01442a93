// System-scope flag stores and bounded flag waits of the peer exchange
// (shared by the exchange kernels and the routing kernel that starts the
// expert-parallel layer).
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace b200moe {

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Threads 0..G-1 wait until flags[thread] >= epoch, then the whole CTA passes
// a barrier: everything the G writers stored before raising their flags is
// visible to the CTA (and to later kernels of the stream) afterwards. Once a
// wait has expired (timeout bit in err), later waits give up after 1 ms, so a
// many-CTA launch whose peer is gone ends in about one limit, not one per wave.
__device__ __forceinline__ void wait_flags(const int32_t* flags, int G, int32_t epoch, int32_t* err,
                                           uint64_t limit_ns) {
  if ((int)threadIdx.x < G) {
    const int32_t* f = flags + threadIdx.x;
    if (ld_acquire_sys(f) < epoch) {
      const uint64_t t0 = globaltimer_ns();
      const uint64_t limit =
          (*reinterpret_cast<volatile int32_t*>(err) & ERR_DEV_TIMEOUT) ? 1000000ull : limit_ns;
      while (ld_acquire_sys(f) < epoch) {
        if (globaltimer_ns() - t0 > limit) {
          atomicOr(err, ERR_DEV_TIMEOUT);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
}

}  // namespace b200moe
