// Cross-GPU and cross-CTA synchronization words: acquire/release loads and
// stores at GPU and system scope, and a bounded wait on a monotonic counter.
// Counters only grow (epochs, cumulative row counts), so no word is ever
// reset between steps and a comparison is wrap-safe.
#pragma once
#include "common.cuh"

namespace qb {

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
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// spin until *p >= want (wrap-safe), with a clock budget
template <bool SYS>
__device__ __forceinline__ bool wait_word(const uint32_t* p, uint32_t want, int* err) {
  const long long t0 = clock64();
  const long long budget = wait_budget(err);
  while (true) {
    const uint32_t v = SYS ? ld_acquire_sys(p) : ld_acquire_gpu(p);
    if ((int32_t)(v - want) >= 0) return true;
    if (clock64() - t0 > budget) {
      atomicCAS(err, 0, kErrTimeoutPeer);
      return false;
    }
  }
}

}  // namespace qb
