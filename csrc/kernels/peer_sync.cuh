// Flag protocol helpers for kernels that synchronise with other CTAs or other GPUs
// through memory (release/acquire at GPU or system scope), with bounded waits.
#pragma once

#include <cstdint>

#include "tc_common.cuh"

namespace axr {

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(int* p, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// bounded wait until *p >= target
template <bool SYS>
__device__ __forceinline__ bool wait_geq(const int* p, int target, volatile int* err, int code) {
  const unsigned long long t0 = tc::globaltimer();
  while ((SYS ? ld_acquire_sys(p) : ld_acquire_gpu(p)) < target) {
    if (*err != 0) return false;
    if (tc::globaltimer() - t0 > tc::kWaitLimitNs) {
      atomicCAS(const_cast<int*>(err), 0, code);
      return false;
    }
  }
  return true;
}

}  // namespace axr
