// Flag protocol helpers for kernels that synchronise with other CTAs or other GPUs
// through memory (release/acquire at GPU or system scope), with bounded waits.
#pragma once

#include <cstdint>
#include <cstdlib>

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

// Waits that depend on other GPUs' progress get a longer bound than waits inside one
// GPU: a peer may be late by a host-side stall (a capture mirrored to the CPU tier, a
// slow step) without anything being wrong. The launch passes the bound (default 30 s).
constexpr unsigned long long kPeerWaitLimitNs = 30000000000ull;

// bounded wait until *p >= target
template <bool SYS>
__device__ __forceinline__ bool wait_geq(const int* p, int target, volatile int* err, int code,
                                         unsigned long long limit = kPeerWaitLimitNs) {
  const unsigned long long t0 = tc::globaltimer();
  while ((SYS ? ld_acquire_sys(p) : ld_acquire_gpu(p)) < target) {
    if (*err != 0) return false;
    if (tc::globaltimer() - t0 > limit) {
      atomicCAS(const_cast<int*>(err), 0, code);
      return false;
    }
  }
  return true;
}

// Bound for peer-dependent waits, from AXR_PEER_WAIT_MS (host side).
inline unsigned long long peer_wait_ns() {
  static unsigned long long v = [] {
    const char* e = getenv("AXR_PEER_WAIT_MS");
    const long long ms = e ? atoll(e) : 30000;
    return static_cast<unsigned long long>(ms > 0 ? ms : 30000) * 1000000ull;
  }();
  return v;
}

}  // namespace axr
