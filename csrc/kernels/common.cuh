// Shared device helpers for the sm_100a kernels of axropus_deploy_b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <utility>

namespace axr {

// Storage formats of a KV page unit (one page of P tokens x D dims, one head).
enum PageFmt : int {
  kBF16 = 0,      // bf16 values
  kFP8Page = 1,   // e4m3 codes + one fp32 scale per page unit
  kFP8Token = 2,  // e4m3 codes + one fp32 scale per token row
  kINT4G64 = 3,   // packed nibbles + (scale, zero) fp16 per 64-value group of a row
};

constexpr int kPage = 16;    // tokens per KV page
constexpr int kGroup = 64;   // INT4 group size along head_dim

__host__ __device__ constexpr int page_data_bytes(int fmt, int D) {
  return fmt == kBF16 ? kPage * D * 2 : (fmt == kINT4G64 ? kPage * D / 2 : kPage * D);
}
__host__ __device__ constexpr int page_meta_bytes(int fmt, int D) {
  return fmt == kFP8Page ? 4 : fmt == kFP8Token ? 4 * kPage : fmt == kINT4G64 ? kPage * (D / kGroup) * 4 : 0;
}

// ---- conversions -----------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two e4m3 codes (low byte first) -> two floats.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t v) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  return __half22float2(*reinterpret_cast<__half2*>(&h));
}

// Two floats -> two e4m3 codes, round to nearest even, saturating to +-448.
__device__ __forceinline__ uint16_t float2_to_e4m3x2(float lo, float hi) {
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float half_bits_to_float(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}
__device__ __forceinline__ uint16_t float_to_half_bits(float f) {
  return __half_as_ushort(__float2half_rn(f));
}

// ---- warp reductions ----------------------------------------------------------------
template <int WIDTH = 32>
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int WIDTH = 32>
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int WIDTH = 32>
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- memory helpers ------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_nc_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_nc_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
// Plain (coherent) loads for memory another GPU may have written (peer slabs).
__device__ __forceinline__ uint4 ld_v4(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 ld_v2(const void* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t ld_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// ---- programmatic dependent launch ----------------------------------------------------
// A kernel started with launch_pdl() may begin while the kernel before it in the stream is
// still running (once every CTA of that kernel has called pdl_trigger(), or it has ended).
// Before reading anything an earlier kernel wrote, such a kernel calls pdl_wait(), which
// returns once the kernels before it have completed and their writes are visible; it calls
// pdl_wait() on every path before it ends, so completions stay in stream order (a kernel
// that ended early would otherwise release its own successor's wait while its predecessor
// still runs). pdl_trigger() right after a kernel's set-up lets the next kernel's CTAs come
// up on free SM space and start their independent loads (weights, old KV pages).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// AXR_PDL=0 launches every kernel with plain stream order (for measurements).
inline bool pdl_enabled_env() {
  static const bool on = [] {
    const char* e = std::getenv("AXR_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled_env() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace axr

#define AXR_CHECK_CUDA(expr)                                                          \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error: ", cudaGetErrorString(_e), " at ", \
                __FILE__, ":", __LINE__);                                             \
  } while (0)
