// Allocation-free split-KV decode attention: one extern "C" entry point.
//
// THIS FILE HAS NO COUNTERPART IN THE REFERENCE. It exists for callers that cannot
// allocate GPU memory at call time: code running where cudaMalloc (and allocator
// libraries such as torch's caching allocator) is off limits -- inside a host
// framework that owns the device memory budget, a plugin of another inference
// runtime that only hands over input/output buffers, or a latency-critical path
// that must never enter the driver's allocator. The regular decode_attention needs
// a caller-provided fp32 scratch area for its split-KV partial results; this
// variant keeps that scratch in a fixed device array compiled into the library, so
// the caller passes only inputs and outputs.
//
// Scratch: g_noalloc_scratch, a file-scope static __device__ array of
// kScratchFloats = 2,097,152 floats (8 MiB). Every GPU that loads the library holds
// it until the process exits. One call needs B * Hq * S * (D + 1) floats of it
// (S = number of KV splits, D = head_dim); larger calls are rejected with
// AXR_NOALLOC_TOO_LARGE before anything is launched. With S == 1 no scratch is used.
//
// Set-up: host code cannot use the array's name as a device address (on the host it
// is only a stand-in symbol). The first call on each device runs the set-up with
// that device current: cudaGetSymbolAddress() of the array, return code checked,
// result cached per device. Make that first call before any stream capture.
//
// Sharing: every call uses the same scratch array and leaves its partial results
// there. Nothing has to start at zero -- each call writes every scratch element it
// later reads -- but calls that overlap on the GPU (two streams, or two threads
// launching concurrently on one device) race on the array and corrupt each other's
// results; serialise them.
//
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
//
// Inputs are bf16 KV pages laid out as [block][head][16 tokens][D] per layer (the
// framework's paged cache), q/out are bf16 [B, Hq, D], block_table int32 [B, bt_stride],
// seq_lens int32 [B]. Supported: D = 128, GQA group Hq/Hkv in {1, 2, 4, 8}.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <mutex>

#include "decode_attn_noalloc.h"

namespace {

constexpr int kNoAllocPage = 16;
constexpr int kNoAllocD = 128;
constexpr long long kScratchFloats = AXR_NOALLOC_SCRATCH_FLOATS;  // 8 MiB of fp32 scratch per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

std::mutex g_setup_mu;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
thread_local const char* g_last_error = "ok";

__device__ __forceinline__ float lo_bf16(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

struct NoAllocParams {
  const __nv_bfloat16* q;
  const char* k;
  const char* v;
  long long blk_stride, head_stride;
  const int* block_table;
  int bt_stride;
  const int* seq_lens;
  int Hq, pages_per_split, max_pages;
  float scale_log2;
  __nv_bfloat16* out;
  float* part_o;   // scratch [B, Hq, S, D]
  float* part_lse; // scratch [B, Hq, S]
};

// Grid (splits, kv_heads, batch), 4 warps. Same dataflow as the library's bf16
// decode kernel: warps take pages round-robin with their own online softmax, merged
// at the end; QK lane = (token, half of head_dim), PV lane = 4 output dims.
template <int G>
__global__ void __launch_bounds__(128) noalloc_decode_kernel(NoAllocParams p) {
  constexpr int D = kNoAllocD, HALF = D / 2, QPAD = HALF + 4, DPL = D / 32;
  __shared__ float qs[G][2][QPAD];
  __shared__ float pbuf[4][kNoAllocPage][G];
  __shared__ float wm[4][G], wl[4][G];
  __shared__ float wacc[4][G][D];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, S = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq_len = p.seq_lens[b];
  const int n_pages = (seq_len + kNoAllocPage - 1) / kNoAllocPage;
  const int pg0 = split * p.pages_per_split;
  const int pg1 = min(min(n_pages, p.max_pages), pg0 + p.pages_per_split);  // never past the table row
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    qs[g][d / HALF][d % HALF] = __bfloat162float(p.q[((long long)b * p.Hq + kvh * G + g) * D + d]) * p.scale_log2;
  }
  __syncthreads();
  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -FLT_MAX;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[g][j] = 0.f;
  }
  const int t = lane >> 1, half = lane & 1;
  const int* bt = p.block_table + (long long)b * p.bt_stride;
  for (int pg = pg0 + warp; pg < pg1; pg += 4) {
    const int blk = bt[pg];
    const char* kb = p.k + blk * p.blk_stride + kvh * p.head_stride;
    const char* vb = p.v + blk * p.blk_stride + kvh * p.head_stride;
    const bool valid = pg * kNoAllocPage + t < seq_len;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    const char* row = kb + (long long)t * D * 2 + half * HALF * 2;
#pragma unroll
    for (int j = 0; j < HALF / 8; ++j) {
      const uint4 x = *reinterpret_cast<const uint4*>(row + j * 16);
      const float kv[8] = {lo_bf16(x.x), hi_bf16(x.x), lo_bf16(x.y), hi_bf16(x.y),
                           lo_bf16(x.z), hi_bf16(x.z), lo_bf16(x.w), hi_bf16(x.w)};
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s[g] += qs[g][half][j * 8 + e] * kv[e];
      }
    }
    float pe[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] += __shfl_xor_sync(0xffffffffu, s[g], 1);
      if (!valid) s[g] = -FLT_MAX;
      float mx = s[g];
#pragma unroll
      for (int o = 2; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mnew = fmaxf(m[g], mx);
      const float alpha = exp2f(m[g] - mnew);
      m[g] = mnew;
      pe[g] = valid ? exp2f(s[g] - mnew) : 0.f;
      l[g] = l[g] * alpha + (half == 0 ? pe[g] : 0.f);
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[g][j] *= alpha;
    }
    if (half == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) pbuf[warp][t][g] = pe[g];
    }
    __syncwarp();
    for (int tt = 0; tt < kNoAllocPage; ++tt) {
      const uint2 x = *reinterpret_cast<const uint2*>(vb + (long long)tt * D * 2 + lane * DPL * 2);
      const float vv[4] = {lo_bf16(x.x), hi_bf16(x.x), lo_bf16(x.y), hi_bf16(x.y)};
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pv = pbuf[warp][tt][g];
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[g][j] += pv * vv[j];
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float lw = l[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
    if (lane == 0) {
      wm[warp][g] = m[g];
      wl[warp][g] = lw;
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) wacc[warp][g][lane * DPL + j] = acc[g][j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float M = -FLT_MAX;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float f = wm[w][g] == -FLT_MAX ? 0.f : exp2f(wm[w][g] - M);
      L += wl[w][g] * f;
      O += wacc[w][g][d] * f;
    }
    const int hq = kvh * G + g;
    const float o = L > 0.f ? O / L : 0.f;
    if (S == 1) {
      p.out[((long long)b * p.Hq + hq) * D + d] = __float2bfloat16(o);
    } else {
      const long long base = ((long long)b * p.Hq + hq) * S + split;
      p.part_o[base * D + d] = o;
      if (d == 0) p.part_lse[base] = L > 0.f ? M + log2f(L) : -FLT_MAX;
    }
  }
}

__global__ void noalloc_combine_kernel(const float* part_o, const float* part_lse, __nv_bfloat16* out, int S) {
  const long long bh = blockIdx.x;
  const float* lse = part_lse + bh * S;
  float M = -FLT_MAX;
  for (int s = 0; s < S; ++s) M = fmaxf(M, lse[s]);
  for (int d = threadIdx.x; d < kNoAllocD; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < S; ++s) {
      if (lse[s] == -FLT_MAX) continue;
      const float w = exp2f(lse[s] - M);
      num += w * part_o[(bh * S + s) * kNoAllocD + d];
      den += w;
    }
    out[bh * kNoAllocD + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
  }
}

// Per-device set-up: resolves the device address of the scratch array once, with
// the caller's current device. Returns nullptr (and records why) on failure.
float* scratch_for_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    g_last_error = "no usable current CUDA device";
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (rc != cudaSuccess || ptr == nullptr) {
      g_last_error = "cudaGetSymbolAddress of the decode scratch array failed";
      return nullptr;
    }
    g_scratch_ptr[dev] = static_cast<float*>(ptr);
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" {

// Largest number of fp32 scratch elements one call may use: B * Hq * S * (D + 1).
__attribute__((visibility("default"))) long long axr_decode_noalloc_scratch_floats(void) { return kScratchFloats; }

// Human-readable reason of the last non-zero return code (static string, never freed).
__attribute__((visibility("default"))) const char* axr_decode_noalloc_last_error(void) { return g_last_error; }

// Split-KV decode attention over bf16 KV pages without allocating anything.
// Returns AXR_NOALLOC_OK or an error code; on error nothing has been launched,
// except AXR_NOALLOC_LAUNCH_FAILED (the launch itself reported an error).
__attribute__((visibility("default"))) int axr_decode_attention_noalloc(
    const void* q, void* out, const void* k_pages, const void* v_pages, long long blk_stride,
    long long head_stride, const int* block_table, int bt_stride, const int* seq_lens, int B, int Hq,
    int Hkv, int D, float scale, int num_splits, int max_pages, cudaStream_t stream) {
  if (!q || !out || !k_pages || !v_pages || !block_table || !seq_lens || B <= 0 || Hq <= 0 || Hkv <= 0 ||
      Hq % Hkv != 0 || num_splits < 1 || max_pages < 0 || bt_stride < 0 || max_pages > bt_stride) {
    g_last_error = "invalid arguments";
    return AXR_NOALLOC_BAD_ARGS;
  }
  const int G = Hq / Hkv;
  if (D != kNoAllocD || (G != 1 && G != 2 && G != 4 && G != 8)) {
    g_last_error = "unsupported shape: head_dim must be 128 and Hq/Hkv in {1,2,4,8}";
    return AXR_NOALLOC_BAD_ARGS;
  }
  const long long need = num_splits > 1 ? (long long)B * Hq * num_splits * (D + 1) : 0;
  if (need > kScratchFloats) {
    g_last_error = "call needs more scratch than the fixed 8 MiB array (B*Hq*splits*(head_dim+1) > 2097152)";
    return AXR_NOALLOC_TOO_LARGE;
  }
  if (cudaPeekAtLastError() != cudaSuccess) {  // not ours: leave it for its owner
    g_last_error = "an earlier CUDA error is pending on this thread; nothing launched";
    return AXR_NOALLOC_PENDING_ERROR;
  }
  float* scratch = nullptr;
  if (num_splits > 1) {
    scratch = scratch_for_current_device();
    if (scratch == nullptr) return AXR_NOALLOC_SETUP_FAILED;
  }
  NoAllocParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const char*>(k_pages);
  p.v = static_cast<const char*>(v_pages);
  p.blk_stride = blk_stride;
  p.head_stride = head_stride;
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.Hq = Hq;
  p.pages_per_split = (max_pages + num_splits - 1) / num_splits;
  p.max_pages = max_pages;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.part_o = scratch;
  p.part_lse = scratch ? scratch + (long long)B * Hq * num_splits * D : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_splits, Hkv, B);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaError_t rc;
  switch (G) {
    case 1: rc = cudaLaunchKernelEx(&cfg, noalloc_decode_kernel<1>, p); break;
    case 2: rc = cudaLaunchKernelEx(&cfg, noalloc_decode_kernel<2>, p); break;
    case 4: rc = cudaLaunchKernelEx(&cfg, noalloc_decode_kernel<4>, p); break;
    default: rc = cudaLaunchKernelEx(&cfg, noalloc_decode_kernel<8>, p); break;
  }
  if (rc != cudaSuccess) {
    g_last_error = "decode kernel launch failed";
    return AXR_NOALLOC_LAUNCH_FAILED;
  }
  if (num_splits > 1) {
    cudaLaunchConfig_t c2 = {};
    c2.gridDim = dim3(B * Hq);
    c2.blockDim = dim3(kNoAllocD);
    c2.stream = stream;
    rc = cudaLaunchKernelEx(&c2, noalloc_combine_kernel, static_cast<const float*>(p.part_o),
                            static_cast<const float*>(p.part_lse), p.out, num_splits);
    if (rc != cudaSuccess) {
      g_last_error = "combine kernel launch failed";
      return AXR_NOALLOC_LAUNCH_FAILED;
    }
  }
  g_last_error = "ok";
  return AXR_NOALLOC_OK;
}

}  // extern "C"
