// Device-resident token selection.
//   * argmax_rows: greedy token per logits row, lowest index on ties.
//   * spec_verify: greedy speculative verification entirely on the device — argmax
//     of each target row, compared with the draft tokens, first mismatch found with a
//     ballot; outputs {accepted, first_mismatch, mismatch_token} per sequence. No
//     logits or tokens cross to the host (the reference copies full fp32 logits rows
//     host->device on every call, core/kernels/spec_verify.cu:209-229, and its accept
//     scan syncs the host each call, core/kernels/accept_scan.cu:190-275).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cfloat>

#include "common.cuh"

namespace axr {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Block-wide argmax of one row; returns the index in thread 0.
template <typename T>
__device__ int row_argmax(const T* __restrict__ row, int V) {
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float x = to_f<T>(row[i]);
    if ((__float_as_uint(x) & 0x7fffffffu) > 0x7f800000u) x = -FLT_MAX;  // NaN never wins
    if (x > best || (x == best && i < bi)) { best = x; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sb[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    best = l < (blockDim.x >> 5) ? sb[l] : -FLT_MAX;
    bi = l < (blockDim.x >> 5) ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
  }
  __syncthreads();
  return bi == 0x7fffffff ? 0 : bi;  // a row with no finite entry still yields a valid token
}

template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ logits, int V, long long stride,
                                                      int* __restrict__ out) {
  const int r = row_argmax<T>(logits + blockIdx.x * stride, V);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

void argmax_rows(torch::Tensor logits, torch::Tensor out) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "logits [N, V] with unit stride");
  TORCH_CHECK(out.scalar_type() == torch::kInt32, "out int32");
  const int N = logits.size(0), V = logits.size(1);
  if (N == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == torch::kFloat32)
    argmax_kernel<float><<<N, 1024, 0, st>>>(logits.data_ptr<float>(), V, logits.stride(0), out.data_ptr<int>());
  else if (logits.scalar_type() == torch::kBFloat16)
    argmax_kernel<__nv_bfloat16><<<N, 1024, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), V,
                                                     logits.stride(0), out.data_ptr<int>());
  else TORCH_CHECK(false, "argmax_rows: fp32 or bf16 logits");
  AXR_CHECK_CUDA(cudaGetLastError());
}

// logits: [B, K+1, V] target logits for the K draft positions plus the bonus row;
// draft: [B, K] int32. out: [B, 3] int32 = accepted, first_mismatch (K if none),
// token to emit at the mismatch (target argmax) or the bonus token.
template <typename T>
__global__ void __launch_bounds__(1024) spec_verify_kernel(const T* __restrict__ logits, const int* __restrict__ draft,
                                                           int K, int V, int* __restrict__ out) {
  __shared__ int tgt[65];
  const int b = blockIdx.x;
  for (int k = 0; k <= K; ++k) {
    const int a = row_argmax<T>(logits + ((long long)b * (K + 1) + k) * V, V);
    if (threadIdx.x == 0) tgt[k] = a;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int first = K;
    for (int base = 0; base < K; base += 32) {
      const int k = base + lane;
      const bool mism = k < K && draft[b * K + k] != tgt[k];
      const unsigned m = __ballot_sync(0xffffffffu, mism);
      if (m) { first = base + __ffs(m) - 1; break; }
    }
    if (lane == 0) {
      out[b * 3 + 0] = first;
      out[b * 3 + 1] = first;
      out[b * 3 + 2] = tgt[first];
    }
  }
}

void spec_verify(torch::Tensor logits, torch::Tensor draft, torch::Tensor out) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 3 && logits.is_contiguous(), "logits [B, K+1, V] contiguous");
  TORCH_CHECK(draft.scalar_type() == torch::kInt32 && out.scalar_type() == torch::kInt32, "int32 draft/out");
  const int B = logits.size(0), K = logits.size(1) - 1, V = logits.size(2);
  TORCH_CHECK(K >= 0 && K <= 64, "spec_verify: at most 64 draft tokens");
  if (B == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == torch::kFloat32)
    spec_verify_kernel<float><<<B, 1024, 0, st>>>(logits.data_ptr<float>(), draft.data_ptr<int>(), K, V,
                                                  out.data_ptr<int>());
  else if (logits.scalar_type() == torch::kBFloat16)
    spec_verify_kernel<__nv_bfloat16><<<B, 1024, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()),
                                                          draft.data_ptr<int>(), K, V, out.data_ptr<int>());
  else TORCH_CHECK(false, "spec_verify: fp32 or bf16 logits");
  AXR_CHECK_CUDA(cudaGetLastError());
}

}  // namespace axr
