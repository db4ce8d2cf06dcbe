// Device-resident token selection.
//   * argmax_rows: greedy token per logits row, lowest index on ties.
//   * spec_verify: greedy speculative verification entirely on the device — argmax
//     of every target row on one grid, compared with the draft tokens, first mismatch
//     found with a ballot; outputs {accepted, first_mismatch, mismatch_token} per sequence. No
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

// One element into a thread's running (best, index); NaN never wins, ties keep the lower index.
__device__ __forceinline__ void take(float x, int i, float& best, int& bi) {
  if ((__float_as_uint(x) & 0x7fffffffu) > 0x7f800000u) x = -FLT_MAX;
  if (x > best || (x == best && i < bi)) { best = x; bi = i; }
}

template <typename T>
__device__ __forceinline__ void take_vec(const uint4& v, int i0, float& best, int& bi);
template <>
__device__ __forceinline__ void take_vec<float>(const uint4& v, int i0, float& best, int& bi) {
  take(__uint_as_float(v.x), i0, best, bi);
  take(__uint_as_float(v.y), i0 + 1, best, bi);
  take(__uint_as_float(v.z), i0 + 2, best, bi);
  take(__uint_as_float(v.w), i0 + 3, best, bi);
}
template <>
__device__ __forceinline__ void take_vec<__nv_bfloat16>(const uint4& v, int i0, float& best, int& bi) {
  const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    take(__uint_as_float(w[j] << 16), i0 + 2 * j, best, bi);           // low half = lower index
    take(__uint_as_float(w[j] & 0xffff0000u), i0 + 2 * j + 1, best, bi);
  }
}

// Block-wide argmax of one row; every thread returns the index. A row whose start is
// 16-byte aligned is read as 16-byte vectors, four in flight per thread (a logits row is
// read once, so the kernel is bound by how many loads are outstanding); the remainder
// and misaligned rows are read element by element.
template <typename T>
__device__ int row_argmax(const T* __restrict__ row, int V) {
  constexpr int VEC = 16 / sizeof(T);
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    const int nv = V / VEC;
    int v = threadIdx.x;
    for (; v + 3 * (int)blockDim.x < nv; v += 4 * blockDim.x) {
      uint4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = __ldg(rv + v + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u) take_vec<T>(a[u], (v + u * blockDim.x) * VEC, best, bi);
    }
    for (; v < nv; v += blockDim.x) take_vec<T>(__ldg(rv + v), v * VEC, best, bi);
    done = nv * VEC;
  }
  for (int i = done + threadIdx.x; i < V; i += blockDim.x) take(to_f<T>(row[i]), i, best, bi);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  __shared__ int res;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sb[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    best = l < (int)(blockDim.x >> 5) ? sb[l] : -FLT_MAX;
    bi = l < (int)(blockDim.x >> 5) ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (l == 0) res = bi == 0x7fffffff ? 0 : bi;  // a row with no finite entry still yields a valid token
  }
  __syncthreads();
  return res;
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
// token to emit at the mismatch (target argmax) or the bonus token. The B x (K+1) row
// argmaxes run as one grid (every SM busy), then one warp per sequence finds the first
// mismatch with a ballot.
__global__ void spec_accept_kernel(const int* __restrict__ tgt, const int* __restrict__ draft, int B, int K,
                                   int* __restrict__ out) {
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  int first = K;
  for (int base = 0; base < K; base += 32) {
    const int k = base + lane;
    const bool mism = k < K && draft[b * K + k] != tgt[b * (K + 1) + k];
    const unsigned m = __ballot_sync(0xffffffffu, mism);
    if (m) { first = base + __ffs(m) - 1; break; }
  }
  if (lane == 0) {
    out[b * 3 + 0] = first;
    out[b * 3 + 1] = first;
    out[b * 3 + 2] = tgt[b * (K + 1) + first];
  }
}

void spec_verify(torch::Tensor logits, torch::Tensor draft, torch::Tensor out) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 3 && logits.is_contiguous(), "logits [B, K+1, V] contiguous");
  TORCH_CHECK(draft.scalar_type() == torch::kInt32 && out.scalar_type() == torch::kInt32, "int32 draft/out");
  const int B = logits.size(0), K = logits.size(1) - 1, V = logits.size(2);
  TORCH_CHECK(K >= 0 && K <= 64, "spec_verify: at most 64 draft tokens");
  if (B == 0) return;
  auto tgt = torch::empty({(long long)B * (K + 1)}, out.options());
  argmax_rows(logits.view({(long long)B * (K + 1), V}), tgt);
  auto st = at::cuda::getCurrentCUDAStream();
  spec_accept_kernel<<<(B + 7) / 8, 256, 0, st>>>(tgt.data_ptr<int>(), draft.data_ptr<int>(), B, K, out.data_ptr<int>());
  AXR_CHECK_CUDA(cudaGetLastError());
}

}  // namespace axr
