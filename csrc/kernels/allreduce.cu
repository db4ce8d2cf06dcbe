// One-shot all-reduce (sum, bf16) over NVLink peer memory, for the small activations of
// tensor-parallel decode (a few hundred KB per call, where a collective library's
// latency dominates).
//
// Each GPU stores its input into every peer's receive slot [parity][rank] with plain
// 16-byte peer stores, the last of its CTAs raises this GPU's flag on every peer
// (system-scope release), every CTA waits (bounded) for all GPUs' flags and sums the
// world slots of its range in fp32. The call's epoch lives in device memory and the last
// CTA to finish advances it, so the kernel carries no per-call host state (it can sit in
// a captured CUDA graph). Slots and flags alternate between two parities: a peer can be
// at most one call ahead. No TMA, no multicast; every wait is bounded and reports through
// the error flag.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "peer_sync.cuh"

namespace axr {

struct ArArgs {
  const __nv_bfloat16* in;
  __nv_bfloat16* out;
  long long n8;  // 16-byte vectors
  long long cap;  // elements per slot
  int rank, world;
  const int64_t* peer_buf;   // [world] -> bf16 [2][world][cap]
  const int64_t* peer_flag;  // [world] -> int [2][world]
  const __nv_bfloat16* buf;  // local receive area
  const int* flag;           // local flags
  int* epoch;                // local: epoch of the last completed call
  int* bar;                  // local [2]: CTA arrival counters (zero between calls)
  volatile int* err;
  unsigned long long wait_ns;
};

__global__ void __launch_bounds__(256) peer_allreduce_kernel(ArArgs a) {
  __shared__ int s_ok;
  const int e = ld_acquire_gpu(a.epoch) + 1;
  const int par = e & 1, W = a.world;
  const long long per = (a.n8 + gridDim.x - 1) / gridDim.x;
  const long long v0 = blockIdx.x * per, v1 = min(a.n8, v0 + per);
  // 1. push this GPU's input slice into every peer's slot [par][rank]
  const uint4* src = reinterpret_cast<const uint4*>(a.in);
  for (long long v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const uint4 x = src[v];
    for (int p = 0; p < W; ++p) {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.peer_buf[p]) +
                                            ((long long)par * W + a.rank) * a.cap);
      dst[v] = x;
    }
  }
  __syncthreads();
  // 2. the last CTA to finish its pushes raises this GPU's flag on every peer (the
  //    barrier + system fence order the whole CTA's peer stores before the flags)
  if (threadIdx.x == 0) __threadfence_system();
  if (threadIdx.x == 0 && atomicAdd(&a.bar[0], 1) == gridDim.x - 1) {
    a.bar[0] = 0;
    __threadfence_system();
    for (int p = 0; p < W; ++p) st_release_sys(reinterpret_cast<int*>(a.peer_flag[p]) + par * W + a.rank, e);
  }
  // 3. wait for every GPU's data
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int p = 0; ok && p < W; ++p) ok = wait_geq<true>(a.flag + par * W + p, e, a.err, 61, a.wait_ns);
    s_ok = ok;
  }
  __syncthreads();
  if (s_ok) {
    // 4. sum the world slots of this CTA's range
    for (long long v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int p = 0; p < W; ++p) {
        const uint4 x = reinterpret_cast<const uint4*>(a.buf + ((long long)par * W + p) * a.cap)[v];
        acc[0] += bf16_lo(x.x); acc[1] += bf16_hi(x.x); acc[2] += bf16_lo(x.y); acc[3] += bf16_hi(x.y);
        acc[4] += bf16_lo(x.z); acc[5] += bf16_hi(x.z); acc[6] += bf16_lo(x.w); acc[7] += bf16_hi(x.w);
      }
      reinterpret_cast<uint4*>(a.out)[v] =
          make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                     pack_bf16x2(acc[6], acc[7]));
    }
  }
  // 5. the last CTA out advances the epoch (every CTA has read it by now)
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(&a.bar[1], 1) == gridDim.x - 1) {
    a.bar[1] = 0;
    __threadfence();
    *a.epoch = e;
  }
}

// x (bf16, contiguous, numel % 8 == 0) -> out = sum over the group. peers: int64 [2, world]
// (receive-area and flag addresses of every GPU); buf/flag: this GPU's own; epoch int32 [1],
// bar int32 [2] (zero-initialised once).
void peer_allreduce(torch::Tensor x, torch::Tensor out, int64_t rank, int64_t world, torch::Tensor peers,
                    torch::Tensor buf, torch::Tensor flag, torch::Tensor epoch, torch::Tensor bar, int64_t cap,
                    torch::Tensor err) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "peer_allreduce: bf16 input");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == torch::kBFloat16 && out.numel() == x.numel(),
              "peer_allreduce: out");
  TORCH_CHECK(x.numel() % 8 == 0 && x.numel() <= cap, "peer_allreduce: size must be a multiple of 8 within capacity");
  TORCH_CHECK(peers.scalar_type() == torch::kInt64 && peers.numel() >= 2 * world, "peer_allreduce: peer table");
  if (x.numel() == 0) return;
  ArArgs a{};
  a.in = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.n8 = x.numel() / 8;
  a.cap = cap;
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.peer_buf = peers.data_ptr<int64_t>();
  a.peer_flag = a.peer_buf + world;
  a.buf = reinterpret_cast<const __nv_bfloat16*>(buf.data_ptr());
  a.flag = flag.data_ptr<int>();
  a.epoch = epoch.data_ptr<int>();
  a.bar = bar.data_ptr<int>();
  a.err = err.data_ptr<int>();
  a.wait_ns = peer_wait_ns();
  // A CTA waits for this GPU's own flag, which the last CTA to push raises: every CTA
  // must be resident at once. With at most 32 CTAs of 256 threads
  // they all fit on the GPU at any time, so a plain launch suffices (one CTA per 1024 vectors); were one to be held
  // back anyway, the others' waits end at the bound with an error code, not a hang.
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(32, (a.n8 + 1023) / 1024)));
  peer_allreduce_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  AXR_CHECK_CUDA(cudaGetLastError());
}

}  // namespace axr
