// Host interface of the dense tcgen05 projections (csrc/kernels/gemm_dense.cu).
// Plain C++ (no torch headers), shared by the kernel file and its torch binding.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

namespace axr {
namespace dense {

enum Epi : int { kStore = 0, kResid = 1, kSwiGLU = 2, kRope = 3 };

// One call: out = epilogue(x w^T).
//   x   [M, K] bf16, row stride ldx (elements)
//   w   [N, K] bf16, row stride ldw ("out x in" weights)
//   out [M, N] (STORE/RESID), [M, N/2] (SWIGLU), [M, Hq*128] (ROPE: rotated q)
struct DenseCall {
  const void* x;
  int64_t ldx;
  const void* w;
  int64_t ldw;
  void* out;
  int64_t ldo;
  int M, N, K;
  int epi;
  const void* res;  // RESID: [M, N] bf16 (may equal out)
  int64_t ldr;
  const int* pos;      // ROPE: [M] positions
  const int* slots;    // ROPE: [M] cache slots (block*16 + offset, < 0 = not stored)
  const float* cos_sin;  // ROPE: [n_pos, 128] fp32
  int n_pos;
  void* kc;            // ROPE: bf16 paged cache of the layer (K / V)
  void* vc;
  int64_t blk_stride, head_stride;  // bytes
  int Hq, Hkv;
  float* ws;   // split-K partials (stream kernel, stream_workspace floats)
  int* cnt;    // per-tile arrival counters, zero between calls
  int* err;    // error flag (bounded waits)
  int splits;  // <= 0: stream_splits
  bool force_big;
  bool force_one_cta;  // big-M path on the 1-CTA kernel instead of the CTA-pair kernel
  int device;
};

// Token-column padding of the stream kernel for M rows (0 = M > 256, big kernel).
int stream_nt(int64_t M);
// Largest split count of the stream kernel at token padding nt (its shared-memory stage).
int stream_max_splits(int nt);
// CTAs per 128-row weight tile of the stream kernel.
int stream_splits(int64_t M, int64_t N, int64_t K, int sms);
// {fp32 partial floats, counters} the stream kernel needs.
void stream_workspace(int64_t M, int64_t N, int64_t K, int sms, int64_t* ws_floats, int64_t* counters);
// Timeline of the last traced stream-kernel launch (AXR_DENSE_TRACE=1): 8 stamps per CTA.
int dense_trace(std::vector<unsigned long long>* out);
// Thread-block clusters (CTA pairs) the prefill-sized kernel keeps resident on device `dev`.
int pair_grid_clusters(int dev);
// Checks the call and launches; returns an empty string or the reason it refused.
std::string dense_gemm_launch(const DenseCall& c, cudaStream_t st);

}  // namespace dense
}  // namespace axr
