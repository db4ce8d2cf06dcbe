// Host interface of the tcgen05 prefill attention kernel (csrc/kernels/prefill_tc.cu).
// Plain C++ (no torch headers), shared by the kernel file and its torch binding.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace axr {
namespace fa {

struct PrefillCall {
  const void* q;        // [T, Hq, 128] bf16
  void* out;            // [T, Hq, 128] bf16
  int T, Hq, Hkv;
  const void* k;        // the layer's K / V page regions [num_blocks, Hkv, 16, 128] bf16
  const void* v;
  int64_t num_blocks;
  const int* block_table;
  int bt_stride;
  const int* cu_q;      // [B + 1]
  const int* seq_lens;  // [B]
  int B;
  int max_q;
  float scale;
  int* err;
  int num_splits;       // KV slices per query tile (1: none)
  int gqa_pack;         // > 1: rows = (token, head of the KV group)
  float* part_o;        // [R, Hq, S, 128] (S > 1 or partial_only)
  float* part_lse;      // [R, Hq, S]
  int noncausal;
  const int* q_index;   // nullable
  int partial_only;
};

// Launches the attention (and the split-KV combine when num_splits > 1 and the partials
// are not kept); returns an empty string or the reason it refused.
std::string prefill_launch(const PrefillCall& c, cudaStream_t st);
// Measurement aid: per-KV-tile clock64 stamps of the last launch traced with AXR_PREFILL_TRACE=1.
int prefill_trace(long long* host, int n);

}  // namespace fa
}  // namespace axr
