// Host interface of the GPU codec kernels of the reference's blob formats
// (csrc/kernels/codecs.cu). Plain C++, no torch headers.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace axr {
namespace codec {

enum Format : int { kInt4Sym = 0, kInt4Block = 1, kInt2Sym = 2, kNvfp4 = 3 };
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// Encode x viewed as [rows, D] (last axis D). int4_sym / int2_sym: per-lane scales
// (amax [D], scale32 [D], scale16 [D]). int4_sym_block: x is [S, T, HD] with rows = S*T*HD/D,
// one scale per (s, block of BT tokens): amax / scale32 / scale16 [S * ceil(T/BT)].
// nvfp4: sbytes [rows, ceil(D/16)], amax [1] (the tensor scale). out: packed codes.
struct EncodeCall {
  const void* x;
  int dtype;
  long long rows;
  int D;
  int fmt;
  int S, T, HD, BT;     // int4_sym_block geometry
  uint8_t* out;
  float* amax;
  float* scale32;
  __half* scale16;
  uint8_t* sbytes;
};

struct DecodeCall {
  const uint8_t* in;
  int dtype;  // of out
  long long rows;
  int D;
  int fmt;
  int S, T, HD, BT;
  const __half* scale16;
  const uint8_t* sbytes;
  void* out;
};

std::string encode(const EncodeCall& c, cudaStream_t st);
std::string decode(const DecodeCall& c, cudaStream_t st);

}  // namespace codec
}  // namespace axr
