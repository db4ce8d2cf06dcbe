// Log-sum-exp combine of split-KV attention partials (shared by split-KV decode and
// split-KV prefill).
//
// part_o [R, S, D] fp32 holds each split's normalised output for row r (a (token, head)
// pair), part_lse [R, S] its log2-domain log-sum-exp (max + log2(sum)), -FLT_MAX when
// the split saw no key for that row; out [R, D] bf16.
#pragma once

#include <cuda_bf16.h>

#include <cfloat>

#include "common.cuh"

namespace axr {

template <int D>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                      __nv_bfloat16* __restrict__ out, int S) {
  const long long bh = blockIdx.x;
  pdl_trigger();
  pdl_wait();  // the partials come from the attention kernel before
  const float* lse = part_lse + bh * S;
  float M = -FLT_MAX;
  for (int s = 0; s < S; ++s) M = fmaxf(M, lse[s]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < S; ++s) {
      if (lse[s] == -FLT_MAX) continue;
      const float w = exp2f(lse[s] - M);
      num += w * part_o[(bh * S + s) * D + d];
      den += w;
    }
    out[bh * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
  }
}

// Shared-prefix decode: row bh = (b, head) merges its S own-page partials with the S2
// partials of its row in the grouped shared-prefix pass (row_of[b] = packed row, -1 =
// the sequence shares no prefix), part2_* laid out [R, Hq, S2(, D)].
template <int D>
__global__ void cascade_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int S,
                                       const float* __restrict__ part_o2, const float* __restrict__ part_lse2, int S2,
                                       const int* __restrict__ row_of, int Hq, __nv_bfloat16* __restrict__ out) {
  const long long bh = blockIdx.x;
  pdl_trigger();
  pdl_wait();
  const int b = static_cast<int>(bh / Hq), h = static_cast<int>(bh % Hq);
  const float* lse = part_lse + bh * S;
  const int r = row_of[b];
  const long long bh2 = r >= 0 ? (long long)r * Hq + h : -1;
  const float* lse2 = r >= 0 ? part_lse2 + bh2 * S2 : nullptr;
  float M = -FLT_MAX;
  for (int s = 0; s < S; ++s) M = fmaxf(M, lse[s]);
  for (int s = 0; lse2 && s < S2; ++s) M = fmaxf(M, lse2[s]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < S; ++s) {
      if (lse[s] == -FLT_MAX) continue;
      const float w = exp2f(lse[s] - M);
      num += w * part_o[(bh * S + s) * D + d];
      den += w;
    }
    for (int s = 0; lse2 && s < S2; ++s) {
      if (lse2[s] == -FLT_MAX) continue;
      const float w = exp2f(lse2[s] - M);
      num += w * part_o2[(bh2 * S2 + s) * D + d];
      den += w;
    }
    out[bh * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
  }
}

}  // namespace axr
