// Split-KV flash-decode over the paged KV cache, reading bf16, FP8 (per-token
// scaled) or INT4 g64 (asymmetric) pages directly — the compressed pages are never
// expanded into a bf16 copy.
//
// Reference counterparts: the FP8/INT4 decode kernels fp8_decode_attention.cu:85-201
// and int4_decode_attention.cu:39-177 (contiguous caches, one CTA per (batch, head),
// never wired in) and the SDPA fallback kernels/dispatch.py:117-152.
//
// Grid (splits, kv_heads, batch); 4 warps per CTA. A CTA owns one KV head of one
// sequence and a contiguous range of pages; the G query heads of that KV head
// (GQA group) are processed together so each KV byte is read once. Warps take pages
// round-robin and keep independent online-softmax state, merged once at the end.
// Inside a warp: QK uses lane = (token, half of head_dim); PV uses lane = 4 output
// dims (D=128). With one split the kernel writes bf16 output; with several it writes
// a normalised partial output and its log2-sum-exp, and decode_combine merges them.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cfloat>

#include "common.cuh"

namespace axr {

struct DecodeParams {
  const __nv_bfloat16* q;  // [B, Hq, D]
  const char* k;           // page data base (this layer, K)
  const char* v;
  const char* km;          // page meta base (fp8 scales / int4 scale-zero), may be null
  const char* vm;
  long long blk_stride, head_stride;    // data bytes per block / per head inside a block
  long long mblk_stride, mhead_stride;  // meta bytes
  const int* block_table;  // [B, max_blocks]
  int bt_stride;
  const int* seq_lens;     // [B]
  int Hq, Hkv;
  int pages_per_split;
  float scale_log2;        // softmax scale * log2(e)
  __nv_bfloat16* out;      // [B, Hq, D] when splits == 1
  float* part_o;           // [B, Hq, S, D]
  float* part_lse;         // [B, Hq, S]
};

template <int D, int G, int FMT>
__global__ void __launch_bounds__(128) decode_attn_kernel(DecodeParams p) {
  constexpr int HALF = D / 2;
  constexpr int QPAD = HALF + 4;    // breaks the bank alignment of the two halves
  constexpr int DPL = D / 32;       // output dims per lane in PV
  static_assert(D == 128 || D == 64, "head_dim 64 or 128");
  __shared__ float qs[G][2][QPAD];
  __shared__ float qsum[G][D / kGroup];
  __shared__ float pbuf[4][kPage][G];
  __shared__ float pzbuf[4][kPage][G];
  __shared__ float wm[4][G], wl[4][G];
  __shared__ float wacc[4][G][D];

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int S = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq_len = p.seq_lens[b];
  const int n_pages = (seq_len + kPage - 1) / kPage;
  const int pg0 = split * p.pages_per_split;
  const int pg1 = min(n_pages, pg0 + p.pages_per_split);

  // Stage q (pre-scaled into the log2 domain) for the G heads of this KV head.
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    const float x = __bfloat162float(p.q[((long long)b * p.Hq + kvh * G + g) * D + d]) * p.scale_log2;
    qs[g][d / HALF][d % HALF] = x;
  }
  __syncthreads();
  if constexpr (FMT == kINT4G64) {
    if (threadIdx.x < G * (D / kGroup)) {
      const int g = threadIdx.x / (D / kGroup), grp = threadIdx.x % (D / kGroup);
      float s = 0.f;
      for (int d = grp * kGroup; d < (grp + 1) * kGroup; ++d) s += qs[g][d / HALF][d % HALF];
      qsum[g][grp] = s;
    }
    __syncthreads();
  }

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
    const char* kbase = p.k + blk * p.blk_stride + kvh * p.head_stride;
    const char* vbase = p.v + blk * p.blk_stride + kvh * p.head_stride;
    const int tok = pg * kPage + t;
    const bool valid = tok < seq_len;

    // ---- scores for token t, G heads (this lane: one half of head_dim)
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if constexpr (FMT == kBF16) {
      const char* row = kbase + (long long)t * D * 2 + half * HALF * 2;
#pragma unroll
      for (int j = 0; j < HALF / 8; ++j) {
        const uint4 x = ld_nc_v4(row + j * 16);
        const float kv[8] = {bf16_lo(x.x), bf16_hi(x.x), bf16_lo(x.y), bf16_hi(x.y),
                             bf16_lo(x.z), bf16_hi(x.z), bf16_lo(x.w), bf16_hi(x.w)};
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 qa = *reinterpret_cast<const float4*>(&qs[g][half][j * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&qs[g][half][j * 8 + 4]);
          s[g] += qa.x * kv[0] + qa.y * kv[1] + qa.z * kv[2] + qa.w * kv[3] + qb.x * kv[4] + qb.y * kv[5] +
                  qb.z * kv[6] + qb.w * kv[7];
        }
      }
    } else if constexpr (FMT == kFP8Token) {
      const char* row = kbase + (long long)t * D + half * HALF;
#pragma unroll
      for (int j = 0; j < HALF / 16; ++j) {
        const uint4 x = ld_nc_v4(row + j * 16);
        const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a = e4m3x2_to_float2(w[e] & 0xffff), c = e4m3x2_to_float2(w[e] >> 16);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float4 qa = *reinterpret_cast<const float4*>(&qs[g][half][j * 16 + e * 4]);
            s[g] += qa.x * a.x + qa.y * a.y + qa.z * c.x + qa.w * c.y;
          }
        }
      }
      const float ks = *reinterpret_cast<const float*>(p.km + blk * p.mblk_stride + kvh * p.mhead_stride + t * 4);
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] *= ks;
    } else {  // INT4 g64: lane half == group (D=128) or half a group (D=64)
      const char* row = kbase + (long long)t * (D / 2) + half * (HALF / 2);
#pragma unroll
      for (int j = 0; j < HALF / 32; ++j) {
        const uint4 x = ld_nc_v4(row + j * 16);
        const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
#pragma unroll
          for (int n = 0; n < 8; n += 4) {
            const float n0 = float((w[e] >> (4 * n)) & 0xf), n1 = float((w[e] >> (4 * n + 4)) & 0xf);
            const float n2 = float((w[e] >> (4 * n + 8)) & 0xf), n3 = float((w[e] >> (4 * n + 12)) & 0xf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              const float4 qa = *reinterpret_cast<const float4*>(&qs[g][half][j * 32 + e * 8 + n]);
              s[g] += qa.x * n0 + qa.y * n1 + qa.z * n2 + qa.w * n3;
            }
          }
        }
      }
      const char* mrow = p.km + blk * p.mblk_stride + kvh * p.mhead_stride + (long long)t * (D / kGroup) * 4;
      const int grp = (half * HALF) / kGroup;
      const uint32_t mm = ld_nc_u32(mrow + grp * 4);
      const float sc = half_bits_to_float(mm & 0xffff), zp = half_bits_to_float(mm >> 16);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float qsm = qsum[g][grp];
        if (D == 64) {  // half a group per lane: sum only this lane's half of q
          qsm = 0.f;
#pragma unroll
          for (int d = 0; d < HALF; ++d) qsm += qs[g][half][d];
        }
        s[g] = s[g] * sc + qsm * zp;
      }
    }
    // combine the two halves of head_dim
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] += __shfl_xor_sync(0xffffffffu, s[g], 1);
      if (!valid) s[g] = -FLT_MAX;
    }
    // ---- online softmax over the 16 tokens of the page
    float pexp[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = s[g];
#pragma unroll
      for (int o = 2; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mnew = fmaxf(m[g], mx);
      const float alpha = exp2f(m[g] - mnew);
      m[g] = mnew;
      pexp[g] = valid ? exp2f(s[g] - mnew) : 0.f;
      l[g] = l[g] * alpha + (half == 0 ? pexp[g] : 0.f);
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[g][j] *= alpha;
    }
    // ---- publish p (times the V scale for FP8; p*scale and p*zero for INT4)
    if (half == 0) {
      if constexpr (FMT == kFP8Token) {
        const float vs = *reinterpret_cast<const float*>(p.vm + blk * p.mblk_stride + kvh * p.mhead_stride + t * 4);
#pragma unroll
        for (int g = 0; g < G; ++g) pbuf[warp][t][g] = pexp[g] * vs;
      } else {
#pragma unroll
        for (int g = 0; g < G; ++g) pbuf[warp][t][g] = pexp[g];
      }
    }
    __syncwarp();
    // ---- PV: lane owns dims [lane*DPL, +DPL)
#pragma unroll 4
    for (int tt = 0; tt < kPage; ++tt) {
      float pv[G];
#pragma unroll
      for (int g = 0; g < G; ++g) pv[g] = pbuf[warp][tt][g];
      float vv[DPL];
      if constexpr (FMT == kBF16) {
        const char* vrow = vbase + (long long)tt * D * 2 + lane * DPL * 2;
        if constexpr (DPL == 4) {
          const uint2 x = ld_nc_v2(vrow);
          vv[0] = bf16_lo(x.x); vv[1] = bf16_hi(x.x); vv[2] = bf16_lo(x.y); vv[3] = bf16_hi(x.y);
        } else {
          const uint32_t x = ld_nc_u32(vrow);
          vv[0] = bf16_lo(x); vv[1] = bf16_hi(x);
        }
      } else if constexpr (FMT == kFP8Token) {
        const char* vrow = vbase + (long long)tt * D + lane * DPL;
        if constexpr (DPL == 4) {
          const uint32_t x = ld_nc_u32(vrow);
          const float2 a = e4m3x2_to_float2(x & 0xffff), c = e4m3x2_to_float2(x >> 16);
          vv[0] = a.x; vv[1] = a.y; vv[2] = c.x; vv[3] = c.y;
        } else {
          const uint16_t x = *reinterpret_cast<const uint16_t*>(vrow);
          const float2 a = e4m3x2_to_float2(x);
          vv[0] = a.x; vv[1] = a.y;
        }
      } else {
        const char* vrow = vbase + (long long)tt * (D / 2) + lane * DPL / 2;
        const uint32_t mm = ld_nc_u32(p.vm + blk * p.mblk_stride + kvh * p.mhead_stride +
                                      ((long long)tt * (D / kGroup) + (lane * DPL) / kGroup) * 4);
        const float sc = half_bits_to_float(mm & 0xffff), zp = half_bits_to_float(mm >> 16);
        if constexpr (DPL == 4) {
          const uint16_t x = *reinterpret_cast<const uint16_t*>(vrow);
#pragma unroll
          for (int j = 0; j < 4; ++j) vv[j] = float((x >> (4 * j)) & 0xf) * sc + zp;
        } else {
          const uint8_t x = *reinterpret_cast<const uint8_t*>(vrow);
          vv[0] = float(x & 0xf) * sc + zp;
          vv[1] = float(x >> 4) * sc + zp;
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[g][j] += pv[g] * vv[j];
    }
    __syncwarp();
  }

  // ---- merge the 4 warps
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float lw = warp_sum(l[g]);
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
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = (wm[w][g] == -FLT_MAX) ? 0.f : exp2f(wm[w][g] - M);
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

template <int D>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                      __nv_bfloat16* __restrict__ out, int S) {
  const long long bh = blockIdx.x;
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

// ------------------------------------------------------------------------------- host
template <int D, int FMT>
static void launch_g(int G, dim3 grid, const DecodeParams& p, cudaStream_t st) {
  switch (G) {
    case 1: decode_attn_kernel<D, 1, FMT><<<grid, 128, 0, st>>>(p); break;
    case 2: decode_attn_kernel<D, 2, FMT><<<grid, 128, 0, st>>>(p); break;
    case 4: decode_attn_kernel<D, 4, FMT><<<grid, 128, 0, st>>>(p); break;
    case 8: decode_attn_kernel<D, 8, FMT><<<grid, 128, 0, st>>>(p); break;
    default: TORCH_CHECK(false, "decode_attention: GQA group ", G, " unsupported");
  }
}

// Chooses the number of KV splits so batch x kv_heads x splits fills the GPU.
int64_t decode_num_splits(int64_t batch, int64_t kv_heads, int64_t max_pages, int64_t sms) {
  const int64_t base = std::max<int64_t>(1, batch * kv_heads);
  const int64_t target = sms * 4;  // ~4 resident CTAs per SM
  int64_t s = (target + base - 1) / base;
  s = std::min<int64_t>(s, std::max<int64_t>(1, max_pages / 4));  // >= 4 pages per split
  return std::max<int64_t>(1, std::min<int64_t>(s, 64));
}

// q [B,Hq,D] bf16; k/v: page data of one layer as raw addresses with strides; meta
// addresses (0 for bf16); block_table [B, max_blocks] int32; seq_lens [B] int32.
// part_o / part_lse: fp32 scratch of [B,Hq,S,D] / [B,Hq,S] (ignored when S == 1).
void decode_attention(torch::Tensor q, int64_t k, int64_t v, int64_t km, int64_t vm, int64_t blk_stride,
                      int64_t head_stride, int64_t mblk_stride, int64_t mhead_stride, int64_t fmt,
                      torch::Tensor block_table, torch::Tensor seq_lens, int64_t Hkv, double scale,
                      int64_t num_splits, int64_t max_pages, torch::Tensor out, torch::Tensor part_o,
                      torch::Tensor part_lse) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.is_contiguous(), "q must be contiguous bf16");
  TORCH_CHECK(q.dim() == 3, "q must be [B, Hq, D]");
  const int B = q.size(0), Hq = q.size(1), D = q.size(2);
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && block_table.stride(1) == 1, "block_table int32 rows");
  TORCH_CHECK(seq_lens.scalar_type() == torch::kInt32, "seq_lens int32");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous(), "out must be contiguous bf16");
  const int S = static_cast<int>(std::max<int64_t>(1, num_splits));
  if (S > 1) {
    TORCH_CHECK(part_o.numel() >= (int64_t)B * Hq * S * D && part_lse.numel() >= (int64_t)B * Hq * S,
                "split scratch too small");
  }
  DecodeParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const char*>(k);
  p.v = reinterpret_cast<const char*>(v);
  p.km = reinterpret_cast<const char*>(km);
  p.vm = reinterpret_cast<const char*>(vm);
  p.blk_stride = blk_stride;
  p.head_stride = head_stride;
  p.mblk_stride = mblk_stride;
  p.mhead_stride = mhead_stride;
  p.block_table = block_table.data_ptr<int>();
  p.bt_stride = block_table.stride(0);
  p.seq_lens = seq_lens.data_ptr<int>();
  p.Hq = Hq;
  p.Hkv = static_cast<int>(Hkv);
  p.pages_per_split = static_cast<int>((max_pages + S - 1) / S);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.part_o = S > 1 ? part_o.data_ptr<float>() : nullptr;
  p.part_lse = S > 1 ? part_lse.data_ptr<float>() : nullptr;
  const int G = Hq / static_cast<int>(Hkv);
  dim3 grid(S, Hkv, B);
  auto st = at::cuda::getCurrentCUDAStream();
  if (D == 128) {
    if (fmt == kBF16) launch_g<128, kBF16>(G, grid, p, st);
    else if (fmt == kFP8Token) launch_g<128, kFP8Token>(G, grid, p, st);
    else if (fmt == kINT4G64) launch_g<128, kINT4G64>(G, grid, p, st);
    else TORCH_CHECK(false, "decode_attention: unsupported cache format ", fmt);
  } else if (D == 64) {
    if (fmt == kBF16) launch_g<64, kBF16>(G, grid, p, st);
    else if (fmt == kFP8Token) launch_g<64, kFP8Token>(G, grid, p, st);
    else if (fmt == kINT4G64) launch_g<64, kINT4G64>(G, grid, p, st);
    else TORCH_CHECK(false, "decode_attention: unsupported cache format ", fmt);
  } else {
    TORCH_CHECK(false, "decode_attention: head_dim must be 64 or 128");
  }
  AXR_CHECK_CUDA(cudaGetLastError());
  if (S > 1) {
    if (D == 128) decode_combine_kernel<128><<<B * Hq, 128, 0, st>>>(p.part_o, p.part_lse, p.out, S);
    else decode_combine_kernel<64><<<B * Hq, 64, 0, st>>>(p.part_o, p.part_lse, p.out, S);
    AXR_CHECK_CUDA(cudaGetLastError());
  }
}

}  // namespace axr
