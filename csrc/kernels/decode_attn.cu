// Split-KV flash-decode over the paged KV cache, reading bf16, FP8 (per-token
// scaled) or INT4 g64 (asymmetric) pages directly — the compressed pages are never
// expanded into a bf16 copy.
//
// Reference counterparts: the FP8/INT4 decode kernels fp8_decode_attention.cu:85-201
// and int4_decode_attention.cu:39-177 (contiguous caches, one CTA per (batch, head),
// never wired in) and the SDPA fallback kernels/dispatch.py:117-152.
//
// Two kernels: decode_tc_kernel (tensor cores, head_dim 128, described below) and
// decode_attn_kernel (CUDA cores, head_dim 64). For the latter:
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
#include <cstdlib>

#include "attn_combine.cuh"
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
  // Shared-prefix decode: sequence b attends only to its pages [page_start[b], ...) here
  // (the shared prefix before them is attended by the grouped pass), and the result is
  // always written as partials for the merge. nullptr: every page from 0.
  const int* page_start;
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

  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const int S = gridDim.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq_len = p.seq_lens[b];
  const int n_pages = (seq_len + kPage - 1) / kPage;
  const int pg0 = (p.page_start != nullptr ? p.page_start[b] : 0) + split * p.pages_per_split;
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
    if (S == 1 && p.page_start == nullptr) {
      p.out[((long long)b * p.Hq + hq) * D + d] = __float2bfloat16(o);
    } else {
      const long long base = ((long long)b * p.Hq + hq) * S + split;
      p.part_o[base * D + d] = o;
      if (d == 0) p.part_lse[base] = L > 0.f ? M + log2f(L) : -FLT_MAX;
    }
  }
}


// ======================================================================================
// Tensor-core split-KV decode (head_dim 128): the kernel every D=128 call uses.
//
// A warp owns a stream of pages (pages pg0+warp, pg0+warp+4, ...) and pipelines them
// through a private STAGES-deep ring of shared-memory buffers filled by cp.async, so
// the loads of the next pages are in flight while the current page is computed.
// Per page (16 tokens) the warp runs two warp-level MMAs (m16n8k16, f32 accumulate):
//   S^T[16 tok x 8 heads]  = K[16 x 128] . Q^T[128 x 8]     (GQA heads padded to 8)
//   O^T[128 x 8 heads]    += V^T[128 x 16] . P^T[16 x 8]
// The head_dim axis of the first MMA is permuted (any permutation applied to both K
// and Q leaves QK^T unchanged) so each lane's K fragment is 16 consecutive dims of one
// 64-dim group, read with 128-bit shared loads, and each MMA k-step stays inside one
// group -- which lets INT4 apply its per-group scale/zero to partial accumulators.
// bf16 pages run bf16 MMAs; FP8 and INT4 pages run f16 MMAs on the exact codes (e4m3
// and 0..15 are exact in f16) with the per-token scales applied to the scores, and
// their V page is dequantised into an f16 tile for the ldmatrix.trans PV operand.
// ======================================================================================
constexpr float kDecodeRescaleLog2 = 8.f;

template <int FMT>
struct TcCfg {
  static constexpr int KB = FMT == kBF16 ? 4096 : (FMT == kFP8Token ? 2048 : 1024);  // K (=V) unit bytes
  static constexpr int MB = FMT == kBF16 ? 0 : (FMT == kFP8Token ? 64 : 128);        // meta bytes per unit
  static constexpr int STAGE = 2 * KB + 2 * MB;
  static constexpr int STAGES = FMT == kBF16 ? 3 : 4;
  static constexpr int VT = FMT == kBF16 ? 0 : 4096;  // f16 V tile (the codes as f16)
  static constexpr int PT = FMT == kINT4G64 ? 512 : 256;  // P^T tile(s): INT4 one per 64-dim group
  static constexpr int WARP = STAGES * STAGE + VT + PT;
  static constexpr int SMEM = 4 * WARP;
};

// byte offset of 16B chunk `c` of K row `r` in the LDS-friendly swizzle
template <int FMT>
__device__ __forceinline__ int ksw(int r, int c) {
  if constexpr (FMT == kBF16) return r * 256 + ((c ^ (r & 1)) << 4);
  else if constexpr (FMT == kFP8Token) return r * 128 + ((c ^ ((r & 1) << 2)) << 4);
  else return r * 64 + ((c ^ (((r >> 1) & 1) << 1)) << 4);
}
// ldmatrix-friendly swizzle of a [16 tok][128 dims] 16-bit tile
__device__ __forceinline__ int vsw(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, bool f16) {
  if (f16) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t fp8x2_h2(uint32_t two_codes) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two_codes & 0xffff), __NV_E4M3);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Nibble K (0..3) of both 16-bit halves of `word` -> f16x2 (1024 + n_lo, 1024 + n_hi): a
// shift and one and-or. The halves hold dims K and K + 4 of the word's 8 dims (byte j
// holds dims 2j, 2j+1), so a word yields the pairs (0,4) (1,5) (2,6) (3,7). For K the
// 1024 offset is folded into the zero point: a*(1024 + n) + (z - 1024 a) = a*n + z.
template <int K>
__device__ __forceinline__ uint32_t nib_sh(uint32_t word) {
  return ((word >> (4 * K)) & 0x000F000Fu) | 0x64006400u;
}
// As nib_sh, minus the offset: the exact integers n (one more f16x2 subtraction). The V
// operand takes these, since its scale is folded into P in f16 and an offset of 1024
// would cancel against that rounding.
template <int K>
__device__ __forceinline__ uint32_t nib_sh_exact(uint32_t word) {
  uint32_t w = nib_sh<K>(word);
  __half2 h = __hsub2(*reinterpret_cast<__half2*>(&w), __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int FMT>
__device__ __forceinline__ void tc_issue_page(const DecodeParams& p, int blk, int kvh, char* st, int lane) {
  using C = TcCfg<FMT>;
  const char* ku = p.k + blk * p.blk_stride + kvh * p.head_stride;
  const char* vu = p.v + blk * p.blk_stride + kvh * p.head_stride;
  char* sk = st;
  char* sv = st + C::KB;
#pragma unroll
  for (int i = 0; i < C::KB / 16 / 32; ++i) {
    const int c = lane + i * 32;
    if constexpr (FMT == kBF16) {
      const int r = c >> 4, cc = c & 15;
      cp_async16(sk + ksw<FMT>(r, cc), ku + c * 16);
      cp_async16(sv + vsw(r, cc), vu + c * 16);
    } else if constexpr (FMT == kFP8Token) {
      const int r = c >> 3, cc = c & 7;
      cp_async16(sk + ksw<FMT>(r, cc), ku + c * 16);
      cp_async16(sv + c * 16, vu + c * 16);
    } else {
      const int r = c >> 2, cc = c & 3;
      cp_async16(sk + ksw<FMT>(r, cc), ku + c * 16);
      cp_async16(sv + c * 16, vu + c * 16);
    }
  }
  if constexpr (FMT != kBF16) {
    const char* km = p.km + blk * p.mblk_stride + kvh * p.mhead_stride;
    const char* vm = p.vm + blk * p.mblk_stride + kvh * p.mhead_stride;
    constexpr int MC = C::MB / 16;  // 4 (fp8) or 8 (int4) chunks per meta unit
    if (lane < MC) cp_async16(st + 2 * C::KB + lane * 16, km + lane * 16);
    else if (lane < 2 * MC) cp_async16(st + 2 * C::KB + C::MB + (lane - MC) * 16, vm + (lane - MC) * 16);
  }
}

template <int FMT, int G>
__global__ void __launch_bounds__(128) decode_tc_kernel(DecodeParams p) {
  using C = TcCfg<FMT>;
  constexpr bool F16 = FMT != kBF16;
  extern __shared__ __align__(128) char smem[];
  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z, S = gridDim.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  char* wbase = smem + warp * C::WARP;
  char* vtile = wbase + C::STAGES * C::STAGE;
  uint16_t* pt = reinterpret_cast<uint16_t*>(vtile + C::VT);  // P^T [8 heads][16 tok]

  const int seq_len = p.seq_lens[b];
  const int n_pages = (seq_len + kPage - 1) / kPage;
  const int pg0 = (p.page_start != nullptr ? p.page_start[b] : 0) + split * p.pages_per_split;
  const int pg1 = min(n_pages, pg0 + p.pages_per_split);
  const int my_n = pg1 > pg0 + warp ? (pg1 - pg0 - warp + 3) / 4 : 0;
  const int* bt = p.block_table + (long long)b * p.bt_stride;

  // Programmatic dependent launch: seq_lens, the block table and every page but the
  // sequence's last two were written before this forward began, so the first pages of
  // the ring are fetched before waiting for the kernel before (the projection that
  // writes q and the newest KV row); q and the newest pages are read after the wait.
  pdl_trigger();
  const int stable_pages = max(0, (seq_len - 1) / kPage - 1);
  const bool early = pg0 + warp + 4 * (C::STAGES - 2) < stable_pages;
  auto prologue = [&]() {
#pragma unroll
    for (int s = 0; s < C::STAGES - 1; ++s) {
      if (s < my_n) tc_issue_page<FMT>(p, bt[pg0 + warp + 4 * s], kvh, wbase + s * C::STAGE, lane);
      cp_async_commit();
    }
  };
  if (early) prologue();
  pdl_wait();
  if (!early) prologue();

  // Q^T fragments (B operand), dims permuted: k-step kk, lane t -> dims base..base+3
  uint32_t qb[8][2];
  float qsum[2] = {0.f, 0.f};  // INT4: sum of this lane's q dims per group, head g
  {
    const __nv_bfloat16* qrow = p.q + ((long long)b * p.Hq + kvh * G + (g < G ? g : 0)) * 128;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      // dims of this lane's k-step: 4 consecutive; INT4 takes the nib_sh pairs
      // (d, d+4) and (d+1, d+5) with d = 8 * ((kk & 3) >> 1) + 2 * (kk & 1)
      int dd[4];
      if constexpr (FMT == kINT4G64) {
        const int d0 = (kk >> 2) * 64 + t * 16 + ((kk & 3) >> 1) * 8 + (kk & 1) * 2;
        dd[0] = d0; dd[1] = d0 + 4; dd[2] = d0 + 1; dd[3] = d0 + 5;
      } else {
        const int base = (kk >> 2) * 64 + t * 16 + (kk & 3) * 4;
        dd[0] = base; dd[1] = base + 1; dd[2] = base + 2; dd[3] = base + 3;
      }
      float f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) f[e] = g < G ? __bfloat162float(qrow[dd[e]]) * p.scale_log2 : 0.f;
      if constexpr (F16) {
        qb[kk][0] = pack_h2(f[0], f[1]);
        qb[kk][1] = pack_h2(f[2], f[3]);
        const __half2 h0 = *reinterpret_cast<__half2*>(&qb[kk][0]);
        const __half2 h1 = *reinterpret_cast<__half2*>(&qb[kk][1]);
        qsum[kk >> 2] += __low2float(h0) + __high2float(h0) + __low2float(h1) + __high2float(h1);
      } else {
        qb[kk][0] = pack_bf16x2(f[0], f[1]);
        qb[kk][1] = pack_bf16x2(f[2], f[3]);
      }
    }
  }
  float qs_col[2][2];  // [group][j]: q-sum of head 2t+j (INT4 zero-point term)
  if constexpr (FMT == kINT4G64) {
#pragma unroll
    for (int gr = 0; gr < 2; ++gr) {
      qsum[gr] += __shfl_xor_sync(0xffffffffu, qsum[gr], 1);
      qsum[gr] += __shfl_xor_sync(0xffffffffu, qsum[gr], 2);
#pragma unroll
      for (int j = 0; j < 2; ++j) qs_col[gr][j] = __shfl_sync(0xffffffffu, qsum[gr], 4 * (2 * t + j));
    }
  }

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  // INT4: sum over tokens of p * z per (head 2t+j, group); added to O at the end
  float zacc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  float m[2] = {-FLT_MAX, -FLT_MAX}, l[2] = {0.f, 0.f};

  for (int i = 0; i < my_n; ++i) {
    {
      const int ni = i + C::STAGES - 1;
      if (ni < my_n) tc_issue_page<FMT>(p, bt[pg0 + warp + 4 * ni], kvh, wbase + (ni % C::STAGES) * C::STAGE, lane);
      cp_async_commit();
    }
    cp_async_wait<C::STAGES - 1>();
    __syncwarp();
    const char* st = wbase + (i % C::STAGES) * C::STAGE;
    const char* sk = st;
    const int pg = pg0 + warp + 4 * i;

    // ---- S^T = K . Q^T
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int gr = 0; gr < 2; ++gr) {
      uint32_t ka[2][8];  // [row g | g+8][4 k-steps x (a-lo, a-hi)]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = g + 8 * h;
        if constexpr (FMT == kBF16) {
          const uint4 x = *reinterpret_cast<const uint4*>(sk + ksw<FMT>(r, gr * 8 + t * 2));
          const uint4 y = *reinterpret_cast<const uint4*>(sk + ksw<FMT>(r, gr * 8 + t * 2 + 1));
          ka[h][0] = x.x; ka[h][1] = x.y; ka[h][2] = x.z; ka[h][3] = x.w;
          ka[h][4] = y.x; ka[h][5] = y.y; ka[h][6] = y.z; ka[h][7] = y.w;
        } else if constexpr (FMT == kFP8Token) {
          const uint4 x = *reinterpret_cast<const uint4*>(sk + ksw<FMT>(r, gr * 4 + t));
          const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            ka[h][2 * q] = fp8x2_h2(w[q]);
            ka[h][2 * q + 1] = fp8x2_h2(w[q] >> 16);
          }
        } else {
          const uint2 x = *reinterpret_cast<const uint2*>(sk + ksw<FMT>(r, gr * 2 + (t >> 1)) + (t & 1) * 8);
          ka[h][0] = nib_sh<0>(x.x);
          ka[h][1] = nib_sh<1>(x.x);
          ka[h][2] = nib_sh<2>(x.x);
          ka[h][3] = nib_sh<3>(x.x);
          ka[h][4] = nib_sh<0>(x.y);
          ka[h][5] = nib_sh<1>(x.y);
          ka[h][6] = nib_sh<2>(x.y);
          ka[h][7] = nib_sh<3>(x.y);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int kk = gr * 4 + q;
        if constexpr (FMT == kINT4G64) {
          if (gr == 0) mma16816(s0, ka[0][2 * q], ka[1][2 * q], ka[0][2 * q + 1], ka[1][2 * q + 1], qb[kk][0], qb[kk][1], true);
          else mma16816(s1, ka[0][2 * q], ka[1][2 * q], ka[0][2 * q + 1], ka[1][2 * q + 1], qb[kk][0], qb[kk][1], true);
        } else {
          mma16816(s0, ka[0][2 * q], ka[1][2 * q], ka[0][2 * q + 1], ka[1][2 * q + 1], qb[kk][0], qb[kk][1], F16);
        }
      }
    }
    // ---- per-token scales, masking
    const int tok0 = pg * kPage + g, tok1 = tok0 + 8;
    float sc[4];
    if constexpr (FMT == kBF16) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[e] = s0[e];
    } else if constexpr (FMT == kFP8Token) {
      const float* ks = reinterpret_cast<const float*>(st + 2 * C::KB);
      const float k0 = ks[g], k1 = ks[g + 8];
      sc[0] = s0[0] * k0; sc[1] = s0[1] * k0; sc[2] = s0[2] * k1; sc[3] = s0[3] * k1;
    } else {
      const uint32_t* km = reinterpret_cast<const uint32_t*>(st + 2 * C::KB);  // [tok][group] (scale, zero)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t m0 = km[(g + 8 * h) * 2 + 0], m1 = km[(g + 8 * h) * 2 + 1];
        const float a0 = half_bits_to_float(m0 & 0xffff), z0 = half_bits_to_float(m0 >> 16) - 1024.f * a0;
        const float a1 = half_bits_to_float(m1 & 0xffff), z1 = half_bits_to_float(m1 >> 16) - 1024.f * a1;
#pragma unroll
        for (int j = 0; j < 2; ++j)
          sc[2 * h + j] = s0[2 * h + j] * a0 + qs_col[0][j] * z0 + s1[2 * h + j] * a1 + qs_col[1][j] * z1;
      }
    }
    if (tok0 >= seq_len) { sc[0] = -FLT_MAX; sc[1] = -FLT_MAX; }
    if (tok1 >= seq_len) { sc[2] = -FLT_MAX; sc[3] = -FLT_MAX; }
    // ---- online softmax (columns = heads 2t, 2t+1). The reference maximum only moves
    // when a page's maximum exceeds it by more than 2^8 (log2 units), so p <= 256 and the
    // rescale of O -- 34 multiplies per lane -- is skipped on almost every page.
    float pv[4], alpha[2];
    bool resc = false;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float mx = fmaxf(sc[j], sc[2 + j]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const bool up = mx > m[j] + kDecodeRescaleLog2;
      const float mn = up ? mx : m[j];
      alpha[j] = up ? exp2f(m[j] - mn) : 1.f;
      resc |= up;
      m[j] = mn;
      pv[j] = sc[j] == -FLT_MAX ? 0.f : exp2f(sc[j] - mn);
      pv[2 + j] = sc[2 + j] == -FLT_MAX ? 0.f : exp2f(sc[2 + j] - mn);
      l[j] = l[j] * alpha[j] + pv[j] + pv[2 + j];
    }
    if (__any_sync(0xffffffffu, resc)) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[mt][j] *= alpha[j];
          o[mt][2 + j] *= alpha[j];
        }
        if constexpr (FMT == kINT4G64) {
          zacc[j][0] *= alpha[j];
          zacc[j][1] *= alpha[j];
        }
      }
    }
    // ---- P^T to shared (for the B operand). FP8 / INT4: the V tile holds the raw codes,
    // so each token's V scale is folded into its P entry (INT4: one P^T per 64-dim group,
    // and the zero point of the group goes to zacc).
    if constexpr (FMT == kINT4G64) {
      const uint32_t* vmeta = reinterpret_cast<const uint32_t*>(st + 2 * C::KB + C::MB);  // [tok][group]
      float va[2][2], vz[2][2];  // [token g | g+8][group]
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int gr = 0; gr < 2; ++gr) {
          const uint32_t mm = vmeta[(g + 8 * h) * 2 + gr];
          va[h][gr] = half_bits_to_float(mm & 0xffff);
          vz[h][gr] = half_bits_to_float(mm >> 16);
        }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int hcol = 2 * t + j;
#pragma unroll
        for (int gr = 0; gr < 2; ++gr) {
          pt[gr * 128 + hcol * 16 + g] = __half_as_ushort(__float2half_rn(pv[j] * va[0][gr]));
          pt[gr * 128 + hcol * 16 + g + 8] = __half_as_ushort(__float2half_rn(pv[2 + j] * va[1][gr]));
          zacc[j][gr] += pv[j] * vz[0][gr] + pv[2 + j] * vz[1][gr];
        }
      }
    } else {
      float vs0 = 1.f, vs1 = 1.f;
      if constexpr (FMT == kFP8Token) {
        const float* vsc = reinterpret_cast<const float*>(st + 2 * C::KB + C::MB);
        vs0 = vsc[g];
        vs1 = vsc[g + 8];
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int hcol = 2 * t + j;
        uint16_t a, c;
        if constexpr (F16) {
          a = __half_as_ushort(__float2half_rn(pv[j] * vs0));
          c = __half_as_ushort(__float2half_rn(pv[2 + j] * vs1));
        } else {
          a = __bfloat16_as_ushort(__float2bfloat16(pv[j]));
          c = __bfloat16_as_ushort(__float2bfloat16(pv[2 + j]));
        }
        pt[hcol * 16 + g] = a;
        pt[hcol * 16 + g + 8] = c;
      }
    }
    // ---- V tile (FP8 / INT4: dequantise into the f16 ldmatrix tile)
    const char* vt;
    if constexpr (FMT == kBF16) {
      vt = st + C::KB;
    } else {
      const char* sv = st + C::KB;
      const int cc = lane & 15;
#pragma unroll
      for (int i2 = 0; i2 < 8; ++i2) {
        const int r = (lane >> 4) + 2 * i2;
        uint32_t h4[4];
        if constexpr (FMT == kFP8Token) {  // e4m3 codes are exact in f16
          const uint2 x = *reinterpret_cast<const uint2*>(sv + r * 128 + cc * 8);
          h4[0] = fp8x2_h2(x.x);
          h4[1] = fp8x2_h2(x.x >> 16);
          h4[2] = fp8x2_h2(x.y);
          h4[3] = fp8x2_h2(x.y >> 16);
        } else {  // codes 0..15; tile columns of each 8-dim chunk hold dims 0,4,1,5,2,6,3,7
          const uint32_t x = *reinterpret_cast<const uint32_t*>(sv + r * 64 + cc * 4);
          h4[0] = nib_sh_exact<0>(x);
          h4[1] = nib_sh_exact<1>(x);
          h4[2] = nib_sh_exact<2>(x);
          h4[3] = nib_sh_exact<3>(x);
        }
        *reinterpret_cast<uint4*>(vtile + vsw(r, cc)) = make_uint4(h4[0], h4[1], h4[2], h4[3]);
      }
      vt = vtile;
    }
    __syncwarp();
    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(pt + g * 16 + 2 * t);
    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(pt + g * 16 + 2 * t + 8);
    uint32_t c0 = b0, c1 = b1;  // group 1 (dims 64-127) of INT4
    if constexpr (FMT == kINT4G64) {
      c0 = *reinterpret_cast<const uint32_t*>(pt + 128 + g * 16 + 2 * t);
      c1 = *reinterpret_cast<const uint32_t*>(pt + 128 + g * 16 + 2 * t + 8);
    }
    // ---- O^T += V^T . P^T
    {
      const uint32_t vbase = static_cast<uint32_t>(__cvta_generic_to_shared(vt));
      const int mi = lane >> 3, r = (mi >> 1) * 8 + (lane & 7);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
                     : "r"(vbase + vsw(r, 2 * mt + (mi & 1))));
        mma16816(o[mt], a0, a1, a2, a3, mt < 4 ? b0 : c0, mt < 4 ? b1 : c1, F16);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();

  // ---- merge warps (reuses the stage buffers)
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    l[j] += __shfl_xor_sync(0xffffffffu, l[j], 4);
    l[j] += __shfl_xor_sync(0xffffffffu, l[j], 8);
    l[j] += __shfl_xor_sync(0xffffffffu, l[j], 16);
  }
  __syncthreads();
  float* wm = reinterpret_cast<float*>(smem);          // [4][8]
  float* wl = wm + 32;                                 // [4][8]
  float* wacc = wl + 32;                               // [4][8][128]
  if (g == 0) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      wm[warp * 8 + 2 * t + j] = m[j];
      wl[warp * 8 + 2 * t + j] = l[j];
    }
  }
  if constexpr (FMT == kINT4G64) {
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int gr = 0; gr < 2; ++gr) {
        zacc[j][gr] += __shfl_xor_sync(0xffffffffu, zacc[j][gr], 4);
        zacc[j][gr] += __shfl_xor_sync(0xffffffffu, zacc[j][gr], 8);
        zacc[j][gr] += __shfl_xor_sync(0xffffffffu, zacc[j][gr], 16);
      }
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int head = 2 * t + (e & 1);
      int dim = mt * 16 + g + (e >> 1) * 8;
      float val = o[mt][e];
      if constexpr (FMT == kINT4G64) {
        dim = (dim & ~7) + ((g >> 1) | ((g & 1) << 2));  // tile column -> dim (nib_sh pairs)
        val += zacc[e & 1][mt >> 2];
      }
      wacc[(warp * 8 + head) * 128 + dim] = val;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * 128; i += blockDim.x) {
    const int hh = i / 128, d = i % 128;
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w * 8 + hh]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = wm[w * 8 + hh];
      const float f = mw == -FLT_MAX ? 0.f : exp2f(mw - M);
      L += wl[w * 8 + hh] * f;
      O += wacc[(w * 8 + hh) * 128 + d] * f;
    }
    const int hq = kvh * G + hh;
    const float ov = L > 0.f ? O / L : 0.f;
    if (S == 1 && p.page_start == nullptr) {
      p.out[((long long)b * p.Hq + hq) * 128 + d] = __float2bfloat16(ov);
    } else {
      const long long base = ((long long)b * p.Hq + hq) * S + split;
      p.part_o[base * 128 + d] = ov;
      if (d == 0) p.part_lse[base] = L > 0.f ? M + log2f(L) : -FLT_MAX;
    }
  }
}

template <int FMT>
static void launch_tc(int G, dim3 grid, const DecodeParams& p, cudaStream_t st) {
  constexpr int smem = TcCfg<FMT>::SMEM;
  auto go = [&](auto kern) {
    AXR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    AXR_CHECK_CUDA(launch_pdl(kern, grid, dim3(128), smem, st, p));
  };
  switch (G) {
    case 1: go(decode_tc_kernel<FMT, 1>); break;
    case 2: go(decode_tc_kernel<FMT, 2>); break;
    case 4: go(decode_tc_kernel<FMT, 4>); break;
    case 8: go(decode_tc_kernel<FMT, 8>); break;
    default: TORCH_CHECK(false, "decode_attention: GQA group ", G, " unsupported");
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

// Chooses the number of KV splits so that batch x kv_heads x splits fills the GPU in
// whole waves: with `fmt` given, a wave is SMs x the CTAs of that page format's kernel
// that fit one SM (shared memory bound); the split count in [fill/2, 2*fill] with the
// best last-wave occupancy wins (fewest splits on ties), keeping >= 4 pages per split.
int64_t decode_num_splits(int64_t batch, int64_t kv_heads, int64_t max_pages, int64_t sms, int64_t fmt) {
  // AXR_DECODE_SPLITS=n fixes the count (for measurements)
  static const int64_t forced = [] {
    const char* e = getenv("AXR_DECODE_SPLITS");
    return e ? static_cast<int64_t>(atoi(e)) : 0;
  }();
  const int64_t s_max = std::max<int64_t>(1, std::min<int64_t>(64, max_pages / 4));
  if (forced > 0) return std::min(forced, s_max);
  const int64_t base = std::max<int64_t>(1, batch * kv_heads);
  int64_t per_sm = 4;
  if (fmt == kBF16) per_sm = (227 * 1024) / TcCfg<kBF16>::SMEM;
  else if (fmt == kFP8Token) per_sm = (227 * 1024) / TcCfg<kFP8Token>::SMEM;
  else if (fmt == kINT4G64) per_sm = (227 * 1024) / TcCfg<kINT4G64>::SMEM;
  const int64_t cap = sms * std::max<int64_t>(1, std::min<int64_t>(per_sm, 16));  // resident CTAs
  // the fewest slices with the best wave fill: every extra slice costs partials and a
  // combine (B = 32 x 8448 tokens, bf16: 1 slice 0.127 ms per layer, 2: 0.137, 5: 0.149)
  const int64_t fill = (cap + base - 1) / base;
  int64_t best = 1;
  double best_eff = -1.0;
  for (int64_t s = std::max<int64_t>(1, fill / 2); s <= std::min<int64_t>(s_max, 2 * fill); ++s) {
    const int64_t ctas = base * s;
    const int64_t waves = (ctas + cap - 1) / cap;
    const double eff = static_cast<double>(ctas) / static_cast<double>(waves * cap);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = s;
    }
  }
  return std::max<int64_t>(1, std::min<int64_t>(best, s_max));
}

// q [B,Hq,D] bf16; k/v: page data of one layer as raw addresses with strides; meta
// addresses (0 for bf16); block_table [B, max_blocks] int32; seq_lens [B] int32.
// part_o / part_lse: fp32 scratch of [B,Hq,S,D] / [B,Hq,S] (ignored when S == 1).
void decode_attention(torch::Tensor q, int64_t k, int64_t v, int64_t km, int64_t vm, int64_t blk_stride,
                      int64_t head_stride, int64_t mblk_stride, int64_t mhead_stride, int64_t fmt,
                      torch::Tensor block_table, torch::Tensor seq_lens, int64_t Hkv, double scale,
                      int64_t num_splits, int64_t max_pages, torch::Tensor out, torch::Tensor part_o,
                      torch::Tensor part_lse, c10::optional<torch::Tensor> page_start,
                      c10::optional<torch::Tensor> part_o2, c10::optional<torch::Tensor> part_lse2,
                      c10::optional<torch::Tensor> row_of, int64_t S2) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.is_contiguous(), "q must be contiguous bf16");
  TORCH_CHECK(q.dim() == 3, "q must be [B, Hq, D]");
  const int B = q.size(0), Hq = q.size(1), D = q.size(2);
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && block_table.stride(1) == 1, "block_table int32 rows");
  TORCH_CHECK(seq_lens.scalar_type() == torch::kInt32, "seq_lens int32");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous(), "out must be contiguous bf16");
  const int S = static_cast<int>(std::max<int64_t>(1, num_splits));
  const bool cascade = page_start.has_value();
  if (S > 1 || cascade) {
    TORCH_CHECK(part_o.numel() >= (int64_t)B * Hq * S * D && part_lse.numel() >= (int64_t)B * Hq * S,
                "split scratch too small");
  }
  if (cascade) {
    TORCH_CHECK(page_start->scalar_type() == torch::kInt32 && page_start->numel() >= B && row_of.has_value() &&
                    row_of->scalar_type() == torch::kInt32 && row_of->numel() >= B && part_o2.has_value() &&
                    part_lse2.has_value() && S2 >= 1,
                "decode_attention: shared-prefix inputs (page_start, row_of, shared partials)");
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
  p.part_o = S > 1 || cascade ? part_o.data_ptr<float>() : nullptr;
  p.part_lse = S > 1 || cascade ? part_lse.data_ptr<float>() : nullptr;
  p.page_start = cascade ? page_start->data_ptr<int>() : nullptr;
  const int G = Hq / static_cast<int>(Hkv);
  // KV-slice major: the first slice of every (sequence, KV head) starts together, so
  // sequences that share prefix pages read them at the same time (once from DRAM, the
  // rest from L2), and the later slices backfill SMs as earlier CTAs finish
  dim3 grid(Hkv, B, S);
  auto st = at::cuda::getCurrentCUDAStream();
  if (D == 128) {
    if (fmt == kBF16) launch_tc<kBF16>(G, grid, p, st);
    else if (fmt == kFP8Token) launch_tc<kFP8Token>(G, grid, p, st);
    else if (fmt == kINT4G64) launch_tc<kINT4G64>(G, grid, p, st);
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
  if (cascade) {
    TORCH_CHECK(D == 128, "shared-prefix decode: head_dim 128");
    AXR_CHECK_CUDA(launch_pdl(cascade_combine_kernel<128>, dim3(B * Hq), dim3(128), 0, st,
                              static_cast<const float*>(p.part_o), static_cast<const float*>(p.part_lse),
                              static_cast<int>(S), static_cast<const float*>(part_o2->data_ptr<float>()),
                              static_cast<const float*>(part_lse2->data_ptr<float>()), static_cast<int>(S2),
                              static_cast<const int*>(row_of->data_ptr<int>()), Hq, p.out));
  } else if (S > 1) {
    const float* po = p.part_o;
    const float* pl = p.part_lse;
    if (D == 128) AXR_CHECK_CUDA(launch_pdl(decode_combine_kernel<128>, dim3(B * Hq), dim3(128), 0, st, po, pl, p.out, S));
    else AXR_CHECK_CUDA(launch_pdl(decode_combine_kernel<64>, dim3(B * Hq), dim3(64), 0, st, po, pl, p.out, S));
  }
}

}  // namespace axr
