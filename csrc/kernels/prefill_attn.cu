// Causal prefill attention over the paged KV cache (varlen batch, GQA), written for
// the suffix-after-restore case: the query rows are the new tokens of each sequence
// and the keys/values are every cached token of that sequence (restored prefix pages
// plus the pages the new tokens were just written into).
//
// FlashAttention-2 dataflow on warp-level bf16 tensor-core MMA (m16n8k16): a CTA of 4
// warps owns 64 query rows of one head; KV tiles of 64 tokens (4 pages) are gathered
// from the block table into double-buffered, XOR-swizzled shared memory with
// cp.async (bf16 pages) or dequantised on the way in (FP8 / INT4 pages); S = QK^T and
// O += PV run from ldmatrix fragments with the online softmax in registers.
//
// Split-KV: when the (query tile, head, sequence) grid is too small to fill the GPU --
// a short suffix prefilled against a long restored prefix -- every CTA takes one slice
// of the KV tiles and writes a normalised partial output plus its log-sum-exp; a
// combine kernel merges the slices.
//
// Reference counterpart: the prefill attention inside llama.cpp / vLLM (library
// kernels the reference delegates to); the reference has no prefill kernel of its own.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cfloat>

#include "attn_combine.cuh"
#include "common.cuh"

namespace axr {

struct PrefillParams {
  const __nv_bfloat16* q;  // [T, Hq, D]
  __nv_bfloat16* out;      // [T, Hq, D]
  const char* k;
  const char* v;
  const char* km;
  const char* vm;
  long long blk_stride, head_stride, mblk_stride, mhead_stride;
  const int* block_table;
  int bt_stride;
  const int* cu_q;      // [B+1]
  const int* seq_lens;  // [B] total kv length (cached prefix + new tokens)
  int Hq, Hkv;
  float scale_log2;
  int num_splits;   // KV slices per (query tile, head, sequence); 1 = no split
  float* part_o;    // [T*Hq, S, D] normalised partial outputs (S > 1)
  float* part_lse;  // [T*Hq, S] log2-domain log-sum-exps (S > 1)
};

constexpr int BM = 64, BN = 64, D_ = 128;
constexpr int ROWB = D_ * 2;  // bytes per smem row

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset of a 16B chunk
  return row * ROWB + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Gather one 64-token KV tile (K or V) into swizzled smem.
template <int FMT>
__device__ __forceinline__ void load_kv_tile(const PrefillParams& p, const char* base, const char* mbase,
                                             const int* bt, int kvh, int n0, int kv_len, char* smem) {
  // 64 rows x 16 chunks = 1024 chunks, 8 per thread.
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = threadIdx.x + i * 128;
    const int row = idx >> 4, ch = idx & 15;
    const int tok = n0 + row;
    const bool valid = tok < kv_len;
    const int blk = valid ? bt[tok / kPage] : 0;
    const int r = tok % kPage;
    char* dst = smem + swz(row, ch);
    if constexpr (FMT == kBF16) {
      const char* src = base + blk * p.blk_stride + kvh * p.head_stride + (long long)r * D_ * 2 + ch * 16;
      cp_async16_zfill(dst, valid ? src : base, valid);
    } else {
      uint4 o = make_uint4(0, 0, 0, 0);
      if (valid) {
        const char* unit = base + blk * p.blk_stride + kvh * p.head_stride;
        const char* munit = mbase + blk * p.mblk_stride + kvh * p.mhead_stride;
        float f[8];
        if constexpr (FMT == kFP8Token) {
          const uint2 x = ld_nc_v2(unit + (long long)r * D_ + ch * 8);
          const float sc = *reinterpret_cast<const float*>(munit + r * 4);
          const float2 a = e4m3x2_to_float2(x.x & 0xffff), b = e4m3x2_to_float2(x.x >> 16);
          const float2 c = e4m3x2_to_float2(x.y & 0xffff), d = e4m3x2_to_float2(x.y >> 16);
          f[0] = a.x * sc; f[1] = a.y * sc; f[2] = b.x * sc; f[3] = b.y * sc;
          f[4] = c.x * sc; f[5] = c.y * sc; f[6] = d.x * sc; f[7] = d.y * sc;
        } else {
          const uint32_t x = ld_nc_u32(unit + (long long)r * (D_ / 2) + ch * 4);
          const uint32_t m = ld_nc_u32(munit + ((long long)r * (D_ / kGroup) + ch / 8) * 4);
          const float sc = half_bits_to_float(m & 0xffff), zp = half_bits_to_float(m >> 16);
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = float((x >> (4 * j)) & 0xf) * sc + zp;
        }
        o = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                       pack_bf16x2(f[6], f[7]));
      }
      *reinterpret_cast<uint4*>(dst) = o;
    }
  }
}

template <int FMT>
__global__ void __launch_bounds__(128, 2) prefill_attn_kernel(PrefillParams p) {
  extern __shared__ __align__(128) char smem[];
  char* sQ = smem;
  char* sK[2] = {smem + BM * ROWB, smem + BM * ROWB + 2 * BN * ROWB};
  char* sV[2] = {smem + BM * ROWB + BN * ROWB, smem + BM * ROWB + 3 * BN * ROWB};

  const int S = p.num_splits;
  const int tile_m = blockIdx.x, hq = blockIdx.y, b = blockIdx.z / S, split = blockIdx.z % S;
  const int q0 = p.cu_q[b], nq = p.cu_q[b + 1] - q0;
  if (tile_m * BM >= nq) return;
  const int kv_len = p.seq_lens[b];
  const int pos0 = kv_len - nq;  // absolute position of the first query row
  const int G = p.Hq / p.Hkv;
  const int kvh = hq / G;
  const int* bt = p.block_table + (long long)b * p.bt_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;

  // ---- Q tile -> smem
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = threadIdx.x + i * 128;
    const int row = idx >> 4, ch = idx & 15;
    const int qr = tile_m * BM + row;
    const bool valid = qr < nq;
    const char* src = reinterpret_cast<const char*>(p.q + ((long long)(q0 + (valid ? qr : 0)) * p.Hq + hq) * D_) + ch * 16;
    cp_async16_zfill(sQ + swz(row, ch), src, valid);
  }
  cp_async_commit();

  const int m_last = min(nq, (tile_m + 1) * BM) - 1;  // last valid q row of the tile
  const int kv_end = min(kv_len, pos0 + m_last + 1);
  const int n_all = (kv_end + BN - 1) / BN;
  const int per = (n_all + S - 1) / S;
  const int t_begin = split * per, t_end = min(n_all, t_begin + per);
  if (t_begin >= t_end) {  // this slice has no keys for the tile: mark its partials empty
    cp_async_wait<0>();
    for (int r = threadIdx.x; r < BM; r += blockDim.x) {
      const int qr = tile_m * BM + r;
      if (qr < nq) p.part_lse[((long long)(q0 + qr) * p.Hq + hq) * S + split] = -FLT_MAX;
    }
    return;
  }

  load_kv_tile<FMT>(p, p.k, p.km, bt, kvh, t_begin * BN, kv_len, sK[0]);
  load_kv_tile<FMT>(p, p.v, p.vm, bt, kvh, t_begin * BN, kv_len, sV[0]);
  cp_async_commit();

  cp_async_wait<1>();
  __syncthreads();
  uint32_t qf[8][4];
  {
    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));
    const int mi = lane >> 3, r = lane & 7;
    const int row = warp * 16 + r + (mi & 1) * 8;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int ch = kk * 2 + (mi >> 1);
      ldmatrix_x4(base + swz(row, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-FLT_MAX, -FLT_MAX}, lrow[2] = {0.f, 0.f};
  const int qabs0 = pos0 + tile_m * BM + warp * 16 + g;  // absolute position of row g
  const int qabs1 = qabs0 + 8;

  for (int it = t_begin; it < t_end; ++it) {
    const int buf = (it - t_begin) & 1;
    if (it + 1 < t_end) {
      load_kv_tile<FMT>(p, p.k, p.km, bt, kvh, (it + 1) * BN, kv_len, sK[buf ^ 1]);
      load_kv_tile<FMT>(p, p.v, p.vm, bt, kvh, (it + 1) * BN, kv_len, sV[buf ^ 1]);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    // ---- S = Q K^T  (16 rows x 64 cols per warp)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const uint32_t kb = static_cast<uint32_t>(__cvta_generic_to_shared(sK[buf]));
    {
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
          const int row = jp * 16 + (mi >> 1) * 8 + r;
          const int ch = kk * 2 + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kb + swz(row, ch), b0, b1, b2, b3);
          mma_bf16(s[2 * jp], qf[kk], b0, b1);
          mma_bf16(s[2 * jp + 1], qf[kk], b2, b3);
        }
      }
    }
    // ---- mask + online softmax
    const int n0 = it * BN;
    const bool need_mask = (n0 + BN - 1 > pos0 + tile_m * BM + warp * 16) || (n0 + BN > kv_len);
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * p.scale_log2;
        if (need_mask) {
          const int col = n0 + j * 8 + 2 * t4 + (e & 1);
          const int qa = (e < 2) ? qabs0 : qabs1;
          if (col > qa || col >= kv_len) x = -FLT_MAX;
        }
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      alpha[h] = exp2f(mrow[h] - mx[h]);
      mrow[h] = mx[h];
      lrow[h] *= alpha[h];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= alpha[0]; o[j][1] *= alpha[0];
      o[j][2] *= alpha[1]; o[j][3] *= alpha[1];
    }
    uint32_t pf[4][4];  // P as A fragments for the 4 k-steps of 16 tokens
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = (s[j][0] == -FLT_MAX) ? 0.f : exp2f(s[j][0] - mrow[0]);
      const float p1 = (s[j][1] == -FLT_MAX) ? 0.f : exp2f(s[j][1] - mrow[0]);
      const float p2 = (s[j][2] == -FLT_MAX) ? 0.f : exp2f(s[j][2] - mrow[1]);
      const float p3 = (s[j][3] == -FLT_MAX) ? 0.f : exp2f(s[j][3] - mrow[1]);
      lrow[0] += p0 + p1;
      lrow[1] += p2 + p3;
      const int ks = j >> 1;
      if ((j & 1) == 0) {
        pf[ks][0] = pack_bf16x2(p0, p1);
        pf[ks][1] = pack_bf16x2(p2, p3);
      } else {
        pf[ks][2] = pack_bf16x2(p0, p1);
        pf[ks][3] = pack_bf16x2(p2, p3);
      }
    }
    // ---- O += P V
    const uint32_t vb = static_cast<uint32_t>(__cvta_generic_to_shared(sV[buf]));
    {
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          const int row = ks * 16 + (mi & 1) * 8 + r;
          const int ch = dp * 2 + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_t(vb + swz(row, ch), b0, b1, b2, b3);
          mma_bf16(o[2 * dp], pf[ks], b0, b1);
          mma_bf16(o[2 * dp + 1], pf[ks], b2, b3);
        }
      }
    }
    __syncthreads();
  }

  // ---- finalize
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 1);
    lrow[h] += __shfl_xor_sync(0xffffffffu, lrow[h], 2);
  }
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f;
  const float inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
  const int r0 = tile_m * BM + warp * 16 + g, r1 = r0 + 8;
  if (S > 1) {
    const long long row0 = ((long long)(q0 + r0) * p.Hq + hq) * S + split;
    const long long row1 = ((long long)(q0 + r1) * p.Hq + hq) * S + split;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int col = j * 8 + 2 * t4;
      if (r0 < nq) *reinterpret_cast<float2*>(p.part_o + row0 * D_ + col) = make_float2(o[j][0] * inv0, o[j][1] * inv0);
      if (r1 < nq) *reinterpret_cast<float2*>(p.part_o + row1 * D_ + col) = make_float2(o[j][2] * inv1, o[j][3] * inv1);
    }
    if (t4 == 0) {
      if (r0 < nq) p.part_lse[row0] = lrow[0] > 0.f ? mrow[0] + __log2f(lrow[0]) : -FLT_MAX;
      if (r1 < nq) p.part_lse[row1] = lrow[1] > 0.f ? mrow[1] + __log2f(lrow[1]) : -FLT_MAX;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int col = j * 8 + 2 * t4;
    if (r0 < nq)
      *reinterpret_cast<uint32_t*>(p.out + ((long long)(q0 + r0) * p.Hq + hq) * D_ + col) =
          pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    if (r1 < nq)
      *reinterpret_cast<uint32_t*>(p.out + ((long long)(q0 + r1) * p.Hq + hq) * D_ + col) =
          pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
  }
}

void prefill_attention(torch::Tensor q, int64_t k, int64_t v, int64_t km, int64_t vm, int64_t blk_stride,
                       int64_t head_stride, int64_t mblk_stride, int64_t mhead_stride, int64_t fmt,
                       torch::Tensor block_table, torch::Tensor cu_q, torch::Tensor seq_lens, int64_t Hkv,
                       double scale, int64_t max_q, torch::Tensor out, int64_t num_splits,
                       c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_lse) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.is_contiguous() && q.dim() == 3,
              "q must be contiguous bf16 [T, Hq, D]");
  TORCH_CHECK(q.size(2) == D_, "prefill_attention: head_dim must be 128");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == torch::kBFloat16, "out must be contiguous bf16");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && cu_q.scalar_type() == torch::kInt32 &&
                  seq_lens.scalar_type() == torch::kInt32,
              "index tensors must be int32");
  const int B = seq_lens.size(0), Hq = q.size(1);
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  PrefillParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
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
  p.cu_q = cu_q.data_ptr<int>();
  p.seq_lens = seq_lens.data_ptr<int>();
  p.Hq = Hq;
  p.Hkv = static_cast<int>(Hkv);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  const int S = static_cast<int>(std::max<int64_t>(1, num_splits));
  p.num_splits = S;
  p.part_o = nullptr;
  p.part_lse = nullptr;
  const int T = q.size(0);
  if (S > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value() && part_o->scalar_type() == torch::kFloat32 &&
                    part_lse->scalar_type() == torch::kFloat32 &&
                    part_o->numel() >= (int64_t)T * Hq * S * D_ && part_lse->numel() >= (int64_t)T * Hq * S,
                "prefill_attention: split-KV scratch too small");
    p.part_o = part_o->data_ptr<float>();
    p.part_lse = part_lse->data_ptr<float>();
  }
  const int smem = BM * ROWB + 4 * BN * ROWB;  // 80 KB
  TORCH_CHECK((int64_t)B * S < 65536, "prefill_attention: too many sequences x splits");
  dim3 grid((max_q + BM - 1) / BM, Hq, B * S);
  auto st = at::cuda::getCurrentCUDAStream();
  if (grid.x == 0 || B == 0) return;
  if (fmt == kBF16) {
    cudaFuncSetAttribute(prefill_attn_kernel<kBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    prefill_attn_kernel<kBF16><<<grid, 128, smem, st>>>(p);
  } else if (fmt == kFP8Token) {
    cudaFuncSetAttribute(prefill_attn_kernel<kFP8Token>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    prefill_attn_kernel<kFP8Token><<<grid, 128, smem, st>>>(p);
  } else if (fmt == kINT4G64) {
    cudaFuncSetAttribute(prefill_attn_kernel<kINT4G64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    prefill_attn_kernel<kINT4G64><<<grid, 128, smem, st>>>(p);
  } else {
    TORCH_CHECK(false, "prefill_attention: unsupported cache format ", fmt);
  }
  AXR_CHECK_CUDA(cudaGetLastError());
  if (S > 1 && T > 0) {
    decode_combine_kernel<128><<<T * Hq, 128, 0, st>>>(p.part_o, p.part_lse, p.out, S);
    AXR_CHECK_CUDA(cudaGetLastError());
  }
}

}  // namespace axr
