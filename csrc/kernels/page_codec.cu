// Page transfer kernel: moves KV page units between any two page stores, converting
// the storage format on the way (dequantise -> requantise in registers).
//
// One kernel serves every KV movement of the framework:
//   restore  : G1 pool chunk slots -> live paged cache blocks (block table scatter)
//   capture  : live paged cache blocks -> G1 pool chunk slots (quantise on write)
//   export   : cache/pool -> dense AMFK layout (disk tier), and back
//   cross-GPU: either side may be another GPU's memory mapped into this process
//              (symmetric/IPC mapping): the loads or stores then travel over NVLink
//              from inside the kernel, so a remote restore is one fused pull +
//              dequantise + scatter, and a capture to a remote owner shard is one
//              fused quantise + push. No TMA is used on peer memory.
//
// Reference counterparts: CompressedVRAMPool.restore_to_vllm / put_from_vllm
// (korith_vllm_ext/compressed_vram_pool.py:434-608) and the connector's per-layer
// slot index-put (amf_kv_connector.py:322-442), which decompress a whole layer in
// PyTorch and scatter with index-put; here it is one pass over HBM.
//
// Work decomposition: one warp per page unit (P=16 tokens x D dims of one head of one
// (layer, K|V)); a lane owns 8 consecutive dims of 16*8/D... rows, so every load is a
// 4-16 byte vector and a warp covers whole 256-byte rows. Units are visited in
// (page, layer*2+kv, head) order with a grid-stride loop over a persistent grid.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace axr {

struct PageSide {
  char* data;
  char* meta;
  long long s_lk, s_blk, s_h;  // data byte strides: (layer*2+kv), block id, head
  long long m_lk, m_blk, m_h;  // meta byte strides
};

template <int D>
struct Lanes {
  static constexpr int CPR = D / 8;       // 8-dim chunks per row
  static constexpr int RPI = 32 / CPR;    // rows covered by one warp pass
  static constexpr int NR = kPage / RPI;  // rows per lane
};

template <int SRC, int D>
__device__ __forceinline__ void load_unit(const PageSide& s, long long doff, long long moff, int lane,
                                          float (&v)[Lanes<D>::NR][8], uint4 (&raw)[Lanes<D>::NR],
                                          float (&rscale)[Lanes<D>::NR], uint32_t (&rmeta)[Lanes<D>::NR]) {
  using L = Lanes<D>;
  const int c = lane % L::CPR, r0 = lane / L::CPR;
#pragma unroll
  for (int i = 0; i < L::NR; ++i) {
    const int r = r0 + i * L::RPI;
    if constexpr (SRC == kBF16) {
      const uint4 x = ld_v4(s.data + doff + (long long)r * D * 2 + c * 16);
      raw[i] = x;
      v[i][0] = bf16_lo(x.x); v[i][1] = bf16_hi(x.x);
      v[i][2] = bf16_lo(x.y); v[i][3] = bf16_hi(x.y);
      v[i][4] = bf16_lo(x.z); v[i][5] = bf16_hi(x.z);
      v[i][6] = bf16_lo(x.w); v[i][7] = bf16_hi(x.w);
    } else if constexpr (SRC == kFP8Page || SRC == kFP8Token) {
      const uint2 x = ld_v2(s.data + doff + (long long)r * D + c * 8);
      raw[i] = make_uint4(x.x, x.y, 0, 0);
      const float sc = (SRC == kFP8Page) ? *reinterpret_cast<const float*>(s.meta + moff)
                                         : *reinterpret_cast<const float*>(s.meta + moff + r * 4);
      rscale[i] = sc;
      float2 a = e4m3x2_to_float2(x.x & 0xffff), b = e4m3x2_to_float2(x.x >> 16);
      float2 e = e4m3x2_to_float2(x.y & 0xffff), f = e4m3x2_to_float2(x.y >> 16);
      v[i][0] = a.x * sc; v[i][1] = a.y * sc; v[i][2] = b.x * sc; v[i][3] = b.y * sc;
      v[i][4] = e.x * sc; v[i][5] = e.y * sc; v[i][6] = f.x * sc; v[i][7] = f.y * sc;
    } else {  // kINT4G64
      const uint32_t x = ld_u32(s.data + doff + (long long)r * (D / 2) + c * 4);
      raw[i] = make_uint4(x, 0, 0, 0);
      const uint32_t m = ld_u32(s.meta + moff + ((long long)r * (D / kGroup) + c / 8) * 4);
      rmeta[i] = m;
      const float sc = half_bits_to_float(m & 0xffff), zp = half_bits_to_float(m >> 16);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = static_cast<float>((x >> (4 * j)) & 0xf) * sc + zp;
    }
  }
}

template <int SRC, int DST, int D>
__global__ void __launch_bounds__(256) page_transfer_kernel(PageSide src, PageSide dst,
                                                            const int* __restrict__ src_ids,
                                                            const int* __restrict__ dst_ids, int n_pages,
                                                            int n_lk, int H) {
  using L = Lanes<D>;
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const long long n_units = (long long)n_pages * n_lk * H;
  const int c = lane % L::CPR, r0 = lane / L::CPR;
  for (long long u = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n_units;
       u += warps_total) {
    const int h = static_cast<int>(u % H);
    const int lk = static_cast<int>((u / H) % n_lk);
    const int p = static_cast<int>(u / ((long long)H * n_lk));
    const int sb = src_ids[p], db = dst_ids[p];
    const long long sdo = lk * src.s_lk + sb * src.s_blk + h * src.s_h;
    const long long smo = lk * src.m_lk + sb * src.m_blk + h * src.m_h;
    const long long ddo = lk * dst.s_lk + db * dst.s_blk + h * dst.s_h;
    const long long dmo = lk * dst.m_lk + db * dst.m_blk + h * dst.m_h;

    float v[L::NR][8];
    uint4 raw[L::NR];
    float rscale[L::NR];
    uint32_t rmeta[L::NR];
    load_unit<SRC, D>(src, sdo, smo, lane, v, raw, rscale, rmeta);

    if constexpr (DST == kBF16) {
#pragma unroll
      for (int i = 0; i < L::NR; ++i) {
        const int r = r0 + i * L::RPI;
        uint4 o;
        if constexpr (SRC == kBF16) {
          o = raw[i];  // bit-exact copy
        } else {
          o = make_uint4(pack_bf16x2(v[i][0], v[i][1]), pack_bf16x2(v[i][2], v[i][3]),
                         pack_bf16x2(v[i][4], v[i][5]), pack_bf16x2(v[i][6], v[i][7]));
        }
        *reinterpret_cast<uint4*>(dst.data + ddo + (long long)r * D * 2 + c * 16) = o;
      }
    } else if constexpr (DST == kFP8Page) {
      if constexpr (SRC == kFP8Page) {
#pragma unroll
        for (int i = 0; i < L::NR; ++i) {
          const int r = r0 + i * L::RPI;
          *reinterpret_cast<uint2*>(dst.data + ddo + (long long)r * D + c * 8) = make_uint2(raw[i].x, raw[i].y);
        }
        if (lane == 0) *reinterpret_cast<float*>(dst.meta + dmo) = rscale[0];
      } else {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < L::NR; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
        amax = warp_max(amax);
        const float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
#pragma unroll
        for (int i = 0; i < L::NR; ++i) {
          const int r = r0 + i * L::RPI;
          uint2 o;
          o.x = float2_to_e4m3x2(v[i][0] * inv, v[i][1] * inv) | (uint32_t(float2_to_e4m3x2(v[i][2] * inv, v[i][3] * inv)) << 16);
          o.y = float2_to_e4m3x2(v[i][4] * inv, v[i][5] * inv) | (uint32_t(float2_to_e4m3x2(v[i][6] * inv, v[i][7] * inv)) << 16);
          *reinterpret_cast<uint2*>(dst.data + ddo + (long long)r * D + c * 8) = o;
        }
        if (lane == 0) *reinterpret_cast<float*>(dst.meta + dmo) = __fdiv_rn(amax, 448.f);
      }
    } else if constexpr (DST == kFP8Token) {
#pragma unroll
      for (int i = 0; i < L::NR; ++i) {
        const int r = r0 + i * L::RPI;
        uint2 o;
        float sc;
        if constexpr (SRC == kFP8Page || SRC == kFP8Token) {
          o = make_uint2(raw[i].x, raw[i].y);  // codes keep their meaning; scale moves per row
          sc = rscale[i];
        } else {
          float amax = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
          amax = warp_max<L::CPR>(amax);
          const float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
          o.x = float2_to_e4m3x2(v[i][0] * inv, v[i][1] * inv) | (uint32_t(float2_to_e4m3x2(v[i][2] * inv, v[i][3] * inv)) << 16);
          o.y = float2_to_e4m3x2(v[i][4] * inv, v[i][5] * inv) | (uint32_t(float2_to_e4m3x2(v[i][6] * inv, v[i][7] * inv)) << 16);
          sc = __fdiv_rn(amax, 448.f);
        }
        *reinterpret_cast<uint2*>(dst.data + ddo + (long long)r * D + c * 8) = o;
        if (c == 0) *reinterpret_cast<float*>(dst.meta + dmo + r * 4) = sc;
      }
    } else {  // kINT4G64
#pragma unroll
      for (int i = 0; i < L::NR; ++i) {
        const int r = r0 + i * L::RPI;
        uint32_t packed, meta;
        if constexpr (SRC == kINT4G64) {
          packed = raw[i].x;
          meta = rmeta[i];
        } else {
          float mn = v[i][0], mx = v[i][0];
#pragma unroll
          for (int j = 1; j < 8; ++j) { mn = fminf(mn, v[i][j]); mx = fmaxf(mx, v[i][j]); }
          mn = warp_min<8>(mn);
          mx = warp_max<8>(mx);
          const uint16_t sh = float_to_half_bits((mx - mn) * (1.0f / 15.0f));
          const uint16_t zh = float_to_half_bits(mn);
          const float sf = half_bits_to_float(sh), zf = half_bits_to_float(zh);
          const float inv = sf > 0.f ? __frcp_rn(sf) : 0.f;
          packed = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float q = rintf((v[i][j] - zf) * inv);
            q = fminf(fmaxf(q, 0.f), 15.f);
            packed |= static_cast<uint32_t>(q) << (4 * j);
          }
          meta = uint32_t(sh) | (uint32_t(zh) << 16);
        }
        *reinterpret_cast<uint32_t*>(dst.data + ddo + (long long)r * (D / 2) + c * 4) = packed;
        if ((c & 7) == 0) *reinterpret_cast<uint32_t*>(dst.meta + dmo + ((long long)r * (D / kGroup) + c / 8) * 4) = meta;
      }
    }
  }
}

// ------------------------------------------------------------------------------- host
namespace {
PageSide side_from(int64_t data, int64_t meta, const std::vector<int64_t>& st) {
  TORCH_CHECK(st.size() == 6, "page side needs 6 strides");
  return PageSide{reinterpret_cast<char*>(data), reinterpret_cast<char*>(meta), st[0], st[1], st[2],
                  st[3], st[4], st[5]};
}

template <int SRC, int DST>
void launch_d(int D, const PageSide& s, const PageSide& d, const int* si, const int* di, int n, int nlk, int H,
              int grid, cudaStream_t st) {
  if (D == 128) page_transfer_kernel<SRC, DST, 128><<<grid, 256, 0, st>>>(s, d, si, di, n, nlk, H);
  else if (D == 64) page_transfer_kernel<SRC, DST, 64><<<grid, 256, 0, st>>>(s, d, si, di, n, nlk, H);
  else if (D == 256) page_transfer_kernel<SRC, DST, 256><<<grid, 256, 0, st>>>(s, d, si, di, n, nlk, H);
  else TORCH_CHECK(false, "page_transfer: unsupported head_dim ", D);
}

template <int SRC>
void launch_dst(int dst_fmt, int D, const PageSide& s, const PageSide& d, const int* si, const int* di, int n,
                int nlk, int H, int grid, cudaStream_t st) {
  switch (dst_fmt) {
    case kBF16: launch_d<SRC, kBF16>(D, s, d, si, di, n, nlk, H, grid, st); break;
    case kFP8Page: launch_d<SRC, kFP8Page>(D, s, d, si, di, n, nlk, H, grid, st); break;
    case kFP8Token: launch_d<SRC, kFP8Token>(D, s, d, si, di, n, nlk, H, grid, st); break;
    case kINT4G64: launch_d<SRC, kINT4G64>(D, s, d, si, di, n, nlk, H, grid, st); break;
    default: TORCH_CHECK(false, "page_transfer: bad destination format ", dst_fmt);
  }
}
}  // namespace

// src/dst: raw device addresses (peer addresses allowed) and strides; ids: int32 CUDA
// tensors of length n_pages (source block/slot id, destination block/slot id).
void page_transfer(int64_t src_data, int64_t src_meta, std::vector<int64_t> src_strides, int64_t src_fmt,
                   int64_t dst_data, int64_t dst_meta, std::vector<int64_t> dst_strides, int64_t dst_fmt,
                   torch::Tensor src_ids, torch::Tensor dst_ids, int64_t n_lk, int64_t H, int64_t D,
                   int64_t max_ctas) {
  TORCH_CHECK(src_ids.is_cuda() && dst_ids.is_cuda(), "page_transfer: ids must be CUDA tensors");
  TORCH_CHECK(src_ids.scalar_type() == torch::kInt32 && dst_ids.scalar_type() == torch::kInt32,
              "page_transfer: ids must be int32");
  TORCH_CHECK(src_ids.numel() == dst_ids.numel(), "page_transfer: id lists differ in length");
  const int n = static_cast<int>(src_ids.numel());
  if (n == 0) return;
  TORCH_CHECK(src_data % 16 == 0 && dst_data % 16 == 0, "page_transfer: data must be 16-byte aligned");
  const PageSide s = side_from(src_data, src_meta, src_strides);
  const PageSide d = side_from(dst_data, dst_meta, dst_strides);
  const long long units = (long long)n * n_lk * H;
  const long long want = (units + 7) / 8;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, src_ids.device().index());
  long long grid = std::min<long long>(want, max_ctas > 0 ? max_ctas : (long long)sms * 8);
  grid = std::max<long long>(grid, 1);
  auto st = at::cuda::getCurrentCUDAStream();
  const int* si = src_ids.data_ptr<int>();
  const int* di = dst_ids.data_ptr<int>();
  switch (src_fmt) {
    case kBF16: launch_dst<kBF16>(dst_fmt, D, s, d, si, di, n, n_lk, H, grid, st); break;
    case kFP8Page: launch_dst<kFP8Page>(dst_fmt, D, s, d, si, di, n, n_lk, H, grid, st); break;
    case kFP8Token: launch_dst<kFP8Token>(dst_fmt, D, s, d, si, di, n, n_lk, H, grid, st); break;
    case kINT4G64: launch_dst<kINT4G64>(dst_fmt, D, s, d, si, di, n, n_lk, H, grid, st); break;
    default: TORCH_CHECK(false, "page_transfer: bad source format ", src_fmt);
  }
  AXR_CHECK_CUDA(cudaGetLastError());
}

}  // namespace axr
