// Fused per-token kernels of the transformer step:
//   * rmsnorm_residual: out = RMSNorm(x + residual) * w, residual <- x + residual
//   * rope_kv_write:    RoPE on q and k of the fused QKV projection, q written out,
//                       k and v stored straight into their KV pages (bf16, FP8 per-token
//                       or INT4 g64), so no separate "write KV cache" pass exists
//   * silu_mul:         SwiGLU activation on the fused gate/up projection
// Reference counterparts: the library ops llama.cpp/vLLM run for these steps and the
// placeholder korith_rmsnorm_linear_kernel (platform/kernels/cuda/kernels.cu:7-26).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace axr {

// ----------------------------------------------------------------------------- RMSNorm
template <int VPT>  // bf16 values per thread (8 per 16-byte vector)
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      __nv_bfloat16* __restrict__ residual,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ out, int H, float eps,
                                                      int early) {
  const long long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  __nv_bfloat16* rr = residual ? residual + row * H : nullptr;
  // A decode-sized norm releases the next projection at once, so its weight stream starts
  // during the norm; a prefill-sized one does not (see the launch).
  if (early) pdl_trigger();
  pdl_wait();  // x / residual come from the kernels before
  float v[VPT];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < VPT / 8; ++c) {
    const int d = (threadIdx.x + c * blockDim.x) * 8;
    if (d >= H) continue;
    uint4 a = *reinterpret_cast<const uint4*>(xr + d);
    float f[8] = {bf16_lo(a.x), bf16_hi(a.x), bf16_lo(a.y), bf16_hi(a.y), bf16_lo(a.z), bf16_hi(a.z),
                  bf16_lo(a.w), bf16_hi(a.w)};
    if (rr) {
      uint4 r = *reinterpret_cast<const uint4*>(rr + d);
      f[0] += bf16_lo(r.x); f[1] += bf16_hi(r.x); f[2] += bf16_lo(r.y); f[3] += bf16_hi(r.y);
      f[4] += bf16_lo(r.z); f[5] += bf16_hi(r.z); f[6] += bf16_lo(r.w); f[7] += bf16_hi(r.w);
      // the residual stream is kept in bf16, like the model's activations
      uint4 o = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                           pack_bf16x2(f[6], f[7]));
      *reinterpret_cast<uint4*>(rr + d) = o;
      f[0] = bf16_lo(o.x); f[1] = bf16_hi(o.x); f[2] = bf16_lo(o.y); f[3] = bf16_hi(o.y);
      f[4] = bf16_lo(o.z); f[5] = bf16_hi(o.z); f[6] = bf16_lo(o.w); f[7] = bf16_hi(o.w);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[c * 8 + j] = f[j];
      ss += f[j] * f[j];
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / H + eps);
#pragma unroll
  for (int c = 0; c < VPT / 8; ++c) {
    const int d = (threadIdx.x + c * blockDim.x) * 8;
    if (d >= H) continue;
    uint4 wv = *reinterpret_cast<const uint4*>(w + d);
    const float wf[8] = {bf16_lo(wv.x), bf16_hi(wv.x), bf16_lo(wv.y), bf16_hi(wv.y),
                         bf16_lo(wv.z), bf16_hi(wv.z), bf16_lo(wv.w), bf16_hi(wv.w)};
    uint4 o;
    o.x = pack_bf16x2(v[c * 8 + 0] * inv * wf[0], v[c * 8 + 1] * inv * wf[1]);
    o.y = pack_bf16x2(v[c * 8 + 2] * inv * wf[2], v[c * 8 + 3] * inv * wf[3]);
    o.z = pack_bf16x2(v[c * 8 + 4] * inv * wf[4], v[c * 8 + 5] * inv * wf[5]);
    o.w = pack_bf16x2(v[c * 8 + 6] * inv * wf[6], v[c * 8 + 7] * inv * wf[7]);
    *reinterpret_cast<uint4*>(out + row * H + d) = o;
  }
}

void rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w, double eps,
             torch::Tensor out) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "x: contiguous bf16");
  const int H = x.size(-1);
  TORCH_CHECK(H % 8 == 0 && H <= 256 * 8 * 8, "rmsnorm: hidden size must be a multiple of 8 and <= 16384");
  const long long rows = x.numel() / H;
  if (rows == 0) return;
  __nv_bfloat16* r = nullptr;
  if (residual.has_value()) {
    TORCH_CHECK(residual->is_contiguous() && residual->scalar_type() == torch::kBFloat16, "residual: bf16");
    r = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr());
  }
  auto st = at::cuda::getCurrentCUDAStream();
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const int per = (H + 256 * 8 - 1) / (256 * 8);
  const dim3 grid(static_cast<unsigned>(rows));
  const float fe = static_cast<float>(eps);
  // Early release only for decode-sized batches (<= 256 rows, the weight-streaming GEMMs):
  // a prefill GEMM launched early parks its CTAs beside thousands of norm CTAs, which cost
  // clock under the power cap.
  const int early = rows <= 256 ? 1 : 0;
  cudaError_t e;
  if (per <= 1) e = launch_pdl(rmsnorm_kernel<8>, grid, dim3(256), 0, st, xp, r, wp, op, H, fe, early);
  else if (per <= 2) e = launch_pdl(rmsnorm_kernel<16>, grid, dim3(256), 0, st, xp, r, wp, op, H, fe, early);
  else if (per <= 4) e = launch_pdl(rmsnorm_kernel<32>, grid, dim3(256), 0, st, xp, r, wp, op, H, fe, early);
  else e = launch_pdl(rmsnorm_kernel<64>, grid, dim3(256), 0, st, xp, r, wp, op, H, fe, early);
  AXR_CHECK_CUDA(e);
}

// ------------------------------------------------------------------------ RoPE + KV
struct RopeKvParams {
  const __nv_bfloat16* qkv;  // [T, (Hq + 2 Hkv) * D]
  const int* pos;            // [T]
  const int* slots;          // [T] block*16 + offset, -1 = do not store
  const float* cos_sin;      // [max_pos, D] : cos[0:D/2] sin[D/2:D]
  __nv_bfloat16* q_out;      // [T, Hq, D]
  char* k;
  char* v;
  char* km;
  char* vm;
  long long blk_stride, head_stride, mblk_stride, mhead_stride;
  int Hq, Hkv, T;
  int n_pos;  // rows of cos_sin; positions are clamped into it (the host checks them first)
};

// One warp per (token, head row). Lane holds dims {2l, 2l+1} and {64+2l, 64+2l+1}
// (D=128), i.e. the two rotate-half partners of each pair.
template <int FMT>
__global__ void __launch_bounds__(256) rope_kv_kernel(RopeKvParams p) {
  constexpr int D = 128;
  pdl_trigger();
  pdl_wait();  // qkv comes from the projection before (and every path waits)
  const int lane = threadIdx.x & 31;
  const long long wid = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int rows_per_tok = p.Hq + 2 * p.Hkv;
  if (wid >= (long long)p.T * rows_per_tok) return;
  const int tok = static_cast<int>(wid / rows_per_tok);
  const int hr = static_cast<int>(wid % rows_per_tok);
  const __nv_bfloat16* src = p.qkv + ((long long)tok * rows_per_tok + hr) * D;
  const uint32_t lo = *reinterpret_cast<const uint32_t*>(src + 2 * lane);
  const uint32_t hi = *reinterpret_cast<const uint32_t*>(src + 64 + 2 * lane);
  float x[4] = {bf16_lo(lo), bf16_hi(lo), bf16_lo(hi), bf16_hi(hi)};  // d, d+1, d+64, d+65
  const bool is_v = hr >= p.Hq + p.Hkv;
  if (!is_v) {
    const int ps = min(max(p.pos[tok], 0), p.n_pos - 1);
    const float* cs = p.cos_sin + (long long)ps * D;
    const float c0 = cs[2 * lane], c1 = cs[2 * lane + 1];
    const float s0 = cs[64 + 2 * lane], s1 = cs[64 + 2 * lane + 1];
    const float a0 = x[0] * c0 - x[2] * s0, b0 = x[2] * c0 + x[0] * s0;
    const float a1 = x[1] * c1 - x[3] * s1, b1 = x[3] * c1 + x[1] * s1;
    x[0] = a0; x[1] = a1; x[2] = b0; x[3] = b1;
  }
  if (hr < p.Hq) {
    __nv_bfloat16* dq = p.q_out + ((long long)tok * p.Hq + hr) * D;
    *reinterpret_cast<uint32_t*>(dq + 2 * lane) = pack_bf16x2(x[0], x[1]);
    *reinterpret_cast<uint32_t*>(dq + 64 + 2 * lane) = pack_bf16x2(x[2], x[3]);
    return;
  }
  const int slot = p.slots[tok];
  if (slot < 0) return;
  const int blk = slot / kPage, off = slot % kPage;
  const int kvh = is_v ? hr - p.Hq - p.Hkv : hr - p.Hq;
  char* unit = (is_v ? p.v : p.k) + blk * p.blk_stride + kvh * p.head_stride;
  char* munit = (is_v ? p.vm : p.km) + blk * p.mblk_stride + kvh * p.mhead_stride;
  if constexpr (FMT == kBF16) {
    char* row = unit + (long long)off * D * 2;
    *reinterpret_cast<uint32_t*>(row + 4 * lane) = pack_bf16x2(x[0], x[1]);
    *reinterpret_cast<uint32_t*>(row + 128 + 4 * lane) = pack_bf16x2(x[2], x[3]);
  } else if constexpr (FMT == kFP8Token) {
    // values must first round to bf16 (the model's activation dtype) so the stored
    // codes match a capture of the same row from a bf16 cache
    float r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = __bfloat162float(__float2bfloat16(x[j]));
    float amax = fmaxf(fmaxf(fabsf(r[0]), fabsf(r[1])), fmaxf(fabsf(r[2]), fabsf(r[3])));
    amax = warp_max(amax);
    const float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
    char* row = unit + (long long)off * D;
    *reinterpret_cast<uint16_t*>(row + 2 * lane) = float2_to_e4m3x2(r[0] * inv, r[1] * inv);
    *reinterpret_cast<uint16_t*>(row + 64 + 2 * lane) = float2_to_e4m3x2(r[2] * inv, r[3] * inv);
    if (lane == 0) *reinterpret_cast<float*>(munit + off * 4) = __fdiv_rn(amax, 448.f);
  } else {  // INT4 g64: group 0 = dims [0,64) (x[0],x[1]), group 1 = [64,128) (x[2],x[3])
    float r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = __bfloat162float(__float2bfloat16(x[j]));
    char* row = unit + (long long)off * (D / 2);
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
      const float e0 = r[2 * grp], e1 = r[2 * grp + 1];
      const float mn = warp_min(fminf(e0, e1)), mx = warp_max(fmaxf(e0, e1));
      const uint16_t sh = float_to_half_bits((mx - mn) * (1.0f / 15.0f));
      const uint16_t zh = float_to_half_bits(mn);
      const float sf = half_bits_to_float(sh), zf = half_bits_to_float(zh);
      const float inv = sf > 0.f ? __frcp_rn(sf) : 0.f;
      const float q0 = fminf(fmaxf(rintf((e0 - zf) * inv), 0.f), 15.f);
      const float q1 = fminf(fmaxf(rintf((e1 - zf) * inv), 0.f), 15.f);
      row[grp * 32 + lane] = static_cast<char>(static_cast<uint32_t>(q0) | (static_cast<uint32_t>(q1) << 4));
      if (lane == 0)
        *reinterpret_cast<uint32_t*>(munit + ((long long)off * (D / kGroup) + grp) * 4) =
            uint32_t(sh) | (uint32_t(zh) << 16);
    }
  }
}

void rope_kv_write(torch::Tensor qkv, torch::Tensor pos, torch::Tensor slots, torch::Tensor cos_sin,
                   torch::Tensor q_out, int64_t k, int64_t v, int64_t km, int64_t vm, int64_t blk_stride,
                   int64_t head_stride, int64_t mblk_stride, int64_t mhead_stride, int64_t fmt, int64_t Hq,
                   int64_t Hkv) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == torch::kBFloat16 && qkv.is_contiguous(), "qkv: bf16");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && slots.scalar_type() == torch::kInt32, "pos/slots int32");
  TORCH_CHECK(cos_sin.scalar_type() == torch::kFloat32 && cos_sin.size(1) == 128, "cos_sin fp32 [P, 128]");
  const int T = qkv.size(0);
  TORCH_CHECK(qkv.numel() == (int64_t)T * (Hq + 2 * Hkv) * 128, "qkv shape mismatch (head_dim 128)");
  if (T == 0) return;
  RopeKvParams p{reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), pos.data_ptr<int>(),
                 slots.data_ptr<int>(), cos_sin.data_ptr<float>(),
                 reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), reinterpret_cast<char*>(k),
                 reinterpret_cast<char*>(v), reinterpret_cast<char*>(km), reinterpret_cast<char*>(vm),
                 blk_stride, head_stride, mblk_stride, mhead_stride, (int)Hq, (int)Hkv, T,
                 static_cast<int>(cos_sin.size(0))};
  const long long warps = (long long)T * (Hq + 2 * Hkv);
  const int grid = static_cast<int>((warps + 7) / 8);
  auto st = at::cuda::getCurrentCUDAStream();
  cudaError_t e;
  if (fmt == kBF16) e = launch_pdl(rope_kv_kernel<kBF16>, dim3(grid), dim3(256), 0, st, p);
  else if (fmt == kFP8Token) e = launch_pdl(rope_kv_kernel<kFP8Token>, dim3(grid), dim3(256), 0, st, p);
  else if (fmt == kINT4G64) e = launch_pdl(rope_kv_kernel<kINT4G64>, dim3(grid), dim3(256), 0, st, p);
  else TORCH_CHECK(false, "rope_kv_write: unsupported cache format ", fmt);
  AXR_CHECK_CUDA(e);
}

// --------------------------------------------------------------------------- SiLU*mul
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu,
                                                       __nv_bfloat16* __restrict__ out, int F, long long n8) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 8;
    const long long row = e / F, col = e % F;
    const uint4 g = *reinterpret_cast<const uint4*>(gu + row * 2 * F + col);
    const uint4 u = *reinterpret_cast<const uint4*>(gu + row * 2 * F + F + col);
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g0 = bf16_lo(gw[j]), g1 = bf16_hi(gw[j]);
      const float s0 = g0 / (1.f + __expf(-g0)), s1 = g1 / (1.f + __expf(-g1));
      o[j] = pack_bf16x2(s0 * bf16_lo(uw[j]), s1 * bf16_hi(uw[j]));
    }
    *reinterpret_cast<uint4*>(out + row * F + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

void silu_mul(torch::Tensor gate_up, torch::Tensor out) {
  TORCH_CHECK(gate_up.is_cuda() && gate_up.scalar_type() == torch::kBFloat16 && gate_up.is_contiguous(), "bf16");
  const int F = gate_up.size(-1) / 2;
  TORCH_CHECK(F % 8 == 0, "silu_mul: width must be a multiple of 8");
  const long long n8 = out.numel() / 8;
  if (n8 == 0) return;
  const int grid = static_cast<int>(std::min<long long>((n8 + 255) / 256, 148LL * 16));
  silu_mul_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gate_up.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      F, n8);
  AXR_CHECK_CUDA(cudaGetLastError());
}

}  // namespace axr
