// GPU encode / decode of the reference's KV blob formats, bit-compatible with the CPU
// codecs (axropus_deploy_b200/codecs/scalar.py, lowbit.py), so a blob written by either
// side restores on the GPU without a CPU round trip:
//
//   int4_sym        per-channel (last-axis lane) scale amax/7, q in [-8, 7] stored q + 8,
//                   two per byte, even index in the low nibble
//   int4_sym_block  one scale per block of 128 tokens (over tokens x heads x dims) of each
//                   leading slice, same nibbles
//   int2_sym        per-channel scale amax/2, q in [-2, 1] stored q + 2, four per byte,
//                   first value in the low bits
//   nvfp4           groups of 16 along the last axis: E2M1 magnitude index (nearest of
//                   {0, .5, 1, 1.5, 2, 3, 4, 6}, first on ties) with the sign in bit 3, two
//                   per byte; one scale byte per group, (1 + m/8) 2^e with e in [-6, 8]
//                   (sign << 7 | (e + 7) << 3 | m) for amax/6 clamped to 448
//
// Quantisation uses the fp32 scale and stores it as fp16 (the CPU codecs' order), so the
// codes match. The extension builds with fast math, so every division that decides a code
// is written as a correctly rounded __fdiv_rn and every power of two as ldexpf. Every kernel is element-wise or a reduction: HBM-bound grid-stride loops.
// (TurboQuant's projections are GEMMs: they run on the dense tcgen05 kernels.)
// Reference formats: korith_vllm_ext/codecs/amf_codec.py:345-538, nvfp4_codec.py:44-158.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "codecs.h"

namespace axr {
namespace codec {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

// non-negative floats order like their bit patterns
__device__ __forceinline__ void atomic_max_pos(float* p, float v) {
  atomicMax(reinterpret_cast<unsigned int*>(p), __float_as_uint(v));
}

// ---- per-lane amax over rows [R, D]
template <typename T>
__global__ void lane_amax_kernel(const T* __restrict__ x, long long R, int D, float* __restrict__ amax) {
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float m = 0.f;
    for (long long r = blockIdx.x; r < R; r += gridDim.x) m = fmaxf(m, fabsf(to_f<T>(x[r * D + d])));
    atomic_max_pos(amax + d, m);
  }
}

// ---- per-block amax: x viewed as [S, T, W] (W = heads x dims), blocks of BT tokens
template <typename T>
__global__ void block_amax_kernel(const T* __restrict__ x, int T_, int W, int BT, int nb, float* __restrict__ amax) {
  const int s = blockIdx.y, b = blockIdx.x;
  const long long t0 = (long long)b * BT;
  const long long t1 = (t0 + BT < (long long)T_) ? t0 + BT : (long long)T_;
  const T* base = x + (long long)s * T_ * W;
  float m = 0.f;
  for (long long i = t0 * W + threadIdx.x; i < t1 * W; i += blockDim.x) m = fmaxf(m, fabsf(to_f<T>(base[i])));
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) amax[(long long)s * nb + b] = m;
  }
}

// scale = max(amax, 1e-8) / qmax in fp32 (used for quantising), stored as fp16
__global__ void scales_kernel(const float* __restrict__ amax, long long n, float qmax, float* __restrict__ s32,
                              __half* __restrict__ s16) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float s = __fdiv_rn(fmaxf(amax[i], 1e-8f), qmax);
    s32[i] = s;
    s16[i] = __float2half_rn(s);
  }
}

// ---- int4 encode: one thread per output byte (two values). scale index per mode.
template <typename T, bool BLOCK>
__global__ void int4_encode_kernel(const T* __restrict__ x, long long R, int D, const float* __restrict__ s32,
                                   int T_, int HD, int BT, int nb, uint8_t* __restrict__ out) {
  const int DB = (D + 1) / 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * DB; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / DB;
    const int c = static_cast<int>(i % DB);
    uint8_t byte = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int d = 2 * c + h;
      int q = -8;  // padding nibble 0, as the CPU packer pads
      if (d < D) {
        float sc;
        if constexpr (BLOCK) {
          const long long flat = r * D + d;  // [S, T, HD]
          const long long s = flat / ((long long)T_ * HD), t = (flat / HD) % T_;
          sc = s32[s * nb + t / BT];
        } else {
          sc = s32[d];
        }
        q = static_cast<int>(rintf(__fdiv_rn(to_f<T>(x[r * D + d]), sc)));
        q = min(max(q, -8), 7);
      }
      byte |= static_cast<uint8_t>((q + 8) & 0xF) << (4 * h);
    }
    out[i] = byte;
  }
}

template <typename O, bool BLOCK>
__global__ void int4_decode_kernel(const uint8_t* __restrict__ in, long long R, int D, const __half* __restrict__ s16,
                                   int T_, int HD, int BT, int nb, O* __restrict__ out) {
  const int DB = (D + 1) / 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * D; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / D;
    const int d = static_cast<int>(i % D);
    const int q = ((in[r * DB + d / 2] >> (4 * (d & 1))) & 0xF) - 8;
    float sc;
    if constexpr (BLOCK) {
      const long long s = i / ((long long)T_ * HD), t = (i / HD) % T_;
      sc = __half2float(s16[s * nb + t / BT]);
    } else {
      sc = __half2float(s16[d]);
    }
    out[i] = from_f<O>(static_cast<float>(q) * sc);
  }
}

// ---- int2 (per lane)
template <typename T>
__global__ void int2_encode_kernel(const T* __restrict__ x, long long R, int D, const float* __restrict__ s32,
                                   uint8_t* __restrict__ out) {
  const int DB = (D + 3) / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * DB; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / DB;
    const int c = static_cast<int>(i % DB);
    uint8_t byte = 0;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int d = 4 * c + h;
      int u = 0;
      if (d < D) {
        int q = static_cast<int>(rintf(__fdiv_rn(to_f<T>(x[r * D + d]), s32[d])));
        u = min(max(q, -2), 1) + 2;
      }
      byte |= static_cast<uint8_t>(u & 3) << (2 * h);
    }
    out[i] = byte;
  }
}

template <typename O>
__global__ void int2_decode_kernel(const uint8_t* __restrict__ in, long long R, int D, const __half* __restrict__ s16,
                                   O* __restrict__ out) {
  const int DB = (D + 3) / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * D; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / D;
    const int d = static_cast<int>(i % D);
    const int u = (in[r * DB + d / 4] >> (2 * (d & 3))) & 3;
    out[i] = from_f<O>(static_cast<float>(u - 2) * __half2float(s16[d]));
  }
}

// ---- NVFP4: one thread per group of 16 values of a row of Dp (padded) values
__constant__ float kE2M1[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};

__device__ __forceinline__ uint8_t scale_byte(float v) {
  v = fminf(fmaxf(v, -448.f), 448.f);
  const float a = fmaxf(fabsf(v), 1e-20f);
  int e = static_cast<int>((__float_as_uint(a) >> 23) & 0xFF) - 127;  // floor(log2 a) of a normal float
  e = min(max(e, -6), 8);
  int m = static_cast<int>(rintf((a * ldexpf(1.f, -e) - 1.f) * 8.f));  // exact power-of-two scaling
  m = min(max(m, 0), 7);
  return static_cast<uint8_t>(((v < 0.f ? 1 : 0) << 7) | (min(max(e + 7, 0), 15) << 3) | m);
}

__device__ __forceinline__ float scale_value(uint8_t b) {
  const float v = ldexpf(1.f + static_cast<float>(b & 7) * 0.125f, ((b >> 3) & 0xF) - 7);
  return (b >> 7) ? -v : v;
}

template <typename T>
__global__ void nvfp4_encode_kernel(const T* __restrict__ x, long long R, int D, int Dp, uint8_t* __restrict__ out,
                                    uint8_t* __restrict__ sbytes, float* __restrict__ amax_all) {
  const int G = Dp / 16;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * G; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / G;
    const int g = static_cast<int>(i % G);
    float v[16];
    float am = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = g * 16 + j;
      v[j] = d < D ? to_f<T>(x[r * D + d]) : 0.f;
      am = fmaxf(am, fabsf(v[j]));
    }
    atomic_max_pos(amax_all, am);
    const float gs = fminf(__fdiv_rn(fmaxf(am, 1e-8f), 6.f), 448.f);
    sbytes[i] = scale_byte(gs);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      uint8_t nib[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float y = __fdiv_rn(v[j + h], gs);
        const float ay = fabsf(y);
        int best = 0;
        float bd = fabsf(ay - kE2M1[0]);
#pragma unroll
        for (int l = 1; l < 8; ++l) {
          const float dd = fabsf(ay - kE2M1[l]);
          if (dd < bd) {
            bd = dd;
            best = l;
          }
        }
        nib[h] = static_cast<uint8_t>(((y < 0.f ? 1 : 0) << 3) | best);
      }
      out[r * (Dp / 2) + (g * 16 + j) / 2] = nib[0] | (nib[1] << 4);
    }
  }
}

template <typename O>
__global__ void nvfp4_decode_kernel(const uint8_t* __restrict__ in, const uint8_t* __restrict__ sbytes, long long R,
                                    int D, int Dp, O* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * D; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / D;
    const int d = static_cast<int>(i % D);
    const uint8_t n = (in[r * (Dp / 2) + d / 2] >> (4 * (d & 1))) & 0xF;
    const float mag = kE2M1[n & 7] * scale_value(sbytes[r * (Dp / 16) + d / 16]);
    out[i] = from_f<O>((n >> 3) ? -mag : mag);
  }
}

int grid_for(long long n, int threads = 256) {
  const long long g = (n + threads - 1) / threads;
  return static_cast<int>(g < 148LL * 32 ? (g > 0 ? g : 1) : 148LL * 32);
}

template <typename T>
std::string encode_t(const EncodeCall& c, cudaStream_t st) {
  const T* x = static_cast<const T*>(c.x);
  const long long R = c.rows;
  const int D = c.D;
  switch (c.fmt) {
    case kInt4Sym:
    case kInt2Sym: {
      cudaMemsetAsync(c.amax, 0, sizeof(float) * D, st);
      lane_amax_kernel<T><<<grid_for(R, 1) > 1024 ? 1024 : grid_for(R, 1), 128, 0, st>>>(x, R, D, c.amax);
      scales_kernel<<<grid_for(D), 256, 0, st>>>(c.amax, D, c.fmt == kInt4Sym ? 7.f : 2.f, c.scale32, c.scale16);
      if (c.fmt == kInt4Sym)
        int4_encode_kernel<T, false><<<grid_for(R * ((D + 1) / 2)), 256, 0, st>>>(x, R, D, c.scale32, 0, 0, 1, 1,
                                                                                  c.out);
      else
        int2_encode_kernel<T><<<grid_for(R * ((D + 3) / 4)), 256, 0, st>>>(x, R, D, c.scale32, c.out);
      break;
    }
    case kInt4Block: {
      const int nb = (c.T + c.BT - 1) / c.BT;
      block_amax_kernel<T><<<dim3(nb, c.S), 256, 0, st>>>(x, c.T, c.HD, c.BT, nb, c.amax);
      scales_kernel<<<grid_for((long long)c.S * nb), 256, 0, st>>>(c.amax, (long long)c.S * nb, 7.f, c.scale32,
                                                                  c.scale16);
      int4_encode_kernel<T, true><<<grid_for(R * ((D + 1) / 2)), 256, 0, st>>>(x, R, D, c.scale32, c.T, c.HD, c.BT,
                                                                               nb, c.out);
      break;
    }
    case kNvfp4: {
      const int Dp = (D + 15) / 16 * 16;
      cudaMemsetAsync(c.amax, 0, sizeof(float), st);
      nvfp4_encode_kernel<T><<<grid_for(R * (Dp / 16)), 256, 0, st>>>(x, R, D, Dp, c.out, c.sbytes, c.amax);
      break;
    }
    default:
      return "unknown format";
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? "" : std::string("launch failed: ") + cudaGetErrorString(e);
}

template <typename O>
std::string decode_t(const DecodeCall& c, cudaStream_t st) {
  O* out = static_cast<O*>(c.out);
  const long long R = c.rows;
  const int D = c.D;
  const long long n = R * D;
  switch (c.fmt) {
    case kInt4Sym:
      int4_decode_kernel<O, false><<<grid_for(n), 256, 0, st>>>(c.in, R, D, c.scale16, 0, 0, 1, 1, out);
      break;
    case kInt4Block: {
      const int nb = (c.T + c.BT - 1) / c.BT;
      int4_decode_kernel<O, true><<<grid_for(n), 256, 0, st>>>(c.in, R, D, c.scale16, c.T, c.HD, c.BT, nb, out);
      break;
    }
    case kInt2Sym:
      int2_decode_kernel<O><<<grid_for(n), 256, 0, st>>>(c.in, R, D, c.scale16, out);
      break;
    case kNvfp4:
      nvfp4_decode_kernel<O><<<grid_for(n), 256, 0, st>>>(c.in, c.sbytes, R, D, (D + 15) / 16 * 16, out);
      break;
    default:
      return "unknown format";
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? "" : std::string("launch failed: ") + cudaGetErrorString(e);
}

}  // namespace

std::string encode(const EncodeCall& c, cudaStream_t st) {
  if (c.rows <= 0 || c.D <= 0) return "";
  switch (c.dtype) {
    case kF32: return encode_t<float>(c, st);
    case kF16: return encode_t<__half>(c, st);
    case kBF16: return encode_t<__nv_bfloat16>(c, st);
    default: return "input dtype must be fp32, fp16 or bf16";
  }
}

std::string decode(const DecodeCall& c, cudaStream_t st) {
  if (c.rows <= 0 || c.D <= 0) return "";
  switch (c.dtype) {
    case kF32: return decode_t<float>(c, st);
    case kF16: return decode_t<__half>(c, st);
    case kBF16: return decode_t<__nv_bfloat16>(c, st);
    default: return "output dtype must be fp32, fp16 or bf16";
  }
}

}  // namespace codec
}  // namespace axr
