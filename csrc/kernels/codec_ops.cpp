// Torch binding of the GPU codec kernels (csrc/kernels/codecs.cu).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "codecs.h"

namespace axr {
namespace codec {

namespace {
int dtype_of(const torch::Tensor& t) {
  if (t.scalar_type() == torch::kFloat32) return kF32;
  if (t.scalar_type() == torch::kFloat16) return kF16;
  if (t.scalar_type() == torch::kBFloat16) return kBF16;
  TORCH_CHECK(false, "codec: tensor must be fp32, fp16 or bf16");
  return -1;
}
}  // namespace

// x: contiguous CUDA tensor, last axis D. fmt: 0 int4_sym, 1 int4_sym_block, 2 int2_sym,
// 3 nvfp4. geom = {S, T, HD, BT} for int4_sym_block. Scratch/outputs sized by the caller.
void codec_encode(torch::Tensor x, int64_t fmt, std::vector<int64_t> geom, torch::Tensor out, torch::Tensor amax,
                  c10::optional<torch::Tensor> scale32, c10::optional<torch::Tensor> scale16,
                  c10::optional<torch::Tensor> sbytes) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() >= 1, "codec_encode: contiguous CUDA input");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kUInt8 && out.is_contiguous(), "codec_encode: uint8 out");
  TORCH_CHECK(amax.is_cuda() && amax.scalar_type() == torch::kFloat32, "codec_encode: fp32 amax scratch");
  EncodeCall c{};
  c.x = x.data_ptr();
  c.dtype = dtype_of(x);
  c.D = static_cast<int>(x.size(-1));
  c.rows = x.numel() / std::max<int64_t>(1, c.D);
  c.fmt = static_cast<int>(fmt);
  c.out = out.data_ptr<uint8_t>();
  c.amax = amax.data_ptr<float>();
  if (fmt != kNvfp4) {
    TORCH_CHECK(scale32.has_value() && scale16.has_value() && scale32->scalar_type() == torch::kFloat32 &&
                    scale16->scalar_type() == torch::kFloat16,
                "codec_encode: scale32 fp32 / scale16 fp16");
    c.scale32 = scale32->data_ptr<float>();
    c.scale16 = reinterpret_cast<__half*>(scale16->data_ptr());
  } else {
    TORCH_CHECK(sbytes.has_value() && sbytes->scalar_type() == torch::kUInt8, "codec_encode: nvfp4 scale bytes");
    c.sbytes = sbytes->data_ptr<uint8_t>();
  }
  if (fmt == kInt4Block) {
    TORCH_CHECK(geom.size() == 4, "codec_encode: int4_sym_block needs {S, T, HD, BT}");
    c.S = geom[0]; c.T = geom[1]; c.HD = geom[2]; c.BT = geom[3];
  }
  const std::string msg = encode(c, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(msg.empty(), "codec_encode: ", msg);
}

void codec_decode(torch::Tensor in, int64_t fmt, std::vector<int64_t> geom, torch::Tensor out,
                  c10::optional<torch::Tensor> scale16, c10::optional<torch::Tensor> sbytes) {
  TORCH_CHECK(in.is_cuda() && in.scalar_type() == torch::kUInt8 && in.is_contiguous(), "codec_decode: uint8 codes");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "codec_decode: contiguous CUDA out");
  DecodeCall c{};
  c.in = in.data_ptr<uint8_t>();
  c.dtype = dtype_of(out);
  c.D = static_cast<int>(out.size(-1));
  c.rows = out.numel() / std::max<int64_t>(1, c.D);
  c.fmt = static_cast<int>(fmt);
  c.out = out.data_ptr();
  if (fmt != kNvfp4) {
    TORCH_CHECK(scale16.has_value() && scale16->scalar_type() == torch::kFloat16, "codec_decode: fp16 scales");
    c.scale16 = reinterpret_cast<const __half*>(scale16->data_ptr());
  } else {
    TORCH_CHECK(sbytes.has_value() && sbytes->scalar_type() == torch::kUInt8, "codec_decode: nvfp4 scale bytes");
    c.sbytes = sbytes->data_ptr<uint8_t>();
  }
  if (fmt == kInt4Block) {
    TORCH_CHECK(geom.size() == 4, "codec_decode: int4_sym_block needs {S, T, HD, BT}");
    c.S = geom[0]; c.T = geom[1]; c.HD = geom[2]; c.BT = geom[3];
  }
  const std::string msg = decode(c, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(msg.empty(), "codec_decode: ", msg);
}

}  // namespace codec
}  // namespace axr
