// Torch binding of the dense tcgen05 projections (kernels in gemm_dense.cu, which stays
// free of torch headers so it compiles in seconds).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "gemm_dense.h"

namespace axr {
namespace dense {

// x [M, K] bf16, w [N, K] bf16 -> epilogue(x w^T). epi: 0 store, 1 residual (res [M, N],
// may be out), 2 SwiGLU (out [M, N/2]), 3 RoPE + bf16 paged KV write (out = q [M, Hq*128]).
// ws fp32 / cnt int32: scratch (the split-K partials of the stream kernel stay in its
// clusters' shared memory; see dense_stream_workspace). splits <= 0: automatic, else the
// stream kernel's CTAs per weight tile (at most 8, one cluster). force_big: 0 automatic,
// 1 the big-M path at any M, 2 the big-M path on the 1-CTA kernel (not the CTA-pair one).
void dense_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t epi, c10::optional<torch::Tensor> res,
                c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> slots,
                c10::optional<torch::Tensor> cos_sin, int64_t kc, int64_t vc, int64_t blk_stride, int64_t head_stride,
                int64_t Hq, int64_t Hkv, torch::Tensor ws, torch::Tensor cnt, torch::Tensor err, int64_t splits,
                int64_t force_big) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "dense_gemm: CUDA tensors");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16 &&
                  out.scalar_type() == torch::kBFloat16,
              "dense_gemm: bf16 operands");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 &&
                  out.stride(1) == 1,
              "dense_gemm: row-major 2D operands");
  TORCH_CHECK(x.size(1) == w.size(1), "dense_gemm: K mismatch");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == torch::kInt32, "dense_gemm: err int32");
  TORCH_CHECK(ws.scalar_type() == torch::kFloat32 && cnt.scalar_type() == torch::kInt32, "dense_gemm: scratch dtypes");
  const int64_t M = x.size(0), N = w.size(0), K = x.size(1);
  TORCH_CHECK(out.size(0) == M, "dense_gemm: out rows");
  const int64_t width = epi == 2 ? N / 2 : epi == 3 ? Hq * 128 : N;
  TORCH_CHECK(out.size(1) == width, "dense_gemm: out has ", out.size(1), " columns, the epilogue writes ", width);
  DenseCall c{};
  c.x = x.data_ptr();
  c.ldx = x.stride(0);
  c.w = w.data_ptr();
  c.ldw = w.stride(0);
  c.out = out.data_ptr();
  c.ldo = out.stride(0);
  c.M = static_cast<int>(M);
  c.N = static_cast<int>(N);
  c.K = static_cast<int>(K);
  c.epi = static_cast<int>(epi);
  if (epi == 1) {
    TORCH_CHECK(res.has_value() && res->scalar_type() == torch::kBFloat16 && res->dim() == 2 && res->stride(1) == 1 &&
                    res->size(0) == M && res->size(1) == N,
                "dense_gemm residual: bf16 [M, N]");
    c.res = res->data_ptr();
    c.ldr = res->stride(0);
  }
  if (epi == 3) {
    TORCH_CHECK(pos.has_value() && slots.has_value() && cos_sin.has_value(), "dense_gemm RoPE: pos, slots, cos_sin");
    TORCH_CHECK(pos->scalar_type() == torch::kInt32 && slots->scalar_type() == torch::kInt32 && pos->numel() >= M &&
                    slots->numel() >= M && pos->is_cuda() && slots->is_cuda(),
                "dense_gemm RoPE: pos / slots int32 [M]");
    TORCH_CHECK(cos_sin->scalar_type() == torch::kFloat32 && cos_sin->dim() == 2 && cos_sin->size(1) == 128 &&
                    cos_sin->is_contiguous(),
                "dense_gemm RoPE: cos_sin fp32 [P, 128]");
    c.pos = pos->data_ptr<int>();
    c.slots = slots->data_ptr<int>();
    c.cos_sin = cos_sin->data_ptr<float>();
    c.n_pos = static_cast<int>(cos_sin->size(0));
    c.kc = reinterpret_cast<void*>(kc);
    c.vc = reinterpret_cast<void*>(vc);
    c.blk_stride = blk_stride;
    c.head_stride = head_stride;
    c.Hq = static_cast<int>(Hq);
    c.Hkv = static_cast<int>(Hkv);
  }
  c.device = x.device().index();
  const int nt = stream_nt(M);
  if (nt != 0 && !force_big) {
    const int sms = at::cuda::getDeviceProperties(c.device)->multiProcessorCount;
    int s = splits > 0 ? static_cast<int>(splits) : stream_splits(M, N, K, sms);
    s = std::max(1, std::min(std::min(s, static_cast<int>((K + 63) / 64)), stream_max_splits(nt)));
    c.splits = s;
  }
  c.err = err.data_ptr<int>();
  c.force_big = force_big != 0;
  c.force_one_cta = force_big == 2;
  const std::string msg = dense_gemm_launch(c, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(msg.empty(), "dense_gemm: ", msg);
}

int64_t dense_stream_nt(int64_t M) { return stream_nt(M); }

int64_t dense_pair_clusters(int64_t device) { return pair_grid_clusters(static_cast<int>(device)); }

std::vector<int64_t> dense_trace_read() {
  std::vector<unsigned long long> v;
  dense_trace(&v);
  return std::vector<int64_t>(v.begin(), v.end());
}

int64_t dense_stream_splits(int64_t M, int64_t N, int64_t K, int64_t sms) {
  return stream_splits(M, N, K, static_cast<int>(sms));
}

std::vector<int64_t> dense_stream_workspace(int64_t M, int64_t N, int64_t K, int64_t sms) {
  int64_t ws = 0, cnt = 0;
  stream_workspace(M, N, K, static_cast<int>(sms), &ws, &cnt);
  return {ws, cnt};
}

}  // namespace dense
}  // namespace axr
