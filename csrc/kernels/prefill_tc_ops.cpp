// Torch binding of the tcgen05 prefill attention (kernel in prefill_tc.cu, which stays free
// of torch headers so it compiles in seconds).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "prefill_tc.h"

namespace axr {

// q [T, Hq, 128] bf16; k/v: the layer's bf16 K and V page regions ([num_blocks, Hkv, 16, 128]
// each, contiguous); block_table [B, max_blocks] int32; cu_q [B+1]; seq_lens [B]; err int32.
void prefill_attention_tc(torch::Tensor q, int64_t k, int64_t v, int64_t blk_stride, int64_t head_stride,
                          int64_t num_blocks, torch::Tensor block_table, torch::Tensor cu_q, torch::Tensor seq_lens,
                          int64_t Hkv, double scale, int64_t max_q, torch::Tensor out, torch::Tensor err,
                          int64_t num_splits, c10::optional<torch::Tensor> part_o,
                          c10::optional<torch::Tensor> part_lse, int64_t gqa_pack, int64_t noncausal,
                          c10::optional<torch::Tensor> q_index, int64_t partial_only) {
  constexpr int HD = 128;
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.is_contiguous() && q.dim() == 3 &&
                  q.size(2) == HD,
              "prefill_tc: q must be contiguous bf16 [T, Hq, 128]");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == torch::kBFloat16, "prefill_tc: out must be contiguous bf16");
  TORCH_CHECK(blk_stride == Hkv * 16 * HD * 2 && head_stride == 16 * HD * 2,
              "prefill_tc: expects contiguous bf16 pages [blocks, Hkv, 16, 128]");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && cu_q.scalar_type() == torch::kInt32 &&
                  seq_lens.scalar_type() == torch::kInt32 && err.scalar_type() == torch::kInt32,
              "prefill_tc: index tensors must be int32");
  const int B = seq_lens.size(0), Hq = q.size(1), T = q.size(0);
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  const int S = static_cast<int>(std::max<int64_t>(1, num_splits));
  fa::PrefillCall c{};
  c.q = q.data_ptr();
  c.out = out.data_ptr();
  c.T = T;
  c.Hq = Hq;
  c.Hkv = static_cast<int>(Hkv);
  c.k = reinterpret_cast<const void*>(k);
  c.v = reinterpret_cast<const void*>(v);
  c.num_blocks = num_blocks;
  c.block_table = block_table.data_ptr<int>();
  c.bt_stride = static_cast<int>(block_table.stride(0));
  c.cu_q = cu_q.data_ptr<int>();
  c.seq_lens = seq_lens.data_ptr<int>();
  c.B = B;
  c.max_q = static_cast<int>(max_q);
  c.scale = static_cast<float>(scale);
  c.err = err.data_ptr<int>();
  c.num_splits = S;
  c.gqa_pack = static_cast<int>(gqa_pack);
  c.noncausal = static_cast<int>(noncausal);
  c.partial_only = static_cast<int>(partial_only);
  // rows of the partials: q rows, or the q_index rows (shared-prefix decode)
  const int64_t R = q_index.has_value() ? q_index->numel() : T;
  if (q_index.has_value()) {
    TORCH_CHECK(q_index->is_cuda() && q_index->scalar_type() == torch::kInt32, "prefill_tc: q_index int32");
    c.q_index = q_index->data_ptr<int>();
  }
  if (S > 1 || partial_only) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value() && part_o->scalar_type() == torch::kFloat32 &&
                    part_lse->scalar_type() == torch::kFloat32 &&
                    part_o->numel() >= R * Hq * S * HD && part_lse->numel() >= R * Hq * S,
                "prefill_tc: split-KV scratch too small");
    c.part_o = part_o->data_ptr<float>();
    c.part_lse = part_lse->data_ptr<float>();
  }
  const std::string msg = fa::prefill_launch(c, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(msg.empty(), "prefill_tc: ", msg);
}

std::vector<int64_t> prefill_trace_read() {
  std::vector<long long> v(12 * 128, 0);
  const int n = fa::prefill_trace(v.data(), static_cast<int>(v.size()));
  if (n <= 0) return {};
  return std::vector<int64_t>(v.begin(), v.begin() + n);
}

}  // namespace axr
