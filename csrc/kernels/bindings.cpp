// Torch bindings of the sm_100a kernels (module axropus_deploy_b200._C).
#include <torch/extension.h>

namespace axr {
void page_transfer(int64_t src_data, int64_t src_meta, std::vector<int64_t> src_strides, int64_t src_fmt,
                   int64_t dst_data, int64_t dst_meta, std::vector<int64_t> dst_strides, int64_t dst_fmt,
                   torch::Tensor src_ids, torch::Tensor dst_ids, int64_t n_lk, int64_t H, int64_t D,
                   int64_t max_ctas);
int64_t decode_num_splits(int64_t batch, int64_t kv_heads, int64_t max_pages, int64_t sms, int64_t fmt);
void decode_attention(torch::Tensor q, int64_t k, int64_t v, int64_t km, int64_t vm, int64_t blk_stride,
                      int64_t head_stride, int64_t mblk_stride, int64_t mhead_stride, int64_t fmt,
                      torch::Tensor block_table, torch::Tensor seq_lens, int64_t Hkv, double scale,
                      int64_t num_splits, int64_t max_pages, torch::Tensor out, torch::Tensor part_o,
                      torch::Tensor part_lse, c10::optional<torch::Tensor> page_start,
                      c10::optional<torch::Tensor> part_o2, c10::optional<torch::Tensor> part_lse2,
                      c10::optional<torch::Tensor> row_of, int64_t S2);
void prefill_attention(torch::Tensor q, int64_t k, int64_t v, int64_t km, int64_t vm, int64_t blk_stride,
                       int64_t head_stride, int64_t mblk_stride, int64_t mhead_stride, int64_t fmt,
                       torch::Tensor block_table, torch::Tensor cu_q, torch::Tensor seq_lens, int64_t Hkv,
                       double scale, int64_t max_q, torch::Tensor out, int64_t num_splits,
                       c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_lse);
void rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w, double eps,
             torch::Tensor out);
void rope_kv_write(torch::Tensor qkv, torch::Tensor pos, torch::Tensor slots, torch::Tensor cos_sin,
                   torch::Tensor q_out, int64_t k, int64_t v, int64_t km, int64_t vm, int64_t blk_stride,
                   int64_t head_stride, int64_t mblk_stride, int64_t mhead_stride, int64_t fmt, int64_t Hq,
                   int64_t Hkv);
void silu_mul(torch::Tensor gate_up, torch::Tensor out);
void argmax_rows(torch::Tensor logits, torch::Tensor out);
void spec_verify(torch::Tensor logits, torch::Tensor draft, torch::Tensor out);
void gemm_tc(torch::Tensor a, torch::Tensor b, torch::Tensor out, c10::optional<torch::Tensor> residual, double alpha,
             torch::Tensor err);
void gemm_tp(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t mode, int64_t rank, int64_t world,
             int64_t rows_per_rank, int64_t epoch, c10::optional<torch::Tensor> peer_a,
             c10::optional<torch::Tensor> staging, c10::optional<torch::Tensor> flags,
             c10::optional<torch::Tensor> ready, c10::optional<torch::Tensor> peer_ready,
             c10::optional<torch::Tensor> peer_recv, c10::optional<torch::Tensor> peer_cnt,
             c10::optional<torch::Tensor> recv, c10::optional<torch::Tensor> cnt, torch::Tensor err);
void prefill_attention_tc(torch::Tensor q, int64_t k, int64_t v, int64_t blk_stride, int64_t head_stride,
                          int64_t num_blocks, torch::Tensor block_table, torch::Tensor cu_q, torch::Tensor seq_lens,
                          int64_t Hkv, double scale, int64_t max_q, torch::Tensor out, torch::Tensor err,
                          int64_t num_splits, c10::optional<torch::Tensor> part_o,
                          c10::optional<torch::Tensor> part_lse, int64_t gqa_pack, int64_t noncausal,
                          c10::optional<torch::Tensor> q_index, int64_t partial_only);
void moe_dispatch(torch::Tensor x, torch::Tensor topk_idx, torch::Tensor topk_w, int64_t E_l, int64_t rank,
                  int64_t world, int64_t epoch, int64_t cap_rows, torch::Tensor pair_pos, torch::Tensor gcount,
                  torch::Tensor grid_bar, torch::Tensor peers, torch::Tensor cnt_all, torch::Tensor cnt_flag,
                  torch::Tensor err);
void moe_gemm(torch::Tensor a, torch::Tensor w, int64_t mode, int64_t E_l, int64_t rank, int64_t world,
              int64_t epoch, torch::Tensor cnt_all, torch::Tensor cnt_flag, torch::Tensor arr_flag,
              c10::optional<torch::Tensor> h, c10::optional<torch::Tensor> recv_meta,
              c10::optional<torch::Tensor> recv_w, c10::optional<torch::Tensor> peer_comb,
              c10::optional<torch::Tensor> peer_comb_flag, torch::Tensor done_ctr, torch::Tensor err);
void moe_combine(torch::Tensor comb, torch::Tensor out, torch::Tensor comb_flag, int64_t world, int64_t epoch,
                 int64_t K, torch::Tensor err);
void peer_allreduce(torch::Tensor x, torch::Tensor out, int64_t rank, int64_t world, torch::Tensor peers,
                    torch::Tensor buf, torch::Tensor flag, torch::Tensor epoch, torch::Tensor bar, int64_t cap,
                    torch::Tensor err);
std::vector<int64_t> prefill_trace_read();
namespace dense {
void dense_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t epi, c10::optional<torch::Tensor> res,
                c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> slots,
                c10::optional<torch::Tensor> cos_sin, int64_t kc, int64_t vc, int64_t blk_stride, int64_t head_stride,
                int64_t Hq, int64_t Hkv, torch::Tensor ws, torch::Tensor cnt, torch::Tensor err, int64_t splits,
                int64_t force_big);
int64_t dense_stream_nt(int64_t M);
int64_t dense_pair_clusters(int64_t device);
std::vector<int64_t> dense_trace_read();
int64_t dense_stream_splits(int64_t M, int64_t N, int64_t K, int64_t sms);
std::vector<int64_t> dense_stream_workspace(int64_t M, int64_t N, int64_t K, int64_t sms);
}  // namespace dense
namespace codec {
void codec_encode(torch::Tensor x, int64_t fmt, std::vector<int64_t> geom, torch::Tensor out, torch::Tensor amax,
                  c10::optional<torch::Tensor> scale32, c10::optional<torch::Tensor> scale16,
                  c10::optional<torch::Tensor> sbytes);
void codec_decode(torch::Tensor in, int64_t fmt, std::vector<int64_t> geom, torch::Tensor out,
                  c10::optional<torch::Tensor> scale16, c10::optional<torch::Tensor> sbytes);
}  // namespace codec
}  // namespace axr

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of axropus_deploy_b200";
  m.def("page_transfer", &axr::page_transfer);
  m.def("decode_num_splits", &axr::decode_num_splits, py::arg("batch"), py::arg("kv_heads"), py::arg("max_pages"),
        py::arg("sms"), py::arg("fmt") = -1);
  m.def("decode_attention", &axr::decode_attention);
  m.def("prefill_attention", &axr::prefill_attention);
  m.def("prefill_attention_tc", &axr::prefill_attention_tc);
  m.def("prefill_trace_read", &axr::prefill_trace_read);
  m.def("rmsnorm", &axr::rmsnorm);
  m.def("rope_kv_write", &axr::rope_kv_write);
  m.def("silu_mul", &axr::silu_mul);
  m.def("argmax_rows", &axr::argmax_rows);
  m.def("spec_verify", &axr::spec_verify);
  m.def("gemm_tc", &axr::gemm_tc);
  m.def("gemm_tp", &axr::gemm_tp);
  m.def("moe_dispatch", &axr::moe_dispatch);
  m.def("peer_allreduce", &axr::peer_allreduce);
  m.def("moe_gemm", &axr::moe_gemm);
  m.def("moe_combine", &axr::moe_combine);
  m.def("dense_gemm", &axr::dense::dense_gemm);
  m.def("dense_stream_nt", &axr::dense::dense_stream_nt);
  m.def("dense_pair_clusters", &axr::dense::dense_pair_clusters);
  m.def("dense_trace_read", &axr::dense::dense_trace_read);
  m.def("dense_stream_splits", &axr::dense::dense_stream_splits);
  m.def("dense_stream_workspace", &axr::dense::dense_stream_workspace);
  m.def("codec_encode", &axr::codec::codec_encode);
  m.def("codec_decode", &axr::codec::codec_decode);
}
