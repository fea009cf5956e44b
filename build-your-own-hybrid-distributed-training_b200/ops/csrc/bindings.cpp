// Python bindings of the native sm_100a kernels (module hybrid_training.ops._C).
#include <torch/extension.h>

namespace ht {
void set_deterministic_reductions(bool on);
void set_gemm_pair(int64_t mode);
bool deterministic_reductions();
void gemm(at::Tensor a, at::Tensor b, at::Tensor d, c10::optional<at::Tensor> bias, c10::optional<at::Tensor> aux,
          c10::optional<at::Tensor> alpha, bool a_mn_major, bool b_mn_major, int64_t epilogue, double beta);
void gemm_swiglu(at::Tensor a, at::Tensor b, at::Tensor h, at::Tensor out, c10::optional<at::Tensor> bias, bool backward);
at::Tensor gemm_error_word(at::Tensor like);
void gemm_collective(at::Tensor a, at::Tensor b, at::Tensor d, c10::optional<at::Tensor> bias, c10::optional<at::Tensor> aux,
                     bool a_mn_major, bool b_mn_major, int64_t epilogue, double beta, int64_t a_mode, std::vector<int64_t> a_ptrs,
                     int64_t b_mode, std::vector<int64_t> b_ptrs, int64_t rs, std::vector<int64_t> out_ptrs, at::Tensor flags_local,
                     std::vector<int64_t> flag_ptrs, at::Tensor counters, int64_t site, int64_t advance, int64_t rank,
                     double timeout_s, c10::optional<at::Tensor> gathered, c10::optional<at::Tensor> block_flags);
void reduce_scatter_sum(at::Tensor recv, at::Tensor out, at::Tensor flags_local, at::Tensor counters, int64_t site, int64_t rank,
                        double timeout_s);
at::Tensor attention_error_word_tensor(at::Tensor like);
void norm_forward(at::Tensor res, c10::optional<at::Tensor> delta, at::Tensor w, c10::optional<at::Tensor> b, at::Tensor r_out,
                  at::Tensor y, at::Tensor mean, at::Tensor rstd, double eps, bool rms);
void norm_backward(c10::optional<at::Tensor> dy, c10::optional<at::Tensor> dr, at::Tensor r, at::Tensor w, at::Tensor mean,
                   at::Tensor rstd, at::Tensor dres, c10::optional<at::Tensor> ddelta, at::Tensor part_w,
                   c10::optional<at::Tensor> part_b, bool rms);
int64_t norm_backward_blocks(int64_t rows);
void sum_rows_pair(at::Tensor part_a, at::Tensor out_a, double beta_a, at::Tensor part_b, at::Tensor out_b, double beta_b);
void exp2_poly_eval(at::Tensor x, at::Tensor poly, at::Tensor mufu);
void sum_rows(at::Tensor part, at::Tensor out, double beta);
void gelu_backward(at::Tensor g, at::Tensor pre, at::Tensor out);
void swiglu_forward(at::Tensor h, at::Tensor out);
void swiglu_backward(at::Tensor h, at::Tensor g, at::Tensor dh);
void column_sum(at::Tensor x, at::Tensor out, double beta);
void embedding_forward(at::Tensor ids, at::Tensor table, c10::optional<at::Tensor> pos, at::Tensor out, int64_t vocab_start);
void embedding_backward(at::Tensor ids, at::Tensor grad, at::Tensor dtable, int64_t vocab_start);
void sum_batch_into(at::Tensor grad, at::Tensor out, double beta);
void rope_(at::Tensor x, at::Tensor cosv, at::Tensor sinv, int64_t heads, int64_t hd, bool inverse);
void cross_entropy_fused(at::Tensor logits, at::Tensor targets, at::Tensor grad, at::Tensor loss, int64_t vocab_start, double scale);
void cross_entropy_stats(at::Tensor logits, at::Tensor targets, at::Tensor stats, int64_t vocab_start);
void cross_entropy_combine(at::Tensor gathered, at::Tensor lse, at::Tensor loss, int64_t world, double scale);
void cross_entropy_grad(at::Tensor logits, at::Tensor targets, at::Tensor lse, at::Tensor grad, int64_t vocab_start, double scale);
void adamw_flat(at::Tensor param, at::Tensor grad, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> copy, at::Tensor hyper,
                double beta1, double beta2, double eps, double wd, bool resident);
void grad_sumsq(at::Tensor g, c10::optional<at::Tensor> w, at::Tensor out, double scale);
void attention_forward(at::Tensor qkv, at::Tensor out, at::Tensor lse, int64_t H, int64_t HKV, int64_t D, bool causal, double scale,
                       int64_t q_begin, int64_t q_len);
void attention_backward(at::Tensor qkv, at::Tensor out, at::Tensor dout, at::Tensor lse, at::Tensor delta, at::Tensor dqkv,
                        int64_t H, int64_t HKV, int64_t D, bool causal, double scale, int64_t q_begin, int64_t q_len);
void bucket_all_reduce(at::Tensor flat, std::vector<int64_t> buffer_ptrs, std::vector<int64_t> pad_ptrs, int64_t multicast_ptr,
                       int64_t start, int64_t numel, double scale, int64_t rank, int64_t slot_base, int64_t max_blocks,
                       at::Tensor status, double timeout_s, bool wide, int64_t min_peer_slots);
void fsdp_reduce_scatter_adamw(at::Tensor staging, std::vector<int64_t> grad_ptrs, std::vector<int64_t> pad_ptrs, int64_t rank,
                               int64_t shard, int64_t valid, double scale, at::Tensor param, at::Tensor exp_avg,
                               at::Tensor exp_avg_sq, at::Tensor shard16, c10::optional<at::Tensor> grad_out, at::Tensor hyper,
                               double beta1, double beta2, double eps, double wd, int64_t slot_base, int64_t max_blocks,
                               at::Tensor status, double timeout_s, int64_t slice);
void fsdp_all_gather(std::vector<int64_t> shard_ptrs, at::Tensor out, int64_t shard, int64_t rank);
void barrier_probe(at::Tensor pads, at::Tensor status, double timeout_s);
void fsdp_all_gather_copy_engine(std::vector<int64_t> shard_ptrs, at::Tensor out, int64_t shard, int64_t rank);
}  // namespace ht

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "hybrid_training native kernels (sm_100a)";
  m.def("gemm", &ht::gemm, "tcgen05 GEMM with fused epilogue");
  m.def("set_gemm_pair", &ht::set_gemm_pair, "1: CTA-pair (cta_group::2) tiles for eligible GEMMs, 0: single-CTA tiles only");
  m.def("gemm_swiglu", &ht::gemm_swiglu, "tcgen05 GEMM with the SwiGLU activation (or its gradient) in the epilogue");
  m.def("gemm_error_word", &ht::gemm_error_word, "device error word written by timed-out GEMM waits");
  m.def("gemm_collective", &ht::gemm_collective, "GEMM with peer-sharded operands or a reduce-scatter epilogue");
  m.def("reduce_scatter_sum", &ht::reduce_scatter_sum, "sum of the reduce-scatter receive slots");
  m.def("attention_error_word", &ht::attention_error_word_tensor, "device error word written by timed-out attention waits");
  m.def("norm_forward", &ht::norm_forward);
  m.def("norm_backward", &ht::norm_backward);
  m.def("norm_backward_blocks", &ht::norm_backward_blocks);
  m.def("sum_rows_pair", &ht::sum_rows_pair, "two column reductions (a norm's weight and bias gradients) in one launch");
  m.def("exp2_poly_eval", &ht::exp2_poly_eval, "the FMA-pipe 2^x of the attention softmax next to exp2f (tests)");
  m.def("sum_rows", &ht::sum_rows);
  m.def("gelu_backward", &ht::gelu_backward);
  m.def("swiglu_forward", &ht::swiglu_forward);
  m.def("swiglu_backward", &ht::swiglu_backward);
  m.def("column_sum", &ht::column_sum);
  m.def("embedding_forward", &ht::embedding_forward);
  m.def("embedding_backward", &ht::embedding_backward);
  m.def("sum_batch_into", &ht::sum_batch_into);
  m.def("rope_", &ht::rope_);
  m.def("cross_entropy_fused", &ht::cross_entropy_fused);
  m.def("cross_entropy_stats", &ht::cross_entropy_stats);
  m.def("cross_entropy_combine", &ht::cross_entropy_combine);
  m.def("cross_entropy_grad", &ht::cross_entropy_grad);
  m.def("adamw_flat", &ht::adamw_flat);
  m.def("set_deterministic_reductions", &ht::set_deterministic_reductions,
        "fixed-order split-K sums (reproducible) or TMA reduce-adds straight into the output (faster)");
  m.def("deterministic_reductions", &ht::deterministic_reductions);
  m.def("grad_sumsq", &ht::grad_sumsq);
  m.def("attention_forward", &ht::attention_forward, py::arg("qkv"), py::arg("out"), py::arg("lse"), py::arg("H"), py::arg("HKV"),
        py::arg("D"), py::arg("causal"), py::arg("scale"), py::arg("q_begin") = 0, py::arg("q_len") = -1);
  m.def("attention_backward", &ht::attention_backward, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"),
        py::arg("delta"), py::arg("dqkv"), py::arg("H"), py::arg("HKV"), py::arg("D"), py::arg("causal"), py::arg("scale"),
        py::arg("q_begin") = 0, py::arg("q_len") = -1);
  m.def("bucket_all_reduce", &ht::bucket_all_reduce, "in-kernel NVLink all-reduce of one DDP bucket");
  m.def("fsdp_reduce_scatter_adamw", &ht::fsdp_reduce_scatter_adamw,
        "FSDP gradient reduce-scatter fused with the cast and the sharded AdamW update (NVLink peer memory)");
  m.def("barrier_probe", &ht::barrier_probe, "one block running the bounded peer barrier against local pads (tests)");
  m.def("fsdp_all_gather", &ht::fsdp_all_gather, "FSDP all-gather of bf16 parameter shards over NVLink peer memory");
  m.def("fsdp_all_gather_copy_engine", &ht::fsdp_all_gather_copy_engine, "FSDP all-gather by one peer cudaMemcpyAsync per rank");
}
