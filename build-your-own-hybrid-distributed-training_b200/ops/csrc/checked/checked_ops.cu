// Bounds-checked build of the element-wise, optimizer and normalisation kernels (module _C_checked).
//
// The same sources as the regular extension, compiled as one translation unit with
// HT_BOUNDS_CHECK defined: every guarded index is compared with the extent of the buffer it
// addresses (HT_IN_BOUNDS in common.cuh), and a violation is recorded in this module's error word
// instead of being performed.  Tests run the checked kernels on the regular tests' inputs, compare
// their outputs with the regular build and require the word to stay zero.  It stands in for a
// memory checker where compute-sanitizer is not available.
#define HT_BOUNDS_CHECK 1

#include "../elementwise.cu"
#include "../norm.cu"
#include "../optim.cu"

namespace ht {

// (flag, code, index, extent) of the first out-of-bounds access a checked kernel skipped.
std::vector<int64_t> bounds_status() {
  long long host[4] = {0, 0, 0, 0};
  HT_CUDA_CHECK(cudaMemcpyFromSymbol(host, ht_bounds_word, sizeof(host)));
  return {host[0], host[1], host[2], host[3]};
}

void bounds_reset() {
  const long long zero[4] = {0, 0, 0, 0};
  HT_CUDA_CHECK(cudaMemcpyToSymbol(ht_bounds_word, zero, sizeof(zero)));
}

}  // namespace ht

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("bounds_status", &ht::bounds_status, "(flag, code, index, extent) of the first skipped out-of-bounds access");
  m.def("bounds_reset", &ht::bounds_reset);
  m.def("gelu_backward", &ht::gelu_backward);
  m.def("swiglu_forward", &ht::swiglu_forward);
  m.def("swiglu_backward", &ht::swiglu_backward);
  m.def("column_sum", &ht::column_sum);
  m.def("embedding_forward", &ht::embedding_forward);
  m.def("embedding_backward", &ht::embedding_backward);
  m.def("rope_", &ht::rope_);
  m.def("norm_forward", &ht::norm_forward);
  m.def("norm_backward", &ht::norm_backward);
  m.def("norm_backward_blocks", &ht::norm_backward_blocks);
  m.def("sum_rows", &ht::sum_rows);
  m.def("sum_rows_pair", &ht::sum_rows_pair);
  m.def("adamw_flat", &ht::adamw_flat);
}
