// pybind11 binding for the reference's 3-bit metadata codec
// (kernel_experiments/sparse_marlin/metadata_decode/codec.cu), compiled from
// the reference source in place by oracle/build_ref.py.  Test infrastructure
// only: tests/ use it to pin the oracle's codec restatement on the GPU box.
#include <torch/extension.h>

torch::Tensor pack_metadata(torch::Tensor x);
torch::Tensor unpack_metadata(torch::Tensor x);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("pack", &pack_metadata);
  m.def("unpack", &unpack_metadata);
}
