// Prefill kernel instances: the dense-expansion kernel and the one-CTA
// structured-sparse kernel (both scale modes, every batch tile and group
// count the launcher picks).
#include "launch_impl.cuh"
namespace sm100 {
#define SM100_INST_PREFILL(BN_, NG_)                                                          \
  template int launch_prefill_dense<BN_, NG_, true>(const PrefillParams&, int, cudaStream_t);  \
  template int launch_prefill_dense<BN_, NG_, false>(const PrefillParams&, int, cudaStream_t); \
  template int launch_prefill_sp<BN_, NG_, true>(const PrefillParams&, int, cudaStream_t);     \
  template int launch_prefill_sp<BN_, NG_, false>(const PrefillParams&, int, cudaStream_t);
SM100_INST_PREFILL(128, 1)
SM100_INST_PREFILL(128, 2)
SM100_INST_PREFILL(128, 4)
SM100_INST_PREFILL(256, 1)
SM100_INST_PREFILL(256, 2)
SM100_INST_PREFILL(256, 4)
#undef SM100_INST_PREFILL
}  // namespace sm100
