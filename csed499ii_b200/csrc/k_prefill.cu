// Prefill kernel instances: the dense-expansion kernel (K not a multiple of
// 128) and, in tuning builds only, the one-CTA structured-sparse kernel
// (both scale modes, every batch tile and group count the launcher picks).
#include "launch_impl.cuh"
#ifndef SM100_MARLIN_TUNING
#define SM100_MARLIN_TUNING 0
#endif
namespace sm100 {
#if SM100_MARLIN_TUNING
#define SM100_INST_PREFILL_SP(BN_, NG_)                                                        \
  template int launch_prefill_sp<BN_, NG_, true>(const PrefillParams&, int, cudaStream_t);     \
  template int launch_prefill_sp<BN_, NG_, false>(const PrefillParams&, int, cudaStream_t);
#else
#define SM100_INST_PREFILL_SP(BN_, NG_)
#endif
#define SM100_INST_PREFILL(BN_, NG_)                                                          \
  template int launch_prefill_dense<BN_, NG_, true>(const PrefillParams&, int, cudaStream_t);  \
  template int launch_prefill_dense<BN_, NG_, false>(const PrefillParams&, int, cudaStream_t); \
  SM100_INST_PREFILL_SP(BN_, NG_)
SM100_INST_PREFILL(128, 1)
SM100_INST_PREFILL(128, 2)
SM100_INST_PREFILL(128, 4)
SM100_INST_PREFILL(256, 1)
SM100_INST_PREFILL(256, 2)
SM100_INST_PREFILL(256, 4)
#undef SM100_INST_PREFILL
#undef SM100_INST_PREFILL_SP
}  // namespace sm100
