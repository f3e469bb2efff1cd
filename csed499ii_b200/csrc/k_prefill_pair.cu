// CTA-pair prefill kernel instances (tcgen05.mma.sp.cta_group::2): both scale
// modes, with and without the fused epilogue, 4- and 3-bit metadata, and the
// metadata-cost diagnostics.
#include "launch_impl.cuh"
namespace sm100 {
#define SM100_INST_PAIR(NG_, G_, E_, M3_, D_) \
  template int launch_prefill_sp2<NG_, G_, E_, M3_, D_>(const PrefillParams&, int, cudaStream_t);
#define SM100_INST_PAIR_NG(NG_)              \
  SM100_INST_PAIR(NG_, true, false, false, 0)  \
  SM100_INST_PAIR(NG_, true, true, false, 0)   \
  SM100_INST_PAIR(NG_, false, false, false, 0) \
  SM100_INST_PAIR(NG_, false, true, false, 0)
SM100_INST_PAIR_NG(1)
SM100_INST_PAIR_NG(2)
SM100_INST_PAIR_NG(4)
SM100_INST_PAIR(4, true, false, true, 0)
SM100_INST_PAIR(4, true, true, true, 0)
SM100_INST_PAIR(4, false, false, true, 0)
SM100_INST_PAIR(4, false, true, true, 0)
SM100_INST_PAIR(4, true, false, false, kDiagNoGmem)
SM100_INST_PAIR(4, true, false, false, kDiagNoReg)
SM100_INST_PAIR(4, true, false, false, kDiagNoGmem | kDiagNoReg)
#undef SM100_INST_PAIR_NG
#undef SM100_INST_PAIR
}  // namespace sm100
