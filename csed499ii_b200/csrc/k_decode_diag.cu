// Decode kernel instances of the metadata-cost diagnostics (uniform-metadata
// ablations; see kDiagNoGmem / kDiagNoReg in marlin24_gemm.cuh).
#include "launch_impl.cuh"
namespace sm100 {
SM100_INST_DECODE(false, true, false, kDiagNoGmem)
SM100_INST_DECODE(false, true, false, kDiagNoReg)
SM100_INST_DECODE(false, true, false, kDiagNoGmem | kDiagNoReg)
}  // namespace sm100
