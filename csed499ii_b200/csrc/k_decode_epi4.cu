// Decode kernel instances: 4-bit metadata, fused bias / activation epilogue.
#include "launch_impl.cuh"
namespace sm100 {
SM100_INST_DECODE(false, true, true, 0)
SM100_INST_DECODE(false, false, true, 0)
}  // namespace sm100
