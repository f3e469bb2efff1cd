// Decode kernel instances: 3-bit metadata, fused bias / activation epilogue.
#include "launch_impl.cuh"
namespace sm100 {
SM100_INST_DECODE(true, true, true, 0)
SM100_INST_DECODE(true, false, true, 0)
}  // namespace sm100
