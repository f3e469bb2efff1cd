// Decode kernel instances: 3-bit metadata, plain store.
#include "launch_impl.cuh"
namespace sm100 {
SM100_INST_DECODE(true, true, false, 0)
SM100_INST_DECODE(true, false, false, 0)
}  // namespace sm100
