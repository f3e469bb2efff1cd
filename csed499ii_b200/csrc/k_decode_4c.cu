// Decode kernel instances: 4-bit metadata, one scale per column, plain store.
#include "launch_impl.cuh"
namespace sm100 {
SM100_INST_DECODE(false, false, false, 0)
}  // namespace sm100
