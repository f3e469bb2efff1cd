// Decode kernel instances: 4-bit metadata, group scales, plain store.
#include "launch_impl.cuh"
namespace sm100 {
SM100_INST_DECODE(false, true, false, 0)
}  // namespace sm100
