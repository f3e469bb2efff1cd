// Tensor-memory decode kernel instances (marlin24_decode_tc.cuh): batch tiles
// of 16/32/48/64 rows, 4- and 3-bit metadata, both scale modes; and the
// cluster-occupancy query the launcher plans with.
#include "launch_impl.cuh"
namespace sm100 {
#define SM100_INST_TC(NR_)                                                                      \
  template int launch_decode_tc<NR_, false, true>(const DecodeTcParams&, int, int, cudaStream_t);  \
  template int launch_decode_tc<NR_, false, false>(const DecodeTcParams&, int, int, cudaStream_t); \
  template int launch_decode_tc<NR_, true, true>(const DecodeTcParams&, int, int, cudaStream_t);   \
  template int launch_decode_tc<NR_, true, false>(const DecodeTcParams&, int, int, cudaStream_t);
SM100_INST_TC(16)
SM100_INST_TC(32)
SM100_INST_TC(48)
SM100_INST_TC(64)
#undef SM100_INST_TC

// Clusters of `split` CTAs of the kernel (one CTA per SM) that run at once;
// the planner launches at most that many, so that a call runs in one wave.
int decode_tc_max_clusters(int split, int dev) {
  static int cache[64][5] = {};
  if (dev >= 0 && dev < 64 && split >= 1 && split <= 4 && cache[dev][split] > 0)
    return cache[dev][split];
  auto kern = marlin24_decode_tc_kernel<16, false, true>;
  const int smem = DecodeTcCfg<16, false>::SMEM;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (split == 1) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    n = sms;
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(split * 64);
    cfg.blockDim = dim3(DecodeTcCfg<16, false>::THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
  }
  if (dev >= 0 && dev < 64 && split >= 1 && split <= 4) cache[dev][split] = n;
  return n;
}
}  // namespace sm100
