// Definitions of the kernel launch functions declared in launch.cuh.
// Included only by the k_*.cu translation units, each of which explicitly
// instantiates one group of kernel configurations.
#pragma once

#include "../../include/sm100_marlin.h"
#include "launch.cuh"
#include "marlin24_decode_tc.cuh"
#include "marlin24_prefill_sparse.cuh"

namespace sm100 {

// cudaFuncSetAttribute once per (kernel instance, device): the attribute is
// per function and device, and setting it costs host time on every call.
template <typename Kern>
int set_smem_once(Kern kern, int smem, bool (&attr_set)[64], int dev) {
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  return SM100_MARLIN_OK;
}

template <int NC, int MB, int NH, bool META3, bool GROUPED, bool EPI, int DIAG>
int launch_decode(const GemmParams& p, int grid, int dev, cudaStream_t stream) {
  using Cfg = DecodeCfg<NC, MB, META3>;
  static bool attr_set[64] = {};
  auto kern = marlin24_decode_kernel<NC, MB, NH, META3, GROUPED, EPI, DIAG>;
  int rc = set_smem_once(kern, Cfg::SMEM, attr_set, dev);
  if (rc != SM100_MARLIN_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  int na = 1;
  if (p.cluster > 1) {  // cluster split-K: one cluster of p.cluster CTAs per column tile
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = p.cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

template <int NR, bool META3, bool GROUPED>
int launch_decode_tc(const DecodeTcParams& p, int grid, int dev, cudaStream_t stream) {
  using Cfg = DecodeTcCfg<NR, META3>;
  static bool attr_set[64] = {};
  auto kern = marlin24_decode_tc_kernel<NR, META3, GROUPED>;
  int rc = set_smem_once(kern, Cfg::SMEM, attr_set, dev);
  if (rc != SM100_MARLIN_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  ++na;
  if (p.split > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = p.split;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

template <int BN, int NG, bool GROUPED>
int launch_prefill_dense(const PrefillParams& p, int dev, cudaStream_t stream) {
  using Cfg = PrefillCfg<BN, NG>;
  static bool attr_set[64] = {};
  auto kern = marlin24_prefill_kernel<BN, NG, GROUPED>;
  int rc = set_smem_once(kern, Cfg::SMEM, attr_set, dev);
  if (rc != SM100_MARLIN_OK) return rc;
  const dim3 grid(p.N / 128, (p.M + BN - 1) / BN);
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

template <int BN, int NG, bool GROUPED>
int launch_prefill_sp(const PrefillParams& p, int dev, cudaStream_t stream) {
  using Cfg = PrefillSpCfg<BN, NG>;
  static bool attr_set[64] = {};
  auto kern = marlin24_prefill_sp_kernel<BN, NG, GROUPED>;
  int rc = set_smem_once(kern, Cfg::SMEM, attr_set, dev);
  if (rc != SM100_MARLIN_OK) return rc;
  const dim3 grid(p.N / 128, (p.M + BN - 1) / BN);
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

// 2-CTA clusters along the features, grid (N/128, M/256).
template <int NG, bool GROUPED, bool EPI, bool META3, int DIAG>
int launch_prefill_sp2(const PrefillParams& p, int dev, cudaStream_t stream) {
  using Cfg = PrefillSp2Cfg<NG>;
  static bool attr_set[64] = {};
  auto kern = marlin24_prefill_sp2_kernel<NG, GROUPED, EPI, META3, DIAG>;
  int rc = set_smem_once(kern, Cfg::SMEM, attr_set, dev);
  if (rc != SM100_MARLIN_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.N / 128, (p.M + 255) / 256);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

// Explicit instantiation helpers for the k_*.cu files: every decode
// configuration the launcher dispatches to (see dispatch_decode in
// sm100_marlin.cu) for one (META3, GROUPED, EPI, DIAG).
#define SM100_INST_DECODE_ONE(NC_, MB_, NH_, META3_, GROUPED_, EPI_, DIAG_)        \
  template int launch_decode<NC_, MB_, NH_, META3_, GROUPED_, EPI_, DIAG_>(        \
      const GemmParams&, int, int, cudaStream_t);
#define SM100_INST_DECODE_NC(NC_, META3_, GROUPED_, EPI_, DIAG_)    \
  SM100_INST_DECODE_ONE(NC_, 1, 1, META3_, GROUPED_, EPI_, DIAG_)   \
  SM100_INST_DECODE_ONE(NC_, 1, 2, META3_, GROUPED_, EPI_, DIAG_)   \
  SM100_INST_DECODE_ONE(NC_, 2, 2, META3_, GROUPED_, EPI_, DIAG_)   \
  SM100_INST_DECODE_ONE(NC_, 4, 2, META3_, GROUPED_, EPI_, DIAG_)
#define SM100_INST_DECODE(META3_, GROUPED_, EPI_, DIAG_) \
  SM100_INST_DECODE_NC(1, META3_, GROUPED_, EPI_, DIAG_) \
  SM100_INST_DECODE_NC(2, META3_, GROUPED_, EPI_, DIAG_) \
  SM100_INST_DECODE_NC(4, META3_, GROUPED_, EPI_, DIAG_)

}  // namespace sm100
