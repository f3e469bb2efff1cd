// Internal host interface between the library's translation units.
//
// sm100_marlin.cu (the C ABI and the launch planning) calls the launch
// functions declared here; their definitions (launch_impl.cuh) are compiled
// and explicitly instantiated in the k_*.cu files, several translation units
// that nvcc builds in parallel.  Nothing here is exported from the library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "marlin24_decode_tc.cuh"
#include "marlin24_gemm.cuh"
#include "marlin24_prefill.cuh"

namespace sm100 {

// Records the CUDA error text (returned by sm100_marlin_last_cuda_error on
// this thread) and returns SM100_MARLIN_ERR_CUDA.
int cuda_fail(cudaError_t e);

// One launch of the decode kernel (marlin24_gemm.cuh) on `grid` CTAs.
template <int NC, int MB, int NH, bool META3, bool GROUPED, bool EPI, int DIAG>
int launch_decode(const GemmParams& p, int grid, int dev, cudaStream_t stream);

// One launch of the tensor-memory decode kernel (marlin24_decode_tc.cuh):
// `grid` CTAs in clusters of p.split.
template <int NR, bool META3, bool GROUPED>
int launch_decode_tc(const DecodeTcParams& p, int grid, int dev, cudaStream_t stream);

// Clusters of `split` CTAs (1 CTA per SM) of the tensor-memory decode kernel
// that the device runs at once (0 on error).
int decode_tc_max_clusters(int split, int dev);

// Dense-expansion prefill kernel (marlin24_prefill.cuh).
template <int BN, int NG, bool GROUPED>
int launch_prefill_dense(const PrefillParams& p, int dev, cudaStream_t stream);

// One-CTA structured-sparse prefill kernel (marlin24_prefill_sparse.cuh).
template <int BN, int NG, bool GROUPED>
int launch_prefill_sp(const PrefillParams& p, int dev, cudaStream_t stream);

// CTA-pair structured-sparse prefill kernel (marlin24_prefill_sparse.cuh).
template <int NG, bool GROUPED, bool EPI, bool META3, int DIAG>
int launch_prefill_sp2(const PrefillParams& p, int dev, cudaStream_t stream);

// GPU packer and 3-bit metadata codec (k_misc.cu).
int launch_pack_2_4(const void* w, const void* s, int prob_k, int prob_m, int groupsize, void* B,
                    void* meta, void* s_out, cudaStream_t stream);
int launch_meta3_pack(const void* meta, void* out, int64_t pairs, void* err_count,
                      cudaStream_t stream);
int launch_meta3_unpack(const void* in, void* out, int64_t lanes, cudaStream_t stream);
int launch_meta3_decode_words(const void* in, void* out_high, void* out_low, int64_t n,
                              cudaStream_t stream);

}  // namespace sm100
