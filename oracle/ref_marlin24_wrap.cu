// C-ABI wrapper around the reference's own Sparse-Marlin 2:4 launcher,
// compiled from the reference sources in place (never copied) by
// oracle/build_ref.py into oracle/_ref/libref_marlin24.so.
//
// Test infrastructure only: used by tests/ to pin the oracle against the
// reference kernel running on the B200 and to time that kernel beside this
// library's.  REF_NM_CU is the path of
// kernel_experiments/sparse_marlin/src/marlin/marlin_cuda_kernel_nm.cu.
#include REF_NM_CU

extern "C" int ref_marlin_cuda_2_4(const void* A, const void* B, const void* meta, void* C,
                                   void* s, int prob_m, int prob_n, int prob_k, void* workspace,
                                   int groupsize, int dev, void* stream, int thread_k,
                                   int thread_m, int sms, int max_par) {
  return marlin::marlin_cuda_2_4(A, B, meta, C, s, prob_m, prob_n, prob_k, workspace, groupsize,
                                 dev, reinterpret_cast<cudaStream_t>(stream), thread_k, thread_m,
                                 sms, max_par);
}
