/*
 * C ABI of the sm_100a 2:4 sparse W4A16 GEMM library (libsm100_marlin.so).
 *
 * Drop-in for the CUDA entry points of hyeonu453/CSED499II's Sparse-Marlin
 * path.  Plain pointers and sizes only; every function returns an int status
 * (0 = success, see SM100_MARLIN_* below) and never throws.  Streams are
 * passed as `void*` holding a cudaStream_t (NULL = legacy default stream).
 *
 * Naming: `prob_m` is the number of OUTPUT FEATURES (N), `prob_n` the number
 * of BATCH ROWS (M) and `prob_k` the number of input features (K), exactly as
 * the reference launcher names them.
 */
#ifndef SM100_MARLIN_H_
#define SM100_MARLIN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  1 and 2 have the meaning of the reference's ERR_PROB_SHAPE /
 * ERR_KERN_SHAPE (kernel_experiments/sparse_marlin/src/marlin/
 * marlin_cuda_kernel_nm.cu:748-749). */
#define SM100_MARLIN_OK 0
#define SM100_MARLIN_ERR_PROB_SHAPE 1
#define SM100_MARLIN_ERR_KERN_SHAPE 2
#define SM100_MARLIN_ERR_CUDA 3
#define SM100_MARLIN_ERR_ALIGNMENT 4
#define SM100_MARLIN_ERR_ARGUMENT 5
#define SM100_MARLIN_ERR_SCRATCH 6

/* Bits of the device status word (sm100_marlin_device_status). */
#define SM100_MARLIN_STATUS_FULL_WAIT_TIMEOUT 1
#define SM100_MARLIN_STATUS_EMPTY_WAIT_TIMEOUT 2
#define SM100_MARLIN_STATUS_FINISH_WAIT_TIMEOUT 4
#define SM100_MARLIN_STATUS_GATHER_WAIT_TIMEOUT 8

/* Fused-epilogue activations (sm100_marlin_mul_2_4_epilogue). */
#define SM100_MARLIN_ACT_NONE 0
#define SM100_MARLIN_ACT_RELU 1
#define SM100_MARLIN_ACT_SILU 2      /* x * sigmoid(x) */
#define SM100_MARLIN_ACT_GELU_TANH 3 /* 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) */

/*
 * C[prob_n, prob_m] (fp16, row-major) = A[prob_n, prob_k] (fp16, row-major)
 *     x dequant(B, meta, s)[prob_k, prob_m].
 *
 * Replaces `int marlin::marlin_cuda_2_4(const void*A, const void*B, const
 * void*meta, void*C, void*s, int prob_m, int prob_n, int prob_k, void*
 * workspace, int groupsize, int dev, cudaStream_t stream, int thread_k, int
 * thread_m, int sms, int max_par)` (marlin_cuda_kernel_nm.cu:751-755, bound by
 * marlin_cuda.cpp:25-29), with the same arguments and validation:
 *   B          int32 (prob_k/32, 2*prob_m), Sparse-Marlin packed INT4 nonzeros
 *   meta       int16 (prob_m, prob_k/16), reordered 2:4 metadata
 *   s          fp16 (prob_k/128, prob_m) group scales, or (1, prob_m)
 *   workspace  int32 array of >= prob_m/128*max_par entries, all zero on
 *              entry; left all zero on exit
 *   groupsize  compressed group size prob_k/2/s_rows (64 for 128-wide groups)
 *              or -1 for one scale per column
 *   thread_k, thread_m  -1 (auto) or one of the reference tiles (128,128)
 *              for prob_n <= 16 and (64,256); they only select the reference's
 *              shape checks, the B200 kernel picks its own tiling
 *   sms        number of persistent CTAs (-1 = all SMs of `dev`)
 * The call is asynchronous on `stream`.  Split-K scratch is taken from a
 * per-(device, stream) cache owned by the library (allocated on first use; call
 * once before any stream capture).  Concurrent calls on different streams
 * need distinct workspaces, as in the reference.
 */
int sm100_marlin_mul_2_4(const void* A, const void* B, const void* meta, void* C, const void* s,
                         int prob_m, int prob_n, int prob_k, void* workspace, int groupsize,
                         int dev, void* stream, int thread_k, int thread_m, int sms, int max_par);

/*
 * Same GEMM with 3-bit metadata: `meta3` is int32 of prob_m*prob_k*3/128
 * words produced by sm100_marlin_meta3_pack.  Replaces the reference's
 * `metadata_decode.fetch` / `metadata_decode.matmul` variants
 * (kernel_experiments/sparse_marlin/metadata_decode/setup.py:36-51), which
 * accept the same arguments as mul_2_4.
 */
int sm100_marlin_mul_2_4_meta3(const void* A, const void* B, const void* meta3, void* C,
                               const void* s, int prob_m, int prob_n, int prob_k, void* workspace,
                               int groupsize, int dev, void* stream, int thread_k, int thread_m,
                               int sms, int max_par);

/* Split-K scratch bytes needed by a call with these sizes (for _ex). */
size_t sm100_marlin_scratch_bytes(int prob_m, int prob_n, int prob_k, int dev, int sms);

/* mul_2_4 / mul_2_4_meta3 with caller-provided split-K scratch (device memory,
 * 16-byte aligned, >= sm100_marlin_scratch_bytes bytes, contents irrelevant).
 * `meta_bits` is 4 or 3.  No counterpart in the reference: it exists for
 * integrators that manage device memory themselves. */
int sm100_marlin_mul_2_4_ex(const void* A, const void* B, const void* meta, void* C, const void* s,
                            int prob_m, int prob_n, int prob_k, void* workspace, int groupsize,
                            int dev, void* stream, int thread_k, int thread_m, int sms,
                            int max_par, int meta_bits, void* scratch, size_t scratch_bytes);

/*
 * mul_2_4 / mul_2_4_meta3 (`meta_bits` 4 or 3) with a fused epilogue:
 * C = act(A . dequant(B, meta, s) + bias), computed in fp32 and rounded once
 * to fp16.  `bias`: fp16 of prob_m (= N) values, 16-byte aligned, or NULL;
 * `activation`: SM100_MARLIN_ACT_*.  No counterpart in the reference, whose
 * Layer_2_4 is "without bias" (SRC/marlin/__init__.py:275) and whose callers
 * apply bias and activation as separate PyTorch ops; this is the step after
 * the GEMM fused into its store.  Errors as sm100_marlin_mul_2_4, plus
 * SM100_MARLIN_ERR_ARGUMENT for an unknown activation or meta_bits and
 * SM100_MARLIN_ERR_ALIGNMENT for an unaligned bias.
 */
int sm100_marlin_mul_2_4_epilogue(const void* A, const void* B, const void* meta, void* C,
                                  const void* s, int prob_m, int prob_n, int prob_k,
                                  void* workspace, int groupsize, int dev, void* stream,
                                  int thread_k, int thread_m, int sms, int max_par, int meta_bits,
                                  const void* bias, int activation);

/*
 * sm100_marlin_mul_2_4 without any device allocation.  No counterpart in the
 * reference.  The regular entry point gets its split-K scratch from a cache
 * it fills with cudaMalloc on first use; callers that may not allocate device
 * memory at call time -- code running inside CUDA graph capture, serving
 * runtimes and plugins whose host framework owns all device memory, or
 * real-time loops that forbid allocation after start-up -- call this one
 * instead.  Its scratch is a fixed 8 MiB static device buffer inside the
 * library (one per device, kept until the process exits), enough for every
 * call with prob_n (batch rows) <= 16 on up to 148 SMs.  Calls that need more
 * return SM100_MARLIN_ERR_SCRATCH (see sm100_marlin_last_cuda_error).
 * Arguments and results are those of sm100_marlin_mul_2_4.
 * The first call on a device looks up the buffer's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  The address stays cached for the life of the
 * process: after cudaDeviceReset on a device (which destroys the buffer with
 * the context) this entry point must not be used on that device again.  All
 * noalloc calls on a device share the buffer: calls that overlap on the GPU
 * (different streams, no ordering between them) race and must be avoided;
 * calls on one stream are safe.
 */
int sm100_marlin_mul_2_4_noalloc(const void* A, const void* B, const void* meta, void* C,
                                 const void* s, int prob_m, int prob_n, int prob_k,
                                 void* workspace, int groupsize, int dev, void* stream,
                                 int thread_k, int thread_m, int sms, int max_par);

/*
 * Metadata-cost diagnostics: mul_2_4 (4-bit metadata, group-128 scales) with
 * the metadata path partly removed, to measure what it costs.  Replaces the
 * reference's `metadata_diagnostics` extension and its `no_gmem` / `no_reg`
 * / `no_all` kernels (kernel_experiments/sparse_marlin/kernel_profile/
 * setup.py:14-38, driven by run.py:62-70).
 *   variant 1  "no_gmem": no metadata copy from global memory; the kernel's
 *              shared-memory metadata is the constant 0xEEEE from its start
 *   variant 2  "no_reg": metadata copied as usual, but the constant 0xEEEE is
 *              used in place of the shared-memory (or tensor-memory) load
 *   variant 3  "no_all": both
 * The result is only meaningful, and then bit-identical to mul_2_4, when every
 * metadata word of `meta` is 0xEEEE (int16 -4370).  Runs the decode kernel for
 * prob_n <= 64 and the CTA-pair tensor-memory kernel above (prob_m % 256 ==
 * 0).  SM100_MARLIN_ERR_ARGUMENT for another variant or groupsize -1.
 */
int sm100_marlin_mul_2_4_meta_diag(const void* A, const void* B, const void* meta, void* C,
                                   const void* s, int prob_m, int prob_n, int prob_k,
                                   void* workspace, int groupsize, int dev, void* stream,
                                   int variant);

/*
 * Column-parallel GEMM with the all-gather of C fused into its epilogue.  No
 * counterpart in the reference (which has no multi-GPU code); it replaces
 * "local mul_2_4 + all-gather of C" across `world` ranks (one GPU each) that
 * hold column shards of one layer (prob_m columns each, batch prob_n <= 64).
 *   gathered_c[q]  rank q's gathered output, fp16 (prob_n, world*prob_m)
 *                  row-major, mapped into this process (sm100_marlin_ipc_open)
 *   arrival[q]     rank q's uint64 arrival counter for that buffer (zero at
 *                  creation, never reset)
 *   target         this rank's uint64 cumulative target for that buffer (zero
 *                  at creation; the call adds its blocks, world x tiles, on
 *                  the device)
 *   wait_arrival,  the launch ends once *wait_arrival >= *wait_target
 *   wait_target    (bounded wait, SM100_MARLIN_STATUS_GATHER_WAIT_TIMEOUT on
 *                  expiry); both null: no wait
 *   release_arrival  the previous call's arrival counters (all ranks) when
 *                  that call deferred its release, else null
 *   defer          0: every CTA releases its own stores (system-scope fence,
 *                  then its tile count on every rank's counter); 1: this
 *                  call's stores are released later, by the next call
 *                  (release_arrival) or by sm100_marlin_gather_wait, which
 *                  add 1 per rank once this launch has completed
 * Every C row this rank computes is stored into all ranks' gathered buffers
 * (peer stores over NVLink) at column block `rank`.  Completion, chosen by the
 * caller:
 *   - per call (defer = 0, no release_arrival): wait_arrival =
 *     arrival[rank], wait_target = target; the call completes on the stream
 *     once this rank's buffer holds every rank's block.  A rank may already
 *     store its next call's block while another still reads this one, so
 *     alternate two buffers between calls.
 *   - pipelined (defer = 1): release_arrival and the wait are the PREVIOUS
 *     call's (its counters; its arrival[rank] and target), both null for the
 *     first call, and a sequence ends with sm100_marlin_gather_wait on the
 *     last call (releasing it).  A call's exchange then overlaps the next
 *     GEMM and no CTA waits for its own peer stores; a call's output is
 *     complete once a later launch waited on it.  Rotate three buffers (a
 *     rank can be one call further ahead) and read a call's output before
 *     issuing the next call.
 * All ranks must issue the same sequence of calls on a buffer (shapes may
 * differ between calls).
 */
int sm100_marlin_mul_2_4_gather(const void* A, const void* B, const void* meta, const void* s,
                                int prob_m, int prob_n, int prob_k, void* workspace, int groupsize,
                                int dev, void* stream, int meta_bits, void* const* gathered_c,
                                void* const* arrival, void* target, const void* wait_arrival,
                                const void* wait_target, void* const* release_arrival, int defer,
                                int world, int rank);

/* On `stream` (one-thread kernel): the deferred release of the last call
 * (release_arrival: its counters on all `world` ranks, or null), then a
 * bounded wait until *arrival >= *target -- the completion point of a
 * pipelined fused all-gather (see above).  No counterpart in the reference. */
int sm100_marlin_gather_wait(const void* arrival, const void* target, void* const* release_arrival,
                             int world, int dev, void* stream);

/* Device buffers shared between processes (CUDA IPC) for the fused all-gather:
 * allocate (zeroed), export a 64-byte handle, map a peer's buffer, unmap,
 * free.  No counterpart in the reference. */
int sm100_marlin_ipc_alloc(size_t bytes, int dev, void** ptr);
int sm100_marlin_ipc_free(void* ptr, int dev);
int sm100_marlin_ipc_get_handle(void* ptr, int dev, void* handle);
int sm100_marlin_ipc_open(const void* handle, int dev, void** ptr);
int sm100_marlin_ipc_close(void* ptr, int dev);

/*
 * GPU packer: fp16 weight w (prob_k, prob_m) row-major and unpermuted fp16
 * scales s (prob_k/groupsize or 1, prob_m) -> B int32 (prob_k/32, 2*prob_m),
 * meta int16 (prob_m, prob_k/16), s_out fp16 (same shape as s, permuted),
 * bit-identical to `Layer_2_4.pack(linear, scales, trans=True)`
 * (kernel_experiments/sparse_marlin/src/marlin/__init__.py:331-388: quantise
 * clamp(round(w/s)+8, 0, 15), 2:4 mask on the biased codes, CUTLASS
 * compression and metadata reorder, Marlin tiling and nibble packing), which
 * the reference runs on the CPU.  groupsize is the uncompressed group (128)
 * or -1; prob_k % 128 == 0 and prob_m % 64 == 0.  Asynchronous on `stream`.
 */
int sm100_marlin_pack_2_4(const void* w, const void* s, int prob_k, int prob_m, int groupsize,
                          void* B, void* meta, void* s_out, int dev, void* stream);

/*
 * 3-bit metadata codec.  Replaces `pack_metadata` / `unpack_metadata`
 * (kernel_experiments/sparse_marlin/metadata_decode/codec.cu:30-41).
 * pack:   meta int16[n_int16] (n_int16 % 128 == 0) -> out int32[n_int16*3/8];
 *         illegal 2:4 nibbles are counted into *err_count (device uint32,
 *         caller zeroes it; the reference raises when it is nonzero).
 * unpack: in int32[n_int32] (n_int32 % 48 == 0) -> out int16[n_int32*8/3].
 */
int sm100_marlin_meta3_pack(const void* meta, void* out, int64_t n_int16, void* err_count,
                            void* stream);
int sm100_marlin_meta3_unpack(const void* in, void* out, int64_t n_int32, void* stream);

/* Applies the device 3-bit decoders to n words: out_high[i] = high-table
 * decode of in[i] bits [0,24), out_low[i] = low-table decode.  Exposes the
 * in-kernel decoders (kernel_experiments/sparse_marlin/decoder_dependency/
 * pair.cuh:3-23, decoder.cuh:46-76) for known-answer tests. */
int sm100_marlin_meta3_decode_words(const void* in, void* out_high, void* out_low, int64_t n,
                                    void* stream);

/* Reads and clears the device status word of `dev` (synchronises the
 * device).  Nonzero bits mean a kernel gave up a bounded wait.  The library
 * looks up the word's device address once per device and keeps it for the
 * life of the process, so none of its entry points may be used on a device
 * after cudaDeviceReset there. */
int sm100_marlin_device_status(int dev, int* status);

/* Static description of a status code. */
const char* sm100_marlin_error_string(int code);

/* Message of the last CUDA error seen by this library on this thread. */
const char* sm100_marlin_last_cuda_error(void);

/* Launch overlap between consecutive GEMM calls on one stream (programmatic
 * dependent launch; on by default, or per SM100_MARLIN_PDL=0 in the
 * environment).  With overlap on, a call may start streaming its WEIGHTS
 * (B, meta, s) while the previous GEMM call on the stream is still running,
 * so those buffers must not be written by that previous call; activations,
 * C, workspace and scratch are only touched after it has completed.  No
 * counterpart in the reference (whose launches never overlap). */
int sm100_marlin_set_overlap(int enable);

/* Which kernel takes batches of at most 64 rows (process-wide):
 *   SM100_MARLIN_DECODE_AUTO (0, default): the tensor-memory kernel for 17-64
 *     rows (33-64 with 3-bit metadata) where N % 128 == 0 and K % 256 == 0,
 *     the warp-level stream-K kernel otherwise;
 *   SM100_MARLIN_DECODE_STREAM_K (1): always the warp-level kernel (or the
 *     CTA-pair kernel for 33-64 rows where it applies);
 *   SM100_MARLIN_DECODE_TMEM (2): the tensor-memory kernel for every batch of
 *     1-64 rows whose shape it takes.
 * Results of the two kernels agree within fp32 summation order; each is
 * deterministic.  Returns SM100_MARLIN_ERR_ARGUMENT for other values. */
#define SM100_MARLIN_DECODE_AUTO 0
#define SM100_MARLIN_DECODE_STREAM_K 1
#define SM100_MARLIN_DECODE_TMEM 2
int sm100_marlin_set_decode_kernel(int which);

/* Debug timelines: in a library built with -DSM100_MARLIN_TRACE=1 the k-th
 * GEMM launch after this call writes into `buf` (device memory, zeroed by the
 * caller, 36 KiB per launch) at offset k * 36 KiB: per CTA 16 uint64 words
 * (%globaltimer at kernel entry, first TMA issue, first and last stage
 * consumed, end of the CTA, stage count, fixup count, return from the
 * programmatic-launch wait, then inside the last epilogue: warps reduced,
 * finisher partials ready, C stores issued, past the dependency wait; words
 * 12-15 unused), then per-stage clock64 stamps of CTA 0.
 * Returns SM100_MARLIN_ERR_ARGUMENT in normal builds (nothing is recorded).
 * No counterpart in the reference (its profiling is external, via ncu). */
int sm100_marlin_set_trace_buffer(void* buf);

#ifdef __cplusplus
}
#endif

#endif /* SM100_MARLIN_H_ */
