// Host launcher and C ABI of the sm_100a 2:4 sparse W4A16 GEMM library.
//
// Entry points are declared in include/sm100_marlin.h.  The argument
// validation mirrors the reference launcher
// (kernel_experiments/sparse_marlin/src/marlin/marlin_cuda_kernel_nm.cu:751-830)
// so that shapes it rejects are rejected with the same status; the kernel
// tiling behind it is this library's own.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/sm100_marlin.h"
#include "device_primitives.cuh"
#include "marlin24_gemm.cuh"
#include "meta3_codec.cuh"

namespace sm100 {

__device__ int g_device_status = 0;

namespace {

thread_local std::string t_last_cuda_error;

int cuda_fail(cudaError_t e) {
  t_last_cuda_error = cudaGetErrorString(e);
  return SM100_MARLIN_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      ok = false;
      return;
    }
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// Split-K scratch owned by the library, one buffer per (device, stream):
// calls on one stream are ordered, so they can share it.
struct ScratchCache {
  std::mutex mu;
  std::map<std::pair<int, void*>, std::pair<void*, size_t>> bufs;
};
ScratchCache& scratch_cache() {
  static ScratchCache* c = new ScratchCache();  // never destroyed: no teardown-order issues
  return *c;
}

int get_scratch(int dev, cudaStream_t stream, size_t need, void** out) {
  ScratchCache& c = scratch_cache();
  std::lock_guard<std::mutex> lock(c.mu);
  auto& slot = c.bufs[{dev, reinterpret_cast<void*>(stream)}];
  if (slot.second >= need) {
    *out = slot.first;
    return SM100_MARLIN_OK;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) return cuda_fail(cudaGetLastError());
  if (cap != cudaStreamCaptureStatusNone) {
    t_last_cuda_error = "split-K scratch must be sized by one call before stream capture";
    return SM100_MARLIN_ERR_SCRATCH;
  }
  if (slot.first) {
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e);
    cudaFree(slot.first);
    slot = {nullptr, 0};
  }
  size_t bytes = need < (1u << 20) ? (1u << 20) : need;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e);
  slot = {p, bytes};
  *out = p;
  return SM100_MARLIN_OK;
}

int device_sms(int dev, int* sms) {
  cudaError_t e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int choose_nc(int n_out) { return (n_out % 256 == 0) ? 4 : ((n_out % 128 == 0) ? 2 : 1); }

struct Plan {
  int nc, mb, nh_last, grid;
  long long units;
  size_t scratch;
};

Plan make_plan(int n_out, int m_rows, int k_in, int sms) {
  Plan pl;
  pl.nc = choose_nc(n_out);
  pl.mb = (m_rows + 15) / 16;
  pl.nh_last = (m_rows - 16 * (pl.mb - 1)) > 8 ? 2 : 1;
  const long long n_tiles = n_out / (64 * pl.nc);
  pl.units = n_tiles * (k_in / 64);
  pl.grid = static_cast<int>(pl.units < sms ? pl.units : sms);
  pl.scratch = static_cast<size_t>(pl.grid) * pl.nc * pl.mb * 8192;
  return pl;
}

template <int NC, int MB, int NH, bool META3>
int launch_one(const GemmParams& p, int grid, int dev, cudaStream_t stream) {
  using Cfg = DecodeCfg<NC, MB, META3>;
  static bool attr_set[64] = {};
  auto kern = marlin24_decode_kernel<NC, MB, NH, META3>;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  kern<<<grid, kThreads, Cfg::SMEM, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

template <bool META3>
int dispatch(const GemmParams& p, const Plan& pl, int dev, cudaStream_t stream) {
#define SM100_CASE(NC_, MB_, NH_)                                   \
  if (pl.nc == NC_ && pl.mb == MB_ && pl.nh_last == NH_)            \
    return launch_one<NC_, MB_, NH_, META3>(p, pl.grid, dev, stream);
#define SM100_CASES_NC(NC_) \
  SM100_CASE(NC_, 1, 1)     \
  SM100_CASE(NC_, 1, 2)     \
  SM100_CASE(NC_, 2, 1)     \
  SM100_CASE(NC_, 2, 2)     \
  SM100_CASE(NC_, 3, 1)     \
  SM100_CASE(NC_, 3, 2)     \
  SM100_CASE(NC_, 4, 1)     \
  SM100_CASE(NC_, 4, 2)
  SM100_CASES_NC(4)
  SM100_CASES_NC(2)
  SM100_CASES_NC(1)
#undef SM100_CASES_NC
#undef SM100_CASE
  return SM100_MARLIN_ERR_KERN_SHAPE;
}

// Reference shape rules (marlin_cuda_kernel_nm.cu:763-783,811-823).
int check_reference_shape(int prob_m, int prob_n, int prob_k, int groupsize, int* thread_k,
                          int* thread_m) {
  if (*thread_k == -1 || *thread_m == -1) {
    if (prob_n <= 16) {
      *thread_k = 128;
      *thread_m = 128;
    } else {
      *thread_k = 64;
      *thread_m = 256;
    }
  }
  if (*thread_k <= 0 || *thread_m <= 0) return SM100_MARLIN_ERR_KERN_SHAPE;
  const int group_blocks = (groupsize == -1) ? -1 : groupsize / 16;
  if (prob_m % *thread_m != 0 || prob_k % *thread_k != 0 ||
      (group_blocks != -1 && (group_blocks == 0 || (prob_k / 2) % group_blocks != 0)))
    return SM100_MARLIN_ERR_PROB_SHAPE;
  const bool tile_small = (*thread_k == 128 && *thread_m == 128);
  const bool tile_large = (*thread_k == 64 && *thread_m == 256);
  if (!tile_small && !tile_large) return SM100_MARLIN_ERR_KERN_SHAPE;
  if (tile_small && prob_n > 16) return SM100_MARLIN_ERR_KERN_SHAPE;
  if (group_blocks != -1 && group_blocks != 4) return SM100_MARLIN_ERR_KERN_SHAPE;
  return SM100_MARLIN_OK;
}

int mul_impl(const void* A, const void* B, const void* meta, void* C, const void* s, int prob_m,
             int prob_n, int prob_k, void* workspace, int groupsize, int dev, void* stream_v,
             int thread_k, int thread_m, int sms, int max_par, int meta_bits, void* scratch,
             size_t scratch_bytes) {
  (void)max_par;
  if (prob_m < 0 || prob_n < 0 || prob_k < 0) return SM100_MARLIN_ERR_ARGUMENT;
  int rc = check_reference_shape(prob_m, prob_n, prob_k, groupsize, &thread_k, &thread_m);
  if (rc != SM100_MARLIN_OK) return rc;
  if (prob_m == 0 || prob_n == 0 || prob_k == 0) return SM100_MARLIN_OK;
  if (groupsize != -1 && prob_k % 128 != 0) return SM100_MARLIN_ERR_PROB_SHAPE;
  if (!A || !B || !meta || !C || !s || !workspace) return SM100_MARLIN_ERR_ARGUMENT;
  if (!aligned16(A) || !aligned16(B) || !aligned16(meta) || !aligned16(C) || !aligned16(s) ||
      (reinterpret_cast<uintptr_t>(workspace) & 3u))
    return SM100_MARLIN_ERR_ALIGNMENT;

  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_v);
  if (sms == -1) {
    rc = device_sms(dev, &sms);
    if (rc != SM100_MARLIN_OK) return rc;
  }
  if (sms <= 0) return SM100_MARLIN_ERR_ARGUMENT;

  const int chunk_rows = prob_n < 64 ? prob_n : 64;
  Plan big = make_plan(prob_m, chunk_rows, prob_k, sms);
  if (scratch == nullptr) {
    rc = get_scratch(dev, stream, big.scratch, &scratch);
    if (rc != SM100_MARLIN_OK) return rc;
  } else if (scratch_bytes < big.scratch || !aligned16(scratch)) {
    return SM100_MARLIN_ERR_SCRATCH;
  }
  int* status = nullptr;
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_device_status);
  if (e != cudaSuccess) return cuda_fail(e);

  for (int r0 = 0; r0 < prob_n; r0 += 64) {
    const int rows = (prob_n - r0) < 64 ? (prob_n - r0) : 64;
    Plan pl = make_plan(prob_m, rows, prob_k, sms);
    GemmParams p;
    p.A = static_cast<const uint8_t*>(A) + static_cast<size_t>(r0) * prob_k * 2;
    p.B = static_cast<const uint8_t*>(B);
    p.meta = static_cast<const uint8_t*>(meta);
    p.s = static_cast<const uint8_t*>(s);
    p.C = reinterpret_cast<half*>(static_cast<uint8_t*>(C) + static_cast<size_t>(r0) * prob_m * 2);
    p.partials = static_cast<float4*>(scratch);
    p.counters = static_cast<int*>(workspace);
    p.status = status;
    p.M = rows;
    p.N = prob_m;
    p.K = prob_k;
    p.grouped = groupsize != -1 ? 1 : 0;
    p.n_tiles = prob_m / (64 * pl.nc);
    p.kk_total = prob_k / 32;
    p.units = pl.units;
    rc = meta_bits == 3 ? dispatch<true>(p, pl, dev, stream) : dispatch<false>(p, pl, dev, stream);
    if (rc != SM100_MARLIN_OK) return rc;
  }
  return SM100_MARLIN_OK;
}

}  // namespace
}  // namespace sm100

using namespace sm100;

extern "C" {

int sm100_marlin_mul_2_4(const void* A, const void* B, const void* meta, void* C, const void* s,
                         int prob_m, int prob_n, int prob_k, void* workspace, int groupsize,
                         int dev, void* stream, int thread_k, int thread_m, int sms, int max_par) {
  return mul_impl(A, B, meta, C, s, prob_m, prob_n, prob_k, workspace, groupsize, dev, stream,
                  thread_k, thread_m, sms, max_par, 4, nullptr, 0);
}

int sm100_marlin_mul_2_4_meta3(const void* A, const void* B, const void* meta3, void* C,
                               const void* s, int prob_m, int prob_n, int prob_k, void* workspace,
                               int groupsize, int dev, void* stream, int thread_k, int thread_m,
                               int sms, int max_par) {
  return mul_impl(A, B, meta3, C, s, prob_m, prob_n, prob_k, workspace, groupsize, dev, stream,
                  thread_k, thread_m, sms, max_par, 3, nullptr, 0);
}

int sm100_marlin_mul_2_4_ex(const void* A, const void* B, const void* meta, void* C, const void* s,
                            int prob_m, int prob_n, int prob_k, void* workspace, int groupsize,
                            int dev, void* stream, int thread_k, int thread_m, int sms,
                            int max_par, int meta_bits, void* scratch, size_t scratch_bytes) {
  if (meta_bits != 3 && meta_bits != 4) return SM100_MARLIN_ERR_ARGUMENT;
  if (scratch == nullptr) return SM100_MARLIN_ERR_SCRATCH;
  return mul_impl(A, B, meta, C, s, prob_m, prob_n, prob_k, workspace, groupsize, dev, stream,
                  thread_k, thread_m, sms, max_par, meta_bits, scratch, scratch_bytes);
}

size_t sm100_marlin_scratch_bytes(int prob_m, int prob_n, int prob_k, int dev, int sms) {
  if (prob_m <= 0 || prob_n <= 0 || prob_k <= 0) return 0;
  if (sms == -1 && device_sms(dev, &sms) != SM100_MARLIN_OK) return 0;
  if (sms <= 0) return 0;
  const int rows = prob_n < 64 ? prob_n : 64;
  return make_plan(prob_m, rows, prob_k, sms).scratch;
}

int sm100_marlin_meta3_pack(const void* meta, void* out, int64_t n_int16, void* err_count,
                            void* stream) {
  if (n_int16 < 0 || n_int16 % 128 != 0) return SM100_MARLIN_ERR_ARGUMENT;
  if (n_int16 == 0) return SM100_MARLIN_OK;
  if (!meta || !out || !err_count) return SM100_MARLIN_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(meta) & 3u) || (reinterpret_cast<uintptr_t>(out) & 3u) ||
      (reinterpret_cast<uintptr_t>(err_count) & 3u))
    return SM100_MARLIN_ERR_ALIGNMENT;
  const int64_t pairs = n_int16 / 8;
  const int threads = 256;
  const int64_t blocks = (pairs + threads - 1) / threads;
  meta3_pack_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                      reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(meta), static_cast<uint32_t*>(out), pairs,
      static_cast<uint32_t*>(err_count));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_meta3_unpack(const void* in, void* out, int64_t n_int32, void* stream) {
  if (n_int32 < 0 || n_int32 % 48 != 0) return SM100_MARLIN_ERR_ARGUMENT;
  if (n_int32 == 0) return SM100_MARLIN_OK;
  if (!in || !out) return SM100_MARLIN_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(in) & 3u) || (reinterpret_cast<uintptr_t>(out) & 3u))
    return SM100_MARLIN_ERR_ALIGNMENT;
  const int64_t lanes = n_int32 / 48 * 32;
  const int threads = 256;
  const int64_t blocks = (lanes + threads - 1) / threads;
  meta3_unpack_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out), lanes);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_meta3_decode_words(const void* in, void* out_high, void* out_low, int64_t n,
                                    void* stream) {
  if (n < 0) return SM100_MARLIN_ERR_ARGUMENT;
  if (n == 0) return SM100_MARLIN_OK;
  if (!in || !out_high || !out_low) return SM100_MARLIN_ERR_ARGUMENT;
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  meta3_decode_words_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                              reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out_high),
      static_cast<uint32_t*>(out_low), n);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_device_status(int dev, int* status) {
  if (!status) return SM100_MARLIN_ERR_ARGUMENT;
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e);
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e);
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e);
  *status = v;
  return SM100_MARLIN_OK;
}

const char* sm100_marlin_error_string(int code) {
  switch (code) {
    case SM100_MARLIN_OK: return "ok";
    case SM100_MARLIN_ERR_PROB_SHAPE: return "problem shape not compatible with the tile shape";
    case SM100_MARLIN_ERR_KERN_SHAPE: return "no kernel implementation for this tile / group shape";
    case SM100_MARLIN_ERR_CUDA: return "CUDA error";
    case SM100_MARLIN_ERR_ALIGNMENT: return "a pointer is not 16-byte aligned";
    case SM100_MARLIN_ERR_ARGUMENT: return "invalid argument";
    case SM100_MARLIN_ERR_SCRATCH: return "split-K scratch missing or too small";
    default: return "unknown status";
  }
}

const char* sm100_marlin_last_cuda_error(void) { return t_last_cuda_error.c_str(); }

}  // extern "C"
