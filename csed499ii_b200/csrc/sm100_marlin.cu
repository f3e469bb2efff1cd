// Host launcher and C ABI of the sm_100a 2:4 sparse W4A16 GEMM library.
//
// Entry points are declared in include/sm100_marlin.h.  The argument
// validation mirrors the reference launcher
// (kernel_experiments/sparse_marlin/src/marlin/marlin_cuda_kernel_nm.cu:751-830)
// so that shapes it rejects are rejected with the same status; the kernel
// tiling behind it is this library's own.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <unordered_map>
#include <string>
#include <utility>

#include "../../include/sm100_marlin.h"
#include "launch.cuh"

namespace sm100 {

__device__ int g_device_status = 0;

// Split-K scratch of the allocation-free entry point
// (sm100_marlin_mul_2_4_noalloc).  One copy per device that loads the
// library, held until the process exits.  Every noalloc call on a device uses
// the same bytes; the kernel writes each partial before any CTA reads it, so
// nothing in it has to start at zero.
constexpr size_t kNoAllocScratchBytes = 8u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
thread_local std::string t_last_cuda_error;
}  // namespace

int cuda_fail(cudaError_t e) {
  t_last_cuda_error = cudaGetErrorString(e);
  return SM100_MARLIN_ERR_CUDA;
}

namespace {

// Programmatic dependent launch between consecutive GEMM launches (on by
// default; SM100_MARLIN_PDL=0 or sm100_marlin_set_overlap(0) turns it off).
int g_pdl_override = -1;
bool pdl_enabled() {
  if (g_pdl_override >= 0) return g_pdl_override != 0;
  static const bool env_on = [] {
    const char* e = std::getenv("SM100_MARLIN_PDL");
    return !(e && e[0] == '0');
  }();
  return env_on;
}

// Tuning knobs.  Builds with -DSM100_MARLIN_TUNING=1 (experiments only) read
// them from the environment once per process; the default build compiles
// them out and uses the measured defaults given at each call site.  The one
// supported environment switch is SM100_MARLIN_PDL (above).
#ifndef SM100_MARLIN_TUNING
#define SM100_MARLIN_TUNING 0
#endif
int tuning_knob(const char* name, int dflt) {
#if SM100_MARLIN_TUNING
  const char* e = std::getenv(name);
  return e ? std::atoi(e) : dflt;
#else
  (void)name;
  return dflt;
#endif
}

// Stages whose weights a kernel may stream before the previous kernel on the
// stream has completed (default: the whole ring; knob SM100_MARLIN_PREFETCH).
int prefetch_stages() {
  static const int v = tuning_knob("SM100_MARLIN_PREFETCH", 1 << 30);
  return v;
}

// Device buffer for per-CTA timelines (only written by SM100_MARLIN_TRACE builds).
unsigned long long* g_trace_buffer = nullptr;
// Trace builds: launch k writes its records at g_trace_buffer + k * kTraceLaunchWords.
long long g_trace_launch = 0;


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

// Device address of g_noalloc_scratch on `dev` (the host-side symbol is only
// a stand-in, never a device pointer).  Resolved once per device, with that
// device current; the first noalloc call on a device does it.  The cached
// address is valid as long as the device's primary context lives: after a
// cudaDeviceReset it would point at freed memory (documented in the header).
int noalloc_scratch(int dev, void** out) {
  static std::mutex mu;
  static void* ptr[64] = {};
  if (dev < 0 || dev >= 64) return SM100_MARLIN_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e);
    ptr[dev] = p;
  }
  *out = ptr[dev];
  return SM100_MARLIN_OK;
}

// Per-call host costs are on the eager path's critical path (an eager
// decode step issues ~10 us of host work per ~10 us GEMM), so what never
// changes between calls is looked up once: the SM count, the address of the
// device status word, and encoded tensor maps.
int device_sms(int dev, int* sms) {
  static std::atomic<int> cache[64] = {};
  if (dev >= 0 && dev < 64) {
    const int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) {
      *sms = v;
      return SM100_MARLIN_OK;
    }
  }
  cudaError_t e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev >= 0 && dev < 64) cache[dev].store(*sms, std::memory_order_relaxed);
  return SM100_MARLIN_OK;
}

// Device address of g_device_status on the current device (looked up once
// per device; the caller has made `dev` current).
int device_status_ptr(int dev, int** out) {
  static std::atomic<int*> cache[64] = {};
  if (dev >= 0 && dev < 64) {
    int* v = cache[dev].load(std::memory_order_acquire);
    if (v != nullptr) {
      *out = v;
      return SM100_MARLIN_OK;
    }
  }
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_device_status);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev >= 0 && dev < 64) cache[dev].store(*out, std::memory_order_release);
  return SM100_MARLIN_OK;
}

// Column-tile width (in 64-column chunks).  Wider tiles re-read the
// activations less often, but when there are fewer tiles than CTAs some CTA
// works entirely inside one tile and finishes at the same time as the CTA
// that completes the tile, which puts the split-K hand-over on the critical
// path.  So: the widest tile that still gives every CTA at least one tile
// boundary, else one chunk (measured best for every Llama-2-7B shape).
// Knob SM100_MARLIN_NC=1|2|4 forces a width.
int choose_nc(int n_out, int sms) {
  static const int forced = tuning_knob("SM100_MARLIN_NC", 0);
  const int chunks = n_out / 64;
  if ((forced == 1 || forced == 2 || forced == 4) && chunks % forced == 0) return forced;
  for (int nc : {4, 2})
    if (chunks % nc == 0 && chunks / nc >= sms) return nc;
  return 1;
}

struct Plan {
  int nc, mb, nh_last, grid, unit_kk, sk;
  long long units;
  size_t scratch;
  int cluster;  // > 1: cluster split-K with clusters of this many CTAs
};

bool cluster_split_enabled() {
  static const bool v = tuning_knob("SM100_MARLIN_CLUSTER", 1) != 0;
  return v;
}

// A unit is one full stage (sk rows of 32 K) when K allows it; scale groups
// (4 rows) stay aligned to stage starts.
int unit_rows(int kk, int sk) {
  for (int u = sk; u >= 4; u /= 2)
    if (kk % u == 0) return u;
  return 2;
}

Plan make_plan(int n_out, int m_rows, int k_in, int sms, bool allow_cluster = true) {
  Plan pl;
  pl.cluster = 1;
  pl.mb = (m_rows + 15) / 16;
  if (pl.mb == 3) pl.mb = 4;
  pl.nh_last = (pl.mb == 1 && m_rows <= 8) ? 1 : 2;
  const int kk = k_in / 32;
  // Cluster split-K (batch <= 16): the CTAs of a column tile form a cluster
  // of S = 2 or 3 and hand their partials to the tile's finisher through
  // distributed shared memory -- no scratch, no counters, no GPU-scope
  // fence, and the contributors leave at once.  Taken when the tiles times S
  // fill at least 80 % of the SMs and a CTA streams at most 48 blocks of
  // 32 x 64 (~1 us at ~18 ns a block) and 25 % above its stream-K share.
  // Llama step at M = 16 on B200: 7B 2269 vs 2124 GB/s; per call
  // (K, N) = (11008, 4096) 8.7 vs 9.4 us, (8192, 8192) 10.9 vs 11.2; with
  // (28672, 8192) at 896 vs 775 blocks it was 25.7 vs 24.6 us.
  if (allow_cluster && pl.mb == 1 && cluster_split_enabled()) {
    const long long chunks = n_out / 64;
    const double sk_blocks = static_cast<double>(kk) * chunks / sms;  // 32x64 blocks per CTA
    long long best_blocks = -1;
    for (int nc : {1, 2}) {  // 256-column tiles stream too slowly (4-row stages)
      if (chunks % nc != 0) continue;
      const int sk = consumer_warps(1) * rows_per_warp(nc, 1) / nc;
      const int ukk = unit_rows(kk, sk);
      const long long upt = kk / ukk, tiles = chunks / nc;
      for (int S : {2, 3}) {
        const long long ctas = tiles * S;
        if (upt < S || ctas > sms || ctas * 5 < static_cast<long long>(sms) * 4) continue;
        const long long blocks = static_cast<long long>(nc) * ukk * ((upt + S - 1) / S);
        if (blocks > 1.25 * sk_blocks || blocks > sk_blocks + 48 ||
            (best_blocks >= 0 && blocks >= best_blocks))
          continue;
        best_blocks = blocks;
        pl.nc = nc;
        pl.sk = sk;
        pl.unit_kk = ukk;
        pl.units = tiles * upt;
        pl.grid = static_cast<int>(ctas);
        pl.cluster = S;
      }
    }
    if (pl.cluster > 1) {
      pl.scratch = 0;
      return pl;
    }
  }
  pl.nc = choose_nc(n_out, sms);
  pl.sk = consumer_warps(pl.mb) * rows_per_warp(pl.nc, pl.mb) / pl.nc;
  pl.unit_kk = unit_rows(kk, pl.sk);
  const long long n_tiles = n_out / (64 * pl.nc);
  pl.units = n_tiles * (kk / pl.unit_kk);
  pl.grid = static_cast<int>(pl.units < sms ? pl.units : sms);
  // Whole column tiles (no split-K) when they fit the SMs in one wave and a
  // tile is at most 4 stages deep: the split-K hand-over costs ~3-4 us per
  // call (per-CTA traces), more than the fewer SMs lose on short tiles.
  // Measured at M = 16: K = N = 4096 5.87 vs 7.24 us; deeper tiles stream too
  // slowly on fewer SMs (K = 11008, N = 4096: 11.0 vs 10.0 us).
  if (n_tiles <= sms && kk <= 4 * pl.sk) pl.grid = static_cast<int>(n_tiles);
  // Split-K happens when some CTA's unit range starts inside a tile: never
  // with one unit per tile or when the CTAs divide the tiles evenly.  Then
  // one fp32 partial tile (nc chunks x 16*mb rows x 64 columns) per CTA.
  const long long upt = kk / pl.unit_kk;
  const bool split = upt > 1 && n_tiles % pl.grid != 0;
  pl.scratch = split ? static_cast<size_t>(pl.grid) * pl.nc * pl.mb * 4096 : 0;
  return pl;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// An encoded tensor map is a pure function of its arguments, so a cache keyed
// on all of them is always valid (a freed and reused address with the same
// dims and box encodes to the same map).  Cleared when it grows past 4096.
struct TmapKey {
  uint64_t w[12];
  bool operator==(const TmapKey& o) const { return std::memcmp(w, o.w, sizeof(w)) == 0; }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t x : k.w) h = (h ^ x) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};
struct TmapCache {
  std::mutex mu;
  std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> maps;
};
TmapCache& tmap_cache() {
  static TmapCache c;
  return c;
}

int encode_nd_uncached(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank,
                       const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                       CUtensorMapSwizzle swizzle);

int encode_nd(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swizzle) {
  TmapKey key = {};
  key.w[0] = static_cast<uint64_t>(dtype) | (static_cast<uint64_t>(rank) << 16) |
             (static_cast<uint64_t>(swizzle) << 32);
  key.w[1] = reinterpret_cast<uint64_t>(base);
  for (int i = 0; i < rank; ++i) {
    key.w[2 + i] = dims[i];
    key.w[5 + i] = box[i];
    if (i + 1 < rank) key.w[8 + i] = strides_bytes[i];
  }
  TmapCache& c = tmap_cache();
  {
    std::lock_guard<std::mutex> lock(c.mu);
    auto it = c.maps.find(key);
    if (it != c.maps.end()) {
      *map = it->second;
      return SM100_MARLIN_OK;
    }
  }
  const int rc = encode_nd_uncached(map, dtype, base, rank, dims, strides_bytes, box, swizzle);
  if (rc != SM100_MARLIN_OK) return rc;
  std::lock_guard<std::mutex> lock(c.mu);
  if (c.maps.size() >= 4096) c.maps.clear();
  c.maps.emplace(key, *map);
  return SM100_MARLIN_OK;
}

int encode_nd_uncached(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank,
                       const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                       CUtensorMapSwizzle swizzle) {
  auto enc = tensor_map_encoder();
  if (!enc) {
    t_last_cuda_error = "cuTensorMapEncodeTiled unavailable";
    return SM100_MARLIN_ERR_CUDA;
  }
  cuuint64_t d[3];
  cuuint64_t st[2];
  cuuint32_t b[3], es[3];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = enc(map, dtype, rank, const_cast<void*>(base), d, st, b, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")";
    return SM100_MARLIN_ERR_CUDA;
  }
  return SM100_MARLIN_OK;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return encode_nd(map, dtype, base, 2, dims, strides, box, swizzle);
}

// Fills the four tensor maps of `p` for this launch's plan.
int encode_maps(GemmParams& p, const Plan& pl, const void* A, const void* B, const void* meta,
                const void* s, int meta_bits) {
  const int nc = pl.nc, sk = pl.sk;
  const uint64_t N = p.N, K = p.K, KK = K / 32;
  // activations as (64 halves, M rows, K/64 slices): one box per stage holds
  // the SK/2 64-wide K slices of all (padded) rows, 128B-swizzled
  const uint64_t a_dims[3] = {64, static_cast<uint64_t>(p.M), K / 64};
  const uint64_t a_strides[2] = {2 * K, 128};
  const uint32_t a_box[3] = {64, static_cast<uint32_t>(16 * pl.mb), static_cast<uint32_t>(sk / 2)};
  int rc = encode_nd(&p.tm_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, 3, a_dims, a_strides, a_box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT64, B, N, KK, 8 * N, 64 * nc, sk,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (meta_bits == 3)
    rc = encode_2d(&p.tm_meta, CU_TENSOR_MAP_DATA_TYPE_UINT64, meta, 3 * N / 8, KK, 3 * N,
                   24 * nc, sk, CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    rc = encode_2d(&p.tm_meta, CU_TENSOR_MAP_DATA_TYPE_UINT64, meta, N / 2, KK, 4 * N, 32 * nc,
                   sk, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (p.grouped) {
    const uint32_t s_rows = sk / 4;
    rc = encode_2d(&p.tm_s, CU_TENSOR_MAP_DATA_TYPE_UINT64, s, N / 4, K / 128, 2 * N, 16 * nc,
                   s_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    std::memset(&p.tm_s, 0, sizeof(p.tm_s));
  }
  return SM100_MARLIN_OK;
}

template <bool META3, bool GROUPED, bool EPI, int DIAG = 0>
int dispatch_g(const GemmParams& p, const Plan& pl, int dev, cudaStream_t stream) {
#define SM100_CASE(NC_, MB_, NH_)                                            \
  if (pl.nc == NC_ && pl.mb == MB_ && pl.nh_last == NH_)                     \
    return launch_decode<NC_, MB_, NH_, META3, GROUPED, EPI, DIAG>(p, pl.grid, dev, stream);
#define SM100_CASES_NC(NC_) \
  SM100_CASE(NC_, 1, 1)     \
  SM100_CASE(NC_, 1, 2)     \
  SM100_CASE(NC_, 2, 2)     \
  SM100_CASE(NC_, 4, 2)
  SM100_CASES_NC(4)
  SM100_CASES_NC(2)
  SM100_CASES_NC(1)
#undef SM100_CASES_NC
#undef SM100_CASE
  return SM100_MARLIN_ERR_KERN_SHAPE;
}

template <bool META3>
int dispatch(const GemmParams& p, const Plan& pl, int dev, cudaStream_t stream, int diag) {
  if (!META3 && diag != 0) {
    // metadata diagnostics: grouped scales, plain store only
    if (!p.grouped || p.bias != nullptr || p.act != kActNone) return SM100_MARLIN_ERR_ARGUMENT;
    if (diag == kDiagNoGmem) return dispatch_g<false, true, false, kDiagNoGmem>(p, pl, dev, stream);
    if (diag == kDiagNoReg) return dispatch_g<false, true, false, kDiagNoReg>(p, pl, dev, stream);
    if (diag == (kDiagNoGmem | kDiagNoReg))
      return dispatch_g<false, true, false, kDiagNoGmem | kDiagNoReg>(p, pl, dev, stream);
    return SM100_MARLIN_ERR_ARGUMENT;
  }
  if (p.bias != nullptr || p.act != kActNone)
    return p.grouped ? dispatch_g<META3, true, true>(p, pl, dev, stream)
                     : dispatch_g<META3, false, true>(p, pl, dev, stream);
  return p.grouped ? dispatch_g<META3, true, false>(p, pl, dev, stream)
                   : dispatch_g<META3, false, false>(p, pl, dev, stream);
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

// Batches above this many rows go to the tensor-memory (tcgen05) kernel in
// one launch instead of 64-row decode launches (knob SM100_MARLIN_PREFILL_MIN;
// a very large value disables the prefill kernel).
int prefill_min_rows() {
  static const int v = tuning_knob("SM100_MARLIN_PREFILL_MIN", 64);
  return v;
}

// Groups of dequantising warps per prefill CTA (knob SM100_MARLIN_PREFILL_GROUPS
// = 1|2|4).  Default 4: measured 928 / 1003 / 1041 TFLOP/s for 1 / 2 / 4
// groups over the prefill sweep.
int prefill_groups() {
  static const int v = [] {
    const int g = tuning_knob("SM100_MARLIN_PREFILL_GROUPS", 4);
    return (g == 1 || g == 2) ? g : 4;
  }();
  return v;
}

// Groups of dequantising warps for the sparse prefill kernel (knob
// SM100_MARLIN_PREFILL_SPARSE_GROUPS = 1|2|4).  Default 4: 1199 / 1246 / 1294
// TFLOP/s for 1 / 2 / 4 groups over the prefill sweep.
int prefill_groups_sparse() {
  static const int v = [] {
    const int g = tuning_knob("SM100_MARLIN_PREFILL_SPARSE_GROUPS", 4);
    return (g == 1 || g == 2) ? g : 4;
  }();
  return v;
}

// Structured-sparse prefill kernel (tcgen05.mma.sp) for K % 128 == 0 (knob
// SM100_MARLIN_PREFILL_SPARSE=0 selects the dense-expansion kernel; knob
// SM100_MARLIN_PREFILL_BN=128|256 forces its batch tile).
bool prefill_sparse_enabled() {
  static const bool v = tuning_knob("SM100_MARLIN_PREFILL_SPARSE", 1) != 0;
  return v;
}

int prefill_forced_bn() {
  static const int v = [] {
    const int b = tuning_knob("SM100_MARLIN_PREFILL_BN", 0);
    return (b == 128 || b == 256) ? b : 0;
  }();
  return v;
}

// Knob SM100_MARLIN_PREFILL_PAIR=0 keeps 256-row prefill tiles on one CTA
// (default: CTA pairs whenever N % 256 == 0).
bool prefill_pair_enabled() {
  static const bool v = tuning_knob("SM100_MARLIN_PREFILL_PAIR", 1) != 0;
  return v;
}

// The structured-sparse form: K steps of 64 (as the dense form).
int mul_prefill_sparse(PrefillParams& p, const void* A, const void* B, const void* meta,
                       const void* s, int dev, int sms, cudaStream_t stream, int meta_bits,
                       int diag) {
  const uint64_t N = p.N, K = p.K;
  const int n_tiles = p.N / 128;
  // CTA pairs (256 features x 256 rows, 128-K steps) whenever the pair's 256
  // features divide N: per SM they do twice the work per K step of a one-CTA
  // tile, so they win even where half of the pair's rows lie past M.  Else
  // one CTA per tile: 256-row tiles unless they would leave more than a
  // quarter of the SMs idle (the 128-row tile is ~2x slower per CTA).
  int bn = prefill_forced_bn();
  const bool pair = p.N % 256 == 0 && prefill_pair_enabled() && bn != 128;
  // 3-bit metadata and the metadata diagnostics: CTA-pair kernel only (the
  // caller routes nothing else here)
  if ((meta_bits == 3 || diag != 0) && (!pair || p.K % 128 != 0)) return SM100_MARLIN_ERR_KERN_SHAPE;
  if (bn == 0)
    bn = pair || (p.M > 128 && 4ll * n_tiles * ((p.M + 255) / 256) >= 3ll * sms) ? 256 : 128;
  int rc;
  if (pair) {
    // (64 halves, M rows, K/64 slices), box 64 x 128 rows x 2 slices: the two
    // 128-byte-swizzled 64-K atoms of one 128-K step for one CTA's 128 rows
    const uint64_t a_dims[3] = {64, static_cast<uint64_t>(p.M), K / 64};
    const uint64_t a_strides[2] = {2 * K, 128};
    const uint32_t a_box[3] = {64, 128, 2};
    rc = encode_nd(&p.tm_act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, 3, a_dims, a_strides, a_box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    rc = encode_2d(&p.tm_act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, K, static_cast<uint64_t>(p.M),
                   2 * K, 64, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  // packed codes / metadata: 2 rows of 32 K per 64-K step, 4 per 128-K step (pair)
  const uint32_t rows32 = pair ? 4 : 2;
  rc = encode_2d(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT64, B, N, K / 32, 8 * N, 128, rows32,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (meta_bits == 3)  // 48 words per 64 features and 32-K row: 3N/8 u64 per row
    rc = encode_2d(&p.tm_meta, CU_TENSOR_MAP_DATA_TYPE_UINT64, meta, 3 * N / 8, K / 32, 3 * N, 48,
                   rows32, CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    rc = encode_2d(&p.tm_meta, CU_TENSOR_MAP_DATA_TYPE_UINT64, meta, N / 2, K / 32, 4 * N, 64,
                   rows32, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (p.grouped) {
    rc = encode_2d(&p.tm_s, CU_TENSOR_MAP_DATA_TYPE_UINT64, s, N / 4, K / 128, 2 * N, 32, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    std::memset(&p.tm_s, 0, sizeof(p.tm_s));
  }
  const int ng = prefill_groups_sparse();
  if (pair) {
    // C as (N, M) fp16, box 128 features x 256 rows: one TMA store per CTA
    rc = encode_2d(&p.tm_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, p.C, N, static_cast<uint64_t>(p.M),
                   2 * N, 128, 256, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    const bool epi = p.bias != nullptr || p.act != kActNone;
    if (diag != 0) {
      if (!p.grouped || epi || meta_bits != 4) return SM100_MARLIN_ERR_ARGUMENT;
      if (diag == kDiagNoGmem) return launch_prefill_sp2<4, true, false, false, kDiagNoGmem>(p, dev, stream);
      if (diag == kDiagNoReg) return launch_prefill_sp2<4, true, false, false, kDiagNoReg>(p, dev, stream);
      if (diag == (kDiagNoGmem | kDiagNoReg))
        return launch_prefill_sp2<4, true, false, false, kDiagNoGmem | kDiagNoReg>(p, dev, stream);
      return SM100_MARLIN_ERR_ARGUMENT;
    }
    if (meta_bits == 3)
      return p.grouped ? (epi ? launch_prefill_sp2<4, true, true, true, 0>(p, dev, stream)
                              : launch_prefill_sp2<4, true, false, true, 0>(p, dev, stream))
                       : (epi ? launch_prefill_sp2<4, false, true, true, 0>(p, dev, stream)
                              : launch_prefill_sp2<4, false, false, true, 0>(p, dev, stream));
#define SM100_PREFILL_SP2(NG_)                                                            \
  if (ng == NG_)                                                                          \
    return p.grouped ? (epi ? launch_prefill_sp2<NG_, true, true, false, 0>(p, dev, stream)   \
                            : launch_prefill_sp2<NG_, true, false, false, 0>(p, dev, stream)) \
                     : (epi ? launch_prefill_sp2<NG_, false, true, false, 0>(p, dev, stream)  \
                            : launch_prefill_sp2<NG_, false, false, false, 0>(p, dev, stream));
    SM100_PREFILL_SP2(1)
    SM100_PREFILL_SP2(2)
    SM100_PREFILL_SP2(4)
#undef SM100_PREFILL_SP2
    return SM100_MARLIN_ERR_KERN_SHAPE;
  }
#if SM100_MARLIN_TUNING
  // One CTA per 128-feature tile.  Unreachable with the default settings:
  // batches above 16 rows need N % 256 == 0 (the reference's shape rule),
  // which always allows CTA pairs; kept for experiments (knobs
  // SM100_MARLIN_PREFILL_PAIR=0, SM100_MARLIN_PREFILL_BN=128).
#define SM100_PREFILL_SP(BN_, NG_)                                                   \
  if (bn == BN_ && ng == NG_)                                                        \
    return p.grouped ? launch_prefill_sp<BN_, NG_, true>(p, dev, stream)        \
                     : launch_prefill_sp<BN_, NG_, false>(p, dev, stream);
  SM100_PREFILL_SP(128, 1)
  SM100_PREFILL_SP(128, 2)
  SM100_PREFILL_SP(128, 4)
  SM100_PREFILL_SP(256, 1)
  SM100_PREFILL_SP(256, 2)
  SM100_PREFILL_SP(256, 4)
#undef SM100_PREFILL_SP
#endif
  return SM100_MARLIN_ERR_KERN_SHAPE;
}

// C[M, N] = A . dequant(B, meta, s) for M > prefill_min_rows() (4-bit
// metadata): one 128 x BN output tile per CTA on the tcgen05 kernels.
int mul_prefill(const void* A, const void* B, const void* meta, void* C, const void* s, int n_out,
                int m_rows, int k_in, int groupsize, int dev, int sms, cudaStream_t stream,
                int* status, const void* bias, int act, int meta_bits, int diag) {
  PrefillParams p;
  p.s = static_cast<const uint8_t*>(s);
  p.C = static_cast<half*>(C);
  p.bias = static_cast<const half*>(bias);
  p.act = act;
  p.status = status;
  p.M = m_rows;
  p.N = n_out;
  p.K = k_in;
  p.grouped = groupsize != -1 ? 1 : 0;
  if (meta_bits == 3 || diag != 0 || (prefill_sparse_enabled() && k_in % 128 == 0))
    return mul_prefill_sparse(p, A, B, meta, s, dev, sms, stream, meta_bits, diag);
  const int n_tiles = n_out / 128;
  const int bn = (m_rows >= 256 && static_cast<long long>(n_tiles) * ((m_rows + 255) / 256) >= sms)
                     ? 256 : 128;
  const uint64_t N = n_out, K = k_in;
  int rc = encode_2d(&p.tm_act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, K, static_cast<uint64_t>(m_rows),
                     2 * K, 64, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT64, B, N, K / 32, 8 * N, 128, 2,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_2d(&p.tm_meta, CU_TENSOR_MAP_DATA_TYPE_UINT64, meta, N / 2, K / 32, 4 * N, 64, 2,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (p.grouped) {
    rc = encode_2d(&p.tm_s, CU_TENSOR_MAP_DATA_TYPE_UINT64, s, N / 4, K / 128, 2 * N, 32, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    std::memset(&p.tm_s, 0, sizeof(p.tm_s));
  }
#define SM100_PREFILL(BN_, NG_)                                                      \
  if (bn == BN_ && prefill_groups() == NG_)                                         \
    return p.grouped ? launch_prefill_dense<BN_, NG_, true>(p, dev, stream)           \
                     : launch_prefill_dense<BN_, NG_, false>(p, dev, stream);
  SM100_PREFILL(256, 2)
  SM100_PREFILL(256, 1)
  SM100_PREFILL(256, 4)
  SM100_PREFILL(128, 2)
  SM100_PREFILL(128, 1)
  SM100_PREFILL(128, 4)
#undef SM100_PREFILL
  return SM100_MARLIN_ERR_KERN_SHAPE;
}

// Which kernel takes batches of at most 64 rows (sm100_marlin_set_decode_kernel).
int g_decode_kernel = SM100_MARLIN_DECODE_AUTO;

// Whether a batch of `rows` (<= 64) goes to the tensor-memory decode kernel
// (marlin24_decode_tc.cuh).  Its single-thread MMA issue costs the same at
// 16 rows as at 64, so smaller batches stream faster on the warp-level kernel
// (Llama-7B step, 4-bit: 1666 vs 2174 GB/s at 16 rows, 1544 vs 1338 at 32,
// 973 vs 785 at 64; 3-bit: 990 vs 1156 at 32, 716 vs 679 at 64).
bool decode_tc_rows(int rows, int meta_bits) {
  if (g_decode_kernel == SM100_MARLIN_DECODE_TMEM) return true;
  if (g_decode_kernel == SM100_MARLIN_DECODE_STREAM_K) return false;
  return rows > (meta_bits == 3 ? 32 : 16);
}

// Plan: clusters of S CTAs (S = 1, 2, 4) split K S ways over `bpc`
// consecutive 128-feature blocks each.  At most one CTA per SM (clusters of
// four fit only 33 to a B200 that way), the fewest K steps per CTA wins;
// ties go to the smaller cluster.
struct TcPlan {
  int split, bpc, clusters;
};

TcPlan plan_decode_tc(int n_out, int k_in, int kstage, int sms, int dev) {
  const int nblocks = n_out / 128, ksteps = k_in / kstage;  // stages of kstage K
  TcPlan best{1, nblocks, 1};
  long long best_cost = -1;
  for (int split : {1, 2, 4}) {
    if (ksteps < split) continue;
    int maxcl = split == 1 ? sms : decode_tc_max_clusters(split, dev);
    if (split > 1 && maxcl > sms / split) maxcl = sms / split;
    if (maxcl <= 0) continue;
    int cl = nblocks < maxcl ? nblocks : maxcl;
    const int bpc = (nblocks + cl - 1) / cl;
    cl = (nblocks + bpc - 1) / bpc;
    const long long cost = static_cast<long long>(bpc) * ((ksteps + split - 1) / split);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = TcPlan{split, bpc, cl};
    }
  }
  return best;
}

template <int NR, bool META3>
int dispatch_decode_tc(const DecodeTcParams& p, int grid, int dev, cudaStream_t stream, bool grouped) {
  return grouped ? launch_decode_tc<NR, META3, true>(p, grid, dev, stream)
                 : launch_decode_tc<NR, META3, false>(p, grid, dev, stream);
}

// C[M, N] = A . dequant(B, meta, s) for M <= 64, N % 128 == 0, K % 256 == 0
// on the tensor-memory decode kernel (stages of 256 K, or 128 K for tiles of
// 48 and 64 rows: tc_stage_ks).
int mul_decode_tc(const void* A, const void* B, const void* meta, void* C, const void* s,
                  int n_out, int m_rows, int k_in, int groupsize, int dev, int sms,
                  cudaStream_t stream, int* status, const void* bias, int act, int meta_bits) {
  const int nr = (m_rows + 15) / 16 * 16;
  const int ks = tc_stage_ks(nr);  // 128-K sub-steps per stage
  const TcPlan pl = plan_decode_tc(n_out, k_in, 128 * ks, sms, dev);
  const uint64_t N = n_out, K = k_in;
  DecodeTcParams p;
  const uint64_t a_dims[3] = {64, static_cast<uint64_t>(m_rows), K / 64};
  const uint64_t a_strides[2] = {2 * K, 128};
  const uint32_t a_box[3] = {64, static_cast<uint32_t>(nr), static_cast<uint32_t>(2 * ks)};
  int rc = encode_nd(&p.tm_act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, 3, a_dims, a_strides, a_box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT64, B, N, K / 32, 8 * N, 128, 4 * ks,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (meta_bits == 3)
    rc = encode_2d(&p.tm_meta, CU_TENSOR_MAP_DATA_TYPE_UINT64, meta, 3 * N / 8, K / 32, 3 * N, 48,
                   4 * ks, CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    rc = encode_2d(&p.tm_meta, CU_TENSOR_MAP_DATA_TYPE_UINT64, meta, N / 2, K / 32, 4 * N, 64,
                   4 * ks, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  const bool grouped = groupsize != -1;
  if (grouped) {
    rc = encode_2d(&p.tm_s, CU_TENSOR_MAP_DATA_TYPE_UINT64, s, N / 4, K / 128, 2 * N, 32, ks,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    std::memset(&p.tm_s, 0, sizeof(p.tm_s));
  }
  p.s = static_cast<const uint8_t*>(s);
  p.C = static_cast<half*>(C);
  p.bias = static_cast<const half*>(bias);
  p.act = act;
  p.status = status;
  p.M = m_rows;
  p.N = n_out;
  p.ksteps = k_in / (128 * ks);
  p.split = pl.split;
  p.bpc = pl.bpc;
  p.nblocks = n_out / 128;
  p.pdl = pdl_enabled() ? 1 : 0;
  p.trace = g_trace_buffer ? g_trace_buffer + g_trace_launch++ * kTraceLaunchWords : nullptr;
  const int grid = pl.clusters * pl.split;
  const bool m3 = meta_bits == 3;
  switch (nr) {
    case 16: return m3 ? dispatch_decode_tc<16, true>(p, grid, dev, stream, grouped)
                       : dispatch_decode_tc<16, false>(p, grid, dev, stream, grouped);
    case 32: return m3 ? dispatch_decode_tc<32, true>(p, grid, dev, stream, grouped)
                       : dispatch_decode_tc<32, false>(p, grid, dev, stream, grouped);
    case 48: return m3 ? dispatch_decode_tc<48, true>(p, grid, dev, stream, grouped)
                       : dispatch_decode_tc<48, false>(p, grid, dev, stream, grouped);
    case 64: return m3 ? dispatch_decode_tc<64, true>(p, grid, dev, stream, grouped)
                       : dispatch_decode_tc<64, false>(p, grid, dev, stream, grouped);
    default: return SM100_MARLIN_ERR_KERN_SHAPE;
  }
}

// Fused all-gather targets of one call (see sm100_marlin_mul_2_4_gather).
struct GatherArgs {
  int world, rank;
  void* const* c;
  void* const* flag;
  void* target;
  const void* wait_arrival;
  const void* wait_target;
  void* const* release;  // previous call's counters (deferred release), or null
  int defer;
};

int mul_impl(const void* A, const void* B, const void* meta, void* C, const void* s, int prob_m,
             int prob_n, int prob_k, void* workspace, int groupsize, int dev, void* stream_v,
             int thread_k, int thread_m, int sms, int max_par, int meta_bits, void* scratch,
             size_t scratch_bytes, const GatherArgs* gather = nullptr, const void* bias = nullptr,
             int act = 0, int diag = 0) {
  (void)max_par;
  if (act < 0 || act > 3) return SM100_MARLIN_ERR_ARGUMENT;
  if (bias != nullptr && !aligned16(bias)) return SM100_MARLIN_ERR_ALIGNMENT;
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

  if (gather && prob_n > 64) return SM100_MARLIN_ERR_ARGUMENT;
  // Batches of 17 (3-bit metadata: 33) to 64 rows: the tensor-memory decode
  // kernel, unless the call brings its own split-K scratch (_ex, _noalloc:
  // the stream-K kernel below), gathers across GPUs, runs a metadata
  // diagnostic, or has N not a multiple of 128 or K not a multiple of 256.
  if (prob_n <= 64 && decode_tc_rows(prob_n, meta_bits) && !gather && scratch == nullptr &&
      diag == 0 && prob_m % 128 == 0 && prob_k % 256 == 0) {
    int* status = nullptr;
    rc = device_status_ptr(dev, &status);
    if (rc != SM100_MARLIN_OK) return rc;
    return mul_decode_tc(A, B, meta, C, s, prob_m, prob_n, prob_k, groupsize, dev, sms, stream,
                         status, bias, act, meta_bits);
  }
  // The tcgen05 prefill kernels take batches above 64 rows, and 33-64 rows
  // where the CTA-pair kernel's tiles fit one wave and K <= 8192: there the
  // mma.sync decode kernel (4 row blocks) is compute-bound (Llama-7B at
  // M = 64: 32.4 / 23.0 us for (4096, 12288) / (4096, 4096) against 20.7 /
  // 20.4 on the pair kernel; longer K or two waves stay on decode).
  const bool mid_batch_pair = !gather && prob_n > 32 && prob_m % 256 == 0 &&
                              prob_k % 128 == 0 && prob_k <= 8192 && prob_m / 128 <= sms &&
                              prefill_min_rows() == 64 && prefill_pair_enabled();
  // 3-bit metadata: the CTA-pair kernel decodes it (N % 256, K % 128);
  // other shapes stay on the decode kernel in 64-row chunks.
  const bool pair_meta3 = meta_bits == 3 && prob_m % 256 == 0 && prob_k % 128 == 0 &&
                          prefill_pair_enabled() && prefill_sparse_enabled() &&
                          prefill_forced_bn() != 128;
  if (((meta_bits == 4 && prob_m % 128 == 0 && prob_k % 64 == 0) || pair_meta3) &&
      (prob_n > prefill_min_rows() || mid_batch_pair)) {
    int* status = nullptr;
    rc = device_status_ptr(dev, &status);
    if (rc != SM100_MARLIN_OK) return rc;
    return mul_prefill(A, B, meta, C, s, prob_m, prob_n, prob_k, groupsize, dev, sms, stream,
                       status, bias, act, meta_bits, diag);
  }

  const int chunk_rows = prob_n < 64 ? prob_n : 64;
  Plan big = make_plan(prob_m, chunk_rows, prob_k, sms);
  if (scratch == nullptr) {
    rc = get_scratch(dev, stream, big.scratch, &scratch);
    if (rc != SM100_MARLIN_OK) return rc;
  } else if (scratch_bytes < big.scratch || !aligned16(scratch)) {
    return SM100_MARLIN_ERR_SCRATCH;
  }
  int* status = nullptr;
  rc = device_status_ptr(dev, &status);
  if (rc != SM100_MARLIN_OK) return rc;

  for (int r0 = 0; r0 < prob_n; r0 += 64) {
    const int rows = (prob_n - r0) < 64 ? (prob_n - r0) : 64;
    Plan pl = make_plan(prob_m, rows, prob_k, sms);
    GemmParams p;
    const uint8_t* a_rows = static_cast<const uint8_t*>(A) + static_cast<size_t>(r0) * prob_k * 2;
    p.s = static_cast<const uint8_t*>(s);
    p.C = reinterpret_cast<half*>(static_cast<uint8_t*>(C) + static_cast<size_t>(r0) * prob_m * 2);
    p.partials = static_cast<float4*>(scratch);
    p.counters = static_cast<int*>(workspace);
    p.status = status;
    p.M = rows;
    p.N = prob_m;
    p.K = prob_k;
    p.grouped = groupsize != -1 ? 1 : 0;
    p.kk_total = prob_k / 32;
    p.unit_kk = pl.unit_kk;
    p.units = pl.units;
    p.trace = g_trace_buffer ? g_trace_buffer + g_trace_launch++ * kTraceLaunchWords : nullptr;
    p.pdl = pdl_enabled() ? 1 : 0;
    p.prefetch = prefetch_stages();
    p.cluster = pl.cluster;
    p.bias = static_cast<const half*>(bias);
    p.act = act;
    p.gather_world = 0;
    p.gather_rank = 0;
    p.gather_target = nullptr;
    p.gather_wait_arrival = nullptr;
    p.gather_wait_target = nullptr;
    p.gather_ldc = 0;
    p.tiles_per_rank = 0;
    p.gather_defer = 0;
    for (int q = 0; q < kMaxGatherRanks; ++q) {
      p.gather_c[q] = nullptr;
      p.gather_flag[q] = nullptr;
      p.gather_release[q] = nullptr;
    }
    if (gather) {
      p.gather_world = gather->world;
      p.gather_rank = gather->rank;
      p.gather_target = static_cast<unsigned long long*>(gather->target);
      p.gather_wait_arrival = static_cast<const unsigned long long*>(gather->wait_arrival);
      p.gather_wait_target = static_cast<const unsigned long long*>(gather->wait_target);
      p.gather_ldc = static_cast<long long>(gather->world) * prob_m;
      p.tiles_per_rank = prob_m / (64 * pl.nc);
      p.gather_defer = gather->defer;
      for (int q = 0; q < gather->world; ++q) {
        p.gather_c[q] = static_cast<half*>(gather->c[q]);
        p.gather_flag[q] = static_cast<unsigned long long*>(gather->flag[q]);
        if (gather->release) p.gather_release[q] = static_cast<unsigned long long*>(gather->release[q]);
      }
      p.C = p.gather_c[gather->rank];
    }
    rc = encode_maps(p, pl, a_rows, B, meta, s, meta_bits);
    if (rc != SM100_MARLIN_OK) return rc;
    rc = meta_bits == 3 ? dispatch<true>(p, pl, dev, stream, 0)
                        : dispatch<false>(p, pl, dev, stream, diag);
    if (rc != SM100_MARLIN_OK) return rc;
  }
  return SM100_MARLIN_OK;
}

}  // namespace
}  // namespace sm100

namespace sm100 {
namespace {

struct GatherWaitParams {
  const unsigned long long* arrival;
  const unsigned long long* target;
  unsigned long long* release[kMaxGatherRanks];  // deferred release to do first, or null
  int world;
  int* status;
};

// One thread: the deferred release of the last fused all-gather call (when
// given; the previous launch on the stream has completed, so its peer stores
// are done), then a bounded wait until this rank's arrival counter of a
// buffer reaches the buffer's target (sm100_marlin_gather_wait).
__global__ void gather_wait_kernel(const __grid_constant__ GatherWaitParams p) {
  if (p.release[0] != nullptr) {
    fence_acq_rel_sys();
    for (int q = 0; q < p.world; ++q) red_add_relaxed_sys_u64(p.release[q], 1ull);
  }
  const unsigned long long* arrival = p.arrival;
  int* status = p.status;
  const unsigned long long want = *p.target;
  unsigned long long t0 = 0;
  uint32_t polls = 0;
  while (ld_acquire_sys_u64(arrival) < want) {
    if ((++polls & 63u) != 0) continue;
    const unsigned long long now = global_timer_ns();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > kWaitLimitNs) {
      atomicOr(status, kStatusGatherWaitTimeout);
      break;
    }
  }
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

int sm100_marlin_mul_2_4_epilogue(const void* A, const void* B, const void* meta, void* C,
                                  const void* s, int prob_m, int prob_n, int prob_k,
                                  void* workspace, int groupsize, int dev, void* stream,
                                  int thread_k, int thread_m, int sms, int max_par, int meta_bits,
                                  const void* bias, int activation) {
  if (meta_bits != 3 && meta_bits != 4) return SM100_MARLIN_ERR_ARGUMENT;
  return mul_impl(A, B, meta, C, s, prob_m, prob_n, prob_k, workspace, groupsize, dev, stream,
                  thread_k, thread_m, sms, max_par, meta_bits, nullptr, 0, nullptr, bias,
                  activation);
}

int sm100_marlin_mul_2_4_noalloc(const void* A, const void* B, const void* meta, void* C,
                                 const void* s, int prob_m, int prob_n, int prob_k,
                                 void* workspace, int groupsize, int dev, void* stream,
                                 int thread_k, int thread_m, int sms, int max_par) {
  int rc;
  void* scratch = nullptr;
  {
    DeviceGuard guard(dev);
    if (!guard.ok) return cuda_fail(cudaGetLastError());
    rc = noalloc_scratch(dev, &scratch);
  }
  if (rc != SM100_MARLIN_OK) return rc;
  rc = mul_impl(A, B, meta, C, s, prob_m, prob_n, prob_k, workspace, groupsize, dev, stream,
                thread_k, thread_m, sms, max_par, 4, scratch, kNoAllocScratchBytes);
  if (rc == SM100_MARLIN_ERR_SCRATCH)
    t_last_cuda_error = "problem needs more split-K scratch than the " +
                        std::to_string(kNoAllocScratchBytes >> 20) +
                        " MiB static buffer of sm100_marlin_mul_2_4_noalloc";
  return rc;
}

int sm100_marlin_mul_2_4_meta_diag(const void* A, const void* B, const void* meta, void* C,
                                   const void* s, int prob_m, int prob_n, int prob_k,
                                   void* workspace, int groupsize, int dev, void* stream,
                                   int variant) {
  if (variant < 1 || variant > 3) return SM100_MARLIN_ERR_ARGUMENT;
  if (groupsize == -1) return SM100_MARLIN_ERR_ARGUMENT;
  return mul_impl(A, B, meta, C, s, prob_m, prob_n, prob_k, workspace, groupsize, dev, stream, -1,
                  -1, -1, 16, 4, nullptr, 0, nullptr, nullptr, 0, variant);
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
  return launch_meta3_pack(meta, out, n_int16 / 8, err_count, reinterpret_cast<cudaStream_t>(stream));
}

int sm100_marlin_meta3_unpack(const void* in, void* out, int64_t n_int32, void* stream) {
  if (n_int32 < 0 || n_int32 % 48 != 0) return SM100_MARLIN_ERR_ARGUMENT;
  if (n_int32 == 0) return SM100_MARLIN_OK;
  if (!in || !out) return SM100_MARLIN_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(in) & 3u) || (reinterpret_cast<uintptr_t>(out) & 3u))
    return SM100_MARLIN_ERR_ALIGNMENT;
  return launch_meta3_unpack(in, out, n_int32 / 48 * 32, reinterpret_cast<cudaStream_t>(stream));
}

int sm100_marlin_meta3_decode_words(const void* in, void* out_high, void* out_low, int64_t n,
                                    void* stream) {
  if (n < 0) return SM100_MARLIN_ERR_ARGUMENT;
  if (n == 0) return SM100_MARLIN_OK;
  if (!in || !out_high || !out_low) return SM100_MARLIN_ERR_ARGUMENT;
  return launch_meta3_decode_words(in, out_high, out_low, n, reinterpret_cast<cudaStream_t>(stream));
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

int sm100_marlin_pack_2_4(const void* w, const void* s, int prob_k, int prob_m, int groupsize,
                          void* B, void* meta, void* s_out, int dev, void* stream_v) {
  if (prob_k <= 0 || prob_m <= 0 || prob_k % 128 != 0 || prob_m % 64 != 0)
    return SM100_MARLIN_ERR_PROB_SHAPE;
  if (groupsize != -1 && (groupsize <= 0 || prob_k % groupsize != 0))
    return SM100_MARLIN_ERR_PROB_SHAPE;
  if (!w || !s || !B || !meta || !s_out) return SM100_MARLIN_ERR_ARGUMENT;
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  return launch_pack_2_4(w, s, prob_k, prob_m, groupsize, B, meta, s_out,
                         reinterpret_cast<cudaStream_t>(stream_v));
}

int sm100_marlin_mul_2_4_gather(const void* A, const void* B, const void* meta, const void* s,
                                int prob_m, int prob_n, int prob_k, void* workspace, int groupsize,
                                int dev, void* stream, int meta_bits, void* const* gathered_c,
                                void* const* arrival, void* target, const void* wait_arrival,
                                const void* wait_target, void* const* release_arrival, int defer,
                                int world, int rank) {
  if (world < 1 || world > kMaxGatherRanks || rank < 0 || rank >= world) return SM100_MARLIN_ERR_ARGUMENT;
  if (meta_bits != 3 && meta_bits != 4) return SM100_MARLIN_ERR_ARGUMENT;
  if (!gathered_c || !arrival || !target || (wait_arrival == nullptr) != (wait_target == nullptr))
    return SM100_MARLIN_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(target) & 7u) || (reinterpret_cast<uintptr_t>(wait_arrival) & 7u) ||
      (reinterpret_cast<uintptr_t>(wait_target) & 7u))
    return SM100_MARLIN_ERR_ALIGNMENT;
  if (defer != 0 && defer != 1) return SM100_MARLIN_ERR_ARGUMENT;
  for (int q = 0; q < world; ++q) {
    if (!gathered_c[q] || !arrival[q] || (reinterpret_cast<uintptr_t>(gathered_c[q]) & 15u) ||
        (reinterpret_cast<uintptr_t>(arrival[q]) & 7u))
      return SM100_MARLIN_ERR_ALIGNMENT;
    if (release_arrival &&
        (!release_arrival[q] || (reinterpret_cast<uintptr_t>(release_arrival[q]) & 7u)))
      return SM100_MARLIN_ERR_ALIGNMENT;
  }
  const GatherArgs g{world,       rank,        gathered_c,      arrival, target,
                     wait_arrival, wait_target, release_arrival, defer};
  return mul_impl(A, B, meta, gathered_c[rank], s, prob_m, prob_n, prob_k, workspace, groupsize,
                  dev, stream, -1, -1, -1, 16, meta_bits, nullptr, 0, &g);
}

int sm100_marlin_gather_wait(const void* arrival, const void* target, void* const* release_arrival,
                             int world, int dev, void* stream) {
  if (!arrival || !target) return SM100_MARLIN_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(arrival) & 7u) || (reinterpret_cast<uintptr_t>(target) & 7u))
    return SM100_MARLIN_ERR_ALIGNMENT;
  if (release_arrival && (world < 1 || world > kMaxGatherRanks)) return SM100_MARLIN_ERR_ARGUMENT;
  GatherWaitParams wp{};
  wp.arrival = static_cast<const unsigned long long*>(arrival);
  wp.target = static_cast<const unsigned long long*>(target);
  wp.world = release_arrival ? world : 0;
  for (int q = 0; q < wp.world; ++q) {
    if (!release_arrival[q] || (reinterpret_cast<uintptr_t>(release_arrival[q]) & 7u))
      return SM100_MARLIN_ERR_ALIGNMENT;
    wp.release[q] = static_cast<unsigned long long*>(release_arrival[q]);
  }
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  int rc = device_status_ptr(dev, &wp.status);
  if (rc != SM100_MARLIN_OK) return rc;
  gather_wait_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(wp);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_ipc_alloc(size_t bytes, int dev, void** ptr) {
  if (!ptr || bytes == 0) return SM100_MARLIN_ERR_ARGUMENT;
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_ipc_free(void* ptr, int dev) {
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_ipc_get_handle(void* ptr, int dev, void* handle) {
  if (!ptr || !handle) return SM100_MARLIN_ERR_ARGUMENT;
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e);
  std::memcpy(handle, &h, sizeof(h));
  return SM100_MARLIN_OK;
}

int sm100_marlin_ipc_open(const void* handle, int dev, void** ptr) {
  if (!ptr || !handle) return SM100_MARLIN_ERR_ARGUMENT;
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_ipc_close(void* ptr, int dev) {
  DeviceGuard guard(dev);
  if (!guard.ok) return cuda_fail(cudaGetLastError());
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

int sm100_marlin_set_overlap(int enable) {
  g_pdl_override = enable ? 1 : 0;
  return SM100_MARLIN_OK;
}

int sm100_marlin_set_decode_kernel(int which) {
  if (which < SM100_MARLIN_DECODE_AUTO || which > SM100_MARLIN_DECODE_TMEM)
    return SM100_MARLIN_ERR_ARGUMENT;
  g_decode_kernel = which;
  return SM100_MARLIN_OK;
}

int sm100_marlin_set_trace_buffer(void* buf) {
  g_trace_buffer = static_cast<unsigned long long*>(buf);
  g_trace_launch = 0;
  return SM100_MARLIN_TRACE ? SM100_MARLIN_OK : SM100_MARLIN_ERR_ARGUMENT;
}

}  // extern "C"
