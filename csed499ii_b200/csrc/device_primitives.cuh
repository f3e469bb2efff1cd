// Device primitives for the sm_100a 2:4 sparse W4A16 GEMM.
//
// Replaces the reference's Ampere helpers
// (kernel_experiments/sparse_marlin/src/marlin/common/{base,mma,mem}.h):
// cp.async / ldmatrix / unbounded lock spins become TMA bulk copies tracked by
// mbarriers with *bounded* waits; the dequant and sparse MMA fragments are
// written from the PTX ISA fragment layouts.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace sm100 {

// ----------------------------------------------------------------------------
// Status bits written by kernels that gave up waiting (read by the host via
// sm100_marlin_device_status).  A kernel never traps: it records the bit and
// runs to completion without waiting any further.
// ----------------------------------------------------------------------------
enum : int {
  kStatusFullWaitTimeout = 1,    // consumer waited too long for a stage
  kStatusEmptyWaitTimeout = 2,   // producer waited too long for a free slot
  kStatusFinishWaitTimeout = 4,  // split-K finisher waited too long for partials
  kStatusGatherWaitTimeout = 8,  // fused all-gather waited too long for other ranks' blocks
};

// Metadata-cost diagnostics (a kernel template parameter DIAG, a bit set; 0
// in every production instance).  They measure what the metadata path costs,
// as the reference's constant-metadata ablations do
// (kernel_experiments/sparse_marlin/kernel_profile/setup.py:14-38), and are
// only correct for inputs whose metadata is the uniform pattern 0xEEEE:
//   kDiagNoGmem  the metadata is not copied from global memory; every stage's
//                metadata region holds 0xEEEE from kernel start and is read
//                from shared memory as usual;
//   kDiagNoReg   the metadata is copied as usual, but the kernel takes a
//                constant register instead of loading it from shared memory.
enum : int { kDiagNoGmem = 1, kDiagNoReg = 2 };
constexpr uint32_t kDiagMetaWord = 0xEEEEEEEEu;

// Timeline recording into a caller's buffer, compiled in only with
// -DSM100_MARLIN_TRACE=1 (sm100_marlin_set_trace_buffer; off by default).
#ifndef SM100_MARLIN_TRACE
#define SM100_MARLIN_TRACE 0
#endif

// Upper bound for any single wait, in nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 500ull * 1000ull * 1000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar), "r"(bytes)
      : "memory");
}

// One non-blocking-ish poll of the phase with parity `parity` (returns true
// once that phase has completed).  No suspend-time hint: on B200 a hinted
// try_wait costs ~50 cycles on a completed phase against ~15 without.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `parity` to complete.  Returns false (and leaves the
// wait) when `*abort` is raised by another thread of the CTA or when the wait
// exceeds kWaitLimitNs; in the latter case it raises `*abort` itself.
// %globaltimer is slow to read, so the abort flag and the clock are only
// checked every 1024 unsuccessful polls: a normal wait never touches them.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int* abort) {
  unsigned long long t0 = 0;
  uint32_t polls = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++polls & 1023u) != 0) continue;
    if (*abort) return false;
    const unsigned long long now = global_timer_ns();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > kWaitLimitNs) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// The same wait for warps that are not on the critical path: each poll
// suspends the thread in hardware (suspend-time hint) until the phase
// completes or ~20 us pass, so a waiting warp takes no issue slots from the
// warps that share its sub-partition.  A poll of a completed phase costs ~50
// cycles instead of ~15.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_sleep_bounded(uint32_t bar, uint32_t parity,
                                                        volatile int* abort) {
  unsigned long long t0 = 0;
  while (!mbar_try_wait_sleep(bar, parity)) {
    if (*abort) return false;
    const unsigned long long now = global_timer_ns();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > kWaitLimitNs) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// A critical-path wait that may also be long (e.g. for the previous kernel on
// the stream): polls without a hint first, then sleeps in hardware between
// polls so that a long wait takes no issue slots.
__device__ __forceinline__ bool mbar_wait_spin_sleep_bounded(uint32_t bar, uint32_t parity,
                                                             volatile int* abort) {
#pragma unroll 1
  for (int i = 0; i < 64; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_sleep_bounded(bar, parity, abort);
}

// ---------------------------------------------------------------------------
// Fused epilogue: C = act(acc [* column scale] + bias), in fp32, rounded once
// to fp16.  Activation codes match SM100_MARLIN_ACT_* of the C header.
// ---------------------------------------------------------------------------
enum : int { kActNone = 0, kActRelu = 1, kActSilu = 2, kActGeluTanh = 3 };

// Out of line: inlined, the activations' math grew the decode kernel enough
// to cost it 7 % even with the epilogue off (2048 vs 1904 GB/s, same box).
static __device__ __noinline__ float epilogue_act_call(float x, int act) {
  if (act == kActRelu) return fmaxf(x, 0.f);
  if (act == kActSilu) return x / (1.f + __expf(-x));
  if (act == kActGeluTanh) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.f + tanhf(u));
  }
  return x;
}

__device__ __forceinline__ float epilogue_act(float x, int act) {
  return act == kActNone ? x : epilogue_act_call(x, act);
}

// ---------------------------------------------------------------------------
// GPU-scope counters for the split-K hand-over between CTAs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Orders this thread's earlier (generic-proxy) accesses of global memory
// before its later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Fire-and-forget add (no return value, so the issuing thread does not wait
// for the round trip).  Callers order their earlier writes with a fence.
__device__ __forceinline__ void red_add_relaxed_gpu(int* p, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// System-scope counters for the fused all-gather between GPUs (peer memory
// over NVLink).
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void red_add_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Poll `*p` (acquire) until it reaches `target`.  Bounded like
// mbar_wait_bounded: gives up (and raises `*abort`) after kWaitLimitNs, or
// returns false when another thread raised `*abort`.
__device__ __forceinline__ bool wait_counter_bounded(const int* p, int target,
                                                     volatile int* abort) {
  unsigned long long t0 = 0;
  uint32_t polls = 0;
  while (ld_acquire_gpu(p) < target) {
    if ((++polls & 63u) != 0) continue;
    if (*abort) return false;
    const unsigned long long now = global_timer_ns();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > kWaitLimitNs) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Bulk (non-tensor) TMA copies global -> shared, completing on an mbarrier.
// Both addresses must be 16-byte aligned and `bytes` a multiple of 16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// 2-D tiled TMA load global -> shared (no multicast), completing on an
// mbarrier.  (x, y) are element coordinates of the box origin; x times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// 3-D tiled TMA load (no multicast); x is the innermost coordinate.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  launch_dependents lets the next kernel of
// the stream (launched with the programmatic-serialization attribute) begin
// once every CTA of this grid has issued it; wait blocks until the previous
// grid has completed and its memory operations are visible.  Both are no-ops
// for kernels launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dependency_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Thread-block clusters: rank, distributed shared memory, cluster barrier.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The two halves of a cluster barrier, for a CTA whose threads arrive early
// and wait later (each thread waits once per arrival, in order).  The
// relaxed arrival orders nothing by itself: mbarrier initialisations are
// published to the cluster by fence.mbarrier_init.release.cluster first.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 16 bytes into another CTA's shared memory (shared::cluster address), the
// bytes counted on that CTA's mbarrier (shared::cluster address).
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, const float4& v, uint32_t cluster_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          cluster_addr),
      "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
      "r"(__float_as_uint(v.w)), "r"(cluster_bar)
      : "memory");
}

// ---------------------------------------------------------------------------
// Named barriers for subsets of warps (id 0 is __syncthreads).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Arrive without waiting (the producer side of a named barrier whose other
// participants bar.sync): memory accesses before the arrival are performed
// for the waiting threads.
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// Four 8x8 b16 matrices; lane l supplies the row address of matrix l/8.
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Two 8x8 b16 matrices (lanes 0..15 supply row addresses).
__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}

// ---------------------------------------------------------------------------
// INT4 -> fp16.  Magic-number construction (FasterTransformer's published
// method): OR a nibble into the mantissa of 1024.0 (0x6400) to get 1024+n, or
// 1024+16n for the high nibble of a byte, then remove the offset and the
// symmetric zero point 8 with one half2 op.
//   lo(q) = (n0 - 8, n4 - 8)     hi(q) = (n1 - 8, n5 - 8)
// where n_i is nibble i of q.
// ---------------------------------------------------------------------------
// A pure function of its operands: not volatile, so the compiler may schedule
// and combine it like any other ALU operation.
template <int LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(r) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return r;
}

constexpr int kLutAndOr = (0xF0 & 0xCC) | 0xAA;  // (a & b) | c

__device__ __forceinline__ void dequant_pair(uint32_t q, half2& lo, half2& hi) {
  const uint32_t l = lop3<kLutAndOr>(q, 0x000f000fu, 0x64006400u);
  const uint32_t h = lop3<kLutAndOr>(q, 0x00f000f0u, 0x64006400u);
  const uint32_t kSub = 0x64086408u;  // (1032, 1032)
  const uint32_t kMul = 0x2c002c00u;  // (1/16, 1/16)
  const uint32_t kAdd = 0xd480d480u;  // (-72, -72)
  lo = __hsub2(*reinterpret_cast<const half2*>(&l), *reinterpret_cast<const half2*>(&kSub));
  hi = __hfma2(*reinterpret_cast<const half2*>(&h), *reinterpret_cast<const half2*>(&kMul),
               *reinterpret_cast<const half2*>(&kAdd));
}

// ---------------------------------------------------------------------------
// Sparse tensor-core MMA m16n8k32 (fp16 x fp16 -> fp32), 2:4 on operand A.
// a: 4 regs of the compressed 16x16 A tile; b: 4 regs of the dense 32x8 B
// tile; e: metadata register; SEL: sparsity selector (which thread pair of
// each quad supplies metadata).
// ---------------------------------------------------------------------------
template <int SEL>
__device__ __forceinline__ void mma_sp_16832(float (&c)[4], const uint32_t (&a)[4],
                                             uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3,
                                             uint32_t e) {
  asm volatile(
      "mma.sp::ordered_metadata.sync.aligned.m16n8k32.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9,%10,%11}, {%0,%1,%2,%3}, %12, %13;"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(b2), "r"(b3),
        "r"(e), "n"(SEL));
}

// Same MMA with a zero accumulator input (d = A.B): starts a fresh partial
// sum without clearing registers first.
template <int SEL>
__device__ __forceinline__ void mma_sp_16832_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1, uint32_t b2, uint32_t b3, uint32_t e) {
  const float z = 0.f;
  asm volatile(
      "mma.sp::ordered_metadata.sync.aligned.m16n8k32.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9,%10,%11}, {%12,%12,%12,%12}, %13, %14;"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(b2), "r"(b3), "f"(z),
        "r"(e), "n"(SEL));
}

// ---------------------------------------------------------------------------
// 3-bit metadata decode.
//
// Eight 3-bit codes in bits [0,24) are spread to nibbles (code i in bits
// [4i, 4i+3), bit 3 of every nibble clear), and each nibble then selects one
// byte of an 8-entry table with prmt (codes 0-3 from the first table word,
// 4-7 from the second); two prmts give the eight looked-up values as bytes,
// which are merged pairwise into nibbles and gathered by a third prmt.  The
// two tables are the codec's "high" map [E,D,8,D,3,4,9,C] and "low" map
// [C,D,E,A,8,9,4,0] (codes 3/4 resp. 3/7 are never produced by the packer).
// Bits [24,32) of the input are ignored.  15 instructions per word (the
// earlier form, one lop3 per output bit position, took ~23).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t spread24(uint32_t x) {
  constexpr int kSel = ((0xAA & 0xF0) | (~0xAA & 0xCC)) & 0xFF;  // c ? a : b (bitwise)
  x = lop3<kSel>(x << 4, x, 0x0fff0000u);
  x = lop3<kSel>(x << 2, x, 0x3f003f00u);
  x = lop3<kSel>(x << 1, x, 0x70707070u);
  return x;
}

__device__ __forceinline__ uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

template <uint32_t LUT_LO, uint32_t LUT_HI>
__device__ __forceinline__ uint32_t decode24_lut(uint32_t x) {
  // bit 3 of each nibble would switch prmt to sign replication: keep it clear
  const uint32_t sel = spread24(x) & 0x77777777u;
  uint32_t r0 = prmt_b32(LUT_LO, LUT_HI, sel);        // bytes: values of codes 0-3
  uint32_t r1 = prmt_b32(LUT_LO, LUT_HI, sel >> 16);  // codes 4-7
  r0 |= r0 >> 4;  // byte 0 = v0 | v1 << 4, byte 2 = v2 | v3 << 4
  r1 |= r1 >> 4;
  return prmt_b32(r0, r1, 0x6420u);
}

__device__ __forceinline__ uint32_t decode24_high(uint32_t x) {
  return decode24_lut<0x0D080D0Eu, 0x0C090403u>(x);  // [E,D,8,D | 3,4,9,C]
}

__device__ __forceinline__ uint32_t decode24_low(uint32_t x) {
  return decode24_lut<0x0A0E0D0Cu, 0x00040908u>(x);  // [C,D,E,A | 8,9,4,0]
}

// Lane-pair decode: lanes 0..15 hold (X, Y) words of their 48-bit pair,
// lanes 16..31 hold (Y, Z).  Produces the lane's two 4-bit metadata words
// (original words `lane` and `32 + lane` of the 64-word block).
__device__ __forceinline__ void meta3_pair_decode(uint32_t a, uint32_t b, bool upper,
                                                  uint32_t& w0, uint32_t& w1) {
  const uint32_t hi_in = upper ? __funnelshift_r(a, b, 16) : a;
  const uint32_t lo_in = upper ? (b >> 8) : __funnelshift_r(a, b, 24);
  w0 = decode24_high(hi_in);
  w1 = decode24_low(lo_in);
}

}  // namespace sm100
