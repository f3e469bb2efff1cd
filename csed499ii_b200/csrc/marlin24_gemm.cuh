// 2:4 sparse W4A16 GEMM for the decode regime (batch rows M <= 64 per launch),
// sm_100a.
//
//   C[M, N] (fp16) = A[M, K] (fp16) . dequant(B, meta, s)[K, N]
//
// Consumes the Sparse-Marlin packed layout unchanged (reference:
// kernel_experiments/sparse_marlin/src/marlin/__init__.py:331-388 for B/s,
// _semi_structured_conversions.py:54-179 for meta, and the 3-bit metadata of
// kernel_experiments/sparse_marlin/metadata_decode/codec.cu:18-24).
//
// Design (B200-first, not a translation of marlin_cuda_kernel_nm.cu):
//  * Work = column tiles of 64*NC out-features x K.  The (tile, K-slice)
//    "units" are laid out tile-major and split evenly over a persistent grid
//    of one CTA per SM, so every SM streams the same number of weight bytes
//    whatever the shape (stream-K style split).
//  * Producer warps stream each stage -- SK rows of 32 dense K of B,
//    metadata and scales of the tile, plus the activation slice -- with one
//    TMA tensor copy per operand into a deep shared-memory ring (mbarrier
//    full/empty pairs, evict-first L2 policy for the weight stream; the
//    activation box is 128-byte swizzled so ldmatrix is bank-conflict free).
//    A warp can only keep about one stage per ~0.3 us in flight on B200, so
//    kProducerWarps warps take the stages round-robin.  Every wait is bounded
//    (%globaltimer) and records a status bit instead of hanging.
//  * Eight consumer warps each own one (32-K row, 64-column chunk) block per
//    stage: one 16-byte B load, the metadata words (ldmatrix.x2 for 4-bit,
//    two 32-bit loads + lop3 decode for 3-bit), INT4 -> fp16 magic-number
//    dequant with the group scale fused, and mma.sp m16n8k32 with fp32
//    accumulators.
//  * Split-K partials are reduced in fp32: warps of a CTA through shared
//    memory (a tree), CTAs of a tile through a scratch buffer and a per-tile
//    counter in the caller's workspace.  The CTA holding a tile's first K
//    units (for it always its last segment) finishes the tile: the others
//    publish their partials and count them without waiting, a producer thread
//    of the finisher polls the counter while its consumers still compute, and
//    the finisher adds the partials in CTA order (deterministic) and writes C.
//    When the tiles times 2 or 3 fill the SMs, the CTAs of a tile form one
//    thread-block cluster instead and send their partials into the
//    finisher's shared memory with st.async (cluster split-K, no scratch).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "device_primitives.cuh"

namespace sm100 {

constexpr int kMaxGatherRanks = 8;

struct GemmParams {
  CUtensorMap tm_a;     // A  fp16 (64, M rows, K/64) box (64, 16*MB, SK/2), 128B swizzle
  CUtensorMap tm_b;     // B  u64  (K/32 rows, N)     box (64*NC, SK)
  CUtensorMap tm_meta;  // meta u64 (K/32 rows, N/2 or 3N/8) box (32*NC or 24*NC, SK)
  CUtensorMap tm_s;     // s  u64  (K/128 rows, N/4)  box (16*NC, S_ROWS)   (grouped only)
  const uint8_t* s;     // fp16 scales (per-column epilogue reads)
  half* C;              // fp16 (M, N) row-major
  float4* partials;     // split-K scratch
  int* counters;        // one int per column tile; zero on entry and on exit
  int* status;          // device status word (timeouts)
  int M;                // rows in this launch, 1..64
  int N;
  int K;
  int grouped;          // 1: group of 128 dense K; 0: one scale per column
  int kk_total;         // K / 32
  int unit_kk;          // 32-K rows per unit (2, 4 or 8); divides kk_total
  long long units;      // n_tiles * kk_total / unit_kk
  unsigned long long* trace;  // optional per-CTA timestamps (SM100_MARLIN_TRACE builds)
  int pdl;              // launched with programmatic dependent launch
  const half* bias;     // fused epilogue: fp16 bias per output column, or null
  int act;              // fused epilogue: activation (kAct*)
  int prefetch;         // stages whose weights may be issued before griddepcontrol.wait
  // Fused all-gather of column-parallel shards (gather_world > 0): every C row
  // this launch computes is stored into each rank's gathered buffer (peer
  // memory over NVLink) at this rank's column block, then counted on each
  // rank's arrival counter:
  //  - per-call release (gather_defer = 0): each CTA, after its stores, with a
  //    system-scope fence and the number of tiles it stored;
  //  - deferred release (gather_defer = 1): no CTA waits for its stores; a
  //    later launch (the next call's CTA 0, right after its programmatic-
  //    launch wait, through gather_release; or the completion wait) fences
  //    once, when this launch has completed, and adds 1 per rank.
  // CTA 0 adds this call's count (world x tiles_per_rank, or world) to the
  // buffer's cumulative target, then returns only once the counter
  // gather_wait_arrival has reached *gather_wait_target: this call's own
  // counter and target (the call completes with its all-gather), an earlier
  // call's (pipelined completion), or nothing (null).
  half* gather_c[kMaxGatherRanks];                   // each rank's gathered C (row 0 of this launch)
  unsigned long long* gather_flag[kMaxGatherRanks];  // each rank's arrival counter
  unsigned long long* gather_target;                 // this rank's cumulative target of this buffer
  const unsigned long long* gather_wait_arrival;     // counter this launch waits on, or null
  const unsigned long long* gather_wait_target;      // the target it waits for
  unsigned long long* gather_release[kMaxGatherRanks];  // previous call's counters (deferred), or null
  int gather_defer;                                  // 1: deferred release of this call
  long long gather_ldc;                              // row stride of the gathered C (elements)
  int gather_world;                                  // 0: plain stores to C
  int gather_rank;
  int tiles_per_rank;                                // tiles each rank stores per call
  // Cluster split-K (batch <= 16): 0 or 1 for the stream-K split over the
  // whole grid; S = 2 or 3 when the grid is n_tiles * S CTAs launched as
  // clusters of S, one cluster per column tile.  The CTAs of a tile then
  // hand their partials to the tile's finisher (cluster rank 0) through
  // distributed shared memory instead of the scratch and counters.
  int cluster;
};

// Per-CTA timeline written when the library is built with
// -DSM100_MARLIN_TRACE=1 (off by default): %globaltimer at kernel entry, first
// TMA issue, first stage consumed, last stage consumed, end of epilogue, the
// number of stages and fixups of the CTA, the time its consumers returned
// from the programmatic-launch wait, and inside the epilogue of the last
// segment: [11] past the dependency wait, [8] warps reduced, [9] finisher
// partials ready, [10] C stores issued (warp 0 of chunk 0).
constexpr int kTraceWords = 16;
// CTA 0 additionally records per-stage SM clock cycles (clock64, cheap to
// read) after the per-CTA words: [stage][0] producer issue, [1..3] consumer
// warp 0 wait start / data ready / done, [4..6] the same for the last
// consumer warp, [7] the CTA's clock at entry (for the offsets).
constexpr int kTraceStages = 64;
constexpr int kTraceStageWords = 8;
// Words per launch in a trace buffer (grid <= 256 CTAs).
constexpr long long kTraceLaunchWords = 256 * kTraceWords + kTraceStages * kTraceStageWords;

// Warp roles per configuration: 8 consumer warps; 2 producer warps for batch
// rows <= 16 (24 KB weight stages) and 4 for larger batches (smaller stages).
constexpr int consumer_warps(int mb) { return 8; }
constexpr int producer_warps(int nc, int mb) { return (mb == 1 || (nc == 1 && mb == 4)) ? 2 : 4; }
// Consecutive 32-K rows of one chunk per consumer warp per stage: 2, except
// for narrow tiles with many batch rows (64 columns above 16 rows, 128 columns
// at 64 rows), whose activation slices would not fit a useful ring.
constexpr int rows_per_warp(int nc, int mb) {
  return mb == 1 ? 4 : (((nc == 1 && mb > 1) || (nc == 2 && mb == 4)) ? 1 : 2);
}
// Group scales are applied to the dequantised weights (fp16 multiply, as the
// reference does) rather than to per-group fp32 temporaries: on B200 the
// temporaries' extra accumulator traffic costs more than the multiplies
// (118 vs 69 cycles per 32x64 block per sub-partition, measured).  The
// accumulator variant stays available for experiments.
constexpr bool scale_on_accumulator(int mb) { return false; }

constexpr int kSmemBudget = 227 * 1024;

template <int NC, int MB, bool META3>
struct DecodeCfg {
  static constexpr int CW = consumer_warps(MB);
  static constexpr int PW = producer_warps(NC, MB);
  static constexpr int THREADS = (CW + PW) * 32;
  static constexpr int WPC = CW / NC;                            // consumer warps per chunk
  static constexpr int RPW = rows_per_warp(NC, MB);
  static constexpr bool SCALE_ACC = scale_on_accumulator(MB);
  static constexpr int SK = CW * RPW / NC;                       // 32-K rows per stage
  static constexpr int B_ROW = 512 * NC;                         // bytes of B per row
  static constexpr int M_BLK = META3 ? 192 : 256;                // meta bytes per (row, chunk)
  static constexpr int M_ROW = M_BLK * NC;
  static constexpr int S_ROW = 128 * NC;                         // scale bytes per group row
  static constexpr int S_ROWS = SK / 4;                          // group rows per stage
  static constexpr int A_BOXES = SK / 2;                         // 64-K activation boxes
  static constexpr int A_BOX = 16 * MB * 128;                    // bytes per activation box
  static constexpr int OFF_A = 0;                                // 1024-aligned (swizzle atom)
  static constexpr int OFF_B = OFF_A + A_BOXES * A_BOX;
  static constexpr int OFF_M = OFF_B + SK * B_ROW;
  static constexpr int OFF_S = OFF_M + SK * M_ROW;
  static constexpr int STAGE_RAW = OFF_S + S_ROWS * S_ROW;
  static constexpr int STAGE = (STAGE_RAW + 1023) / 1024 * 1024;
  static constexpr int ACC_F4 = 8 * MB;                          // float4 per thread of acc
  static constexpr int ACC_BYTES = ACC_F4 * 32 * 16;             // one warp's accumulators
  static constexpr int HEADER = 1024;                            // barriers + flags
  // The warps sharing a chunk reduce pairwise (a tree); WPC/2 shared-memory
  // slots per chunk let each level run in one pass, unless they would cost the
  // ring more than one stage.
  static constexpr int ring_depth(int slots) {
    return (kSmemBudget - (HEADER + NC * slots * ACC_BYTES + 1023) / 1024 * 1024 -
            (MB == 1 ? 2 * NC * ACC_BYTES : 0) - 1024) / STAGE;
  }
  // Batch <= 16: one flat pass instead (every warp but the leader writes its
  // accumulators, the leader adds them in warp order) when the WPC-1 slots
  // cost the ring no stage.
  static constexpr bool FLAT_RED = MB == 1 && WPC > 2 && ring_depth(WPC - 1) >= ring_depth(WPC / 2);
  static constexpr int RED_SLOTS =
      FLAT_RED ? WPC - 1
               : ((WPC / 2 > 1 && ring_depth(WPC / 2) + 1 >= ring_depth(1)) ? WPC / 2 : 1);
  static constexpr int RED_BYTES = NC * RED_SLOTS * ACC_BYTES;
  // Split-K finisher: room for the partials of up to FIN_SLOTS other CTAs of
  // its tile, bulk-copied in while the finisher still computes (batch <= 16;
  // larger partials are read from global memory at the end).
  static constexpr int FIN_SLOTS = MB == 1 ? 2 : 0;
  static constexpr int FIN_BYTES = FIN_SLOTS * NC * ACC_BYTES;
  static constexpr int FIN_OFF = (HEADER + RED_BYTES + 1023) / 1024 * 1024;
  static constexpr int RING_OFF = (FIN_OFF + FIN_BYTES + 1023) / 1024 * 1024;
  static constexpr int DEPTH_FIT = (kSmemBudget - RING_OFF - 1024) / STAGE;
  static constexpr int DEPTH = DEPTH_FIT > 16 ? 16 : DEPTH_FIT;
  static constexpr int SMEM = RING_OFF + DEPTH * STAGE + 1024;   // +1024: base alignment slack
  static constexpr uint32_t STAGE_TX_NOSCALE = A_BOXES * A_BOX + SK * (B_ROW + M_ROW);
  static_assert(DEPTH >= PW, "ring too shallow for the producer warps");
  static constexpr uint32_t STAGE_TX_SCALE = STAGE_TX_NOSCALE + S_ROWS * S_ROW;
  static_assert(DEPTH >= 2, "ring too shallow");
  static_assert(SK % 4 == 0, "stage must hold whole scale groups");
  static_assert(!SCALE_ACC || RPW == 4, "accumulator scaling needs whole groups per warp");
  static_assert(THREADS <= 1024, "too many threads");
};

// floor(num / den) for 0 <= num < 2^53, den > 0, without the slow 64-bit
// integer division: a double quotient corrected by at most one step.
__device__ __forceinline__ long long floor_div(long long num, long long den) {
  long long q = static_cast<long long>(static_cast<double>(num) / static_cast<double>(den));
  if (q * den > num) --q;
  if ((q + 1) * den <= num) ++q;
  return q;
}
// Unit range of CTA c in a split of `units` over `grid` CTAs.
__device__ __forceinline__ long long unit_begin(long long c, long long units, long long grid) {
  return floor_div(c * units, grid);
}
// CTA owning unit u (the largest c with unit_begin(c) <= u).
__device__ __forceinline__ long long unit_owner(long long u, long long units, long long grid) {
  return floor_div((u + 1) * grid - 1, units);
}

__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// EPI: the fused bias / activation epilogue is compiled in (a separate
// instantiation: even out of line, the epilogue code cost the plain kernel
// 3.5 %, 2059 vs 1988 GB/s on the same box).
template <int NC, int MB, int NH_LAST, bool META3, bool GROUPED, bool EPI, int DIAG = 0>
__global__ void __launch_bounds__(DecodeCfg<NC, MB, META3>::THREADS, 1)
    marlin24_decode_kernel(const __grid_constant__ GemmParams p) {
  static_assert(DIAG == 0 || (!META3 && !EPI), "diagnostics: 4-bit metadata, plain store");
  using Cfg = DecodeCfg<NC, MB, META3>;
  constexpr int SK = Cfg::SK;
  constexpr int D = Cfg::DEPTH;
  constexpr int kConsumerWarps = Cfg::CW;
  constexpr int kProducerWarps = Cfg::PW;

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment of the ring (128B-swizzle atoms).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty_bar = full_bar + D;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 512);
  // Split-K finisher hand-over: a producer thread arrives once the partials
  // of every other CTA of the finisher's tile are published.
  uint64_t* fin_bar = reinterpret_cast<uint64_t*>(smem + 520);
  uint8_t* red = smem + Cfg::HEADER;
  uint8_t* fin = smem + Cfg::FIN_OFF;
  uint8_t* ring = smem + Cfg::RING_OFF;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.cluster > 1 ? p.cluster : 1;
  const uint32_t crank = S > 1 ? cluster_cta_rank() : 0u;
  unsigned long long* trace =
      SM100_MARLIN_TRACE && p.trace ? p.trace + static_cast<long long>(blockIdx.x) * kTraceWords : nullptr;
  if (trace && threadIdx.x == 0) {
    trace[0] = global_timer_ns();
    if (blockIdx.x == 0) p.trace[gridDim.x * kTraceWords + 7] = clock64();
  }

  if (threadIdx.x < D) {
    mbar_init(smem_addr(&full_bar[threadIdx.x]), 1);
    mbar_init(smem_addr(&empty_bar[threadIdx.x]), kConsumerWarps);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(smem_addr(fin_bar), 1);
    fence_mbar_init();
    // cluster split-K: rank 0 finishes the tile and receives the S - 1
    // partials of the other ranks, counted as bytes on fin_bar
    if (S > 1 && crank == 0)
      mbar_arrive_expect_tx(smem_addr(fin_bar), static_cast<uint32_t>((S - 1) * NC * Cfg::ACC_BYTES));
  }
  if constexpr ((DIAG & kDiagNoGmem) != 0) {
    // uniform metadata in every stage's region, written once (never copied)
    for (int st = 0; st < D; ++st) {
      uint32_t* mreg = reinterpret_cast<uint32_t*>(smem + Cfg::RING_OFF + st * Cfg::STAGE + Cfg::OFF_M);
      for (int i = threadIdx.x; i < SK * Cfg::M_ROW / 4; i += blockDim.x) mreg[i] = kDiagMetaWord;
    }
  }
  // Let the next kernel on the stream start its prologue and weight prefetch
  // while this one runs (it waits for this grid before touching anything
  // this kernel reads or writes besides the weights).
  if (p.pdl && threadIdx.x == 0) grid_dependency_launch();
  if (threadIdx.x == kConsumerWarps * 32) {
    prefetch_tmap(&p.tm_a);
    prefetch_tmap(&p.tm_b);
    prefetch_tmap(&p.tm_meta);
    if (GROUPED) prefetch_tmap(&p.tm_s);
  }
  __syncthreads();
  // the peers' barriers exist before any st.async (waited on by each warp
  // before its first remote store, or before it leaves)
  if (S > 1) cluster_arrive_relaxed();
  bool cluster_waited = false;

  const long long grid = gridDim.x;
  const long long cta = blockIdx.x;
  const long long u_begin = unit_begin(cta, p.units, grid);
  const long long u_end = unit_begin(cta + 1, p.units, grid);
  const int units_per_tile = p.kk_total / p.unit_kk;
  const int ukk = p.unit_kk;
  const uint32_t ring_base = smem_addr(ring);

  if (warp >= kConsumerWarps) {
    // ------------------------------------------------------------------ producers
    // Producer warp pw (lane 0) issues every stage s with s % PW == pw.
    const int pw = warp - kConsumerWarps;
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      const uint32_t tx = (GROUPED ? Cfg::STAGE_TX_SCALE : Cfg::STAGE_TX_NOSCALE) -
                          ((DIAG & kDiagNoGmem) ? SK * Cfg::M_ROW : 0);
      // With programmatic dependent launch the previous kernel on the stream
      // may still be running: the weight parts of the first ring's worth of
      // stages are issued before griddepcontrol.wait; the activation parts,
      // which the previous kernel may have produced, only after it.
      constexpr int kPre = (D + kProducerWarps - 1) / kProducerWarps;
      int pre_slot[kPre], pre_kk[kPre];
      int n_pre = 0;
      bool waited = !p.pdl;
      auto issue_a = [&](int slot, int kk0) {
        const uint32_t full = smem_addr(&full_bar[slot]);
        tma_load_3d(ring_base + slot * Cfg::STAGE + Cfg::OFF_A, &p.tm_a, 0, 0, kk0 >> 1, full,
                    pol_keep);
      };
      // Deferred all-gather release of the previous call (CTA 0): once the
      // previous launch has completed (programmatic-launch wait, or a launch
      // without overlap), its peer stores are done; one system-scope fence
      // orders them before the counts.
      auto release_previous_gather = [&]() {
        if (blockIdx.x == 0 && pw == 0 && p.gather_release[0] != nullptr) {
          fence_acq_rel_sys();
          for (int q = 0; q < p.gather_world; ++q) red_add_relaxed_sys_u64(p.gather_release[q], 1ull);
        }
      };
      if (waited) release_previous_gather();
      auto release_deferred = [&]() {
        grid_dependency_wait();
        waited = true;
        release_previous_gather();
        for (int i = 0; i < n_pre; ++i) issue_a(pre_slot[i], pre_kk[i]);
        n_pre = 0;
      };
      uint32_t stage = 0;
      bool ok = true;
      for (long long u = u_begin; u < u_end && ok;) {
        const int ui = static_cast<int>(u);
        const int tile = ui / units_per_tile;
        const int ub = ui - tile * units_per_tile;
        const long long ue_ll = ub + (u_end - u);
        const int ue = ue_ll < units_per_tile ? static_cast<int>(ue_ll) : units_per_tile;
        u += ue - ub;
        const int kb = ub * ukk, ke = ue * ukk;
        for (int kk0 = kb; kk0 < ke; kk0 += SK, ++stage) {
          if (static_cast<int>(stage % kProducerWarps) != pw) continue;
          const int slot = stage % D;
          const uint32_t parity = ((stage / D) & 1u) ^ 1u;
          // a slot can only be free again after its stage was consumed, which
          // needs the deferred activation loads: release them first
          if (!waited && static_cast<int>(stage) >= (p.prefetch < D ? p.prefetch : D))
            release_deferred();
          if (!mbar_wait_bounded(smem_addr(&empty_bar[slot]), parity, abort_flag)) {
            atomicOr(p.status, kStatusEmptyWaitTimeout);
            ok = false;
            break;
          }
          if (trace && stage == 0) trace[1] = global_timer_ns();
          if (trace && blockIdx.x == 0 && stage < kTraceStages)
            p.trace[gridDim.x * kTraceWords + stage * kTraceStageWords] = clock64();
          const uint32_t full = smem_addr(&full_bar[slot]);
          const uint32_t st = ring_base + slot * Cfg::STAGE;
          mbar_arrive_expect_tx(full, tx);
          tma_load_2d(st + Cfg::OFF_B, &p.tm_b, tile * 64 * NC, kk0, full, pol_stream);
          if constexpr ((DIAG & kDiagNoGmem) == 0)
            tma_load_2d(st + Cfg::OFF_M, &p.tm_meta, tile * (Cfg::M_BLK / 8) * NC, kk0, full,
                        pol_stream);
          if (GROUPED)
            tma_load_2d(st + Cfg::OFF_S, &p.tm_s, tile * 16 * NC, kk0 >> 2, full, pol_keep);
          if (waited) {
            issue_a(slot, kk0);
          } else {
            pre_slot[n_pre] = slot;
            pre_kk[n_pre] = kk0;
            ++n_pre;
          }
        }
      }
      if (!waited) release_deferred();
      // Split-K finisher: when this CTA's last segment starts a tile that
      // other CTAs finish, wait (here, while the consumers still compute) for
      // their partials to be published, then hand over to the consumers.
      // The counters are only read after griddepcontrol.wait (above), so the
      // previous kernel's use of them is over.
      if (pw == 0 && ok && S == 1) {
        const long long last_tile = (u_end - 1) / units_per_tile;
        const long long t0 = last_tile * units_per_tile;
        if (u_begin <= t0 && u_end < t0 + units_per_tile) {
          const int others =
              static_cast<int>(unit_owner(t0 + units_per_tile - 1, p.units, grid) - cta);
          const uint32_t fb = smem_addr(fin_bar);
          if (!wait_counter_bounded(&p.counters[last_tile], others, abort_flag)) {
            atomicOr(p.status, kStatusFinishWaitTimeout);
            mbar_arrive(fb);
          } else {
            // bring the first FIN_SLOTS partials next to the consumers
            const int n_fin = others < Cfg::FIN_SLOTS ? others : Cfg::FIN_SLOTS;
            constexpr uint32_t kPart = NC * Cfg::ACC_BYTES;
            if (n_fin > 0) {
              fence_proxy_async_global();
              mbar_arrive_expect_tx(fb, n_fin * kPart);
              for (int i = 0; i < n_fin; ++i)
                bulk_g2s(smem_addr(fin) + i * kPart,
                         p.partials + ((cta + 1 + i) * NC) * Cfg::ACC_F4 * 32, kPart, fb,
                         policy_evict_first());
            } else {
              mbar_arrive(fb);
            }
          }
        }
      }
    }
    if (S > 1) cluster_wait();
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cc = warp % NC;                // 64-column chunk inside the tile
  const int kl = (warp / NC) * Cfg::RPW;  // first of this warp's 32-K rows in a stage
  const int g = lane >> 2;
  const int t = lane & 3;
  float acc[MB][4][2][4];
  uint32_t stage = 0;
  bool aborted = false;
  bool epi_waited = !p.pdl;
  int tiles_stored = 0;  // tiles this CTA wrote to C (counted by thread 0)

  // Per-warp shared-memory offsets inside a stage, computed once: every
  // per-stage load is then (stage base + constant) with an immediate row
  // offset.  Activations: row ar of the 128B-swizzled box keeps 16-byte chunk
  // c at chunk c ^ (ar & 7).  a_off[p][mb][h] addresses, for a 32-K row of
  // parity p, the 8 batch rows 16mb+8h.. with lane group q = lane/8 on K
  // 8q..8q+7, so one ldmatrix.x4 returns a complete mma B operand in order
  // (assembling it from two loads costs ~30 % of the inner loop).
  const uint32_t b_off = Cfg::OFF_B + kl * Cfg::B_ROW + cc * 512 + lane * 16;
  const uint32_t m_off = Cfg::OFF_M + kl * Cfg::M_ROW + cc * Cfg::M_BLK +
                         (META3 ? lane * 4 : (lane & 15) * 16);
  const uint32_t s_off = Cfg::OFF_S + (kl >> 2) * Cfg::S_ROW + cc * 128 + g * 16;
  uint32_t a_off[2][MB][2];
#pragma unroll
  for (int par = 0; par < 2; ++par)
#pragma unroll
    for (int mb = 0; mb < MB; ++mb)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int ar = 16 * mb + 8 * h + (lane & 7);
        const int c = par * 4 + (lane >> 3);
        a_off[par][mb][h] = Cfg::OFF_A + (kl >> 1) * Cfg::A_BOX + ar * 128 + ((c ^ (ar & 7)) << 4);
      }

  for (long long u = u_begin; u < u_end;) {
    const int ui = static_cast<int>(u);
    const int tile = ui / units_per_tile;
    const int ub = ui - tile * units_per_tile;
    const long long ue_ll = ub + (u_end - u);
    const int ue = ue_ll < units_per_tile ? static_cast<int>(ue_ll) : units_per_tile;
    u += ue - ub;
    const int kb = ub * ukk, ke = ue * ukk;

#pragma unroll
    for (int mb = 0; mb < MB; ++mb)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mb][j][h][e] = 0.f;

    for (int kk0 = kb; kk0 < ke; kk0 += SK, ++stage) {
      const int rows = min(SK, ke - kk0);
      const int slot = stage % D;
      const uint32_t parity = (stage / D) & 1u;
      unsigned long long* st_trace =
          (trace && blockIdx.x == 0 && stage < kTraceStages && lane == 0 &&
           (warp == 0 || warp == kConsumerWarps - 1))
              ? p.trace + gridDim.x * kTraceWords + stage * kTraceStageWords + (warp == 0 ? 1 : 4)
              : nullptr;
      if (st_trace) st_trace[0] = clock64();
      if (!aborted && !mbar_wait_bounded(smem_addr(&full_bar[slot]), parity, abort_flag)) {
        aborted = true;
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
      }
      if (st_trace) st_trace[1] = clock64();
      if (!aborted && kl < rows) {
        const uint32_t st = ring_base + slot * Cfg::STAGE;
        const int nr = min(Cfg::RPW, rows - kl);  // rows of this warp in this stage
        // one scale row serves the warp's rows (kl is a multiple of RPW, stage
        // starts are multiples of 4 when grouped, groups are 4 rows)
        uint4 sv = make_uint4(0, 0, 0, 0);
        if (GROUPED) sv = lds128(st + s_off);
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
        constexpr bool kTmp = GROUPED && Cfg::SCALE_ACC;
        float tmp[kTmp ? MB : 1][4][2][4];
        auto rows_body = [&](auto full) {
          constexpr bool kFull = decltype(full)::value;
#pragma unroll
          for (int r = 0; r < Cfg::RPW; ++r) {
            if (!kFull && r >= nr) break;
            const uint4 q = lds128(st + b_off + r * Cfg::B_ROW);
            uint32_t mw[2];
            if constexpr (META3) {
              const uint32_t a = lds32(st + m_off + r * Cfg::M_ROW);
              const uint32_t b = lds32(st + m_off + r * Cfg::M_ROW + 64);
              meta3_pair_decode(a, b, (lane & 16) != 0, mw[0], mw[1]);
            } else if constexpr ((DIAG & kDiagNoReg) != 0) {
              mw[0] = kDiagMetaWord;
              mw[1] = kDiagMetaWord;
            } else {
              ldmatrix_x2(mw, st + m_off + r * Cfg::M_ROW);
            }
            // row parity / box index: compile-time when kl is even (RPW even)
            const int par = (Cfg::RPW % 2 == 0) ? (r & 1) : ((kl + r) & 1);
            const uint32_t abox = st + (((kl & 1) + r) >> 1) * Cfg::A_BOX;
            uint32_t bf[MB][2][4];
#pragma unroll
            for (int mb = 0; mb < MB; ++mb)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (h == 1 && mb == MB - 1 && NH_LAST == 1) continue;
                ldmatrix_x4(bf[mb][h], abox + (par ? a_off[1][mb][h] : a_off[0][mb][h]));
              }
            const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              half2 lo0, hi0, lo1, hi1;
              dequant_pair(qw[j], lo0, hi0);
              dequant_pair(qw[j] >> 8, lo1, hi1);
              if (GROUPED && !kTmp) {
                const half2 s2 = *reinterpret_cast<const half2*>(&sw[j]);
                const half2 sx = __low2half2(s2), sy = __high2half2(s2);
                lo0 = __hmul2(lo0, sx);
                hi0 = __hmul2(hi0, sx);
                lo1 = __hmul2(lo1, sy);
                hi1 = __hmul2(hi1, sy);
              }
              const uint32_t af[4] = {*reinterpret_cast<uint32_t*>(&lo0), *reinterpret_cast<uint32_t*>(&lo1),
                                      *reinterpret_cast<uint32_t*>(&hi0), *reinterpret_cast<uint32_t*>(&hi1)};
              const uint32_t e = mw[j >> 1];
#pragma unroll
              for (int mb = 0; mb < MB; ++mb) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  if (h == 1 && mb == MB - 1 && NH_LAST == 1) continue;
                  float(&d)[4] = kTmp ? tmp[kTmp ? mb : 0][j][h] : acc[mb][j][h];
                  if (kTmp && r == 0) {
                    if (j & 1)
                      mma_sp_16832_z<1>(d, af, bf[mb][h][0], bf[mb][h][1], bf[mb][h][2], bf[mb][h][3], e);
                    else
                      mma_sp_16832_z<0>(d, af, bf[mb][h][0], bf[mb][h][1], bf[mb][h][2], bf[mb][h][3], e);
                  } else {
                    if (j & 1)
                      mma_sp_16832<1>(d, af, bf[mb][h][0], bf[mb][h][1], bf[mb][h][2], bf[mb][h][3], e);
                    else
                      mma_sp_16832<0>(d, af, bf[mb][h][0], bf[mb][h][1], bf[mb][h][2], bf[mb][h][3], e);
                  }
                }
              }
            }
          }
        };
        if (nr == Cfg::RPW)
          rows_body(std::true_type{});
        else
          rows_body(std::false_type{});
        if constexpr (kTmp) {
          // acc += s (group scale of the output column) * tmp, in fp32.
          // frag_s[j] = (scale of out-feature 8g+j, of 8g+j+4): x for the
          // accumulator rows g (elements 0,1), y for rows g+8 (elements 2,3).
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const half2 s2 = *reinterpret_cast<const half2*>(&sw[j]);
            const float sx = __low2float(s2), sy = __high2float(s2);
#pragma unroll
            for (int mb = 0; mb < MB; ++mb)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (h == 1 && mb == MB - 1 && NH_LAST == 1) continue;
                acc[mb][j][h][0] = fmaf(sx, tmp[mb][j][h][0], acc[mb][j][h][0]);
                acc[mb][j][h][1] = fmaf(sx, tmp[mb][j][h][1], acc[mb][j][h][1]);
                acc[mb][j][h][2] = fmaf(sy, tmp[mb][j][h][2], acc[mb][j][h][2]);
                acc[mb][j][h][3] = fmaf(sy, tmp[mb][j][h][3], acc[mb][j][h][3]);
              }
          }
        }
      }
      __syncwarp();
      if (st_trace) st_trace[2] = clock64();
      if (lane == 0) mbar_arrive(smem_addr(&empty_bar[slot]));
      if (trace && threadIdx.x == 0) {
        if (stage == 0) trace[2] = global_timer_ns();
        trace[3] = global_timer_ns();
        trace[5] = stage + 1;
      }
    }

    // ---------------------------------------------------------------- epilogue
    // C, the split-K scratch and the workspace tickets may still be in use by
    // the previous kernel on the stream until it has completed.
    if (!epi_waited) {
      grid_dependency_wait();
      epi_waited = true;
      if (trace && threadIdx.x == 0) trace[7] = global_timer_ns();
    }
    if (trace && threadIdx.x == 0) trace[11] = global_timer_ns();
    // 1) reduce the WPC warps of each chunk through shared memory, flat (see
    //    FLAT_RED) or as a tree:
    //    at each level warps [h, 2h) add into warps [0, h) (slot-limited
    //    passes); the summation order is fixed, so results are deterministic.
    float4* acc4 = reinterpret_cast<float4*>(&acc[0][0][0][0]);
    const int wk = warp / NC;  // warp index among the warps sharing this chunk
    if constexpr (Cfg::FLAT_RED) {
      float4* red4 = reinterpret_cast<float4*>(red) + (cc * Cfg::RED_SLOTS * Cfg::ACC_F4) * 32 + lane;
      if (wk != 0) {
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) red4[((wk - 1) * Cfg::ACC_F4 + v) * 32] = acc4[v];
      }
      named_bar_sync(1, kConsumerWarps * 32);
      if (wk == 0) {
#pragma unroll
        for (int w = 0; w < Cfg::RED_SLOTS; ++w)
#pragma unroll
          for (int v = 0; v < Cfg::ACC_F4; ++v) {
            const float4 x = red4[(w * Cfg::ACC_F4 + v) * 32];
            acc4[v].x += x.x; acc4[v].y += x.y; acc4[v].z += x.z; acc4[v].w += x.w;
          }
      }
      named_bar_sync(1, kConsumerWarps * 32);
    }
    for (int h = Cfg::FLAT_RED ? 0 : Cfg::WPC / 2; h >= 1; h /= 2) {
      for (int base = 0; base < h; base += Cfg::RED_SLOTS) {
        const int slot_w = wk - h - base;  // writer's slot this pass
        const int slot_r = wk - base;      // reader's slot this pass
        float4* red4w = reinterpret_cast<float4*>(red) +
                        ((cc * Cfg::RED_SLOTS + slot_w) * Cfg::ACC_F4) * 32;
        float4* red4r = reinterpret_cast<float4*>(red) +
                        ((cc * Cfg::RED_SLOTS + slot_r) * Cfg::ACC_F4) * 32;
        if (slot_w >= 0 && slot_w < Cfg::RED_SLOTS) {
#pragma unroll
          for (int v = 0; v < Cfg::ACC_F4; ++v) red4w[v * 32 + lane] = acc4[v];
        }
        named_bar_sync(1, kConsumerWarps * 32);
        if (slot_r >= 0 && slot_r < Cfg::RED_SLOTS) {
#pragma unroll
          for (int v = 0; v < Cfg::ACC_F4; ++v) {
            const float4 x = red4r[v * 32 + lane];
            acc4[v].x += x.x; acc4[v].y += x.y; acc4[v].z += x.z; acc4[v].w += x.w;
          }
        }
        named_bar_sync(1, kConsumerWarps * 32);
      }
    }

    if (trace && threadIdx.x == 0) trace[8] = global_timer_ns();
    const bool complete = (kb == 0 && ke == p.kk_total);
    if (!complete && kb != 0 && S > 1) {
      // 2a') cluster contributor (rank r > 0): the leader warp of each chunk
      //      stores its partial into slot r - 1 of the finisher's (rank 0)
      //      partial buffer, the bytes counted on the finisher's fin_bar.
      //      Nothing aims at this CTA afterwards, so it may leave at once.
      if (wk == 0) {
        cluster_wait();
        cluster_waited = true;
        const uint32_t dst = mapa_shared(
            smem_addr(fin) + (((crank - 1) * NC + cc) * Cfg::ACC_F4 * 32 + lane) * 16, 0);
        const uint32_t rbar = mapa_shared(smem_addr(fin_bar), 0);
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) st_async_v4(dst + v * 512, acc4[v], rbar);
      }
      continue;
    }
    if (!complete && kb != 0) {
      // 2a) contributor: this segment ends a tile that another CTA (the one
      //     holding the tile's first K units) finishes.  Publish the partial
      //     in this CTA's scratch slot and count it; nobody waits here.
      //     (Such a segment is always the CTA's first.)
      if (wk == 0) {
        float4* part = p.partials + ((cta * NC + cc) * Cfg::ACC_F4) * 32;
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) part[v * 32 + lane] = acc4[v];
      }
      named_bar_sync(1, kConsumerWarps * 32);
      if (threadIdx.x == 0) {
        fence_acq_rel_gpu();
        red_add_relaxed_gpu(&p.counters[tile], 1);
      }
      continue;
    }
    if (wk != 0) continue;
    if (!complete) {
      // 2b) finisher (always the CTA's last segment): a producer thread has
      //     waited for the other CTAs' partials; add them in CTA order.
      if (aborted || !mbar_wait_bounded(smem_addr(fin_bar), 0, abort_flag) || *abort_flag) {
        if (!aborted && lane == 0) atomicOr(p.status, kStatusFinishWaitTimeout);
        continue;
      }
      if (trace && threadIdx.x == 0) {
        trace[6] += 1;
        trace[9] = global_timer_ns();
      }
      const long long t0 = static_cast<long long>(tile) * units_per_tile;
      const long long c_hi = unit_owner(t0 + units_per_tile - 1, p.units, grid);
      // partials already in shared memory (bulk-copied by the producer)
      const long long c_fin = cta + Cfg::FIN_SLOTS < c_hi ? cta + Cfg::FIN_SLOTS : c_hi;
      for (long long c = cta + 1; c <= c_fin; ++c) {
        const uint32_t src = smem_addr(fin) +
                             ((static_cast<int>(c - cta - 1) * NC + cc) * Cfg::ACC_F4 * 32 + lane) * 16;
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) {
          const uint4 x = lds128(src + v * 512);
          float4& a = acc4[v];
          a.x += __uint_as_float(x.x); a.y += __uint_as_float(x.y);
          a.z += __uint_as_float(x.z); a.w += __uint_as_float(x.w);
        }
      }
      // the rest from global memory: two contributors' loads in flight at a
      // time, 8 float4 per lane each
      constexpr int VB = Cfg::ACC_F4 < 8 ? Cfg::ACC_F4 : 8;
      for (long long c = c_fin + 1; c <= c_hi; c += 2) {
        const bool two = c + 1 <= c_hi;
        const float4* src0 = p.partials + ((c * NC + cc) * Cfg::ACC_F4) * 32 + lane;
        const float4* src1 = two ? src0 + NC * Cfg::ACC_F4 * 32 : src0;
#pragma unroll
        for (int vb = 0; vb < Cfg::ACC_F4; vb += VB) {
          float4 x0[VB], x1[VB];
#pragma unroll
          for (int v = 0; v < VB; ++v) {
            x0[v] = __ldcg(src0 + (vb + v) * 32);
            x1[v] = two ? __ldcg(src1 + (vb + v) * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int v = 0; v < VB; ++v) {
            float4& a = acc4[vb + v];
            a.x += x0[v].x; a.y += x0[v].y; a.z += x0[v].z; a.w += x0[v].w;
            if (two) {
              a.x += x1[v].x; a.y += x1[v].y; a.z += x1[v].z; a.w += x1[v].w;
            }
          }
        }
      }
      // every contribution has arrived and been counted: re-arm the counter
      if (cc == 0 && lane == 0 && S == 1) p.counters[tile] = 0;
    }
    // 3) the leader warp of each chunk converts and stores 16-byte rows of C.
    if (threadIdx.x == 0) ++tiles_stored;
    if (trace && threadIdx.x == 0) trace[10] = global_timer_ns();
    {
      const int n0 = (tile * NC + cc) * 64 + 8 * g;
      float colscale[8];
      if (!GROUPED) {
        const uint4 sv = *reinterpret_cast<const uint4*>(p.s + 2ll * n0);
        const half2* sh = reinterpret_cast<const half2*>(&sv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          colscale[2 * i] = __low2float(sh[i]);
          colscale[2 * i + 1] = __high2float(sh[i]);
        }
      }
#pragma unroll
      for (int mb = 0; mb < MB; ++mb)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int r = 16 * mb + 8 * h + 2 * t + e;
            if (r >= p.M) continue;
            float v[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[j] = acc[mb][j][h][e];
              v[4 + j] = acc[mb][j][h][2 + e];
            }
            if (!GROUPED) {
#pragma unroll
              for (int i = 0; i < 8; ++i) v[i] *= colscale[i];
            }
            if (EPI) {
              float bv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
              if (p.bias != nullptr) {
                const uint4 braw = *reinterpret_cast<const uint4*>(p.bias + n0);
                const half2* bh = reinterpret_cast<const half2*>(&braw);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  bv[2 * i] = __low2float(bh[i]);
                  bv[2 * i + 1] = __high2float(bh[i]);
                }
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) v[i] = epilogue_act(v[i] + bv[i], p.act);
            }
            uint4 o;
            half2* oh = reinterpret_cast<half2*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            if (p.gather_world == 0) {
              *reinterpret_cast<uint4*>(p.C + static_cast<long long>(r) * p.N + n0) = o;
            } else {
              const long long off = static_cast<long long>(r) * p.gather_ldc +
                                    static_cast<long long>(p.gather_rank) * p.N + n0;
              for (int q = 0; q < p.gather_world; ++q)
                *reinterpret_cast<uint4*>(p.gather_c[q] + off) = o;
            }
          }
    }
  }
  if (p.gather_world > 0) {
    // every consumer warp's C stores precede thread 0's system-scope release
    named_bar_sync(1, kConsumerWarps * 32);
    if (threadIdx.x == 0) {
      if (!p.gather_defer && tiles_stored > 0) {
        fence_acq_rel_sys();
        for (int q = 0; q < p.gather_world; ++q)
          red_add_relaxed_sys_u64(p.gather_flag[q], static_cast<unsigned long long>(tiles_stored));
      }
      if (blockIdx.x == 0) {
        // Arrival counters and targets only grow (device memory, so graph
        // replays advance them too).  The target moves by this call's blocks
        // whether or not a wait below expires: late arrivals still count
        // toward this call, so a later wait on the buffer is for later calls'
        // blocks, not for this call's stragglers.  The buffer's previous
        // target was written by an earlier launch, visible since this thread
        // passed the programmatic-launch wait in its epilogue.
        *p.gather_target += static_cast<unsigned long long>(p.gather_world) *
                            (p.gather_defer ? 1ull : static_cast<unsigned long long>(p.tiles_per_rank));
        if (p.gather_wait_arrival != nullptr) {
          const unsigned long long want = *p.gather_wait_target;
          unsigned long long t0 = 0;
          uint32_t polls = 0;
          while (ld_acquire_sys_u64(p.gather_wait_arrival) < want) {
            if ((++polls & 63u) != 0) continue;
            const unsigned long long now = global_timer_ns();
            if (t0 == 0) {
              t0 = now;
            } else if (now - t0 > kWaitLimitNs) {
              atomicOr(p.status, kStatusGatherWaitTimeout);  // the waited-for output is incomplete
              break;
            }
          }
        }
      }
    }
  }
  if (S > 1 && !cluster_waited) cluster_wait();
  if (trace && threadIdx.x == 0) trace[4] = global_timer_ns();
}

}  // namespace sm100
