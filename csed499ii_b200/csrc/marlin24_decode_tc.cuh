// 2:4 sparse W4A16 GEMM for batches of up to 64 rows on the tensor-memory
// tensor cores (sm_100a): tcgen05.mma.sp kind::f16 with the COMPRESSED
// weights as operand A read from tensor memory, activations as operand B
// from shared memory, fp32 accumulators in tensor memory.
//
//   C[M, N] (fp16) = A[M, K] (fp16) . dequant(B, meta, s)[K, N]
//
// Inputs are the Sparse-Marlin packed layout (reference:
// kernel_experiments/sparse_marlin/src/marlin/__init__.py:331-388 and
// _semi_structured_conversions.py:54-179), 4-bit or 3-bit metadata
// (kernel_experiments/sparse_marlin/metadata_decode/codec.cu:18-24).
//
// Work split.  Output features come in 128-feature blocks (one MMA's M).  A
// cluster of S CTAs (S = 1, 2 or 4) owns `bpc` consecutive blocks and splits
// K S ways: CTA r of the cluster streams K steps [r*ks/S, (r+1)*ks/S) of every
// block of the cluster, block after block.  The S partial sums of a block are
// reduced through distributed shared memory: CTA r owns rows
// [r*128/S, (r+1)*128/S) of every block, every other CTA sends it those rows
// of its partial (st.async, counted on the owner's mbarrier; the owner's own
// rows are plain shared-memory stores), and the owner adds the S partials in
// rank order (deterministic) and stores its part of C.  No global scratch, no
// split-K counters: the workspace is never touched.
//
// Warp roles (one CTA per SM).  Every single-thread issue of a TMA copy,
// barrier wait, MMA or commit costs ~100-200 cycles on B200, so stages are
// 256 K deep (8 MMAs of K = 32 per 128-feature block; 128 K for the 48- and
// 64-row tiles, whose activation slices are larger) and the issuing roles are
// doubled (the counts per tile are in DecodeTcCfg):
//   warps 0-1    TMA, stages in turn: the packed codes, metadata and scale
//                rows of the block (before the programmatic-launch wait:
//                weights do not depend on the previous kernel), then the
//                activation slice.
//   MMA_WARPS    MMA issue (one thread each), a block's stages in turn, each
//                into its own accumulator (the epilogue adds them in a
//                fixed order); tensor-memory allocation.
//   4 x DG       dequantise, DG groups of four taking the stages in turn:
//                each thread owns one MMA row (one output feature): INT4
//                codes -> fp16 (magic-number method), group scale applied,
//                the 16 compressed values of each 32-K row written to its
//                tensor-memory lane (tcgen05.st), and its metadata word
//                copied (3-bit metadata decoded first).
//   last 4       epilogue: accumulators -> registers, the DSMEM exchange,
//                sums and the 16-byte stores of C.
// With two accumulator sets (16 and 32 rows) consecutive blocks alternate
// between them, so the epilogue of one block overlaps the MMAs of the next.
//
// Row order.  MMA row m (tensor-memory lane m) of a block holds output feature
// 32q + phi(l) of the block, q = m / 32, l = m % 32,
//   phi(l) = 8 ((l & 7) >> 1) + 2 (l & 1) + (l >> 4) + 4 ((l >> 3) & 1).
// Rows m and m + 8 (m % 16 < 8) are then features f and f + 4, whose 2:4
// metadata share one packed 32-bit word per dense-K half, which is exactly
// what one metadata lane of the sparse MMA holds (lane (m % 8) + 8h + 16(m/16):
// row m in bits 0-15, row m + 8 in bits 16-31, for dense-K half h); the lane
// -> feature map also spreads each warp's code-word loads over 8 banks, and
// each 32-lane quarter covers 32 consecutive features.  Operand A in tensor
// memory: row m at lane m, compressed K pair (2j, 2j+1) in 32-bit column j.
// Both layouts were checked bit-exact against a CPU GEMM by a one-tile probe
// before this kernel was written.
#pragma once

#include "marlin24_prefill_sparse.cuh"

namespace sm100 {

struct DecodeTcParams {
  CUtensorMap tm_act;   // A fp16 (64, M, K/64), box (64, NR, 4), 128-byte swizzle
  CUtensorMap tm_b;     // B u64 (N, K/32), box (128, 8): one block's codes, 8 rows of 32 K
  CUtensorMap tm_meta;  // meta u64 (N/2 or 3N/8, K/32), box (64 or 48, 8)
  CUtensorMap tm_s;     // s u64 (N/4, K/128), box (32, 2)  (grouped only)
  const uint8_t* s;     // fp16 scales (per-column mode: applied in the epilogue)
  half* C;              // fp16 (M, N) row-major
  const half* bias;     // fused epilogue: fp16 per output column, or null
  int act;              // fused epilogue activation (kAct*)
  int* status;          // device status word
  int M;
  int N;
  int ksteps;           // K / (128 * tc_stage_ks(NR)) (stages per block)
  int split;            // S: CTAs of a cluster splitting K (1, 2 or 4)
  int bpc;              // 128-feature blocks per cluster
  int nblocks;          // N / 128
  int pdl;              // launched with programmatic dependent launch
  unsigned long long* trace;  // per-stage clock64 stamps of CTA 0 (SM100_MARLIN_TRACE builds)
};

// Trace builds (-DSM100_MARLIN_TRACE=1): CTA 0 records, per stage s < 64,
// words [16s + i]: 0 producer issue, 1 dequant start (weights landed),
// 2 dequant done (tensor memory written), 3 MMA start (operands ready),
// 4 MMA issued, 5 epilogue got the block's accumulator (first stage of the
// block's slot), 6 epilogue stored C, 8-14 inside the MMA warp's step (loop
// top, tensor stage ready, activations ready, after the fence, after the
// first and the last MMA, after the commits); word 1024 the CTA's clock at
// entry, then setup stamps: 1025 barriers initialised (thread 0), 1026 tensor
// memory allocated, 1027 past the CTA barrier, 1028 TMA warp 0 past the
// programmatic-launch wait, 1029 epilogue past the cluster wait, 1030
// epilogue past the programmatic-launch wait; in the dequantising warps word
// 7 = first half stored to tensor memory, 15 = stores complete.
// Every CTA c also records %globaltimer (ns, comparable across SMs) at words
// kTcCtaBase + 8c + i: 0 entry, 1 first dequantisation start, 2 TMA warp
// past the programmatic-launch wait, 3 first activations landed (MMA warp
// 0), 4 last MMA issued, 5 last block's accumulators read, 6 last C stores
// issued, 7 exit.
constexpr int kTcCtaBase = 1088;
constexpr int kTcTraceStages = 64;
constexpr int kTcTraceWords = 16;

// 128-K sub-steps per stage: 2 (256-K stages), or 1 for the 48- and 64-row
// tiles, whose activation slice (24 or 32 KB per 256 K) would otherwise leave
// room for only two stages.
__host__ __device__ constexpr int tc_stage_ks(int nr) { return nr >= 48 ? 1 : 2; }

template <int NR, bool META3>
struct DecodeTcCfg {
  static_assert(NR == 16 || NR == 32 || NR == 48 || NR == 64, "batch tile");
  static constexpr int KS = tc_stage_ks(NR);           // 128-K sub-steps per stage
  static constexpr int SMEM_BUDGET = 227 * 1024;       // one CTA per SM
  static constexpr int TMEM_COLS = 512;
  static constexpr int ACT = 2 * KS * NR * 128;        // 64-K atoms of NR rows
  static constexpr int CODES = KS * 4 * 1024;          // 32-K rows x 2 chunks x 512 B
  static constexpr int META_ROW = META3 ? 384 : 512;   // per 32-K row, both chunks
  static constexpr int META = KS * 4 * META_ROW;
  static constexpr int SCALES = KS * 256;
  static constexpr int OFF_ACT = 0;                    // 1024-aligned (swizzle atoms)
  static constexpr int OFF_B = ACT;
  static constexpr int OFF_M = OFF_B + CODES;
  static constexpr int OFF_S = OFF_M + META;
  static constexpr int STAGE = (OFF_S + SCALES + 1023) / 1024 * 1024;
  static constexpr int HEADER = 1024;
  // Accumulator (and exchange-buffer) sets.  Two let the epilogue of block j
  // overlap the MMAs of block j + 1; the 48- and 64-row tiles keep one, so
  // that four MMA warps' accumulators still leave four tensor-memory stages,
  // and the freed exchange buffer deepens the shared-memory ring (6 -> 8).
  static constexpr int NACC = NR >= 48 ? 1 : 2;
  static constexpr int RECV = 128 * NR * 4;            // one exchange buffer
  static constexpr int OFF_RECV = HEADER;
  static constexpr int OFF_RING = HEADER + NACC * RECV;
  // MMA-issuing warps: a thread issues one tcgen05.mma per ~90-160 cycles
  // whatever N is, and separate warps issue in parallel, so the 16-row tile
  // (the least work per MMA) gets four, one per SM sub-partition.  So do the
  // 48- and 64-row tiles: their 128-K stages carry four MMAs and two barrier
  // waits and two commits each (~1400 cycles of one thread per stage in a
  // trace with two MMA warps, which set the stage rate); four warps took the
  // 64-row step from 1391 to 1474 GB/s.
  static constexpr int MMA_WARPS = (NR == 16 || NR >= 48) ? 4 : 2;
  // Dequantising groups of four warps (one per tensor-memory lane quarter).
  // The dequantisation is latency-bound (a warp issues ~0.25 instructions
  // per cycle), so the 16-row tile, whose stages carry the least MMA work,
  // runs four groups, and so do the 48- and 64-row tiles, whose 128-K stages
  // and eight tensor-memory stages keep four groups busy.  The 32-row tile
  // keeps two groups and 256-K stages (the 48/64-row configuration measured
  // 1458 vs 1721 GB/s on its step).
  static constexpr int DG = (NR == 16 || NR >= 48) ? 4 : 2;
  // Ring depths are multiples of every role's warp count (two TMA warps, DG
  // dequantising groups, MMA_WARPS MMA warps): each role takes stages in
  // turn, so each warp (group) then owns a fixed subset of the slots and
  // waits on a slot only after it waited on the slot's previous use (a
  // barrier waited on by phase parity must never be two phases behind its
  // waiter).
  static constexpr int DS_FIT = (SMEM_BUDGET - OFF_RING - 1024) / STAGE;
  static constexpr int RING_MULT = MMA_WARPS > DG ? MMA_WARPS : DG;  // both powers of two
  static constexpr int DS = (DS_FIT > 12 ? 12 : DS_FIT) / RING_MULT * RING_MULT;  // shared-memory stages
  static constexpr int SMEM = OFF_RING + DS * STAGE + 1024;
  // tensor memory: per stage 8 MMAs x (8 A + 4 metadata) columns; two
  // accumulators (consecutive blocks) for each MMA-issuing warp
  static constexpr int TSLOT = KS * 48;
  static constexpr int ACC_COLS = MMA_WARPS * NACC * NR;
  static constexpr int DT_FIT = (TMEM_COLS - ACC_COLS) / TSLOT;
  static constexpr int DT_CAP = 4 * 2 / KS;  // at most 1024 K in tensor memory
  static constexpr int DT = (DT_FIT > DT_CAP ? DT_CAP : DT_FIT) / RING_MULT * RING_MULT;  // tensor-memory stages
  // warps: 0-1 TMA, MMA_WARPS MMA, then DG groups of four dequantising warps,
  // then four epilogue warps
  static constexpr int WARP_MMA = 2;
  static constexpr int WARP_DQ = WARP_MMA + MMA_WARPS;
  static constexpr int WARP_EPI = WARP_DQ + 4 * DG;
  static constexpr int THREADS = (WARP_EPI + 4) * 32;
  // Epilogue columns read from tensor memory at a time: the whole row unless
  // the register budget of a larger CTA (above 640 threads) forbids it.
  static constexpr int EPI_CHUNK = (THREADS > 640 && NR > 16) ? 16 : NR;
  static_assert(DS >= RING_MULT && DT >= RING_MULT && DS % RING_MULT == 0 &&
                    DT % RING_MULT == 0 && DS % 2 == 0,
                "ring depths");
  static constexpr int NBAR = 3 * DS + 2 * DT + 8;
  static_assert(NBAR * 8 <= 1000, "barriers exceed the header");
};

// Row m = 32q + l of a block holds feature 32q + phi(l) (see the file comment).
__device__ __forceinline__ int tc_row_feature(int l) {
  return 8 * ((l & 7) >> 1) + 2 * (l & 1) + (l >> 4) + 4 * ((l >> 3) & 1);
}

__device__ __forceinline__ void tmem_st32_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
      "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The sparse MMA with operand A in tensor memory.
__device__ __forceinline__ void umma_sp_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                               uint32_t e_tmem, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.sp.cta_group::1.kind::f16 [%0], [%1], %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, const float4& v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float2 lds_f32x2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// INT4 -> fp16 pair, the magic-number method of dequant_pair in plain C++
// (no volatile asm): the compiler fuses the masks into LOP3s and is free to
// schedule the 16 independent word chains of a stage together.
__device__ __forceinline__ void dequant_pair_sched(uint32_t q, half2& lo, half2& hi) {
  const uint32_t l = (q & 0x000f000fu) | 0x64006400u;
  const uint32_t h = (q & 0x00f000f0u) | 0x64006400u;
  const uint32_t kSub = 0x64086408u;  // (1032, 1032)
  const uint32_t kMul = 0x2c002c00u;  // (1/16, 1/16)
  const uint32_t kAdd = 0xd480d480u;  // (-72, -72)
  lo = __hsub2(*reinterpret_cast<const half2*>(&l), *reinterpret_cast<const half2*>(&kSub));
  hi = __hfma2(*reinterpret_cast<const half2*>(&h), *reinterpret_cast<const half2*>(&kMul),
               *reinterpret_cast<const half2*>(&kAdd));
}

template <int NR, bool META3, bool GROUPED>
__global__ void __launch_bounds__(DecodeTcCfg<NR, META3>::THREADS, 1)
    marlin24_decode_tc_kernel(const __grid_constant__ DecodeTcParams p) {
  using Cfg = DecodeTcCfg<NR, META3>;
  constexpr int DS = Cfg::DS;
  constexpr int DT = Cfg::DT;
  constexpr int KS = Cfg::KS;
  constexpr int NACC = Cfg::NACC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* sfull = reinterpret_cast<uint64_t*>(smem);  // codes/meta/scales landed (1 + tx)
  uint64_t* afull = sfull + DS;                         // activations landed (1 + tx)
  uint64_t* sempty = afull + DS;                        // stage free (4 dequant warps + MMA commit)
  uint64_t* tready = sempty + DS;                       // tensor-memory stage written (4 warps)
  uint64_t* tempty = tready + DT;                       // tensor-memory stage consumed (commit)
  uint64_t* accfull = tempty + DT;                      // accumulators complete (MMA warps' commits)
  uint64_t* accempty = accfull + 2;                     // accumulators read out (4 epilogue warps)
  uint64_t* recvb = accempty + 2;                       // exchange buffer filled (1 + tx)
  uint64_t* freeb = recvb + 2;                          // exchange buffers released (S owners)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::HEADER - 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::HEADER - 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned long long* const trace = (SM100_MARLIN_TRACE && p.trace && blockIdx.x == 0) ? p.trace : nullptr;
  unsigned long long* const cta_trace =
      (SM100_MARLIN_TRACE && p.trace) ? p.trace + kTcCtaBase + 8 * blockIdx.x : nullptr;
  auto gstamp = [&](int i) {
    if (cta_trace) cta_trace[i] = global_timer_ns();
  };
  if (threadIdx.x == 0) gstamp(0);
  if (trace && threadIdx.x == 0) trace[kTcTraceWords * kTcTraceStages] = clock64();
  auto stamp = [&](int s, int i) {
    if (trace && lane == 0 && s < kTcTraceStages) trace[kTcTraceWords * s + i] = clock64();
  };
  const int S = p.split;
  const uint32_t rank = S > 1 ? cluster_cta_rank() : 0u;
  const int b0 = static_cast<int>(blockIdx.x) / S * p.bpc;
  const int nb = min(b0 + p.bpc, p.nblocks) - b0;  // blocks of this cluster (>= 1)
  const int k_lo = static_cast<int>(rank) * p.ksteps / S;
  const int kn = (static_cast<int>(rank) + 1) * p.ksteps / S - k_lo;  // stages per block (>= 1)
  const int T = nb * kn;                                              // stages of this CTA
  // MMA warp w takes the stages s with s % mma_warps == w; mma_warps (1, 2 or
  // 4, a divisor of both ring depths) is at most the stages per block, so
  // every active MMA warp writes every block's accumulator
  const int mma_warps = kn >= Cfg::MMA_WARPS ? Cfg::MMA_WARPS : (kn >= 2 ? 2 : 1);

  if (warp == 0) {
    // the barriers are contiguous from sfull: lane i initialises i, i + 32, ...
    for (int i = lane; i < Cfg::NBAR; i += 32) {
      uint32_t count = 1;  // sfull, afull, tempty, recvb
      if (i >= 2 * DS && i < 3 * DS) count = 5;  // sempty
      else if (i >= 3 * DS && i < 3 * DS + DT) count = 4;  // tready
      else if (i >= 3 * DS + 2 * DT && i < 3 * DS + 2 * DT + 2) count = mma_warps;  // accfull
      else if (i >= 3 * DS + 2 * DT + 2 && i < 3 * DS + 2 * DT + 4) count = 4;  // accempty
      else if (i >= 3 * DS + 2 * DT + 6) count = S;  // freeb
      mbar_init(smem_addr(&sfull[i]), count);
    }
    fence_mbar_init();
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    prefetch_tmap(&p.tm_act);
    prefetch_tmap(&p.tm_b);
    prefetch_tmap(&p.tm_meta);
    if (GROUPED) prefetch_tmap(&p.tm_s);
    if (trace) trace[kTcTraceWords * kTcTraceStages + 1] = clock64();
  }
  if (warp == Cfg::WARP_MMA) {
    tmem_alloc(smem_addr(tmem_slot), Cfg::TMEM_COLS);
    if (trace && lane == 0) trace[kTcTraceWords * kTcTraceStages + 2] = clock64();
  }
  // let the next kernel on the stream start streaming its weights
  if (p.pdl && threadIdx.x == 0) grid_dependency_launch();
  // Start-up.  The TMA warps need only the barriers, which warp 0 has
  // initialised: they pass named barrier 2 together and start streaming.
  // The other warps also need the tensor-memory address: they wait on named
  // barrier 3, where warps 0-1 only arrive.
  uint32_t tmem = 0;
  if (warp < Cfg::WARP_MMA) {
    named_bar_sync(2, 64);
    named_bar_arrive(3, Cfg::THREADS);
  } else {
    tc_fence_before();
    named_bar_sync(3, Cfg::THREADS);
    tc_fence_after();
    tmem = *tmem_slot;
  }
  if (trace && threadIdx.x == 0) trace[kTcTraceWords * kTcTraceStages + 3] = clock64();
  // The weight stream needs only this CTA's barriers; the cluster barrier
  // (peers' barriers exist before any remote arrive or st.async) is waited
  // on by the epilogue warps before their first exchange, and by the others
  // at teardown.
  if (S > 1) cluster_arrive_relaxed();  // after the barrier-init fences
  const uint32_t ring = smem_addr(smem + Cfg::OFF_RING);

  if (warp < Cfg::WARP_MMA) {
    // ------------------------------------------------------------- TMA issue
    // Two warps take the stages in turn (one warp issues a stage's four
    // copies in ~700 cycles); lane 0 issues.  Weight parts of the first
    // stages go out before griddepcontrol.wait, activation parts after it.
    const int pw = warp;
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const uint32_t tx_w = Cfg::CODES + Cfg::META + (GROUPED ? Cfg::SCALES : 0);
    bool waited = p.pdl == 0;
    int n_pend = 0;
    int pend_slot[DS / 2 + 1], pend_ks[DS / 2 + 1];
    auto issue_act = [&](int slot, int ks) {
      const uint32_t af = smem_addr(&afull[slot]);
      mbar_arrive_expect_tx(af, Cfg::ACT);
      tma_load_3d(ring + slot * Cfg::STAGE + Cfg::OFF_ACT, &p.tm_act, 0, 0, 2 * KS * ks, af, pol_keep);
    };
    int b = b0, ks = k_lo;
    if (pw == 1 && T > 1) {  // start at stage 1
      if (++ks == k_lo + kn) {
        ks = k_lo;
        ++b;
      }
    }
    for (int s = pw; s < T && !*abort_flag; s += 2) {
      const int slot = s % DS;
      if (s >= DS) {
        if (!waited) {  // a stage frees only after its MMAs, which need the activations
          grid_dependency_wait();
          waited = true;
          if (trace && threadIdx.x == 0) trace[kTcTraceWords * kTcTraceStages + 4] = clock64();
          if (threadIdx.x == 0) gstamp(2);
          if (lane == 0)
            for (int i = 0; i < n_pend; ++i) issue_act(pend_slot[i], pend_ks[i]);
          n_pend = 0;
        }
        const bool ok = mbar_wait_sleep_bounded(smem_addr(&sempty[slot]), ((s / DS) - 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) atomicOr(p.status, kStatusEmptyWaitTimeout);
          break;
        }
      }
      stamp(s, 0);
      if (lane == 0) {
        const uint32_t st = ring + slot * Cfg::STAGE;
        const uint32_t sf = smem_addr(&sfull[slot]);
        mbar_arrive_expect_tx(sf, tx_w);
        tma_load_2d(st + Cfg::OFF_B, &p.tm_b, b * 128, ks * 4 * KS, sf, pol_stream);
        tma_load_2d(st + Cfg::OFF_M, &p.tm_meta, b * (META3 ? 48 : 64), ks * 4 * KS, sf, pol_stream);
        if (GROUPED) tma_load_2d(st + Cfg::OFF_S, &p.tm_s, b * 32, ks * KS, sf, pol_keep);
        if (waited) {
          issue_act(slot, ks);
        } else {
          pend_slot[n_pend] = slot;
          pend_ks[n_pend] = ks;
        }
      }
      if (!waited) ++n_pend;
      __syncwarp();
      // advance two stages
      for (int a = 0; a < 2; ++a)
        if (++ks == k_lo + kn) {
          ks = k_lo;
          ++b;
        }
    }
    if (!waited) {
      grid_dependency_wait();
      if (trace && threadIdx.x == 0) trace[kTcTraceWords * kTcTraceStages + 4] = clock64();
      if (threadIdx.x == 0) gstamp(2);
      if (lane == 0)
        for (int i = 0; i < n_pend; ++i) issue_act(pend_slot[i], pend_ks[i]);
    }
  } else if (warp < Cfg::WARP_DQ) {
    // ------------------------------------------------------------- MMA issue
    // MMA_WARPS warps, one thread each, take the stages in turn, each
    // accumulating into its own accumulator: the warps' MMA issue, barrier
    // waits and commits (100-200 cycles each) overlap.  The epilogue adds the
    // accumulators in warp order.
    const int w = warp - Cfg::WARP_MMA;
    constexpr uint32_t idesc = umma_idesc_f16_f32(NR) | (1u << 2);  // sparse
    constexpr uint64_t kAtom = (NR * 128) >> 4;                     // next 64-K atom
    if (w < mma_warps) {
      int j = 0, i_in = 0, slot = 0, t = 0;
      uint32_t sph = 0, tph = 0;  // phase parities of slot / t
      bool first = true;          // this warp's first stage of block j
      for (int s = 0; s < T; ++s) {
        if ((s & (mma_warps - 1)) == w) {
          bool ok = true;
          stamp(s, 8);
          if (first && j >= NACC)  // the epilogue has read this accumulator out
            ok = mbar_wait_spin_sleep_bounded(smem_addr(&accempty[j % NACC]), ((j / NACC) - 1) & 1, abort_flag);
          ok = ok && mbar_wait_spin_sleep_bounded(smem_addr(&tready[t]), tph, abort_flag);
          stamp(s, 9);
          ok = ok && mbar_wait_spin_sleep_bounded(smem_addr(&afull[slot]), sph, abort_flag);
          stamp(s, 10);
          if (s == 0 && lane == 0) gstamp(3);
          if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
            break;
          }
          tc_fence_after();
          stamp(s, 3);
          if (lane == 0) {
            const uint32_t acc = tmem + (w * NACC + j % NACC) * NR;
            const uint32_t ta = tmem + Cfg::ACC_COLS + t * Cfg::TSLOT;
            const uint64_t bd = umma_desc_sw128_k(ring + slot * Cfg::STAGE + Cfg::OFF_ACT);
#pragma unroll
            for (int i = 0; i < 4 * KS; ++i)
              umma_sp_f16_ts(acc, ta + 8 * i, bd + (i >> 1) * kAtom + (i & 1) * 4,
                             ta + 32 * KS + 4 * i, idesc, (first && i == 0) ? 0u : 1u);
            stamp(s, 13);
            if (s + mma_warps >= T) gstamp(4);
            umma_commit(smem_addr(&tempty[t]));
            umma_commit(smem_addr(&sempty[slot]));
            // this warp's last stage of the block
            if (i_in + mma_warps >= kn) umma_commit(smem_addr(&accfull[j % NACC]));
          }
          stamp(s, 4);
          __syncwarp();
          first = false;
        }
        if (++slot == DS) {
          slot = 0;
          sph ^= 1u;
        }
        if (++t == DT) {
          t = 0;
          tph ^= 1u;
        }
        if (++i_in == kn) {
          i_in = 0;
          ++j;
          first = true;
        }
      }
    }
  } else if (warp < Cfg::WARP_EPI) {
    // -------------------------------------------------------------- dequantise
    const int q = warp & 3;                       // tensor-memory lanes 32q .. 32q+31
    const int grp = (warp - Cfg::WARP_DQ) >> 2;   // stages s % DG == grp
    const int l = lane;
    const int c = q >> 1;                           // 64-feature chunk of the block
    const int g = 4 * (q & 1) + ((l & 7) >> 1);     // 8-feature group in the chunk
    const int jp = 2 * (l & 1) + (l >> 4);          // feature in the group (and +4)
    const int e = (l >> 3) & 1;                     // 0: feature 8g + jp, 1: + 4
    // code words 16g + 4t + jp of chunk c (t = 0..3), nibbles of this feature
    const uint32_t code_off = Cfg::OFF_B + c * 512 + 4 * (16 * g + jp);
    const uint32_t scale_off = Cfg::OFF_S + 2 * (64 * c + 8 * g + 2 * jp + e);
    // metadata word of this lane: pair (f, f + 4), dense-K half e
    const int w4 = 32 * (l & 1) + 4 * g + 2 * (l >> 4) + e;
    const uint32_t meta_off = META3 ? (Cfg::OFF_M + c * 192 + 4 * (w4 & 31))
                                    : (Cfg::OFF_M + c * 256 + 4 * w4);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * q) << 16) + Cfg::ACC_COLS;
    for (int s = grp; s < T; s += Cfg::DG) {
      const int slot = s % DS;
      const int t = s % DT;
      bool ok = mbar_wait_sleep_bounded(smem_addr(&sfull[slot]), (s / DS) & 1, abort_flag);
      if (s >= DT)
        ok = ok && mbar_wait_sleep_bounded(smem_addr(&tempty[t]), ((s / DT) - 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
        break;
      }
      tc_fence_after();
      if (q == 0) stamp(s, 1);
      if (s == 0 && q == 0 && lane == 0) gstamp(1);
      const uint8_t* stp = smem + Cfg::OFF_RING + slot * Cfg::STAGE;
      const uint32_t tslot = lane_base + t * Cfg::TSLOT;
      // four sub-steps of 64 K (two 32-K rows each; a small register
      // footprint leaves room for four dequantising groups)
#pragma unroll
      for (int u = 0; u < 2 * KS; ++u) {
        const int h = u >> 1;        // 128-K half of the stage
        const int kb = 2 * (u & 1);  // first 32-K row of the sub-step in the half
        // plain loads (ordered after the barrier wait by its memory clobber),
        // all issued before any use so that their latencies overlap
        uint32_t words[8];
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2)
#pragma unroll
          for (int tt = 0; tt < 4; ++tt)
            words[k2 * 4 + tt] = *reinterpret_cast<const uint32_t*>(
                stp + code_off + (4 * h + kb + k2) * 1024 + 16 * tt);
        uint32_t mraw[META3 ? 4 : 2];
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          const uint8_t* mp = stp + meta_off + (4 * h + kb + k2) * Cfg::META_ROW;
          mraw[k2] = *reinterpret_cast<const uint32_t*>(mp);
          if constexpr (META3) mraw[2 + k2] = *reinterpret_cast<const uint32_t*>(mp + 64);
        }
        half2 s2 = __float2half2_rn(1.f);
        if (GROUPED) {
          const half sh = *reinterpret_cast<const half*>(stp + scale_off + 256 * h);
          s2 = __halves2half2(sh, sh);
        }
        uint32_t v[16];
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
#pragma unroll
          for (int tt = 0; tt < 4; ++tt) {
            const uint32_t wd = words[k2 * 4 + tt];
            half2 lo, hi;
            dequant_pair_sched(e ? (wd >> 8) : wd, lo, hi);  // (kc 2tt, 2tt+1), (kc 8+2tt, 9+2tt)
            if (GROUPED) {
              lo = __hmul2(lo, s2);
              hi = __hmul2(hi, s2);
            }
            v[k2 * 8 + tt] = *reinterpret_cast<uint32_t*>(&lo);
            v[k2 * 8 + 4 + tt] = *reinterpret_cast<uint32_t*>(&hi);
          }
        }
        uint32_t mw[2];
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          if constexpr (META3) {
            // 4-bit word w4 of the chunk is the high (w4 < 32) or low decode of
            // 3-bit words w4 % 32 and w4 % 32 + 16 (meta3_pair_decode)
            const uint32_t a = mraw[k2], bb = mraw[2 + k2];
            const bool upper = (w4 & 31) >= 16;
            if (w4 >= 32)
              mw[k2] = decode24_low(upper ? (bb >> 8) : __funnelshift_r(a, bb, 24));
            else
              mw[k2] = decode24_high(upper ? __funnelshift_r(a, bb, 16) : a);
          } else {
            mw[k2] = mraw[k2];
          }
        }
        tmem_st32_x16(tslot + 32 * h + 8 * kb, v);
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2)
          tmem_st32(tslot + 32 * KS + 16 * h + 4 * (kb + k2), mw[k2]);
        if (q == 0 && u == 1) stamp(s, 7);
      }
      tmem_wait_st();
      if (q == 0) stamp(s, 15);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_addr(&tready[t]));
        mbar_arrive(smem_addr(&sempty[slot]));
      }
      if (q == 0) stamp(s, 2);
    }
  } else {
    // ----------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int row = 32 * q + lane;                   // accumulator lane
    const int feat = 32 * q + tc_row_feature(lane);  // feature of that row in the block
    const int slice = 128 / S;                       // rows (features) each CTA owns
    const uint32_t owner = static_cast<uint32_t>(row / slice);
    const int et = threadIdx.x - Cfg::WARP_EPI * 32;  // 0 .. 127
    const uint32_t recv = smem_addr(smem + Cfg::OFF_RECV);
    const uint32_t lane_acc = tmem + (static_cast<uint32_t>(32 * q) << 16);
    // C may still be read by the previous kernel on the stream
    if (p.pdl) grid_dependency_wait();
    if (trace && et == 0) trace[kTcTraceWords * kTcTraceStages + 6] = clock64();
    if (S > 1) cluster_wait();
    if (trace && et == 0) trace[kTcTraceWords * kTcTraceStages + 5] = clock64();
    for (int j = 0; j < nb; ++j) {
      const int buf = j % NACC;
      const uint32_t par = static_cast<uint32_t>(j / NACC) & 1u;
      bool ok = mbar_wait_spin_sleep_bounded(smem_addr(&accfull[buf]), par, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
        break;
      }
      tc_fence_after();
      if (q == 0) stamp(j * kn, 5);
      if (j == nb - 1 && et == 0) gstamp(5);
      // this row of the partial -> its owner's buffer, at [rank][feature in slice]
      const uint32_t dst = recv + buf * Cfg::RECV +
                           ((rank * slice + (feat - static_cast<int>(owner) * slice)) * NR) * 4;
      const uint32_t rdst = S > 1 ? mapa_shared(dst, owner) : dst;
      const uint32_t rbar = S > 1 ? mapa_shared(smem_addr(&recvb[buf]), owner) : 0u;
      // The sum of the MMA warps' accumulators (warp 0 first), ECH columns at
      // a time: the accumulators are released after the last chunk is read,
      // and exchange buffer `buf` must be free (all owners done with block
      // j - NACC) before the first chunk is sent.
      constexpr int ECH = Cfg::EPI_CHUNK;
      bool failed = false;
#pragma unroll
      for (int e0 = 0; e0 < NR; e0 += ECH) {
        uint32_t r[ECH];
        float acc[ECH];
#pragma unroll
        for (int c0 = 0; c0 < ECH; c0 += 16) tmem_ld16(lane_acc + buf * NR + e0 + c0, r + c0);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < ECH; ++u) acc[u] = __uint_as_float(r[u]);
        for (int w = 1; w < mma_warps; ++w) {
#pragma unroll
          for (int c0 = 0; c0 < ECH; c0 += 16)
            tmem_ld16(lane_acc + (NACC * w + buf) * NR + e0 + c0, r + c0);
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < ECH; ++u) acc[u] += __uint_as_float(r[u]);
        }
        if (e0 + ECH == NR) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(&accempty[buf]));
        }
        if (e0 == 0 && S > 1 && j >= NACC) {
          ok = mbar_wait_sleep_bounded(smem_addr(&freeb[buf]), (par - 1u) & 1u, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(p.status, kStatusFinishWaitTimeout);
            failed = true;
            break;
          }
        }
        if (owner != rank) {  // warp-uniform: a warp's 32 rows have one owner
#pragma unroll
          for (int c0 = 0; c0 < ECH; c0 += 4)
            st_async_v4(rdst + 4 * (e0 + c0), make_float4(acc[c0], acc[c0 + 1], acc[c0 + 2], acc[c0 + 3]),
                        rbar);
        } else {
#pragma unroll
          for (int c0 = 0; c0 < ECH; c0 += 4)
            sts128(dst + 4 * (e0 + c0), make_float4(acc[c0], acc[c0 + 1], acc[c0 + 2], acc[c0 + 3]));
        }
      }
      if (failed) break;
      if (S > 1) {
        if (q == 0) stamp(j * kn, 11);
        // the peers' slices; this CTA's own slice was stored locally (ordered
        // by the named barrier below)
        if (et == 0) mbar_arrive_expect_tx(smem_addr(&recvb[buf]), Cfg::RECV - Cfg::RECV / S);
        ok = mbar_wait_spin_sleep_bounded(smem_addr(&recvb[buf]), par, abort_flag);
        if (q == 0) stamp(j * kn, 12);
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) atomicOr(p.status, kStatusFinishWaitTimeout);
          break;
        }
      }
      named_bar_sync(1, 128);
      // sums of this CTA's slice: 8 features x 2 batch rows per item, the S
      // partials added in rank order; 16-byte stores of C.  Lanes take
      // consecutive row pairs of one feature group, so each warp-wide 8-byte
      // load reads one contiguous run of the buffer (no bank conflicts).
      const int n0 = (b0 + j) * 128 + static_cast<int>(rank) * slice;
      const int groups = slice / 8;
      const int pairs = (p.M + 1) >> 1;
      for (int it = et; it < groups * pairs; it += 128) {
        const int fg = it / pairs;
        const int rp = it - fg * pairs;
        float sum[2][8];
#pragma unroll
        for (int u = 0; u < 8; ++u) sum[0][u] = sum[1][u] = 0.f;
        for (int src = 0; src < S; ++src) {
          const uint32_t base = recv + buf * Cfg::RECV + ((src * slice + fg * 8) * NR + 2 * rp) * 4;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float2 v = lds_f32x2(base + u * NR * 4);
            sum[0][u] += v.x;
            sum[1][u] += v.y;
          }
        }
        const int n = n0 + fg * 8;
        float sc[8], bv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          sc[u] = 1.f;
          bv[u] = 0.f;
        }
        if (!GROUPED) {
          const uint4 sv = *reinterpret_cast<const uint4*>(p.s + 2ll * n);
          const half2* sh = reinterpret_cast<const half2*>(&sv);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            sc[2 * u] = __low2float(sh[u]);
            sc[2 * u + 1] = __high2float(sh[u]);
          }
        }
        const bool fused = p.bias != nullptr || p.act != kActNone;
        if (p.bias != nullptr) {
          const uint4 braw = *reinterpret_cast<const uint4*>(p.bias + n);
          const half2* bh = reinterpret_cast<const half2*>(&braw);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            bv[2 * u] = __low2float(bh[u]);
            bv[2 * u + 1] = __high2float(bh[u]);
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int rr = 2 * rp + h;
          if (rr >= p.M) break;
          float o8[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            o8[u] = GROUPED ? sum[h][u] : sum[h][u] * sc[u];
            if (fused) o8[u] = epilogue_act(o8[u] + bv[u], p.act);
          }
          uint4 o;
          half2* oh = reinterpret_cast<half2*>(&o);
#pragma unroll
          for (int u = 0; u < 4; ++u) oh[u] = __floats2half2_rn(o8[2 * u], o8[2 * u + 1]);
          *reinterpret_cast<uint4*>(p.C + static_cast<long long>(rr) * p.N + n) = o;
        }
      }
      named_bar_sync(1, 128);
      if (q == 0) stamp(j * kn, 6);
      if (j == nb - 1 && et == 0) gstamp(6);
      // release buffer `buf` to every CTA of the cluster (needed only when a
      // block j + NACC follows)
      if (S > 1 && j + NACC < nb && et < S)
        mbar_arrive_remote(mapa_shared(smem_addr(&freeb[buf]), static_cast<uint32_t>(et)));
    }
  }

  // Teardown: all MMAs complete before the tensor memory is released.  No
  // cluster barrier: every remote write aimed at a CTA (its peers' st.async
  // partials, counted on its recvb, and their freeb arrivals, which it waits
  // for before its exchange of block j + NACC) precedes a wait that the CTA has
  // passed by the end of its last exchange, so a CTA may leave as soon as it
  // is done.  Each thread completes its start-up cluster arrival.
  if (S > 1 && warp < Cfg::WARP_EPI) cluster_wait();
  tc_fence_before();
  __syncthreads();
  if (warp == Cfg::WARP_MMA) {
    if (*abort_flag == 0)  // the last block's accumulators are complete
      mbar_wait_sleep_bounded(smem_addr(&accfull[(nb - 1) % NACC]), ((nb - 1) / NACC) & 1, abort_flag);
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0) gstamp(7);
}

}  // namespace sm100
