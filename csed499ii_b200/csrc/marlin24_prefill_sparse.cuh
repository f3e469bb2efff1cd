// 2:4 sparse W4A16 GEMM for batches above 64 rows on the structured-sparse
// tensor-core instruction: tcgen05.mma.sp kind::f16, fp32 accumulator and the
// 2:4 metadata in tensor memory.  Same inputs and host contract as
// marlin24_prefill_kernel (the dense-expansion form, kept for K not a
// multiple of 128).
//
// Two forms.  The CTA-pair form further below (tcgen05.mma.sp.cta_group::2,
// 128-K steps) runs every prefill whose N is a multiple of 256.  The
// one-CTA form here (128-feature x BN-row tile, 64-K steps: a 64-byte-
// swizzled tile of compressed weights, one 128-byte swizzle atom of
// activations, two MMAs of K = 32, 4-8 stages) runs when pairs are off.
//
//  * warp 0 (lane 0 issues): TMA of the activation atom (counted on the
//    ready barrier) and of the packed codes (2 x 32-K rows), metadata and
//    scale row of the 128 features (counted on the weight barrier);
//  * warps 2.. (NG groups of four, K steps in turn): dequantise the INT4
//    codes and apply the group scale (fp16, as the reference), storing the
//    COMPRESSED values (two per group of four; no zero fill) into the UMMA
//    K-major 64-byte-swizzled tile, and copy the metadata words of the step
//    into tensor memory (tcgen05.st; one 4-column-aligned slot per MMA);
//  * warp 1 (lane 0 issues): one wait per K step on the ready barrier, then
//    tcgen05.mma.sp.cta_group::1.kind::f16 with the compressed weights as
//    operand A, the activations as operand B and the metadata slot of each
//    MMA; tcgen05.commit frees the stage.
//
// Metadata layout in tensor memory (M = 128, K = 32 per MMA): lane
// L = (m mod 8) + 8h + 16(m div 16) holds, in bits 0-15, the four nibbles of
// row m for dense K half h and, in bits 16-31, those of row m + 8 (derived from
// CUTLASS 4.x `tmem_e_frg`, checked bit-exact by a one-tile probe).  The
// packed int32 metadata words pair out-features n and n + 4 per K half, so
// with the weight-tile row of feature 64c + 8a + 2cc' + d (+4) chosen as
// a + 16(4c + 2cc' + d) (+8), every tensor-memory lane receives exactly one
// packed metadata word: the copy is a permutation of 32-bit words.
#pragma once

#include "marlin24_prefill.cuh"

namespace sm100 {

// Warp roles: one TMA producer warp, one MMA warp, then the dequantising
// warps.  (One producer warp per tensor was measured 5 % slower.)
constexpr int kSpProducerWarps = 1;
constexpr int kSpMmaWarp = 1;
constexpr int kSpDequantWarp0 = 2;

template <int BN, int NG>
struct PrefillSpCfg {
  static_assert(BN == 128 || BN == 256, "batch tile");
  static constexpr int ACT = BN * 128;                 // one 64-K activation atom
  static constexpr int ATILE = 128 * 64;               // compressed weights: 128 rows x 32 halves
  static constexpr int OFF_ACT = 0;
  static constexpr int OFF_A = ACT;
  static constexpr int OFF_B = OFF_A + ATILE;          // 2 rows x 1024 B of packed codes
  static constexpr int OFF_M = OFF_B + 2048;           // 2 rows x 512 B of metadata
  static constexpr int OFF_S = OFF_M + 1024;           // one scale row (128 features)
  static constexpr int STAGE = (OFF_S + 256 + 1023) / 1024 * 1024;
  static constexpr int HEADER = 1024;
  static constexpr int DEPTH_FIT = (kPrefillSmemBudget - HEADER - 1024) / STAGE;
  static constexpr int DEPTH_CAP = DEPTH_FIT > 8 ? 8 : DEPTH_FIT;
  static constexpr int DEPTH = DEPTH_CAP / NG * NG;
  static constexpr int SMEM = HEADER + DEPTH * STAGE + 1024;
  static constexpr int THREADS = (kSpProducerWarps + 1 + 4 * NG) * 32;
  static constexpr int META_COLS = 8;  // per stage: 2 MMAs x 4-column-aligned metadata slots
  static constexpr int TMEM_NEED = BN + DEPTH * META_COLS;
  static constexpr int TMEM_COLS = TMEM_NEED <= 128 ? 128 : (TMEM_NEED <= 256 ? 256 : 512);
  static_assert(DEPTH >= 2 && DEPTH % NG == 0, "sparse prefill ring too shallow");
  static_assert(TMEM_NEED <= 512, "tensor memory");
};

// Shared-memory descriptor of a K-major operand in the 64-byte swizzled
// canonical layout (rows of 64 bytes, 8-row groups 512 bytes apart, swizzle
// mode 4).
__device__ __forceinline__ uint64_t umma_desc_sw64_k(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;
  return d;
}

__device__ __forceinline__ void umma_sp_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t e_tmem, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.sp.cta_group::1.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

template <int BN, int NG, bool GROUPED>
__global__ void __launch_bounds__(PrefillSpCfg<BN, NG>::THREADS, 1)
    marlin24_prefill_sp_kernel(const __grid_constant__ PrefillParams p) {
  using Cfg = PrefillSpCfg<BN, NG>;
  constexpr int D = Cfg::DEPTH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* aready_bar = full_bar + D;
  uint64_t* empty_bar = aready_bar + D;
  uint64_t* acc_bar = empty_bar + D;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 256);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 260);
  uint8_t* ring = smem + Cfg::HEADER;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x;
  const int m_tile = blockIdx.y;
  const int ksteps = p.K / 64;

  if (threadIdx.x < D) {
    mbar_init(smem_addr(&full_bar[threadIdx.x]), 1);    // packed codes, metadata, scales
    mbar_init(smem_addr(&aready_bar[threadIdx.x]), 5);  // activations (tx) + 4 dequant warps
    mbar_init(smem_addr(&empty_bar[threadIdx.x]), 1);
  }
  if (threadIdx.x == 32) {
    mbar_init(smem_addr(acc_bar), 1);
    *abort_flag = 0;
  }
  if (threadIdx.x < D || threadIdx.x == 32) fence_mbar_init();
  if (warp == kSpMmaWarp) tmem_alloc(smem_addr(tmem_slot), Cfg::TMEM_COLS);
  if (threadIdx.x == 0) {
    prefetch_tmap(&p.tm_act);
    prefetch_tmap(&p.tm_b);
    prefetch_tmap(&p.tm_meta);
    if (GROUPED) prefetch_tmap(&p.tm_s);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_e = tmem + BN;  // metadata slots after the accumulator columns
  const uint32_t ring_base = smem_addr(ring);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp runs the loop (lane 0 issues): a lone lane looping while
    // the rest of its warp waits at the CTA barrier below runs slowly.
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const uint32_t txw = 2048 + 1024 + (GROUPED ? 256 : 0);
    for (int ks = 0; ks < ksteps; ++ks) {
      const int slot = ks % D;
      const uint32_t parity = ((ks / D) & 1) ^ 1;
      const bool ok = mbar_wait_bounded(smem_addr(&empty_bar[slot]), parity, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicOr(p.status, kStatusEmptyWaitTimeout);
        break;
      }
      if (lane == 0) {
        const uint32_t full = smem_addr(&full_bar[slot]);
        const uint32_t ready = smem_addr(&aready_bar[slot]);
        const uint32_t st = ring_base + slot * Cfg::STAGE;
        mbar_arrive_expect_tx(full, txw);
        mbar_arrive_expect_tx(ready, Cfg::ACT);
        tma_load_2d(st + Cfg::OFF_ACT, &p.tm_act, ks * 64, m_tile * BN, ready, pol_keep);
        tma_load_2d(st + Cfg::OFF_B, &p.tm_b, n_tile * 128, ks * 2, full, pol_stream);
        tma_load_2d(st + Cfg::OFF_M, &p.tm_meta, n_tile * 64, ks * 2, full, pol_stream);
        if (GROUPED) tma_load_2d(st + Cfg::OFF_S, &p.tm_s, n_tile * 32, ks >> 1, full, pol_keep);
      }
      __syncwarp();
    }
  } else if (warp == kSpMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // The issuing warp shares its sub-partition with busy dequantising warps
    // and gets few issue slots, so its per-step instruction count is the
    // kernel's critical path (per-step clock64 traces: ~750 cycles per step
    // spent in this loop with every stage already complete).  Descriptors,
    // barrier addresses and metadata slots therefore advance by one stage per
    // K step and wrap with the ring instead of being recomputed.
    {
      constexpr uint32_t idesc = umma_idesc_f16_f32(BN) | (1u << 2);  // sparse
      constexpr uint64_t kStageDesc = Cfg::STAGE >> 4;  // start-address field step
      const uint64_t ad0 = umma_desc_sw64_k(ring_base + Cfg::OFF_A);
      const uint64_t bd0 = umma_desc_sw128_k(ring_base + Cfg::OFF_ACT);
      const uint32_t ready0 = smem_addr(aready_bar);
      const uint32_t empty0 = smem_addr(empty_bar);
      uint64_t ad = ad0, bd = bd0;
      uint32_t e = tmem_e, slot = 0, parity = 0;
      for (int ks = 0; ks < ksteps; ++ks) {
        // one wait per step: activations landed and the tile dequantised
        const bool ok = mbar_wait_bounded(ready0 + 8 * slot, parity, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          // two MMAs of K = 32: the second half of the 64-byte weight rows
          // (+32 B) and of the 128-byte activation rows (+64 B)
          umma_sp_f16(tmem, ad, bd, e, idesc, ks ? 1u : 0u);
          umma_sp_f16(tmem, ad + 2, bd + 4, e + 4, idesc, 1u);
          umma_commit(empty0 + 8 * slot);
        }
        __syncwarp();
        if (++slot == D) {
          slot = 0;
          parity ^= 1;
          ad = ad0;
          bd = bd0;
          e = tmem_e;
        } else {
          ad += kStageDesc;
          bd += kStageDesc;
          e += Cfg::META_COLS;
        }
      }
      if (lane == 0) umma_commit(smem_addr(acc_bar));
    }
  } else {
    // ---------------------------------------------- dequantise, then epilogue
    // 0 .. 4*NG-1; the mask (a no-op here) tells the compiler the K-step
    // index below is never negative (without it: 80 registers and spills)
    const int dw = static_cast<int>(static_cast<uint32_t>(warp - kSpDequantWarp0) & (4u * NG - 1u));
    const int grp = dw >> 2;        // K steps ks % NG == grp
    const int r = dw & 1;           // 32-K row of the step whose codes this warp converts
    const int cc = (dw >> 1) & 1;   // and its 64-feature chunk
    const int quarter = warp & 3;   // tensor-memory lanes this warp may access
    const int g = lane >> 2, t = lane & 3;
    // metadata word of TMEM lane 32*quarter + lane: chunk quarter/2, word
    // 32*(quarter&1) + 4a + 2d + h with a = lane%8, h = (lane/8)%2, d = lane/16
    const uint32_t m_word = (quarter >> 1) * 256 +
                            4 * (32 * (quarter & 1) + 4 * (lane & 7) + 2 * (lane >> 4) + ((lane >> 3) & 1));
    const uint32_t e_lane = tmem_e + (static_cast<uint32_t>(32 * quarter) << 16);
    bool ok = true;
    for (int ks = grp; ks < ksteps; ks += NG) {
      const int slot = ks % D;
      const uint32_t parity = (ks / D) & 1;
      if (!mbar_wait_bounded(smem_addr(&full_bar[slot]), parity, abort_flag)) {
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
        ok = false;
        break;
      }
      const uint32_t st = ring_base + slot * Cfg::STAGE;
      // metadata of the two MMAs into this warp's lanes of the stage's slots
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
        tmem_st32(e_lane + slot * Cfg::META_COLS + 4 * kk, lds32(st + Cfg::OFF_M + kk * 512 + m_word));
      // compressed weights of 32-K row r, chunk cc
      {
        const uint4 q = lds128(st + Cfg::OFF_B + r * 1024 + cc * 512 + lane * 16);
        uint4 sv = make_uint4(0, 0, 0, 0);
        if (GROUPED) sv = lds128(st + Cfg::OFF_S + cc * 128 + g * 16);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          half2 lo0, hi0, lo1, hi1;
          dequant_pair(qw[j], lo0, hi0);       // feature 8g+j: kc 2t.., 8+2t..
          dequant_pair(qw[j] >> 8, lo1, hi1);  // feature 8g+j+4
          if (GROUPED) {
            const half2 s2 = *reinterpret_cast<const half2*>(&sw[j]);
            const half2 sx = __low2half2(s2), sy = __high2half2(s2);
            lo0 = __hmul2(lo0, sx);
            hi0 = __hmul2(hi0, sx);
            lo1 = __hmul2(lo1, sy);
            hi1 = __hmul2(hi1, sy);
          }
          // rows: feature 64cc + 8g + j -> g + 16(4cc + j), feature + 4 -> + 8
          const int m_lo = g + 16 * (4 * cc + j);
          const uint32_t row_lo = st + Cfg::OFF_A + m_lo * 64;
          const uint32_t row_hi = row_lo + 8 * 64;
          // compressed columns 16r + 2t (16-byte chunk 2r) and 16r + 8 + 2t
          // (chunk 2r+1) of a 64-byte row, swizzled with (row / 2) mod 4;
          // rows m and m + 8 share the pattern
          const uint32_t sx = (g >> 1) & 3;
          const uint32_t ca = ((2 * r) ^ sx) << 4, cb = ((2 * r + 1) ^ sx) << 4;
          const uint32_t wo = 4 * t;
          sts32(row_lo + ca + wo, *reinterpret_cast<uint32_t*>(&lo0));
          sts32(row_lo + cb + wo, *reinterpret_cast<uint32_t*>(&hi0));
          sts32(row_hi + ca + wo, *reinterpret_cast<uint32_t*>(&lo1));
          sts32(row_hi + cb + wo, *reinterpret_cast<uint32_t*>(&hi1));
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&aready_bar[slot]));
    }

    // ------------------------------------------------------------ epilogue
    if (ok && mbar_wait_bounded(smem_addr(acc_bar), 0, abort_flag)) {
      tc_fence_after();
      const int rr = 32 * quarter + lane;  // accumulator row
      const int m2 = rr >> 4;
      const int feat = 64 * (m2 >> 2) + 8 * (rr & 7) + (m2 & 3) + 4 * ((rr >> 3) & 1);
      const int n = n_tile * 128 + feat;
      float cs = 1.f;
      if (!GROUPED) cs = __half2float(reinterpret_cast<const half*>(p.s)[n]);
      const float col_bias = p.bias != nullptr ? __half2float(p.bias[n]) : 0.f;
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
#pragma unroll 1
      for (int cb2 = grp; cb2 < BN / 32; cb2 += NG) {
        uint32_t v[32];
        tmem_ld32(lane_addr + cb2 * 32, v);
        const int b0 = m_tile * BN + cb2 * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int b = b0 + j;
          if (b < p.M)
            p.C[static_cast<long long>(b) * p.N + n] =
                __float2half_rn(epilogue_act(__uint_as_float(v[j]) * cs + col_bias, p.act));
        }
      }
    } else if (ok && lane == 0) {
      atomicOr(p.status, kStatusFullWaitTimeout);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kSpMmaWarp) {
    mbar_wait_bounded(smem_addr(acc_bar), 0, abort_flag);
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ===========================================================================
// CTA-pair form: tcgen05.mma.sp.cta_group::2 (M = 256 features, N = 256 batch
// rows per MMA, issued by the even CTA of a 2-CTA cluster), K in steps of 128.
//
// Each CTA of the pair dequantises its own 128 features and holds half of the
// pair's 256-row activation tile; the MMA reads operand A (weights) and B
// (activations) from both CTAs' shared memory at the same offsets and
// accumulates each CTA's 128 features x 256 rows in that CTA's tensor memory;
// each CTA's metadata slots hold its own 128 rows in the one-CTA layout
// (CUTLASS 4.x SM100_MMA_F16BF16_2x1SM_SS_SPARSE: A, B and C split over the
// pair along M, N and M; checked bit-exact by a one-tile probe).
//
// Why: per-step clock64 traces of the one-CTA kernel show a fixed ~700-cycle
// cost per K step in its issuing threads (barrier polls, TMA and MMA issue),
// independent of the stage's bytes and of the MMA work.  Halving the
// activation bytes per SM lets a 128-K step (four MMAs, a 128-byte-swizzled
// compressed weight tile) fit 4 stages deep, so that cost is paid once per
// 128 K instead of once per 64 K.
//
// Barriers per ring slot:
//   wfull  (each CTA)  packed codes, metadata, scales landed     (count 1 + tx)
//   aready (even CTA)  both CTAs' activation halves landed and both CTAs'
//                      tiles dequantised (count 9 + tx): the MMA thread's
//                      only wait per step (each wait costs it ~250 cycles)
//   empty  (each CTA)  MMAs of the slot done (commit, multicast to the pair)
// ===========================================================================

template <int NG>
struct PrefillSp2Cfg {
  static constexpr int ROWS = 128;                     // activation rows held per CTA
  static constexpr int ATOM = ROWS * 128;              // one 64-K activation atom
  static constexpr int ACT = 2 * ATOM;                 // the step's two atoms
  static constexpr int ATILE = 128 * 128;              // compressed weights: 128 rows x 64 halves
  static constexpr int OFF_ACT = 0;
  static constexpr int OFF_A = ACT;
  static constexpr int OFF_B = OFF_A + ATILE;          // 4 rows x 1024 B of packed codes
  static constexpr int OFF_M = OFF_B + 4096;           // 4 rows x 512 B of metadata
  static constexpr int OFF_S = OFF_M + 2048;           // one scale row (128 features)
  static constexpr int STAGE = (OFF_S + 256 + 1023) / 1024 * 1024;
  static constexpr int HEADER = 1024;
  static constexpr int DEPTH_FIT = (kPrefillSmemBudget - HEADER - 1024) / STAGE;
  static constexpr int DEPTH_CAP = DEPTH_FIT > 8 ? 8 : DEPTH_FIT;
  static constexpr int DEPTH = DEPTH_CAP / NG * NG;
  static constexpr int SMEM = HEADER + DEPTH * STAGE + 1024;
  static constexpr uint32_t TX_ACT_PAIR = 2 * ACT;
  static constexpr uint32_t TX_W = 4096 + 2048;        // + 256 with group scales
  static constexpr int THREADS = (2 + 4 * NG) * 32;
  static constexpr int META_COLS = 16;                 // 4 MMAs x 4-column-aligned slots
  static constexpr int BN = 256;                       // accumulator columns (the pair's rows)
  static constexpr int TMEM_NEED = BN + DEPTH * META_COLS;
  static constexpr int TMEM_COLS = TMEM_NEED <= 256 ? 256 : 512;
  static_assert(DEPTH >= 2 && DEPTH % NG == 0, "paired sparse prefill ring too shallow");
  static_assert(TMEM_NEED <= 512, "tensor memory");
  static_assert((3 * DEPTH + 1) * 8 <= HEADER - 8, "barriers exceed the header");
};

__device__ __forceinline__ uint32_t ld_shared_cluster_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or
// the peer's), release at CTA scope.  What the arrive publishes - shared
// memory made visible to the async proxy and completed tensor-memory stores
// of this CTA - never leaves this SM: the pair's tensor cores read it here.
// (A cluster-scope release costs a membar of ~1k cycles per arrive on B200.)
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// 2-D TMA load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (`cluster_bar`: shared::cluster
// address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, int x, int y,
                                                 uint32_t cluster_bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(cluster_bar), "l"(policy)
      : "memory");
}

// 3-D form of tma_load_2d_pair (x innermost).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* tmap, int x, int y, int z,
                                                 uint32_t cluster_bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(cluster_bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void sts16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

// 2-D tiled TMA store shared -> global (rows past the tensor's end are
// clipped by the copy), then wait until it has completed.
__device__ __forceinline__ void tma_store_2d_wait(const void* tmap, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

__device__ __forceinline__ void umma_sp_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t e_tmem, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.sp.cta_group::2.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at the same offset in both CTAs of the pair once
// every previously issued MMA of this thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], m;\n\t}" ::"r"(bar)
      : "memory");
}

// EPI: fused bias / activation compiled in (a separate instantiation; the
// epilogue code cost the plain kernel 1-3 %).
// META3: 3-bit metadata (kernel_experiments/sparse_marlin/metadata_decode):
// per 32-K row and 64-feature chunk 48 words instead of 64; each dequantising
// thread decodes its one 4-bit word from two of them before the copy into
// tensor memory, so the MMAs are unchanged.
// DIAG: metadata-cost diagnostics (kDiagNoGmem / kDiagNoReg of
// device_primitives.cuh; 0 in production instances).
template <int NG, bool GROUPED, bool EPI, bool META3 = false, int DIAG = 0>
__global__ void __launch_bounds__(PrefillSp2Cfg<NG>::THREADS, 1)
    marlin24_prefill_sp2_kernel(const __grid_constant__ PrefillParams p) {
  using Cfg = PrefillSp2Cfg<NG>;
  static_assert(DIAG == 0 || (!META3 && !EPI), "diagnostics: 4-bit metadata, plain store");
  constexpr int D = Cfg::DEPTH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* wfull_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* aready_bar = wfull_bar + D;
  uint64_t* empty_bar = aready_bar + D;
  uint64_t* acc_bar = empty_bar + D;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 1024 - 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 1024 - 4);
  uint8_t* ring = smem + Cfg::HEADER;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();   // 0: issues the pair's MMAs
  const int n_tile = blockIdx.x;              // this CTA's 128 features
  const int m_tile = blockIdx.y;              // the pair's 256 batch rows
  const int ksteps = p.K / 128;

  if (threadIdx.x < D) {
    mbar_init(smem_addr(&wfull_bar[threadIdx.x]), 1);
    // the pair's 8 dequantising-group warps + the even CTA's activation expect_tx
    mbar_init(smem_addr(&aready_bar[threadIdx.x]), 9);
    mbar_init(smem_addr(&empty_bar[threadIdx.x]), 1);
  }
  if (threadIdx.x == 32) {
    mbar_init(smem_addr(acc_bar), 1);
    *abort_flag = 0;
  }
  if (threadIdx.x < D || threadIdx.x == 32) fence_mbar_init();
  if constexpr ((DIAG & kDiagNoGmem) != 0) {
    // uniform metadata in every stage's region, written once (never copied)
    for (int st = 0; st < D; ++st) {
      uint32_t* mreg = reinterpret_cast<uint32_t*>(smem + Cfg::HEADER + st * Cfg::STAGE + Cfg::OFF_M);
      for (int i = threadIdx.x; i < 2048 / 4; i += blockDim.x) mreg[i] = kDiagMetaWord;
    }
  }
  if (warp == 1) tmem_alloc_pair(smem_addr(tmem_slot), Cfg::TMEM_COLS);
  if (threadIdx.x == 0) {
    prefetch_tmap(&p.tm_act);
    prefetch_tmap(&p.tm_b);
    prefetch_tmap(&p.tm_meta);
    if (GROUPED) prefetch_tmap(&p.tm_s);
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // both CTAs must see the same tensor-memory columns (the MMA addresses both)
  if (threadIdx.x == 0 && ld_shared_cluster_u32(mapa_shared(smem_addr(tmem_slot), rank ^ 1u)) != tmem) {
    atomicOr(p.status, kStatusFullWaitTimeout);
    *abort_flag = 1;
  }
  __syncthreads();
  const bool run = *abort_flag == 0;
  const uint32_t tmem_e = tmem + Cfg::BN;
  const uint32_t ring_base = smem_addr(ring);

  if (!run) {
    // nothing issued: fall through to the teardown
  } else if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp runs the loop, lane 0 issues (a lone lane looping while
    // the rest of its warp waits at the CTA barrier runs slower).
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    // packed codes 4 x 1 KB, metadata 4 x 512 B (4-bit) or 4 x 384 B (3-bit)
    const uint32_t txw = 4096 + ((DIAG & kDiagNoGmem) ? 0 : (META3 ? 1536 : 2048)) + (GROUPED ? 256 : 0);
    const int act_row = m_tile * 256 + static_cast<int>(rank) * Cfg::ROWS;
    for (int ks = 0; ks < ksteps; ++ks) {
      const int slot = ks % D;
      const uint32_t parity = ((ks / D) & 1) ^ 1;
      const bool ok = mbar_wait_bounded(smem_addr(&empty_bar[slot]), parity, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicOr(p.status, kStatusEmptyWaitTimeout);
        break;
      }
      if (lane == 0) {
        const uint32_t st = ring_base + slot * Cfg::STAGE;
        const uint32_t wfull = smem_addr(&wfull_bar[slot]);
        mbar_arrive_expect_tx(wfull, txw);
        tma_load_2d(st + Cfg::OFF_B, &p.tm_b, n_tile * 128, ks * 4, wfull, pol_stream);
        if constexpr ((DIAG & kDiagNoGmem) == 0)
          tma_load_2d(st + Cfg::OFF_M, &p.tm_meta, n_tile * (META3 ? 48 : 64), ks * 4, wfull,
                      pol_stream);
        if (GROUPED) tma_load_2d(st + Cfg::OFF_S, &p.tm_s, n_tile * 32, ks, wfull, pol_keep);
        // both CTAs' activation halves count on the even CTA's ready barrier
        const uint32_t ready = smem_addr(&aready_bar[slot]);
        if (rank == 0) mbar_arrive_expect_tx(ready, Cfg::TX_ACT_PAIR);
        // (64 halves, rows, K/64 slices): both 64-K atoms of the step in one copy
        tma_load_3d_pair(st + Cfg::OFF_ACT, &p.tm_act, 0, act_row, ks * 2, mapa_shared(ready, 0),
                         pol_keep);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (even CTA)
    if (rank == 0) {
      constexpr uint32_t idesc =
          (1u << 2) | (1u << 4) | (static_cast<uint32_t>(256 >> 3) << 17) | ((256u >> 4) << 24);
      constexpr uint64_t kStageDesc = Cfg::STAGE >> 4;  // start-address field step
      constexpr uint64_t kAtomDesc = Cfg::ATOM >> 4;
      const uint64_t ad0 = umma_desc_sw128_k(ring_base + Cfg::OFF_A);
      const uint64_t bd0 = umma_desc_sw128_k(ring_base + Cfg::OFF_ACT);
      const uint32_t ready0 = smem_addr(aready_bar);
      const uint32_t empty0 = smem_addr(empty_bar);
      uint32_t parity = 0;
      bool ok = true;
      // The loop runs a ring's worth of steps per iteration, so slot numbers
      // and descriptor offsets are compile-time constants.
      for (int ks0 = 0; ks0 < ksteps && ok; ks0 += D, parity ^= 1) {
#pragma unroll
        for (int slot = 0; slot < D; ++slot) {
          const int ks = ks0 + slot;
          if (ks >= ksteps) break;
          // one wait per step: activations landed and both CTAs' tiles dequantised
          ok = mbar_wait_bounded(ready0 + 8 * slot, parity, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            // four MMAs of K = 32: 32 compressed bytes of each 128-byte weight
            // row; 64 bytes of each 128-byte activation row, two atoms
            const uint64_t ad = ad0 + slot * kStageDesc, bd = bd0 + slot * kStageDesc;
            const uint32_t e = tmem_e + slot * Cfg::META_COLS;
            umma_sp_f16_pair(tmem, ad, bd, e, idesc, ks ? 1u : 0u);
            umma_sp_f16_pair(tmem, ad + 2, bd + 4, e + 4, idesc, 1u);
            umma_sp_f16_pair(tmem, ad + 4, bd + kAtomDesc, e + 8, idesc, 1u);
            umma_sp_f16_pair(tmem, ad + 6, bd + kAtomDesc + 4, e + 12, idesc, 1u);
            umma_commit_pair(empty0 + 8 * slot);
          }
          __syncwarp();
        }
      }
      if (lane == 0) umma_commit_pair(smem_addr(acc_bar));
    }
  } else {
    // ---------------------------------------------- dequantise, then epilogue
    const int dw = warp - 2;        // 0 .. 4*NG-1
    const int grp = dw >> 2;        // K steps ks % NG == grp
    const int r = dw & 3;           // 32-K row of the step whose codes this warp converts
    const int quarter = warp & 3;   // tensor-memory lanes this warp may access
    const int g = lane >> 2, t = lane & 3;
    const uint32_t m_word = (quarter >> 1) * 256 +
                            4 * (32 * (quarter & 1) + 4 * (lane & 7) + 2 * (lane >> 4) + ((lane >> 3) & 1));
    // 3-bit: word l = (4-bit word) mod 32 of the chunk's 48-word block
    const uint32_t m3_l = 4 * (lane & 7) + 2 * (lane >> 4) + ((lane >> 3) & 1);
    const uint32_t m3_word = (quarter >> 1) * 192 + 4 * m3_l;
    const bool m3_upper = m3_l >= 16;
    const uint32_t e_lane = tmem_e + (static_cast<uint32_t>(32 * quarter) << 16);
    const uint32_t ready_own = smem_addr(aready_bar);
    bool ok = true;
    for (int ks = grp; ks < ksteps; ks += NG) {
      const int slot = ks % D;
      const uint32_t parity = (ks / D) & 1;
      if (!mbar_wait_bounded(smem_addr(&wfull_bar[slot]), parity, abort_flag)) {
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
        ok = false;
        break;
      }
      const uint32_t st = ring_base + slot * Cfg::STAGE;
      // metadata of the four MMAs into this warp's lanes of the stage's slots
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t mw;
        if constexpr (META3) {
          // 4-bit word w of chunk quarter/2 (w >= 32 exactly in odd quarters)
          // is the high (w < 32) or low (w >= 32) decode of 3-bit words
          // l = w mod 32 and l + 16 of the chunk's 48 (see meta3_pair_decode)
          const uint32_t a = lds32(st + Cfg::OFF_M + kk * 384 + m3_word);
          const uint32_t b = lds32(st + Cfg::OFF_M + kk * 384 + m3_word + 64);
          if (quarter & 1)
            mw = decode24_low(m3_upper ? (b >> 8) : __funnelshift_r(a, b, 24));
          else
            mw = decode24_high(m3_upper ? __funnelshift_r(a, b, 16) : a);
        } else if constexpr ((DIAG & kDiagNoReg) != 0) {
          mw = kDiagMetaWord;
        } else {
          mw = lds32(st + Cfg::OFF_M + kk * 512 + m_word);
        }
        tmem_st32(e_lane + slot * Cfg::META_COLS + 4 * kk, mw);
      }
      // compressed weights of 32-K row r, both 64-feature chunks
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const uint4 q = lds128(st + Cfg::OFF_B + r * 1024 + cc * 512 + lane * 16);
        uint4 sv = make_uint4(0, 0, 0, 0);
        if (GROUPED) sv = lds128(st + Cfg::OFF_S + cc * 128 + g * 16);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          half2 lo0, hi0, lo1, hi1;
          dequant_pair(qw[j], lo0, hi0);       // feature 8g+j: kc 2t.., 8+2t..
          dequant_pair(qw[j] >> 8, lo1, hi1);  // feature 8g+j+4
          if (GROUPED) {
            const half2 s2 = *reinterpret_cast<const half2*>(&sw[j]);
            const half2 sx = __low2half2(s2), sy = __high2half2(s2);
            lo0 = __hmul2(lo0, sx);
            hi0 = __hmul2(hi0, sx);
            lo1 = __hmul2(lo1, sy);
            hi1 = __hmul2(hi1, sy);
          }
          // rows: feature 64cc + 8g + j -> g + 16(4cc + j), feature + 4 -> + 8;
          // compressed columns 16r + 2t (16-byte chunk 2r) and 16r + 8 + 2t
          // (chunk 2r+1) of a 128-byte row, swizzled with row mod 8 = g
          const int m_lo = g + 16 * (4 * cc + j);
          const uint32_t row_lo = st + Cfg::OFF_A + m_lo * 128;
          const uint32_t row_hi = row_lo + 8 * 128;
          const uint32_t ca = ((2 * r) ^ g) << 4, cb = ((2 * r + 1) ^ g) << 4;
          const uint32_t wo = 4 * t;
          sts32(row_lo + ca + wo, *reinterpret_cast<uint32_t*>(&lo0));
          sts32(row_lo + cb + wo, *reinterpret_cast<uint32_t*>(&hi0));
          sts32(row_hi + ca + wo, *reinterpret_cast<uint32_t*>(&lo1));
          sts32(row_hi + cb + wo, *reinterpret_cast<uint32_t*>(&hi1));
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(ready_own + 8 * slot);
        else
          mbar_arrive_remote(mapa_shared(ready_own + 8 * slot, 0));
      }
    }

    // ------------------------------------------------------------ epilogue
    // The ring is idle once the last MMA has completed: the CTA's 256 x 128
    // fp16 block of C is assembled there (row b at 256 B, feature f at 2f;
    // the 32 lanes of a store hit 16 distinct banks) and written by one TMA
    // tensor store, which also clips rows past M.
    bool stored = false;
    if (ok && mbar_wait_bounded(smem_addr(acc_bar), 0, abort_flag)) {
      tc_fence_after();
      const int rr = 32 * quarter + lane;
      const int m2 = rr >> 4;
      const int feat = 64 * (m2 >> 2) + 8 * (rr & 7) + (m2 & 3) + 4 * ((rr >> 3) & 1);
      float cs = 1.f;
      if (!GROUPED) cs = __half2float(reinterpret_cast<const half*>(p.s)[n_tile * 128 + feat]);
      const float col_bias =
          EPI && p.bias != nullptr ? __half2float(p.bias[n_tile * 128 + feat]) : 0.f;
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
      const uint32_t c_col = ring_base + 2 * feat;
#pragma unroll 1
      for (int cb2 = grp; cb2 < Cfg::BN / 32; cb2 += NG) {
        uint32_t v[32];
        tmem_ld32(lane_addr + cb2 * 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          sts16(c_col + (cb2 * 32 + j) * 256,
                __half_as_ushort(__float2half_rn(
                    EPI ? epilogue_act(__uint_as_float(v[j]) * cs + col_bias, p.act)
                        : __uint_as_float(v[j]) * cs)));
      }
      fence_proxy_async_smem();
      stored = true;
    } else if (ok && lane == 0) {
      atomicOr(p.status, kStatusFullWaitTimeout);
    }
    // all dequantising warps' parts of the block are in shared memory
    named_bar_sync(1, 4 * NG * 32);
    if (stored && warp == 2 && lane == 0 && *abort_flag == 0)
      tma_store_2d_wait(&p.tm_c, ring_base, n_tile * 128, m_tile * 256);
  }

  // Teardown: every MMA of the pair must be complete (acc_bar, bounded) before
  // either CTA releases its shared or tensor memory.
  tc_fence_before();
  __syncthreads();
  if (warp == 1 && run) mbar_wait_bounded(smem_addr(acc_bar), 0, abort_flag);
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
}

}  // namespace sm100
