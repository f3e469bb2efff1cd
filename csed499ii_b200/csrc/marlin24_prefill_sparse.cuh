// 2:4 sparse W4A16 GEMM for batches above 64 rows on the structured-sparse
// tensor-core instruction: tcgen05.mma.sp kind::f16, fp32 accumulator and the
// 2:4 metadata in tensor memory.  Same inputs and host contract as
// marlin24_prefill_kernel (the dense-expansion form, kept for K not a
// multiple of 128).
//
// Per CTA: one 128-feature x BN-row output tile over the whole K range, K in
// steps of 64 (a 64-byte-swizzled tile of compressed weights, one 128-byte
// swizzle atom of activations, two MMAs of K = 32), so 4-8 stages fit.
//
//  * warp 0 (one thread): TMA of the activation atom and of the packed codes
//    (2 x 32-K rows), metadata and scale row of the 128 features;
//  * warps 2.. (NG groups of four, K steps in turn): dequantise the INT4
//    codes and apply the group scale (fp16, as the reference), storing the
//    COMPRESSED values (two per group of four; no zero fill) into the UMMA
//    K-major 64-byte-swizzled tile, and copy the metadata words of the step
//    into tensor memory (tcgen05.st; one 4-column-aligned slot per MMA);
//  * warp 1 (one thread): tcgen05.mma.sp.cta_group::1.kind::f16 with the
//    compressed weights as operand A, the activations as operand B and the
//    metadata slot of each MMA; tcgen05.commit frees the stage.
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
  static constexpr uint32_t TX_NOSCALE = ACT + 2048 + 1024;
  static constexpr uint32_t TX_SCALE = TX_NOSCALE + 256;
  static constexpr int THREADS = (2 + 4 * NG) * 32;
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
    mbar_init(smem_addr(&full_bar[threadIdx.x]), 1);
    mbar_init(smem_addr(&aready_bar[threadIdx.x]), 4);
    mbar_init(smem_addr(&empty_bar[threadIdx.x]), 1);
  }
  if (threadIdx.x == 32) {
    mbar_init(smem_addr(acc_bar), 1);
    *abort_flag = 0;
  }
  if (threadIdx.x < D || threadIdx.x == 32) fence_mbar_init();
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), Cfg::TMEM_COLS);
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
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      const uint32_t tx = GROUPED ? Cfg::TX_SCALE : Cfg::TX_NOSCALE;
      for (int ks = 0; ks < ksteps; ++ks) {
        const int slot = ks % D;
        const uint32_t parity = ((ks / D) & 1) ^ 1;
        if (!mbar_wait_bounded(smem_addr(&empty_bar[slot]), parity, abort_flag)) {
          atomicOr(p.status, kStatusEmptyWaitTimeout);
          break;
        }
        const uint32_t full = smem_addr(&full_bar[slot]);
        const uint32_t st = ring_base + slot * Cfg::STAGE;
        mbar_arrive_expect_tx(full, tx);
        tma_load_2d(st + Cfg::OFF_ACT, &p.tm_act, ks * 64, m_tile * BN, full, pol_keep);
        tma_load_2d(st + Cfg::OFF_B, &p.tm_b, n_tile * 128, ks * 2, full, pol_stream);
        tma_load_2d(st + Cfg::OFF_M, &p.tm_meta, n_tile * 64, ks * 2, full, pol_stream);
        if (GROUPED) tma_load_2d(st + Cfg::OFF_S, &p.tm_s, n_tile * 32, ks >> 1, full, pol_keep);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_f32(BN) | (1u << 2);  // sparse
      bool ok = true;
      for (int ks = 0; ks < ksteps && ok; ++ks) {
        const int slot = ks % D;
        const uint32_t parity = (ks / D) & 1;
        ok = mbar_wait_bounded(smem_addr(&full_bar[slot]), parity, abort_flag) &&
             mbar_wait_bounded(smem_addr(&aready_bar[slot]), parity, abort_flag);
        if (!ok) {
          atomicOr(p.status, kStatusFullWaitTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t st = ring_base + slot * Cfg::STAGE;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t ad = umma_desc_sw64_k(st + Cfg::OFF_A + kk * 32);
          const uint64_t bd = umma_desc_sw128_k(st + Cfg::OFF_ACT + kk * 64);
          umma_sp_f16(tmem, ad, bd, tmem_e + slot * Cfg::META_COLS + 4 * kk, idesc,
                      (ks | kk) ? 1u : 0u);
        }
        umma_commit(smem_addr(&empty_bar[slot]));
      }
      umma_commit(smem_addr(acc_bar));
    }
  } else {
    // ---------------------------------------------- dequantise, then epilogue
    const int dw = warp - 2;        // 0 .. 4*NG-1
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
            p.C[static_cast<long long>(b) * p.N + n] = __float2half_rn(__uint_as_float(v[j]) * cs);
        }
      }
    } else if (ok && lane == 0) {
      atomicOr(p.status, kStatusFullWaitTimeout);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mbar_wait_bounded(smem_addr(acc_bar), 0, abort_flag);
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace sm100
