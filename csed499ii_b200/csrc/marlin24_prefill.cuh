// 2:4 sparse W4A16 GEMM for the compute-bound regime (batch rows M > 64),
// sm_100a, on the 5th-generation tensor cores (tcgen05 / TMEM).
//
//   C[M, N] (fp16) = A[M, K] (fp16) . dequant(B, meta, s)[K, N]
//
// Same packed inputs as the decode kernel (Sparse-Marlin layout, reference:
// kernel_experiments/sparse_marlin/src/marlin/__init__.py:331-388 and
// _semi_structured_conversions.py:54-179).  Where the reference runs its
// batch-64 Ampere kernel in parallel slices (marlin_cuda_kernel_nm.cu:792-808)
// this kernel computes one 128-feature x BN-row output tile per CTA over the
// whole K range:
//
//  * warp 0 (one thread) streams, per 64-wide K step, the activation tile
//    (TMA, 128-byte swizzle: already the UMMA K-major canonical layout) and
//    the packed weights, metadata and scales of the 128 output features into
//    a ring of stages (mbarrier full / empty pairs, bounded waits);
//  * warps 2.. (NG groups of four, taking the K steps in turn) dequantise
//    the packed INT4 codes (magic-number conversion,
//    group scale applied in fp16 as in the reference) and expand each 2:4
//    pair to its four dense positions with byte permutes, writing the dense
//    fp16 weight tile (128 x 64) into the stage in the UMMA K-major 128-byte
//    swizzled layout;
//  * warp 1 (one thread) issues tcgen05.mma kind::f16 (M = 128, N = BN,
//    K = 16 per instruction) with the weights as operand A and the
//    activations as operand B, accumulating in fp32 in tensor memory, and
//    frees each stage with tcgen05.commit;
//  * the same warps then read the accumulator (tcgen05.ld) and store C.
//
// The dense expansion doubles the tensor work against a sparse MMA (the
// structured-sparse form needs the metadata in tensor memory in a layout
// not used here); the kernel is bounded by the dense tensor peak.
// Rows of the weight tile hold output features in the order
// 64c + 8j + g for feature 64c + 8g + j (c chunk, g group, j in 0..7), which
// makes the dequantising warps' stores bank-conflict free; the epilogue maps
// accumulator lanes back.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "device_primitives.cuh"

namespace sm100 {

struct PrefillParams {
  CUtensorMap tm_act;   // A fp16, dims (K, M), box (64, BN), 128-byte swizzle
  CUtensorMap tm_b;     // B as u64, dims (N, K/32), box (128, 2)
  CUtensorMap tm_meta;  // meta as u64, dims (N/2, K/32), box (64, 2)
  CUtensorMap tm_s;     // s as u64, dims (N/4, K/128), box (32, 1)   (grouped only)
  CUtensorMap tm_c;     // C fp16, dims (N, M), box (128, 256)        (CTA-pair form only)
  const uint8_t* s;     // fp16 scales (per-column scaling in the epilogue)
  half* C;              // fp16 (M, N) row-major
  const half* bias;     // fused epilogue: fp16 bias per output column, or null
  int act;              // fused epilogue: activation (kAct*)
  int* status;          // device status word
  int M;
  int N;
  int K;
  int grouped;
};

constexpr int kPrefillSmemBudget = 227 * 1024;

// NG groups of four dequantising warps take the K steps in turn (group
// ks % NG).  The ring depth is a multiple of NG, so every slot belongs to one
// group, which visits each of its uses in order (an mbarrier parity wait must
// never skip a phase).
template <int BN, int NG>
struct PrefillCfg {
  static_assert(BN == 128 || BN == 256, "batch tile");
  static constexpr int ACT = BN * 128;                 // activation tile (BN rows x 64 K)
  static constexpr int ATILE = 128 * 128;              // dense weight tile (128 rows x 64 K)
  static constexpr int OFF_ACT = 0;
  static constexpr int OFF_A = ACT;
  static constexpr int OFF_B = OFF_A + ATILE;          // 2 rows x 1024 B of packed codes
  static constexpr int OFF_M = OFF_B + 2048;           // 2 rows x 512 B of metadata
  static constexpr int OFF_S = OFF_M + 1024;           // 128 scales
  static constexpr int STAGE = (OFF_S + 256 + 1023) / 1024 * 1024;
  static constexpr int HEADER = 1024;
  static constexpr int DEPTH_FIT = (kPrefillSmemBudget - HEADER - 1024) / STAGE;
  static constexpr int DEPTH_CAP = DEPTH_FIT > 8 ? 8 : DEPTH_FIT;
  static constexpr int DEPTH = DEPTH_CAP / NG * NG;
  static constexpr int SMEM = HEADER + DEPTH * STAGE + 1024;
  static constexpr uint32_t TX_NOSCALE = ACT + 2048 + 1024;
  static constexpr uint32_t TX_SCALE = TX_NOSCALE + 256;
  static constexpr int THREADS = (2 + 4 * NG) * 32;
  static_assert(DEPTH >= 2 && DEPTH % NG == 0, "prefill ring too shallow");
};

// ---------------------------------------------------------------------------
// tcgen05 helpers
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzled
// canonical layout: 8-row groups 1024 bytes apart (stride byte offset),
// descriptor version 1, swizzle mode 2.  The leading byte offset is unused
// for swizzled K-major operands.
__device__ __forceinline__ uint64_t umma_desc_sw128_k(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Byte-permute selectors that place a kept pair (v0 at idx0, v1 at idx1) of a
// 2:4 group into its four dense fp16 slots, zero elsewhere: low 16 bits for
// slots 0-1, high 16 bits for slots 2-3 (prmt with a zero second operand).
__device__ __forceinline__ uint32_t expand_selector(uint32_t nib) {
  const uint32_t i0 = nib & 3u, i1 = nib >> 2;
  uint32_t sel = 0;
#pragma unroll
  for (uint32_t pos = 0; pos < 4; ++pos) {
    const uint32_t s = pos == i0 ? 0x10u : (pos == i1 ? 0x32u : 0x44u);
    sel |= s << (8 * pos);
  }
  return (sel & 0xFFFFu) | ((sel >> 16) << 16);
}

template <int BN, int NG, bool GROUPED>
__global__ void __launch_bounds__(PrefillCfg<BN, NG>::THREADS, 1)
    marlin24_prefill_kernel(const __grid_constant__ PrefillParams p) {
  using Cfg = PrefillCfg<BN, NG>;
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
  uint32_t* sel_tab = reinterpret_cast<uint32_t*>(smem + 512);
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
  if (threadIdx.x >= 64 && threadIdx.x < 80) sel_tab[threadIdx.x - 64] = expand_selector(threadIdx.x - 64);
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), BN);
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
      constexpr uint32_t idesc = umma_idesc_f16_f32(BN);
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
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = umma_desc_sw128_k(st + Cfg::OFF_A + kk * 32);
          const uint64_t bd = umma_desc_sw128_k(st + Cfg::OFF_ACT + kk * 32);
          umma_f16(tmem, ad, bd, idesc, (ks | kk) ? 1u : 0u);
        }
        umma_commit(smem_addr(&empty_bar[slot]));
      }
      // completes once every MMA issued above has finished
      umma_commit(smem_addr(acc_bar));
    }
  } else {
    // ---------------------------------------------- dequantise, then epilogue
    const int dw = warp - 2;       // 0 .. 4*NG-1
    const int grp = dw >> 2;       // this warp's group: K steps ks % NG == grp
    const int pr = dw & 1;         // 32-K row inside the 64-K step
    const int cc = (dw >> 1) & 1;  // 64-feature chunk inside the 128-feature tile
    const int g = lane >> 2;
    const int t = lane & 3;
    const uint32_t q_off = Cfg::OFF_B + pr * 1024 + cc * 512 + lane * 16;
    const uint32_t m_off = Cfg::OFF_M + pr * 512 + cc * 256 + g * 16;
    const uint32_t s_off = Cfg::OFF_S + cc * 128 + g * 16;
    // destination rows (feature 64cc + 8g + j lives in row 64cc + 8j + g) and
    // swizzled 16-byte chunks of dense groups t and t + 4 of this 32-K row
    const uint32_t row0 = Cfg::OFF_A + (64 * cc + g) * 128;
    const uint32_t ch_a = ((4 * pr + (t >> 1)) ^ g) << 4;
    const uint32_t ch_b = ((4 * pr + 2 + (t >> 1)) ^ g) << 4;
    const uint32_t half_off = 8 * (t & 1);
    const uint32_t sel_base = smem_addr(sel_tab);
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
      const uint4 q = lds128(st + q_off);
      const uint4 ma = lds128(st + m_off);
      const uint4 mb = lds128(st + m_off + 128);
      uint4 sv = make_uint4(0, 0, 0, 0);
      if (GROUPED) sv = lds128(st + s_off);
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
      const uint32_t mw[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        half2 lo0, hi0, lo1, hi1;
        dequant_pair(qw[j], lo0, hi0);       // feature 8g+j: groups t, t+4
        dequant_pair(qw[j] >> 8, lo1, hi1);  // feature 8g+j+4: groups t, t+4
        if (GROUPED) {
          const half2 s2 = *reinterpret_cast<const half2*>(&sw[j]);
          const half2 sx = __low2half2(s2), sy = __high2half2(s2);
          lo0 = __hmul2(lo0, sx);
          hi0 = __hmul2(hi0, sx);
          lo1 = __hmul2(lo1, sy);
          hi1 = __hmul2(hi1, sy);
        }
        // metadata words of the pair (c, d) = (j >> 1, j & 1): dense K half 0 / 1
        const uint32_t w0 = mw[4 * (j >> 1) + 2 * (j & 1)];
        const uint32_t w1 = mw[4 * (j >> 1) + 2 * (j & 1) + 1];
        const uint32_t n_lo_a = (w0 >> (4 * t)) & 15u, n_lo_b = (w1 >> (4 * t)) & 15u;
        const uint32_t n_hi_a = (w0 >> (16 + 4 * t)) & 15u, n_hi_b = (w1 >> (16 + 4 * t)) & 15u;
        const uint32_t s_lo_a = lds32(sel_base + 4 * n_lo_a), s_lo_b = lds32(sel_base + 4 * n_lo_b);
        const uint32_t s_hi_a = lds32(sel_base + 4 * n_hi_a), s_hi_b = lds32(sel_base + 4 * n_hi_b);
        const uint32_t v_lo_a = *reinterpret_cast<uint32_t*>(&lo0);
        const uint32_t v_lo_b = *reinterpret_cast<uint32_t*>(&hi0);
        const uint32_t v_hi_a = *reinterpret_cast<uint32_t*>(&lo1);
        const uint32_t v_hi_b = *reinterpret_cast<uint32_t*>(&hi1);
        const uint32_t r_lo = st + row0 + (8 * j) * 128;
        const uint32_t r_hi = st + row0 + (8 * (j + 4)) * 128;
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(r_lo + ch_a + half_off),
                     "r"(prmt(v_lo_a, 0u, s_lo_a)), "r"(prmt(v_lo_a, 0u, s_lo_a >> 16)) : "memory");
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(r_lo + ch_b + half_off),
                     "r"(prmt(v_lo_b, 0u, s_lo_b)), "r"(prmt(v_lo_b, 0u, s_lo_b >> 16)) : "memory");
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(r_hi + ch_a + half_off),
                     "r"(prmt(v_hi_a, 0u, s_hi_a)), "r"(prmt(v_hi_a, 0u, s_hi_a >> 16)) : "memory");
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(r_hi + ch_b + half_off),
                     "r"(prmt(v_hi_b, 0u, s_hi_b)), "r"(prmt(v_hi_b, 0u, s_hi_b >> 16)) : "memory");
      }
      // make the generic-proxy stores visible to the tensor core, then signal
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&aready_bar[slot]));
    }

    // ------------------------------------------------------------ epilogue
    if (ok && mbar_wait_bounded(smem_addr(acc_bar), 0, abort_flag)) {
      tc_fence_after();
      const int quarter = warp & 3;   // TMEM lanes this warp may access
      const int r = 32 * quarter + lane;
      const int feat = 64 * (r >> 6) + 8 * (r & 7) + ((r >> 3) & 7);
      const int n = n_tile * 128 + feat;
      float cs = 1.f;
      if (!GROUPED) cs = __half2float(reinterpret_cast<const half*>(p.s)[n]);
      const float col_bias = p.bias != nullptr ? __half2float(p.bias[n]) : 0.f;
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
#pragma unroll 1
      for (int cb = grp; cb < BN / 32; cb += NG) {
        uint32_t v[32];
        tmem_ld32(lane_addr + cb * 32, v);
        const int b0 = m_tile * BN + cb * 32;
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
  if (warp == 1) {
    // the accumulator must be idle before its columns are released: the
    // epilogue waited for acc_bar; on an aborted run wait (bounded) here
    mbar_wait_bounded(smem_addr(acc_bar), 0, abort_flag);
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

}  // namespace sm100
