// Persistent form of the CTA-pair prefill kernel (marlin24_prefill_sp2_kernel):
// each 2-CTA cluster loops over 256-feature x 256-row output tiles
// (tile c, c + clusters, ...), so the per-tile costs of the one-tile form
// (CTA start-up, barrier and tensor-memory set-up, filling the ring, the
// epilogue) stop being serial.  A fit of the one-tile kernel's sweep puts
// them at ~3.8 us per tile: 12 % of a K = 8192 tile, 22 % of a K = 4096 tile.
//
//  * warp 0: TMA producer, one continuous stream of 128-K steps over all of
//    the cluster's tiles (it runs up to a ring ahead across tile ends);
//  * warp 1: MMA issuer (even CTA), as in the one-tile form, plus one wait
//    per tile for the accumulator to be drained before the tile's first MMA
//    (`acc_empty`) and one commit after its last (`acc_full`);
//  * warps 2-17: four groups of four dequantising warps, one continuous
//    stream of steps (they never see tile boundaries);
//  * warps 18-21: epilogue, one warp per tensor-memory lane quarter, each
//    reading the eight 32-column blocks of the 256-column accumulator and
//    storing them to C, then arriving on `acc_empty`.
//
// Barriers: wfull / aready / empty per ring slot as in the one-tile form;
// acc_full (each CTA, count 1, commit multicast to the pair) per tile;
// acc_empty (even CTA, count 8: the pair's epilogue warps) per tile;
// done (each CTA, count 1, commit multicast) once all MMAs are issued.
#pragma once

#include "marlin24_prefill_sparse.cuh"

namespace sm100 {

template <int NG>
struct PrefillSp2pCfg : PrefillSp2Cfg<NG> {
  // 8 (two per lane quarter) spill at the 72-register cap of 832 threads
  static constexpr int EPI_WARPS = 4;
  static constexpr int DQ_WARP0 = 2;
  static constexpr int EPI_WARP0 = 2 + 4 * NG;
  static constexpr int THREADS = (2 + 4 * NG + EPI_WARPS) * 32;
  static_assert((3 * PrefillSp2Cfg<NG>::DEPTH + 3) * 8 <= PrefillSp2Cfg<NG>::HEADER - 8,
                "barriers exceed the header");
  static_assert(THREADS <= 1024, "too many threads");
};

template <int NG, bool GROUPED, bool EPI>
__global__ void __launch_bounds__(PrefillSp2pCfg<NG>::THREADS, 1)
    marlin24_prefill_sp2p_kernel(const __grid_constant__ PrefillParams p) {
  using Cfg = PrefillSp2pCfg<NG>;
  constexpr int D = Cfg::DEPTH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* wfull_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* aready_bar = wfull_bar + D;
  uint64_t* empty_bar = aready_bar + D;
  uint64_t* acc_full = empty_bar + D;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* done_bar = acc_empty + 1;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 1024 - 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 1024 - 4);
  uint8_t* ring = smem + Cfg::HEADER;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();  // 0: issues the pair's MMAs
  const int ksteps = p.K / 128;
  // the cluster's tiles: id = cluster + j * clusters, n fastest
  const int n_pairs = p.N / 256;
  const int m_tiles = (p.M + 255) / 256;
  const int tiles = n_pairs * m_tiles;
  const int cluster = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;
  const int my_tiles = cluster < tiles ? (tiles - cluster + clusters - 1) / clusters : 0;
  const long long total_steps = static_cast<long long>(my_tiles) * ksteps;

  if (threadIdx.x < D) {
    mbar_init(smem_addr(&wfull_bar[threadIdx.x]), 1);
    mbar_init(smem_addr(&aready_bar[threadIdx.x]), 9);
    mbar_init(smem_addr(&empty_bar[threadIdx.x]), 1);
  }
  if (threadIdx.x == 32) {
    mbar_init(smem_addr(acc_full), 1);
    mbar_init(smem_addr(acc_empty), 2 * Cfg::EPI_WARPS);
    mbar_init(smem_addr(done_bar), 1);
    *abort_flag = 0;
  }
  if (threadIdx.x < D || threadIdx.x == 32) fence_mbar_init();
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
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const uint32_t txw = Cfg::TX_W + (GROUPED ? 256 : 0);
    long long g = 0;
    bool ok = true;
    for (int j = 0; j < my_tiles && ok; ++j) {
      const int id = cluster + j * clusters;
      const int n_tile = 2 * (id % n_pairs) + static_cast<int>(rank);
      const int act_row = (id / n_pairs) * 256 + static_cast<int>(rank) * Cfg::ROWS;
      for (int ks = 0; ks < ksteps; ++ks, ++g) {
        const int slot = static_cast<int>(g % D);
        const uint32_t parity = static_cast<uint32_t>((g / D) & 1) ^ 1u;
        ok = mbar_wait_bounded(smem_addr(&empty_bar[slot]), parity, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) atomicOr(p.status, kStatusEmptyWaitTimeout);
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t st = ring_base + slot * Cfg::STAGE;
          const uint32_t wfull = smem_addr(&wfull_bar[slot]);
          mbar_arrive_expect_tx(wfull, txw);
          tma_load_2d(st + Cfg::OFF_B, &p.tm_b, n_tile * 128, ks * 4, wfull, pol_stream);
          tma_load_2d(st + Cfg::OFF_M, &p.tm_meta, n_tile * 64, ks * 4, wfull, pol_stream);
          if (GROUPED) tma_load_2d(st + Cfg::OFF_S, &p.tm_s, n_tile * 32, ks, wfull, pol_keep);
          // both CTAs' activation halves count on the even CTA's ready barrier
          const uint32_t ready = smem_addr(&aready_bar[slot]);
          if (rank == 0) mbar_arrive_expect_tx(ready, Cfg::TX_ACT_PAIR);
          tma_load_3d_pair(st + Cfg::OFF_ACT, &p.tm_act, 0, act_row, ks * 2, mapa_shared(ready, 0),
                           pol_keep);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (even CTA)
    if (rank == 0) {
      constexpr uint32_t idesc =
          (1u << 2) | (1u << 4) | (static_cast<uint32_t>(256 >> 3) << 17) | ((256u >> 4) << 24);
      constexpr uint64_t kStageDesc = Cfg::STAGE >> 4;
      constexpr uint64_t kAtomDesc = Cfg::ATOM >> 4;
      const uint64_t ad0 = umma_desc_sw128_k(ring_base + Cfg::OFF_A);
      const uint64_t bd0 = umma_desc_sw128_k(ring_base + Cfg::OFF_ACT);
      const uint32_t ready0 = smem_addr(aready_bar);
      const uint32_t empty0 = smem_addr(empty_bar);
      uint64_t ad = ad0, bd = bd0;
      uint32_t e = tmem_e, slot = 0, parity = 0;
      bool ok = true;
      for (int j = 0; j < my_tiles && ok; ++j) {
        if (j > 0) {
          // the epilogue warps of both CTAs have read the previous tile
          ok = mbar_wait_bounded(smem_addr(acc_empty), static_cast<uint32_t>((j - 1) & 1),
                                 abort_flag);
          if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (int ks = 0; ks < ksteps; ++ks) {
          ok = mbar_wait_bounded(ready0 + 8 * slot, parity, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            umma_sp_f16_pair(tmem, ad, bd, e, idesc, ks ? 1u : 0u);
            umma_sp_f16_pair(tmem, ad + 2, bd + 4, e + 4, idesc, 1u);
            umma_sp_f16_pair(tmem, ad + 4, bd + kAtomDesc, e + 8, idesc, 1u);
            umma_sp_f16_pair(tmem, ad + 6, bd + kAtomDesc + 4, e + 12, idesc, 1u);
            umma_commit_pair(empty0 + 8 * slot);
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
        // the tile's accumulator is complete once its MMAs are
        if (ok && lane == 0) umma_commit_pair(smem_addr(acc_full));
        __syncwarp();
      }
    }
  } else if (warp < Cfg::EPI_WARP0) {
    // ---------------------------------------------------------- dequantise
    // (the mask, a no-op here, tells the compiler the step index is never
    // negative; without it the kernel needs more registers)
    const int dw = static_cast<int>(static_cast<uint32_t>(warp - Cfg::DQ_WARP0) & (4u * NG - 1u));
    const int grp = dw >> 2;
    const int r = dw & 3;
    const int quarter = warp & 3;
    const int g8 = lane >> 2, t = lane & 3;
    const uint32_t m_word = (quarter >> 1) * 256 +
                            4 * (32 * (quarter & 1) + 4 * (lane & 7) + 2 * (lane >> 4) + ((lane >> 3) & 1));
    const uint32_t e_lane = tmem_e + (static_cast<uint32_t>(32 * quarter) << 16);
    const uint32_t ready_own = smem_addr(aready_bar);
    for (long long g = grp; g < total_steps; g += NG) {
      const int slot = static_cast<int>(g % D);
      const uint32_t parity = static_cast<uint32_t>((g / D) & 1);
      if (!mbar_wait_bounded(smem_addr(&wfull_bar[slot]), parity, abort_flag)) {
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
        break;
      }
      const uint32_t st = ring_base + slot * Cfg::STAGE;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tmem_st32(e_lane + slot * Cfg::META_COLS + 4 * kk, lds32(st + Cfg::OFF_M + kk * 512 + m_word));
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const uint4 q = lds128(st + Cfg::OFF_B + r * 1024 + cc * 512 + lane * 16);
        uint4 sv = make_uint4(0, 0, 0, 0);
        if (GROUPED) sv = lds128(st + Cfg::OFF_S + cc * 128 + g8 * 16);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          half2 lo0, hi0, lo1, hi1;
          dequant_pair(qw[jj], lo0, hi0);
          dequant_pair(qw[jj] >> 8, lo1, hi1);
          if (GROUPED) {
            const half2 s2 = *reinterpret_cast<const half2*>(&sw[jj]);
            const half2 sx = __low2half2(s2), sy = __high2half2(s2);
            lo0 = __hmul2(lo0, sx);
            hi0 = __hmul2(hi0, sx);
            lo1 = __hmul2(lo1, sy);
            hi1 = __hmul2(hi1, sy);
          }
          // same row order and 128-byte swizzle as the one-tile pair kernel
          const int m_lo = g8 + 16 * (4 * cc + jj);
          const uint32_t row_lo = st + Cfg::OFF_A + m_lo * 128;
          const uint32_t row_hi = row_lo + 8 * 128;
          const uint32_t ca = ((2 * r) ^ g8) << 4, cb = ((2 * r + 1) ^ g8) << 4;
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
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - Cfg::EPI_WARP0;   // 0 .. EPI_WARPS-1
    const int quarter = warp & 3;
    const int blk0 = ew >> 2;               // column blocks blk0, blk0 + EPI_WARPS / 4, ...
    const int rr = 32 * quarter + lane;
    const int m2 = rr >> 4;
    const int feat = 64 * (m2 >> 2) + 8 * (rr & 7) + (m2 & 3) + 4 * ((rr >> 3) & 1);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
    const uint32_t acc_empty_own = smem_addr(acc_empty);
    for (int j = 0; j < my_tiles; ++j) {
      if (!mbar_wait_bounded(smem_addr(acc_full), static_cast<uint32_t>(j & 1), abort_flag)) {
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
        break;
      }
      tc_fence_after();
      const int id = cluster + j * clusters;
      const int n = (2 * (id % n_pairs) + static_cast<int>(rank)) * 128 + feat;
      const int m0 = (id / n_pairs) * 256;
      float cs = 1.f;
      if (!GROUPED) cs = __half2float(reinterpret_cast<const half*>(p.s)[n]);
      const float col_bias = EPI && p.bias != nullptr ? __half2float(p.bias[n]) : 0.f;
#pragma unroll 1
      for (int cb2 = blk0; cb2 < Cfg::BN / 32; cb2 += Cfg::EPI_WARPS / 4) {
        uint32_t v[32];
        tmem_ld32(lane_addr + cb2 * 32, v);
        const int b0 = m0 + cb2 * 32;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int b = b0 + jj;
          if (b < p.M) {
            const float x = __uint_as_float(v[jj]) * cs;
            p.C[static_cast<long long>(b) * p.N + n] =
                __float2half_rn(EPI ? epilogue_act(x + col_bias, p.act) : x);
          }
        }
      }
      // this warp's reads of the accumulator are complete (tcgen05.ld waits)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(acc_empty_own);
        else
          mbar_arrive_remote(mapa_shared(acc_empty_own, 0));
      }
    }
  }

  // Teardown: every MMA of the pair has completed (done, bounded) before
  // either CTA releases its shared or tensor memory.
  if (warp == 1 && rank == 0 && lane == 0) umma_commit_pair(smem_addr(done_bar));
  tc_fence_before();
  __syncthreads();
  if (warp == 1) mbar_wait_bounded(smem_addr(done_bar), 0, abort_flag);
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
}

}  // namespace sm100
