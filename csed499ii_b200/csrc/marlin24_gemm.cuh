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
//  * Work = column tiles of 64*NC out-features x K.  The (tile, kk) "units"
//    (kk = 32 dense K) are laid out tile-major and split evenly over a
//    persistent grid of one CTA per SM, so every SM streams the same number
//    of weight bytes whatever the shape (stream-K style split).
//  * One producer warp streams B rows, metadata rows, scale rows and the
//    activation slice of each stage with cp.async.bulk into a deep
//    shared-memory ring (mbarrier full/empty pairs, evict-first L2 policy for
//    the weight stream).  Every wait is bounded (%globaltimer) and records a
//    status bit instead of hanging.
//  * Eight consumer warps each own one (kk, 64-column chunk) block per stage:
//    one 16-byte B load, the metadata words (ldmatrix.x2 for 4-bit, two
//    32-bit loads + lop3 decode for 3-bit), INT4 -> fp16 magic-number dequant
//    with the group scale fused, and mma.sp m16n8k32 with fp32 accumulators.
//  * Split-K partials are reduced in fp32: warps of a CTA through shared
//    memory, CTAs of a tile through a scratch buffer and a per-tile ticket in
//    the caller's workspace; the last CTA to arrive sums all partials in CTA
//    order (deterministic, no CTA ever waits for another) and writes C.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "device_primitives.cuh"

namespace sm100 {

struct GemmParams {
  const uint8_t* A;     // fp16 (M, K) row-major, this launch's rows
  const uint8_t* B;     // int32 (K/32, 2N)
  const uint8_t* meta;  // K/32 rows of 4N bytes (4-bit) or 3N bytes (3-bit)
  const uint8_t* s;     // fp16 (K/128, N) permuted, or (1, N)
  half* C;              // fp16 (M, N) row-major
  float4* partials;     // split-K scratch
  int* counters;        // one int per column tile; zero on entry and on exit
  int* status;          // device status word (timeouts)
  int M;                // rows in this launch, 1..64
  int N;
  int K;
  int grouped;          // 1: group of 128 dense K; 0: one scale per column
  int n_tiles;          // N / (64*NC)
  int kk_total;         // K / 32
  long long units;      // n_tiles * kk_total / 2   (a unit = 2 kk rows)
};

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSmemBudget = 200 * 1024;

template <int NC, int MB, bool META3>
struct DecodeCfg {
  static constexpr int SK = kConsumerWarps / NC;                 // kk rows per stage
  static constexpr int B_ROW = 512 * NC;                         // bytes of B per kk row
  static constexpr int M_BLK = META3 ? 192 : 256;                // meta bytes per (kk, chunk)
  static constexpr int M_ROW = M_BLK * NC;
  static constexpr int S_ROW = 128 * NC;                         // scale bytes per group row
  static constexpr int S_ROWS = SK == 2 ? 1 : (SK == 4 ? 2 : 3); // groups a stage can touch
  static constexpr int A_STRIDE = SK * 64 + 16;                  // padded activation row
  static constexpr int OFF_B = 0;
  static constexpr int OFF_M = OFF_B + SK * B_ROW;
  static constexpr int OFF_S = OFF_M + SK * M_ROW;
  static constexpr int OFF_A = OFF_S + S_ROWS * S_ROW;
  static constexpr int STAGE_RAW = OFF_A + 16 * MB * A_STRIDE;
  static constexpr int STAGE = (STAGE_RAW + 127) / 128 * 128;
  static constexpr int ACC_F4 = 8 * MB;                          // float4 per thread of acc
  static constexpr int RED_BYTES = NC * ACC_F4 * 32 * 16;        // one slot per chunk
  static constexpr int HEADER = 1024;                            // barriers + flags
  static constexpr int DEPTH_FIT = (kSmemBudget - HEADER - RED_BYTES) / STAGE;
  static constexpr int DEPTH = DEPTH_FIT > 16 ? 16 : DEPTH_FIT;
  static constexpr int SMEM = HEADER + RED_BYTES + DEPTH * STAGE;
  static_assert(DEPTH >= 4, "ring too shallow");
};

// Unit range of CTA c in a split of `units` over `grid` CTAs.
__device__ __forceinline__ long long unit_begin(long long c, long long units, long long grid) {
  return (c * units) / grid;
}
// CTA owning unit u (the largest c with unit_begin(c) <= u).
__device__ __forceinline__ long long unit_owner(long long u, long long units, long long grid) {
  return ((u + 1) * grid - 1) / units;
}

template <int NC, int MB, int NH_LAST, bool META3>
__global__ void __maxnreg__(224)
    marlin24_decode_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = DecodeCfg<NC, MB, META3>;
  constexpr int SK = Cfg::SK;
  constexpr int D = Cfg::DEPTH;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty_bar = full_bar + D;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 512);
  volatile int* ticket_sh = reinterpret_cast<volatile int*>(smem + 516);
  uint8_t* red = smem + Cfg::HEADER;
  uint8_t* ring = red + Cfg::RED_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < D; ++i) {
      mbar_init(smem_addr(&full_bar[i]), 1);
      mbar_init(smem_addr(&empty_bar[i]), kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const long long grid = gridDim.x;
  const long long cta = blockIdx.x;
  const long long u_begin = unit_begin(cta, p.units, grid);
  const long long u_end = unit_begin(cta + 1, p.units, grid);
  const int units_per_tile = p.kk_total >> 1;
  const uint32_t ring_base = smem_addr(ring);

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------ producer
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const long long b_row_stride = 8ll * p.N;                     // bytes per kk row of B
    const long long m_row_stride = (META3 ? 3ll : 4ll) * p.N;      // bytes per kk row of meta
    const long long s_row_stride = 2ll * p.N;
    const long long a_row_stride = 2ll * p.K;
    uint32_t stage = 0;
    bool ok = true;
    for (long long u = u_begin; u < u_end && ok;) {
      const int tile = static_cast<int>(u / units_per_tile);
      const int ub = static_cast<int>(u % units_per_tile);
      const long long ue_ll = ub + (u_end - u);
      const int ue = ue_ll < units_per_tile ? static_cast<int>(ue_ll) : units_per_tile;
      u += ue - ub;
      const int kb = 2 * ub, ke = 2 * ue;
      for (int kk0 = kb; kk0 < ke; kk0 += SK, ++stage) {
        const int rows = min(SK, ke - kk0);
        const int slot = stage % D;
        const uint32_t parity = ((stage / D) & 1u) ^ 1u;
        if (!mbar_wait_bounded(smem_addr(&empty_bar[slot]), parity, abort_flag)) {
          if (lane == 0) atomicOr(p.status, kStatusEmptyWaitTimeout);
          ok = false;
          break;
        }
        const int g_lo = kk0 >> 2, g_hi = (kk0 + rows - 1) >> 2;
        const int n_srows = p.grouped ? (g_hi - g_lo + 1) : 0;
        const uint32_t bytes = rows * (Cfg::B_ROW + Cfg::M_ROW) + n_srows * Cfg::S_ROW +
                               p.M * rows * 64;
        const uint32_t full = smem_addr(&full_bar[slot]);
        if (lane == 0) mbar_arrive_expect_tx(full, bytes);
        __syncwarp();
        const uint32_t st = ring_base + slot * Cfg::STAGE;
        const long long col_b = static_cast<long long>(tile) * Cfg::B_ROW;
        const long long col_m = static_cast<long long>(tile) * Cfg::M_ROW;
        if (lane < rows) {
          bulk_g2s(st + Cfg::OFF_B + lane * Cfg::B_ROW,
                   p.B + (kk0 + lane) * b_row_stride + col_b, Cfg::B_ROW, full, pol_stream);
        } else if (lane >= 8 && lane < 8 + rows) {
          const int r = lane - 8;
          bulk_g2s(st + Cfg::OFF_M + r * Cfg::M_ROW, p.meta + (kk0 + r) * m_row_stride + col_m,
                   Cfg::M_ROW, full, pol_stream);
        } else if (lane >= 16 && lane < 16 + n_srows) {
          const int r = lane - 16;
          bulk_g2s(st + Cfg::OFF_S + r * Cfg::S_ROW,
                   p.s + (g_lo + r) * s_row_stride + static_cast<long long>(tile) * Cfg::S_ROW,
                   Cfg::S_ROW, full, pol_keep);
        }
        for (int m = lane; m < p.M; m += 32) {
          bulk_g2s(st + Cfg::OFF_A + m * Cfg::A_STRIDE, p.A + m * a_row_stride + kk0 * 64,
                   rows * 64, full, pol_keep);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cc = warp % NC;  // 64-column chunk inside the tile
  const int kl = warp / NC;  // kk row inside a stage
  const int g = lane >> 2;
  const int t = lane & 3;
  float acc[MB][4][2][4];
  uint32_t stage = 0;
  bool aborted = false;

  for (long long u = u_begin; u < u_end;) {
    const int tile = static_cast<int>(u / units_per_tile);
    const int ub = static_cast<int>(u % units_per_tile);
    const long long ue_ll = ub + (u_end - u);
      const int ue = ue_ll < units_per_tile ? static_cast<int>(ue_ll) : units_per_tile;
    const bool first_seg = (u == u_begin);
    u += ue - ub;
    const bool last_seg = (u == u_end);
    const int kb = 2 * ub, ke = 2 * ue;

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
      if (!aborted && !mbar_wait_bounded(smem_addr(&full_bar[slot]), parity, abort_flag)) {
        aborted = true;
        if (lane == 0) atomicOr(p.status, kStatusFullWaitTimeout);
      }
      if (!aborted && kl < rows) {
        const uint32_t st = ring_base + slot * Cfg::STAGE;
        const uint4 q = lds128(st + Cfg::OFF_B + kl * Cfg::B_ROW + cc * 512 + lane * 16);
        uint32_t mw[2];
        if constexpr (META3) {
          const uint32_t mbase = st + Cfg::OFF_M + kl * Cfg::M_ROW + cc * Cfg::M_BLK;
          const uint32_t a = lds32(mbase + lane * 4);
          const uint32_t b = lds32(mbase + (16 + lane) * 4);
          meta3_pair_decode(a, b, (lane & 16) != 0, mw[0], mw[1]);
        } else {
          ldmatrix_x2(mw, st + Cfg::OFF_M + kl * Cfg::M_ROW + cc * Cfg::M_BLK + (lane & 15) * 16);
        }
        uint4 sv = make_uint4(0, 0, 0, 0);
        if (p.grouped) {
          const int srow = ((kk0 + kl) >> 2) - (kk0 >> 2);
          sv = lds128(st + Cfg::OFF_S + srow * Cfg::S_ROW + cc * 128 + g * 16);
        }
        uint32_t bf[MB][2][4];
#pragma unroll
        for (int mb = 0; mb < MB; ++mb) {
          uint32_t r0[4], r1[4];
          const uint32_t aaddr =
              st + Cfg::OFF_A + (16 * mb + (lane & 15)) * Cfg::A_STRIDE + kl * 64 + (lane >> 4) * 16;
          ldmatrix_x4(r0, aaddr);
          ldmatrix_x4(r1, aaddr + 32);
          bf[mb][0][0] = r0[0]; bf[mb][0][1] = r0[2]; bf[mb][0][2] = r1[0]; bf[mb][0][3] = r1[2];
          bf[mb][1][0] = r0[1]; bf[mb][1][1] = r0[3]; bf[mb][1][2] = r1[1]; bf[mb][1][3] = r1[3];
        }
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          half2 lo0, hi0, lo1, hi1;
          dequant_pair(qw[j], lo0, hi0);
          dequant_pair(qw[j] >> 8, lo1, hi1);
          if (p.grouped) {
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
              if (j & 1)
                mma_sp_16832<1>(acc[mb][j][h], af, bf[mb][h][0], bf[mb][h][1], bf[mb][h][2],
                                bf[mb][h][3], e);
              else
                mma_sp_16832<0>(acc[mb][j][h], af, bf[mb][h][0], bf[mb][h][1], bf[mb][h][2],
                                bf[mb][h][3], e);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&empty_bar[slot]));
    }

    // ---------------------------------------------------------------- epilogue
    // 1) reduce the SK warps of each chunk through shared memory, one kl at a
    //    time in increasing order (deterministic summation order).
    float4* acc4 = reinterpret_cast<float4*>(&acc[0][0][0][0]);
    float4* red4 = reinterpret_cast<float4*>(red) + cc * Cfg::ACC_F4 * 32;
    for (int k2 = 1; k2 < SK; ++k2) {
      if (kl == k2) {
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) red4[v * 32 + lane] = acc4[v];
      }
      named_bar_sync(1, kConsumerWarps * 32);
      if (kl == 0) {
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) {
          const float4 x = red4[v * 32 + lane];
          acc4[v].x += x.x; acc4[v].y += x.y; acc4[v].z += x.z; acc4[v].w += x.w;
        }
      }
      named_bar_sync(1, kConsumerWarps * 32);
    }
    if (kl != 0) continue;

    // 2) leaders (one warp per chunk) finish the tile.
    const bool complete = (kb == 0 && ke == p.kk_total);
    bool write = complete;
    if (!complete) {
      const long long my_slot = 2 * cta + ((first_seg) ? 0 : 1);
      (void)last_seg;
      float4* part = p.partials + ((my_slot * NC + cc) * Cfg::ACC_F4) * 32;
#pragma unroll
      for (int v = 0; v < Cfg::ACC_F4; ++v) part[v * 32 + lane] = acc4[v];
      __threadfence();
      named_bar_sync(2, NC * 32);
      if (warp == 0 && lane == 0) {
        const long long t0 = static_cast<long long>(tile) * units_per_tile;
        const long long c_lo = unit_owner(t0, p.units, grid);
        const long long c_hi = unit_owner(t0 + units_per_tile - 1, p.units, grid);
        const int n_part = static_cast<int>(c_hi - c_lo + 1);
        const int prev = atomicAdd(&p.counters[tile], 1);
        *ticket_sh = (prev == n_part - 1) ? 1 : 0;
      }
      named_bar_sync(2, NC * 32);
      write = (*ticket_sh != 0);
      if (write) {
        __threadfence();
        const long long t0 = static_cast<long long>(tile) * units_per_tile;
        const long long c_lo = unit_owner(t0, p.units, grid);
        const long long c_hi = unit_owner(t0 + units_per_tile - 1, p.units, grid);
        float4 sum[Cfg::ACC_F4];
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) sum[v] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (long long c = c_lo; c <= c_hi; ++c) {
          const bool started_here = unit_begin(c, p.units, grid) >= t0;
          const long long slot = 2 * c + (started_here ? 0 : 1);
          const float4* src = p.partials + ((slot * NC + cc) * Cfg::ACC_F4) * 32;
#pragma unroll
          for (int v = 0; v < Cfg::ACC_F4; ++v) {
            const float4 x = (c == cta) ? acc4[v] : __ldcg(&src[v * 32 + lane]);
            sum[v].x += x.x; sum[v].y += x.y; sum[v].z += x.z; sum[v].w += x.w;
          }
        }
#pragma unroll
        for (int v = 0; v < Cfg::ACC_F4; ++v) acc4[v] = sum[v];
        if (warp == 0 && lane == 0) p.counters[tile] = 0;
      }
    }
    if (write) {
      // 3) fp32 -> fp16, per-column scale when not grouped, 16-byte stores.
      const int n0 = (tile * NC + cc) * 64 + 8 * g;
      float colscale[8];
      if (!p.grouped) {
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
            if (!p.grouped) {
#pragma unroll
              for (int i = 0; i < 8; ++i) v[i] *= colscale[i];
            }
            uint4 o;
            half2* oh = reinterpret_cast<half2*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            *reinterpret_cast<uint4*>(p.C + static_cast<long long>(r) * p.N + n0) = o;
          }
    }
  }
}

}  // namespace sm100
