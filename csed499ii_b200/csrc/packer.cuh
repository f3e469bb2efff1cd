// GPU packer: fp16 weight (K, N) + group scales -> Sparse-Marlin 2:4 INT4
// operands (B, meta, permuted s), bit-identical to the reference's
// Layer_2_4.pack(linear, scales, trans=True)
// (kernel_experiments/sparse_marlin/src/marlin/__init__.py:331-388), which
// quantises, builds the 2:4 mask on the biased codes (mask_creator,
// _semi_structured_conversions.py:286-314), compresses with the CUTLASS
// metadata reorder (_semi_structured_conversions.py:21-179), tiles and
// nibble-packs on the CPU.  Here every output word is computed independently
// from the 16 codes it depends on, so each kernel is a single streaming pass.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace sm100 {

// Biased 4-bit code clamp(rint(fp16(w / s)) + 8, 0, 15): the reference divides
// fp16 tensors (fp32 arithmetic, one rounding to fp16) and rounds half to
// even.
__device__ __forceinline__ int quant_code(half w, half s) {
  const half q = __float2half_rn(__half2float(w) / __half2float(s));
  int c = static_cast<int>(rintf(__half2float(q))) + 8;
  return c < 0 ? 0 : (c > 15 ? 15 : c);
}

// Compressed pair (v0, v1) and nibble idx0 | idx1 << 2 of one group of four
// codes: keep the two largest codes (ties: the lower index is dropped first,
// as a stable ascending sort does), then the reference's flag logic
// (_semi_structured_conversions.py:133-141; a kept code of 0 counts as zero).
__device__ __forceinline__ void compress_group(const int (&c)[4], int& v0, int& v1, int& nib) {
  int mv[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    int rank = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) rank += (c[q] < c[p]) || (c[q] == c[p] && q < p);
    mv[p] = rank >= 2 ? c[p] : 0;
  }
  const bool m0 = mv[0] != 0, m1 = mv[1] != 0, m3 = mv[3] != 0;
  const bool e0 = m0 && m1, e1 = !m0 && m1, e2 = !m0 && !m1;
  const int idx0 = (e1 ? 1 : 0) | (e2 ? 2 : 0);
  const int idx1 = ((e0 || e2 || m3) ? 1 : 0) | ((e1 || !m1) ? 2 : 0);
  v0 = mv[idx0];
  v1 = mv[idx1];
  nib = idx0 | (idx1 << 2);
}

// Codes of dense group gk (k = 4gk .. 4gk+3) of out-feature n.
__device__ __forceinline__ void load_group(const half* __restrict__ w, const half* __restrict__ s,
                                           int N, int g_rows, int n, int gk, int (&c)[4]) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int k = 4 * gk + p;
    c[p] = quant_code(w[static_cast<long long>(k) * N + n], s[static_cast<long long>(k / g_rows) * N + n]);
  }
}

// B word (kk, 128cc + 16g + 4t + j): nibble i = 4ib + 2rh + ia holds the
// compressed value ib of dense group 8kk + 4ia + t of out-feature
// 64cc + 8g + j + 4rh.
__global__ void pack_b_kernel(const half* __restrict__ w, const half* __restrict__ s, int K, int N,
                              int g_rows, uint32_t* __restrict__ B) {
  const long long total = static_cast<long long>(K / 32) * 2 * N;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int kk = static_cast<int>(idx / (2 * N));
    const int word = static_cast<int>(idx % (2 * N));
    const int cc = word >> 7, g = (word >> 4) & 7, t = (word >> 2) & 3, j = word & 3;
    uint32_t q = 0;
#pragma unroll
    for (int rh = 0; rh < 2; ++rh)
#pragma unroll
      for (int ia = 0; ia < 2; ++ia) {
        int c[4], v0, v1, nib;
        load_group(w, s, N, g_rows, 64 * cc + 8 * g + j + 4 * rh, 8 * kk + 4 * ia + t, c);
        compress_group(c, v0, v1, nib);
        q |= static_cast<uint32_t>(v0) << (4 * (2 * rh + ia));
        q |= static_cast<uint32_t>(v1) << (4 * (4 + 2 * rh + ia));
      }
    B[idx] = q;
  }
}

// Metadata int16 of (out-feature n, 16-K column col): the nibbles of groups
// 4col .. 4col+3, stored at the CUTLASS interleaved offset
// (_semi_structured_conversions.py:21-48).
__global__ void pack_meta_kernel(const half* __restrict__ w, const half* __restrict__ s, int K,
                                 int N, int g_rows, uint16_t* __restrict__ meta) {
  const int cols = K / 16;
  const long long total = static_cast<long long>(N) * cols;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(idx / cols);
    const int col = static_cast<int>(idx % cols);
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int c[4], v0, v1, nib;
      load_group(w, s, N, g_rows, n, 4 * col + i, c);
      compress_group(c, v0, v1, nib);
      m |= static_cast<uint32_t>(nib) << (4 * i);
    }
    int dr = (n / 64) * 64 + (n % 2) * 2 + (n % 8) / 4 + ((n % 4) / 2) * 32 + ((n % 64) / 8) * 4;
    int dc = col;
    const int tr = (dr % 2 == 0 && dc % 2 == 1) ? 1 : 0;
    const int bl = (dr % 2 == 1 && dc % 2 == 0) ? 1 : 0;
    dr += tr - bl;
    dc -= tr - bl;
    meta[static_cast<long long>(dc / 2) * N * 2 + dr * 2 + dc % 2] = static_cast<uint16_t>(m);
  }
}

// Scales: grouped -> columns permuted inside each 8-column block by
// (0,4,1,5,2,6,3,7) (__init__.py:242-268, 359-365); per-column -> copied.
__global__ void pack_scales_kernel(const half* __restrict__ s, int rows, int N, int grouped,
                                   half* __restrict__ out) {
  const long long total = static_cast<long long>(rows) * N;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(idx & 7);
    const int src = grouped ? ((p & 1) ? 4 + (p >> 1) : (p >> 1)) : p;
    out[idx] = s[(idx & ~7ll) + src];
  }
}

}  // namespace sm100
