// 3-bit 2:4 metadata codec kernels (sm_100a).
//
// Format (kernel_experiments/sparse_marlin/metadata_decode/codec.cu:7-29):
// the metadata is processed in blocks of 64 32-bit words (one warp's 256-byte
// share of a 32-deep K slice of a 64-column chunk).  Each word is 8 nibbles,
// each nibble one of the six legal 2:4 patterns, so it fits in 3 bits.  Lane
// pair p (0..15) of a block packs words p and p+32 into the 48-bit value
// `first` and words p+16 and p+48 into `second` (first word of each pair with
// the "high" code table, second with the "low" one) and stores them in three
// planes of 16 words: X = first[0:32], Y = first[32:48] | second[0:16] << 16,
// Z = second[16:48].  A block shrinks from 256 to 192 bytes.
#pragma once

#include <stdint.h>

#include "device_primitives.cuh"

namespace sm100 {

// nibble -> 3-bit code; 8 marks an illegal nibble.
__constant__ uint8_t c_enc_high[16] = {8, 8, 8, 8, 5, 8, 8, 8, 2, 6, 8, 8, 7, 1, 0, 8};
__constant__ uint8_t c_enc_low[16] = {8, 8, 8, 8, 6, 8, 8, 8, 4, 5, 8, 8, 0, 1, 2, 8};

__device__ __forceinline__ uint32_t encode_word(uint32_t w, const uint8_t* table, uint32_t& bad) {
  uint32_t out = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t c = table[(w >> (4 * i)) & 15u];
    if (c == 8u) {
      ++bad;
      c = 0;
    }
    out |= c << (3 * i);
  }
  return out;
}

__global__ void meta3_pack_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                  int64_t pairs, uint32_t* err_count) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= pairs) return;
  const int64_t blk = idx >> 4;
  const int p = static_cast<int>(idx & 15);
  const uint32_t* w = in + blk * 64;
  uint32_t bad = 0;
  const uint64_t first = encode_word(w[p], c_enc_high, bad) |
                         (static_cast<uint64_t>(encode_word(w[p + 32], c_enc_low, bad)) << 24);
  const uint64_t second = encode_word(w[p + 16], c_enc_high, bad) |
                          (static_cast<uint64_t>(encode_word(w[p + 48], c_enc_low, bad)) << 24);
  uint32_t* o = out + blk * 48;
  o[p] = static_cast<uint32_t>(first);
  o[16 + p] = static_cast<uint32_t>(first >> 32) | (static_cast<uint32_t>(second) << 16);
  o[32 + p] = static_cast<uint32_t>(second >> 16);
  if (bad) atomicAdd(err_count, bad);
}

__global__ void meta3_unpack_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                    int64_t lanes) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= lanes) return;
  const int64_t blk = idx >> 5;
  const int lane = static_cast<int>(idx & 31);
  const uint32_t a = in[blk * 48 + lane];
  const uint32_t b = in[blk * 48 + 16 + lane];
  uint32_t w0, w1;
  meta3_pair_decode(a, b, (lane & 16) != 0, w0, w1);
  out[blk * 64 + lane] = w0;
  out[blk * 64 + 32 + lane] = w1;
}

__global__ void meta3_decode_words_kernel(const uint32_t* __restrict__ in,
                                          uint32_t* __restrict__ out_high,
                                          uint32_t* __restrict__ out_low, int64_t n) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n) return;
  const uint32_t x = in[idx];
  out_high[idx] = decode24_high(x);
  out_low[idx] = decode24_low(x);
}

}  // namespace sm100
