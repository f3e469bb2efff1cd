// Launches of the GPU packer (packer.cuh) and the 3-bit metadata codec
// (meta3_codec.cuh); argument checks are done by the C ABI in sm100_marlin.cu.
#include "../../include/sm100_marlin.h"
#include "launch.cuh"
#include "meta3_codec.cuh"
#include "packer.cuh"

namespace sm100 {

namespace {
int last_launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SM100_MARLIN_OK : cuda_fail(e);
}

// grid-stride kernels: enough blocks to fill the GPU, no more
int grid_for(long long items, int threads) {
  const long long b = (items + threads - 1) / threads;
  return static_cast<int>(b < 148 * 16 ? b : 148 * 16);
}
}  // namespace

int launch_pack_2_4(const void* w, const void* s, int prob_k, int prob_m, int groupsize, void* B,
                    void* meta, void* s_out, cudaStream_t stream) {
  const int g_rows = groupsize == -1 ? prob_k : groupsize;
  const int s_rows = prob_k / g_rows;
  const long long b_words = static_cast<long long>(prob_k / 32) * 2 * prob_m;
  const long long meta_words = static_cast<long long>(prob_m) * (prob_k / 16);
  const long long s_words = static_cast<long long>(s_rows) * prob_m;
  pack_b_kernel<<<grid_for(b_words, 256), 256, 0, stream>>>(
      static_cast<const half*>(w), static_cast<const half*>(s), prob_k, prob_m, g_rows,
      static_cast<uint32_t*>(B));
  pack_meta_kernel<<<grid_for(meta_words, 256), 256, 0, stream>>>(
      static_cast<const half*>(w), static_cast<const half*>(s), prob_k, prob_m, g_rows,
      static_cast<uint16_t*>(meta));
  pack_scales_kernel<<<grid_for(s_words, 256), 256, 0, stream>>>(
      static_cast<const half*>(s), s_rows, prob_m, groupsize != -1 ? 1 : 0,
      static_cast<half*>(s_out));
  return last_launch_status();
}

int launch_meta3_pack(const void* meta, void* out, int64_t pairs, void* err_count,
                      cudaStream_t stream) {
  const int threads = 256;
  const int64_t blocks = (pairs + threads - 1) / threads;
  meta3_pack_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<const uint32_t*>(meta), static_cast<uint32_t*>(out), pairs,
      static_cast<uint32_t*>(err_count));
  return last_launch_status();
}

int launch_meta3_unpack(const void* in, void* out, int64_t lanes, cudaStream_t stream) {
  const int threads = 256;
  const int64_t blocks = (lanes + threads - 1) / threads;
  meta3_unpack_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out), lanes);
  return last_launch_status();
}

int launch_meta3_decode_words(const void* in, void* out_high, void* out_low, int64_t n,
                              cudaStream_t stream) {
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  meta3_decode_words_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out_high),
      static_cast<uint32_t*>(out_low), n);
  return last_launch_status();
}

}  // namespace sm100
