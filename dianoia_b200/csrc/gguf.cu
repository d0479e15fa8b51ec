// GGUF Q4_0 / Q8_0 blocks split on the device into the engine's layout:
// dianoia's loader does this on the CPU (gguf.dart:206-215 splitQ4_0,
// gguf.dart:269-283 splitQ8_0), a byte loop over the whole matrix.
//
// GGUF stores each 32-value block interleaved: a little-endian fp16 scale,
// then the values (Q4_0: 16 nibble bytes, low nibble = value k, high =
// value k + 16; Q8_0: 32 int8). The engine keeps them in two arrays: the
// values block after block, and the scales (Q4_0: the fp16 bytes as they
// are; Q8_0: widened to f32, which is exact). A block starts 2-byte aligned
// (18 or 34 bytes apart), so each thread assembles 32-bit words of values
// from 16-bit loads and stores them 4-byte aligned; the scales go one per
// thread. Bit-exact by construction: nothing is computed but the widening.
#include "dn_common.cuh"
#include "dn_launch.h"

namespace dn {
namespace {

constexpr int kSplitThreads = 256;

// Word w (of kWords) of block b's values, and block b's scale.
template <bool Q4>
__global__ void __launch_bounds__(kSplitThreads)
    gguf_split_kernel(const uint16_t* __restrict__ blocks, int64_t count, uint32_t* __restrict__ qs,
                      void* __restrict__ scales) {
  constexpr int kBlockHalves = Q4 ? 9 : 17;  // 18 / 34 bytes
  constexpr int kWords = Q4 ? 4 : 8;         // 16 / 32 value bytes
  const int64_t i = (int64_t)blockIdx.x * kSplitThreads + threadIdx.x;
  if (i < count * kWords) {
    const int64_t b = i / kWords;
    const int w = (int)(i % kWords);
    const uint16_t* src = blocks + b * kBlockHalves + 1 + 2 * w;  // past the scale
    qs[i] = (uint32_t)__ldg(src) | ((uint32_t)__ldg(src + 1) << 16);
  }
  if (i < count) {
    const uint16_t h = __ldg(blocks + i * kBlockHalves);
    if (Q4)
      static_cast<uint16_t*>(scales)[i] = h;
    else
      static_cast<float*>(scales)[i] = half_bits_to_float(h);
  }
}

}  // namespace

cudaError_t launch_gguf_split(bool q4, const void* blocks, int64_t count, void* qs, void* scales,
                              cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  const int64_t threads = count * (q4 ? 4 : 8);
  const unsigned grid = (unsigned)((threads + kSplitThreads - 1) / kSplitThreads);
  if (q4)
    gguf_split_kernel<true><<<grid, kSplitThreads, 0, stream>>>(
        static_cast<const uint16_t*>(blocks), count, static_cast<uint32_t*>(qs), scales);
  else
    gguf_split_kernel<false><<<grid, kSplitThreads, 0, stream>>>(
        static_cast<const uint16_t*>(blocks), count, static_cast<uint32_t*>(qs), scales);
  return cudaGetLastError();
}

}  // namespace dn
