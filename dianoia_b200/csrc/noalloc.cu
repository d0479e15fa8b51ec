// dn_linear_noalloc: dn_linear (mode 1, automatic path) without any memory
// allocation by this library, for callers that cannot allocate: an engine
// that reserves all of its device memory up front and must not see it grow,
// or a code path that may not call cudaMalloc and friends.
//
// The tensor-core path needs scratch for the quantized activations (n * cols
// int8 and their f32 block scales) and every kernel needs a word to record a
// bounded wait that ran out. dn_linear takes the scratch from the caller and
// the status word from per-device pinned memory that it allocates on first
// use; here both live in one file-scope __device__ array, created with the
// module, whose address is looked up once per device.
#include <mutex>

#include "dianoia_b200.h"
#include "dn_common.cuh"
#include "dn_launch.h"

namespace {

constexpr int64_t kStatusBytes = 256;                     // the status word, padded
constexpr int64_t kMaxActs = int64_t(8) << 20;            // n * cols quantized activations
constexpr int64_t kScaleBytes = kMaxActs / dn::kBlock * 4;  // their f32 block scales

// [status word | xq: kMaxActs int8 | xsc: kMaxActs / 32 f32]. Device globals
// without an initializer start at zero, which is what the status word needs;
// xq and xsc are written by the activation quantize before anything reads
// them, so their contents never matter.
__device__ __align__(256) uint8_t g_scratch[kStatusBytes + kMaxActs + kScaleBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint8_t* g_base[kMaxDevices] = {};

// g_scratch's device address on the current device (looked up on the first
// call for each device).
uint8_t* scratch_base() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_base[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return nullptr;
    }
    g_base[dev] = static_cast<uint8_t*>(p);
  }
  return g_base[dev];
}

}  // namespace

extern "C" int64_t dn_linear_noalloc(int64_t format, const void* qs, const void* scales,
                                     const float* xs, float* ys, int64_t rows, int64_t cols,
                                     int64_t n, int64_t ldy, int64_t flags, void* stream) {
  if (format != DN_Q8 && format != DN_Q4) return DN_ERR_ARGS;
  if (rows < 0 || cols < 0 || n < 0 || ldy < rows) return DN_ERR_ARGS;
  if (n > 0 && cols > kMaxActs / n) return DN_ERR_TOO_LARGE;
  uint8_t* base = scratch_base();
  if (base == nullptr) return DN_ERR_NO_DEVICE;
  int8_t* xq = reinterpret_cast<int8_t*>(base + kStatusBytes);
  float* xsc = reinterpret_cast<float*>(base + kStatusBytes + kMaxActs);
  uint32_t* status = reinterpret_cast<uint32_t*>(base);
  const dn::LinearArgs a{format == DN_Q4, qs, scales, xs, xq, xsc, ys, rows, cols, n, ldy, 1, status};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((flags & DN_FLAG_PDL) && dn::path_for(a) == 0) return dn::launch_gemv(a, st, true);
  return dn::launch_linear(a, st);
}

extern "C" int64_t dn_linear_noalloc_status(int64_t clear) {
  uint8_t* base = scratch_base();
  if (base == nullptr) return DN_ERR_NO_DEVICE;
  uint32_t v = 0;
  if (cudaMemcpy(&v, base, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return DN_ERR_CUDA;
  }
  if (clear && v != 0 && cudaMemset(base, 0, sizeof v) != cudaSuccess) {
    cudaGetLastError();
    return DN_ERR_CUDA;
  }
  return (int64_t)v;
}
