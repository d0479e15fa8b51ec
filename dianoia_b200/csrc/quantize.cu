// Activation -> Q8_0 quantization (lab_quantize_q8) and the Q4_0 weight
// quantizer (lab_quantize_q4), as standalone sm_100a kernels.
//
// Each is HBM-bound integer/float byte work: one pass that reads the floats
// once with 16-byte loads and writes the int8 (or nibble) bytes and the block
// scales once. A block of 32 values is handled by 8 (Q8) or 16 (Q4) adjacent
// lanes that combine their partial maxima with warp shuffles.
#include "dn_common.cuh"
#include "dn_launch.h"

namespace dn {
namespace {

constexpr int kQuantThreads = 256;

// lab_quantize_q8 (lab_native.c:407-429). Eight lanes per block, four values
// each; lane `sub` holds values 4*sub .. 4*sub+3 of its block.
__global__ void __launch_bounds__(kQuantThreads)
    quantize_q8_kernel(const float* __restrict__ xs, int8_t* __restrict__ xq,
                       float* __restrict__ xsc, int64_t n, int64_t cols, int64_t blocks,
                       bool vec) {
  // The product after this (a programmatic dependent launch) may start its
  // weight stream now; it waits for this grid's completion before reading
  // the quantized activations.
  pdl_launch_dependents();
  const int64_t gid = (int64_t)blockIdx.x * kQuantThreads + threadIdx.x;
  const int64_t blk = gid >> 3;
  const int sub = (int)(gid & 7);
  const bool active = blk < n * blocks;
  const int64_t t = active ? blk / blocks : 0, b = active ? blk % blocks : 0;
  const float* src = xs + t * cols + b * kBlock + sub * 4;
  float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (active) {
    if (vec) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(src));
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
      for (int i = 0; i < 4; i++) v[i] = __ldg(src + i);
    }
  }
  // amax starts at 0 and NaN never raises it, as the reference's strict '>'.
  float amax = 0.0f;
  for (int i = 0; i < 4; i++) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  float scale, inv;
  q8_scale(amax, scale, inv);
  if (!active) return;
  int32_t q[4];
  for (int i = 0; i < 4; i++) q[i] = quant_q8_elem(v[i], inv);
  int8_t* dst = xq + t * cols + b * kBlock + sub * 4;
  if (vec) {
    *reinterpret_cast<uint32_t*>(dst) = pack4(q[0], q[1], q[2], q[3]);
  } else {
    for (int i = 0; i < 4; i++) dst[i] = (int8_t)q[i];
  }
  if (sub == 0) xsc[t * blocks + b] = scale;
}

// The same quantization into QA blocks (32 int8, then the f32 scale):
// token t's block b at xa + t * xa_stride + 36 * b.
__global__ void __launch_bounds__(kQuantThreads)
    quantize_qa_kernel(const float* __restrict__ xs, uint8_t* __restrict__ xa, int64_t n,
                       int64_t cols, int64_t blocks, int64_t xa_stride, bool vec) {
  // The product after this (a programmatic dependent launch) may start its
  // weight stream now; it waits for this grid's completion before reading
  // the quantized activations.
  pdl_launch_dependents();
  const int64_t gid = (int64_t)blockIdx.x * kQuantThreads + threadIdx.x;
  const int64_t blk = gid >> 3;
  const int sub = (int)(gid & 7);
  const bool active = blk < n * blocks;
  const int64_t t = active ? blk / blocks : 0, b = active ? blk % blocks : 0;
  const float* src = xs + t * cols + b * kBlock + sub * 4;
  float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (active) {
    if (vec) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(src));
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
      for (int i = 0; i < 4; i++) v[i] = __ldg(src + i);
    }
  }
  float amax = 0.0f;
  for (int i = 0; i < 4; i++) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  float scale, inv;
  q8_scale(amax, scale, inv);
  if (!active) return;
  uint8_t* dst = xa + t * xa_stride + b * kQABytes;
  *reinterpret_cast<uint32_t*>(dst + sub * 4) =
      pack4(quant_q8_elem(v[0], inv), quant_q8_elem(v[1], inv), quant_q8_elem(v[2], inv),
            quant_q8_elem(v[3], inv));
  if (sub == 0) *reinterpret_cast<float*>(dst + 32) = scale;
}

// lab_quantize_q4 (lab_native.c:928-955): sixteen lanes per block, lane k
// holds values k and k + 16, which share byte k of the block.
__global__ void __launch_bounds__(kQuantThreads)
    quantize_q4_kernel(const float* __restrict__ w, uint8_t* __restrict__ qs,
                       uint16_t* __restrict__ scales, int64_t rows, int64_t cols,
                       int64_t blocks) {
  const int64_t gid = (int64_t)blockIdx.x * kQuantThreads + threadIdx.x;
  const int64_t blk = gid >> 4;
  const int k = (int)(gid & 15);
  const bool active = blk < rows * blocks;
  const int64_t r = active ? blk / blocks : 0, b = active ? blk % blocks : 0;
  const float* src = w + r * cols + b * kBlock;
  const float x0 = active ? __ldg(src + k) : 0.0f;
  const float x1 = active ? __ldg(src + k + 16) : 0.0f;
  // The first value of largest magnitude (strict '>' in index order): keep
  // (|x|, x, index) and prefer the lower index on ties; |x| = 0 or NaN never
  // qualifies, so an all-zero block keeps max = +0.
  float a = 0.0f, m = 0.0f;
  int idx = 1 << 30;
  const float a0 = fabsf(x0), a1 = fabsf(x1);
  if (a0 > 0.0f) { a = a0; m = x0; idx = k; }
  if (a1 > a) { a = a1; m = x1; idx = k + 16; }
  for (int off = 8; off >= 1; off >>= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, a, off);
    const float om = __shfl_xor_sync(0xffffffffu, m, off);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
    if (oa > a || (oa == a && oi < idx)) { a = oa; m = om; idx = oi; }
  }
  if (!active) return;
  const float d = __fdiv_rn(m, -8.0f);
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  const int8_t lo = (int8_t)trunc_i32_x86(__fadd_rn(__fmul_rn(x0, id), 8.5f));
  const int8_t hi = (int8_t)trunc_i32_x86(__fadd_rn(__fmul_rn(x1, id), 8.5f));
  const int loc = lo > 15 ? 15 : lo, hic = hi > 15 ? 15 : hi;
  qs[(r * cols + b * kBlock) / 2 + k] = (uint8_t)(loc | (hic << 4));
  if (k == 0) scales[r * blocks + b] = __half_as_ushort(__float2half_rn(d));
}

}  // namespace

cudaError_t launch_quantize_q8(const float* xs, int8_t* xq, float* xsc, int64_t n, int64_t cols,
                               cudaStream_t stream) {
  const int64_t blocks = cols / kBlock;
  if (n <= 0 || blocks <= 0) return cudaSuccess;
  const bool vec = cols % 4 == 0 && ((uintptr_t)xs & 15) == 0 && ((uintptr_t)xq & 3) == 0;
  const int64_t threads = n * blocks * 8;
  const int64_t grid = (threads + kQuantThreads - 1) / kQuantThreads;
  quantize_q8_kernel<<<(unsigned)grid, kQuantThreads, 0, stream>>>(xs, xq, xsc, n, cols, blocks,
                                                                   vec);
  return cudaGetLastError();
}

cudaError_t launch_quantize_qa(const float* xs, uint8_t* xa, int64_t n, int64_t cols,
                               int64_t xa_stride, cudaStream_t stream) {
  const int64_t blocks = cols / kBlock;
  if (n <= 0 || blocks <= 0) return cudaSuccess;
  const bool vec = cols % 4 == 0 && ((uintptr_t)xs & 15) == 0;
  const int64_t grid = (n * blocks * 8 + kQuantThreads - 1) / kQuantThreads;
  quantize_qa_kernel<<<(unsigned)grid, kQuantThreads, 0, stream>>>(xs, xa, n, cols, blocks,
                                                                   xa_stride, vec);
  return cudaGetLastError();
}

cudaError_t launch_quantize_q4(const float* w, uint8_t* qs, uint16_t* scales, int64_t rows,
                               int64_t cols, cudaStream_t stream) {
  const int64_t blocks = cols / kBlock;
  if (rows <= 0 || blocks <= 0) return cudaSuccess;
  const int64_t threads = rows * blocks * 16;
  const int64_t grid = (threads + kQuantThreads - 1) / kQuantThreads;
  quantize_q4_kernel<<<(unsigned)grid, kQuantThreads, 0, stream>>>(w, qs, scales, rows, cols,
                                                                   blocks);
  return cudaGetLastError();
}

}  // namespace dn
