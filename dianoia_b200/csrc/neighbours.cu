// RMSNorm, SwiGLU and the residual add, the decode path's neighbours of the
// quantized products, as dianoia's GPU layer encodes them
// (lab_gpu_enc_rms_norm, lab_gpu_enc_swiglu and lab_gpu_enc_add,
// src/vulkan/lab_vulkan.c:899-907, 974-978 and 993-998) but with the
// arithmetic of its CPU path, which the GPU layer's tests hold as the truth:
//
//  * RMSNorm (lib/src/ops.dart:12-31): the sum of squares and
//    r = 1 / sqrt(sum / cols + eps) in double, x * r in double stored to f32,
//    then an f32 product with the weight; with accumulate, an f32 add into the
//    output (the residual add of lib/src/model.dart:946-950). The sum runs in
//    the order of norm_factor (dn_common.cuh), which the GEMV prologue that
//    runs a norm itself shares.
//  * SwiGLU (lib/src/shard.dart:456-460): silu_mul (dn_common.cuh).
//  * the residual add (lib/src/model.dart:946-950): one f32 add per value.
//
// Both kernels can also write their outputs as QA blocks (32 int8 of
// lab_quantize_q8 and their f32 scale), so that the products reading them
// take quantized activations without a quantize of their own: the fused
// norm -> quantize and SwiGLU -> quantize of the decode path. A product whose
// f32 input is quantized by the CTA gets the same bits, so nothing changes
// but the time. Both are HBM-bound: the norm reads its row twice (the second
// time from L1) and writes it once, SwiGLU reads two values and writes one.
#include "dn_common.cuh"
#include "dn_launch.h"
#include "gemv_core.cuh"

namespace dn {
namespace {

constexpr int kNormThreads = kNormLanes;  // 4 warps: the shared summation order
constexpr int kNormWarps = kNormThreads / 32;

// One CTA per row. Warp w handles 32-value blocks w, w + 4, ...: lane j holds
// value j of the block, so its QA block comes out of one warp reduction.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const NormArgs a) {
  pdl_launch_dependents();  // the next product may start streaming weights
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row = blockIdx.x;
  const float* x = a.x + row * a.cols;
  float* out = a.out + row * a.cols;
  __shared__ double red[kNormWarps];
  const double r = norm_factor(x, a.cols, a.eps, tid, red, [] { __syncthreads(); });

  // Blocks in chunks: every load of a chunk is issued before its stores (a
  // store to out could alias the next load, so the compiler would not hoist it).
  constexpr int kChunk = 8;
  const int64_t blocks = a.cols / kBlock;
  for (int64_t b0 = warp; b0 < blocks; b0 += kNormWarps * kChunk) {
    float xv[kChunk], wv[kChunk], ov[kChunk];
#pragma unroll
    for (int u = 0; u < kChunk; u++) {
      const int64_t b = b0 + u * kNormWarps, j = b * kBlock + lane;
      if (b < blocks) {
        xv[u] = x[j];
        wv[u] = a.w[j];
        ov[u] = a.accumulate ? out[j] : 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < kChunk; u++) {
      const int64_t b = b0 + u * kNormWarps, j = b * kBlock + lane;
      if (b < blocks) {  // the same in every lane
        float v = norm_value(xv[u], wv[u], r);
        if (a.accumulate) v = __fadd_rn(ov[u], v);
        out[j] = v;
        if (a.qa != nullptr) gemv::quantize_block_out(v, a.qa + row * a.qa_stride + b * kQABytes, lane);
      }
    }
  }
  // A trailing part block (no QA: the planner links only whole blocks).
  const int64_t j = blocks * kBlock + lane;
  if (warp == kNormWarps - 1 && j < a.cols) {
    float v = norm_value(x[j], a.w[j], r);
    if (a.accumulate) v = __fadd_rn(out[j], v);
    out[j] = v;
  }
}

constexpr int kGluThreads = 256;

// Grid-stride over 32-value blocks, one per warp and lane j on value j.
__global__ void __launch_bounds__(kGluThreads) swiglu_kernel(const SwigluArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kGluThreads / 32);
  const int64_t blocks = (a.count + kBlock - 1) / kBlock;
  for (int64_t b = (int64_t)blockIdx.x * (kGluThreads / 32) + (threadIdx.x >> 5); b < blocks; b += warps) {
    const int64_t j = b * kBlock + lane;
    float h = 0.0f;
    if (j < a.count) {
      h = silu_mul(a.g[j], a.u[j]);
      a.g[j] = h;
    }
    // Whole blocks only; the branch is uniform across the warp.
    if (a.qa != nullptr && (b + 1) * kBlock <= a.count)
      gemv::quantize_block_out(h, a.qa + b * kQABytes, lane);
  }
}

// dst += src (src/vulkan/shaders/add.comp; the CPU's _addInto,
// lib/src/model.dart:946-950): an f32 add per value.
__global__ void __launch_bounds__(kGluThreads) add_kernel(const float* src, float* dst, int64_t count) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * kGluThreads;
  for (int64_t i = (int64_t)blockIdx.x * kGluThreads + threadIdx.x; i < count; i += stride)
    dst[i] = __fadd_rn(dst[i], src[i]);
}

cudaError_t launch_ex(const void* kern, void** args, dim3 grid, int threads, cudaStream_t stream,
                      bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3((unsigned)threads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

}  // namespace

cudaError_t launch_rms_norm(const NormArgs& a, cudaStream_t stream, bool pdl) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.rows > 0x7fffffff) return cudaErrorInvalidValue;
  NormArgs copy = a;
  void* args[] = {&copy};
  return launch_ex(reinterpret_cast<const void*>(rms_norm_kernel), args, dim3((unsigned)a.rows),
                   kNormThreads, stream, pdl);
}

cudaError_t launch_swiglu(const SwigluArgs& a, cudaStream_t stream, bool pdl) {
  if (a.count <= 0) return cudaSuccess;
  const int64_t blocks = (a.count + kBlock - 1) / kBlock;
  const int64_t per_cta = kGluThreads / 32;
  // One block per warp up to 8 CTAs per SM, then grid-stride.
  int64_t grid = (blocks + per_cta - 1) / per_cta;
  if (grid > 148 * 8) grid = 148 * 8;
  SwigluArgs copy = a;
  void* args[] = {&copy};
  return launch_ex(reinterpret_cast<const void*>(swiglu_kernel), args, dim3((unsigned)grid),
                   kGluThreads, stream, pdl);
}

cudaError_t launch_add(const float* src, float* dst, int64_t count, cudaStream_t stream, bool pdl) {
  if (count <= 0) return cudaSuccess;
  int64_t grid = (count + kGluThreads - 1) / kGluThreads;
  if (grid > 148 * 8) grid = 148 * 8;
  void* args[] = {&src, &dst, &count};
  return launch_ex(reinterpret_cast<const void*>(add_kernel), args, dim3((unsigned)grid), kGluThreads,
                   stream, pdl);
}

}  // namespace dn
