// The rest of the decode layer that dianoia's GPU layer encodes around the
// quantized products (src/vulkan/lab_vulkan.c:916-1016): the per-head
// RMSNorm + RoPE of q and k, causal grouped-query attention over the KV
// cache, the gated short convolution of LFM2-style layers, copies and the
// control vector. Each follows the arithmetic of dianoia's CPU path, which
// computes in double where Dart's doubles do and stores to f32 where it
// stores into a Float32List:
//
//  * head norm + RoPE: rmsNorm per head (lib/src/ops.dart:12-31, the shared
//    norm_factor order) then Rope.apply (ops.dart:62-71): x1 * cos - x2 * sin
//    as a double difference of exact products, stored to f32;
//  * attention (lib/src/shard.dart:589-628): q.k and the scores in double,
//    exp in double, the softmax sum and the value sums in double, the output
//    acc / sum stored to f32 and, gated, times the double sigmoid of the gate;
//  * conv (shard.dart:476-516): z = B * X in f32, the causal depthwise sum in
//    double over the kernel taps in order, y = C * acc stored to f32;
//  * steer (lib/src/control_vector.dart:176-203): add in f32, or the double
//    dot with the direction and x - scale * dot * v in double, stored to f32.
//
// Sums the CPU runs left to right are trees here where the work is spread
// over threads (the head norm's and the steer's dot, attention's q.k and its
// max / sum): every term is exact or a double, so they differ from the CPU's
// by a few double ulps and move an f32 output only within that of a rounding
// boundary. The attention's value sums run in the CPU's key order within a
// slice of the keys, and the slices add in order.
#include <cooperative_groups.h>

#include "dn_common.cuh"
#include "dn_launch.h"

namespace dn {
namespace {

// ------------------------------------------------------------------- copy

__global__ void __launch_bounds__(256) copy_kernel(const float* src, float* dst, int64_t count) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * 256;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < count; i += stride) dst[i] = src[i];
}

// -------------------------------------------------------------- head norm

// One CTA of 128 threads per (head, token); thread j holds dimensions j and
// j + hd / 2 of the head (hd <= 256, even).
// With a second set of heads, CTAs heads .. heads + heads2 - 1 take those.
__global__ void __launch_bounds__(kNormLanes) head_norm_rope_kernel(const HeadNormRopeArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const bool second = blockIdx.x >= a.heads;
  const int head = second ? blockIdx.x - (int)a.heads : blockIdx.x;
  const int64_t t = blockIdx.y;
  const int tid = threadIdx.x, pair = (int)(a.hd / 2);
  float* x = second ? a.x2 + t * a.x2_stride + (int64_t)head * a.hd : a.x + t * a.x_stride + (int64_t)head * a.hd;
  const float* w = second ? a.w2 : a.w;
  const float* tab = a.rope + t * a.rope_stride;
  __shared__ double red[kNormLanes / 32];
  const double r = norm_factor(x, a.hd, a.eps, tid, red, [] { __syncthreads(); });
  if (tid < pair) {
    const float n1 = norm_value(x[tid], w[tid], r);
    const float n2 = norm_value(x[tid + pair], w[tid + pair], r);
    const double c = (double)tab[tid], s = (double)tab[pair + tid];
    x[tid] = __double2float_rn(__dsub_rn(__dmul_rn((double)n1, c), __dmul_rn((double)n2, s)));
    x[tid + pair] = __double2float_rn(__dadd_rn(__dmul_rn((double)n2, c), __dmul_rn((double)n1, s)));
  }
}

// -------------------------------------------------------------- attention

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// A cluster of kAttnSplit CTAs per (head, token), each owning a contiguous
// slice of the keys, so that decode attention runs on many SMs:
//  1. each CTA scores its keys (a warp per key, lanes across head_dim) into
//     shared memory and takes their max; the cluster's max comes from every
//     CTA's through distributed shared memory;
//  2. each CTA turns its scores into exp(score - max) and sums them, and sums
//     score * value over its keys, each thread four dimensions of a part of
//     the keys in order (eight keys' loads issued together);
//  3. CTA 0 adds the slices' sums in rank order and writes the outputs.
// The arithmetic is the CPU's (the same exp(score - max) of every key); only
// the sums are split, by warps and by slices.
constexpr int kAttnSplit = 8;
constexpr int kAttnMaxHd = 256;

__global__ void __cluster_dims__(kAttnSplit, 1, 1) __launch_bounds__(kAttnThreads)
    attention_kernel(const AttentionArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ double scores[];
  __shared__ double part[kAttnWarps];
  __shared__ double slice_max, slice_sum;
  __shared__ double slice_acc[kAttnMaxHd];
  __shared__ double part_acc[kAttnThreads * 4];  // kgroups x hd partial sums
  const int rank = (int)cluster.block_rank();
  const int head = blockIdx.x / kAttnSplit;
  const int64_t t = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t pos = a.position + t;
  const int64_t start = a.window > 0 && pos - a.window + 1 > 0 ? pos - a.window + 1 : 0;
  const int64_t count = pos - start + 1;
  const int64_t per = (count + kAttnSplit - 1) / kAttnSplit;
  const int64_t k0 = min64(count, rank * per), k1 = min64(count, k0 + per);  // this CTA's keys
  const int64_t mine = k1 - k0;
  const int64_t q_dim = (int64_t)a.heads * a.hd, kv_dim = (int64_t)a.kv_heads * a.hd;
  const int64_t kvo = (int64_t)(head / (a.heads / a.kv_heads)) * a.hd;
  const float* q = a.q + t * q_dim + (int64_t)head * a.hd;
  const double scale = __ddiv_rn(1.0, __dsqrt_rn((double)a.hd));

  // 1. scores and the max. Lane l holds q[l + 32 u]; a warp loads four keys
  // at once, then reduces each (the same per-lane order for every key).
  constexpr int kJ = kAttnMaxHd / 32;
  constexpr int kKeys = 4;
  double qd[kJ];
#pragma unroll
  for (int u = 0; u < kJ; u++) {
    const int j = lane + 32 * u;
    qd[u] = j < a.hd ? (double)q[j] : 0.0;
  }
  for (int64_t i0 = warp; i0 < mine; i0 += kAttnWarps * kKeys) {
    float kk[kKeys][kJ];
#pragma unroll
    for (int c = 0; c < kKeys; c++) {
      const int64_t i = i0 + c * kAttnWarps;
      const float* k = a.keys + (start + k0 + min64(i, mine - 1)) * kv_dim + kvo;
#pragma unroll
      for (int u = 0; u < kJ; u++) {
        const int j = lane + 32 * u;
        kk[c][u] = j < a.hd ? k[j] : 0.0f;
      }
    }
#pragma unroll
    for (int c = 0; c < kKeys; c++) {
      double d = 0.0;
#pragma unroll
      for (int u = 0; u < kJ; u++)
        if (lane + 32 * u < a.hd) d = __dadd_rn(d, __dmul_rn(qd[u], (double)kk[c][u]));
      d = warp_sum_d(d);
      const int64_t i = i0 + c * kAttnWarps;
      if (lane == 0 && i < mine) scores[i] = __dmul_rn(d, scale);
    }
  }
  __syncthreads();
  double m = -INFINITY;
  for (int64_t i = tid; i < mine; i += kAttnThreads) m = fmax(m, scores[i]);
  m = warp_max_d(m);
  if (lane == 0) part[warp] = m;
  __syncthreads();
  if (tid == 0) {
    double mm = part[0];
    for (int w = 1; w < kAttnWarps; w++) mm = fmax(mm, part[w]);
    slice_max = mm;
  }
  cluster.sync();
  m = -INFINITY;
  for (int r = 0; r < kAttnSplit; r++) m = fmax(m, *cluster.map_shared_rank(&slice_max, r));

  // 2. exp and the slice's sum
  double sum = 0.0;
  for (int64_t i = tid; i < mine; i += kAttnThreads) {
    const double e = exp(__dsub_rn(scores[i], m));
    scores[i] = e;
    sum = __dadd_rn(sum, e);
  }
  sum = warp_sum_d(sum);
  if (lane == 0) part[warp] = sum;
  __syncthreads();
  if (tid == 0) {
    double ss = 0.0;
    for (int w = 0; w < kAttnWarps; w++) ss = __dadd_rn(ss, part[w]);
    slice_sum = ss;
  }
  // ... and the slice's weighted values: thread (kg, dg) sums dimensions
  // 4 dg .. 4 dg + 3 (one 16-byte load per key) over part kg of the slice's
  // keys, in order, eight keys' loads at a time; the parts add in order.
  const int dgroups = (int)(a.hd / 4), kgroups = kAttnThreads / dgroups;
  const int dg = tid % dgroups, kg = tid / dgroups;
  const int64_t part_keys = (mine + kgroups - 1) / kgroups;
  const int64_t i_lo = min64(mine, kg * part_keys), i_hi = min64(mine, i_lo + part_keys);
  if (kg < kgroups) {
    const float* v = a.values + (start + k0) * kv_dim + kvo + 4 * dg;
    double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0, acc3 = 0.0;
    int64_t i = i_lo;
    for (; i + 8 <= i_hi; i += 8) {
      float4 vv[8];
#pragma unroll
      for (int u = 0; u < 8; u++) vv[u] = *reinterpret_cast<const float4*>(v + (i + u) * kv_dim);
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const double e = scores[i + u];
        acc0 = __dadd_rn(acc0, __dmul_rn(e, (double)vv[u].x));
        acc1 = __dadd_rn(acc1, __dmul_rn(e, (double)vv[u].y));
        acc2 = __dadd_rn(acc2, __dmul_rn(e, (double)vv[u].z));
        acc3 = __dadd_rn(acc3, __dmul_rn(e, (double)vv[u].w));
      }
    }
    for (; i < i_hi; i++) {
      const float4 vv = *reinterpret_cast<const float4*>(v + i * kv_dim);
      const double e = scores[i];
      acc0 = __dadd_rn(acc0, __dmul_rn(e, (double)vv.x));
      acc1 = __dadd_rn(acc1, __dmul_rn(e, (double)vv.y));
      acc2 = __dadd_rn(acc2, __dmul_rn(e, (double)vv.z));
      acc3 = __dadd_rn(acc3, __dmul_rn(e, (double)vv.w));
    }
    double* pa = part_acc + kg * a.hd + 4 * dg;
    pa[0] = acc0;
    pa[1] = acc1;
    pa[2] = acc2;
    pa[3] = acc3;
  }
  __syncthreads();
  for (int d = tid; d < a.hd; d += kAttnThreads) {
    double acc = 0.0;
    for (int p = 0; p < kgroups; p++) acc = __dadd_rn(acc, part_acc[p * a.hd + d]);
    slice_acc[d] = acc;
  }
  cluster.sync();

  // 3. CTA 0 adds the slices in rank order
  if (rank == 0) {
    double total = 0.0;
    for (int r = 0; r < kAttnSplit; r++) total = __dadd_rn(total, *cluster.map_shared_rank(&slice_sum, r));
    const bool gated = a.gate != nullptr;
    const double g = gated ? __ddiv_rn(1.0, __dadd_rn(1.0, exp(-(double)a.gate[t * a.heads + head]))) : 1.0;
    float* out = a.out + t * q_dim + (int64_t)head * a.hd;
    for (int d = tid; d < a.hd; d += kAttnThreads) {
      double acc = 0.0;
      for (int r = 0; r < kAttnSplit; r++) acc = __dadd_rn(acc, cluster.map_shared_rank(slice_acc, r)[d]);
      float o = __double2float_rn(__ddiv_rn(acc, total));
      if (gated) o = __double2float_rn(__dmul_rn((double)o, g));
      out[d] = o;
    }
  }
  cluster.sync();  // the other CTAs' shared memory stays until CTA 0 has read it
}

// ------------------------------------------------------------------- conv

// One thread per channel, walking the tokens in order. The taps of token t:
// s = 0 .. k-1 steps back, z of the chunk or a history row before it.
__global__ void __launch_bounds__(256) conv_kernel(const ConvArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t ch = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (ch >= a.width) return;
  const int64_t w = a.width;
  const int k = a.k;
  float past[kMaxConvTaps];  // the last k - 1 inputs z, oldest first
  for (int r = 0; r + 1 < k; r++) past[r] = a.history[r * w + ch];
  const float* kern = a.weight + ch * k;
  for (int64_t t = 0; t < a.n; t++) {
    const float* row = a.bcx + t * 3 * w;
    const float z = __fmul_rn(row[ch], row[2 * w + ch]);
    // From 0.0, as the CPU's sum starts (a first term of -0.0 then gives +0.0).
    double acc = __dadd_rn(0.0, __dmul_rn((double)kern[k - 1], (double)z));  // s = 0
    for (int s = 1; s < k; s++) acc = __dadd_rn(acc, __dmul_rn((double)kern[k - 1 - s], (double)past[k - 1 - s]));
    a.y[t * w + ch] = __double2float_rn(__dmul_rn((double)row[w + ch], acc));
    for (int r = 0; r + 2 < k; r++) past[r] = past[r + 1];
    if (k >= 2) past[k - 2] = z;
  }
  for (int r = 0; r + 1 < k; r++) a.history[r * w + ch] = past[r];
}

// ------------------------------------------------------------------ steer

// One CTA of 128 threads per row.
__global__ void __launch_bounds__(kNormLanes) steer_kernel(const SteerArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  float* x = a.x + (int64_t)blockIdx.x * a.cols;
  const int tid = threadIdx.x;
  if (a.mode == 0) {
    for (int64_t j = tid; j < a.cols; j += kNormLanes) x[j] = __fadd_rn(x[j], a.v[j]);
    return;
  }
  double d = 0.0;
  for (int64_t j = tid; j < a.cols; j += kNormLanes) d = __dadd_rn(d, __dmul_rn((double)x[j], (double)a.v[j]));
  d = warp_sum_d(d);
  __shared__ double part[kNormLanes / 32];
  if ((tid & 31) == 0) part[tid >> 5] = d;
  __syncthreads();
  double dot = 0.0;
#pragma unroll
  for (int w = 0; w < kNormLanes / 32; w++) dot = __dadd_rn(dot, part[w]);
  const double c = __dmul_rn(a.scale, dot);
  for (int64_t j = tid; j < a.cols; j += kNormLanes)
    x[j] = __double2float_rn(__dsub_rn((double)x[j], __dmul_rn(c, (double)a.v[j])));
}

cudaError_t launch_cfg(const void* kern, void** args, dim3 grid, int threads, size_t smem,
                       cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3((unsigned)threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

}  // namespace

cudaError_t launch_copy(const float* src, float* dst, int64_t count, cudaStream_t stream, bool pdl) {
  if (count <= 0) return cudaSuccess;
  int64_t grid = (count + 255) / 256;
  if (grid > 148 * 8) grid = 148 * 8;
  void* args[] = {&src, &dst, &count};
  return launch_cfg(reinterpret_cast<const void*>(copy_kernel), args, dim3((unsigned)grid), 256, 0,
                    stream, pdl);
}

cudaError_t launch_head_norm_rope(const HeadNormRopeArgs& a, cudaStream_t stream, bool pdl) {
  const int64_t heads = a.heads + (a.x2 != nullptr ? a.heads2 : 0);
  if (heads <= 0 || a.n <= 0) return cudaSuccess;
  if (a.hd <= 0 || a.hd % 2 != 0 || a.hd > 2 * kNormLanes || a.n > 65535 || heads > 0x7fffffff)
    return cudaErrorInvalidValue;
  HeadNormRopeArgs c = a;
  void* args[] = {&c};
  return launch_cfg(reinterpret_cast<const void*>(head_norm_rope_kernel), args,
                    dim3((unsigned)heads, (unsigned)a.n), kNormLanes, 0, stream, pdl);
}

cudaError_t launch_attention(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  if (a.heads <= 0 || a.n <= 0) return cudaSuccess;
  // The value sums load four dimensions at a time: hd a multiple of 4 (as the
  // reference's shader reads vec4s) and 16-byte aligned values.
  if (a.hd <= 0 || a.hd > kAttnMaxHd || a.hd % 4 != 0 || a.kv_heads <= 0 || a.heads % a.kv_heads != 0 ||
      a.n > 65535 || a.position < 0 || a.heads > 65535 / kAttnSplit || ((uintptr_t)a.values & 15) != 0)
    return cudaErrorInvalidValue;
  // Keys a token sees: all before it, or the window; a CTA scores its slice.
  const int64_t longest = a.window > 0 ? (a.window < a.position + a.n ? a.window : a.position + a.n)
                                       : a.position + a.n;
  if (longest > kMaxAttnKeys) return cudaErrorInvalidValue;
  const size_t smem = (size_t)((longest + kAttnSplit - 1) / kAttnSplit) * sizeof(double);
  AttentionArgs c = a;
  void* args[] = {&c};
  return launch_cfg(reinterpret_cast<const void*>(attention_kernel), args,
                    dim3((unsigned)(a.heads * kAttnSplit), (unsigned)a.n), kAttnThreads, smem, stream, pdl);
}

cudaError_t launch_conv(const ConvArgs& a, cudaStream_t stream, bool pdl) {
  if (a.width <= 0 || a.n < 0) return cudaSuccess;
  if (a.k < 1 || a.k > kMaxConvTaps) return cudaErrorInvalidValue;
  ConvArgs c = a;
  void* args[] = {&c};
  return launch_cfg(reinterpret_cast<const void*>(conv_kernel), args,
                    dim3((unsigned)((a.width + 255) / 256)), 256, 0, stream, pdl);
}

cudaError_t launch_steer(const SteerArgs& a, cudaStream_t stream, bool pdl) {
  if (a.rows <= 0 || a.cols <= 0) return cudaSuccess;
  if (a.rows > 0x7fffffff) return cudaErrorInvalidValue;
  SteerArgs c = a;
  void* args[] = {&c};
  return launch_cfg(reinterpret_cast<const void*>(steer_kernel), args, dim3((unsigned)a.rows),
                    kNormLanes, 0, stream, pdl);
}

}  // namespace dn
