// Decode GEMV for Q8_0 and Q4_0 weights times Q8_0-quantized activations
// (lab_gemm_q8 / lab_gemm_q4 with small n, lab_native.c:553-579, 1059-1080).
//
// Bit-exact with the reference, not just within tolerance. The reference
// computes every output as four f32 accumulator chains over the blocks in
// order, acc_l = fma(f32(d_l), f32(sw * sx), acc_l), where d_l is the int32
// sum over bytes 4l..4l+3 of both 16-byte halves of a block, and ends with
// (acc0 + acc1) + (acc2 + acc3) (lab_native.c:456-466, 503-512, 987-1002,
// 1025-1034). Here each warp lane owns exactly one chain: lane (r, l) of a
// warp computes accumulator l of row r (8 rows per warp), so the chain runs
// in the reference's order with the reference's roundings, and the four
// lanes of a row finish with two shuffles in the reference's pairing.
//
// The Q4 nibble layout lines up with the lanes: word l of a 16-byte Q4 block
// holds, in its low nibbles, weights 4l..4l+3 and, in its high nibbles,
// weights 16+4l..16+4l+3 - exactly lane l's eight weights. The unsigned
// nibbles go straight into dp4a and the "- 8" is folded in as -8 * (sum of the
// lane's eight activations), precomputed once per token and block.
//
// Memory path: weights stream from HBM with 1-D TMA bulk copies
// (cp.async.bulk) of one 512-byte row chunk each into a 4-stage shared-memory
// ring, completing on an mbarrier per stage; rows sit 16 bytes apart in
// shared memory beyond their 512 bytes so the lanes' 4-byte reads are free of
// bank conflicts. Every CTA quantizes the activations itself (they are small
// and L2-resident), which fuses the activation quantize into the GEMV; CTA
// column 0 also writes xq / xsc out, as lab_gemm_* does.
#include <algorithm>

#include "dn_common.cuh"
#include "dn_launch.h"

namespace dn {
namespace {

constexpr int kStages = 4;
constexpr int kWarps = 4;
constexpr int kRows = 8 * kWarps;  // rows per CTA: one Q8_0 block of the output
constexpr int kThreads = 32 * kWarps;
constexpr int kRowPad = 16;        // bytes between consecutive rows of a stage
constexpr int kChunkBytes = 512;   // weight bytes per row per stage
constexpr int kMaxSmem = 227 * 1024;

template <bool Q4>
struct Fmt {
  static constexpr int kWB = Q4 ? 16 : 32;          // weight bytes per block
  static constexpr int kSB = Q4 ? 2 : 4;            // scale bytes per block
  static constexpr int kKC = kChunkBytes / kWB;     // blocks per stage
  static constexpr int kWStride = kKC * kWB + kRowPad;
  static constexpr int kSStride = kKC * kSB + kRowPad;
};

__host__ __device__ inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

struct SmemPlan {
  int64_t w_off, s_off, bar_off, xa_off, xa_stride, xs8_off, yt_off, xf_off, total;
};

// bars: kStages weight stages, then two activation barriers.
template <bool Q4>
__host__ __device__ inline SmemPlan plan(int nt, int64_t cols, bool f32_in) {
  using F = Fmt<Q4>;
  const int64_t blocks = cols / kBlock;
  SmemPlan p;
  p.w_off = 0;
  p.s_off = p.w_off + (int64_t)kStages * kRows * F::kWStride;
  p.bar_off = p.s_off + (int64_t)kStages * kRows * F::kSStride;
  p.xa_off = round_up(p.bar_off + 8 * (kStages + 2), 128);
  p.xa_stride = round_up(blocks * kQABytes, 16);
  p.xs8_off = p.xa_off + nt * p.xa_stride;
  p.yt_off = p.xs8_off + (Q4 ? (int64_t)nt * blocks * 16 : 0);
  p.xf_off = round_up(p.yt_off + (int64_t)nt * kRows * 4, 128);
  p.total = p.xf_off + (f32_in ? 2 * cols * 4 : 0);
  return p;
}

// Quantizes one token of f32 activations (in shared memory) into QA blocks in
// shared memory, eight lanes per block (lab_quantize_q8 semantics). With
// `xq`, also writes lab_gemm's xq / xsc outputs for that token.
__device__ __forceinline__ void quantize_token(const float* xf, uint8_t* xa, int64_t blocks,
                                               int8_t* xq, float* xsc) {
  const int tid = threadIdx.x, sub = tid & 7;
  for (int64_t base = 0; base < blocks; base += kThreads / 8) {
    const int64_t b = base + (tid >> 3);
    const bool active = b < blocks;
    const float4 v = active ? *reinterpret_cast<const float4*>(xf + b * kBlock + sub * 4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    float amax = fmaxf(fmaxf(fmaxf(0.0f, fabsf(v.x)), fmaxf(fabsf(v.y), fabsf(v.z))), fabsf(v.w));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    float scale, inv;
    q8_scale(amax, scale, inv);
    const uint32_t word = pack4(quant_q8_elem(v.x, inv), quant_q8_elem(v.y, inv),
                                quant_q8_elem(v.z, inv), quant_q8_elem(v.w, inv));
    if (active) {
      *reinterpret_cast<uint32_t*>(xa + b * kQABytes + sub * 4) = word;
      if (sub == 0) *reinterpret_cast<float*>(xa + b * kQABytes + 32) = scale;
      if (xq != nullptr) {
        *reinterpret_cast<uint32_t*>(xq + b * kBlock + sub * 4) = word;
        if (sub == 0) xsc[b] = scale;
      }
    }
  }
}

template <bool Q4, int NT, bool TMA_SCALES, bool F32_IN>
__global__ void __launch_bounds__(kThreads) gemv_i8_kernel(const GemvArgs a) {
  using F = Fmt<Q4>;
  extern __shared__ __align__(128) uint8_t smem[];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r8 = lane >> 2, l = lane & 3;
  const int64_t blocks = a.cols / kBlock;
  const int64_t row0 = (int64_t)blockIdx.x * kRows;
  const int tile_rows = (int)min64(kRows, a.rows - row0);
  const int64_t t0 = (int64_t)blockIdx.y * NT;
  const int nt = (int)min64(NT, a.n - t0);
  const int nchunks = (int)((blocks + F::kKC - 1) / F::kKC);
  const SmemPlan sp = plan<Q4>(NT, a.cols, F32_IN);
  uint8_t* w_s = smem + sp.w_off;
  uint8_t* s_s = smem + sp.s_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sp.bar_off);
  uint64_t* xbars = bars + kStages;
  uint8_t* xa_s = smem + sp.xa_off;
  int32_t* xs8_s = reinterpret_cast<int32_t*>(smem + sp.xs8_off);
  float* yt_s = reinterpret_cast<float*>(smem + sp.yt_off);
  float* xf_s = reinterpret_cast<float*>(smem + sp.xf_off);

  if (tid == 0) {
    for (int s = 0; s < kStages + 2; s++) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const uint8_t* qs = static_cast<const uint8_t*>(a.qs);
  const uint8_t* sc = static_cast<const uint8_t*>(a.scales);
  const int64_t wrow_bytes = blocks * F::kWB, srow_bytes = blocks * F::kSB;
  // Warp 0 issues one stage: a bulk copy per row of its weight chunk (and of
  // its scale chunk when those are 16-byte aligned).
  auto issue = [&](int c) {
    const int s = c % kStages;
    const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
    const uint32_t wbytes = nb * F::kWB, sbytes = TMA_SCALES ? nb * F::kSB : 0;
    if (lane == 0) mbar_arrive_expect_tx(&bars[s], (uint32_t)tile_rows * (wbytes + sbytes));
    __syncwarp();
    for (int r = lane; r < tile_rows; r += 32) {
      bulk_g2s(w_s + (s * kRows + r) * F::kWStride,
               qs + (row0 + r) * wrow_bytes + (int64_t)c * F::kKC * F::kWB, wbytes, &bars[s]);
      if (TMA_SCALES)
        bulk_g2s(s_s + (s * kRows + r) * F::kSStride,
                 sc + (row0 + r) * srow_bytes + (int64_t)c * F::kKC * F::kSB, sbytes, &bars[s]);
    }
  };
  int issued = 0;
  if (warp == 0) {
    for (; issued < min(kStages, nchunks); issued++) issue(issued);
  }

  // The weights do not depend on the previous kernel; the activations do.
  pdl_wait();
  bool ok = true;
  if (F32_IN) {
    // Token by token through two f32 buffers: the bulk copy of token t+2
    // runs while token t+1 is quantized.
    const uint32_t xbytes = (uint32_t)(a.cols * 4);
    auto issue_x = [&](int tt) {
      mbar_arrive_expect_tx(&xbars[tt & 1], xbytes);
      bulk_g2s(xf_s + (tt & 1) * a.cols, a.xs + (t0 + tt) * a.cols, xbytes, &xbars[tt & 1]);
    };
    if (tid == 0) {
      for (int tt = 0; tt < min(2, nt); tt++) issue_x(tt);
    }
    const bool writer = blockIdx.x == 0 && a.xq != nullptr;
    for (int tt = 0; tt < nt; tt++) {
      const bool got = mbar_wait_bounded(&xbars[tt & 1], (uint32_t)(tt >> 1) & 1u, a.status,
                                         kStatusTmaTimeout);
      if (got)
        quantize_token(xf_s + (tt & 1) * a.cols, xa_s + tt * sp.xa_stride, blocks,
                       writer ? a.xq + (t0 + tt) * a.cols : nullptr,
                       writer ? a.xsc + (t0 + tt) * blocks : nullptr);
      if (__syncthreads_or(!got)) {
        ok = false;
        break;
      }
      if (tid == 0 && tt + 2 < nt) issue_x(tt + 2);
    }
  } else {
    const int64_t row_bytes = blocks * kQABytes;
    const bool bulk = (row_bytes % 16) == 0 && ((uintptr_t)a.xa & 15) == 0 && (a.xa_stride % 16) == 0;
    if (bulk) {
      if (tid == 0) {
        mbar_arrive_expect_tx(&xbars[0], (uint32_t)(nt * row_bytes));
        for (int tt = 0; tt < nt; tt++)
          bulk_g2s(xa_s + tt * sp.xa_stride, a.xa + (t0 + tt) * a.xa_stride, (uint32_t)row_bytes,
                   &xbars[0]);
      }
      ok = mbar_wait_bounded(&xbars[0], 0, a.status, kStatusTmaTimeout);
    } else {
      for (int tt = 0; tt < nt; tt++) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(a.xa + (t0 + tt) * a.xa_stride);
        uint32_t* dst = reinterpret_cast<uint32_t*>(xa_s + tt * sp.xa_stride);
        for (int64_t i = tid; i < row_bytes / 4; i += kThreads) dst[i] = __ldg(src + i);
      }
    }
    ok = __syncthreads_or(!ok) == 0;
  }
  if (Q4 && ok) {
    // -8 * (sum of lane l's eight activations) per token and block: the
    // nibbles enter dp4a unsigned and this term subtracts the offset of 8.
    for (int64_t i = tid; i < (int64_t)nt * blocks * 4; i += kThreads) {
      const int64_t tt = i / (blocks * 4), rem = i % (blocks * 4), b = rem >> 2;
      const int ll = (int)(rem & 3);
      const uint8_t* xb = xa_s + tt * sp.xa_stride + b * kQABytes + 4 * ll;
      xs8_s[i] = -8 * __dp4a((int32_t)lds_u32(xb), 0x01010101, __dp4a((int32_t)lds_u32(xb + 16), 0x01010101, 0));
    }
    __syncthreads();
  }
  pdl_launch_dependents();

  const int row_local = warp * 8 + r8;
  const int64_t row = row0 + min(row_local, tile_rows - 1);
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; t++) acc[t] = 0.0f;

  bool failed = !ok;
  int c = 0;
  for (; c < nchunks && !failed; c++) {
    const int s = c % kStages;
    const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
    const bool got = mbar_wait_bounded(&bars[s], (uint32_t)(c / kStages) & 1u, a.status,
                                       kStatusTmaTimeout);
    if (got) {
      const uint8_t* wrow = w_s + (s * kRows + row_local) * F::kWStride + 4 * l;
      const int64_t b0 = (int64_t)c * F::kKC;
#pragma unroll 4
      for (int bb = 0; bb < nb; bb++) {
        const int64_t b = b0 + bb;
        float sw;
        if (TMA_SCALES) {
          const uint8_t* srow = s_s + (s * kRows + row_local) * F::kSStride;
          sw = Q4 ? half_bits_to_float(reinterpret_cast<const uint16_t*>(srow)[bb])
                  : reinterpret_cast<const float*>(srow)[bb];
        } else {
          sw = Q4 ? half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(sc) + row * blocks + b))
                  : __ldg(reinterpret_cast<const float*>(sc) + row * blocks + b);
        }
        int32_t w0, w1;
        if (Q4) {
          const uint32_t wv = lds_u32(wrow + bb * 16);
          w0 = (int32_t)(wv & 0x0f0f0f0fu);          // weights 4l..4l+3, as 0..15
          w1 = (int32_t)((wv >> 4) & 0x0f0f0f0fu);   // weights 16+4l..16+4l+3
        } else {
          w0 = (int32_t)lds_u32(wrow + bb * 32);
          w1 = (int32_t)lds_u32(wrow + bb * 32 + 16);
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
          const uint8_t* xb = xa_s + t * sp.xa_stride + b * kQABytes;
          const int32_t base = Q4 ? xs8_s[((int64_t)t * blocks + b) * 4 + l] : 0;
          const int32_t d = __dp4a(w0, (int32_t)lds_u32(xb + 4 * l),
                                   __dp4a(w1, (int32_t)lds_u32(xb + 16 + 4 * l), base));
          const float s2 = __fmul_rn(sw, *reinterpret_cast<const float*>(xb + 32));
          acc[t] = __fmaf_rn(__int2float_rn(d), s2, acc[t]);
        }
      }
    }
    failed = __syncthreads_or(!got) != 0;
    if (!failed && warp == 0 && issued < nchunks) issue(issued++);
  }
  if (failed) {
    // Let copies still in flight land before the CTA's shared memory goes.
    if (tid == 0) {
      for (int k = c; k < issued; k++)
        mbar_wait_bounded(&bars[k % kStages], (uint32_t)(k / kStages) & 1u, a.status,
                          kStatusTmaTimeout);
    }
    __syncthreads();
    return;
  }

#pragma unroll
  for (int t = 0; t < NT; t++) {
    const float v = acc[t];
    const float s01 = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1));
    const float y = __fadd_rn(s01, __shfl_down_sync(0xffffffffu, s01, 2));
    if (l == 0 && row_local < tile_rows && t < nt) {
      if (a.ys != nullptr) a.ys[(t0 + t) * a.ldy + row0 + row_local] = y;
      yt_s[t * kRows + row_local] = y;
    }
  }
  if (a.ya != nullptr && tile_rows == kRows) {
    // The CTA's 32 outputs of a token are one Q8_0 block of the next
    // projection's input: quantize them here (lab_quantize_q8 semantics).
    __syncthreads();
    for (int t = warp; t < nt; t += kWarps) {
      const float v = yt_s[t * kRows + lane];
      float amax = fmaxf(0.0f, fabsf(v));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      float scale, inv;
      q8_scale(amax, scale, inv);
      uint8_t* dst = a.ya + (t0 + t) * a.ya_stride + (int64_t)blockIdx.x * kQABytes;
      dst[lane] = (uint8_t)(int8_t)quant_q8_elem(v, inv);
      if (lane == 0) *reinterpret_cast<float*>(dst + 32) = scale;
    }
  }
}

// ------------------------------------------------------------------ generic
//
// Any alignment, any cols (the reference ignores a trailing partial block),
// both modes. Same lane-per-chain mapping; weights come straight from global
// memory a byte at a time, so it is slow, but exact. Mode 1 reads the
// activations already quantized into xq / xsc.

__device__ __forceinline__ int32_t gather_word(const uint8_t* p) {
  return (int32_t)((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                   ((uint32_t)p[3] << 24));
}

__device__ __forceinline__ int q4_weight(const uint8_t* blk, int j) {
  return (j < 16 ? (blk[j] & 15) : (blk[j - 16] >> 4)) - 8;
}

__global__ void __launch_bounds__(128) generic_kernel(const LinearArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r8 = lane >> 2, l = lane & 3;
  const int64_t blocks = a.cols / kBlock;
  const int64_t row_raw = ((int64_t)blockIdx.x * 4 + warp) * 8 + r8;
  const int64_t row = min(row_raw, a.rows - 1);
  const int64_t t = blockIdx.y;
  const uint8_t* qs = static_cast<const uint8_t*>(a.qs);
  const uint8_t* rowp = a.q4 ? qs + row * a.cols / 2 : qs + row * a.cols;
  float acc = 0.0f;
  for (int64_t b = 0; b < blocks; b++) {
    const float sw = a.q4 ? half_bits_to_float(static_cast<const uint16_t*>(a.scales)[row * blocks + b])
                          : static_cast<const float*>(a.scales)[row * blocks + b];
    if (a.mode == 1) {
      const int8_t* xb = a.xq + t * a.cols + b * kBlock;
      int32_t d = 0;
      for (int h = 0; h < 32; h += 16) {
        for (int i = 0; i < 4; i++) {
          const int j = h + 4 * l + i;
          const int w = a.q4 ? q4_weight(rowp + b * 16, j) : (int)(int8_t)rowp[b * kBlock + j];
          d += w * xb[j];
        }
      }
      acc = __fmaf_rn(__int2float_rn(d), __fmul_rn(sw, a.xsc[t * blocks + b]), acc);
    } else {
      const float* xb = a.xs + t * a.cols + b * kBlock;
      float s = 0.0f;
      for (int m = 0; m < 8; m++) {
        const int j = 4 * m + l;
        const int w = a.q4 ? q4_weight(rowp + b * 16, j) : (int)(int8_t)rowp[b * kBlock + j];
        s = __fmaf_rn((float)w, xb[j], s);
      }
      acc = __fmaf_rn(s, sw, acc);
    }
  }
  const float s01 = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
  const float y = __fadd_rn(s01, __shfl_down_sync(0xffffffffu, s01, 2));
  if (l == 0 && row_raw < a.rows) a.ys[t * a.ldy + row_raw] = y;
}

template <bool Q4, int NT, bool TMA_SCALES, bool F32_IN>
int64_t launch_gemv_t(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  const SmemPlan sp = plan<Q4>(NT, a.cols, F32_IN);
  if (sp.total > kMaxSmem) return kErrTooLarge;
  auto kern = gemv_i8_kernel<Q4, NT, TMA_SCALES, F32_IN>;
  static bool configured[64] = {};  // per device: the opt-in smem limit is set
  int dev = 0;
  cudaGetDevice(&dev);
  if (sp.total > 48 * 1024 && !configured[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return kErrCuda;
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.rows + kRows - 1) / kRows), (unsigned)((a.n + NT - 1) / NT), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)sp.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? kOk : kErrCuda;
}

template <bool Q4, int NT>
int64_t launch_gemv_s(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  const int64_t blocks = a.cols / kBlock;
  const bool tma_scales = ((uintptr_t)a.scales & 15) == 0 && (blocks * Fmt<Q4>::kSB) % 16 == 0;
  const bool f32_in = a.xs != nullptr;
  if (tma_scales)
    return f32_in ? launch_gemv_t<Q4, NT, true, true>(a, stream, pdl)
                  : launch_gemv_t<Q4, NT, true, false>(a, stream, pdl);
  return f32_in ? launch_gemv_t<Q4, NT, false, true>(a, stream, pdl)
                : launch_gemv_t<Q4, NT, false, false>(a, stream, pdl);
}

// Tokens per CTA: enough for n (up to 8), fewer if shared memory runs out.
template <bool Q4>
int64_t launch_gemv_q(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  const bool f32_in = a.xs != nullptr;
  auto fits = [&](int nt) { return plan<Q4>(nt, a.cols, f32_in).total <= kMaxSmem; };
  if (a.n <= 1 || !fits(2)) return fits(1) ? launch_gemv_s<Q4, 1>(a, stream, pdl) : kErrTooLarge;
  if (a.n <= 2 || !fits(4)) return launch_gemv_s<Q4, 2>(a, stream, pdl);
  if (a.n <= 4 || !fits(8)) return launch_gemv_s<Q4, 4>(a, stream, pdl);
  return launch_gemv_s<Q4, 8>(a, stream, pdl);
}

}  // namespace

bool gemv_ex_supported(const GemvArgs& g) {
  if (g.cols % kBlock != 0 || g.cols <= 0 || ((uintptr_t)g.qs & 15) != 0 ||
      ((uintptr_t)g.scales & (g.q4 ? 1 : 3)) != 0)
    return false;
  if ((g.xs == nullptr) == (g.xa == nullptr)) return false;
  if (g.xs != nullptr && (((uintptr_t)g.xs & 15) != 0 || (g.xq != nullptr && ((uintptr_t)g.xq & 3) != 0)))
    return false;
  if (g.xa != nullptr && (((uintptr_t)g.xa & 3) != 0 || (g.xa_stride & 3) != 0)) return false;
  if (g.ya != nullptr && (((uintptr_t)g.ya & 3) != 0 || (g.ya_stride & 3) != 0)) return false;
  return (g.q4 ? plan<true>(1, g.cols, g.xs != nullptr).total
               : plan<false>(1, g.cols, g.xs != nullptr).total) <= kMaxSmem;
}

int64_t launch_gemv_ex(const GemvArgs& g, cudaStream_t stream, bool pdl) {
  if (!gemv_ex_supported(g)) return kErrUnsupported;
  if (g.rows <= 0 || g.n <= 0) return kOk;
  if (g.n > 65535 * 8) return kErrTooLarge;
  return g.q4 ? launch_gemv_q<true>(g, stream, pdl) : launch_gemv_q<false>(g, stream, pdl);
}

static GemvArgs from_linear(const LinearArgs& a) {
  GemvArgs g{};
  g.q4 = a.q4;
  g.qs = a.qs;
  g.scales = a.scales;
  g.xs = a.xs;
  g.xq = a.xq;
  g.xsc = a.xsc;
  g.ys = a.ys;
  g.ldy = a.ldy;
  g.rows = a.rows;
  g.cols = a.cols;
  g.n = a.n;
  g.status = a.status;
  return g;
}

bool gemv_supported(const LinearArgs& a) {
  return a.mode == 1 && a.xs != nullptr && gemv_ex_supported(from_linear(a));
}

int64_t launch_gemv(const LinearArgs& a, cudaStream_t stream, bool pdl) {
  if (!gemv_supported(a)) return kErrUnsupported;
  return launch_gemv_ex(from_linear(a), stream, pdl);
}

int64_t launch_generic(const LinearArgs& a, cudaStream_t stream) {
  if (a.rows <= 0 || a.n <= 0) return kOk;
  if (a.mode == 1) {
    if (a.xq == nullptr || a.xsc == nullptr) return kErrArgs;
    if (launch_quantize_q8(a.xs, a.xq, a.xsc, a.n, a.cols, stream) != cudaSuccess) return kErrCuda;
  }
  const dim3 grid((unsigned)((a.rows + 31) / 32), (unsigned)a.n, 1);
  generic_kernel<<<grid, 128, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace dn
