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
constexpr int kRowPad = 16;        // bytes between consecutive rows of a stage
constexpr int kChunkBytes = 512;   // weight bytes per row per stage

template <bool Q4>
struct Fmt {
  static constexpr int kWB = Q4 ? 16 : 32;          // weight bytes per block
  static constexpr int kSB = Q4 ? 2 : 4;            // scale bytes per block
  static constexpr int kKC = kChunkBytes / kWB;     // blocks per stage
  static constexpr int kWStride = kKC * kWB + kRowPad;
  static constexpr int kSStride = kKC * kSB + kRowPad;
};

struct SmemPlan {
  int64_t w_off, s_off, bar_off, xq_off, xsc_off, xs8_off, total;
};

template <bool Q4>
__host__ __device__ inline SmemPlan plan(int rows_per_cta, int nt, int64_t blocks) {
  using F = Fmt<Q4>;
  SmemPlan p;
  p.w_off = 0;
  p.s_off = p.w_off + (int64_t)kStages * rows_per_cta * F::kWStride;
  p.bar_off = p.s_off + (int64_t)kStages * rows_per_cta * F::kSStride;
  p.xq_off = p.bar_off + 8 * kStages + 64;
  p.xq_off = (p.xq_off + 127) & ~(int64_t)127;
  p.xsc_off = p.xq_off + (int64_t)nt * blocks * kBlock;
  p.xs8_off = p.xsc_off + (int64_t)nt * blocks * 4;
  p.total = p.xs8_off + (Q4 ? (int64_t)nt * blocks * 16 : 0);
  return p;
}

// Quantizes tokens [t0, t0 + nt) into shared memory, eight lanes per block
// (lab_quantize_q8 semantics). Q4 also gets -8 * the lane sums of each block.
// CTA column 0 copies the result to xq / xsc in global memory when given.
template <bool Q4, int THREADS>
__device__ __forceinline__ void quantize_to_smem(const LinearArgs& a, int64_t t0, int nt,
                                                 int64_t blocks, int8_t* xq_s, float* xsc_s,
                                                 int32_t* xs8_s) {
  const int tid = threadIdx.x, sub = tid & 7;
  const bool writer = blockIdx.x == 0 && a.xq != nullptr;
  const int64_t jobs = (int64_t)nt * blocks;
  for (int64_t base = 0; base < jobs; base += THREADS / 8) {
    const int64_t job = base + (tid >> 3);
    const bool active = job < jobs;
    const int64_t t = active ? job / blocks : 0, b = active ? job % blocks : 0;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (active) v = __ldg(reinterpret_cast<const float4*>(a.xs + (t0 + t) * a.cols + b * kBlock + sub * 4));
    float amax = fmaxf(fmaxf(fmaxf(0.0f, fabsf(v.x)), fmaxf(fabsf(v.y), fabsf(v.z))), fabsf(v.w));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    float scale, inv;
    q8_scale(amax, scale, inv);
    const int32_t q0 = quant_q8_elem(v.x, inv), q1 = quant_q8_elem(v.y, inv),
                  q2 = quant_q8_elem(v.z, inv), q3 = quant_q8_elem(v.w, inv);
    const uint32_t word = pack4(q0, q1, q2, q3);
    int32_t part = q0 + q1 + q2 + q3;
    if (Q4) part += __shfl_down_sync(0xffffffffu, part, 4);  // sub l < 4: lane sum l
    if (active) {
      *reinterpret_cast<uint32_t*>(xq_s + (t * blocks + b) * kBlock + sub * 4) = word;
      if (sub == 0) xsc_s[t * blocks + b] = scale;
      if (Q4 && sub < 4) xs8_s[(t * blocks + b) * 4 + sub] = -8 * part;
      if (writer) {
        *reinterpret_cast<uint32_t*>(a.xq + (t0 + t) * a.cols + b * kBlock + sub * 4) = word;
        if (sub == 0) a.xsc[(t0 + t) * blocks + b] = scale;
      }
    }
  }
}

template <bool Q4, int WARPS, int NT, bool TMA_SCALES>
__global__ void __launch_bounds__(WARPS * 32) gemv_i8_kernel(const LinearArgs a) {
  using F = Fmt<Q4>;
  constexpr int ROWS = 8 * WARPS;
  constexpr int THREADS = WARPS * 32;
  extern __shared__ __align__(128) uint8_t smem[];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r8 = lane >> 2, l = lane & 3;
  const int64_t blocks = a.cols / kBlock;
  const int64_t row0 = (int64_t)blockIdx.x * ROWS;
  const int tile_rows = (int)min64(ROWS, a.rows - row0);
  const int64_t t0 = (int64_t)blockIdx.y * NT;
  const int nt = (int)min64(NT, a.n - t0);
  const int nchunks = (int)((blocks + F::kKC - 1) / F::kKC);
  const SmemPlan sp = plan<Q4>(ROWS, NT, blocks);
  uint8_t* w_s = smem + sp.w_off;
  uint8_t* s_s = smem + sp.s_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sp.bar_off);
  int8_t* xq_s = reinterpret_cast<int8_t*>(smem + sp.xq_off);
  float* xsc_s = reinterpret_cast<float*>(smem + sp.xsc_off);
  int32_t* xs8_s = reinterpret_cast<int32_t*>(smem + sp.xs8_off);

  if (tid == 0) {
    for (int s = 0; s < kStages; s++) mbar_init(&bars[s], 1);
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
      bulk_g2s(w_s + (s * ROWS + r) * F::kWStride,
               qs + (row0 + r) * wrow_bytes + (int64_t)c * F::kKC * F::kWB, wbytes, &bars[s]);
      if (TMA_SCALES)
        bulk_g2s(s_s + (s * ROWS + r) * F::kSStride,
                 sc + (row0 + r) * srow_bytes + (int64_t)c * F::kKC * F::kSB, sbytes, &bars[s]);
    }
  };
  int issued = 0;
  if (warp == 0) {
    for (; issued < min(kStages, nchunks); issued++) issue(issued);
  }
  // The weights do not depend on the previous kernel; the activations do.
  pdl_wait();
  quantize_to_smem<Q4, THREADS>(a, t0, nt, blocks, xq_s, xsc_s, xs8_s);
  __syncthreads();
  pdl_launch_dependents();

  const int row_local = warp * 8 + r8;
  const int64_t row = row0 + min(row_local, tile_rows - 1);
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; t++) acc[t] = 0.0f;

  bool failed = false;
  int c = 0;
  for (; c < nchunks; c++) {
    const int s = c % kStages;
    const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
    const bool ok = mbar_wait_bounded(&bars[s], (uint32_t)(c / kStages) & 1u, a.status,
                                      kStatusTmaTimeout);
    if (ok) {
      const uint8_t* wrow = w_s + (s * ROWS + row_local) * F::kWStride + 4 * l;
      const int64_t b0 = (int64_t)c * F::kKC;
#pragma unroll 4
      for (int bb = 0; bb < nb; bb++) {
        const int64_t b = b0 + bb;
        float sw;
        if (TMA_SCALES) {
          const uint8_t* srow = s_s + (s * ROWS + row_local) * F::kSStride;
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
          const int8_t* xb = xq_s + ((int64_t)t * blocks + b) * kBlock + 4 * l;
          const int32_t base = Q4 ? xs8_s[((int64_t)t * blocks + b) * 4 + l] : 0;
          const int32_t d = __dp4a(w0, (int32_t)lds_u32(xb), __dp4a(w1, (int32_t)lds_u32(xb + 16), base));
          const float s2 = __fmul_rn(sw, xsc_s[(int64_t)t * blocks + b]);
          acc[t] = __fmaf_rn(__int2float_rn(d), s2, acc[t]);
        }
      }
    }
    failed = __syncthreads_or(!ok) != 0;
    if (failed) break;
    if (warp == 0 && issued < nchunks) issue(issued++);
  }
  if (failed) {
    // Let copies still in flight land before the CTA's shared memory goes.
    if (tid == 0) {
      for (int k = c + 1; k < issued; k++)
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
    if (l == 0 && row_local < tile_rows && t < nt) a.ys[(t0 + t) * a.ldy + row0 + row_local] = y;
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

template <bool Q4, int WARPS, int NT, bool TMA_SCALES>
int64_t launch_gemv_t(const LinearArgs& a, cudaStream_t stream, bool pdl) {
  constexpr int ROWS = 8 * WARPS;
  const int64_t blocks = a.cols / kBlock;
  const SmemPlan sp = plan<Q4>(ROWS, NT, blocks);
  if (sp.total > 227 * 1024) return kErrTooLarge;
  auto kern = gemv_i8_kernel<Q4, WARPS, NT, TMA_SCALES>;
  static bool configured[64] = {};  // per device: the opt-in smem limit is set
  int dev = 0;
  cudaGetDevice(&dev);
  if (sp.total > 48 * 1024 && !configured[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess)
      return kErrCuda;
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.rows + ROWS - 1) / ROWS), (unsigned)((a.n + NT - 1) / NT), 1);
  cfg.blockDim = dim3(WARPS * 32, 1, 1);
  cfg.dynamicSmemBytes = (size_t)sp.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? kOk : kErrCuda;
}

template <bool Q4, int WARPS, int NT>
int64_t launch_gemv_s(const LinearArgs& a, cudaStream_t stream, bool pdl) {
  const int64_t blocks = a.cols / kBlock;
  const bool tma_scales = ((uintptr_t)a.scales & 15) == 0 && (blocks * Fmt<Q4>::kSB) % 16 == 0;
  return tma_scales ? launch_gemv_t<Q4, WARPS, NT, true>(a, stream, pdl)
                    : launch_gemv_t<Q4, WARPS, NT, false>(a, stream, pdl);
}

template <bool Q4, int NT>
int64_t launch_gemv_w(const LinearArgs& a, cudaStream_t stream, bool pdl) {
  // Rows per CTA: the most (up to 32) that still leaves two CTAs per SM.
  const int64_t target = 2 * 148;
  if ((a.rows + 31) / 32 >= target) return launch_gemv_s<Q4, 4, NT>(a, stream, pdl);
  if ((a.rows + 15) / 16 >= target) return launch_gemv_s<Q4, 2, NT>(a, stream, pdl);
  return launch_gemv_s<Q4, 1, NT>(a, stream, pdl);
}

template <bool Q4>
int64_t launch_gemv_q(const LinearArgs& a, cudaStream_t stream, bool pdl) {
  if (a.n <= 1) return launch_gemv_w<Q4, 1>(a, stream, pdl);
  if (a.n <= 2) return launch_gemv_w<Q4, 2>(a, stream, pdl);
  if (a.n <= 4) return launch_gemv_w<Q4, 4>(a, stream, pdl);
  return launch_gemv_w<Q4, 8>(a, stream, pdl);
}

}  // namespace

bool gemv_supported(const LinearArgs& a) {
  return a.mode == 1 && a.cols % kBlock == 0 && a.cols > 0 && ((uintptr_t)a.qs & 15) == 0 &&
         ((uintptr_t)a.xs & 15) == 0 && (a.xq == nullptr || ((uintptr_t)a.xq & 3) == 0) &&
         ((uintptr_t)a.scales & (a.q4 ? 1 : 3)) == 0;
}

int64_t launch_gemv(const LinearArgs& a, cudaStream_t stream, bool pdl) {
  if (!gemv_supported(a)) return kErrUnsupported;
  if (a.rows <= 0 || a.n <= 0) return kOk;
  return a.q4 ? launch_gemv_q<true>(a, stream, pdl) : launch_gemv_q<false>(a, stream, pdl);
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
