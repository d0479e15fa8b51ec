// Shared pieces of the decode GEMV kernels (gemv.cu): tile geometry, the
// lane-interleaved activation layout, the exact per-block dot-product step
// over one shared-memory stage, and the output helpers. See gemv.cu for the
// design.
#pragma once

#include "dn_common.cuh"
#include "dn_launch.h"

namespace dn {
namespace gemv {

constexpr int kConsumerWarps = 4;
constexpr int kRows = 8 * kConsumerWarps;   // rows per tile: one Q8_0 block of the output
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kThreads = kConsumers + 32;   // + one producer warp
constexpr int kChunkBytes = 512;            // weight bytes per row per stage
constexpr int kBoxBytes = 128;              // inner box width (the 128-byte swizzle span)
constexpr int kBox = kRows * kBoxBytes;     // 4 KB per box in shared memory
constexpr int kWBoxes = kChunkBytes / kBoxBytes;
constexpr int kScaleRow = 64;               // scale bytes per row per stage (16 f32 / 32 fp16)
constexpr int kStageBytes = kWBoxes * kBox + kRows * kScaleRow;  // weight boxes + scale box
constexpr int kMaxSmem = 226 * 1024;  // dynamic; leaves room for static smem
constexpr int kSmemPerSM = 228 * 1024;
constexpr int kSMs = 148;
constexpr int kMaxStages = 16;

// dp4a sums seeded with kMagic: the bits 0x4B400000 + d are the float
// 1.5 * 2^23 + d, exact for |d| < 2^22, so subtracting kMagicF converts d to
// float exactly, without the slower int-to-float conversion.
constexpr int32_t kMagic = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

// Packed f32x2 arithmetic (two floats per instruction).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// Two biased dp4a results as exact floats.
__device__ __forceinline__ uint64_t exact_d2(int32_t a, int32_t b) {
  return f2_add(f2_pack(__int_as_float(a), __int_as_float(b)), f2_pack(-kMagicF, -kMagicF));
}

template <bool Q4>
struct Fmt {
  static constexpr int kWB = Q4 ? 16 : 32;          // weight bytes per block
  static constexpr int kSB = Q4 ? 2 : 4;            // scale bytes per block
  static constexpr int kKC = kChunkBytes / kWB;     // blocks per stage (scales: 64 bytes)
};

__host__ __device__ inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

struct SmemPlan {
  int64_t bar_off, xw_off, xw_stride, xs_off, xs_stride, yt_off, stg_off, stg_stride, nw_off, total;
};

// Activations in shared memory, lane-interleaved: for block b, lane l's two
// words (bytes 4l..4l+3 and 16+4l..16+4l+3 of the block) sit together, so a
// lane reads its block operand with one 64-bit load (Q8). Q4 adds the lane's
// -8 * sum term: 16 bytes per lane, one 128-bit load. Block scales are a
// separate f32 array.
template <bool Q4>
struct XLayout {
  static constexpr int kLaneBytes = Q4 ? 16 : 8;
  static constexpr int kBlockBytes = 4 * kLaneBytes;
  // Offset of word w (0..7) of a block.
  __device__ static __forceinline__ int word_off(int w) { return (w & 3) * kLaneBytes + (w >> 2) * 4; }
};

// Layout from a 1024-byte aligned base: the stages, the barriers (`stages`
// full, `stages` empty, three activation, two epilogue), the activations, the
// epilogue's outputs, the input staging and, for a product that runs an
// RMSNorm in its prologue, the norm's weights. `total` includes the slack to
// align the base.
template <bool Q4>
__host__ __device__ inline SmemPlan plan(int stages, int nt, int64_t cols, bool f32_in, bool norm) {
  const int64_t blocks = cols / kBlock;
  SmemPlan p;
  p.bar_off = (int64_t)stages * kStageBytes;
  p.xw_off = round_up(p.bar_off + 8 * (2 * stages + 5), 128);
  p.xw_stride = blocks * XLayout<Q4>::kBlockBytes;
  p.xs_off = p.xw_off + nt * p.xw_stride;
  p.xs_stride = round_up(blocks, 4);
  p.yt_off = p.xs_off + nt * p.xs_stride * 4;
  p.stg_off = round_up(p.yt_off + 2 * (int64_t)nt * kRows * 4, 128);
  p.stg_stride = f32_in ? cols * 4 : round_up(blocks * kQABytes, 16);
  p.nw_off = round_up(p.stg_off + (f32_in ? 2 : nt) * p.stg_stride, 16);
  p.total = p.nw_off + (norm ? cols * 4 : 0) + 1024;
  return p;
}

// In a 128-byte-swizzled box of 32 rows x 128 bytes, byte `col` of row r
// sits at r * 128 + (((col / 16) ^ (r % 8)) * 16) + col % 16: the 16-byte
// chunk index is XORed with r mod 8.
// A bounded wait whose result is the same on every lane of the warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  const bool got = mbar_wait_bounded(bar, parity, status, kStatusTmaTimeout);
  return __all_sync(0xffffffffu, got) != 0;
}

// warp_wait whose waiting lanes sleep in hardware (mbarrier try_wait with a
// suspend-time hint) instead of spinning, so warps that wait leave the issue
// slots to warps that compute.
__device__ __forceinline__ bool warp_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t* status,
                                                uint32_t mult = 1) {
  const bool got = mbar_wait_bounded_sleep(bar, parity, status, kStatusTmaTimeout, mult);
  return __all_sync(0xffffffffu, got) != 0;
}

// Named barrier over the consumer warps only (the producer never joins);
// used in the prologue, which every consumer thread always reaches.
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

// True in every consumer thread when `v` is true in all of them (a named
// barrier with an AND reduction; every consumer thread must reach it).
__device__ __forceinline__ bool consumers_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kConsumers)
      : "memory");
  return r != 0;
}

template <typename T>
__device__ __forceinline__ T lds(const void* p) {
  return *reinterpret_cast<const T*>(p);
}

// -8 * (sum of the eight int8 a lane multiplies in one block).
__device__ __forceinline__ int32_t lane_sum8(uint32_t w0, uint32_t w1) {
  return -8 * __dp4a((int32_t)w0, 0x01010101, __dp4a((int32_t)w1, 0x01010101, 0));
}

// Quantizes one token of f32 activations (in shared memory) into the
// lane-interleaved layout, eight lanes per block (lab_quantize_q8
// semantics). With `xq`, also writes lab_gemm's xq / xsc outputs; with `qa`,
// the same values as QA blocks (32 int8 and the f32 scale per block).
template <bool Q4>
__device__ __forceinline__ void quantize_token(const float* xf, uint8_t* xw, float* xs,
                                               int64_t blocks, int8_t* xq, float* xsc,
                                               uint8_t* qa = nullptr) {
  using X = XLayout<Q4>;
  const int tid = threadIdx.x, sub = tid & 7;
  for (int64_t base = 0; base < blocks; base += kConsumers / 8) {
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
    const uint32_t hi_word = __shfl_down_sync(0xffffffffu, word, 4);  // sub < 4: word sub + 4
    if (active) {
      uint8_t* blk = xw + b * X::kBlockBytes;
      *reinterpret_cast<uint32_t*>(blk + X::word_off(sub)) = word;
      if (Q4 && sub < 4) *reinterpret_cast<int32_t*>(blk + sub * 16 + 8) = lane_sum8(word, hi_word);
      if (sub == 0) xs[b] = scale;
      if (xq != nullptr) {
        *reinterpret_cast<uint32_t*>(xq + b * kBlock + sub * 4) = word;
        if (sub == 0) xsc[b] = scale;
      }
      if (qa != nullptr) {
        *reinterpret_cast<uint32_t*>(qa + b * kQABytes + sub * 4) = word;
        if (sub == 0) *reinterpret_cast<float*>(qa + b * kQABytes + 32) = scale;
      }
    }
  }
}

// QA blocks (staged in shared memory) -> the lane-interleaved layout.
template <bool Q4>
__device__ __forceinline__ void unpack_qa(const uint8_t* qa, uint8_t* xw, float* xs, int64_t blocks) {
  using X = XLayout<Q4>;
  for (int64_t i = threadIdx.x; i < blocks * 4; i += kConsumers) {
    const int64_t b = i >> 2;
    const int ll = (int)(i & 3);
    const uint8_t* src = qa + b * kQABytes;
    const uint32_t w0 = lds<uint32_t>(src + 4 * ll), w1 = lds<uint32_t>(src + 16 + 4 * ll);
    uint8_t* dst = xw + b * X::kBlockBytes + ll * X::kLaneBytes;
    if (Q4) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(w0, w1, (uint32_t)lane_sum8(w0, w1), 0u);
    } else {
      *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);
    }
    if (ll == 0) xs[b] = lds<float>(src + 32);
  }
}


// Per-consumer-lane context of the dot products: lane (r8, l) of consumer
// warp w owns accumulator chain l of tile row 8w + r8.
struct LaneCtx {
  int row_local, r8, l;
  uint32_t rowoff;         // the row's offset in a weight box
  const uint8_t* xw_l;     // this lane's slot in the lane-interleaved activations
  int64_t xw_stride;       // bytes between tokens there
  const float* xs_s;       // activation block scales
  int64_t xs_stride;       // floats between tokens
  const uint8_t* sc;       // weight scales in global memory (path without a scale box)
  int64_t row, blocks;     // the lane's weight row (clamped) and blocks per row
};

// Runs the reference's per-block step over the nb blocks of one stage
// (blocks b0 .. b0 + nb - 1 of the row) for every token.
template <bool Q4, int NT, bool TMA_SCALES>
__device__ __forceinline__ void gemv_stage(const uint8_t* stage, int nb, int b0, const LaneCtx& c,
                                           float (&acc)[NT]) {
  using F = Fmt<Q4>;
  using X = XLayout<Q4>;
  constexpr int kPerBox = kBoxBytes / F::kWB;  // blocks per weight box: 4 (Q8) or 8 (Q4)
  const int r8 = c.r8, l = c.l, row_local = c.row_local;
  const uint32_t rowoff = c.rowoff;
  const uint8_t* xw_l = c.xw_l;
  const float* xs_s = c.xs_s;
  const uint8_t* sc = c.sc;
  const int64_t row = c.row, blocks = c.blocks;
  struct {
    int64_t xw_stride, xs_stride;
  } sp{c.xw_stride, c.xs_stride};
  // One block: weights w0 / w1 (as int8 for Q8, nibbles for Q4), its
  // scale, and the activations of every token.
  // The dot products are seeded with kMagic and converted to float two at a
  // time (exact), the scale products taken two at a time (f32x2, the same
  // roundings); each token keeps its own fma chain in the reference's order.
  auto block_step = [&](int b, int32_t w0, int32_t w1, float sw, const float* xsc_b) {
    int32_t d[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const uint8_t* xb = xw_l + t * sp.xw_stride + b * X::kBlockBytes;
      if (Q4) {
        const uint4 xv = lds<uint4>(xb);
        d[t] = __dp4a(w0, (int32_t)xv.x, __dp4a(w1, (int32_t)xv.y, (int32_t)xv.z + kMagic));
      } else {
        const uint2 xv = lds<uint2>(xb);
        d[t] = __dp4a(w0, (int32_t)xv.x, __dp4a(w1, (int32_t)xv.y, kMagic));
      }
    }
    const uint64_t sw2 = f2_pack(sw, sw);
#pragma unroll
    for (int t = 0; t + 1 < NT; t += 2) {
      const uint64_t dd = exact_d2(d[t], d[t + 1]);
      const uint64_t ss = f2_mul(sw2, f2_pack(xsc_b[t], xsc_b[t + 1]));
      acc[t] = __fmaf_rn(f2_lo(dd), f2_lo(ss), acc[t]);
      acc[t + 1] = __fmaf_rn(f2_hi(dd), f2_hi(ss), acc[t + 1]);
    }
    if (NT & 1)
      acc[NT - 1] = __fmaf_rn(__fsub_rn(__int_as_float(d[NT - 1]), kMagicF), __fmul_rn(sw, xsc_b[NT - 1]),
                              acc[NT - 1]);
  };
  auto weights_of = [&](const uint8_t* stage, int bb, int32_t& w0, int32_t& w1) {
    if (Q4) {
      const uint32_t wv = lds<uint32_t>(stage + (bb / 8) * kBox + rowoff +
                                        ((((bb & 7) ^ r8) & 7) << 4) + 4 * l);
      w0 = (int32_t)(wv & 0x0f0f0f0fu);          // weights 4l..4l+3, as 0..15
      w1 = (int32_t)((wv >> 4) & 0x0f0f0f0fu);   // weights 16+4l..16+4l+3
    } else {
      const uint8_t* line = stage + (bb / 4) * kBox + rowoff;
      w0 = (int32_t)lds<uint32_t>(line + (((((bb & 3) * 2) ^ r8) & 7) << 4) + 4 * l);
      w1 = (int32_t)lds<uint32_t>(line + (((((bb & 3) * 2 + 1) ^ r8) & 7) << 4) + 4 * l);
    }
  };
  auto scale_of = [&](const uint8_t* stage, int bb, int64_t b) -> float {
    if (TMA_SCALES) {
      const uint8_t* sline = stage + kWBoxes * kBox + row_local * kScaleRow;
      return Q4 ? half_bits_to_float(lds<uint16_t>(sline + bb * 2)) : lds<float>(sline + bb * 4);
    }
    return Q4 ? half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(sc) + row * blocks + b))
              : __ldg(reinterpret_cast<const float*>(sc) + row * blocks + b);
  };

      const int full_boxes = nb / kPerBox;
  // A whole box: kPerBox consecutive blocks, their scales in one 16-byte
  // load, the activation scales in 16-byte loads.
  auto do_box = [&](int j) {
    const uint8_t* line = stage + j * kBox + rowoff;
    float sws[kPerBox];
    if (TMA_SCALES) {
      const uint4 sv = lds<uint4>(stage + kWBoxes * kBox + row_local * kScaleRow + 16 * j);
      if (Q4) {
        const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int q = 0; q < 8; q++) sws[q] = half_bits_to_float((uint16_t)(u[q >> 1] >> (16 * (q & 1))));
      } else {
        sws[0] = __uint_as_float(sv.x);
        sws[1] = __uint_as_float(sv.y);
        sws[2] = __uint_as_float(sv.z);
        sws[3] = __uint_as_float(sv.w);
      }
    } else {
#pragma unroll
      for (int q = 0; q < kPerBox; q++) sws[q] = scale_of(stage, j * kPerBox + q, b0 + j * kPerBox + q);
    }
#pragma unroll
    for (int q4 = 0; q4 < kPerBox; q4 += 4) {
      const int bq = b0 + j * kPerBox + q4;
      float xsc[4][NT];
#pragma unroll
      for (int t = 0; t < NT; t++) {
        const float4 xv = lds<float4>(xs_s + t * sp.xs_stride + bq);
        xsc[0][t] = xv.x;
        xsc[1][t] = xv.y;
        xsc[2][t] = xv.z;
        xsc[3][t] = xv.w;
      }
#pragma unroll
      for (int q = 0; q < 4; q++) {
        int32_t w0, w1;
        if (Q4) {
          const uint32_t wv = lds<uint32_t>(line + ((((q4 + q) ^ r8) & 7) << 4) + 4 * l);
          w0 = (int32_t)(wv & 0x0f0f0f0fu);
          w1 = (int32_t)((wv >> 4) & 0x0f0f0f0fu);
        } else {
          w0 = (int32_t)lds<uint32_t>(line + (((2 * q ^ r8) & 7) << 4) + 4 * l);
          w1 = (int32_t)lds<uint32_t>(line + ((((2 * q + 1) ^ r8) & 7) << 4) + 4 * l);
        }
        block_step(bq + q, w0, w1, sws[q4 + q], xsc[q]);
      }
    }
  };
  if (full_boxes == kWBoxes) {
    // A full stage as straight-line code: later blocks' loads and dot
    // products can be scheduled under the serial FMA chain.
#pragma unroll
    for (int j = 0; j < kWBoxes; j++) do_box(j);
  } else {
    for (int j = 0; j < full_boxes; j++) do_box(j);
  }
  // Blocks after the last whole box (only when cols is not a multiple of
  // the box: 128 weights for Q8, 256 for Q4).
  for (int bb = full_boxes * kPerBox; bb < nb; bb++) {
    int32_t w0, w1;
    weights_of(stage, bb, w0, w1);
    float xsc[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) xsc[t] = xs_s[t * sp.xs_stride + b0 + bb];
    block_step(b0 + bb, w0, w1, scale_of(stage, bb, b0 + bb), xsc);
  }
}

// The reference's lane pairing (acc0 + acc1) + (acc2 + acc3) across the four
// lanes of a row; the sum is valid on lane l = 0.
__device__ __forceinline__ float lane_reduce(float v) {
  const float s01 = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1));
  return __fadd_rn(s01, __shfl_down_sync(0xffffffffu, s01, 2));
}

// Quantizes the 32 outputs of a tile for one token (one per lane of the
// calling warp) into a QA block (lab_quantize_q8 semantics).
__device__ __forceinline__ void quantize_block_out(float v, uint8_t* dst, int lane) {
  float amax = fmaxf(0.0f, fabsf(v));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  float scale, inv;
  q8_scale(amax, scale, inv);
  dst[lane] = (uint8_t)(int8_t)quant_q8_elem(v, inv);
  if (lane == 0) *reinterpret_cast<float*>(dst + 32) = scale;
}

// Producer side: the TMA boxes of one stage (chunk c of the 32-row tile at
// row y0): boxes of the weights and, with TMA_SCALES, one of the scales.
template <bool Q4, bool TMA_SCALES>
__device__ __forceinline__ void issue_stage(uint8_t* stage, const void* tw, const void* tsc, int c,
                                            int nb, int32_t y0, uint64_t* full) {
  using F = Fmt<Q4>;
  const int boxes = (nb * F::kWB + kBoxBytes - 1) / kBoxBytes;
  // Boxes past the matrix edge are zero-filled and count in full.
  mbar_arrive_expect_tx(full, (uint32_t)(boxes * kBox + (TMA_SCALES ? kRows * kScaleRow : 0)));
  for (int j = 0; j < boxes; j++) tma_load_2d(stage + j * kBox, tw, c * kChunkBytes + j * kBoxBytes, y0, full);
  if (TMA_SCALES) tma_load_2d(stage + kWBoxes * kBox, tsc, c * F::kKC, y0, full);
}

}  // namespace gemv
}  // namespace dn
