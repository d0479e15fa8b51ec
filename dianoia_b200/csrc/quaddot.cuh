// Quad-lane decode dot products: four lanes per weight row, lane l keeping
// the reference's accumulator l, eight rows per warp, four consumer warps per
// 32-row tile. This spreads a tile over 128 lanes, so the serial part of a
// decode step (one tile's dot products after its input arrives) is short.
//
// For block b of row r the reference (lab_native.c:456-466 NEON,
// :483-512 AVX2) forms four int32 lane sums d_l over bytes 4l..4l+3 and
// 16+4l..16+4l+3 of the block and accumulates
//   acc_l = fma(float(d_l), float(sw[b] * sx[b]), acc_l)     (l = 0..3)
// in block order, finishing with y = (acc0 + acc1) + (acc2 + acc3). Here lane
// l of the row loads its two words of the block from the 128-byte-swizzled
// stage and its eight activation bytes from a lane-interleaved copy of the
// input. float(d_l) is formed exactly without an int->float instruction: the
// dp4a chain starts from 0x4B400000 (the bits of 1.5 * 2^23, whose ulp is 1),
// so for |d| < 2^22 the result's bits are the float 12582912 + d and one exact
// subtraction (two blocks per packed f32x2 add) leaves d. (|d| <= 8 * 127 * 127
// for Q8_0, 8 * 8 * 127 for Q4_0.) The scale products sw * sx are also formed
// two at a time (mul.rn.f32x2: two independent round-to-nearest products).
#pragma once

#include "gemv_core.cuh"

namespace dn {
namespace quad {

using gemv::Fmt;
using gemv::kBox;
using gemv::kBoxBytes;
using gemv::kStageBytes;
using gemv::kWBoxes;
using gemv::lds;

constexpr int kRows = 32;  // rows per tile
constexpr int kWarps = 4;  // consumer warps per tile, 8 rows each
using gemv::exact_d2;
using gemv::f2_add;
using gemv::f2_hi;
using gemv::f2_lo;
using gemv::f2_mul;
using gemv::f2_pack;
using gemv::kMagic;
using gemv::kMagicF;

// --------------------------------------------------------- activation layout
// One token's activations in shared memory, lane-interleaved per block b:
//   Q8_0: 32 bytes; lane l's 8 at b * 32 + 8 l (its words 4l..4l+3 and
//         16+4l..16+4l+3 of the block);
//   Q4_0: 64 bytes; lane l's 16 at b * 64 + 16 l: the same two words,
//         -8 * (sum of those eight int8) (the nibbles enter the dot products
//         unsigned, 0..15; kMagic is added where it seeds the dp4a) and a pad
//         word (the layout gemv_core.cuh's XLayout also uses);
// and the block scales as a float array.
template <bool Q4>
struct XQ {
  static constexpr int kLane = Q4 ? 16 : 8;
  static constexpr int kBlock = 4 * kLane;
};

__host__ __device__ inline int64_t x_bytes(int64_t blocks, bool q4) {
  return blocks * (q4 ? 64 : 32) + gemv::round_up(blocks * 4, 16);
}

// QA blocks in global memory (4-byte aligned) -> the lane-interleaved
// layout, read through L2 (ld.global.cg: the input may have been written by
// another SM during this kernel): item i = (block i / 4, lane i % 4) takes
// words l and 4 + l of its block (and the scale, for l = 0). The loads of up
// to U items per thread are in flight together.
template <bool Q4>
__device__ __forceinline__ void load_unpack(const uint8_t* qa, int64_t blocks, uint8_t* xw, float* xs,
                                            int t, int nthreads) {
  constexpr int U = 4;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(qa);
  const int64_t items = blocks * 4;
  for (int64_t i0 = 0; i0 < items; i0 += (int64_t)nthreads * U) {
    uint32_t lo[U], hi[U], sc[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int64_t i = i0 + (int64_t)u * nthreads + t;
      if (i < items) {
        const uint32_t* w = src + (i >> 2) * (kQABytes / 4);
        const int l = (int)(i & 3);
        lo[u] = __ldcg(w + l);
        hi[u] = __ldcg(w + 4 + l);
        if (l == 0) sc[u] = __ldcg(w + 8);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int64_t i = i0 + (int64_t)u * nthreads + t;
      if (i < items) {
        const int64_t b = i >> 2;
        const int l = (int)(i & 3);
        if (Q4) {
          const int32_t seed =
              -8 * __dp4a((int32_t)lo[u], 0x01010101, __dp4a((int32_t)hi[u], 0x01010101, 0));
          *reinterpret_cast<uint4*>(xw + b * 64 + 16 * l) = make_uint4(lo[u], hi[u], (uint32_t)seed, 0u);
        } else {
          *reinterpret_cast<uint2*>(xw + b * 32 + 8 * l) = make_uint2(lo[u], hi[u]);
        }
        if (l == 0) xs[b] = __uint_as_float(sc[u]);
      }
    }
  }
}

// ------------------------------------------------------------- dot products
// Per-lane constants: lane (r8, l) of consumer warp w owns accumulator l of
// tile row r = 8 w + r8.
struct Lane {
  uint32_t off[8];  // byte offset of word l of 16-byte chunk c of row r in a 128-byte-swizzled box
  uint32_t soff;    // row r's line in the 64-byte-swizzled scale box (chunk 0)
  int r, l;
  // off[k] for a k known only at run time (indexing off[] with one would
  // move the array to local memory).
  __device__ __forceinline__ uint32_t off_rt(int k) const {
    return r * 128 + (((k ^ r) & 7) << 4) + 4 * l;
  }
};
__device__ __forceinline__ Lane lane_ctx(int warp, int lane) {
  Lane c;
  c.l = lane & 3;
  c.r = warp * 8 + (lane >> 2);
#pragma unroll
  for (int k = 0; k < 8; k++) c.off[k] = c.r * 128 + (((k ^ c.r) & 7) << 4) + 4 * c.l;
  c.soff = c.r * 64 + (((c.r >> 1) & 3) << 4);
  return c;
}

// Accumulator l over one stage of nb blocks. xwb / xsb: the activations of
// the stage's first block (xwb offset to the lane's slot); with TMA_SCALES
// the weight scales come from the stage's 64-byte-swizzled scale box,
// otherwise from global memory (gsc: the row's scale of the stage's first
// block). The callers advance these pointers chunk by chunk: forming them
// here from a block index made the compiler issue the shared-memory loads
// late (measured: twice the time per stage).
// Accumulator l over one whole stage (Fmt<Q4>::kKC blocks) whose weight
// scales are in the stage's 64-byte-swizzled scale box. xwb / xsb: the
// activations of the stage's first block (xwb offset to the lane's slot).
// Callers advance these pointers chunk by chunk, and keep whole stages and
// the general case (stage_part) in separate loops: forming the pointers here
// from a block index, or branching between the two cases per stage, made the
// compiler issue the shared-memory loads late (measured: up to twice the
// time per stage).
template <bool Q4>
__device__ __forceinline__ void stage_full(const uint8_t* stage, const Lane& c, const uint8_t* xwb,
                                           const float* xsb, float& acc) {
  using X = XQ<Q4>;
  const uint8_t* sbox = stage + kWBoxes * kBox;
  // A whole stage, straight-line: 4 boxes of 4 (Q8_0) or 8 (Q4_0) blocks.
#pragma unroll
  for (int j = 0; j < kWBoxes; j++) {
    const uint8_t* box = stage + j * kBox;
    const uint4 sv = lds<uint4>(sbox + (c.soff ^ (j << 4)));
    if (Q4) {
      const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int h = 0; h < 2; h++) {  // blocks 8j + 4h .. 8j + 4h + 3
        const float4 x4 = lds<float4>(xsb + 8 * j + 4 * h);
        const uint64_t s01 = f2_mul(f2_pack(half_bits_to_float((uint16_t)u[2 * h]),
                                            half_bits_to_float((uint16_t)(u[2 * h] >> 16))),
                                    f2_pack(x4.x, x4.y));
        const uint64_t s23 = f2_mul(f2_pack(half_bits_to_float((uint16_t)u[2 * h + 1]),
                                            half_bits_to_float((uint16_t)(u[2 * h + 1] >> 16))),
                                    f2_pack(x4.z, x4.w));
        int32_t d[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const int bb = 4 * h + q;  // block within the box = 16-byte chunk
          const uint32_t w = lds<uint32_t>(box + c.off[bb]);
          const uint4 xv = lds<uint4>(xwb + (8 * j + bb) * X::kBlock);
          d[q] = __dp4a((int32_t)((w >> 4) & 0x0f0f0f0fu), (int32_t)xv.y,
                        __dp4a((int32_t)(w & 0x0f0f0f0fu), (int32_t)xv.x, (int32_t)xv.z + kMagic));
        }
        const uint64_t d01 = exact_d2(d[0], d[1]), d23 = exact_d2(d[2], d[3]);
        acc = __fmaf_rn(f2_lo(d01), f2_lo(s01), acc);
        acc = __fmaf_rn(f2_hi(d01), f2_hi(s01), acc);
        acc = __fmaf_rn(f2_lo(d23), f2_lo(s23), acc);
        acc = __fmaf_rn(f2_hi(d23), f2_hi(s23), acc);
      }
    } else {
      const float4 x4 = lds<float4>(xsb + 4 * j);
      const uint64_t s01 = f2_mul(f2_pack(__uint_as_float(sv.x), __uint_as_float(sv.y)), f2_pack(x4.x, x4.y));
      const uint64_t s23 = f2_mul(f2_pack(__uint_as_float(sv.z), __uint_as_float(sv.w)), f2_pack(x4.z, x4.w));
      int32_t d[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint32_t w0 = lds<uint32_t>(box + c.off[2 * q]);
        const uint32_t w1 = lds<uint32_t>(box + c.off[2 * q + 1]);
        const uint2 xv = lds<uint2>(xwb + (4 * j + q) * X::kBlock);
        d[q] = __dp4a((int32_t)w1, (int32_t)xv.y, __dp4a((int32_t)w0, (int32_t)xv.x, kMagic));
      }
      const uint64_t d01 = exact_d2(d[0], d[1]), d23 = exact_d2(d[2], d[3]);
      acc = __fmaf_rn(f2_lo(d01), f2_lo(s01), acc);
      acc = __fmaf_rn(f2_hi(d01), f2_hi(s01), acc);
      acc = __fmaf_rn(f2_lo(d23), f2_lo(s23), acc);
      acc = __fmaf_rn(f2_hi(d23), f2_hi(s23), acc);
    }
  }
}

// Accumulator l over any stage of nb blocks: a partial last stage, or
// scales read from global memory (TMA_SCALES false; gsc: the row's scale of
// the stage's first block).
template <bool Q4, bool TMA_SCALES>
__device__ __forceinline__ void stage_part(const uint8_t* stage, int nb, const Lane& c,
                                           const uint8_t* xwb, const float* xsb, const void* gsc,
                                           float& acc) {
  using F = Fmt<Q4>;
  using X = XQ<Q4>;
  const uint8_t* sbox = stage + kWBoxes * kBox;
  constexpr int kPerBox = kBoxBytes / F::kWB;
  for (int bb = 0; bb < nb; bb++) {
    const uint8_t* box = stage + (bb / kPerBox) * kBox;
    const int q = bb % kPerBox;
    float sw;
    if (TMA_SCALES) {
      sw = Q4 ? half_bits_to_float(lds<uint16_t>(sbox + (c.soff ^ ((bb / 8) << 4)) + (bb % 8) * 2))
              : lds<float>(sbox + (c.soff ^ ((bb / 4) << 4)) + (bb % 4) * 4);
    } else {
      sw = Q4 ? half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(gsc) + bb))
              : __ldg(reinterpret_cast<const float*>(gsc) + bb);
    }
    int32_t d;
    if (Q4) {
      const uint32_t w = lds<uint32_t>(box + c.off_rt(q));
      const uint4 xv = lds<uint4>(xwb + bb * X::kBlock);
      d = __dp4a((int32_t)((w >> 4) & 0x0f0f0f0fu), (int32_t)xv.y,
                 __dp4a((int32_t)(w & 0x0f0f0f0fu), (int32_t)xv.x, (int32_t)xv.z + kMagic));
    } else {
      const uint32_t w0 = lds<uint32_t>(box + c.off_rt(2 * q));
      const uint32_t w1 = lds<uint32_t>(box + c.off_rt(2 * q + 1));
      const uint2 xv = lds<uint2>(xwb + bb * X::kBlock);
      d = __dp4a((int32_t)w1, (int32_t)xv.y, __dp4a((int32_t)w0, (int32_t)xv.x, kMagic));
    }
    acc = __fmaf_rn(__fsub_rn(__int_as_float(d), kMagicF), __fmul_rn(sw, xsb[bb]), acc);
  }
}

}  // namespace quad
}  // namespace dn
