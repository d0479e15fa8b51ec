// Row-per-lane decode dot products: one consumer warp owns a 32-row tile,
// lane r owns row r and keeps all four of the reference's accumulators, so a
// tile needs no shuffles or barriers beyond its own warp.
//
// For block b of row r the reference (lab_native.c:456-466 NEON,
// :483-512 AVX2) forms four int32 lane sums d_l over bytes 4l..4l+3 and
// 16+4l..16+4l+3 of the block, and accumulates
//   acc_l = fma(float(d_l), float(sw[b] * sx[b]), acc_l)     (l = 0..3)
// in block order, finishing with y = (acc0 + acc1) + (acc2 + acc3). Here the
// lane reads its row's 32-byte block with 128-bit loads from the swizzled
// stage, and the activation block (the same for every lane: a broadcast)
// likewise. float(d_l) is formed exactly without an int->float instruction:
// the dp4a chain starts from 0x4B400000 (the bits of 1.5 * 2^23, whose ulp is
// 1), so for |d| < 2^22 the result's bits are the float 12582912 + d, and one
// exact subtraction leaves d. (|d| <= 8 * 127 * 127 for Q8_0, 8 * 8 * 127 for
// Q4_0.)
#pragma once

#include "gemv_core.cuh"

namespace dn {
namespace rowdot {

using gemv::Fmt;
using gemv::kBox;
using gemv::kBoxBytes;
using gemv::kChunkBytes;
using gemv::kScaleRow;
using gemv::kStageBytes;
using gemv::kWBoxes;
using gemv::lds;

constexpr int kRows = 32;  // tile rows: one per lane of the consumer warp
constexpr int32_t kMagic = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t sw128(int r, int c) { return r * 128 + (((c ^ r) & 7) << 4); }
// Byte offset of 16-byte chunk j of row r in the 64-byte-swizzled scale box.
__device__ __forceinline__ uint32_t sw64(int r, int j) { return r * 64 + (((j ^ (r >> 1)) & 3) << 4); }

__device__ __forceinline__ float exact_d(int32_t biased) {
  return __fsub_rn(__int_as_float(biased), kMagicF);
}

// Activations of one token in shared memory, per block b: the 32 int8 at
// q + 32 b (16-byte aligned), the scale at s[b], and for Q4_0 the four dp4a
// seeds kMagic - 8 * (sum of the eight int8 accumulator l multiplies) at
// seed[b] (the nibbles enter the dot products unsigned, 0..15).
struct XBuf {
  uint8_t* q;
  float* s;
  int4* seed;
};

// Bytes of an XBuf for `blocks` blocks (each part 16-byte aligned).
__host__ __device__ inline int64_t xbuf_bytes(int64_t blocks, bool q4) {
  return blocks * 32 + gemv::round_up(blocks * 4, 16) + (q4 ? blocks * 16 : 0);
}
__device__ __forceinline__ XBuf xbuf_at(uint8_t* base, int64_t blocks, bool q4) {
  XBuf x;
  x.q = base;
  x.s = reinterpret_cast<float*>(base + blocks * 32);
  x.seed = q4 ? reinterpret_cast<int4*>(base + blocks * 32 + gemv::round_up(blocks * 4, 16)) : nullptr;
  return x;
}

// Bytes of the raw staging area load_qa_warp needs for `blocks` QA blocks.
__host__ __device__ inline int64_t qa_raw_bytes(int64_t blocks) {
  return gemv::round_up(blocks * kQABytes + 16, 16);
}

// Loads `blocks` QA blocks (36 bytes: 32 int8 then the f32 scale; the input
// 4-byte aligned) from global memory through L2 into x, by one warp: the
// bytes are copied with 16-byte loads (words up to the first 16-byte
// boundary and after the last one singly, so nothing outside the input is
// read) into `raw` at the input's offset modulo 16, then unpacked.
template <bool Q4>
__device__ __forceinline__ void load_qa_warp(const uint8_t* qa, int64_t blocks, const XBuf& x,
                                             uint8_t* raw, int lane) {
  const uint32_t mis = (uint32_t)((uintptr_t)qa & 15);  // a multiple of 4
  const int64_t words = blocks * (kQABytes / 4);
  const int64_t head = mis == 0 ? 0 : min64((16 - mis) / 4, words);
  const int64_t vecs = (words - head) / 4;
  const int64_t tail0 = head + vecs * 4;
  const uint32_t* src = reinterpret_cast<const uint32_t*>(qa);
  uint32_t* dst = reinterpret_cast<uint32_t*>(raw + mis);
  if (lane < head) dst[lane] = __ldcg(src + lane);
  if (lane < words - tail0) dst[tail0 + lane] = __ldcg(src + tail0 + lane);
  const uint4* vsrc = reinterpret_cast<const uint4*>(src + head);
  uint4* vdst = reinterpret_cast<uint4*>(dst + head);
  constexpr int U = 4;
  for (int64_t i0 = 0; i0 < vecs; i0 += 32 * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++)
      if (i0 + u * 32 + lane < vecs) v[u] = __ldcg(vsrc + i0 + u * 32 + lane);
#pragma unroll
    for (int u = 0; u < U; u++)
      if (i0 + u * 32 + lane < vecs) vdst[i0 + u * 32 + lane] = v[u];
  }
  __syncwarp();
  for (int64_t b = lane; b < blocks; b += 32) {
    const uint32_t* w = dst + b * (kQABytes / 4);
    uint32_t v[9];
#pragma unroll
    for (int i = 0; i < 9; i++) v[i] = w[i];
    *reinterpret_cast<uint4*>(x.q + b * 32) = make_uint4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<uint4*>(x.q + b * 32 + 16) = make_uint4(v[4], v[5], v[6], v[7]);
    x.s[b] = __uint_as_float(v[8]);
    if (Q4) {
      int32_t sd[4];
#pragma unroll
      for (int l = 0; l < 4; l++)
        sd[l] = kMagic - 8 * __dp4a((int32_t)v[l], 0x01010101, __dp4a((int32_t)v[4 + l], 0x01010101, 0));
      x.seed[b] = make_int4(sd[0], sd[1], sd[2], sd[3]);
    }
  }
}

// One block: the lane's 32 weight bytes as (wa, wb) = bytes 0..15, 16..31
// (Q8_0), or its 16 nibble bytes in wa (Q4_0).
template <bool Q4>
__device__ __forceinline__ void block_dot(const uint4& wa, const uint4& wb, const XBuf& x, int64_t b,
                                          float s, float (&acc)[4]) {
  const uint4 xa = lds<uint4>(x.q + b * 32);
  const uint4 xb = lds<uint4>(x.q + b * 32 + 16);
  const uint32_t xl[4] = {xa.x, xa.y, xa.z, xa.w};
  const uint32_t xh[4] = {xb.x, xb.y, xb.z, xb.w};
  if (Q4) {
    const int4 sd4 = lds<int4>(x.seed + b);
    const int32_t sd[4] = {sd4.x, sd4.y, sd4.z, sd4.w};
    const uint32_t w[4] = {wa.x, wa.y, wa.z, wa.w};
#pragma unroll
    for (int l = 0; l < 4; l++) {
      // byte 4l+i: low nibble = weight 4l+i, high nibble = weight 16+4l+i
      const int32_t d = __dp4a((int32_t)((w[l] >> 4) & 0x0f0f0f0fu), (int32_t)xh[l],
                               __dp4a((int32_t)(w[l] & 0x0f0f0f0fu), (int32_t)xl[l], sd[l]));
      acc[l] = __fmaf_rn(exact_d(d), s, acc[l]);
    }
  } else {
    const uint32_t w0[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t w1[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int l = 0; l < 4; l++) {
      const int32_t d =
          __dp4a((int32_t)w1[l], (int32_t)xh[l], __dp4a((int32_t)w0[l], (int32_t)xl[l], kMagic));
      acc[l] = __fmaf_rn(exact_d(d), s, acc[l]);
    }
  }
}

// The weights of block bb (0-based within the stage) for row r.
template <bool Q4>
__device__ __forceinline__ void weights_at(const uint8_t* stage, int r, int bb, uint4& wa, uint4& wb) {
  constexpr int kPerBox = kBoxBytes / Fmt<Q4>::kWB;
  const uint8_t* box = stage + (bb / kPerBox) * kBox;
  const int q = bb % kPerBox;
  if (Q4) {
    wa = lds<uint4>(box + sw128(r, q));
  } else {
    wa = lds<uint4>(box + sw128(r, 2 * q));
    wb = lds<uint4>(box + sw128(r, 2 * q + 1));
  }
}

// The scale of block bb (0-based within the stage) for row r from the
// stage's scale box.
template <bool Q4>
__device__ __forceinline__ float scale_at(const uint8_t* stage, int r, int bb) {
  const uint8_t* sbox = stage + kWBoxes * kBox;
  if (Q4) return half_bits_to_float(lds<uint16_t>(sbox + sw64(r, bb / 8) + (bb % 8) * 2));
  return lds<float>(sbox + sw64(r, bb / 4) + (bb % 4) * 4);
}

// Lane r's dot products over one stage: blocks b0 .. b0 + nb - 1 of row
// `row` (nb == Fmt<Q4>::kKC for a whole stage). With TMA_SCALES the scales
// come from the stage's scale box, otherwise from global memory
// (scales + row * blocks + b).
template <bool Q4, bool TMA_SCALES>
__device__ __forceinline__ void stage_dot(const uint8_t* stage, int nb, int64_t b0, int r, const XBuf& x,
                                          const void* scales, int64_t row, int64_t blocks,
                                          float (&acc)[4]) {
  using F = Fmt<Q4>;
  auto gscale = [&](int64_t b) -> float {
    return Q4 ? half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(scales) + row * blocks + b))
              : __ldg(reinterpret_cast<const float*>(scales) + row * blocks + b);
  };
  if (nb == F::kKC && TMA_SCALES) {
    // A whole stage as straight-line code: 4 boxes of 4 (Q8_0) or 8 (Q4_0)
    // blocks; one 16-byte scale load per box (Q8_0: 4 f32; Q4_0: 8 fp16).
    constexpr int kPerBox = kBoxBytes / F::kWB;
    const uint8_t* sbox = stage + kWBoxes * kBox;
#pragma unroll
    for (int j = 0; j < kWBoxes; j++) {
      const uint4 sv = lds<uint4>(sbox + sw64(r, j));
      float sw[kPerBox];
      if (Q4) {
        const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int q = 0; q < 8; q++) sw[q] = half_bits_to_float((uint16_t)(u[q >> 1] >> (16 * (q & 1))));
      } else {
        sw[0] = __uint_as_float(sv.x);
        sw[1] = __uint_as_float(sv.y);
        sw[2] = __uint_as_float(sv.z);
        sw[3] = __uint_as_float(sv.w);
      }
#pragma unroll
      for (int q4 = 0; q4 < kPerBox; q4 += 4) {
        const int64_t bq = b0 + j * kPerBox + q4;
        const float4 xs = lds<float4>(x.s + bq);
        const float xsv[4] = {xs.x, xs.y, xs.z, xs.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          uint4 wa, wb;
          weights_at<Q4>(stage, r, j * kPerBox + q4 + q, wa, wb);
          block_dot<Q4>(wa, wb, x, bq + q, __fmul_rn(sw[q4 + q], xsv[q]), acc);
        }
      }
    }
  } else {
    for (int bb = 0; bb < nb; bb++) {
      uint4 wa, wb;
      weights_at<Q4>(stage, r, bb, wa, wb);
      const float sw = TMA_SCALES ? scale_at<Q4>(stage, r, bb) : gscale(b0 + bb);
      block_dot<Q4>(wa, wb, x, b0 + bb, __fmul_rn(sw, x.s[b0 + bb]), acc);
    }
  }
}

__device__ __forceinline__ float finish(const float (&acc)[4]) {
  return __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
}

}  // namespace rowdot
}  // namespace dn
