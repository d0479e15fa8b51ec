// One-token decode GEMV on quantized activations: the product a decode step
// runs once per projection (lab_gemm_q8 / lab_gemm_q4 with n = 1 on the
// previous projection's output, lab_native.c:553-579, 1059-1080), with its
// input as QA blocks (the 32 int8 and f32 scale of lab_quantize_q8 per 32
// values) and its outputs in f32 and/or QA blocks for the next product.
//
// Bit-exact with the reference. Every output is four f32 accumulator chains
// over the blocks in order, acc_l = fma(f32(d_l), f32(sw * sx), acc_l), d_l
// the int32 sum over bytes 4l..4l+3 of both 16-byte halves of the block,
// ending with (acc0 + acc1) + (acc2 + acc3) (lab_native.c:456-466, 503-512,
// 987-1002, 1025-1034). Here two threads share a weight row: thread h keeps
// chains 2h and 2h + 1, whose weights are the eight contiguous bytes 8h..8h+7
// of each 16-byte half of a Q8_0 block (of the 16-byte Q4_0 block: low
// nibbles weights 8h..8h+3 and 8h+4..8h+7 of the first half, high nibbles the
// same of the second). So a block costs a thread two 8-byte weight loads (one
// for Q4_0), one 16-byte activation load, four dp4a, one scale product for
// both chains and two fma, about a third of the instructions of one thread
// per chain, which matters because a decode projection is a chain of
// dependent launches whose length is set by each tile's serial work.
//
// Memory path as in gemv.cu: a persistent, warp-specialized kernel; each CTA
// owns 32-row tiles (one Q8_0 block of the output each) and a producer warp
// streams their weights through a shared-memory ring of 2-D TMA boxes (32
// rows x 128 bytes, 128-byte swizzle, and a 64-byte-swizzled box of the
// stage's scales) before the previous kernel has finished. Two consumer warps
// of 16 rows compute. After the dependent-launch wait the input vector comes
// in by one bulk copy and is rearranged so that thread h's four activation
// words of a block are one 16-byte load.
#include <stdlib.h>
#include <string.h>

#include "dn_common.cuh"
#include "dn_launch.h"
#include "dn_tmap.h"
#include "gemv_core.cuh"

namespace dn {
namespace {

using gemv::exact_d2;
using gemv::f2_hi;
using gemv::f2_lo;
using gemv::f2_mul;
using gemv::f2_pack;
using gemv::Fmt;
using gemv::kBox;
using gemv::kBoxBytes;
using gemv::kMagic;
using gemv::kMaxSmem;
using gemv::kMaxStages;
using gemv::kRows;
using gemv::kSMs;
using gemv::kSmemPerSM;
using gemv::kStageBytes;
using gemv::kWBoxes;
using gemv::lds;

constexpr int kCWarps = 2;                 // consumer warps, 16 rows each
constexpr int kCThreads = 32 * kCWarps;
constexpr int kThreads1 = kCThreads + 32;  // + the producer warp

// One block of the input in shared memory, per half h (chains 2h, 2h + 1):
// activation words 2h, 2h + 1, 4 + 2h, 5 + 2h (16 bytes); Q4 adds each
// chain's dp4a seed, kMagic - 8 * (sum of its eight int8), and a pad word
// pair (the unsigned nibbles n enter the dot product as n, the "- 8" through
// the seed).
template <bool Q4>
struct XH {
  static constexpr int kHalf = Q4 ? 32 : 16;
  static constexpr int kBlock = 2 * kHalf;
};

// Shared memory from a 1024-byte aligned base: the stages; `stages` full and
// `stages` empty barriers, two epilogue barriers and the input's barrier; the
// input blocks; their scales; the two warps' amax per epilogue buffer; the
// input's QA blocks as copied in.
struct Plan1 {
  int64_t bar_off, xw_off, xs_off, am_off, stg_off, total;
};

template <bool Q4>
__host__ __device__ inline Plan1 plan1(int stages, int64_t blocks) {
  Plan1 p;
  p.bar_off = (int64_t)stages * kStageBytes;
  p.xw_off = gemv::round_up(p.bar_off + 8 * (2 * stages + 4), 128);
  p.xs_off = p.xw_off + blocks * XH<Q4>::kBlock;
  p.am_off = gemv::round_up(p.xs_off + gemv::round_up(blocks, 4) * 4, 16);
  p.stg_off = p.am_off + 16;
  p.total = p.stg_off + gemv::round_up(blocks * kQABytes, 16) + 1024;
  return p;
}

// Shared-memory loads at a 32-bit shared address plus an immediate offset,
// so that a stage's loads need no address arithmetic beyond one base register
// per weight chunk (set once per stage).
template <int kOff>
__device__ __forceinline__ uint2 ld2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(addr), "n"(kOff));
  return v;
}
template <int kOff>
__device__ __forceinline__ uint4 ld4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+%5];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr), "n"(kOff));
  return v;
}
__device__ __forceinline__ uint2 ld2rt(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 ld4rt(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t ld1rt(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// Per-thread constants: thread (r, h) of the tile, r = 16 * warp + lane / 2.
struct Lane1 {
  uint32_t w[8];  // offset in a weight box of bytes 8h..8h+7 of 16-byte chunk k of row r (128-byte swizzle)
  uint32_t sc[4];  // offset in the stage of row r's chunk j of the 64-byte-swizzled scale box
  int r, h;
};

__device__ __forceinline__ Lane1 lane1(int warp, int lane) {
  Lane1 c;
  c.h = lane & 1;
  c.r = 16 * warp + (lane >> 1);
#pragma unroll
  for (int k = 0; k < 8; k++) c.w[k] = c.r * 128 + (((k ^ c.r) & 7) << 4) + 8 * c.h;
#pragma unroll
  for (int j = 0; j < 4; j++) c.sc[j] = kWBoxes * kBox + c.r * 64 + ((((c.r >> 1) ^ j) & 3) << 4);
  return c;
}

// c.w[k] and c.sc[j] for k, j known only at run time (indexing the arrays
// with one would move them to local memory).
__device__ __forceinline__ uint32_t w_off_rt(const Lane1& c, int k) {
  return c.r * 128 + (((k ^ c.r) & 7) << 4) + 8 * c.h;
}
__device__ __forceinline__ uint32_t sc_off_rt(const Lane1& c, int j) {
  return kWBoxes * kBox + c.r * 64 + ((((c.r >> 1) ^ j) & 3) << 4);
}

// One block's two chains, d seeded with kMagic (Q4: kMagic - 8 * sum(x)) so
// that the bits of d are the float 1.5 * 2^23 + dot, made exact by one f32
// subtraction. Q8: weight words (2h, 2h+1) of the first half in wa, (4+2h,
// 5+2h) of the second in wb. Q4: the eight nibble bytes in wa, the seeds in sd.
template <bool Q4>
__device__ __forceinline__ void block2(uint2 wa, uint2 wb, uint4 xv, uint2 sd, float s, float& a0,
                                       float& a1) {
  int32_t d0, d1;
  if (Q4) {
    d0 = __dp4a((int32_t)((wa.x >> 4) & 0x0f0f0f0fu), (int32_t)xv.z,
                __dp4a((int32_t)(wa.x & 0x0f0f0f0fu), (int32_t)xv.x, (int32_t)sd.x));
    d1 = __dp4a((int32_t)((wa.y >> 4) & 0x0f0f0f0fu), (int32_t)xv.w,
                __dp4a((int32_t)(wa.y & 0x0f0f0f0fu), (int32_t)xv.y, (int32_t)sd.y));
  } else {
    d0 = __dp4a((int32_t)wb.x, (int32_t)xv.z, __dp4a((int32_t)wa.x, (int32_t)xv.x, kMagic));
    d1 = __dp4a((int32_t)wb.y, (int32_t)xv.w, __dp4a((int32_t)wa.y, (int32_t)xv.y, kMagic));
  }
  a0 = __fmaf_rn(__fsub_rn(__int_as_float(d0), gemv::kMagicF), s, a0);
  a1 = __fmaf_rn(__fsub_rn(__int_as_float(d1), gemv::kMagicF), s, a1);
}

// A whole stage (Fmt<Q4>::kKC blocks) with its scales in the stage's scale
// box, straight-line. st: the stage's shared address; xh: this thread's half
// of the stage's first input block; xsa: that block's scale.
template <bool Q4>
__device__ __forceinline__ void stage_full1(uint32_t st, const Lane1& c, uint32_t xh, uint32_t xsa,
                                            float& a0, float& a1) {
  using X = XH<Q4>;
  uint32_t wk[8];
#pragma unroll
  for (int k = 0; k < 8; k++) wk[k] = st + c.w[k];
#pragma unroll
  for (int j = 0; j < kWBoxes; j++) {
    const uint4 sv = ld4rt(st + c.sc[j]);
    if (Q4) {
      const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
      const uint4 xa = j == 0 ? ld4<0>(xsa) : j == 1 ? ld4<32>(xsa) : j == 2 ? ld4<64>(xsa) : ld4<96>(xsa);
      const uint4 xb = j == 0 ? ld4<16>(xsa) : j == 1 ? ld4<48>(xsa) : j == 2 ? ld4<80>(xsa) : ld4<112>(xsa);
      const float xsv[8] = {__uint_as_float(xa.x), __uint_as_float(xa.y), __uint_as_float(xa.z),
                            __uint_as_float(xa.w), __uint_as_float(xb.x), __uint_as_float(xb.y),
                            __uint_as_float(xb.z), __uint_as_float(xb.w)};
#pragma unroll
      for (int bb = 0; bb < 8; bb++) {  // block within the box = 16-byte chunk
        const uint32_t xo = xh + (8 * j + bb) * X::kBlock;
        const float sw = half_bits_to_float((uint16_t)(u[bb >> 1] >> (16 * (bb & 1))));
        const uint2 w = ld2rt(wk[bb] + j * kBox);
        block2<true>(w, w, ld4rt(xo), ld2rt(xo + 16), __fmul_rn(sw, xsv[bb]), a0, a1);
      }
    } else {
      const uint4 x4 = j == 0 ? ld4<0>(xsa) : j == 1 ? ld4<16>(xsa) : j == 2 ? ld4<32>(xsa) : ld4<48>(xsa);
      const float sw[4] = {__uint_as_float(sv.x), __uint_as_float(sv.y), __uint_as_float(sv.z),
                           __uint_as_float(sv.w)};
      const float sx[4] = {__uint_as_float(x4.x), __uint_as_float(x4.y), __uint_as_float(x4.z),
                           __uint_as_float(x4.w)};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint2 wa = ld2rt(wk[2 * q] + j * kBox);
        const uint2 wb = ld2rt(wk[2 * q + 1] + j * kBox);
        const uint4 xv = ld4rt(xh + (4 * j + q) * X::kBlock);
        block2<false>(wa, wb, xv, make_uint2(0u, 0u), __fmul_rn(sw[q], sx[q]), a0, a1);
      }
    }
  }
}

// Any stage of nb blocks (a partial last stage).
template <bool Q4>
__device__ __forceinline__ void stage_part1(uint32_t st, int nb, const Lane1& c, uint32_t xh, uint32_t xsa,
                                            float& a0, float& a1) {
  using X = XH<Q4>;
  constexpr int kPerBox = kBoxBytes / Fmt<Q4>::kWB;
  for (int bb = 0; bb < nb; bb++) {
    const uint32_t box = st + (bb / kPerBox) * kBox;
    const int q = bb % kPerBox;
    const uint32_t sl = st + sc_off_rt(c, Q4 ? bb / 8 : bb / 4);
    const float sw = Q4 ? half_bits_to_float((uint16_t)(ld1rt(sl + (bb % 8) / 2 * 4) >> (16 * (bb & 1))))
                        : __uint_as_float(ld1rt(sl + (bb % 4) * 4));
    const float s = __fmul_rn(sw, __uint_as_float(ld1rt(xsa + bb * 4)));
    const uint32_t xo = xh + bb * X::kBlock;
    if (Q4) {
      const uint2 w = ld2rt(box + w_off_rt(c, q));
      block2<true>(w, w, ld4rt(xo), ld2rt(xo + 16), s, a0, a1);
    } else {
      block2<false>(ld2rt(box + w_off_rt(c, 2 * q)), ld2rt(box + w_off_rt(c, 2 * q + 1)), ld4rt(xo),
                    make_uint2(0u, 0u), s, a0, a1);
    }
  }
}

// The input's QA blocks, bulk-copied into shared memory (qa), into the
// layout above. One bulk copy per CTA is the fastest way in: the same few
// lines are read by every CTA of the launch, and per-thread loads of them
// measured up to twice as slow.
template <bool Q4>
__device__ __forceinline__ void unpack_qa1(const uint8_t* qa, int64_t blocks, uint8_t* xw, float* xs,
                                           int t) {
  using X = XH<Q4>;
  for (int64_t i = t; i < blocks * 2; i += kCThreads) {
    const int64_t b = i >> 1;
    const int h = (int)(i & 1);
    const uint8_t* src = qa + b * kQABytes;
    const uint32_t v0 = lds<uint32_t>(src + 8 * h), v1 = lds<uint32_t>(src + 8 * h + 4);
    const uint32_t v2 = lds<uint32_t>(src + 16 + 8 * h), v3 = lds<uint32_t>(src + 20 + 8 * h);
    uint8_t* dst = xw + b * X::kBlock + h * X::kHalf;
    *reinterpret_cast<uint4*>(dst) = make_uint4(v0, v1, v2, v3);
    if (Q4) {
      const int32_t s0 = kMagic - 8 * __dp4a((int32_t)v0, 0x01010101, __dp4a((int32_t)v2, 0x01010101, 0));
      const int32_t s1 = kMagic - 8 * __dp4a((int32_t)v1, 0x01010101, __dp4a((int32_t)v3, 0x01010101, 0));
      *reinterpret_cast<uint2*>(dst + 16) = make_uint2((uint32_t)s0, (uint32_t)s1);
    }
    if (h == 0) xs[b] = lds<float>(src + 32);
  }
}

template <bool Q4>
__global__ void __launch_bounds__(kThreads1, 4)
    gemv1_kernel(const GemvArgs a, const int stages, const __grid_constant__ CUtensorMap tw,
                 const __grid_constant__ CUtensorMap tsc, const __grid_constant__ CUtensorMap tw3,
                 const int wide) {
  using F = Fmt<Q4>;
  using X = XH<Q4>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t blocks = a.cols / kBlock;
  const int64_t ntiles = (a.rows + kRows - 1) / kRows;
  const int nch = (int)((blocks + F::kKC - 1) / F::kKC);
  const int64_t my_tiles = (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const Plan1 sp = plan1<Q4>(stages, blocks);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sp.bar_off);
  uint64_t* empty = full + stages;
  uint64_t* epi = empty + stages;
  uint64_t* xbar = epi + 2;
  uint64_t* gbar = xbar + 1;  // the fused all-gather: every consumer's stores are issued
  uint8_t* xw = smem + sp.xw_off;
  uint8_t* stg = smem + sp.stg_off;
  float* xs = reinterpret_cast<float*>(smem + sp.xs_off);
  float* am = reinterpret_cast<float*>(smem + sp.am_off);
  __shared__ volatile int abort_flag;

  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    mbar_init(&epi[0], kCThreads);
    mbar_init(&epi[1], kCThreads);
    mbar_init(xbar, 1);
    mbar_init(gbar, kCThreads);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kCWarps) {
    // ------------------------------------------------------------ producer
    // The weights do not depend on the previous kernel: no dependent-launch
    // wait here, so they stream while it finishes.
    if (lane == 0) {
      prefetch_tmap(wide ? &tw3 : &tw);
      prefetch_tmap(&tsc);
    }
    const int64_t total = my_tiles * nch;
    int64_t k = 0, tile = blockIdx.x;
    int s = 0, c = 0;
    uint32_t eph = 1;
    for (; k < total; k++) {
      if (k >= stages && !mbar_wait_bounded(&empty[s], eph, a.status, kStatusTmaTimeout)) abort_flag = 1;
      if (abort_flag) break;
      if (lane == 0) {
        const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
        uint8_t* stage = smem + (int64_t)s * kStageBytes;
        if (wide) {
          // The stage's four weight boxes in one copy (chunks past the row are
          // zero-filled and count in full), then its scales.
          mbar_arrive_expect_tx(&full[s], (uint32_t)(kStageBytes));
          tma_load_3d(stage, &tw3, 0, (int32_t)(tile * kRows), c * kWBoxes, &full[s]);
          tma_load_2d(stage + kWBoxes * kBox, &tsc, c * F::kKC, (int32_t)(tile * kRows), &full[s]);
        } else {
          gemv::issue_stage<Q4, true>(stage, &tw, &tsc, c, nb, (int32_t)(tile * kRows), &full[s]);
        }
      }
      __syncwarp();
      if (++s == stages) {
        s = 0;
        eph ^= 1u;
      }
      if (++c == nch) {
        c = 0;
        tile += gridDim.x;
      }
    }
    if (abort_flag && lane == 0) {
      // Let the copies still in flight land before the CTA's shared memory goes.
      for (int64_t j = k - 1; j >= 0 && j >= k - stages; j--)
        mbar_wait_bounded(&full[j % stages], (uint32_t)(j / stages) & 1u, a.status, kStatusTmaTimeout);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // The next product may start streaming its weights right away.
  pdl_launch_dependents();
  pdl_wait();  // the input comes from the previous kernel
  const int64_t in_bytes = blocks * kQABytes;
  if (((uintptr_t)a.xa & 15) == 0 && (in_bytes & 15) == 0) {
    if (tid == 0) {
      mbar_arrive_expect_tx(xbar, (uint32_t)in_bytes);
      bulk_g2s(stg, a.xa, (uint32_t)in_bytes, xbar);
    }
    if (!gemv::warp_wait(xbar, 0, a.status)) abort_flag = 1;
  } else {
    for (int64_t i = tid; i < in_bytes / 4; i += kCThreads)
      reinterpret_cast<uint32_t*>(stg)[i] = __ldcg(reinterpret_cast<const uint32_t*>(a.xa) + i);
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory");  // every consumer thread gets here
  if (abort_flag) return;
  unpack_qa1<Q4>(stg, blocks, xw, xs, tid);
  asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory");

  const Lane1 c = lane1(warp, lane);
  const int nfull = (int)(blocks / F::kKC);
  const uint32_t smem32 = smem_u32(smem);
  const uint32_t xw32 = smem_u32(xw) + c.h * X::kHalf, xs32 = smem_u32(xs);
  int s = 0;
  uint32_t ph = 0, e = 0;
  for (int64_t i = 0; i < my_tiles; i++) {
    const int64_t tile = blockIdx.x + i * gridDim.x;
    float a0 = 0.0f, a1 = 0.0f;
    uint32_t xwp = xw32, xsp = xs32;
    int ch = 0;
    for (; ch < nfull; ch++) {
      if (!gemv::warp_wait(&full[s], ph, a.status)) {
        abort_flag = 1;
        return;  // the producer drains what it issued; every other wait is bounded
      }
      stage_full1<Q4>(smem32 + (uint32_t)s * kStageBytes, c, xwp, xsp, a0, a1);
      xwp += F::kKC * X::kBlock;
      xsp += F::kKC * 4;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    for (; ch < nch; ch++) {
      if (!gemv::warp_wait(&full[s], ph, a.status)) {
        abort_flag = 1;
        return;
      }
      const int nb = (int)min64(F::kKC, blocks - (int64_t)ch * F::kKC);
      stage_part1<Q4>(smem32 + (uint32_t)s * kStageBytes, nb, c, xwp, xsp, a0, a1);
      xwp += F::kKC * X::kBlock;
      xsp += F::kKC * 4;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    // (acc0 + acc1) + (acc2 + acc3): each thread its pair, then the partner's
    // (an f32 add is commutative, so both threads of a row hold the same y).
    const float p = __fadd_rn(a0, a1);
    const float o = __shfl_xor_sync(0xffffffffu, p, 1);
    const float y = c.h == 0 ? __fadd_rn(p, o) : __fadd_rn(o, p);
    const int tile_rows = (int)min64(kRows, a.rows - tile * kRows);
    if (c.h == 0 && c.r < tile_rows && a.ys != nullptr) a.ys[tile * kRows + c.r] = y;
    if (c.h == 0 && c.r < tile_rows) {
      // The fused all-gather: the row into every rank's copy of the output.
      for (int p = 0; p < a.gather_n; p++) a.gather_ys[p][a.gather_row0 + tile * kRows + c.r] = y;
    }
    if (a.ya != nullptr && tile_rows == kRows) {
      // The tile's 32 outputs are one Q8_0 block of the next product's input
      // (lab_quantize_q8 semantics): the two warps' amax meet in shared
      // memory behind a bounded barrier, whose buffer alternates.
      float m = fmaxf(0.0f, fabsf(y));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      float* amb = am + (e & 1) * 2;
      if (lane == 0) amb[warp] = m;
      mbar_arrive(&epi[e & 1]);
      if (!gemv::warp_wait(&epi[e & 1], (e >> 1) & 1u, a.status)) {
        abort_flag = 1;
        return;
      }
      float scale, inv;
      q8_scale(fmaxf(amb[0], amb[1]), scale, inv);
      uint8_t* dst = a.ya + tile * kQABytes;
      if (c.h == 0) dst[c.r] = (uint8_t)(int8_t)quant_q8_elem(y, inv);
      if (tid == 0) *reinterpret_cast<float*>(dst + 32) = scale;
      e++;
    }
  }
  if (a.gather_n > 0) {
    // Every consumer's stores of this CTA (a bounded barrier: a warp that
    // gave up never arrives), then one system-scope fence and the CTA's tile
    // count into every rank's counter (the waiting side acquires).
    mbar_arrive(gbar);
    const bool all = tid >= 32 || gemv::warp_wait(gbar, 0, a.status);
    if (tid == 0 && all && !abort_flag) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int p = 0; p < a.gather_n; p++)
        asm volatile("red.relaxed.sys.global.add.s32 [%0], %1;" ::"l"(a.gather_cnt[p]), "r"((int)my_tiles)
                     : "memory");
    }
  }
}

__global__ void peer_wait_kernel(const int* cnt, int* expect, int count, uint32_t* status) {
  const int target = *expect + count;
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
  if (v - target < 0) {
    const uint64_t start = globaltimer_ns();
    for (uint32_t i = 1;; i++) {
      __nanosleep(64);
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
      if (v - target >= 0) break;
      if ((i & 63u) == 0 && globaltimer_ns() - start > wait_limit_ns()) {
        report(status, kStatusPeerTimeout);
        break;
      }
    }
  }
  *expect = target;
}

// DN_WIDE_COPIES=0 loads a stage as four 2-D boxes instead of one 3-D copy.
bool wide_copies() {
  static const bool on = [] {
    const char* e = getenv("DN_WIDE_COPIES");
    return e == nullptr || atoi(e) != 0;
  }();
  return on;
}

template <bool Q4>
int64_t launch1(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  using F = Fmt<Q4>;
  const int64_t ntiles = (a.rows + kRows - 1) / kRows;
  const int64_t blocks = a.cols / kBlock;
  const int nch = (int)((blocks + F::kKC - 1) / F::kKC);
  const Plan1 base = plan1<Q4>(0, blocks);
  // One CTA per SM when the tiles fit one wave (each CTA holds all of its
  // stages), two otherwise; the ring never holds more stages than the CTA
  // loads, so the next kernel's CTAs find room and start streaming early.
  const int per_sm = ntiles <= kSMs ? 1 : 2;
  const int64_t slots = (int64_t)kSMs * per_sm;
  const int64_t grid = ntiles < slots ? ntiles : slots;
  const int64_t waves = (ntiles + slots - 1) / slots;
  const int64_t budget = per_sm == 1 ? kMaxSmem : kSmemPerSM / 2 - 1024;
  int64_t stages = (budget - base.total) / (kStageBytes + 16);
  stages = stages > kMaxStages ? kMaxStages : stages;
  const int64_t chunks = waves * nch;
  if (chunks < stages) stages = chunks < 2 ? 2 : chunks;
  if (stages < 2) return kErrTooLarge;
  const Plan1 sp = plan1<Q4>((int)stages, blocks);
  if (sp.total > kMaxSmem) return kErrTooLarge;
  CUtensorMap tw, tsc;
  const uint64_t row_bytes = (uint64_t)blocks * F::kWB;
  if (!encode_tmap_2d(&tw, a.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, row_bytes, (uint64_t)a.rows, row_bytes,
                      kBoxBytes, kRows, true) ||
      !encode_tmap_2d_sw64(&tsc, a.scales,
                           Q4 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                           (uint64_t)blocks, (uint64_t)a.rows, (uint64_t)blocks * F::kSB, F::kKC, kRows))
    return kErrUnsupported;
  // Whole stages in one copy where the rows are whole 128-byte chunks.
  CUtensorMap tw3 = tw;
  int wide = wide_copies() && encode_tmap_row_chunks(&tw3, a.qs, (uint64_t)a.rows, row_bytes, kRows, kWBoxes) ? 1 : 0;
  const void* kern = reinterpret_cast<const void*>(gemv1_kernel<Q4>);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess)
      return kErrCuda;
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads1, 1, 1);
  cfg.dynamicSmemBytes = (size_t)sp.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GemvArgs args = a;
  int nstages = (int)stages;
  void* params[] = {&args, &nstages, &tw, &tsc, &tw3, &wide};
  return cudaLaunchKernelExC(&cfg, kern, params) == cudaSuccess ? kOk : kErrCuda;
}

// Plain one-token products run on the general GEMV kernel (gemv.cu) unless
// DN_GEMV1=1: chained the way a decode step chains them, that kernel measured
// 1704 against this one's 1658 tokens/s on the config-3 stack, although this
// one is faster launch for launch on one shape. This kernel is the one that
// fuses the all-gather (gather_n > 0), which it always serves.
bool gemv1_enabled() {
  static const bool on = [] {
    const char* e = getenv("DN_GEMV1");
    return e != nullptr && atoi(e) != 0;
  }();
  return on;
}

}  // namespace

// One token, QA input, plain outputs (f32 and/or QA), scales the TMA can
// address (16-byte aligned arrays, rows a multiple of 16 bytes).
bool gemv1_eligible(const GemvArgs& g) {
  if (!gemv1_enabled() && g.gather_n == 0) return false;
  if (g.gather_n < 0 || g.gather_n > kMaxGatherRanks) return false;
  for (int p = 0; p < g.gather_n; p++)
    if (g.gather_ys[p] == nullptr || g.gather_cnt[p] == nullptr || ((uintptr_t)g.gather_ys[p] & 3) != 0 ||
        ((uintptr_t)g.gather_cnt[p] & 3) != 0)
      return false;
  if (g.n != 1 || g.xa == nullptr || g.xs != nullptr || g.groups > 1 || g.qs2 != nullptr ||
      g.glu_out != nullptr || g.res != nullptr || g.norm_w != nullptr || g.xa_out != nullptr)
    return false;
  const int64_t blocks = g.cols / kBlock;
  if (g.cols <= 0 || g.cols % kBlock != 0 || ((uintptr_t)g.qs & 15) != 0 ||
      ((uintptr_t)g.scales & 15) != 0 || (blocks * (g.q4 ? 2 : 4)) % 16 != 0 ||
      ((uintptr_t)g.xa & 3) != 0 || (g.ya != nullptr && ((uintptr_t)g.ya & 3) != 0) ||
      (g.ys != nullptr && ((uintptr_t)g.ys & 3) != 0))
    return false;
  return (g.q4 ? plan1<true>(2, blocks).total : plan1<false>(2, blocks).total) <= kMaxSmem;
}

int64_t launch_gemv1(const GemvArgs& g, cudaStream_t stream, bool pdl) {
  if (g.rows <= 0) return kOk;
  return g.q4 ? launch1<true>(g, stream, pdl) : launch1<false>(g, stream, pdl);
}

cudaError_t launch_peer_wait(const int* cnt, int* expect, int count, uint32_t* status, cudaStream_t stream) {
  peer_wait_kernel<<<1, 1, 0, stream>>>(cnt, expect, count, status);
  return cudaGetLastError();
}

}  // namespace dn
