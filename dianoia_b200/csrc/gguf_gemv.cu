// One-token decode GEMV straight on GGUF Q8_0 / Q4_0 blocks: the weights stay
// in the file's interleaved layout (Q8_0: an fp16 scale then 32 int8, 34
// bytes; Q4_0: an fp16 scale then 16 bytes of nibbles, 18 bytes - weight k of
// a block in the low nibble of byte k, k + 16 in the high nibble), so a
// loader needs neither dianoia's CPU split (gguf.dart:206-215 splitQ4_0,
// 269-283 splitQ8_0) nor dn_gguf_split's device copy before the products.
//
// Results equal lab_gemm_q8 / lab_gemm_q4 (mode 1, n = 1, lab_native.c:553-
// 579, 1059-1080) on the split weights, bit for bit: the Q8_0 scale widens
// exactly to the f32 the split would store, the Q4_0 one is used as fp16 as
// the split keeps it, and each row runs the reference's four accumulators in
// block order, acc_l = fma(f32(d_l), f32(sw * sx), acc_l), ending with (acc0 +
// acc1) + (acc2 + acc3) (lab_native.c:456-466, 987-1002). Four lanes per row,
// eight rows per warp, as in the other decode kernels; d_l comes from a dp4a
// chain seeded with 0x4B400000 and one exact subtraction.
//
// Memory path: a persistent, warp-specialized kernel; a CTA owns 32-row tiles
// and a producer warp streams them through a shared-memory ring, one 2-D TMA
// copy per stage: 32 rows x 8 Q8_0 blocks (272 bytes) or 16 Q4_0 blocks (288
// bytes), the tensor map's element a 16-bit word so a stage's row is one box
// line. Blocks are only 2-byte aligned: in a pair of blocks (68 or 36 bytes,
// 4-byte aligned) the odd block's values are word-aligned and the even
// block's are two bytes off, so a lane forms each of its even-block words
// from two aligned shared-memory words (one byte permute).
#include <stdlib.h>
#include <string.h>

#include "dn_common.cuh"
#include "dn_launch.h"
#include "dn_tmap.h"
#include "gemv_core.cuh"
#include "quaddot.cuh"

namespace dn {
namespace {

using gemv::exact_d2;
using gemv::f2_hi;
using gemv::f2_lo;
using gemv::f2_mul;
using gemv::f2_pack;
using gemv::kMagic;
using gemv::kMaxSmem;
using gemv::kSMs;
using gemv::kSmemPerSM;
using gemv::lds;

constexpr int kTRows = 32;                // rows per tile
constexpr int kCWarps = 4;                // consumer warps, 8 rows each
constexpr int kCThreads = 32 * kCWarps;
constexpr int kThreads = kCThreads + 32;  // + the producer warp
constexpr int kMaxStages = 16;

template <bool Q4>
struct GG {
  static constexpr int kBlockBytes = Q4 ? 18 : 34;
  static constexpr int kBlocks = Q4 ? 16 : 8;               // blocks per stage
  static constexpr int kRowBytes = kBlocks * kBlockBytes;   // 288 / 272: one box line
  static constexpr int kBoxElems = kRowBytes / 2;           // 16-bit words
  static constexpr int kStageBytes = (kTRows * kRowBytes + 1023) / 1024 * 1024;
  static constexpr int kXBlock = Q4 ? 64 : 32;              // activation bytes per block (quaddot layout)
};

// Shared memory from a 1024-byte aligned base: the stages; full and empty
// barriers; the activations (lane-interleaved) and their block scales.
struct Plan {
  int64_t bar_off, xw_off, xs_off, total;
};
template <bool Q4>
__host__ __device__ inline Plan plan(int stages, int64_t blocks) {
  Plan p;
  p.bar_off = (int64_t)stages * GG<Q4>::kStageBytes;
  p.xw_off = gemv::round_up(p.bar_off + 16 * stages, 128);
  p.xs_off = p.xw_off + blocks * GG<Q4>::kXBlock;
  p.total = gemv::round_up(p.xs_off + blocks * 4, 16) + 1024;  // + alignment slack
  return p;
}

// Bytes 2..5 of the pair (lo, hi): the word that starts two bytes into lo.
__device__ __forceinline__ uint32_t off2(uint32_t lo, uint32_t hi) { return __byte_perm(lo, hi, 0x5432); }

// One pair of blocks (b, b + 1) of row r, lane l: weight words, scales, then
// the two fma steps. pr: the pair's 4-byte aligned start in the stage; xb:
// the lane's activation slot of block b; sx2: the two activation scales.
template <bool Q4>
__device__ __forceinline__ void pair_step(const uint8_t* pr, int l, const uint8_t* xb, float2 sx2, float& acc) {
  int32_t d0, d1;
  float sw0, sw1;
  if (Q4) {
    // Even block: scale at 0, nibbles at 2..17; odd: scale at 18, nibbles at 20..35.
    const uint32_t w0 = off2(lds<uint32_t>(pr + 4 * l), lds<uint32_t>(pr + 4 * l + 4));
    const uint32_t w1 = lds<uint32_t>(pr + 20 + 4 * l);
    sw0 = half_bits_to_float(lds<uint16_t>(pr));
    sw1 = half_bits_to_float(lds<uint16_t>(pr + 18));
    const uint4 x0 = lds<uint4>(xb), x1 = lds<uint4>(xb + 64);
    d0 = __dp4a((int32_t)((w0 >> 4) & 0x0f0f0f0fu), (int32_t)x0.y,
                __dp4a((int32_t)(w0 & 0x0f0f0f0fu), (int32_t)x0.x, (int32_t)x0.z + kMagic));
    d1 = __dp4a((int32_t)((w1 >> 4) & 0x0f0f0f0fu), (int32_t)x1.y,
                __dp4a((int32_t)(w1 & 0x0f0f0f0fu), (int32_t)x1.x, (int32_t)x1.z + kMagic));
  } else {
    // Even block: scale at 0, values at 2..33; odd: scale at 34, values at 36..67.
    const uint32_t a0 = off2(lds<uint32_t>(pr + 4 * l), lds<uint32_t>(pr + 4 * l + 4));
    const uint32_t a1 = off2(lds<uint32_t>(pr + 16 + 4 * l), lds<uint32_t>(pr + 20 + 4 * l));
    const uint32_t b0 = lds<uint32_t>(pr + 36 + 4 * l), b1 = lds<uint32_t>(pr + 52 + 4 * l);
    sw0 = half_bits_to_float(lds<uint16_t>(pr));
    sw1 = half_bits_to_float(lds<uint16_t>(pr + 34));
    const uint2 x0 = lds<uint2>(xb), x1 = lds<uint2>(xb + 32);
    d0 = __dp4a((int32_t)a1, (int32_t)x0.y, __dp4a((int32_t)a0, (int32_t)x0.x, kMagic));
    d1 = __dp4a((int32_t)b1, (int32_t)x1.y, __dp4a((int32_t)b0, (int32_t)x1.x, kMagic));
  }
  const uint64_t dd = exact_d2(d0, d1);
  const uint64_t ss = f2_mul(f2_pack(sw0, sw1), f2_pack(sx2.x, sx2.y));
  acc = __fmaf_rn(f2_lo(dd), f2_lo(ss), acc);
  acc = __fmaf_rn(f2_hi(dd), f2_hi(ss), acc);
}

template <bool Q4>
__global__ void __launch_bounds__(kThreads, 2)
    gguf_gemv_kernel(const uint8_t* xa, float* ys, const int64_t rows, const int64_t cols, const int stages,
                     const __grid_constant__ CUtensorMap tw, uint32_t* status) {
  using G = GG<Q4>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t blocks = cols / kBlock;
  const int nst = (int)(blocks / G::kBlocks);
  const int64_t ntiles = (rows + kTRows - 1) / kTRows;
  const int64_t my_tiles = (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const Plan pl = plan<Q4>(stages, blocks);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pl.bar_off);
  uint64_t* empty = full + stages;
  uint8_t* xw = smem + pl.xw_off;
  float* xs = reinterpret_cast<float*>(smem + pl.xs_off);
  __shared__ volatile int abort_flag;

  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kCWarps) {
    // ------------------------------------------------------------ producer
    // The weights do not depend on the previous kernel: they stream while it
    // finishes.
    if (lane == 0) {
      prefetch_tmap(&tw);
      const int64_t total = my_tiles * nst;
      int64_t k = 0, tile = blockIdx.x;
      int s = 0, c = 0;
      uint32_t eph = 1;
      for (; k < total; k++) {
        if (k >= stages && (abort_flag || !mbar_wait_bounded(&empty[s], eph, status, kStatusTmaTimeout))) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], (uint32_t)(kTRows * G::kRowBytes));
        tma_load_2d(smem + (int64_t)s * G::kStageBytes, &tw, c * G::kBoxElems, (int32_t)(tile * kTRows), &full[s]);
        if (++s == stages) {
          s = 0;
          eph ^= 1u;
        }
        if (++c == nst) {
          c = 0;
          tile += gridDim.x;
        }
      }
      if (abort_flag) {
        // Let the copies still in flight land before the CTA's shared memory goes.
        for (int64_t j = k - 1; j >= 0 && j >= k - stages; j--)
          mbar_wait_bounded(&full[j % stages], (uint32_t)(j / stages) & 1u, status, kStatusTmaTimeout);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_launch_dependents();
  pdl_wait();  // the input comes from the previous kernel
  // The QA blocks, read through L2, into the lane-interleaved layout (Q4:
  // with each lane's seed).
  quad::load_unpack<Q4>(xa, blocks, xw, xs, tid, kCThreads);
  asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory");

  const int r = 8 * warp + (lane >> 2), l = lane & 3;
  const uint8_t* xw_l = xw + l * (Q4 ? 16 : 8);
  int s = 0;
  uint32_t ph = 0;
  for (int64_t i = 0; i < my_tiles; i++) {
    const int64_t tile = blockIdx.x + i * gridDim.x;
    float acc = 0.0f;
    for (int c = 0; c < nst; c++) {
      if (!gemv::warp_wait(&full[s], ph, status)) {
        abort_flag = 1;
        return;  // the producer drains what it issued; every other wait is bounded
      }
      const uint8_t* row = smem + (int64_t)s * G::kStageBytes + r * G::kRowBytes;
      const int b0 = c * G::kBlocks;
#pragma unroll
      for (int p = 0; p < G::kBlocks / 2; p++)
        pair_step<Q4>(row + p * 2 * G::kBlockBytes, l, xw_l + (b0 + 2 * p) * G::kXBlock,
                      lds<float2>(xs + b0 + 2 * p), acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    const float y = gemv::lane_reduce(acc);  // (acc0 + acc1) + (acc2 + acc3) on l == 0
    const int64_t row = tile * kTRows + r;
    if (l == 0 && row < rows) ys[row] = y;
  }
}

template <bool Q4>
int64_t launch_t(const uint8_t* blocks_ptr, const uint8_t* xa, float* ys, int64_t rows, int64_t cols,
                 uint32_t* status, cudaStream_t stream, bool pdl) {
  using G = GG<Q4>;
  const int64_t blocks = cols / kBlock;
  const int64_t ntiles = (rows + kTRows - 1) / kTRows;
  const int nst = (int)(blocks / G::kBlocks);
  const int per_sm = ntiles <= kSMs ? 1 : 2;
  const int64_t slots = (int64_t)kSMs * per_sm;
  const int64_t grid = ntiles < slots ? ntiles : slots;
  const int64_t budget = per_sm == 1 ? kMaxSmem : kSmemPerSM / 2 - 1024;
  const Plan base = plan<Q4>(0, blocks);
  int64_t stages = (budget - base.total) / (G::kStageBytes + 16);
  stages = stages > kMaxStages ? kMaxStages : stages;
  const int64_t loads = ((ntiles + grid - 1) / grid) * nst;  // stages the busiest CTA loads
  if (loads < stages) stages = loads < 2 ? 2 : loads;
  if (stages < 2) return kErrTooLarge;
  const Plan sp = plan<Q4>((int)stages, blocks);
  if (sp.total > kMaxSmem) return kErrTooLarge;
  CUtensorMap tw;
  if (!encode_tmap_2d(&tw, blocks_ptr, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)(blocks * G::kBlockBytes / 2),
                      (uint64_t)rows, (uint64_t)(blocks * G::kBlockBytes), G::kBoxElems, kTRows, false))
    return kErrUnsupported;
  const void* kern = reinterpret_cast<const void*>(gguf_gemv_kernel<Q4>);
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
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)sp.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nstages = (int)stages;
  int64_t r = rows, c = cols;
  void* params[] = {&xa, &ys, &r, &c, &nstages, &tw, &status};
  return cudaLaunchKernelExC(&cfg, kern, params) == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace

int64_t launch_gguf_gemv(bool q4, const void* blocks, const uint8_t* xa, float* ys, int64_t rows, int64_t cols,
                         uint32_t* status, cudaStream_t stream, bool pdl) {
  const int64_t per_stage = q4 ? GG<true>::kBlocks : GG<false>::kBlocks;
  if (rows < 0 || cols <= 0 || cols % (kBlock * per_stage) != 0 || cols > (1 << 20) || blocks == nullptr ||
      xa == nullptr || ys == nullptr || ((uintptr_t)blocks & 15) != 0 || ((uintptr_t)xa & 3) != 0 ||
      ((uintptr_t)ys & 3) != 0)
    return kErrArgs;
  if (rows == 0) return kOk;
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  return q4 ? launch_t<true>(b, xa, ys, rows, cols, status, stream, pdl)
            : launch_t<false>(b, xa, ys, rows, cols, status, stream, pdl);
}

}  // namespace dn
