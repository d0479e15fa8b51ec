// Prefill / vision GEMM on the 5th-generation tensor cores (tcgen05, kind::i8)
// for Q8_0 and Q4_0 weights times Q8_0 activations (lab_gemm_q8 / lab_gemm_q4
// with many tokens, lab_native.c:553-579, 1059-1080).
//
// One tcgen05.mma of K = 32 int8 is exactly one Q8_0 block: D_b[r, t] =
// sum_k W[r, k] * xq[t, k] over block b, in int32 in TMEM - bit-exact block
// dots. Every block has its own scale product sw[r, b] * sx[t, b], so each
// block's D tile must leave TMEM and be scaled and accumulated in f32 on the
// CUDA cores (acc += f32(d) * f32(sw * sx), the reference's per-block
// operations). The f32 sums therefore run over whole blocks rather than the
// reference's four lanes, and match it within its own 1e-5 relative bound.
//
// Tile: 128 weight rows (MMA M, TMEM lanes) x 64 tokens (MMA N, TMEM
// columns); TMEM holds 8 such D slots, so the MMA warp runs two stages (8
// blocks) ahead of the drain. Warp roles:
//   warp 0      producer: per stage, TMA copies of the weights (Q8: a 128 x
//               128-byte box, 128-byte swizzle = the UMMA K-major SW128
//               layout; Q4: the raw 128 x 64-byte nibbles), the activations
//               (64 tokens x 128 bytes, SW128) and both block-scale boxes
//               for 4 blocks of K, all completing on one mbarrier. (Shapes
//               whose scale rows TMA cannot address - blocks per row not a
//               multiple of 4 (Q8) or 8 (Q4), or unaligned scale arrays -
//               stage the scales with per-lane cp.async copies instead, a
//               path several times slower per stage.)
//   warp 1      MMA issuer: allocates 512 TMEM columns = eight D slots of 64
//               columns; transposes the stage's activation scales to the
//               block-major order the drain reads; from an elected lane
//               issues the stage's MMAs (one per block, each into its own D
//               slot) and commits the stage to its "dready" barrier. A
//               stage's slots are reused two stages later, once the drain
//               has released that stage: one handshake per stage each way,
//               since every mbarrier operation costs far more than the math
//               it guards
//   warps 2-17  drain ("epilogue"): four warps per TMEM lane quarter (even
//               or odd blocks x low or high 32 token columns), each owning
//               one weight row per lane; per block a TMEM load, then the
//               scale-and-accumulate in packed f32x2 math
//   warps 18-19 (Q4) nibble expansion: raw nibbles -> int8 (q - 8) in the
//               SW128 K-major layout the MMA reads
// Every mbarrier wait is bounded; on a timeout the kernel records it, lets
// its copies and MMAs finish (bounded), frees its TMEM and returns.
#include <string.h>

#include <type_traits>

#include "dn_common.cuh"
#include "dn_launch.h"
#include "dn_tmap.h"

namespace dn {
namespace {

constexpr int kTileRows = 128;                 // MMA M
constexpr int kTileTok = 64;                   // MMA N
constexpr int kStageK = 128;                   // int8 of K per stage = 4 blocks
constexpr int kBlocksPerStage = kStageK / kBlock;
constexpr int kABytes = kTileRows * kStageK;   // 16 KB
constexpr int kBBytes = kTileTok * kStageK;    // 8 KB
constexpr int kRawBytes = kTileRows * (kStageK / 2);  // Q4 nibbles: 8 KB
constexpr int kEpiWarps = 16;
constexpr int kConvWarps = 2;
constexpr int kEpiCols = kTileTok * 8 / kEpiWarps;  // token columns per drain warp (32 or 64)
static_assert(kEpiCols % 32 == 0 && kEpiCols <= kTileTok, "whole 32-column TMEM loads");
constexpr uint32_t kTmemCols = 512;
constexpr int kSlots = (int)kTmemCols / kTileTok;  // D slots: blocks in flight between MMA and drain
constexpr int kMaxSmemTc = 226 * 1024;

// The odd-block drain warps hand their f32 sums to the even ones here:
// 128 rows x 64 tokens.
constexpr int kXchgBytes = kTileRows * kTileTok * 4;
constexpr int kSxBytes = kBlocksPerStage * kTileTok * 4;   // activation scales, block-major
constexpr int kSwBytes = kTileRows * kBlocksPerStage * 4;   // weight scales, row-major (f32)

template <bool Q4>
struct TcShape {
  static constexpr int kWarps = 2 + kEpiWarps + (Q4 ? kConvWarps : 0);
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kRawOff = kABytes + kBBytes;
  static constexpr int kSxOff = kRawOff + (Q4 ? kRawBytes : 0);
  static constexpr int kSwOff = kSxOff + kSxBytes;
  static constexpr int kSxbOff = kSwOff + kSwBytes;   // block-major copy of sx (TMA scales)
  static constexpr int kStageBytes = kSxbOff + kSxBytes;
  static_assert(kStageBytes % 1024 == 0, "SW128 operand tiles need 1024-byte aligned stages");
};

struct TcArgs {
  const void* scales;
  const float* xsc;
  float* ys;
  int64_t rows, cols, n, ldy;
  uint32_t* status;
  int tma_scales;  // scales arrive by TMA (tsw, tsx) rather than cp.async
  int64_t row_tiles, tiles;  // the narrow kernel's tile walk
};

// The kernels' arguments when the all-gather of a row-sharded output is
// fused into the epilogue (a compile-time variant; the plain kernels take
// TcArgs itself, unchanged): this GPU's rows are rows gather_row0 .. + rows
// of the whole output, and each value goes to every rank's copy of it,
// gather_ys[p][t * ldy + gather_row0 + row] (plain stores, over NVLink for
// the peers); peer_signal_kernel then counts the product on every rank.
struct TcGatherArgs : TcArgs {
  int gather_n;
  int64_t gather_row0;
  float* gather_ys[kMaxGatherRanks];
};
template <bool GATHER>
using TcArgsOf = typename std::conditional<GATHER, TcGatherArgs, TcArgs>::type;

// ----------------------------------------------------------- tcgen05 PTX

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] = A * B (+ D when `accumulate`): one K = 32 step of int8 x int8
// -> s32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The Q4 kernel seeds every D slot with this int32 and accumulates onto it:
// 0x4B400000 + d, read as a float, is 1.5 * 2^23 + d exactly for |d| < 2^22,
// so the tensor core's own int32 sum does the first step of the exact
// int -> float conversion and the drain skips an integer add per value. (The
// Q8 kernel, with fewer registers to spare per thread, adds the seed itself.)
constexpr uint32_t kSeed = 0x4B400000u;
// 32 lanes x 32 consecutive 32-bit columns of TMEM set to `v` (four stores
// of 8 columns: a store reads its values from consecutive registers).
__device__ __forceinline__ void tmem_fill32(uint32_t taddr, uint32_t v) {
#pragma unroll
  for (int c = 0; c < 32; c += 8)
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(
                     taddr + (uint32_t)c),
                 "r"(v)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// The mbarrier arrives once every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// Waits for this thread's TMEM loads, tied to the registers an earlier
// tcgen05.ld writes, so the compiler cannot move their reads above it.
__device__ __forceinline__ void tmem_wait_ld_regs(int32_t (&v)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]),
        "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]),
        "+r"(v[14]), "+r"(v[15]), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]),
        "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]),
        "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
      :
      : "memory");
}
// Asynchronous global -> shared copy of `bytes` (4, 8 or 16); fewer source
// bytes (`src_bytes`, possibly 0) zero-fill the rest without reading them.
__device__ __forceinline__ void cp_async(void* dst, const void* src, int bytes, int src_bytes) {
  if (bytes == 16)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes) : "memory");
  else if (bytes == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes) : "memory");
}
// Arrives on the mbarrier once this thread's earlier cp.async copies landed
// (the arrival counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major, 128-byte-swizzled operand
// tile whose rows are 128 bytes: 8-row groups 1024 bytes apart (SBO), version
// 1, layout SWIZZLE_128B. `addr` may be advanced by 32 bytes within the
// swizzle span to select a K = 32 step.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: s32 accumulator, signed int8 A and B, both K-major,
// N = 64, M = 128.
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileTok >> 3) << 17) |
                              ((uint32_t)(kTileRows >> 4) << 24);

// Packed f32x2 arithmetic (sm_100): two lanes of float math per instruction.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
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
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// Two int32 block dots (|d| < 2^22) as floats, exactly, from slot values that
// hold 0x4B400000 + d (seeded slots) or d: the bits 0x4B400000 + d are the
// float 1.5 * 2^23 + d, and subtracting 1.5 * 2^23 is exact. One packed float
// add per pair (and an integer add per value for unseeded slots), instead of
// the slower int-to-float conversion.
template <bool kSeeded>
__device__ __forceinline__ uint64_t slot_to_f2(int32_t v0, int32_t v1) {
  const uint32_t b0 = kSeeded ? (uint32_t)v0 : (uint32_t)(v0 + (int32_t)kSeed);
  const uint32_t b1 = kSeeded ? (uint32_t)v1 : (uint32_t)(v1 + (int32_t)kSeed);
  return f2_add((uint64_t)b0 | ((uint64_t)b1 << 32), f2_pack(-12582912.0f, -12582912.0f));
}

__device__ __forceinline__ bool wait_tc(uint64_t* bar, uint32_t parity, uint32_t* status,
                                        uint32_t bits, volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (!mbar_wait_bounded(bar, parity, status, bits)) {
    *abort_flag = 1;
    return false;
  }
  return true;
}

// kPartial: all tokens in one partial tile (n < 64), and drain warps whose
// token columns are all beyond n skip their work.
template <bool Q4, bool kPartial, bool GATHER = false>
__global__ void __launch_bounds__(TcShape<Q4>::kThreads, 1)
    gemm_tc_kernel(const TcArgsOf<GATHER> a, const int stages, const __grid_constant__ CUtensorMap tw,
                   const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tsw,
                   const __grid_constant__ CUtensorMap tsx) {
  using S = TcShape<Q4>;
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* smem = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  float* xchg = reinterpret_cast<float*>(smem + (int64_t)stages * S::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (int64_t)stages * S::kStageBytes + kXchgBytes);
  uint64_t* conv = full + stages;
  uint64_t* empty = conv + stages;
  uint64_t* dready = empty + stages;
  uint64_t* tinit = dready + stages;
  uint64_t* done = tinit + 1;
  uint64_t* xbar = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 1);
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t blocks = a.cols / kBlock;
  const int nst = (int)((blocks + kBlocksPerStage - 1) / kBlocksPerStage);
  const int64_t row0 = (int64_t)blockIdx.x * kTileRows;
  const int64_t tok0 = (int64_t)blockIdx.y * kTileTok;
  auto stage_a = [&](int s) { return smem + (int64_t)s * S::kStageBytes; };
  auto stage_b = [&](int s) { return smem + (int64_t)s * S::kStageBytes + kABytes; };
  auto stage_raw = [&](int s) { return smem + (int64_t)s * S::kStageBytes + S::kRawOff; };
  auto stage_sx = [&](int s) { return reinterpret_cast<float*>(smem + (int64_t)s * S::kStageBytes + S::kSxOff); };
  auto stage_sw = [&](int s) { return reinterpret_cast<float*>(smem + (int64_t)s * S::kStageBytes + S::kSwOff); };
  auto stage_sxb = [&](int s) { return reinterpret_cast<float*>(smem + (int64_t)s * S::kStageBytes + S::kSxbOff); };
  const bool tma_scales = a.tma_scales != 0;

  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      // TMA bytes (+ the producer lanes' cp.async scale copies on that path)
      mbar_init(&full[s], tma_scales ? 1 : 1 + 32);
      mbar_init(&conv[s], kConvWarps * 32);
      mbar_init(&empty[s], 1 + kEpiWarps * 32);  // MMA commit + every drain lane
      // The stage's MMAs have completed (commit), and with TMA scales the MMA
      // warp's lanes have written the block-major activation scales.
      mbar_init(&dready[s], tma_scales ? 1 + 32 : 1);
    }
    mbar_init(tinit, kEpiWarps * 32);  // every drain lane has seeded its part of all D slots
    mbar_init(done, 1);
    mbar_init(xbar, (kEpiWarps / 2) * 32);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One elected lane of the converged warp issues the stage's TMA copies.
    // Stage index and phase are running counters (no division in the loop).
    if (lane == 0) {
      prefetch_tmap(&tw);
      prefetch_tmap(&tx);
      if (tma_scales) {
        prefetch_tmap(&tsw);
        prefetch_tmap(&tsx);
      }
    }
    // Launched as a programmatic dependent of the activation quantize: the
    // CTA's setup above overlapped it; the quantized activations and their
    // scales are read only after it completed.
    pdl_wait();
    __syncwarp();
    int k = 0, s = 0;
    uint32_t eph = 1;  // parity of empty[s] to wait for, from the ring's second pass on
    for (; k < nst; k++) {
      if (k >= stages) {
        const bool got = !abort_flag && mbar_wait_bounded(&empty[s], eph, a.status, kStatusMmaTimeout);
        if (!__all_sync(0xffffffffu, got)) {
          abort_flag = 1;
          break;
        }
      }
      if (elect_one()) {
        mbar_arrive_expect_tx(&full[s], (uint32_t)((Q4 ? kRawBytes : kABytes) + kBBytes +
                                                   (tma_scales ? kSxBytes + kSwBytes : 0)));
        if (Q4)
          tma_load_2d(stage_raw(s), &tw, k * (kStageK / 2), (int32_t)row0, &full[s]);
        else
          tma_load_2d(stage_a(s), &tw, k * kStageK, (int32_t)row0, &full[s]);
        tma_load_2d(stage_b(s), &tx, k * kStageK, (int32_t)tok0, &full[s]);
        if (tma_scales) {
          // Weight scales: Q8 the stage's 4 f32 per row; Q4 the 8 fp16 per
          // row of the pair of stages holding this one (a box starting on a
          // 16-byte boundary), of which the drain reads its half.
          tma_load_2d(stage_sw(s), &tsw, Q4 ? (k >> 1) * 2 * kBlocksPerStage : k * kBlocksPerStage,
                      (int32_t)row0, &full[s]);
          // Activation scales, token-major: 64 tokens x 4 blocks.
          tma_load_2d(stage_sx(s), &tsx, k * kBlocksPerStage, (int32_t)tok0, &full[s]);
        }
      }
      __syncwarp();
      if (tma_scales) {
        if (++s == stages) {
          s = 0;
          eph ^= 1u;
        }
        continue;
      }
      float* sx = stage_sx(s);
      float* sw = stage_sw(s);
      const int64_t b0 = (int64_t)k * kBlocksPerStage;
      // Asynchronous copies (cp.async), so the producer never waits for the
      // scales' latency: activation scales transposed to block-major, one
      // 4-byte copy each; weight scales 16 (f32) or 8 (fp16) bytes per row.
      // Out-of-range tokens, rows or blocks are zero-filled.
      for (int i = lane; i < kTileTok; i += 32) {
        const int64_t t = tok0 + i;
#pragma unroll
        for (int q = 0; q < kBlocksPerStage; q++) {
          const bool in = t < a.n && b0 + q < blocks;
          cp_async(sx + q * kTileTok + i, in ? (const void*)(a.xsc + t * blocks + b0 + q) : (const void*)a.xsc,
                   4, in ? 4 : 0);
        }
      }
      const bool vec_w = (blocks % kBlocksPerStage) == 0 && ((uintptr_t)a.scales & (Q4 ? 7 : 15)) == 0;
      for (int i = lane; i < kTileRows; i += 32) {
        const int64_t r = row0 + i;
        if (Q4) {
          uint16_t* sw16 = reinterpret_cast<uint16_t*>(sw) + i * kBlocksPerStage;
          const uint16_t* src = static_cast<const uint16_t*>(a.scales) + r * blocks + b0;
          if (vec_w) {
            cp_async(sw16, r < a.rows ? (const void*)src : a.scales, 8, r < a.rows ? 8 : 0);
          } else {
#pragma unroll
            for (int q = 0; q < kBlocksPerStage; q++)
              sw16[q] = (r < a.rows && b0 + q < blocks) ? __ldg(src + q) : (uint16_t)0;
          }
        } else {
          const float* src = static_cast<const float*>(a.scales) + r * blocks + b0;
          if (vec_w) {
            cp_async(sw + i * kBlocksPerStage, r < a.rows ? (const void*)src : a.scales, 16,
                     r < a.rows ? 16 : 0);
          } else {
#pragma unroll
            for (int q = 0; q < kBlocksPerStage; q++) {
              const bool in = r < a.rows && b0 + q < blocks;
              cp_async(sw + i * kBlocksPerStage + q, in ? (const void*)(src + q) : a.scales, 4, in ? 4 : 0);
            }
          }
        }
      }
      if (Q4 && !vec_w) {
        // The fp16 scales went through plain stores: arrive after everything landed.
        asm volatile("cp.async.wait_all;" ::: "memory");
        mbar_arrive(&full[s]);
      } else {
        cp_async_arrive(&full[s]);
      }
      if (++s == stages) {
        s = 0;
        eph ^= 1u;
      }
    }
    if (abort_flag && lane == 0) {
      // Let the copies already issued land before the CTA's memory goes.
      for (int j = k - 1; j >= 0 && j >= k - stages; j--)
        mbar_wait_bounded(&full[j % stages], (uint32_t)(j / stages) & 1u, a.status,
                          kStatusTmaTimeout);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // The whole warp runs the loop; one elected lane issues. The stage's
    // operand descriptors are formed once and the blocks' K offsets (32
    // bytes = 2 descriptor units) and D slots are constants: block b of the
    // tile goes to D slot b % 8 = 4 * (k & 1) + q, on its (k / 2)-th use.
    static_assert(kSlots == 2 * kBlocksPerStage, "two stages of D slots");
    const uint32_t smem0 = smem_u32(smem);
    int s = 0, s2 = 0;  // ring indices of stages k and k - 2
    uint32_t ph = 0, ph2 = 0;
    for (int k = 0; k < nst; k++) {
      bool got = !abort_flag && mbar_wait_bounded(&full[s], ph, a.status, kStatusTmaTimeout);
      if (Q4) got = got && mbar_wait_bounded(&conv[s], ph, a.status, kStatusTmaTimeout);
      if (!__all_sync(0xffffffffu, got)) {
        abort_flag = 1;
        break;
      }
      if (tma_scales) {
        // Activation scales [64 tokens][4 blocks] -> [4 blocks][64 tokens],
        // so a drain warp reads four tokens of one block in one 16-byte load.
        const float* src = stage_sx(s);
        float* dst = stage_sxb(s);
#pragma unroll
        for (int t = lane; t < kTileTok; t += 32) {
          const float4 v = *reinterpret_cast<const float4*>(src + t * kBlocksPerStage);
          dst[0 * kTileTok + t] = v.x;
          dst[1 * kTileTok + t] = v.y;
          dst[2 * kTileTok + t] = v.z;
          dst[3 * kTileTok + t] = v.w;
        }
        mbar_arrive(&dready[s]);
      }
      tc_fence_after();
      const uint32_t a_addr = smem0 + (uint32_t)s * (uint32_t)S::kStageBytes;
      const uint64_t ad = sw128_desc(a_addr), bd = sw128_desc(a_addr + kABytes);
      const int slot0 = (k & 1) * kBlocksPerStage;
      const int nq = (int)min64(kBlocksPerStage, blocks - (int64_t)k * kBlocksPerStage);
      bool ok = true;
      if (Q4 && k == 0) {
        ok = !abort_flag && mbar_wait_bounded(tinit, 0, a.status, kStatusMmaTimeout);
        ok = __all_sync(0xffffffffu, ok) != 0;
        if (!ok) abort_flag = 1;
      }
      if (k >= 2) {
        // The stage's D slots held stage k - 2's blocks: they are free (and
        // seeded again) once the drain has released stage k - 2 (its
        // `empty` phase completes).
        ok = !abort_flag && mbar_wait_bounded(&empty[s2], ph2, a.status, kStatusMmaTimeout);
        ok = __all_sync(0xffffffffu, ok) != 0;
        if (!ok) abort_flag = 1;
        if (++s2 == stages) {
          s2 = 0;
          ph2 ^= 1u;
        }
      }
      tc_fence_after();
      // One elected section per stage: the control flow around single-lane
      // instructions costs more than the MMAs themselves.
      if (elect_one()) {
        if (ok) {
#pragma unroll
          for (int q = 0; q < kBlocksPerStage; q++) {
            if (q < nq) {
              mma_i8(tmem + (uint32_t)((slot0 + q) * kTileTok), ad + (uint64_t)(2 * q),
                     bd + (uint64_t)(2 * q), kIdescI8, Q4 ? 1u : 0u);
            }
          }
        }
        mma_commit(&dready[s]);  // the drain may read the stage's D slots
        mma_commit(&empty[s]);   // the producer may refill the stage (with the drain's arrivals)
      }
      __syncwarp();
      if (!ok) break;
      if (++s == stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    // Every MMA issued has completed once `done` arrives.
    if (elect_one()) mma_commit(done);
    __syncwarp();
    mbar_wait_bounded(done, 0, a.status, kStatusMmaTimeout);
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ drain
    // Four warps per TMEM lane quarter: even or odd blocks times the low or
    // high 32 token columns. Each block's step is a short serial chain in
    // one warp (barrier probe, TMEM load, arrival, 32 columns of math), so
    // four such warps per scheduler hide one another's latencies
    // (tcgen05.wait::ld waits for all of a thread's loads, so a warp cannot
    // keep a second one in flight). The even and odd partial f32 sums are
    // added at the end.
    const int quarter = warp & 3;               // TMEM lanes this warp may access
    const int sub = (warp - 2) >> 2;            // 0 .. 3
    const int parity = sub & 1;                 // even or odd blocks
    const int col0 = (sub >> 1) * kEpiCols;     // first token column of this warp (0 with 8 warps)
    const int row_local = quarter * 32 + lane;
    const int64_t row = row0 + row_local;
    uint64_t acc[kEpiCols / 2];                 // f32 pairs: tokens col0 + 2i, col0 + 2i + 1
#pragma unroll
    for (int j = 0; j < kEpiCols / 2; j++) acc[j] = 0;
    const int nblk = (int)blocks;
    int32_t dn[kEpiCols];
    const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0;
    // Token columns of this warp that hold real tokens (kPartial: fewer than
    // 64 tokens, e.g. a short prompt or a few sequences at the lm_head): a
    // warp without any still keeps every barrier step, but loads and scales
    // nothing.
    const int64_t ncols = a.n - (tok0 + col0);
    const int valid = !kPartial || ncols >= kEpiCols ? kEpiCols : (ncols <= 0 ? 0 : (int)ncols);
    if (Q4 && valid > 0) {
#pragma unroll
      for (int q = 0; q < kSlots; q++)
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 32) tmem_fill32(tlane + (uint32_t)(q * kTileTok + c), kSeed);
      tmem_wait_st();
      tc_fence_before();
    }
    if (Q4) mbar_arrive(tinit);
    int st = 0;
    uint32_t sph = 0;
    for (int k = 0; k < nst; k++) {
      // One wait per stage: the stage's scales have landed, its MMAs have
      // completed and (with TMA scales) the block-major activation scales
      // are written.
      bool got = !abort_flag && mbar_wait_bounded(&full[st], sph, a.status, kStatusTmaTimeout);
      got = got && mbar_wait_bounded(&dready[st], sph, a.status, kStatusMmaTimeout);
      if (!__all_sync(0xffffffffu, got)) {
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int slot0 = (k & 1) * kBlocksPerStage;
      float sws[kBlocksPerStage];
      if (Q4) {
        // TMA scales: 8 fp16 per row covering stages 2j and 2j + 1.
        const uint16_t* w16 = reinterpret_cast<const uint16_t*>(stage_sw(st)) +
                              (tma_scales ? row_local * 2 * kBlocksPerStage + (k & 1) * kBlocksPerStage
                                          : row_local * kBlocksPerStage);
        const uint2 h = *reinterpret_cast<const uint2*>(w16);
        sws[0] = half_bits_to_float((uint16_t)h.x);
        sws[1] = half_bits_to_float((uint16_t)(h.x >> 16));
        sws[2] = half_bits_to_float((uint16_t)h.y);
        sws[3] = half_bits_to_float((uint16_t)(h.y >> 16));
      } else {
        const float4 f = *reinterpret_cast<const float4*>(stage_sw(st) + row_local * kBlocksPerStage);
        sws[0] = f.x; sws[1] = f.y; sws[2] = f.z; sws[3] = f.w;
      }
      if (valid > 0) {
#pragma unroll
        for (int q = parity; q < kBlocksPerStage; q += 2) {
          const int blk = k * kBlocksPerStage + q;
          if (blk >= nblk) break;
#pragma unroll
          for (int c = 0; c < kEpiCols; c += 32)
            tmem_ld32(tlane + (uint32_t)((slot0 + q) * kTileTok + c), *reinterpret_cast<int32_t(*)[32]>(dn + c));
#pragma unroll
          for (int c = 0; c < kEpiCols; c += 32) tmem_wait_ld_regs(*reinterpret_cast<int32_t(*)[32]>(dn + c));
          if (Q4) {  // seed for the slot's next block
#pragma unroll
            for (int c = 0; c < kEpiCols; c += 32) tmem_fill32(tlane + (uint32_t)((slot0 + q) * kTileTok + c), kSeed);
          }
          const uint64_t sw2 = f2_pack(sws[q], sws[q]);
          const float* sxq = (tma_scales ? stage_sxb(st) : stage_sx(st)) + q * kTileTok + col0;
#pragma unroll
          for (int j = 0; j < kEpiCols; j += 4) {
            const float4 x4 = *reinterpret_cast<const float4*>(sxq + j);
            // acc += f32(d) * f32(sw * sx), as the reference's per-block step.
            acc[j / 2] = f2_fma(slot_to_f2<Q4>(dn[j], dn[j + 1]), f2_mul(sw2, f2_pack(x4.x, x4.y)), acc[j / 2]);
            acc[j / 2 + 1] = f2_fma(slot_to_f2<Q4>(dn[j + 2], dn[j + 3]), f2_mul(sw2, f2_pack(x4.z, x4.w)),
                                    acc[j / 2 + 1]);
          }
        }
      }
      if (Q4 && valid > 0) tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&empty[st]);  // every lane: done with the stage's scales and D slots (seeded again)
      if (++st == stages) {
        st = 0;
        sph ^= 1u;
      }
    }
    // The odd warp hands its sums to the even warp of its lane quarter
    // (token-major in the exchange buffer, so a warp's stores hit 32 banks).
    float* x = xchg + (int64_t)quarter * 32 * kTileTok + col0 * 32;
    if (parity == 1) {
#pragma unroll
      for (int j = 0; j < kEpiCols / 2; j++) {
        x[(2 * j) * 32 + lane] = __uint_as_float((uint32_t)acc[j]);
        x[(2 * j + 1) * 32 + lane] = __uint_as_float((uint32_t)(acc[j] >> 32));
      }
      mbar_arrive(xbar);
    } else {
      const bool got = !abort_flag && mbar_wait_bounded(xbar, 0, a.status, kStatusMmaTimeout);
      if (got && row < a.rows) {
#pragma unroll
        for (int j = 0; j < kEpiCols / 2; j++) {
          const int64_t t = tok0 + col0 + 2 * j;
          const float y0 = __fadd_rn(__uint_as_float((uint32_t)acc[j]), x[(2 * j) * 32 + lane]);
          const float y1 = __fadd_rn(__uint_as_float((uint32_t)(acc[j] >> 32)), x[(2 * j + 1) * 32 + lane]);
          if constexpr (GATHER) {
            // (A compile-time variant: a run-time index into the argument
            // struct would move the whole struct to local memory in the plain
            // kernels too - measured 3-12 % slower.)
            for (int p = 0; p < a.gather_n; p++) {
              float* g = a.gather_ys[p] + a.gather_row0 + row;
              if (t < a.n) g[t * a.ldy] = y0;
              if (t + 1 < a.n) g[(t + 1) * a.ldy] = y1;
            }
          } else {
            if (t < a.n) a.ys[t * a.ldy + row] = y0;
            if (t + 1 < a.n) a.ys[(t + 1) * a.ldy + row] = y1;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ Q4 expansion
    const int ct = tid - (2 + kEpiWarps) * 32;  // 0 .. 63
    int s = 0;
    uint32_t ph = 0;
    for (int k = 0; k < nst; k++) {
      if (!wait_tc(&full[s], ph, a.status, kStatusTmaTimeout, &abort_flag)) break;
      const uint8_t* raw = stage_raw(s);
      uint8_t* dst = stage_a(s);
      // One (row, block) per task: 16 nibble bytes -> two swizzled 16-byte
      // chunks of int8 (q - 8): low nibbles are weights 0..15 of the block,
      // high nibbles weights 16..31 (GGUF order).
      for (int task = ct; task < kTileRows * kBlocksPerStage; task += kConvWarps * 32) {
        const int r = task >> 2, q = task & 3;
        const uint4 v = *reinterpret_cast<const uint4*>(raw + r * (kStageK / 2) + q * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          // (n & 15) + 0x78, then ^ 0x80, is n - 8 as a two's-complement byte.
          lo[i] = ((w[i] & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
          hi[i] = (((w[i] >> 4) & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
        }
        uint8_t* line = dst + (r >> 3) * 1024 + (r & 7) * 128;
        *reinterpret_cast<uint4*>(line + (((2 * q) ^ (r & 7)) << 4)) =
            make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(line + (((2 * q + 1) ^ (r & 7)) << 4)) =
            make_uint4(hi[0], hi[1], hi[2], hi[3]);
      }
      fence_proxy_async_smem();  // generic-proxy writes -> the tensor core's reads
      mbar_arrive(&conv[s]);
      if (++s == stages) {
        s = 0;
        ph ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// After the gathering GEMM (the previous kernel in the stream, complete, so
// every store it made is ordered before this one): one system-scope fence
// makes those stores visible to the peers, then one count on every rank's
// counter (the waiting side acquires). One fence per product instead of one
// per CTA: a fence per CTA measured +21 us on a 45 us GEMM. After a bounded
// wait ran out anywhere (the status word is set) nothing is counted, so the
// peers' waits run out too rather than read a partial output.
struct PeerCounters {
  int* p[kMaxGatherRanks];
};
__global__ void peer_signal_kernel(const PeerCounters c, int world, const uint32_t* status) {
  if (status != nullptr && *reinterpret_cast<const volatile uint32_t*>(status) != 0) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int p = 0; p < world; p++)
    asm volatile("red.relaxed.sys.global.add.s32 [%0], 1;" ::"l"(c.p[p]) : "memory");
}

// The fused all-gather's destinations (launch_tc; null: plain outputs).
struct TcGather {
  int world;
  int64_t row0;
  float* const* ys;
  int* const* cnt;
};

template <bool Q4>
int64_t launch_tc(const LinearArgs& a, cudaStream_t stream, const TcGather* gather = nullptr) {
  using S = TcShape<Q4>;
  const int64_t blocks = a.cols / kBlock;
  const int64_t bar_bytes = 8 * (4 * 16 + 2 * kSlots + 3) + 16;  // up to 16 stages
  int stages = (int)((kMaxSmemTc - 1024 - kXchgBytes - bar_bytes) / S::kStageBytes);
  stages = stages > 12 ? 12 : stages;
  if (stages < 2) return kErrTooLarge;
  const size_t smem = 1024 + (size_t)stages * S::kStageBytes + kXchgBytes + (size_t)bar_bytes;
  CUtensorMap tw, tx;
  if (Q4) {
    if (!encode_tmap_2d(&tw, a.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)blocks * 16,
                        (uint64_t)a.rows, (uint64_t)blocks * 16, kStageK / 2, kTileRows, false))
      return kErrUnsupported;
  } else {
    if (!encode_tmap_2d(&tw, a.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)blocks * 32,
                        (uint64_t)a.rows, (uint64_t)blocks * 32, kStageK, kTileRows, true))
      return kErrUnsupported;
  }
  if (!encode_tmap_2d(&tx, a.xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)a.cols, (uint64_t)a.n,
                      (uint64_t)a.cols, kStageK, kTileTok, true))
    return kErrUnsupported;
  // Scales by TMA when their rows are addressable: 16-byte aligned arrays and
  // rows whose byte length is a multiple of 16 (the Q4 box is 8 fp16 wide).
  const bool tma_scales = blocks % (Q4 ? 8 : 4) == 0 && ((uintptr_t)a.scales & 15) == 0 &&
                          ((uintptr_t)a.xsc & 15) == 0;
  CUtensorMap tsw = tw, tsx = tx;  // unused copies unless tma_scales
  if (tma_scales) {
    const bool ok_w =
        Q4 ? encode_tmap_2d(&tsw, a.scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)blocks,
                            (uint64_t)a.rows, (uint64_t)blocks * 2, 2 * kBlocksPerStage, kTileRows, false)
           : encode_tmap_2d(&tsw, a.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)blocks,
                            (uint64_t)a.rows, (uint64_t)blocks * 4, kBlocksPerStage, kTileRows, false);
    if (!ok_w || !encode_tmap_2d(&tsx, a.xsc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)blocks,
                                 (uint64_t)a.n, (uint64_t)blocks * 4, kBlocksPerStage, kTileTok, false))
      return kErrUnsupported;
  }
  const void* kern =
      gather != nullptr
          ? (a.n < kTileTok ? (const void*)gemm_tc_kernel<Q4, true, true> : (const void*)gemm_tc_kernel<Q4, false, true>)
          : (a.n < kTileTok ? (const void*)gemm_tc_kernel<Q4, true> : (const void*)gemm_tc_kernel<Q4, false>);
  static bool configured[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int variant = (a.n < kTileTok ? 1 : 0) + (gather != nullptr ? 2 : 0);
  if (!configured[variant][dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemTc) !=
        cudaSuccess)
      return kErrCuda;
    configured[variant][dev & 63] = true;
  }
  TcGatherArgs t{};
  static_cast<TcArgs&>(t) = TcArgs{a.scales, a.xsc, a.ys, a.rows, a.cols, a.n, a.ldy, a.status, tma_scales ? 1 : 0};
  if (gather != nullptr) {
    t.gather_n = gather->world;
    t.gather_row0 = gather->row0;
    for (int p = 0; p < gather->world; p++) t.gather_ys[p] = gather->ys[p];
  }
  const dim3 grid((unsigned)((a.rows + kTileRows - 1) / kTileRows),
                  (unsigned)((a.n + kTileTok - 1) / kTileTok), 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(S::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nstages = stages;
  void* params[] = {&t, &nstages, &tw, &tx, &tsw, &tsx};
  return cudaLaunchKernelExC(&cfg, kern, params) == cudaSuccess ? kOk : kErrCuda;
}

// ------------------------------------------------------------ narrow tiles
//
// Few tokens (the lm_head M sweep, a short prompt): the 64-token tile leaves
// TMEM room for two stages only, and at one handshake round trip per two
// stages (~2 k cycles each) the kernel streams far below HBM speed however
// little there is to compute. A narrow tile of TOK = 16 or 32 tokens leaves
// room for 512 / TOK D slots = 8 or 4 stages in flight, so the round trip
// hides behind the weight stream. The kernel is persistent (one CTA per SM
// walks tiles blockIdx.x, + gridDim.x, ...; every ring runs on across
// tiles) and its drain is stage-parallel: drain warp (quarter, sub) takes
// the stages g with g % 4 == sub, all 4 blocks x TOK tokens of them, so the
// four subs of a quarter work on different stages and meet only at a tile's
// end. There each warp leaves its partial sums in shared memory, and the
// producer warp, which otherwise waits for free stages, adds the four subs'
// sums and writes the tile. Roles otherwise as in gemm_tc_kernel: warp 0
// producer, warp 1 MMA issuer (and the activation-scale transpose), warps
// 2-17 drain, warps 18-19 (Q4) nibble expansion.
template <bool Q4, int TOK>
struct NarrowShape {
  static constexpr int kSlots = (int)kTmemCols / TOK;
  static constexpr int kLookahead = kSlots / kBlocksPerStage;  // stages TMEM can hold: 8 or 4
  static constexpr int kWarps = 2 + kEpiWarps + (Q4 ? kConvWarps : 0);
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kBBytes = TOK * kStageK;
  static constexpr int kSxBytes = kBlocksPerStage * TOK * 4;
  static constexpr int kRawOff = kABytes + kBBytes;
  static constexpr int kSxOff = kRawOff + (Q4 ? kRawBytes : 0);
  static constexpr int kSwOff = kSxOff + kSxBytes;
  static constexpr int kSxbOff = kSwOff + kSwBytes;
  static constexpr int kStageBytes = (kSxbOff + kSxBytes + 1023) / 1024 * 1024;
  static constexpr int kXchgBytes = 4 * kTileRows * TOK * 4;  // each sub's sums of a tile
  static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TOK >> 3) << 17) |
                                     ((uint32_t)(kTileRows >> 4) << 24);
  static_assert(kLookahead % 4 == 0, "each sub owns whole slot groups");
};

// 32 lanes x TOK consecutive 32-bit TMEM columns.
template <int TOK>
__device__ __forceinline__ void tmem_ld_tok(uint32_t taddr, int32_t (&v)[TOK]);
template <>
__device__ __forceinline__ void tmem_ld_tok<32>(uint32_t taddr, int32_t (&v)[32]) {
  tmem_ld32(taddr, v);
}
template <>
__device__ __forceinline__ void tmem_ld_tok<16>(uint32_t taddr, int32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
template <int TOK>
__device__ __forceinline__ void tmem_wait_ld_tok(int32_t (&v)[TOK]);
template <>
__device__ __forceinline__ void tmem_wait_ld_tok<32>(int32_t (&v)[32]) {
  tmem_wait_ld_regs(v);
}
template <>
__device__ __forceinline__ void tmem_wait_ld_tok<16>(int32_t (&v)[16]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]),
        "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]),
        "+r"(v[14]), "+r"(v[15])
      :
      : "memory");
}
// TMEM columns set to the seed: TOK of them for the calling warp's 32 lanes.
template <int TOK>
__device__ __forceinline__ void tmem_fill_tok(uint32_t taddr) {
#pragma unroll
  for (int c = 0; c < TOK; c += 8)
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(
                     taddr + (uint32_t)c),
                 "r"(kSeed)
                 : "memory");
}
// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

template <bool Q4, int TOK, bool GATHER = false>
__global__ void __launch_bounds__(NarrowShape<Q4, TOK>::kThreads, 1)
    gemm_narrow_kernel(const TcArgsOf<GATHER> a, const int stages, const int L, const __grid_constant__ CUtensorMap tw,
                       const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tsw,
                       const __grid_constant__ CUtensorMap tsx) {
  using S = NarrowShape<Q4, TOK>;
  // L: stages held in TMEM (slot groups of 4 D slots), 4 or 8; at most the
  // ring's stage count, so a stage's `tfree` phase is waited for before
  // the ring slot's next use can complete it again.
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* smem = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  float* xchg = reinterpret_cast<float*>(smem + (int64_t)stages * S::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (int64_t)stages * S::kStageBytes + S::kXchgBytes);
  uint64_t* conv = full + stages;
  uint64_t* empty = conv + stages;
  uint64_t* dready = empty + stages;
  uint64_t* tfree = dready + stages;
  uint64_t* tinit = tfree + stages;
  uint64_t* done = tinit + 1;
  uint64_t* xbar = done + 1;
  uint64_t* xfree = xbar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfree + 1);
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t blocks = a.cols / kBlock;
  const int nst = (int)((blocks + kBlocksPerStage - 1) / kBlocksPerStage);
  auto stage_a = [&](int s) { return smem + (int64_t)s * S::kStageBytes; };
  auto stage_b = [&](int s) { return smem + (int64_t)s * S::kStageBytes + kABytes; };
  auto stage_raw = [&](int s) { return smem + (int64_t)s * S::kStageBytes + S::kRawOff; };
  auto stage_sx = [&](int s) { return reinterpret_cast<float*>(smem + (int64_t)s * S::kStageBytes + S::kSxOff); };
  auto stage_sw = [&](int s) { return reinterpret_cast<float*>(smem + (int64_t)s * S::kStageBytes + S::kSwOff); };
  auto stage_sxb = [&](int s) { return reinterpret_cast<float*>(smem + (int64_t)s * S::kStageBytes + S::kSxbOff); };

  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);                // TMA bytes
      mbar_init(&conv[s], kConvWarps * 32);  // (Q4) the stage's weights expanded
      // The stage's drain sub (4 warps) is done with its scales; the MMAs
      // that read its operands completed before that sub saw `dready`.
      mbar_init(&empty[s], 4 * 32);
      // The stage's MMAs have completed and the MMA warp's lanes have written
      // its block-major activation scales.
      mbar_init(&dready[s], 1 + 32);
      // The stage's drain sub has read (and, Q4, seeded again) its D slots.
      mbar_init(&tfree[s], 4 * 32);
    }
    mbar_init(tinit, kEpiWarps * 32);
    mbar_init(done, 1);
    mbar_init(xbar, kEpiWarps * 32);  // every drain lane has left a tile's partial sums
    mbar_init(xfree, 32);             // the producer has written that tile's outputs
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tw);
      prefetch_tmap(&tx);
      prefetch_tmap(&tsw);
      prefetch_tmap(&tsx);
    }
    // A programmatic dependent of the activation quantize: only the copies
    // below wait for it.
    pdl_wait();
    __syncwarp();
    // Tile outputs: the oldest tile whose sums are not written yet.
    int64_t ep_tile = blockIdx.x;
    uint32_t ep_it = 0;
    bool vec_y = (a.ldy & 3) == 0;
    if constexpr (GATHER) {
      vec_y = vec_y && (a.gather_row0 & 3) == 0;
      for (int p = 0; p < a.gather_n; p++) vec_y = vec_y && ((uintptr_t)a.gather_ys[p] & 15) == 0;
    } else {
      vec_y = vec_y && ((uintptr_t)a.ys & 15) == 0;
    }
    auto finish_tile = [&]() {
      // Every lane observes the completed phase itself (no wait: it is).
      mbar_wait_bounded(xbar, ep_it & 1u, a.status, kStatusMmaTimeout);
      const int64_t row0 = (ep_tile % a.row_tiles) * kTileRows;
      const int64_t tok0 = (ep_tile / a.row_tiles) * TOK;
      const int64_t r = row0 + 4 * lane;
      // The four subs' sums, token-major: a lane's 4 rows are 16 bytes.
      const float4* p = reinterpret_cast<const float4*>(xchg) + lane;
      constexpr int kSub = TOK * kTileRows / 4;  // float4s per sub
      for (int t = 0; t < TOK; t++) {
        const int64_t tok = tok0 + t;
        if (tok >= a.n) break;
        const float4 u0 = p[t * (kTileRows / 4)], u1 = p[kSub + t * (kTileRows / 4)];
        const float4 u2 = p[2 * kSub + t * (kTileRows / 4)], u3 = p[3 * kSub + t * (kTileRows / 4)];
        const float4 y = make_float4(__fadd_rn(__fadd_rn(u0.x, u1.x), __fadd_rn(u2.x, u3.x)),
                                     __fadd_rn(__fadd_rn(u0.y, u1.y), __fadd_rn(u2.y, u3.y)),
                                     __fadd_rn(__fadd_rn(u0.z, u1.z), __fadd_rn(u2.z, u3.z)),
                                     __fadd_rn(__fadd_rn(u0.w, u1.w), __fadd_rn(u2.w, u3.w)));
        // Into this GPU's output, or (the fused all-gather, a compile-time
        // variant) into every rank's.
        int ncopies = 1;
        if constexpr (GATHER) ncopies = a.gather_n;
        for (int p = 0; p < ncopies; p++) {
          float* dst;
          if constexpr (GATHER)
            dst = a.gather_ys[p] + a.gather_row0 + tok * a.ldy + r;
          else
            dst = a.ys + tok * a.ldy + r;
          if (vec_y && r + 3 < a.rows) {
            *reinterpret_cast<float4*>(dst) = y;
          } else {
            if (r < a.rows) dst[0] = y.x;
            if (r + 1 < a.rows) dst[1] = y.y;
            if (r + 2 < a.rows) dst[2] = y.z;
            if (r + 3 < a.rows) dst[3] = y.w;
          }
        }
      }
      __syncwarp();
      mbar_arrive(xfree);
      ep_it++;
      ep_tile += gridDim.x;
    };
    int64_t g = 0;
    int s = 0;
    uint32_t eph = 1;  // parity of empty[s] to wait for, from the ring's second pass on
    bool stop = false;
    for (int64_t tile = blockIdx.x; tile < a.tiles && !stop; tile += gridDim.x) {
      const int64_t row0 = (tile % a.row_tiles) * kTileRows;
      const int64_t tok0 = (tile / a.row_tiles) * TOK;
      for (int k = 0; k < nst; k++, g++) {
        if (g >= stages) {
          // Wait for the stage to come free (sleeping in the wait, not
          // spinning); meanwhile write any tile whose sums are complete - the
          // drain needs that buffer back before it can finish its next tile.
          // Lane 0 probes and the warp follows its decision.
          bool got = false;
          const uint64_t t_start = globaltimer_ns();
          for (;;) {
            int what = 0;  // 1: stage free, 2: give up, 3: a tile to write
            if (lane == 0) {
              if (abort_flag) {
                what = 2;
              } else if (mbar_try_wait_sleep(&empty[s], eph, 1000u)) {
                what = 1;
              } else if (ep_tile < tile && mbar_test(xbar, ep_it & 1u)) {
                what = 3;
              } else if (globaltimer_ns() - t_start > wait_limit_ns()) {
                report(a.status, kStatusMmaTimeout);
                what = 2;
              }
            }
            what = __shfl_sync(0xffffffffu, what, 0);
            if (what == 1) {
              got = true;
              break;
            }
            if (what == 2) break;
            if (what == 3) finish_tile();
          }
          if (!__all_sync(0xffffffffu, got)) {
            abort_flag = 1;
            stop = true;
            break;
          }
        }
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], (uint32_t)((Q4 ? kRawBytes : kABytes) + S::kBBytes + S::kSxBytes + kSwBytes));
          if (Q4)
            tma_load_2d(stage_raw(s), &tw, k * (kStageK / 2), (int32_t)row0, &full[s]);
          else
            tma_load_2d(stage_a(s), &tw, k * kStageK, (int32_t)row0, &full[s]);
          tma_load_2d(stage_b(s), &tx, k * kStageK, (int32_t)tok0, &full[s]);
          // Weight scales: Q8 the stage's 4 f32 per row; Q4 the 8 fp16 per
          // row of the pair of stages holding this one, of which the drain
          // reads its half. Activation scales token-major: TOK x 4.
          tma_load_2d(stage_sw(s), &tsw, Q4 ? (k >> 1) * 2 * kBlocksPerStage : k * kBlocksPerStage,
                      (int32_t)row0, &full[s]);
          tma_load_2d(stage_sx(s), &tsx, k * kBlocksPerStage, (int32_t)tok0, &full[s]);
        }
        __syncwarp();
        if (++s == stages) {
          s = 0;
          eph ^= 1u;
        }
      }
    }
    while (!stop && ep_tile < a.tiles) {
      const bool got = !abort_flag && mbar_wait_bounded(xbar, ep_it & 1u, a.status, kStatusMmaTimeout);
      if (!__all_sync(0xffffffffu, got)) {
        abort_flag = 1;
        break;
      }
      finish_tile();
    }
    if (abort_flag && lane == 0) {
      // Let the copies already issued land before the CTA's memory goes.
      for (int64_t j = g - 1; j >= 0 && j >= g - stages; j--)
        mbar_wait_bounded(&full[j % stages], (uint32_t)(j / stages) & 1u, a.status, kStatusTmaTimeout);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // Stage g's block q goes to D slot 4 * (g % L) + q.
    const uint32_t smem0 = smem_u32(smem);
    int s = 0, sl = 0;  // ring indices of stages g and g - L
    uint32_t ph = 0, phl = 0;
    int grp = 0;        // g % L
    int64_t g = 0;
    bool stop = false;
    for (int64_t tile = blockIdx.x; tile < a.tiles && !stop; tile += gridDim.x) {
      for (int k = 0; k < nst; k++, g++) {
        bool ok = !abort_flag && mbar_wait_bounded(&full[s], ph, a.status, kStatusTmaTimeout);
        if (Q4) ok = ok && mbar_wait_bounded(&conv[s], ph, a.status, kStatusTmaTimeout);
        if (!__all_sync(0xffffffffu, ok)) {
          abort_flag = 1;
          stop = true;
          break;
        }
        // Activation scales [TOK tokens][4 blocks] -> [4 blocks][TOK tokens],
        // so a drain warp reads four tokens of one block in one 16-byte load.
        if (lane < TOK) {
          const float4 v = reinterpret_cast<const float4*>(stage_sx(s))[lane];
          float* dst = stage_sxb(s);
          dst[0 * TOK + lane] = v.x;
          dst[1 * TOK + lane] = v.y;
          dst[2 * TOK + lane] = v.z;
          dst[3 * TOK + lane] = v.w;
        }
        mbar_arrive(&dready[s]);
        if (g == 0) ok = ok && mbar_wait_bounded(tinit, 0, a.status, kStatusMmaTimeout);
        if (g >= L) {
          // The slot group held stage g - L's blocks: free (and seeded
          // again) once that stage's drain sub has read them.
          ok = ok && mbar_wait_bounded(&tfree[sl], phl, a.status, kStatusMmaTimeout);
          if (++sl == stages) {
            sl = 0;
            phl ^= 1u;
          }
        }
        if (!__all_sync(0xffffffffu, ok)) {
          abort_flag = 1;
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem0 + (uint32_t)s * (uint32_t)S::kStageBytes;
        const uint64_t ad = sw128_desc(a_addr), bd = sw128_desc(a_addr + kABytes);
        const int nq = (int)min64(kBlocksPerStage, blocks - (int64_t)k * kBlocksPerStage);
        if (elect_one()) {
          const uint32_t d0 = tmem + (uint32_t)(grp * kBlocksPerStage * TOK);
#pragma unroll
          for (int q = 0; q < kBlocksPerStage; q++) {
            // Every slot holds the seed 0x4B400000; the MMA adds the dot.
            if (q < nq)
              mma_i8(d0 + (uint32_t)(q * TOK), ad + (uint64_t)(2 * q), bd + (uint64_t)(2 * q), S::kIdesc, 1u);
          }
          mma_commit(&dready[s]);  // the drain may read the stage's D slots
        }
        __syncwarp();
        grp = grp + 1 == L ? 0 : grp + 1;
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    if (elect_one()) mma_commit(done);
    __syncwarp();
    mbar_wait_bounded(done, 0, a.status, kStatusMmaTimeout);
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ drain
    const int quarter = warp & 3;               // TMEM lanes this warp may access
    const int sub = (warp - 2) >> 2;            // 0 .. 3: the stages g with g % 4 == sub
    const int row_local = quarter * 32 + lane;
    const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16);
    uint64_t acc[TOK / 2];                      // f32 pairs: tokens 2i, 2i + 1
    int32_t dn[TOK];
    // Seed this warp's part of its slot groups (sub, sub + 4, ...).
#pragma unroll
    for (int gg = sub; gg < L; gg += 4)
#pragma unroll
      for (int q = 0; q < kBlocksPerStage; q++) tmem_fill_tok<TOK>(tlane + (uint32_t)((gg * kBlocksPerStage + q) * TOK));
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(tinit);
    int st = 0, grp = 0, g4 = 0;  // ring index, g % L, g % 4
    uint32_t sph = 0;
    uint32_t it = 0;  // tiles done by this CTA
    bool stop = false;
    for (int64_t tile = blockIdx.x; tile < a.tiles && !stop; tile += gridDim.x, it++) {
#pragma unroll
      for (int j = 0; j < TOK / 2; j++) acc[j] = 0;
      for (int k = 0; k < nst; k++) {
        if (g4 == sub) {
          bool got = !abort_flag && mbar_wait_bounded(&dready[st], sph, a.status, kStatusMmaTimeout);
          if (!__all_sync(0xffffffffu, got)) {
            abort_flag = 1;
            stop = true;
            break;
          }
          tc_fence_after();
          // This row's weight scales of the stage, read per block (Q4: 8 fp16
          // per row covering stages 2j and 2j + 1).
          const float* sw32 = stage_sw(st) + row_local * kBlocksPerStage;
          const uint16_t* sw16 = reinterpret_cast<const uint16_t*>(stage_sw(st)) + row_local * 2 * kBlocksPerStage +
                                 (k & 1) * kBlocksPerStage;
          const int nq = (int)min64(kBlocksPerStage, blocks - (int64_t)k * kBlocksPerStage);
          const float* sxs = stage_sxb(st);
          const uint32_t slots = tlane + (uint32_t)(grp * kBlocksPerStage * TOK);
#pragma unroll
          for (int q = 0; q < kBlocksPerStage; q++) {
            if (q < nq) {
              const uint32_t slot = slots + (uint32_t)(q * TOK);
              tmem_ld_tok<TOK>(slot, dn);
              tmem_wait_ld_tok<TOK>(dn);
              tmem_fill_tok<TOK>(slot);  // seed for the slot's next block
              if (q == nq - 1) {
                // The whole slot group is in registers or done: back to the MMA.
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&tfree[st]);
              }
              const float sw = Q4 ? half_bits_to_float(sw16[q]) : sw32[q];
              const uint64_t sw2 = f2_pack(sw, sw);
              const float* sxq = sxs + q * TOK;
#pragma unroll
              for (int j = 0; j < TOK; j += 4) {
                const float4 x4 = *reinterpret_cast<const float4*>(sxq + j);
                // acc += f32(d) * f32(sw * sx), as the reference's per-block step.
                acc[j / 2] = f2_fma(slot_to_f2<true>(dn[j], dn[j + 1]), f2_mul(sw2, f2_pack(x4.x, x4.y)), acc[j / 2]);
                acc[j / 2 + 1] = f2_fma(slot_to_f2<true>(dn[j + 2], dn[j + 3]), f2_mul(sw2, f2_pack(x4.z, x4.w)),
                                        acc[j / 2 + 1]);
              }
            }
          }
          mbar_arrive(&empty[st]);  // every lane: done with the stage's scales
        }
        grp = grp + 1 == L ? 0 : grp + 1;
        g4 = (g4 + 1) & 3;
        if (++st == stages) {
          st = 0;
          sph ^= 1u;
        }
      }
      if (stop) break;
      // This sub's partial sums of the tile, token-major (a warp's stores hit
      // 32 banks), once the producer has written the previous tile's.
      const bool got = it == 0 || (!abort_flag && mbar_wait_bounded(xfree, (it - 1) & 1u, a.status, kStatusMmaTimeout));
      if (!__all_sync(0xffffffffu, got)) {
        abort_flag = 1;
        break;
      }
      float* x = xchg + (int64_t)sub * TOK * kTileRows + row_local;
#pragma unroll
      for (int j = 0; j < TOK / 2; j++) {
        x[(2 * j) * kTileRows] = __uint_as_float((uint32_t)acc[j]);
        x[(2 * j + 1) * kTileRows] = __uint_as_float((uint32_t)(acc[j] >> 32));
      }
      mbar_arrive(xbar);
    }
  } else {
    // ------------------------------------------------------------ Q4 expansion
    const int ct = tid - (2 + kEpiWarps) * 32;  // 0 .. 63
    int s = 0;
    uint32_t ph = 0;
    bool stop = false;
    for (int64_t tile = blockIdx.x; tile < a.tiles && !stop; tile += gridDim.x) {
      for (int k = 0; k < nst; k++) {
        if (!wait_tc(&full[s], ph, a.status, kStatusTmaTimeout, &abort_flag)) {
          stop = true;
          break;
        }
        const uint8_t* raw = stage_raw(s);
        uint8_t* dst = stage_a(s);
        // One (row, block) per task: 16 nibble bytes -> two swizzled 16-byte
        // chunks of int8 (q - 8): low nibbles are weights 0..15 of the block,
        // high nibbles weights 16..31 (GGUF order).
        for (int task = ct; task < kTileRows * kBlocksPerStage; task += kConvWarps * 32) {
          const int r = task >> 2, q = task & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(raw + r * (kStageK / 2) + q * 16);
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            // (n & 15) + 0x78, then ^ 0x80, is n - 8 as a two's-complement byte.
            lo[i] = ((wv[i] & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
            hi[i] = (((wv[i] >> 4) & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u;
          }
          uint8_t* line = dst + (r >> 3) * 1024 + (r & 7) * 128;
          *reinterpret_cast<uint4*>(line + (((2 * q) ^ (r & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(line + (((2 * q + 1) ^ (r & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
        fence_proxy_async_smem();  // generic-proxy writes -> the tensor core's reads
        mbar_arrive(&conv[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int& c = counts[dev & 63];
  if (c == 0 && cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) c = 0;
  return c > 0 ? c : 148;
}

// The narrow kernel needs the scales by TMA (blocks a multiple of 4 for Q8,
// 8 for Q4; 16-byte aligned scale arrays).
template <bool Q4, int TOK>
int64_t launch_narrow(const LinearArgs& a, cudaStream_t stream, const TcGather* gather = nullptr) {
  using S = NarrowShape<Q4, TOK>;
  const int64_t blocks = a.cols / kBlock;
  if (blocks % (Q4 ? 8 : 4) != 0 || ((uintptr_t)a.scales & 15) != 0 || ((uintptr_t)a.xsc & 15) != 0)
    return kErrUnsupported;
  constexpr int kMaxStages = 12;
  // Barrier rings (full, conv, empty, dready, tfree), tinit, done, xbar, xfree,
  // the TMEM slot address.
  const int64_t bar_bytes = 8 * (5 * kMaxStages + 4) + 16;
  int stages = (int)((kMaxSmemTc - 1024 - S::kXchgBytes - bar_bytes) / S::kStageBytes);
  stages = stages > kMaxStages ? kMaxStages : stages;
  if (stages < 4) return kErrTooLarge;
  // Stages in TMEM: all it holds when the ring has as many stages, else 4.
  int lookahead = stages >= S::kLookahead ? S::kLookahead : 4;
  const size_t smem = 1024 + (size_t)stages * S::kStageBytes + S::kXchgBytes + (size_t)bar_bytes;
  CUtensorMap tw, tx, tsw, tsx;
  if (Q4) {
    if (!encode_tmap_2d(&tw, a.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)blocks * 16,
                        (uint64_t)a.rows, (uint64_t)blocks * 16, kStageK / 2, kTileRows, false))
      return kErrUnsupported;
  } else {
    if (!encode_tmap_2d(&tw, a.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)blocks * 32,
                        (uint64_t)a.rows, (uint64_t)blocks * 32, kStageK, kTileRows, true))
      return kErrUnsupported;
  }
  if (!encode_tmap_2d(&tx, a.xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)a.cols, (uint64_t)a.n,
                      (uint64_t)a.cols, kStageK, TOK, true))
    return kErrUnsupported;
  const bool ok_w =
      Q4 ? encode_tmap_2d(&tsw, a.scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)blocks,
                          (uint64_t)a.rows, (uint64_t)blocks * 2, 2 * kBlocksPerStage, kTileRows, false)
         : encode_tmap_2d(&tsw, a.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)blocks,
                          (uint64_t)a.rows, (uint64_t)blocks * 4, kBlocksPerStage, kTileRows, false);
  if (!ok_w || !encode_tmap_2d(&tsx, a.xsc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)blocks,
                               (uint64_t)a.n, (uint64_t)blocks * 4, kBlocksPerStage, TOK, false))
    return kErrUnsupported;
  const void* kern = gather != nullptr ? (const void*)gemm_narrow_kernel<Q4, TOK, true>
                                       : (const void*)gemm_narrow_kernel<Q4, TOK>;
  static bool configured[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int variant = gather != nullptr ? 1 : 0;
  if (!configured[variant][dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemTc) != cudaSuccess)
      return kErrCuda;
    configured[variant][dev & 63] = true;
  }
  const int64_t row_tiles = (a.rows + kTileRows - 1) / kTileRows;
  const int64_t tiles = row_tiles * ((a.n + TOK - 1) / TOK);
  TcGatherArgs t{};
  static_cast<TcArgs&>(t) = TcArgs{a.scales, a.xsc, a.ys, a.rows, a.cols, a.n, a.ldy, a.status, 1, row_tiles, tiles};
  if (gather != nullptr) {
    t.gather_n = gather->world;
    t.gather_row0 = gather->row0;
    for (int p = 0; p < gather->world; p++) t.gather_ys[p] = gather->ys[p];
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)min64(tiles, (int64_t)sm_count()), 1, 1);
  cfg.blockDim = dim3(S::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nstages = stages;
  void* params[] = {&t, &nstages, &lookahead, &tw, &tx, &tsw, &tsx};
  return cudaLaunchKernelExC(&cfg, kern, params) == cudaSuccess ? kOk : kErrCuda;
}

// The drain step alone, for measuring the GEMM's own ceiling: the drain warps
// of one CTA per SM run the GEMM's per-block step - TMEM load of a block's
// 32 x 32 int32 tile, exact conversion, rank-1 scale product and f32x2
// accumulate - over `nst` stages of four blocks, with no MMA, no TMA and no
// barrier between them (the D slots hold the seed value). Each thread's sums
// go to out[] so that nothing is optimized away.
__global__ void __launch_bounds__(TcShape<false>::kThreads, 1)
    drain_probe_kernel(int nst, float* out) {
  __shared__ __align__(16) float sx_s[kBlocksPerStage * kTileTok];
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < kBlocksPerStage * kTileTok; i += blockDim.x) sx_s[i] = 1.0f + 1e-3f * (float)i;
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (warp >= 2 && warp < 2 + kEpiWarps) {
    const int quarter = warp & 3, sub = (warp - 2) >> 2, parity = sub & 1, col0 = (sub >> 1) * kEpiCols;
    const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0;
#pragma unroll
    for (int q = 0; q < kSlots; q++)
#pragma unroll
      for (int c = 0; c < kEpiCols; c += 32) tmem_fill32(tlane + (uint32_t)(q * kTileTok + c), kSeed);
    tmem_wait_st();
    uint64_t acc[kEpiCols / 2];
#pragma unroll
    for (int j = 0; j < kEpiCols / 2; j++) acc[j] = 0;
    int32_t dn[kEpiCols];
    const float sw = 0.01f + 1e-5f * (float)lane;
    for (int k = 0; k < nst; k++) {
      const int slot0 = (k & 1) * kBlocksPerStage;
#pragma unroll
      for (int q = parity; q < kBlocksPerStage; q += 2) {
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 32)
          tmem_ld32(tlane + (uint32_t)((slot0 + q) * kTileTok + c), *reinterpret_cast<int32_t(*)[32]>(dn + c));
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 32) tmem_wait_ld_regs(*reinterpret_cast<int32_t(*)[32]>(dn + c));
        const uint64_t sw2 = f2_pack(sw, sw);
        const float* sxq = sx_s + q * kTileTok + col0;
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
          const float4 x4 = *reinterpret_cast<const float4*>(sxq + j);
          acc[j / 2] = f2_fma(slot_to_f2<true>(dn[j], dn[j + 1]), f2_mul(sw2, f2_pack(x4.x, x4.y)), acc[j / 2]);
          acc[j / 2 + 1] = f2_fma(slot_to_f2<true>(dn[j + 2], dn[j + 3]), f2_mul(sw2, f2_pack(x4.z, x4.w)),
                                  acc[j / 2 + 1]);
        }
      }
    }
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kEpiCols / 2; j++)
      sum += __uint_as_float((uint32_t)acc[j]) + __uint_as_float((uint32_t)(acc[j] >> 32));
    out[(int64_t)blockIdx.x * blockDim.x + tid] = sum;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// The drain ceiling probe (see drain_probe_kernel): `ctas` CTAs, one per
// SM, `nst` stages of four blocks each; out holds ctas x kThreads floats.
// Each stage is 128 weight rows x 64 tokens x 4 blocks per CTA.
int64_t launch_drain_probe(int64_t ctas, int64_t nst, float* out, cudaStream_t stream) {
  if (ctas <= 0 || nst <= 0 || out == nullptr) return kErrArgs;
  drain_probe_kernel<<<(unsigned)ctas, TcShape<false>::kThreads, 0, stream>>>((int)nst, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// The tensor-core path needs 16-byte aligned weights and quantized
// activations (TMA), cols a multiple of 32, and the quantized activations
// written to device memory first (xq / xsc).
bool gemm_tc_supported(const LinearArgs& a) {
  return a.mode == 1 && a.cols % kBlock == 0 && a.cols > 0 && a.xq != nullptr &&
         a.xsc != nullptr && ((uintptr_t)a.qs & 15) == 0 && ((uintptr_t)a.xq & 15) == 0 &&
         ((uintptr_t)a.xs & 15) == 0 && ((uintptr_t)a.scales & (a.q4 ? 1 : 3)) == 0 &&
         ((uintptr_t)a.xsc & 3) == 0;
}

// Up to this many tokens the narrow kernel runs (16-token tiles up to 16,
// 32-token tiles above); DN_GEMM_NARROW overrides it (0: never).
static int64_t gemm_narrow_max() {
  static int64_t v = -1;
  if (v < 0) {
    const char* e = getenv("DN_GEMM_NARROW");
    v = e != nullptr ? atoll(e) : 32;
    if (v < 0) v = 0;
  }
  return v;
}

int64_t launch_gemm_tc(const LinearArgs& a, cudaStream_t stream) {
  if (!gemm_tc_supported(a)) return kErrUnsupported;
  if (a.rows <= 0 || a.n <= 0) return kOk;
  if (launch_quantize_q8(a.xs, a.xq, a.xsc, a.n, a.cols, stream) != cudaSuccess) return kErrCuda;
  if (a.n <= gemm_narrow_max()) {
    const int64_t rc = a.n <= 16 ? (a.q4 ? launch_narrow<true, 16>(a, stream) : launch_narrow<false, 16>(a, stream))
                                 : (a.q4 ? launch_narrow<true, 32>(a, stream) : launch_narrow<false, 32>(a, stream));
    if (rc != kErrUnsupported) return rc;
  }
  return a.q4 ? launch_tc<true>(a, stream) : launch_tc<false>(a, stream);
}

int64_t launch_gemm_tc_allgather(const LinearArgs& a, int64_t row0, float* const* ys, int* const* cnt, int world,
                                 cudaStream_t stream) {
  if (!gemm_tc_supported(a) || world < 1 || world > kMaxGatherRanks) return kErrArgs;
  if (a.rows <= 0 || a.n <= 0) return kOk;
  for (int p = 0; p < world; p++)
    if (ys[p] == nullptr || cnt[p] == nullptr || ((uintptr_t)ys[p] & 3) != 0 || ((uintptr_t)cnt[p] & 3) != 0)
      return kErrArgs;
  if (launch_quantize_q8(a.xs, a.xq, a.xsc, a.n, a.cols, stream) != cudaSuccess) return kErrCuda;
  const TcGather g{world, row0, ys, cnt};
  int64_t rc = kErrUnsupported;
  if (a.n <= gemm_narrow_max())  // the same kernel choice as launch_gemm_tc
    rc = a.n <= 16 ? (a.q4 ? launch_narrow<true, 16>(a, stream, &g) : launch_narrow<false, 16>(a, stream, &g))
                   : (a.q4 ? launch_narrow<true, 32>(a, stream, &g) : launch_narrow<false, 32>(a, stream, &g));
  if (rc == kErrUnsupported) rc = a.q4 ? launch_tc<true>(a, stream, &g) : launch_tc<false>(a, stream, &g);
  if (rc != kOk) return rc;
  // The counters' addresses travel by value.
  PeerCounters c{};
  for (int p = 0; p < world; p++) c.p[p] = cnt[p];
  peer_signal_kernel<<<1, 1, 0, stream>>>(c, world, a.status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace dn
