// Decode stack: the one-token Q8_0 products of a decode step (a token's
// projections, each the lab_gemm_q8 mode-1 product of lab_native.c:553-579
// on the previous projection's f32 output) run by ONE persistent kernel with
// one CTA per SM, every product's rows split evenly over all SMs.
//
// Why this shape. A batch-1 token is a chain of dependent products: each
// needs all of its predecessor's outputs. Per product the time is then
// (hand-off latency) + (the slowest SM's dot products after its input
// arrives), while the weights, which never depend on activations, can stream
// ahead through each SM's shared-memory ring. So:
//   * every product's rows are divided over all SMs in equal contiguous
//     slices (T rows per tile, T <= 32, nt tiles per CTA), so that no SM has
//     more than its share of either the stream or the serial work;
//   * the producer warp streams the CTA's slices of all products in order,
//     whole stages of T rows x 512 or 1024 bytes in one 3-D TMA copy
//     (T <= 16 rows take 1024-byte stages, so a short slice is few stages);
//   * a product's outputs are plain f32 stores; the CTA then adds one to the
//     product's counter with a gpu-scope release. A dependent CTA's thread 0
//     polls that counter (relaxed, then one acquire), and every consumer
//     thread reads the f32 input through L2 and quantizes it itself
//     (lab_quantize_q8 semantics), so the hand-off is one counter round trip
//     and one L2 read: no per-tile quantized blocks, no grid completion.
//
// Arithmetic (bit-exact with the reference): per row, the reference's four
// accumulators over the blocks in order, acc_l = fma(f32(d_l), f32(sw * sx),
// acc_l), d_l the int32 sum over bytes 4l..4l+3 and 16+4l..16+4l+3 of the
// block, and y = (acc0 + acc1) + (acc2 + acc3) (lab_native.c:456-466 NEON,
// 483-512 AVX2). d_l comes exactly from a dp4a chain seeded with 0x4B400000
// (the float 1.5 * 2^23, ulp 1) and one exact subtraction; sw * sx is one
// round-to-nearest product. A row's result does not depend on the row split
// (lab_native.c:550-552).
//
// Inside a CTA, four consumer warps of eight rows, four lanes per row: lane
// l of row r keeps the reference's accumulator l. Only the fma chain is
// serial; a lane first loads half a stage (4 chunks: 16 blocks' weight words,
// activation words and both scales) into registers and then does the math,
// so the shared-memory latency is paid once per half stage, not per block.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "dn_common.cuh"
#include "dn_launch.h"
#include "dn_tmap.h"
#include "gemv_core.cuh"

namespace dn {

struct alignas(64) StackOpDev {
  CUtensorMap tw;   // weights: {128 bytes, rows, chunks of a row}, box {128, T, cpr}
  CUtensorMap tsc;  // scales: {blocks, rows} f32, box {4 * cpr, T}
  const float* x;   // f32 input [cols]
  float* y;         // f32 output [rows]
  int32_t rows, cols;
  int32_t dep;      // earlier op to wait for, or -1 (input written before the launch)
  int32_t T;        // rows per tile (the box height), <= 32
  int32_t nt;       // tiles per CTA
  int32_t cpr;      // 128-byte lines per row per stage: 4 (16 blocks) or 8 (32 blocks)
  int32_t nctas;    // CTAs holding rows of the op (the counter's count per run)
  int32_t pad;
};

struct StackHost {
  StackOpDev* ops_dev = nullptr;
  int* counters = nullptr;  // nops per-op counts, then CTAs done, then the run index
  int nops = 0;
  int grid = 0;
  int64_t max_blocks = 0;
};

namespace {

using gemv::exact_d2;
using gemv::f2_hi;
using gemv::f2_lo;
using gemv::f2_mul;
using gemv::f2_pack;
using gemv::kMagic;
using gemv::kMaxSmem;
using gemv::lds;

constexpr int kCWarps = 4;                // consumer warps: 8 rows each, 32-row tiles at most
constexpr int kCThreads = 32 * kCWarps;
constexpr int kThreads = kCThreads + 32;  // + the producer warp
constexpr int kSlotBytes = 18 * 1024;
constexpr int kScaleOff = 16 * 1024;
constexpr int kMaxT = 32;
constexpr int kMaxStagesS = 16;
constexpr int64_t kMaxCols = 8192;  // the quantized input sits in shared memory beside the ring

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const int* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ld_acquire_gpu(const int* p) {
  asm volatile("{\n\t.reg .b32 t;\n\tld.acquire.gpu.global.b32 t, [%0];\n\t}" ::"l"(p) : "memory");
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The producer's wait for a free slot: a spin (a sleeping try_wait woke up
// measurably late), bounded at `mult` times the limit because the consumers
// free slots only after their own bounded waits.
__device__ __forceinline__ bool spin_wait(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t mult) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - start > mult * wait_limit_ns()) {
      report(status, kStatusTmaTimeout);
      return false;
    }
  }
}

// Barrier of the consumer warps with an AND of `v` (every consumer thread
// reaches each one: a thread that gave up a wait carries on to the next
// barrier with v false, and all leave together).
__device__ __forceinline__ bool cons_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kCThreads)
      : "memory");
  return r != 0;
}

// Shared memory after the slots: full and empty barriers, the quantized
// input (32 bytes per block, lane l's words l and 4 + l at 8 l) and its
// block scales.
struct Plan {
  int64_t bar_off, xw_off, xs_off, total;
};
__host__ __device__ inline Plan plan(int stages, int64_t max_blocks) {
  Plan p;
  p.bar_off = (int64_t)stages * kSlotBytes;
  p.xw_off = gemv::round_up(p.bar_off + 16 * stages, 128);
  p.xs_off = p.xw_off + max_blocks * 32;
  p.total = gemv::round_up(p.xs_off + max_blocks * 4, 16) + 1024;  // + alignment slack
  return p;
}

// The f32 input (written by another SM in this kernel, or before it) read
// through L2 and quantized per 32-block with lab_quantize_q8's arithmetic
// (lab_native.c:407-429) into the lane-interleaved layout. Two threads per
// block, thread h holding values 16h..16h+15 (words 4h..4h+3 of the block):
// a 2048-value input is one round of 64 blocks. The loads of every round are
// issued before any is used; this step sits between a product's input
// arriving and its dot products, so its latency is the hop's.
__device__ __forceinline__ void quantize_input(const float* x, int64_t blocks, uint8_t* xw, float* xs, int t) {
  constexpr int kPer = kCThreads / 2;  // blocks per round
  constexpr int kMaxRounds = (int)(kMaxCols / kBlock / kPer);
  const int h = t & 1;
  const int rounds = (int)((blocks + kPer - 1) / kPer);
  float4 v[kMaxRounds][4];
#pragma unroll
  for (int u = 0; u < kMaxRounds; u++) {
    if (u < rounds) {
      const int64_t b = (int64_t)u * kPer + (t >> 1);
      const float4* src = reinterpret_cast<const float4*>(x + b * kBlock + 16 * h);
#pragma unroll
      for (int k = 0; k < 4; k++) v[u][k] = b < blocks ? __ldcg(src + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int u = 0; u < kMaxRounds; u++) {
    if (u < rounds) {
      const int64_t b = (int64_t)u * kPer + (t >> 1);
      float amax = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; k++)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[u][k].x), fabsf(v[u][k].y)), fmaxf(fabsf(v[u][k].z), fabsf(v[u][k].w))));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      float scale, inv;
      q8_scale(amax, scale, inv);
      if (b < blocks) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const uint32_t word = pack4(quant_q8_elem(v[u][k].x, inv), quant_q8_elem(v[u][k].y, inv),
                                      quant_q8_elem(v[u][k].z, inv), quant_q8_elem(v[u][k].w, inv));
          // word w = 4h + k of the block: lane w % 4's slot, first or second half.
          *reinterpret_cast<uint32_t*>(xw + b * 32 + 8 * k + 4 * h) = word;
        }
        if (h == 0) xs[b] = scale;
      }
    }
  }
}

// Accumulator l of row r over one stage of 4 * CPR blocks of a T-row tile,
// four 128-byte chunks (16 blocks) at a time: every load of the four chunks
// first, then their math. st: the slot; xb: the lane's activation words of
// the stage's first block (8 bytes per block at 32-byte steps); xsb: that
// block's activation scale.
template <int CPR>
__device__ __forceinline__ void stage_q8(const uint8_t* st, int T, int r, int l, const uint8_t* xb,
                                         const float* xsb, float& acc) {
  const uint8_t* sbase = st + kScaleOff + (CPR == 4 ? r * 64 : r * 128);
#pragma unroll
  for (int c0 = 0; c0 < CPR; c0 += 4) {
    uint32_t w0[16], w1[16];
    uint2 xv[16];
    float4 sv[4], x4[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int c = c0 + j;
      const int L = c * T + r;
      const uint8_t* line = st + L * 128 + 4 * l;
      const int x7 = L & 7;
      sv[j] = lds<float4>(sbase + ((CPR == 4 ? (c ^ ((r >> 1) & 3)) : (c ^ (r & 7))) << 4));
      x4[j] = lds<float4>(xsb + 4 * c);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        w0[4 * j + q] = lds<uint32_t>(line + (((2 * q) ^ x7) << 4));
        w1[4 * j + q] = lds<uint32_t>(line + (((2 * q + 1) ^ x7) << 4));
        xv[4 * j + q] = lds<uint2>(xb + (4 * c + q) * 32);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint64_t s01 = f2_mul(f2_pack(sv[j].x, sv[j].y), f2_pack(x4[j].x, x4[j].y));
      const uint64_t s23 = f2_mul(f2_pack(sv[j].z, sv[j].w), f2_pack(x4[j].z, x4[j].w));
      int32_t d[4];
#pragma unroll
      for (int q = 0; q < 4; q++)
        d[q] = __dp4a((int32_t)w1[4 * j + q], (int32_t)xv[4 * j + q].y,
                      __dp4a((int32_t)w0[4 * j + q], (int32_t)xv[4 * j + q].x, kMagic));
      const uint64_t d01 = exact_d2(d[0], d[1]), d23 = exact_d2(d[2], d[3]);
      acc = __fmaf_rn(f2_lo(d01), f2_lo(s01), acc);
      acc = __fmaf_rn(f2_hi(d01), f2_hi(s01), acc);
      acc = __fmaf_rn(f2_lo(d23), f2_lo(s23), acc);
      acc = __fmaf_rn(f2_hi(d23), f2_hi(s23), acc);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    stack_kernel(const StackOpDev* __restrict__ ops, const int nops, int* counters, uint32_t* status,
                 const int stages, const int64_t max_blocks) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const Plan pl = plan(stages, max_blocks);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pl.bar_off);
  uint64_t* empty = full + stages;
  uint8_t* xw = smem + pl.xw_off;
  float* xs = reinterpret_cast<float*>(smem + pl.xs_off);
  __shared__ volatile int abort_flag;
  __shared__ uint32_t run_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bid = blockIdx.x, G = gridDim.x;
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
    // Weights never depend on the previous kernel: no dependent-launch wait.
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int64_t k = 0;
      bool ok = true;
      for (int op = 0; op < nops && ok; op++) {
        const StackOpDev& o = ops[op];
        if (bid >= o.nctas) continue;
        prefetch_tmap(&o.tw);
        prefetch_tmap(&o.tsc);
        const int nst = o.cols / (kBlock * 4 * o.cpr);
        const uint32_t bytes = (uint32_t)(o.T * o.cpr * 144);
        const int32_t r0 = bid * o.nt * o.T;
        for (int t = 0; t < o.nt && ok; t++) {
          for (int c = 0; c < nst; c++) {
            // Consumers free a slot only after their own bounded waits (a
            // counter, then a barrier), so this wait runs three times the limit.
            if (k >= stages && (abort_flag || !spin_wait(&empty[s], ph ^ 1u, status, 3))) {
              abort_flag = 1;
              ok = false;
              break;
            }
            uint8_t* slot = smem + (int64_t)s * kSlotBytes;
            mbar_arrive_expect_tx(&full[s], bytes);
            tma_load_3d(slot, &o.tw, 0, r0 + t * o.T, c * o.cpr, &full[s]);
            tma_load_2d(slot + kScaleOff, &o.tsc, c * 4 * o.cpr, r0 + t * o.T, &full[s]);
            k++;
            if (++s == stages) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land (bounded) before the CTA's memory goes.
        for (int j = 0; j < stages; j++) {
          const int64_t kk = k - 1 - j;
          if (kk < 0) break;
          mbar_wait_bounded(&full[kk % stages], (uint32_t)(kk / stages) & 1u, status, kStatusTmaTimeout);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_launch_dependents();
  pdl_wait();  // inputs written before the launch, and the run index
  if (tid == 0) run_s = ld_relaxed_gpu(counters + nops + 1);
  bool ok = cons_all(true);
  const uint32_t run = run_s;
  const int r = 8 * warp + (lane >> 2), l = lane & 3;
  const uint8_t* xw_l = xw + 8 * l;
  int s = 0;
  uint32_t ph = 0;
  for (int op = 0; op < nops && ok; op++) {
    const StackOpDev& o = ops[op];
    if (bid >= o.nctas) continue;
    if (o.dep >= 0 && tid == 0) {
      // This run's completions of op dep: (run + 1) x its CTAs (wrap-around
      // differences).
      const uint32_t target = (run + 1u) * (uint32_t)ops[o.dep].nctas;
      const int* cnt = counters + o.dep;
      if ((int32_t)(ld_relaxed_gpu(cnt) - target) < 0) {
        const uint64_t start = globaltimer_ns();
        for (uint32_t it = 1;; it++) {
          if ((int32_t)(ld_relaxed_gpu(cnt) - target) >= 0) break;
          if ((it & 63u) == 0 && globaltimer_ns() - start > wait_limit_ns()) {
            report(status, kStatusPeerTimeout);
            ok = false;
            break;
          }
        }
      }
      ld_acquire_gpu(cnt);
    }
    ok = cons_all(ok && !abort_flag);
    if (!ok) break;
    const int64_t blocks = o.cols / kBlock;
    quantize_input(o.x, blocks, xw, xs, tid);
    ok = cons_all(true);
    const int T = o.T, bps = 4 * o.cpr;
    const int nst = (int)(blocks / bps);
    const int32_t r0 = bid * o.nt * T;
    const bool rows_here = 8 * warp < T;  // warp-uniform: this warp holds rows of the tile
    for (int t = 0; t < o.nt && ok; t++) {
      float acc = 0.0f;
      const uint8_t* xb = xw_l;
      const float* xsb = xs;
      for (int c = 0; c < nst; c++) {
        if (!gemv::warp_wait(&full[s], ph, status)) {
          ok = false;
          break;
        }
        if (rows_here) {
          const uint8_t* st = smem + (int64_t)s * kSlotBytes;
          if (o.cpr == 8)
            stage_q8<8>(st, T, r, l, xb, xsb, acc);
          else
            stage_q8<4>(st, T, r, l, xb, xsb, acc);
        }
        xb += bps * 32;
        xsb += bps;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
      const float y = gemv::lane_reduce(acc);  // (acc0 + acc1) + (acc2 + acc3) on l == 0
      const int64_t row = (int64_t)r0 + (int64_t)t * T + r;
      if (rows_here && l == 0 && r < T && row < o.rows) o.y[row] = y;
    }
    // Every consumer's outputs of the op, then one release per CTA.
    ok = cons_all(ok);
    if (ok && tid == 0) red_release_gpu_add(counters + op, 1);
  }
  if (!ok) {
    abort_flag = 1;
    return;
  }
  // The last CTA out advances the run index for the next launch (every wait
  // of this launch on the counters is behind it).
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(counters + nops, 1) == G - 1) {
      counters[nops] = 0;
      counters[nops + 1] = (int)(run + 1u);
      __threadfence();
    }
  }
}

// Rows per tile and tiles per CTA for `rows` rows over `grid` CTAs: the
// fewest 32-row-or-smaller tiles per CTA, then the smallest tile that covers
// the rows, so the slices are as even as the tile height allows.
void split_rows(int64_t rows, int grid, int* T, int* nt, int* nctas) {
  const int64_t per = (int64_t)grid * kMaxT;
  const int64_t n = (rows + per - 1) / per;
  const int64_t t = (rows + (int64_t)grid * n - 1) / ((int64_t)grid * n);
  *T = (int)t;
  *nt = (int)n;
  *nctas = (int)((rows + t * n - 1) / (t * n));
}

}  // namespace

int64_t stack_create(const StackOpSpec* specs, int64_t nops, StackHost** out) {
  if (nops <= 0 || nops > (1 << 20) || specs == nullptr || out == nullptr) return kErrArgs;
  int dev = 0, sms = gemv::kSMs;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kErrCuda;
  std::vector<StackOpDev> table((size_t)nops);
  int64_t max_blocks = 0;
  for (int64_t i = 0; i < nops; i++) {
    const StackOpSpec& sp = specs[i];
    StackOpDev& d = table[(size_t)i];
    memset(&d, 0, sizeof d);
    const int64_t blocks = sp.cols / kBlock;
    if (sp.rows <= 0 || sp.cols <= 0 || sp.cols % (16 * kBlock) != 0 || sp.rows > INT32_MAX / 2 ||
        sp.cols > kMaxCols || sp.qs == nullptr || sp.scales == nullptr || sp.x == nullptr ||
        sp.y == nullptr || ((uintptr_t)sp.qs & 15) != 0 || ((uintptr_t)sp.scales & 15) != 0 ||
        ((uintptr_t)sp.x & 15) != 0 || ((uintptr_t)sp.y & 3) != 0 || sp.dep < -1 || sp.dep >= i)
      return kErrArgs;
    int T, nt, nctas;
    split_rows(sp.rows, sms, &T, &nt, &nctas);
    const int cpr = (T <= 16 && blocks % 32 == 0) ? 8 : 4;
    if (!encode_tmap_row_chunks(&d.tw, sp.qs, (uint64_t)sp.rows, (uint64_t)sp.cols, (uint32_t)T, (uint32_t)cpr) ||
        !(cpr == 4 ? encode_tmap_2d_sw64(&d.tsc, sp.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)blocks,
                                         (uint64_t)sp.rows, (uint64_t)blocks * 4, 16, (uint32_t)T)
                   : encode_tmap_2d(&d.tsc, sp.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)blocks,
                                    (uint64_t)sp.rows, (uint64_t)blocks * 4, 32, (uint32_t)T, true)))
      return kErrUnsupported;
    d.x = sp.x;
    d.y = sp.y;
    d.rows = (int32_t)sp.rows;
    d.cols = (int32_t)sp.cols;
    d.dep = (int32_t)sp.dep;
    d.T = T;
    d.nt = nt;
    d.cpr = cpr;
    d.nctas = nctas;
    max_blocks = blocks > max_blocks ? blocks : max_blocks;
  }
  // Each output belongs to one op: it may not overlap another op's output or
  // any weights, and an op may read it only through a dep edge to its writer.
  auto lo = [](const void* p) { return (uintptr_t)p; };
  for (int64_t i = 0; i < nops; i++) {
    const uintptr_t ylo = lo(specs[i].y), yhi = ylo + (uintptr_t)specs[i].rows * 4;
    for (int64_t j = 0; j < nops; j++) {
      const StackOpSpec& o = specs[j];
      const uintptr_t blocks = (uintptr_t)(o.cols / kBlock);
      const uintptr_t spans[3][2] = {{lo(o.qs), lo(o.qs) + (uintptr_t)o.rows * blocks * 32},
                                     {lo(o.scales), lo(o.scales) + (uintptr_t)o.rows * blocks * 4},
                                     {lo(o.y), lo(o.y) + (uintptr_t)o.rows * 4}};
      for (int k = 0; k < 3; k++) {
        if (k == 2 && j == i) continue;
        if (ylo < spans[k][1] && spans[k][0] < yhi) return kErrArgs;
      }
      const uintptr_t xlo = lo(o.x), xhi = xlo + (uintptr_t)o.cols * 4;
      if (j != i && xlo < yhi && ylo < xhi && o.dep != i) return kErrArgs;
      if (j == i && xlo < yhi && ylo < xhi) return kErrArgs;
    }
  }
  StackHost* h = new StackHost();
  h->nops = (int)nops;
  h->grid = sms;
  h->max_blocks = max_blocks;
  if (cudaMalloc(&h->counters, sizeof(int) * (size_t)(nops + 2)) != cudaSuccess ||
      cudaMemset(h->counters, 0, sizeof(int) * (size_t)(nops + 2)) != cudaSuccess ||
      cudaMalloc(&h->ops_dev, sizeof(StackOpDev) * (size_t)nops) != cudaSuccess ||
      cudaMemcpy(h->ops_dev, table.data(), sizeof(StackOpDev) * (size_t)nops, cudaMemcpyHostToDevice) !=
          cudaSuccess) {
    cudaGetLastError();
    stack_destroy(h);
    return kErrCuda;
  }
  *out = h;
  return kOk;
}

void stack_destroy(StackHost* h) {
  if (h == nullptr) return;
  if (h->ops_dev != nullptr) cudaFree(h->ops_dev);
  if (h->counters != nullptr) cudaFree(h->counters);
  delete h;
}

int64_t stack_launch(StackHost* h, uint32_t* status, cudaStream_t stream, bool pdl) {
  if (h == nullptr) return kErrArgs;
  const Plan base = plan(0, h->max_blocks);
  int stages = (int)((kMaxSmem - base.total) / (kSlotBytes + 16));
  stages = stages > kMaxStagesS ? kMaxStagesS : stages;
  if (stages < 2) return kErrTooLarge;
  const Plan sp = plan(stages, h->max_blocks);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    if (cudaFuncSetAttribute(stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess)
      return kErrCuda;
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)h->grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)sp.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they wait on one another
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const StackOpDev* ops = h->ops_dev;
  return cudaLaunchKernelEx(&cfg, stack_kernel, ops, h->nops, h->counters, status, stages, h->max_blocks) ==
                 cudaSuccess
             ? kOk
             : kErrCuda;
}

int64_t stack_reset(StackHost* h, cudaStream_t stream) {
  if (h == nullptr) return kErrArgs;
  return cudaMemsetAsync(h->counters, 0, sizeof(int) * (size_t)(h->nops + 2), stream) == cudaSuccess ? kOk
                                                                                                    : kErrCuda;
}

}  // namespace dn
