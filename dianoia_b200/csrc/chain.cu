// Decode chain: a sequence of quantized products (a token's projections) run
// by one persistent kernel, so HBM keeps streaming across the dependencies
// between them.
//
// Each op is a decode GEMV (gemv_core.cuh: exact reference order, 32-row
// tiles, QA activations in and optionally QA activations out). The ops' tiles
// are dealt round-robin over the grid, continuing from op to op, so a CTA's
// tiles of consecutive ops rarely coincide. Every CTA's producer warp streams
// the weights of all its tiles of all ops, in order, through the stage ring:
// the weights never depend on the activations, so while the consumers wait
// for an op's input, the next weights are already on their way. An op with a
// dependency waits for that op's completion counter (one increment per
// finished tile, published after the tile's QA output with a gpu-scope
// release) - a bounded spin by one thread, then a CTA barrier - and reads its
// input through L2 (ld.global.cg), never a stale L1 line. The dependency is
// either a data edge (the input is the earlier op's QA output) or an ordering
// edge (the input was written before the launch; the op still starts only
// after the earlier one, as it would with a step outside the chain between
// them).
//
// The grid is launched cooperatively (all CTAs co-resident), so no CTA can
// wait on one that has not started; every wait is bounded anyway. The last
// CTA to finish resets the counters for the next launch.
#include <stdio.h>
#include <string.h>

#include <vector>

#include "dn_tmap.h"
#include "gemv_core.cuh"

namespace dn {

// Device-side op table entry (tensor maps first: 64-byte aligned).
struct alignas(64) ChainOpDev {
  CUtensorMap tw;         // weights: boxes of 32 rows x 128 bytes, 128-byte swizzle
  CUtensorMap tsc;        // scales: boxes of 32 rows x 64 bytes (when tma_scales)
  const void* scales;     // scales in global memory (when not tma_scales)
  const uint8_t* xa;      // QA input of the op
  float* ys;              // f32 outputs or null
  uint8_t* ya;            // QA outputs or null
  int32_t rows, cols;
  int32_t dep;            // op to wait for (it produces xa, or only precedes this op), or -1
  int32_t ext_input;      // xa was written before the launch (wait for the previous kernel)
  int32_t ntiles;         // 32-row tiles of the op
  int32_t tile_base;      // global index of the op's first tile (round-robin deal)
  int32_t tma_scales;
};

struct ChainHost {
  ChainOpDev* ops_dev = nullptr;  // nops entries
  int* counters = nullptr;        // nops + 1 ints (the last: CTAs done)
  int nops = 0;
  bool q4 = false;
  int64_t max_cols = 0;
  int device = 0;
};

namespace {

using namespace gemv;

// A barrier of the consumer warps with a bounded wait (two mbarriers used in
// turn), so a warp that gave up can never leave the others waiting forever.
__device__ __forceinline__ bool consumers_sync_bounded(uint64_t* bars, uint32_t& uses,
                                                       uint32_t* status) {
  uint64_t* b = &bars[uses & 1];
  const uint32_t parity = (uses >> 1) & 1u;
  uses++;
  mbar_arrive(b);
  return warp_wait(b, parity, status);
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <bool Q4>
__global__ void __launch_bounds__(kThreads)
    chain_kernel(const ChainOpDev* __restrict__ ops, const int nops, int* counters,
                 uint32_t* status, const int stages, const int64_t max_cols) {
  using F = Fmt<Q4>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const SmemPlan sp = plan<Q4>(stages, 1, max_cols, false);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sp.bar_off);
  uint64_t* empty = full + stages;
  uint64_t* csync = empty + stages;  // the consumer-group barriers
  uint64_t* epi = csync + 2;
  uint8_t* xw_s = smem + sp.xw_off;
  float* xs_s = reinterpret_cast<float*>(smem + sp.xs_off);
  float* yt_s = reinterpret_cast<float*>(smem + sp.yt_off);
  uint8_t* stg_s = smem + sp.stg_off;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, bid = blockIdx.x;
  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(&csync[0], kConsumers);
    mbar_init(&csync[1], kConsumers);
    mbar_init(&epi[0], kConsumers);
    mbar_init(&epi[1], kConsumers);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // This CTA's tiles of op o: global tile indices tile_base + t with
  // (tile_base + t) % G == bid.
  auto first_tile = [&](const ChainOpDev& o) { return ((bid - o.tile_base) % G + G) % G; };

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int64_t k = 0;
      for (int op = 0; op < nops && !abort_flag; op++) {
        const ChainOpDev& o = ops[op];
        const int64_t blocks = o.cols / kBlock;
        const int nch = (int)((blocks + F::kKC - 1) / F::kKC);
        prefetch_tmap(&o.tw);
        for (int t = first_tile(o); t < o.ntiles && !abort_flag; t += G) {
          for (int c = 0; c < nch; c++) {
            if (k >= stages &&
                !mbar_wait_bounded(&empty[s], ph ^ 1u, status, kStatusTmaTimeout)) {
              abort_flag = 1;
              break;
            }
            const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
            uint8_t* stage = smem + (int64_t)s * kStageBytes;
            if (o.tma_scales)
              issue_stage<Q4, true>(stage, &o.tw, &o.tsc, c, nb, t * kRows, &full[s]);
            else
              issue_stage<Q4, false>(stage, &o.tw, &o.tsc, c, nb, t * kRows, &full[s]);
            k++;
            if (++s == stages) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
      if (abort_flag) {
        // Let the copies already issued land (bounded) before the CTA's memory goes.
        for (int j = 0; j < stages; j++) {
          if (k - 1 - j < 0) break;
          const int64_t kk = k - 1 - j;
          mbar_wait_bounded(&full[kk % stages], (uint32_t)(kk / stages) & 1u, status,
                            kStatusTmaTimeout);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int r8 = lane >> 2, l = lane & 3;
  const int row_local = warp * 8 + r8;
  bool waited_launch = false;
  uint32_t syncs = 0;
  int s = 0;
  uint32_t ph = 0;
  uint32_t e = 0;
  for (int op = 0; op < nops; op++) {
    const ChainOpDev& o = ops[op];
    const int t_first = first_tile(o);
    if (t_first >= o.ntiles) continue;  // no tile of this op here
    const int64_t blocks = o.cols / kBlock;
    const int nch = (int)((blocks + F::kKC - 1) / F::kKC);
    // The op's input: an earlier op's output (its counter) or, for inputs
    // made before the launch, the previous kernel in the stream (PDL).
    if (o.ext_input && !waited_launch) {
      pdl_wait();
      waited_launch = true;
    }
    if (o.dep >= 0) {
      if (tid == 0) {
        const int target = ops[o.dep].ntiles;
        const int* cnt = counters + o.dep;
        if (ld_acquire(cnt) < target) {
          const uint64_t start = globaltimer_ns();
          for (uint32_t it = 1;; it++) {
            if (ld_acquire(cnt) >= target) break;
            if ((it & 63u) == 0 && globaltimer_ns() - start > kWaitLimitNs) {
              report(status, kStatusPeerTimeout);
              abort_flag = 1;
              break;
            }
          }
        }
      }
    }
    if (!consumers_sync_bounded(csync, syncs, status) || abort_flag) {
      abort_flag = 1;
      return;
    }
    // The QA input, through L2, into the lane-interleaved layout. (The
    // previous op's tiles of this CTA are done with the activations: every
    // consumer passed its last stage before reaching the barrier above.)
    {
      const int64_t words = blocks * kQABytes / 4;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(o.xa);
      uint32_t* dst = reinterpret_cast<uint32_t*>(stg_s);
      for (int64_t i = tid; i < words; i += kConsumers) dst[i] = __ldcg(src + i);
      if (!consumers_sync_bounded(csync, syncs, status)) {
        abort_flag = 1;
        return;
      }
      unpack_qa<Q4>(stg_s, xw_s, xs_s, blocks);
      if (!consumers_sync_bounded(csync, syncs, status)) {
        abort_flag = 1;
        return;
      }
    }
    const LaneCtx lc{row_local, r8, l, (uint32_t)row_local * kBoxBytes,
                     xw_s + l * XLayout<Q4>::kLaneBytes, sp.xw_stride, xs_s, sp.xs_stride,
                     static_cast<const uint8_t*>(o.scales), 0, blocks};
    for (int t = t_first; t < o.ntiles; t += G) {
      const int64_t row0 = (int64_t)t * kRows;
      const int tile_rows = (int)min64(kRows, o.rows - row0);
      LaneCtx c = lc;
      c.row = row0 + min(row_local, tile_rows - 1);
      float acc[1] = {0.0f};
      for (int ch = 0; ch < nch; ch++) {
        if (!warp_wait(&full[s], ph, status)) {
          abort_flag = 1;
          return;  // the producer drains what it issued; every other wait is bounded
        }
        const int nb = (int)min64(F::kKC, blocks - (int64_t)ch * F::kKC);
        const uint8_t* stage = smem + (int64_t)s * kStageBytes;
        if (o.tma_scales)
          gemv_stage<Q4, 1, true>(stage, nb, ch * F::kKC, c, acc);
        else
          gemv_stage<Q4, 1, false>(stage, nb, ch * F::kKC, c, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      const float y = lane_reduce(acc[0]);
      float* yt = yt_s + (e & 1) * kRows;
      if (l == 0 && row_local < tile_rows) {
        if (o.ys != nullptr) o.ys[row0 + row_local] = y;
        yt[row_local] = y;
      }
      if (o.ya != nullptr && tile_rows == kRows) {
        mbar_arrive(&epi[e & 1]);
        if (!warp_wait(&epi[e & 1], (e >> 1) & 1u, status)) {
          abort_flag = 1;
          return;
        }
        if (warp == 0) {
          quantize_block_out(yt[lane], o.ya + (int64_t)t * kQABytes, lane);
          __syncwarp();
          if (lane == 0) {
            // Publish the tile: its QA block is visible before the count.
            __threadfence();
            atomicAdd(counters + op, 1);
          }
        }
        e++;
      } else if (o.ya == nullptr) {
        // Outputs only in f32: count the tile once its stores are issued.
        __syncwarp();
        if (warp == 0 && lane == 0) {
          __threadfence();
          atomicAdd(counters + op, 1);
        }
      }
    }
  }
  // The last CTA out resets the counters for the next launch. (When thread 0
  // of every CTA is here, every dependency wait and counter increment of the
  // launch is behind it.)
  if (tid == 0 && !abort_flag) {
    __threadfence();
    if (atomicAdd(counters + nops, 1) == G - 1) {
      for (int i = 0; i <= nops; i++) counters[i] = 0;
      __threadfence();
    }
  }
}

// Ops of different layers run at the same time (a CTA moves on to its tiles
// of the next op as soon as its own are done), so only the dep edges order
// them. Every output must therefore be written by one op and read only by
// ops that wait for it: no output may overlap another op's output, weights
// or scales, nor any op's input except through a dep edge (op j with
// dep == i reading inside i's QA output).
struct Range {
  uintptr_t lo, hi;
  bool overlaps(const Range& o) const { return lo < o.hi && o.lo < hi && lo < hi && o.lo < o.hi; }
};

static bool chain_buffers_disjoint(const ChainOpSpec* specs, int64_t nops, bool q4) {
  auto span = [](const void* p, int64_t bytes) {
    const uintptr_t a = (uintptr_t)p;
    return Range{a, p == nullptr ? a : a + (uintptr_t)bytes};
  };
  std::vector<Range> outs, ins, consts;  // per op: ys, ya; xa; qs, scales
  for (int64_t i = 0; i < nops; i++) {
    const ChainOpSpec& s = specs[i];
    const int64_t blocks = s.cols / kBlock;
    outs.push_back(span(s.ys, s.rows * 4));
    outs.push_back(span(s.ya, s.rows / kRows * kQABytes));
    ins.push_back(span(s.xa, blocks * kQABytes));
    consts.push_back(span(s.qs, s.rows * blocks * (q4 ? 16 : 32)));
    consts.push_back(span(s.scales, s.rows * blocks * (q4 ? 2 : 4)));
  }
  for (int64_t i = 0; i < nops; i++) {
    for (int k = 0; k < 2; k++) {
      const Range& o = outs[(size_t)(2 * i + k)];
      for (int64_t j = 0; j < nops; j++) {
        if (j != i && (o.overlaps(outs[(size_t)(2 * j)]) || o.overlaps(outs[(size_t)(2 * j + 1)])))
          return false;
        if (k == 0 && i == j && o.overlaps(outs[(size_t)(2 * i + 1)])) return false;
        if (o.overlaps(consts[(size_t)(2 * j)]) || o.overlaps(consts[(size_t)(2 * j + 1)]))
          return false;
        // Reading an output is allowed only for the op's dependents, and
        // only its QA output (checked by the caller to contain the input).
        if (o.overlaps(ins[(size_t)j]) && !(k == 1 && specs[j].dep == i)) return false;
      }
    }
  }
  return true;
}

}  // namespace

int64_t chain_create(const ChainOpSpec* specs, int64_t nops, bool q4, ChainHost** out) {
  if (nops <= 0 || specs == nullptr || out == nullptr) return kErrArgs;
  std::vector<ChainOpDev> table((size_t)nops);
  int64_t tile_base = 0, max_cols = 0;
  for (int64_t i = 0; i < nops; i++) {
    const ChainOpSpec& sp = specs[i];
    ChainOpDev& d = table[(size_t)i];
    memset(&d, 0, sizeof d);
    const int64_t blocks = sp.cols / kBlock;
    if (sp.rows <= 0 || sp.cols <= 0 || sp.cols % kBlock != 0 || sp.xa == nullptr ||
        ((uintptr_t)sp.qs & 15) != 0 || ((uintptr_t)sp.xa & 3) != 0 ||
        (sp.ya != nullptr && ((uintptr_t)sp.ya & 3) != 0) || sp.dep >= i || sp.dep < -1 ||
        sp.rows > INT32_MAX / 2 || sp.cols > INT32_MAX / 2)
      return kErrArgs;
    if (sp.ya != nullptr && sp.rows % kRows != 0) return kErrArgs;     // QA outputs: whole blocks
    d.ext_input = 1;
    if (sp.dep >= 0 && specs[sp.dep].ya != nullptr) {
      // A data edge: the input lies inside the QA output of op dep, on a
      // block boundary. An input that does not touch that output was written
      // before the launch (an ordering edge).
      const ChainOpSpec& p = specs[sp.dep];
      const uint8_t *lo = p.ya, *hi = p.ya + p.rows / kRows * kQABytes;
      const uint8_t* end = sp.xa + blocks * kQABytes;
      if (sp.xa < hi && lo < end) {
        if (sp.xa < lo || (sp.xa - lo) % kQABytes != 0 || end > hi) return kErrArgs;
        d.ext_input = 0;
      }
    }
    const int64_t wb = q4 ? 16 : 32, sb = q4 ? 2 : 4;
    if (!encode_tmap_2d(&d.tw, sp.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(blocks * wb),
                        (uint64_t)sp.rows, (uint64_t)(blocks * wb), kBoxBytes, kRows, true))
      return kErrUnsupported;
    d.tma_scales = ((uintptr_t)sp.scales & 15) == 0 && (blocks * sb) % 16 == 0;
    if (d.tma_scales &&
        !encode_tmap_2d(&d.tsc, sp.scales, q4 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        (uint64_t)blocks, (uint64_t)sp.rows, (uint64_t)(blocks * sb),
                        (uint32_t)(kChunkBytes / wb), kRows, false))
      return kErrUnsupported;
    d.scales = sp.scales;
    d.xa = sp.xa;
    d.ys = sp.ys;
    d.ya = sp.ya;
    d.rows = (int32_t)sp.rows;
    d.cols = (int32_t)sp.cols;
    d.dep = (int32_t)sp.dep;
    d.ntiles = (int32_t)((sp.rows + kRows - 1) / kRows);
    d.tile_base = (int32_t)(tile_base % (1 << 30));
    tile_base += d.ntiles;
    max_cols = sp.cols > max_cols ? sp.cols : max_cols;
  }
  if (!chain_buffers_disjoint(specs, nops, q4)) return kErrArgs;
  ChainHost* h = new ChainHost();
  h->nops = (int)nops;
  h->q4 = q4;
  h->max_cols = max_cols;
  cudaGetDevice(&h->device);
  if (cudaMalloc(&h->ops_dev, sizeof(ChainOpDev) * (size_t)nops) != cudaSuccess ||
      cudaMalloc(&h->counters, sizeof(int) * (size_t)(nops + 1)) != cudaSuccess ||
      cudaMemcpy(h->ops_dev, table.data(), sizeof(ChainOpDev) * (size_t)nops,
                 cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(h->counters, 0, sizeof(int) * (size_t)(nops + 1)) != cudaSuccess) {
    chain_destroy(h);
    return kErrCuda;
  }
  *out = h;
  return kOk;
}

void chain_destroy(ChainHost* h) {
  if (h == nullptr) return;
  if (h->ops_dev != nullptr) cudaFree(h->ops_dev);
  if (h->counters != nullptr) cudaFree(h->counters);
  delete h;
}

template <bool Q4>
static int64_t chain_launch_t(ChainHost* h, uint32_t* status, cudaStream_t stream, bool pdl) {
  const SmemPlan base = plan<Q4>(0, 1, h->max_cols, false);
  int per_sm = 2;
  int stages = (int)((kSmemPerSM / per_sm - 1024 - base.total) / (kStageBytes + 16));
  if (stages < 3) {
    per_sm = 1;
    stages = (int)((kMaxSmem - base.total) / (kStageBytes + 16));
  }
  stages = stages > kMaxStages ? kMaxStages : stages;
  if (stages < 2) return kErrTooLarge;
  const SmemPlan sp = plan<Q4>(stages, 1, h->max_cols, false);
  auto kern = chain_kernel<Q4>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return kErrCuda;
    configured[dev & 63] = true;
  }
  int sms = kSMs, max_blocks = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&max_blocks, kern, kThreads, (size_t)sp.total) !=
          cudaSuccess ||
      max_blocks < 1)
    return kErrCuda;
  const int grid = sms * (max_blocks < per_sm ? max_blocks : per_sm);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)sp.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const ChainOpDev* ops = h->ops_dev;
  return cudaLaunchKernelEx(&cfg, kern, ops, h->nops, h->counters, status, stages, h->max_cols) ==
                 cudaSuccess
             ? kOk
             : kErrCuda;
}

int64_t chain_launch(ChainHost* h, uint32_t* status, cudaStream_t stream, bool pdl) {
  if (h == nullptr) return kErrArgs;
  return h->q4 ? chain_launch_t<true>(h, status, stream, pdl)
               : chain_launch_t<false>(h, status, stream, pdl);
}

int64_t chain_reset(ChainHost* h, cudaStream_t stream) {
  if (h == nullptr) return kErrArgs;
  return cudaMemsetAsync(h->counters, 0, sizeof(int) * (size_t)(h->nops + 1), stream) == cudaSuccess
             ? kOk
             : kErrCuda;
}

}  // namespace dn
