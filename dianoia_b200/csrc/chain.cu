// Decode chain: a sequence of quantized products (a token's projections) run
// by one persistent kernel, so HBM keeps streaming across the dependencies
// between them.
//
// Each op is a decode GEMV on QA activations (quaddot.cuh: the reference's
// exact summation order, four lanes per row, 32-row tiles), with f32 and/or
// QA outputs. A CTA is four consumer warps (one 32-row tile at a time) and a
// producer warp; several CTAs share an SM. The ops' tiles are dealt round-robin over the CTAs,
// continuing from op to op, so consecutive ops land on different CTAs. Each
// producer streams the weights of all of its CTA's tiles of all ops, in
// order, through the CTA's stage ring: weights never depend on activations,
// so while the consumer waits for an op's input the next weights are already
// on their way. An op with a dependency waits for that op's completion
// counter (one increment per finished tile, a gpu-scope release after the
// tile's outputs) - a bounded spin by one thread on relaxed loads, one
// acquire, then a bounded CTA barrier - and then reads its input through L2
// (ld.global.cg), never a stale L1 line. The dependency is either
// a data edge (the input is the earlier op's QA output) or an ordering edge
// (the input was written before the launch; the op still starts only after
// the earlier one, as it would with a step outside the chain between them).
//
// The grid is launched cooperatively (all CTAs co-resident), so no CTA can
// wait on one that has not started; every wait is bounded anyway. Counters
// only grow: run e of a chain waits for (e + 1) x the tiles of an op, e being
// a run index the last CTA of each run advances, so a run never has to clear
// what a faster GPU of a sharded chain may already be adding for the next one.
//
// Sharded chains (world > 1 GPUs): each rank computes its row slice of every
// op; a tile's QA block goes to the same place in every rank's region over
// NVLink (plain stores to peer memory), then lane 0 makes them visible
// system-wide (fence.acq_rel.sys) and adds one to every rank's counter of the
// op. No TMA reads or writes peer memory.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "dn_tmap.h"
#include "quaddot.cuh"

namespace dn {

// Device-side op table entry (tensor maps first: 64-byte aligned).
struct alignas(64) ChainOpDev {
  CUtensorMap tw;         // weights: boxes of 32 rows x 128 bytes, 128-byte swizzle
  CUtensorMap tsc;        // scales: boxes of 32 rows x 64 bytes, 64-byte swizzle (when tma_scales)
  const void* scales;     // scales in global memory (when not tma_scales)
  const uint8_t* xa;      // QA input of the op
  float* ys;              // f32 outputs or null
  uint8_t* ya;            // QA outputs or null
  int32_t rows, cols;
  int32_t dep;            // op to wait for (it produces xa, or only precedes this op), or -1
  int32_t ext_input;      // xa was written before the launch (wait for the previous kernel)
  int32_t ntiles;         // this rank's 32-row tiles of the op
  int32_t tile_base;      // index of the op's first tile in the round-robin deal
  int32_t tma_scales;
  int32_t tile0;          // the op's first tile here, in the whole output (0 unsharded)
  int32_t ntiles_total;   // tiles of all ranks (the count dependents wait for)
};

// Where the other ranks' copies of the region are: byte offsets from this
// rank's region to each rank's (0 for itself).
constexpr int kMaxWorld = 8;
struct PeerInfo {
  int32_t world, rank;
  int64_t delta[kMaxWorld];
};

struct ChainHost {
  ChainOpDev* ops_dev = nullptr;  // nops entries
  int* counters = nullptr;        // nops + 2 ints: per op, then CTAs done, then the run index
  bool owns_counters = true;
  int nops = 0;
  bool q4 = false;
  int64_t max_blocks = 0;
  int device = 0;
  PeerInfo peers{1, 0, {0}};
};

namespace {

using quad::kRows;
using gemv::Fmt;
using gemv::kStageBytes;
using gemv::kMaxStages;
using gemv::kSmemPerSM;
using gemv::kMaxSmem;
using gemv::kSMs;
using gemv::kBoxBytes;
using gemv::kChunkBytes;

constexpr int kConsumerWarps = quad::kWarps;
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kThreads = kConsumers + 32;  // + the producer warp

// Counter accesses: gpu scope for one GPU, system scope when other GPUs add
// to the counters over NVLink.
__device__ __forceinline__ uint32_t ld_relaxed(const int* p, bool sys) {
  uint32_t v;
  if (sys)
    asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void ld_acquire(const int* p, bool sys) {
  uint32_t v;
  if (sys)
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  (void)v;
}

__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void red_relaxed_sys_add(int* p, int v) {
  asm volatile("red.relaxed.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ T* at_rank(T* local, const PeerInfo& pi, int p) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(local) + pi.delta[p]);
}

// A barrier of the consumer warps with a bounded wait (two mbarriers used in
// turn), so a warp that gave up can never leave the others waiting forever.
// Thread 0 may reach it only after its own bounded wait for a dependency
// (another GPU's count), so the barrier waits three times as long: that wait
// runs out first and records its own status bit.
__device__ __forceinline__ bool consumers_sync(uint64_t* bars, uint32_t& uses, uint32_t* status) {
  uint64_t* b = &bars[uses & 1];
  const uint32_t parity = (uses >> 1) & 1u;
  uses++;
  mbar_arrive(b);
  return gemv::warp_wait_sleep(b, parity, status, 3);
}

// Shared memory from a 1024-byte aligned base: the stages; `stages` full and
// `stages` empty barriers, two consumer and two epilogue barriers; the
// activations; the epilogue's 2 x 32 outputs.
struct Plan {
  int64_t bar_off, xw_off, xs_off, yt_off, total;
};
__host__ __device__ inline Plan chain_plan(int stages, int64_t max_blocks, bool q4) {
  Plan p;
  p.bar_off = (int64_t)stages * kStageBytes;
  p.xw_off = gemv::round_up(p.bar_off + 8 * (2 * stages + 4), 128);
  p.xs_off = p.xw_off + max_blocks * (q4 ? 64 : 32);
  p.yt_off = p.xs_off + gemv::round_up(max_blocks * 4, 16);
  p.total = p.yt_off + 2 * kRows * 4 + 1024;
  return p;
}

template <bool Q4>
__global__ void __launch_bounds__(kThreads, 3)
    chain_kernel(const ChainOpDev* __restrict__ ops, const int nops, int* counters,
                 uint32_t* status, const int stages, const int64_t max_blocks, const int l2_ahead,
                 const PeerInfo pi) {
  using F = Fmt<Q4>;
  using X = quad::XQ<Q4>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const Plan pl = chain_plan(stages, max_blocks, Q4);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pl.bar_off);
  uint64_t* empty = full + stages;
  uint64_t* csync = empty + stages;
  uint64_t* epi = csync + 2;
  uint8_t* xw = smem + pl.xw_off;
  float* xs = reinterpret_cast<float*>(smem + pl.xs_off);
  float* yt_s = reinterpret_cast<float*>(smem + pl.yt_off);
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, bid = blockIdx.x;
  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&csync[i], kConsumers);
      mbar_init(&epi[i], kConsumers);
    }
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
      // The L2 prefetch cursor: chunk (pop, pt, pc) of this CTA's sequence,
      // kept up to l2_ahead chunks past the end of the ring.
      int pop = 0, pt = first_tile(ops[0]), pc = 0;
      int64_t kp = 0;
      for (int op = 0; op < nops && !abort_flag; op++) {
        const ChainOpDev& o = ops[op];
        const int64_t blocks = o.cols / kBlock;
        const int nch = (int)((blocks + F::kKC - 1) / F::kKC);
        prefetch_tmap(&o.tw);
        for (int t = first_tile(o); t < o.ntiles && !abort_flag; t += G) {
          for (int c = 0; c < nch; c++) {
            while (kp < k + stages + l2_ahead && pop < nops) {
              const ChainOpDev& q = ops[pop];
              if (pt >= q.ntiles) {
                if (++pop < nops) pt = first_tile(ops[pop]);
                pc = 0;
                continue;
              }
              const int64_t qb = q.cols / kBlock;
              const int qnch = (int)((qb + F::kKC - 1) / F::kKC);
              if (kp >= k + stages) {  // chunks inside the ring are loaded anyway
                const int nb = (int)min64(F::kKC, qb - (int64_t)pc * F::kKC);
                const int boxes = (nb * F::kWB + kBoxBytes - 1) / kBoxBytes;
                for (int j = 0; j < boxes; j++)
                  tma_prefetch_l2_2d(&q.tw, pc * kChunkBytes + j * kBoxBytes, pt * kRows);
                if (q.tma_scales) tma_prefetch_l2_2d(&q.tsc, pc * F::kKC, pt * kRows);
              }
              kp++;
              if (++pc == qnch) {
                pc = 0;
                pt += G;
              }
            }
            // The consumers free a stage only after their own bounded waits
            // (a dependency, then a barrier at three times the limit), so
            // this one runs five times the limit.
            if (k >= stages &&
                !mbar_wait_bounded_sleep(&empty[s], ph ^ 1u, status, kStatusTmaTimeout, 5)) {
              abort_flag = 1;
              break;
            }
            const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
            uint8_t* stage = smem + (int64_t)s * kStageBytes;
            if (o.tma_scales)
              gemv::issue_stage<Q4, true>(stage, &o.tw, &o.tsc, c, nb, t * kRows, &full[s]);
            else
              gemv::issue_stage<Q4, false>(stage, &o.tw, &o.tsc, c, nb, t * kRows, &full[s]);
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
  const quad::Lane lc = quad::lane_ctx(warp, lane);
  const uint8_t* xw_l = xw + lc.l * X::kLane;
  const bool sys = pi.world > 1;
  // The run index (thread 0 waits and signals for the CTA): the previous
  // kernel in the stream, hence the previous run, is complete after
  // griddepcontrol.wait.
  uint32_t run = 0;
  if (tid == 0) {
    pdl_wait();
    run = ld_relaxed(counters + nops + 1, false);
  }
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
    // Inputs written before the launch: the previous kernel in the stream
    // (PDL) must be complete. Inputs from an earlier op: its counter.
    if (o.ext_input && !waited_launch) {
      pdl_wait();
      waited_launch = true;
    }
    if (o.dep >= 0 && tid == 0) {
      // This run's tiles of op dep: the counter reaches (run + 1) x its tiles
      // (compared with wrap-around differences).
      const uint32_t target = (run + 1u) * (uint32_t)ops[o.dep].ntiles_total;
      const int* cnt = counters + o.dep;
      // Spin on relaxed loads (an acquire per poll costs this SM an L1
      // invalidation each time, which measurably slows the warps computing
      // beside it), then one acquire load.
      if ((int32_t)(ld_relaxed(cnt, sys) - target) < 0) {
        const uint64_t start = globaltimer_ns();
        for (uint32_t it = 1;; it++) {
          __nanosleep(32);
          if ((int32_t)(ld_relaxed(cnt, sys) - target) >= 0) break;
          if ((it & 63u) == 0 && globaltimer_ns() - start > wait_limit_ns()) {
            report(status, kStatusPeerTimeout);
            abort_flag = 1;
            break;
          }
        }
      }
      ld_acquire(cnt, sys);
    }
    if (!consumers_sync(csync, syncs, status) || abort_flag) {
      abort_flag = 1;
      return;
    }
    quad::load_unpack<Q4>(o.xa, blocks, xw, xs, tid, kConsumers);
    if (!consumers_sync(csync, syncs, status)) {
      abort_flag = 1;
      return;
    }
    for (int t = t_first; t < o.ntiles; t += G) {
      const int64_t row = (int64_t)t * kRows + lc.r;  // row of this rank's slice
      const int64_t grow = (int64_t)o.tile0 * kRows + row;  // row of the whole output
      const int64_t srow = row < o.rows ? row : o.rows - 1;
      const uint8_t* gsc = o.tma_scales ? nullptr
                                        : static_cast<const uint8_t*>(o.scales) + srow * blocks * F::kSB;
      const uint8_t* xwp = xw_l;
      const float* xsp = xs;
      float acc = 0.0f;
      // Whole stages with scales in the stage, then the rest (a partial last
      // stage, or every stage when the scales are read from global memory).
      const int nfull = o.tma_scales ? (int)(blocks / F::kKC) : 0;
      int ch = 0;
      for (; ch < nfull; ch++) {
        if (!gemv::warp_wait(&full[s], ph, status)) {
          abort_flag = 1;
          return;  // the producer drains what it issued; every other wait is bounded
        }
        quad::stage_full<Q4>(smem + (int64_t)s * kStageBytes, lc, xwp, xsp, acc);
        xwp += F::kKC * X::kBlock;
        xsp += F::kKC;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      for (; ch < nch; ch++) {
        if (!gemv::warp_wait(&full[s], ph, status)) {
          abort_flag = 1;
          return;
        }
        const int nb = (int)min64(F::kKC, blocks - (int64_t)ch * F::kKC);
        const uint8_t* stage = smem + (int64_t)s * kStageBytes;
        if (o.tma_scales)
          quad::stage_part<Q4, true>(stage, nb, lc, xwp, xsp, gsc, acc);
        else
          quad::stage_part<Q4, false>(stage, nb, lc, xwp, xsp, gsc + (int64_t)ch * F::kKC * F::kSB, acc);
        xwp += F::kKC * X::kBlock;
        xsp += F::kKC;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      const float y = gemv::lane_reduce(acc);  // valid on l == 0
      float* yt = yt_s + (e & 1) * kRows;
      if (lc.l == 0 && row < o.rows) {
        if (o.ys != nullptr) o.ys[grow] = y;
        yt[lc.r] = y;
      }
      // Every warp's outputs, then (QA outputs: warp 0 quantizes the tile's
      // block) one release per tile.
      mbar_arrive(&epi[e & 1]);
      if (!gemv::warp_wait(&epi[e & 1], (e >> 1) & 1u, status)) {
        abort_flag = 1;
        return;
      }
      if (warp == 0) {
        // QA outputs need whole tiles (rows % 32 == 0, checked at creation).
        uint8_t* blk = o.ya + ((int64_t)o.tile0 + t) * kQABytes;
        if (o.ya != nullptr) gemv::quantize_block_out(yt[lane], blk, lane);
        __syncwarp();
        if (!sys) {
          if (lane == 0) red_release_add(counters + op, 1);
        } else {
          // The block, word by word, into every other rank's region.
          if (o.ya != nullptr) {
            for (int i = lane; i < 9 * pi.world; i += 32) {
              const int p = i / 9, w = i % 9;
              if (p != pi.rank)
                at_rank(reinterpret_cast<uint32_t*>(blk), pi, p)[w] = reinterpret_cast<const uint32_t*>(blk)[w];
            }
          }
          __syncwarp();
          if (lane == 0) {
            fence_acq_rel_sys();  // the block is visible everywhere before any count
            for (int p = 0; p < pi.world; p++) red_relaxed_sys_add(at_rank(counters + op, pi, p), 1);
          }
        }
      }
      e++;
    }
  }
  // The last CTA out advances the run index for the next launch. (Thread 0
  // is here only after its last tile's epilogue barrier, so every consumer of
  // the CTA is past its dependency waits; when every CTA's thread 0 is here,
  // every wait of the launch is behind it.)
  if (tid == 0 && !abort_flag) {
    __threadfence();
    if (atomicAdd(counters + nops, 1) == G - 1) {
      counters[nops] = 0;
      counters[nops + 1] = (int)(run + 1u);
      __threadfence();
    }
  }
}

// Chunks each producer pulls into L2 beyond its stage ring. DN_CHAIN_L2_AHEAD
// overrides (0: none).
static int chain_l2_ahead() {
  static int v = [] {
    const char* e = getenv("DN_CHAIN_L2_AHEAD");
    const int n = e != nullptr ? atoi(e) : -1;
    return n >= 0 && n <= 1024 ? n : 0;
  }();
  return v;
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

static bool chain_buffers_disjoint(const ChainOpSpec* specs, const int64_t* total_rows,
                                   int64_t nops, bool q4) {
  auto span = [](const void* p, int64_t bytes) {
    const uintptr_t a = (uintptr_t)p;
    return Range{a, p == nullptr ? a : a + (uintptr_t)bytes};
  };
  std::vector<Range> outs, ins, consts;  // per op: ys, ya; xa; qs, scales
  for (int64_t i = 0; i < nops; i++) {
    const ChainOpSpec& s = specs[i];
    const int64_t blocks = s.cols / kBlock;
    outs.push_back(span(s.ys, total_rows[i] * 4));
    outs.push_back(span(s.ya, total_rows[i] / kRows * kQABytes));
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

static int64_t create(const ChainOpSpec* specs, const int64_t* row0, const int64_t* total_rows,
                      int64_t nops, bool q4, const ChainShard* shard, ChainHost** out) {
  if (nops <= 0 || specs == nullptr || out == nullptr) return kErrArgs;
  PeerInfo pi{1, 0, {0}};
  const uint8_t *region_lo = nullptr, *region_hi = nullptr;
  if (shard != nullptr) {
    if (shard->world < 1 || shard->world > kMaxWorld || shard->rank < 0 ||
        shard->rank >= shard->world || shard->bases == nullptr || shard->region_bytes <= 0 ||
        shard->counters == nullptr || ((uintptr_t)shard->counters & 3) != 0)
      return kErrArgs;
    pi.world = (int32_t)shard->world;
    pi.rank = (int32_t)shard->rank;
    for (int p = 0; p < pi.world; p++) {
      if (shard->bases[p] == nullptr) return kErrArgs;
      pi.delta[p] = (const char*)shard->bases[p] - (const char*)shard->bases[pi.rank];
    }
    region_lo = static_cast<const uint8_t*>(shard->bases[pi.rank]);
    region_hi = region_lo + shard->region_bytes;
    const uint8_t* c = reinterpret_cast<const uint8_t*>(shard->counters);
    if (c < region_lo || c + 4 * (nops + 2) > region_hi) return kErrArgs;
  }
  std::vector<ChainOpDev> table((size_t)nops);
  int64_t tile_base = 0, max_blocks = 0;
  for (int64_t i = 0; i < nops; i++) {
    const ChainOpSpec& sp = specs[i];
    const int64_t r0 = row0[i], total = total_rows[i];
    ChainOpDev& d = table[(size_t)i];
    memset(&d, 0, sizeof d);
    const int64_t blocks = sp.cols / kBlock;
    if (sp.rows <= 0 || sp.cols <= 0 || sp.cols % kBlock != 0 || sp.xa == nullptr ||
        ((uintptr_t)sp.qs & 15) != 0 || ((uintptr_t)sp.xa & 3) != 0 ||
        (sp.ya != nullptr && ((uintptr_t)sp.ya & 3) != 0) || sp.dep >= i || sp.dep < -1 ||
        total > INT32_MAX / 2 || sp.cols > INT32_MAX / 2 || r0 < 0 || r0 % kRows != 0 ||
        r0 + sp.rows > total)
      return kErrArgs;
    // QA outputs: whole blocks (this rank's rows and the whole output).
    if (sp.ya != nullptr && (sp.rows % kRows != 0 || total % kRows != 0)) return kErrArgs;
    // Other ranks write QA outputs into the region, so they must be inside it.
    if (shard != nullptr && sp.ya != nullptr &&
        (sp.ya < region_lo || sp.ya + total / kRows * kQABytes > region_hi))
      return kErrArgs;
    d.ext_input = 1;
    if (sp.dep >= 0 && specs[sp.dep].ya != nullptr) {
      // A data edge: the input lies inside the QA output of op dep, on a
      // block boundary. An input that does not touch that output was written
      // before the launch (an ordering edge).
      const ChainOpSpec& p = specs[sp.dep];
      const uint8_t *lo = p.ya, *hi = p.ya + total_rows[sp.dep] / kRows * kQABytes;
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
        !encode_tmap_2d_sw64(&d.tsc, sp.scales,
                             q4 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                             (uint64_t)blocks, (uint64_t)sp.rows, (uint64_t)(blocks * sb),
                             (uint32_t)(kChunkBytes / wb), kRows))
      return kErrUnsupported;
    d.scales = sp.scales;
    d.xa = sp.xa;
    d.ys = sp.ys;
    d.ya = sp.ya;
    d.rows = (int32_t)sp.rows;
    d.cols = (int32_t)sp.cols;
    d.dep = (int32_t)sp.dep;
    d.ntiles = (int32_t)((sp.rows + kRows - 1) / kRows);
    d.tile0 = (int32_t)(r0 / kRows);
    d.ntiles_total = (int32_t)((total + kRows - 1) / kRows);
    d.tile_base = (int32_t)(tile_base % (1 << 30));
    tile_base += d.ntiles;
    max_blocks = blocks > max_blocks ? blocks : max_blocks;
  }
  if (!chain_buffers_disjoint(specs, total_rows, nops, q4)) return kErrArgs;
  ChainHost* h = new ChainHost();
  h->nops = (int)nops;
  h->q4 = q4;
  h->max_blocks = max_blocks;
  h->peers = pi;
  cudaGetDevice(&h->device);
  if (shard != nullptr) {
    h->counters = shard->counters;
    h->owns_counters = false;
  } else if (cudaMalloc(&h->counters, sizeof(int) * (size_t)(nops + 2)) != cudaSuccess ||
             cudaMemset(h->counters, 0, sizeof(int) * (size_t)(nops + 2)) != cudaSuccess) {
    chain_destroy(h);
    return kErrCuda;
  }
  if (cudaMalloc(&h->ops_dev, sizeof(ChainOpDev) * (size_t)nops) != cudaSuccess ||
      cudaMemcpy(h->ops_dev, table.data(), sizeof(ChainOpDev) * (size_t)nops,
                 cudaMemcpyHostToDevice) != cudaSuccess) {
    chain_destroy(h);
    return kErrCuda;
  }
  *out = h;
  return kOk;
}

int64_t chain_create(const ChainOpSpec* specs, int64_t nops, bool q4, ChainHost** out) {
  if (nops <= 0 || specs == nullptr) return kErrArgs;
  std::vector<int64_t> row0((size_t)nops, 0), total((size_t)nops);
  for (int64_t i = 0; i < nops; i++) total[(size_t)i] = specs[i].rows;
  return create(specs, row0.data(), total.data(), nops, q4, nullptr, out);
}

int64_t chain_create_sharded(const ChainOpSpec* specs, const int64_t* row0,
                             const int64_t* total_rows, int64_t nops, bool q4,
                             const ChainShard& shard, ChainHost** out) {
  if (row0 == nullptr || total_rows == nullptr) return kErrArgs;
  return create(specs, row0, total_rows, nops, q4, &shard, out);
}

void chain_destroy(ChainHost* h) {
  if (h == nullptr) return;
  if (h->ops_dev != nullptr) cudaFree(h->ops_dev);
  if (h->counters != nullptr && h->owns_counters) cudaFree(h->counters);
  delete h;
}

// CTAs per SM: more CTAs spread an op's tiles over more SMs' worth of
// warps, fewer give each a deeper stage ring. DN_CHAIN_PER_SM overrides.
static int chain_per_sm() {
  static int v = [] {
    const char* e = getenv("DN_CHAIN_PER_SM");
    const int n = e != nullptr ? atoi(e) : 0;
    return n >= 1 && n <= 16 ? n : 2;
  }();
  return v;
}

template <bool Q4>
static int64_t chain_launch_t(ChainHost* h, uint32_t* status, cudaStream_t stream, bool pdl) {
  const Plan base = chain_plan(0, h->max_blocks, Q4);
  int per_sm = chain_per_sm(), stages = 0;
  for (; per_sm >= 1; per_sm--) {
    // 1 KB per CTA is reserved by the system; the static abort flag is small.
    stages = (int)((kSmemPerSM / per_sm - 1024 - 64 - base.total) / (kStageBytes + 16));
    if (stages >= 2) break;
  }
  stages = stages > kMaxStages ? kMaxStages : stages;
  if (per_sm < 1 || stages < 2) return kErrTooLarge;
  const Plan sp = chain_plan(stages, h->max_blocks, Q4);
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
  return cudaLaunchKernelEx(&cfg, kern, ops, h->nops, h->counters, status, stages, h->max_blocks,
                            chain_l2_ahead(), h->peers) ==
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
  return cudaMemsetAsync(h->counters, 0, sizeof(int) * (size_t)(h->nops + 2), stream) == cudaSuccess
             ? kOk
             : kErrCuda;
}

}  // namespace dn
