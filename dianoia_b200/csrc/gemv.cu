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
// Memory path: a persistent, warp-specialized kernel. Each CTA owns a set of
// 32-row tiles (one Q8_0 block of the output each). A producer warp streams
// the weights of all its tiles, chunk by chunk (512 bytes of each row plus
// its scales), through a shared-memory ring with 2-D TMA tensor copies of
// 32 rows x 128 bytes (4 KB boxes, 128-byte swizzle) that complete on a
// "full" mbarrier per stage; four consumer warps compute and release each
// stage on an "empty" mbarrier, so the next tile's weights are in flight
// while the current one is computed. Few, large copies keep enough bytes in
// flight per SM (many 512-byte copies capped the stream near 2 TB/s), and
// the swizzle puts the eight rows a warp reads at once in eight different
// bank groups. The activations are loaded once
// per CTA: f32 inputs are bulk-copied and quantized in the CTA (which fuses
// lab_gemm's input quantize; CTA 0 also writes xq / xsc out), QA inputs are
// bulk-copied as they are. Each tile's 32 outputs per token can be quantized
// again in the epilogue (QA output) for the next product of a chain, and the
// feed-forward's SwiGLU can run there too, on the outputs of the gate / up
// pair's second product and the first one's (glu_* arguments), and so can the
// residual add that follows a layer's output projections (res). With f32
// inputs, the CTA can also run the RMSNorm that produces them (norm_*).
#include <string.h>

#include <algorithm>

#include "dn_common.cuh"
#include "dn_launch.h"
#include "dn_tmap.h"
#include "gemv_core.cuh"
#include "quaddot.cuh"

namespace dn {
namespace {

using namespace gemv;

// Two CTAs per SM, stated so ptxas keeps the unrolled stage in registers
// (without a minimum it capped the kernel at 56 registers).
//
// DUAL (one token only): two matrices of the same shape, the feed-forward's
// gate (qs, scales; tensor maps tw, tsc) and up (qs2, scales2; tw2, tsc2), in
// one launch. A tile streams its 32 gate rows and then the same 32 up rows,
// so the epilogue has g and u of each row in registers and writes
// h = silu(g) * u to ys (and its QA blocks), u to ys2.
// The body of both kernels below (their tensor maps are __grid_constant__
// parameters, passed here by address).
// Tensor maps of a grouped launch, one weight and one scale map per product.
struct GroupMaps {
  CUtensorMap w[kMaxGroups];
  CUtensorMap sc[kMaxGroups];
};

// The product of a grouped launch that tile `tile` belongs to.
__device__ __forceinline__ int group_of(const GemvArgs& a, int64_t tile) {
  int g = 0;
  while (g + 1 < a.groups && tile >= a.group_tile0[g + 1]) g++;
  return g;
}

template <bool Q4, int NT, bool TMA_SCALES, bool F32_IN, bool DUAL, bool EPI, bool GROUP = false>
__device__ __forceinline__ void gemv_body(const GemvArgs& a, const int stages, const CUtensorMap* tw,
                                          const CUtensorMap* tsc, const CUtensorMap* tw2,
                                          const CUtensorMap* tsc2, const GroupMaps* gm = nullptr) {
  static_assert(!GROUP || (NT == 1 && !DUAL && !EPI), "a grouped launch is of plain one-token products");
  static_assert(!DUAL || NT == 1, "the dual product is for one token");
  using F = Fmt<Q4>;
  using X = XLayout<Q4>;
  constexpr int kPerBox = kBoxBytes / F::kWB;  // blocks per weight box: 4 (Q8) or 8 (Q4)
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t blocks = a.cols / kBlock;
  const int64_t ntiles = GROUP ? a.group_tile0[a.groups] : (a.rows + kRows - 1) / kRows;
  const int64_t t0 = (int64_t)blockIdx.y * NT;
  const int nt = (int)min64(NT, a.n - t0);
  const int nch = (int)((blocks + F::kKC - 1) / F::kKC);
  // This CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int64_t my_tiles = (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const int tchunks = DUAL ? 2 * nch : nch;  // stages per tile
  const int64_t total = my_tiles * tchunks;
  const bool norm = F32_IN && a.norm_w != nullptr;
  const SmemPlan sp = plan<Q4>(stages, NT, a.cols, F32_IN, norm);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sp.bar_off);
  uint64_t* empty = full + stages;
  uint64_t* xbars = empty + stages;  // token buffers 0 and 1, the norm's weights
  uint64_t* epi = xbars + 3;
  uint8_t* xw_s = smem + sp.xw_off;
  float* xs_s = reinterpret_cast<float*>(smem + sp.xs_off);
  float* yt_s = reinterpret_cast<float*>(smem + sp.yt_off);
  uint8_t* stg_s = smem + sp.stg_off;
  __shared__ volatile int abort_flag;

  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(&xbars[0], 1);
    mbar_init(&xbars[1], 1);
    mbar_init(&xbars[2], 1);
    mbar_init(&epi[0], kConsumers);
    mbar_init(&epi[1], kConsumers);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    // The weights do not depend on the previous kernel, so no PDL wait here.
    if (lane == 0) {
      prefetch_tmap(tw);
      if (TMA_SCALES) prefetch_tmap(tsc);
      if (DUAL) prefetch_tmap(tw2);
      if (DUAL && TMA_SCALES) prefetch_tmap(tsc2);
    }
    // Ring slot, its phase, chunk and tile are running counters: a 64-bit
    // division per stage would cost more than the stage's own work.
    int64_t k = 0, tile = blockIdx.x;
    int s = 0, c = 0;
    uint32_t eph = 1;  // parity of empty[s] to wait for, from the ring's second pass on
    for (; k < total; k++) {
      if (k >= stages) {
        const bool got = mbar_wait_bounded(&empty[s], eph, a.status, kStatusTmaTimeout);
        if (!got) abort_flag = 1;
      }
      if (abort_flag) break;
      if (lane == 0) {
        const bool second = DUAL && c >= nch;  // the up matrix's half of the tile
        const int cc = second ? c - nch : c;
        const int nb = (int)min64(F::kKC, blocks - (int64_t)cc * F::kKC);
        if constexpr (GROUP) {
          const int g = group_of(a, tile);
          issue_stage<Q4, TMA_SCALES>(smem + (int64_t)s * kStageBytes, &gm->w[g], &gm->sc[g], cc, nb,
                                      (int32_t)((tile - a.group_tile0[g]) * kRows), &full[s]);
        } else {
          issue_stage<Q4, TMA_SCALES>(smem + (int64_t)s * kStageBytes, second ? tw2 : tw,
                                      second ? tsc2 : tsc, cc, nb, (int32_t)(tile * kRows), &full[s]);
        }
      }
      __syncwarp();
      if (++s == stages) {
        s = 0;
        eph ^= 1u;
      }
      if (++c == tchunks) {
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
  const int r8 = lane >> 2, l = lane & 3;
  // A chained product (QA input) lets the next one start its weight stream
  // right away; a single product from f32 inputs triggers after its
  // prologue (back to back, an early start measured slower there).
  if (!F32_IN) pdl_launch_dependents();
  float* nw_s = reinterpret_cast<float*>(smem + sp.nw_off);
  if (norm && tid == 0) {
    // The norm's weights do not come from the previous kernel: fetch them
    // while it finishes.
    mbar_arrive_expect_tx(&xbars[2], (uint32_t)(a.cols * 4));
    bulk_g2s(nw_s, a.norm_w, (uint32_t)(a.cols * 4), &xbars[2]);
  }
  pdl_wait();  // the activations may come from the previous kernel
  bool ok = true;
  if (F32_IN) {
    // Token by token through two f32 buffers: the bulk copy of token t+2
    // runs while token t+1 is quantized.
    const uint32_t xbytes = (uint32_t)(a.cols * 4);
    auto issue_x = [&](int tt) {
      mbar_arrive_expect_tx(&xbars[tt & 1], xbytes);
      bulk_g2s(stg_s + (tt & 1) * sp.stg_stride, a.xs + (t0 + tt) * a.cols, xbytes, &xbars[tt & 1]);
    };
    if (tid == 0) {
      for (int tt = 0; tt < min(2, nt); tt++) issue_x(tt);
    }
    const bool writer = blockIdx.x == 0 && a.xq != nullptr;
    const bool qa_writer = blockIdx.x == 0 && a.xa_out != nullptr;
    float* norm_out = blockIdx.x == 0 ? a.norm_out : nullptr;
    __shared__ double norm_red[kNormLanes / 32];
    const bool wgot = !norm || warp_wait(&xbars[2], 0, a.status);
    int tt = 0;
    for (; tt < nt; tt++) {
      bool got = warp_wait(&xbars[tt & 1], (uint32_t)(tt >> 1) & 1u, a.status);
      float* xf = reinterpret_cast<float*>(stg_s + (tt & 1) * sp.stg_stride);
      // The norm's barriers need every consumer warp: all of them go ahead,
      // or none (a warp whose wait ran out makes every warp skip the token).
      if (norm) got = consumers_all(got && wgot);
      if (got && norm) {
        // The fused RMSNorm, in place in the staging buffer.
        const double r = norm_factor(xf, a.cols, a.norm_eps, tid, norm_red, [] { consumers_sync(); });
        float* out = norm_out == nullptr ? nullptr : norm_out + (t0 + tt) * a.cols;
        for (int64_t j = tid; j < a.cols; j += kConsumers) {
          const float v = norm_value(xf[j], nw_s[j], r);
          xf[j] = v;
          if (out != nullptr) out[j] = v;
        }
        // Generic writes to a buffer the bulk copy of token tt + 2 refills.
        fence_proxy_async_smem();
        consumers_sync();
      }
      if (got)
        quantize_token<Q4>(xf, xw_s + tt * sp.xw_stride, xs_s + tt * sp.xs_stride, blocks,
                           writer ? a.xq + (t0 + tt) * a.cols : nullptr,
                           writer ? a.xsc + (t0 + tt) * blocks : nullptr,
                           qa_writer ? a.xa_out + (t0 + tt) * a.xa_out_stride : nullptr);
      if (!got) abort_flag = 1;
      consumers_sync();
      if (abort_flag) {
        ok = false;
        break;
      }
      if (tid == 0 && tt + 2 < nt) issue_x(tt + 2);
    }
    if (!ok && tid == 0) {
      for (int j = tt + 1; j < min(nt, tt + 2); j++)
        mbar_wait_bounded(&xbars[j & 1], (uint32_t)(j >> 1) & 1u, a.status, kStatusTmaTimeout);
      if (norm) mbar_wait_bounded(&xbars[2], 0, a.status, kStatusTmaTimeout);
    }
  } else {
    const int64_t row_bytes = blocks * kQABytes;
    const bool bulk = (row_bytes % 16) == 0 && ((uintptr_t)a.xa & 15) == 0 && (a.xa_stride % 16) == 0;
    if (bulk) {
      if (tid == 0) {
        mbar_arrive_expect_tx(&xbars[0], (uint32_t)(nt * row_bytes));
        for (int tt = 0; tt < nt; tt++)
          bulk_g2s(stg_s + tt * sp.stg_stride, a.xa + (t0 + tt) * a.xa_stride, (uint32_t)row_bytes,
                   &xbars[0]);
      }
      if (!warp_wait(&xbars[0], 0, a.status)) abort_flag = 1;
    } else {
      for (int tt = 0; tt < nt; tt++) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(a.xa + (t0 + tt) * a.xa_stride);
        uint32_t* dst = reinterpret_cast<uint32_t*>(stg_s + tt * sp.stg_stride);
        for (int64_t i = tid; i < row_bytes / 4; i += kConsumers) dst[i] = __ldg(src + i);
      }
    }
    consumers_sync();
    if (!abort_flag) {
      for (int tt = 0; tt < nt; tt++)
        unpack_qa<Q4>(stg_s + tt * sp.stg_stride, xw_s + tt * sp.xw_stride,
                      xs_s + tt * sp.xs_stride, blocks);
    }
    consumers_sync();
    ok = !abort_flag;
  }
  if (F32_IN) pdl_launch_dependents();
  if (!ok) return;

  const int row_local = warp * 8 + r8;
  const uint32_t rowoff = (uint32_t)row_local * kBoxBytes;
  const uint8_t* sc = static_cast<const uint8_t*>(a.scales);
  const uint8_t* xw_l = xw_s + l * X::kLaneBytes;
  int s = 0;        // ring slot of the next stage
  uint32_t ph = 0;  // and the parity of its full barrier
  uint32_t e = 0;   // epilogue barrier uses so far
  for (int64_t i = 0; i < my_tiles; i++) {
    const int64_t tile = blockIdx.x + i * gridDim.x;
    // A grouped launch: the tile's product and its tile within that product.
    const int gidx = GROUP ? group_of(a, tile) : 0;
    const int64_t ltile = GROUP ? tile - a.group_tile0[gidx] : tile;
    const int64_t rows_g = GROUP ? a.group_rows[gidx] : a.rows;
    const int64_t row0 = ltile * kRows;
    const int tile_rows = (int)min64(kRows, rows_g - row0);
    const int64_t row = row0 + min(row_local, tile_rows - 1);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t] = 0.0f;
    float acc_up = 0.0f;  // DUAL: the up matrix's accumulator

    if constexpr (NT == 1) {
      // One token: the quad-lane core (quaddot.cuh), whole stages and the
      // rest in separate loops (a per-stage branch between them made the
      // compiler issue the shared-memory loads late). DUAL runs them for
      // the gate rows and then for the up rows.
      const quad::Lane qc = quad::lane_ctx(warp, lane);
      // One matrix's rows of the tile (scales scb) into acc_h; false when a
      // wait ran out (the producer drains what it issued; every other wait
      // is bounded). Called once, or for the gate and then the up rows.
      auto run = [&](const uint8_t* scb, float& acc_h) -> bool {
        const uint8_t* xwp = xw_l;
        const float* xsp = xs_s;
        const uint8_t* gsc = TMA_SCALES ? nullptr : scb + row * blocks * F::kSB;
        const int nfull = TMA_SCALES ? (int)(blocks / F::kKC) : 0;
        int c = 0;
        for (; c < nfull; c++) {
          if (!warp_wait(&full[s], ph, a.status)) return false;
          quad::stage_full<Q4>(smem + (int64_t)s * kStageBytes, qc, xwp, xsp, acc_h);
          xwp += F::kKC * X::kBlockBytes;
          xsp += F::kKC;
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        for (; c < nch; c++) {
          const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
          if (!warp_wait(&full[s], ph, a.status)) return false;
          quad::stage_part<Q4, TMA_SCALES>(smem + (int64_t)s * kStageBytes, nb, qc, xwp, xsp,
                                           gsc == nullptr ? nullptr : gsc + (int64_t)c * F::kKC * F::kSB,
                                           acc_h);
          xwp += F::kKC * X::kBlockBytes;
          xsp += F::kKC;
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        return true;
      };
      bool ran = run(GROUP ? static_cast<const uint8_t*>(a.group_scales[gidx]) : sc, acc[0]);
      if constexpr (DUAL) ran = ran && run(static_cast<const uint8_t*>(a.scales2), acc_up);
      if (!ran) {
        abort_flag = 1;
        return;
      }
    } else {
      const LaneCtx lc{row_local, r8, l, rowoff, xw_l, sp.xw_stride, xs_s, sp.xs_stride, sc, row, blocks};
      for (int c = 0; c < nch; c++) {
        const int nb = (int)min64(F::kKC, blocks - (int64_t)c * F::kKC);
        if (!warp_wait(&full[s], ph, a.status)) {
          abort_flag = 1;
          return;  // the producer drains what it issued; every other wait is bounded
        }
        gemv_stage<Q4, NT, TMA_SCALES>(smem + (int64_t)s * kStageBytes, nb, c * F::kKC, lc, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }

    float* yt = yt_s + (e & 1) * NT * kRows;
    const float up = DUAL ? lane_reduce(acc_up) : 0.0f;
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const float y = lane_reduce(acc[t]);
      if (GROUP && l == 0 && row_local < tile_rows && t < nt) {
        float* ys = a.group_ys[gidx];
        if (ys != nullptr) ys[(t0 + t) * rows_g + row0 + row_local] = y;
      } else if (!GROUP && l == 0 && row_local < tile_rows && t < nt) {
        const int64_t at = (t0 + t) * a.ldy + row0 + row_local;
        float v = y;
        if (DUAL) {
          v = silu_mul(y, up);
          if (a.ys2 != nullptr) a.ys2[at] = up;
          if (a.ys != nullptr) a.ys[at] = v;
        } else if (EPI && a.glu_out != nullptr) {
          // The feed-forward's other half was written by the previous kernel,
          // which completed before this one's dependent-launch wait.
          const float other = a.glu_other[at];
          v = a.glu_self_gate ? silu_mul(y, other) : silu_mul(other, y);
          if (!a.glu_self_gate && a.ys != nullptr) a.ys[at] = y;
          a.glu_out[at] = v;
        } else if (a.ys != nullptr) {
          a.ys[at] = y;
        }
        if (EPI && a.res != nullptr) a.res[at] = __fadd_rn(a.res[at], y);
        yt[t * kRows + row_local] = v;
      }
    }
    if (!GROUP && a.ya != nullptr && tile_rows == kRows) {
      // The tile's 32 outputs of a token are one Q8_0 block of the next
      // projection's input: quantize them here (lab_quantize_q8 semantics).
      // All consumers meet on a bounded epilogue barrier; its buffer
      // alternates, and no warp can get two tiles ahead of another.
      mbar_arrive(&epi[e & 1]);
      if (!warp_wait(&epi[e & 1], (e >> 1) & 1u, a.status)) {
        abort_flag = 1;
        return;
      }
      for (int t = warp; t < nt; t += kConsumerWarps)
        quantize_block_out(yt[t * kRows + lane], a.ya + (t0 + t) * a.ya_stride + tile * kQABytes, lane);
      e++;
    }
  }
}

// The kernels: the dual product carries the second matrix's tensor maps.
// EPI: the SwiGLU and residual-add epilogue (glu_* and res arguments) is
// compiled in; without it the plain products keep their own code (its
// branches alone made the plain kernels 2 % slower).
template <bool Q4, int NT, bool TMA_SCALES, bool F32_IN, bool EPI>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_i8_kernel(const GemvArgs a, const int stages, const __grid_constant__ CUtensorMap tw,
                   const __grid_constant__ CUtensorMap tsc) {
  gemv_body<Q4, NT, TMA_SCALES, F32_IN, false, EPI>(a, stages, &tw, &tsc, &tw, &tsc);
}

// Up to kMaxGroups products of one input, one token, in one launch.
template <bool Q4, bool TMA_SCALES, bool F32_IN>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_group_kernel(const GemvArgs a, const int stages, const __grid_constant__ GroupMaps maps) {
  gemv_body<Q4, 1, TMA_SCALES, F32_IN, false, false, true>(a, stages, &maps.w[0], &maps.sc[0], &maps.w[0],
                                                          &maps.sc[0], &maps);
}

template <bool Q4, bool TMA_SCALES, bool F32_IN>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_dual_kernel(const GemvArgs a, const int stages, const __grid_constant__ CUtensorMap tw,
                     const __grid_constant__ CUtensorMap tsc, const __grid_constant__ CUtensorMap tw2,
                     const __grid_constant__ CUtensorMap tsc2) {
  gemv_body<Q4, 1, TMA_SCALES, F32_IN, true, false>(a, stages, &tw, &tsc, &tw2, &tsc2);
}

// ------------------------------------------------------------------ generic
//
// Any alignment, any cols (the reference ignores a trailing partial block),
// both modes. Same lane-per-chain mapping; weights come straight from global
// memory a byte at a time, so it is slow, but exact. Mode 1 reads the
// activations already quantized into xq / xsc.

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

template <bool Q4, int NT, bool TMA_SCALES, bool F32_IN, bool DUAL, bool EPI, bool GROUP = false>
int64_t launch_gemv_t(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  using F = Fmt<Q4>;
  const int64_t ntiles = GROUP ? a.group_tile0[a.groups] : (a.rows + kRows - 1) / kRows;
  const int64_t blocks = a.cols / kBlock;
  // Two CTAs per SM when the ring still gets at least 3 stages that way, and
  // the tiles need more than one CTA per SM; with few tiles (a tall-K matrix
  // such as the MLP down projection) each CTA gets a whole SM's shared memory,
  // so more of its long stream is in flight.
  const bool norm = F32_IN && a.norm_w != nullptr;
  const SmemPlan base = plan<Q4>(0, NT, a.cols, F32_IN, norm);
  int per_sm = ntiles <= kSMs ? 1 : 2;
  int stages = (int)((kSmemPerSM / per_sm - 1024 - base.total) / (kStageBytes + 16));
  if (per_sm == 1) stages = (int)((kMaxSmem - base.total) / (kStageBytes + 16));
  if (stages < 3) {
    per_sm = 1;
    stages = (int)((kMaxSmem - base.total) / (kStageBytes + 16));
  }
  stages = stages > kMaxStages ? kMaxStages : stages;
  if (stages < 2) return kErrTooLarge;
  // Persistent grid of every CTA slot when the tiles need more than one
  // wave: CTA b takes tiles b, b + grid, ..., and CTAs b and b + kSMs share
  // an SM, so no SM holds more than ceil(ntiles / kSMs) + 1 tiles. (Sizing the
  // grid for equal tiles per CTA instead - 192 CTAs of 2 for 384 tiles - left
  // 44 SMs with 4 tiles and the rest with 2.)
  const int64_t slots = (int64_t)kSMs * per_sm;
  const int64_t waves = (ntiles + slots - 1) / slots;
  const int64_t grid = ntiles > slots ? slots : ntiles;
  // No more stages than the stages a CTA will ever load: the shared memory
  // left over lets the next kernel's CTAs become resident early (programmatic
  // dependent launch) and start streaming their weights during this kernel.
  {
    const int64_t chunks = waves * ((blocks + F::kKC - 1) / F::kKC) * (DUAL ? 2 : 1);
    if (chunks < stages) stages = (int)(chunks < 2 ? 2 : chunks);
  }
  const SmemPlan sp = plan<Q4>(stages, NT, a.cols, F32_IN, norm);
  if (sp.total > kMaxSmem) return kErrTooLarge;
  CUtensorMap tw, tsc, tw2, tsc2;
  memset(&tsc, 0, sizeof tsc);
  memset(&tw2, 0, sizeof tw2);
  memset(&tsc2, 0, sizeof tsc2);
  const uint64_t row_bytes = (uint64_t)blocks * F::kWB;
  // The one-token kernel reads its scale box with a 64-byte swizzle (quaddot.cuh).
  const CUtensorMapDataType st = Q4 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  auto maps = [&](CUtensorMap* w, CUtensorMap* sc, const void* qs, const void* scales, int64_t rows) {
    if (!encode_tmap_2d(w, qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, row_bytes, (uint64_t)rows, row_bytes,
                        kBoxBytes, kRows, true))
      return false;
    return !TMA_SCALES ||
           (NT == 1 ? encode_tmap_2d_sw64(sc, scales, st, (uint64_t)blocks, (uint64_t)rows,
                                          (uint64_t)blocks * F::kSB, F::kKC, kRows)
                    : encode_tmap_2d(sc, scales, st, (uint64_t)blocks, (uint64_t)rows,
                                     (uint64_t)blocks * F::kSB, F::kKC, kRows, false));
  };
  GroupMaps gmaps;
  memset(&gmaps, 0, sizeof gmaps);
  if constexpr (GROUP) {
    for (int g = 0; g < a.groups; g++)
      if (!maps(&gmaps.w[g], &gmaps.sc[g], a.group_qs[g], a.group_scales[g], a.group_rows[g]))
        return kErrUnsupported;
  } else if (!maps(&tw, &tsc, a.qs, a.scales, a.rows) ||
             (DUAL && !maps(&tw2, &tsc2, a.qs2, a.scales2, a.rows))) {
    return kErrUnsupported;
  }
  const void* kern = GROUP  ? reinterpret_cast<const void*>(gemv_group_kernel<Q4, TMA_SCALES, F32_IN>)
                     : DUAL ? reinterpret_cast<const void*>(gemv_dual_kernel<Q4, TMA_SCALES, F32_IN>)
                            : reinterpret_cast<const void*>(gemv_i8_kernel<Q4, NT, TMA_SCALES, F32_IN, EPI>);
  static bool configured[64] = {};  // per device: the opt-in smem limit is set
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return kErrCuda;
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, (unsigned)((a.n + NT - 1) / NT), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)sp.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // The plain kernel takes the first four of these, the dual one all six;
  // the grouped one the arguments, the stages and its maps.
  GemvArgs args = a;
  int nstages = stages;
  void* params[] = {&args, &nstages, &tw, &tsc, &tw2, &tsc2};
  if (GROUP) params[2] = &gmaps;
  return cudaLaunchKernelExC(&cfg, kern, params) == cudaSuccess ? kOk : kErrCuda;
}

template <bool Q4, int NT, bool DUAL, bool EPI>
int64_t launch_gemv_d(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  const int64_t blocks = a.cols / kBlock;
  const bool tma_scales = ((uintptr_t)a.scales & 15) == 0 && (blocks * Fmt<Q4>::kSB) % 16 == 0 &&
                          (!DUAL || ((uintptr_t)a.scales2 & 15) == 0);
  const bool f32_in = a.xs != nullptr;
  if (tma_scales)
    return f32_in ? launch_gemv_t<Q4, NT, true, true, DUAL, EPI>(a, stream, pdl)
                  : launch_gemv_t<Q4, NT, true, false, DUAL, EPI>(a, stream, pdl);
  return f32_in ? launch_gemv_t<Q4, NT, false, true, DUAL, EPI>(a, stream, pdl)
                : launch_gemv_t<Q4, NT, false, false, DUAL, EPI>(a, stream, pdl);
}

template <bool Q4, int NT>
int64_t launch_gemv_s(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  if constexpr (NT == 1) {
    if (a.groups > 1) {
      const int64_t blocks = a.cols / kBlock;
      bool tma_scales = (blocks * Fmt<Q4>::kSB) % 16 == 0;
      for (int g = 0; g < a.groups; g++) tma_scales = tma_scales && ((uintptr_t)a.group_scales[g] & 15) == 0;
      const bool f32_in = a.xs != nullptr;
      if (tma_scales)
        return f32_in ? launch_gemv_t<Q4, 1, true, true, false, false, true>(a, stream, pdl)
                      : launch_gemv_t<Q4, 1, true, false, false, false, true>(a, stream, pdl);
      return f32_in ? launch_gemv_t<Q4, 1, false, true, false, false, true>(a, stream, pdl)
                    : launch_gemv_t<Q4, 1, false, false, false, false, true>(a, stream, pdl);
    }
    if (a.qs2 != nullptr) return launch_gemv_d<Q4, 1, true, false>(a, stream, pdl);
  }
  if (a.glu_out != nullptr || a.res != nullptr) return launch_gemv_d<Q4, NT, false, true>(a, stream, pdl);
  return launch_gemv_d<Q4, NT, false, false>(a, stream, pdl);
}

// Tokens per CTA: enough for n (up to 8), fewer if shared memory runs out.
template <bool Q4>
int64_t launch_gemv_q(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  const bool f32_in = a.xs != nullptr;
  auto fits = [&](int nt) {
    return plan<Q4>(2, nt, a.cols, f32_in, a.norm_w != nullptr).total <= kMaxSmem;
  };
  if ((a.qs2 != nullptr || a.groups > 1) && a.n != 1) return kErrUnsupported;  // one token only
  if (a.n <= 1 || !fits(2)) return fits(1) ? launch_gemv_s<Q4, 1>(a, stream, pdl) : kErrTooLarge;
  if (a.n <= 2 || !fits(4)) return launch_gemv_s<Q4, 2>(a, stream, pdl);
  if (a.n <= 4 || !fits(8)) return launch_gemv_s<Q4, 4>(a, stream, pdl);
  return launch_gemv_s<Q4, 8>(a, stream, pdl);
}

}  // namespace

bool gemv_ex_supported(const GemvArgs& g) {
  if (g.cols % kBlock != 0 || g.cols <= 0 || ((uintptr_t)g.qs & 15) != 0 ||
      ((uintptr_t)g.scales & (g.q4 ? 1 : 3)) != 0)
    return false;
  if ((g.xs == nullptr) == (g.xa == nullptr)) return false;
  if (g.xs != nullptr && (((uintptr_t)g.xs & 15) != 0 || (g.xq != nullptr && ((uintptr_t)g.xq & 3) != 0)))
    return false;
  if (g.xa != nullptr && (((uintptr_t)g.xa & 3) != 0 || (g.xa_stride & 3) != 0)) return false;
  if (g.ya != nullptr && (((uintptr_t)g.ya & 3) != 0 || (g.ya_stride & 3) != 0)) return false;
  if (g.glu_out != nullptr &&
      (g.glu_other == nullptr || ((uintptr_t)g.glu_out & 3) != 0 || ((uintptr_t)g.glu_other & 3) != 0))
    return false;
  if (g.ys != nullptr && ((uintptr_t)g.ys & 3) != 0) return false;
  if (g.res != nullptr && ((uintptr_t)g.res & 3) != 0) return false;
  if (g.groups > 1) {
    if (g.groups > kMaxGroups || g.n != 1 || g.ya != nullptr || g.qs2 != nullptr || g.glu_out != nullptr ||
        g.res != nullptr || g.group_tile0[0] != 0)
      return false;
    for (int k = 0; k < g.groups; k++)
      if (g.group_rows[k] <= 0 || ((uintptr_t)g.group_qs[k] & 15) != 0 || g.group_scales[k] == nullptr ||
          ((uintptr_t)g.group_scales[k] & (g.q4 ? 1 : 3)) != 0 || ((uintptr_t)g.group_ys[k] & 3) != 0 ||
          g.group_tile0[k + 1] - g.group_tile0[k] != (g.group_rows[k] + kRows - 1) / kRows)
        return false;
  }
  if (g.qs2 != nullptr && (g.n != 1 || ((uintptr_t)g.qs2 & 15) != 0 || g.scales2 == nullptr ||
                           ((uintptr_t)g.scales2 & (g.q4 ? 1 : 3)) != 0 || ((uintptr_t)g.ys2 & 3) != 0 ||
                           g.glu_out != nullptr))
    return false;
  if (g.xa_out != nullptr && (g.xs == nullptr || ((uintptr_t)g.xa_out & 3) != 0 ||
                              (g.xa_out_stride & 3) != 0 || g.xa_out_stride < g.cols / kBlock * kQABytes))
    return false;
  // The norm's weights come in by one bulk copy.
  if (g.norm_w != nullptr && (g.xs == nullptr || ((uintptr_t)g.norm_w & 15) != 0 ||
                              ((uintptr_t)g.norm_out & 3) != 0))
    return false;
  const bool norm = g.norm_w != nullptr;
  return (g.q4 ? plan<true>(2, 1, g.cols, g.xs != nullptr, norm).total
               : plan<false>(2, 1, g.cols, g.xs != nullptr, norm).total) <= kMaxSmem;
}

int64_t launch_gemv_ex(const GemvArgs& g, cudaStream_t stream, bool pdl) {
  if (!gemv_ex_supported(g)) return kErrUnsupported;
  if (g.rows <= 0 || g.n <= 0) return kOk;
  if (g.n > 65535 * 8) return kErrTooLarge;
  if (g.gather_n > 0) {  // only the one-token kernel fuses the all-gather
    if (!gemv1_eligible(g)) return kErrUnsupported;
    return launch_gemv1(g, stream, pdl);
  }
  if (gemv1_eligible(g)) {
    const int64_t rc = launch_gemv1(g, stream, pdl);
    if (rc != kErrTooLarge && rc != kErrUnsupported) return rc;
  }
  return g.q4 ? launch_gemv_q<true>(g, stream, pdl) : launch_gemv_q<false>(g, stream, pdl);
}

static GemvArgs from_linear(const LinearArgs& a) {
  GemvArgs g{};
  g.q4 = a.q4;
  g.qs = a.qs;
  g.scales = a.scales;
  g.xs = a.xs;
  g.xq = a.xq;
  g.xsc = a.xsc;
  g.ys = a.ys;
  g.ldy = a.ldy;
  g.rows = a.rows;
  g.cols = a.cols;
  g.n = a.n;
  g.status = a.status;
  return g;
}

bool gemv_supported(const LinearArgs& a) {
  return a.mode == 1 && a.xs != nullptr && gemv_ex_supported(from_linear(a));
}

int64_t launch_gemv(const LinearArgs& a, cudaStream_t stream, bool pdl) {
  if (!gemv_supported(a)) return kErrUnsupported;
  return launch_gemv_ex(from_linear(a), stream, pdl);
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
