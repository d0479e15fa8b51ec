// Shared device helpers of the Q4_0 / Q8_0 quantized linear kernels (sm_100a).
//
// Float arithmetic here is spelled with explicit round-to-nearest intrinsics
// (__fmul_rn, __fadd_rn, __fmaf_rn, __fdiv_rn) wherever the reference rounds
// an operation on its own, so that nvcc never contracts a multiply and an add
// that dianoia's CPU kernels (built with -ffp-contract=off) keep apart.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dn {

constexpr int kBlock = 32;  // weights per Q4_0 / Q8_0 block

// Status bits a kernel leaves in the status word when a bounded wait gives up.
enum : uint32_t {
  kStatusTmaTimeout = 1u << 0,   // an mbarrier wait for a bulk copy ran out
  kStatusPeerTimeout = 1u << 1,  // a wait on another GPU's flag ran out
  kStatusMmaTimeout = 1u << 2,   // a wait for a tensor-core commit ran out
};

// How long a bounded wait spins before it records a timeout and returns: 2 s
// unless dn_set_wait_limit_ns changed it for the device.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// The limit as the kernels of this translation unit read it. Every .cu file
// has its own copy of this module variable (no relocatable device code), so
// each registers a setter that dn_set_wait_limit_ns calls for the current
// device (register_wait_limit_setter, abi.cu).
static __device__ uint64_t g_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ uint64_t wait_limit_ns() {
  return *static_cast<volatile uint64_t*>(&g_wait_limit_ns);
}

using WaitLimitSetter = bool (*)(uint64_t ns);
bool register_wait_limit_setter(WaitLimitSetter setter);  // abi.cu

namespace {
// Copies `ns` into this translation unit's g_wait_limit_ns on the current device.
[[maybe_unused]] bool set_wait_limit_here(uint64_t ns) {
  if (cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof ns) == cudaSuccess) return true;
  cudaGetLastError();
  return false;
}
[[maybe_unused]] const bool g_wait_limit_registered = register_wait_limit_setter(&set_wait_limit_here);
}  // namespace

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The status word lives in pinned host memory mapped into the device, so the
// host reads it after a synchronize with no copy. Bits only ever get set, and
// only on failure; a plain read-modify-write (PCIe atomics are not assumed)
// may drop a concurrent bit but never turns a failure into zero.
__device__ __forceinline__ void report(uint32_t* status, uint32_t bits) {
  if (status != nullptr) {
    volatile uint32_t* s = status;
    *s = *s | bits;
    __threadfence_system();
  }
}

// --------------------------------------------------------------- exact math

// The truncating (int) cast of the reference as x86-64 executes it
// (cvttss2si): toward zero, and INT32_MIN for NaN or values outside int32.
__device__ __forceinline__ int32_t trunc_i32_x86(float q) {
  return (q >= -2147483648.0f && q < 2147483648.0f) ? __float2int_rz(q) : INT32_MIN;
}

// One element of lab_quantize_q8 (lab_native.c:420-425): q = x * inv,
// rounded half away from zero by an f32 add of +-0.5 and a truncating cast,
// clamped to [-127, 127].
__device__ __forceinline__ int32_t quant_q8_elem(float x, float inv) {
  float q = __fmul_rn(x, inv);
  q = q < 0.0f ? __fsub_rn(q, 0.5f) : __fadd_rn(q, 0.5f);
  const int32_t v = trunc_i32_x86(q);
  return v > 127 ? 127 : (v < -127 ? -127 : v);
}

// scale = amax / 127 and inv = 1 / scale (0 when scale is 0), both IEEE
// round-to-nearest divisions (lab_native.c:416-417).
__device__ __forceinline__ void q8_scale(float amax, float& scale, float& inv) {
  scale = __fdiv_rn(amax, 127.0f);
  inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
}

__device__ __forceinline__ uint32_t pack4(int32_t a, int32_t b, int32_t c, int32_t d) {
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) |
         ((uint32_t)(d & 0xff) << 24);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  return __half2float(__ushort_as_half(h));  // exact
}

// RMSNorm (lib/src/ops.dart:12-31) pieces shared by the norm kernel and the
// GEMV prologue that runs a norm itself, so that both give the same bits.
// The sum of squares runs over kNormLanes threads in one fixed order: thread
// t adds x[j]^2 (exact in double) for j = t, t + 128, ... left to right, each
// warp reduces with xor shuffles, and the warp sums add in warp order. The
// reference sums left to right; the two sums differ by a few ulps of a double,
// which moves an f32 output only where x * r lies that close to an f32
// rounding boundary.
constexpr int kNormLanes = 128;

// r = 1 / sqrt(sum / cols + eps), in double. Called by threads 0..127 (tid),
// which `sync` (a barrier over exactly them) holds together; `red` is 4
// doubles of shared memory.
template <typename Sync>
__device__ __forceinline__ double norm_factor(const float* x, int64_t cols, double eps, int tid,
                                              double* red, Sync sync) {
  double s = 0.0;
  for (int64_t j = tid; j < cols; j += kNormLanes) {
    const double v = (double)x[j];
    s = __dadd_rn(s, __dmul_rn(v, v));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  if ((tid & 31) == 0) red[tid >> 5] = s;
  sync();
  double sum = 0.0;
#pragma unroll
  for (int w = 0; w < kNormLanes / 32; w++) sum = __dadd_rn(sum, red[w]);
  return __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)cols), eps)));
}

// One normalized value: (x * r) in double stored to f32, times the weight in f32.
__device__ __forceinline__ float norm_value(float x, float w, double r) {
  return __fmul_rn(w, __double2float_rn(__dmul_rn((double)x, r)));
}

// One SwiGLU output, silu(g) * u, as dianoia's CPU feed-forward computes it
// (lib/src/shard.dart:456-460): g / (1 + exp(-g)) in double, stored to f32,
// then an f32 product with u. CUDA's double exp differs from the C library's
// by at most an ulp of a double, which moves the f32 result only when the
// quotient lies within that of an f32 rounding boundary.
__device__ __forceinline__ float silu_mul(float g, float u) {
  const double gd = (double)g;
  const float s = __double2float_rn(__ddiv_rn(gd, __dadd_rn(1.0, exp(-gd))));
  return __fmul_rn(s, u);
}

// --------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// True in exactly one lane of a converged warp, for single-thread
// instructions (tcgen05.mma, TMA copies) issued on behalf of the warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or about `hint_ns` pass, issuing nothing meanwhile.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// mbar_wait_bounded for waits that may be long (a full stage ring): the
// waiting thread sleeps instead of spinning, leaving issue slots to the
// warps that compute. A wait for threads that are themselves in a bounded
// wait (a barrier behind a wait on another GPU) runs `mult` times the limit,
// so the inner wait gives up first and its own status bit is the one set
// (two bits recorded at the same instant could lose one: report() is a plain
// read-modify-write).
__device__ __forceinline__ bool mbar_wait_bounded_sleep(uint64_t* bar, uint32_t parity,
                                                        uint32_t* status, uint32_t bits,
                                                        uint32_t mult = 1) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (globaltimer_ns() - start > mult * wait_limit_ns()) {
      report(status, bits);
      return false;
    }
  }
}

// Waits for phase `parity` of an mbarrier to complete, for at most
// kWaitLimitNs. Returns false (and records `bits`) if it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* status,
                                                  uint32_t bits) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - start > wait_limit_ns()) {
      report(status, bits);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared (TMA engine), completing on `bar` with
// `bytes` transaction bytes. dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled TMA load of the box at (x, y) of a tensor map into shared
// memory, completing on `bar`. x is in elements of the innermost dimension;
// x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int32_t x, int32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load of the box at (x, y, z), as tma_load_2d.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Pulls a box of a tensor map into L2 only (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_l2_2d(const void* tmap, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(x),
               "r"(y)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait until the previous kernel's writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t lds_u32(const void* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

}  // namespace dn
