/*
 * dianoia_b200 - C-ABI of the B200 (sm_100a) Q4_0 / Q8_0 quantized linear path.
 *
 * libdianoia_b200.so exports the symbols dianoia's Dart code binds through
 * dart:ffi for its quantized products (lib/src/native.dart:135-243), with
 * the same signatures and meaning, so the package's NativeQ8Matrix /
 * NativeQ4Matrix / NativeKernels drive CUDA kernels instead of
 * src/c/lab_native.c. All shapes are int64; outputs are token-major,
 * ys[t * rows + r]. Every call is synchronous: results are in place when it
 * returns, as with the CPU kernels.
 *
 * Pointers may be host memory (pageable or pinned: copied to and from the
 * GPU inside the call), memory from lab_alloc (CUDA managed memory; the GPU
 * reads it in place, so weights allocated there stay in HBM between calls)
 * or device memory.
 *
 * The reference's C functions report no errors; neither do these, but a
 * failure is recorded per thread and returned by dn_last_error().
 *
 * The dn_* functions below the lab_* block are this library's own
 * device-resident API (no counterpart in the reference): device pointers,
 * an explicit CUDA stream, asynchronous, with a status code return.
 */
#ifndef DIANOIA_B200_H_
#define DIANOIA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ lab_* (reference ABI) */

/* Zeroed memory, at least 128-byte aligned, that both the host and the GPU
 * can address (CUDA managed memory); NULL on failure.
 * Replaces lab_alloc, src/c/lab_native.c:88-98; bound at lib/src/native.dart:135. */
void* lab_alloc(int64_t bytes);

/* Frees memory from lab_alloc. Replaces lab_free, lab_native.c:100-104;
 * bound at native.dart:236. */
void lab_free(void* p);

/* 1 when the kernels can run here (a CUDA device of compute capability 10.x),
 * else 0. Replaces lab_cpu_supported, lab_native.c:64-84; bound at native.dart:242. */
int64_t lab_cpu_supported(void);

/* Host helpers the Dart side binds from the same library (native.dart:218-240):
 * lab_map_file maps a whole file read-only (private) and stores its length in
 * *size, NULL if it cannot be opened, is empty or cannot be mapped
 * (lab_native.c:109-149); lab_unmap_file unmaps it (:156); lab_evict_file
 * gives its resident pages back to the OS, the mapping staying valid
 * (:169-171); lab_phys_footprint is the process's resident set in bytes, -1
 * if unknown (:876-891, which reports -1 on Linux). */
void* lab_map_file(const char* path, int64_t* size);
void lab_unmap_file(void* p, int64_t size);
void lab_evict_file(void* p, int64_t size);
int64_t lab_phys_footprint(void);

/* Q8_0 quantization of rows x cols floats: per block of 32, scale = amax/127,
 * q = round-half-away(x / scale) clamped to +-127; the trailing cols % 32
 * values of a row are ignored. Replaces lab_quantize_q8, lab_native.c:407-429;
 * bound at native.dart:137-148. */
void lab_quantize_q8(const float* w, int8_t* qs, float* scales, int64_t rows, int64_t cols);

/* Q4_0 quantization (llama.cpp's quantize_row_q4_0_ref) into split nibbles
 * and fp16 scales. Replaces lab_quantize_q4, lab_native.c:928-955; bound at
 * native.dart:177-188. */
void lab_quantize_q4(const float* w, uint8_t* qs, uint16_t* scales, int64_t rows, int64_t cols);

/* ys[t * rows + r] = (W xs[t])[r] for t < n, W in Q8_0 (qs int8[rows*cols],
 * scales f32[rows*cols/32]). mode 1 quantizes xs into xq (n*cols bytes) and
 * xsc (n*cols/32 floats) first and multiplies int8 by int8; mode 0 multiplies
 * the floats. `threads` is accepted and ignored. Replaces lab_gemm_q8,
 * lab_native.c:546-579; bound at native.dart:150-175. */
void lab_gemm_q8(const int8_t* qs, const float* scales, const float* xs, int8_t* xq, float* xsc,
                 float* ys, int64_t rows, int64_t cols, int64_t n, int64_t threads, int64_t mode);

/* The same for Q4_0 weights (qs uint8[rows*cols/2], scales fp16 bits
 * uint16[rows*cols/32]). Replaces lab_gemm_q4, lab_native.c:1057-1080; bound
 * at native.dart:190-216. */
void lab_gemm_q4(const uint8_t* qs, const uint16_t* scales, const float* xs, int8_t* xq,
                 float* xsc, float* ys, int64_t rows, int64_t cols, int64_t n, int64_t threads,
                 int64_t mode);

/* lab_gemm_q8 with n = 1. Replaces lab_gemv_q8, lab_native.c:581-586 (the
 * reference's stage-5a benchmark symbol; not bound in Dart). */
void lab_gemv_q8(const int8_t* qs, const float* scales, const float* x, int8_t* xq, float* xs,
                 float* y, int64_t rows, int64_t cols, int64_t threads, int64_t mode);

/* ------------------------------------------------- lab_gpu_* (reference GPU-layer ABI)
 *
 * The quantized-product part of dianoia's GPU layer (src/vulkan/lab_vulkan.c;
 * bound in lib/src/gpu.dart:36-312 and driven by GpuLinear / GpuForward):
 * buffers are handles to memory the host reads and writes in place through
 * lab_gpu_contents, between command buffers; lab_gpu_begin opens the single
 * process-wide command buffer, lab_gpu_enc_matmul_* record products into it
 * and lab_gpu_commit runs them. Here a buffer is device memory with a pinned
 * host mirror: a commit copies in the input ranges the host may have written,
 * runs the products and copies the written ranges back. A buffer used as
 * weights is copied to the device once, at its first product, so weights must
 * be written before their first use (as dianoia does). Products quantize
 * their inputs to Q8_0 per block, like the reference's integer-dot path, and
 * equal lab_gemm_q8 / lab_gemm_q4 in mode 1. Calls are serialized. */

/* 1 when a usable B200 is present (the first call sets up), else 0.
 * Replaces lab_gpu_init, lab_vulkan.c:295. */
int64_t lab_gpu_init(void);
/* A zeroed buffer of `bytes`; its handle, or -1. Replaces lab_gpu_buffer,
 * lab_vulkan.c:582 (and lab_gpu_readback_buffer, :590, the same here). */
/* Device queries (lab_vulkan.c:507-530; gpu.dart:39-60): the device's name;
 * the longest buffer (all of the device's memory: one allocation may take
 * it); the attention kernel's score capacity as the reference reports it
 * (keys * 4 + 128 bytes, gpu.dart bounds maxSeq by it); the recommended working set (the
 * device's memory); the thermal state (-1: none on CUDA); host RAM bytes. */
void lab_gpu_device_name(char* out, int64_t capacity);
int64_t lab_gpu_max_buffer_length(void);
int64_t lab_gpu_max_shared_memory(void);
int64_t lab_gpu_recommended_working_set(void);
int64_t lab_gpu_thermal_state(void);
int64_t lab_gpu_physical_memory(void);
/* Product tuning knobs (lab_vulkan.c:670-718). set_decode_rows: 1, 2, 4 and
 * negative values keep the one decode GEMV of this library; 0 runs decode
 * products on the generic kernel, a same-device numerical reference.
 * set_q8_group, set_q8_vector and register_q8_head choose Vulkan workgroup
 * sizes and a vectorized head: unavailable here, so they return 0. */
void lab_gpu_set_decode_rows(int64_t rows);
int64_t lab_gpu_set_q8_group(int64_t invocations);
int64_t lab_gpu_set_q8_vector(int64_t on);
int64_t lab_gpu_register_q8_head(int64_t w, int64_t qs, int64_t rows, int64_t cols, int64_t q4Body);
/* Dispatch profiling (lab_vulkan.c:719-733): with profiling on, every launch
 * of a committed command buffer is timed, from the end of the one before it
 * (or of the uploads) to its own end; lab_gpu_profile copies per kind, in the
 * reference's kind order (gemv_q8, gemm_q8, gemv_q4, gemm_q4, rms_norm,
 * head_norm_rope, conv, attention, swiglu, copy, quantize, gemm_q8_i8,
 * gemm_q4_i8, gemv_q8_i8, gemv_q4_i8, gemv_q8_i8_vec, steer, add) the
 * milliseconds and launches since its last call, starts over and returns the
 * number of kinds. Fused ops count within the product that runs them. */
void lab_gpu_set_profiling(int64_t on);
int64_t lab_gpu_profile(double* ms, int64_t* counts, int64_t kinds);
int64_t lab_gpu_buffer(int64_t bytes);
int64_t lab_gpu_readback_buffer(int64_t bytes);
/* A buffer holding a copy of `bytes` bytes at `address`; handle or -1.
 * Replaces lab_gpu_wrap, lab_vulkan.c:598; lab_gpu_wrap_copies (:605) is 1:
 * the wrapped memory may be freed afterwards. */
int64_t lab_gpu_wrap(void* address, int64_t bytes);
int64_t lab_gpu_wrap_copies(void);
/* The host address of a buffer's contents (NULL for a bad handle).
 * Replaces lab_gpu_contents, lab_vulkan.c:607. */
void* lab_gpu_contents(int64_t handle);
/* Frees a buffer once submitted work is done; its handle is reused.
 * Replaces lab_gpu_release, lab_vulkan.c:637. */
void lab_gpu_release(int64_t handle);
/* Buffers not yet released (leak checks). Replaces lab_gpu_live_buffers, :652. */
int64_t lab_gpu_live_buffers(void);
/* Opens the command buffer (waiting for one committed without waiting).
 * Replaces lab_gpu_begin, lab_vulkan.c:655. */
void lab_gpu_begin(void);
/* Runs the recorded operations; with `wait`, blocks until done. Returns 1, or
 * 0 if an operation's buffers, offsets or sizes did not fit or the GPU failed.
 * Replaces lab_gpu_commit, lab_vulkan.c:737; lab_gpu_wait (:761) waits for a
 * command buffer committed without waiting. */
int64_t lab_gpu_commit(int64_t wait);
int64_t lab_gpu_wait(void);
/* GPU time of the last waited command buffer, ms. Replaces lab_gpu_last_ms, :610. */
double lab_gpu_last_ms(void);
/* Y = X W^T for n tokens: W (rows x cols, Q8_0 with f32 scales, or Q4_0
 * with fp16 scales) at byte offsets qsOffset / scalesOffset of buffer w,
 * X [n, cols] f32 at xOffset of buffer x, Y [n, rows] f32 at yOffset of y.
 * Replaces lab_gpu_enc_matmul_q8 / _q4, lab_vulkan.c:879-891. */
void lab_gpu_enc_matmul_q8(int64_t w, int64_t qsOffset, int64_t scalesOffset, int64_t x,
                           int64_t xOffset, int64_t y, int64_t yOffset, int64_t rows, int64_t cols,
                           int64_t n);
void lab_gpu_enc_matmul_q4(int64_t w, int64_t qsOffset, int64_t scalesOffset, int64_t x,
                           int64_t xOffset, int64_t y, int64_t yOffset, int64_t rows, int64_t cols,
                           int64_t n);
/* RMSNorm of `rows` rows of `cols` f32 values at xOffset of buffer x with the
 * weights at wOffset of buffer w, into `out` at outOffset (added into it with
 * `accumulate`), as dianoia's CPU path computes it (lib/src/ops.dart:12-31:
 * the sum of squares and the reciprocal root in double). The weights' buffer
 * is copied to the device once, like a matrix's. When a later product of the
 * same command buffer reads the output, the norm kernel also writes it as
 * quantized activations for that product (the fused norm -> quantize).
 * Replaces lab_gpu_enc_rms_norm, lab_vulkan.c:899-907 (gpu.dart:180-204). */
void lab_gpu_enc_rms_norm(int64_t x, int64_t xOffset, int64_t w, int64_t wOffset, int64_t out,
                          int64_t outOffset, int64_t rows, int64_t cols, double eps,
                          int64_t accumulate);
/* g = silu(g) * u over `count` f32 values at offset 0 of buffers g and u, as
 * dianoia's CPU feed-forward computes it (lib/src/shard.dart:456-460). Right
 * after the two products that wrote g and u it runs in the second one's
 * epilogue and launches nothing; its results are then also quantized there
 * for the product that reads them. Replaces lab_gpu_enc_swiglu,
 * lab_vulkan.c:974-978 (gpu.dart:280-285). */
void lab_gpu_enc_swiglu(int64_t g, int64_t u, int64_t count);
/* dst += src over `count` f32 values at the byte offsets given: the residual
 * add of a layer without sandwich norms (lib/src/model.dart:946-950). Right
 * after the product that wrote all of src (and does not read dst) it runs in
 * that product's epilogue and launches nothing. Replaces lab_gpu_enc_add,
 * lab_vulkan.c:993-998 (gpu.dart:293-297). */
void lab_gpu_enc_add(int64_t src, int64_t srcOffset, int64_t dst, int64_t dstOffset, int64_t count);

/* A zeroed GPU-layer buffer in device memory only, for data the host never
 * reads or writes: a KV cache, scratch between the ops of a command buffer.
 * lab_gpu_contents returns NULL for it and commits copy nothing into or out
 * of it (a lab_gpu_buffer is copied in where the host may have written it
 * and out where the GPU wrote it, every commit). Its handle, or -1. No
 * counterpart in the reference, whose buffers are host-visible memory. */
int64_t dn_gpu_device_buffer(int64_t bytes);

/* A GPU-layer buffer holding bytes [offset, offset + bytes) of the file at
 * `path`, read straight into device memory (slices on up to 8 host threads,
 * each through pinned staging chunks whose reads overlap their device
 * copies); its handle, or -1 if the file cannot be read or is shorter.
 * For weights such as a mapped Q8 cache
 * (lib/src/q8_cache.dart, GpuForward._wrapWeights at gpu.dart:942-979): the
 * buffer has no host mirror (lab_gpu_contents returns NULL) and a commit
 * copies nothing into or out of it. No counterpart in the reference, whose
 * lab_gpu_wrap takes the mapping's address (that works here too, copying). */
int64_t dn_gpu_wrap_file(const char* path, int64_t offset, int64_t bytes);

/* With on = 0, command buffers committed from now on run every operation as
 * its own kernel on f32 inputs, with no QA links and no fusions, as the
 * reference's GPU layer dispatches them; with on = 1 (the default) they run
 * fused. The results are the same bit for bit; only the time differs. No
 * counterpart in the reference. */
void dn_gpu_set_fusion(int64_t on);

/* The rest of a decode layer as dianoia's GpuForward encodes it, with the
 * arithmetic of its CPU path (double where Dart computes in double, f32
 * where it stores into a Float32List). Offsets are bytes; strides floats.
 * lab_gpu_enc_copy: dst = src, count floats (lab_vulkan.c:985-991).
 * lab_gpu_enc_steer: rows of cols floats at x: mode 0 adds v, mode 1
 *   subtracts scale * (x . v) * v (lab_vulkan.c:1010-1016;
 *   control_vector.dart:176-203).
 * lab_gpu_enc_head_norm_rope: per (head, token) RMSNorm over hd values with
 *   weights w, then the half-split RoPE from the token's table
 *   [cos(hd/2), sin(hd/2)] at rope + ropeOffset + token * ropeStride; token t
 *   of x at xOffset + t * xStride (lab_vulkan.c:916-930; shard.dart:548-557,
 *   ops.dart:12-71). hd even, at most 256.
 * lab_gpu_enc_conv: the gated short convolution: bcx [n, 3 width] (B, C, X),
 *   weights [width, k] at weightOffset, history [k - 1, width] read and
 *   updated, y [n, width] = C * causal conv of B * X (lab_vulkan.c:932-941;
 *   shard.dart:476-516). k at most 16.
 * lab_gpu_enc_attention: causal grouped-query attention of n tokens at
 *   positions position.. over the KV cache (rows [position + n, kvHeads *
 *   hd]), q and out [n, heads * hd], gate [n, heads] before the sigmoid or a
 *   negative handle for none, window > 0 keeping the current key and the
 *   window - 1 before it (lab_vulkan.c:949-966; shard.dart:589-628). hd a
 *   multiple of 4 up to 256 (the reference's shader reads vec4s); a token
 *   sees at most 16384 keys (what lab_gpu_max_shared_memory reports). */
void lab_gpu_enc_copy(int64_t src, int64_t srcOffset, int64_t dst, int64_t dstOffset, int64_t count);
void lab_gpu_enc_steer(int64_t x, int64_t xOffset, int64_t v, int64_t vOffset, int64_t rows,
                       int64_t cols, int64_t mode, double scale);
void lab_gpu_enc_head_norm_rope(int64_t x, int64_t xOffset, int64_t xStride, int64_t w, int64_t wOffset,
                                int64_t rope, int64_t ropeOffset, int64_t ropeStride, int64_t heads,
                                int64_t hd, int64_t n, double eps);
void lab_gpu_enc_conv(int64_t bcx, int64_t weight, int64_t weightOffset, int64_t history, int64_t y,
                      int64_t width, int64_t k, int64_t n);
void lab_gpu_enc_attention(int64_t q, int64_t keys, int64_t values, int64_t gate, int64_t out,
                           int64_t position, int64_t n, int64_t heads, int64_t kvHeads, int64_t hd,
                           int64_t window);

/* Kinds of the rows of dn_gpu_enc_batch. */
#define DN_BATCH_Q8 0
#define DN_BATCH_Q4 1
#define DN_BATCH_RMS_NORM 2
#define DN_BATCH_SWIGLU 3
#define DN_BATCH_ADD 4
#define DN_BATCH_COPY 5
#define DN_BATCH_STEER 6
#define DN_BATCH_HEAD_NORM_ROPE 7
#define DN_BATCH_CONV 8
#define DN_BATCH_ATTENTION 9

/* Records `count` operations into the open command buffer in one call,
 * exactly as the same sequence of lab_gpu_enc_* calls would. No counterpart
 * in the reference: it is for callers whose per-call cost is high (a Python
 * ctypes call costs microseconds, a Dart @Native leaf call tens of
 * nanoseconds). Row i of `table` is 11 int64 values, the kind and then the
 * arguments of the call it stands for, in order:
 *   DN_BATCH_Q8 / DN_BATCH_Q4: w, qsOffset, scalesOffset, x, xOffset, y,
 *     yOffset, rows, cols, n (lab_gpu_enc_matmul_q8 / _q4);
 *   DN_BATCH_RMS_NORM: x, xOffset, w, wOffset, out, outOffset, rows, cols,
 *     the bits of eps as a double, accumulate (lab_gpu_enc_rms_norm);
 *   DN_BATCH_SWIGLU: g, u, count, then unused (lab_gpu_enc_swiglu);
 *   DN_BATCH_ADD: src, srcOffset, dst, dstOffset, count, then unused
 *     (lab_gpu_enc_add);
 *   DN_BATCH_COPY: src, srcOffset, dst, dstOffset, count (lab_gpu_enc_copy);
 *   DN_BATCH_STEER: x, xOffset, v, vOffset, rows, cols, mode, the bits of
 *     scale as a double (lab_gpu_enc_steer);
 *   DN_BATCH_HEAD_NORM_ROPE: x, xOffset, xStride, w, wOffset, rope,
 *     ropeOffset, ropeStride, heads | hd << 16 | n << 32, the bits of eps
 *     (lab_gpu_enc_head_norm_rope; heads and hd below 65536);
 *   DN_BATCH_CONV: bcx, weight, weightOffset, history, y, width, k, n
 *     (lab_gpu_enc_conv);
 *   DN_BATCH_ATTENTION: q, keys, values, gate, out, position, n, heads,
 *     kvHeads, hd | window << 32 (lab_gpu_enc_attention).
 * An unknown kind makes the next lab_gpu_commit return 0. */
void dn_gpu_enc_batch(const int64_t* table, int64_t count);

/* ------------------------------------------------------------ dn_* (device API) */

/* Status codes of the dn_* functions and of dn_last_error(). */
#define DN_OK 0
#define DN_ERR_ARGS (-1)        /* a shape, pointer or mode that is not accepted */
#define DN_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define DN_ERR_NO_DEVICE (-3)   /* no usable sm_100 device */
#define DN_ERR_UNSUPPORTED (-4) /* a combination this build does not implement */
#define DN_ERR_TOO_LARGE (-5)   /* a size beyond a stated maximum */

/* Weight formats and kernel paths for dn_linear. */
#define DN_Q8 0
#define DN_Q4 1
#define DN_PATH_AUTO (-1)
#define DN_PATH_GEMV 0    /* decode GEMV: bit-exact with lab_native.c */
#define DN_PATH_TC 1      /* tcgen05 int8 GEMM */
#define DN_PATH_GENERIC 2 /* any alignment / mode, slow */

/* Flags for dn_linear. DN_FLAG_PDL launches with programmatic dependent
 * launch: the kernel may start reading the weights before the previous kernel
 * in the stream has finished, so it is only for weights no kernel in flight
 * writes. */
#define DN_FLAG_PDL 1

/* ys[t * ldy + r] = (W xs[t])[r] on `stream` (a cudaStream_t; NULL = default
 * stream), all pointers device-addressable. `format` DN_Q8 (qs int8, scales
 * f32) or DN_Q4 (qs nibbles, scales fp16 bits). In mode 1, xq / xsc receive the
 * quantized activations; the GEMV path accepts NULL for both. Returns DN_OK or
 * a DN_ERR_* code. */
int64_t dn_linear(int64_t format, const void* qs, const void* scales, const float* xs, int8_t* xq,
                  float* xsc, float* ys, int64_t rows, int64_t cols, int64_t n, int64_t ldy,
                  int64_t mode, int64_t path, int64_t flags, void* stream);

/* Which path DN_PATH_AUTO picks for these arguments; NULL pointers stand for
 * suitably aligned buffers the caller will provide. */
int64_t dn_linear_path(int64_t format, const void* qs, const void* scales, const float* xs,
                       const int8_t* xq, int64_t rows, int64_t cols, int64_t n, int64_t mode);

/* GGUF Q4_0 / Q8_0 blocks in device memory split into the engine's layout
 * on the device, asynchronous: what dianoia's loader does on the CPU
 * (gguf.dart:206-215 splitQ4_0, gguf.dart:269-283 splitQ8_0), so a loader
 * can copy the file's blocks to the GPU as they are. `count` blocks of 18
 * (Q4_0) or 34 (Q8_0) bytes, 2-byte aligned; qs (4-byte aligned) receives
 * 16 or 32 value bytes per block; scales receives the fp16 scale bytes
 * (Q4_0, 2-byte aligned) or the scale widened to f32 (Q8_0, 4-byte aligned). */
int64_t dn_gguf_split(int64_t format, const void* blocks, int64_t count, void* qs, void* scales,
                      void* stream);

/* The one-token product straight on GGUF blocks, with no split: ys[r] for
 * rows r = 0 .. rows - 1 of a matrix stored as the file stores it, `rows`
 * rows of cols / 32 Q4_0 (18-byte) or Q8_0 (34-byte) blocks each, times one
 * token of QA activations xa (cols / 32 blocks of 36 bytes, as
 * dn_quantize_qa writes them; 4-byte aligned). The result equals lab_gemm_q4
 * / lab_gemm_q8 (mode 1, n = 1, lab_native.c:553-579, 1059-1080) on the
 * weights dianoia's loader would split (gguf.dart:206-215, 269-283), bit for
 * bit. `blocks` 16-byte aligned; cols a multiple of 256 (Q8_0) or 512
 * (Q4_0), else DN_ERR_ARGS; asynchronous on `stream`; DN_FLAG_PDL as for
 * dn_linear. */
int64_t dn_gguf_linear_qa(int64_t format, const void* blocks, const uint8_t* xa, float* ys, int64_t rows,
                          int64_t cols, int64_t flags, void* stream);

/* lab_quantize_q8 / lab_quantize_q4 on device memory, asynchronous. */
int64_t dn_quantize_q8(const float* xs, int8_t* xq, float* xsc, int64_t n, int64_t cols,
                       void* stream);
int64_t dn_quantize_q4(const float* w, uint8_t* qs, uint16_t* scales, int64_t rows, int64_t cols,
                       void* stream);

/* Quantized activations ("QA" blocks) for chains of products: per 32 values,
 * the 32 int8 that lab_quantize_q8 gives, then their f32 scale (36 bytes).
 * Token t starts at xa + t * xa_stride. dn_quantize_qa writes them from f32
 * activations [n, cols]. */
int64_t dn_quantize_qa(const float* xs, uint8_t* xa, int64_t n, int64_t cols, int64_t xa_stride,
                       void* stream);

/* The decode path's neighbours of the products on device memory,
 * asynchronous, as dianoia's CPU path computes them:
 * dn_rms_norm: out = w * (x * r) per row, r = 1 / sqrt(mean(x^2) + eps)
 *   (lib/src/ops.dart:12-31; with accumulate, added into out), `rows` rows of
 *   `cols` values; with qa not NULL (cols % 32 == 0) the results also as QA
 *   blocks, row t at qa + t * qa_stride.
 * dn_swiglu: g = silu(g) * u over `count` values (lib/src/shard.dart:456-460);
 *   with qa not NULL (count % 32 == 0) the results also as QA blocks, block
 *   b at qa + 36 * b.
 * flags: DN_FLAG_PDL launches with programmatic dependent launch. */
int64_t dn_rms_norm(const float* x, const float* w, float* out, uint8_t* qa, int64_t qa_stride,
                    int64_t rows, int64_t cols, double eps, int64_t accumulate, int64_t flags,
                    void* stream);
int64_t dn_swiglu(float* g, const float* u, uint8_t* qa, int64_t count, int64_t flags, void* stream);

/* The decode GEMV on QA activations: ys[t * ldy + r] = (W x_t)[r] (ys may be
 * NULL), and, when ya is not NULL, the outputs quantized again into QA blocks
 * (block r / 32 of token t at ya + t * ya_stride; only whole 32-row blocks),
 * ready to be the next product's input. Results equal lab_gemm_q8 /
 * lab_gemm_q4 (mode 1) on the dequantized inputs, bit for bit. */
int64_t dn_linear_qa(int64_t format, const void* qs, const void* scales, const uint8_t* xa,
                     int64_t xa_stride, float* ys, int64_t ldy, uint8_t* ya, int64_t ya_stride,
                     int64_t rows, int64_t cols, int64_t n, int64_t flags, void* stream);

/* A decode chain: the quantized products of one token (or any sequence of
 * GEMVs on QA activations) run by ONE persistent kernel, so HBM keeps
 * streaming weights across the dependencies between them. Op i reads QA
 * activations `xa` (n = 1, stride cols / 32 * 36). If `dep` >= 0, op i
 * starts after op `dep` has finished, inside the kernel: a data edge when xa
 * lies in the QA output `ya` of op dep (from any 36-byte block of it, e.g.
 * the q rows of a fused qkv output), else an ordering edge (xa was written
 * before the launch; a step outside the chain, such as a norm, sits between
 * the two ops). Outputs: f32 `ys` and/or QA `ya` (ya needs rows % 32
 * == 0). Results equal one dn_linear_qa per op, bit for bit. All ops share
 * one format.
 * Only dep edges order the ops: a CTA starts on the next op once its own
 * tiles of the previous one are done, so ops of different layers overlap.
 * Each output buffer therefore belongs to one op; it may not overlap another
 * op's output, weights or scales, nor an input other than a dependent's
 * (DN_ERR_ARGS). A stack of layers gets one output buffer per op. */
typedef struct dn_chain_op {
  const void* qs;
  const void* scales;
  const uint8_t* xa;
  float* ys;
  uint8_t* ya;
  int64_t rows, cols, dep;
} dn_chain_op;

/* Validates the ops, encodes their TMA descriptors and copies the op table to
 * device memory (the chain's only allocations); *chain receives a handle. */
int64_t dn_chain_create(int64_t format, const dn_chain_op* ops, int64_t nops, void** chain);
/* The row-sharded lm_head (or any one-token product on QA input) with the
 * all-gather of its f32 outputs fused into the product, for N GPUs of one
 * node (north_star's row-partitioned weights with an all-gather of each
 * GPU's output slice; the reference shards the LM head's vocabulary rows the
 * same way, lib/src/shard.dart:12-13). This GPU computes rows row0 .. row0 +
 * rows of the whole output from its row slice (qs, scales) and stores each
 * into every rank's copy of the whole output, ys[p] + row0 + row (ys[p]: rank
 * p's buffer as mapped here - dn_peer_alloc / dn_peer_open memory - the
 * local one included; plain stores over NVLink), then adds the number of
 * its 32-row tiles to every rank's counter (counters[p], in the same
 * regions) after a system-scope fence. A rank's copy is complete once its
 * counter has grown by the tiles of all ranks: dn_peer_wait. Results equal
 * dn_linear_qa's rows bit for bit. */
int64_t dn_linear_qa_allgather(int64_t format, const void* qs, const void* scales, const uint8_t* xa,
                               int64_t rows, int64_t cols, int64_t row0, float* const* ys,
                               int32_t* const* counters, int64_t world, int64_t flags, void* stream);
/* The prefill / vision product (the tensor-core GEMM, mode 1 on f32 inputs
 * xs [n, cols], xq / xsc its quantized-input scratch as for dn_linear) on N
 * GPUs of one node with row-partitioned weights (north_star's sharding; the
 * reference's row split, lab_native.c:550-579: a row's result does not
 * depend on it): this GPU holds rows row0 .. row0 + rows of the total_rows
 * of the whole matrix and stores every output value into every rank's copy
 * of Y[n, total_rows], ys[p][t * total_rows + row0 + r] (ys[p]: rank p's
 * buffer as mapped here - dn_peer_alloc / dn_peer_open memory - the local
 * one included; plain stores over NVLink, no TMA on peer memory), inside the
 * GEMM's epilogue. When the GEMM has completed, one thread makes the stores
 * visible system-wide and adds one to every rank's counter (counters[p]), so
 * a rank's copy is complete once its counter has grown by `world` (one per
 * rank): dn_peer_wait. Nothing is counted after a bounded wait ran out (a
 * set dn_device_status). The kernel is the one dn_linear's tensor-core path
 * picks for n tokens (narrow tiles up to 32); its results equal that path's
 * on the whole matrix value for value when cols / 128 is a multiple of 4
 * (the narrow kernel's four partial sums then fall the same way on every
 * slice), and lie within its 1e-5 bound otherwise. */
int64_t dn_linear_allgather(int64_t format, const void* qs, const void* scales, const float* xs, int8_t* xq,
                            float* xsc, int64_t rows, int64_t cols, int64_t n, int64_t row0, int64_t total_rows,
                            float* const* ys, int32_t* const* counters, int64_t world, void* stream);
/* Waits on `stream` (one thread of the GPU, bounded: a timeout sets the
 * peer-timeout bit of dn_device_status) until *counter has grown by `count`
 * since the previous wait with the same `expect` word, a device int32 that
 * holds the count reached last time (zero both before the first wait).
 * Counters only grow, so nothing is reset between steps. */
int64_t dn_peer_wait(const int32_t* counter, int32_t* expect, int64_t count, void* stream);

/* Device memory that the other GPUs of this node can map: dn_peer_alloc
 * allocates `bytes` (zeroed) on the current device and writes a
 * DN_PEER_HANDLE_BYTES-byte handle to pass to the other processes;
 * dn_peer_open maps another process's memory from its handle (on any GPU of
 * the node, reached over NVLink); dn_peer_close unmaps it, dn_peer_free frees
 * one's own. */
#define DN_PEER_HANDLE_BYTES 64
int64_t dn_peer_alloc(int64_t bytes, void** ptr, void* handle);
int64_t dn_peer_open(const void* handle, void** ptr);
int64_t dn_peer_close(void* ptr);
int64_t dn_peer_free(void* ptr);

/* A decode chain split by output rows over `world` GPUs (1..8), one process
 * per GPU: this rank's op i holds rows row0[i] .. row0[i] + rows of the
 * total_rows[i] rows of the whole projection (row0 a multiple of 32; rows too
 * when the op has QA outputs). Its outputs are the WHOLE projection's: ys
 * (here only, indexed by the whole projection's rows) and ya, where every
 * tile's QA block is also stored into every other rank's copy, over NVLink,
 * and the tile counted in every rank's counters, so no collective is needed
 * between ops. bases[p] is rank p's region (dn_peer_alloc memory, the same
 * layout on every rank) as mapped in this process (bases[rank] its own);
 * every ya and `counters` (nops + 2 int32, zero before the first run) must
 * lie in the local region at the same offsets on every rank. Every rank runs
 * the chain once per token; dn_chain_reset must be called on all ranks
 * together. */
int64_t dn_chain_create_sharded(int64_t format, const dn_chain_op* ops, const int64_t* row0,
                                const int64_t* total_rows, int64_t nops, int64_t rank,
                                int64_t world, void* const* bases, int64_t region_bytes,
                                int32_t* counters, void** chain);
/* Runs the chain on `stream` (asynchronous; capturable in a CUDA graph).
 * DN_FLAG_PDL lets the weights start streaming while the previous kernel
 * finishes; inputs with dep = -1 are read only after it completes. */
int64_t dn_chain_run(void* chain, int64_t flags, void* stream);
/* Clears the chain's completion counters and its run index (only needed
 * after a run that reported a bounded-wait timeout). */
int64_t dn_chain_reset(void* chain, void* stream);
int64_t dn_chain_destroy(void* chain);

/* A decode stack: the one-token Q8_0 products of a decode step on f32
 * activations (lab_gemm_q8 mode 1, n = 1, lab_native.c:553-579), run by ONE
 * persistent kernel with one CTA per SM. Every product's rows are split
 * evenly over all SMs; each SM's weights stream ahead through its
 * shared-memory ring while earlier products compute, and a product whose
 * `dep` is op j starts on every SM as soon as op j's last SM has stored its
 * outputs (a counter in device memory, no kernel boundary). Op i reads f32
 * `x` (cols values, 16-byte aligned; with dep = j it may lie inside op j's
 * output `y`, e.g. the q rows of a fused qkv output) and writes f32 `y`
 * (rows values). dep = -1: x was written before the launch (with
 * DN_FLAG_PDL, read after the previous kernel completes); otherwise an
 * earlier op, which then orders the two even when x is elsewhere. Each
 * product quantizes its input itself (lab_quantize_q8), so results equal one
 * lab_gemm_q8 (mode 1, n = 1) per op, bit for bit. Q8_0 only (format DN_Q8;
 * DN_Q4 is DN_ERR_UNSUPPORTED), cols a multiple of 512 and at most 8192.
 * Each output belongs to one op: it may not overlap another op's output or
 * any weights, nor an input other than through a dep edge (DN_ERR_ARGS).
 * No counterpart object in the reference: dianoia runs these products one
 * dispatch each (lib/src/gpu.dart:1130-1190). */
typedef struct dn_stack_op {
  const void* qs;
  const void* scales;
  const float* x;
  float* y;
  int64_t rows, cols, dep;
} dn_stack_op;
/* Validates the ops, encodes their TMA descriptors and copies the op table
 * and zeroed completion counters to device memory (the stack's only
 * allocations); *stack receives a handle. */
int64_t dn_stack_create(int64_t format, const dn_stack_op* ops, int64_t nops, void** stack);
/* Runs every op once, in order, on `stream` (asynchronous; capturable in a
 * CUDA graph). Runs of one stack must not overlap in time. */
int64_t dn_stack_run(void* stack, int64_t flags, void* stream);
/* Clears the completion counters (only needed after a run that reported a
 * bounded-wait timeout in dn_device_status). */
int64_t dn_stack_reset(void* stack, void* stream);
int64_t dn_stack_destroy(void* stack);

/* dn_linear in mode 1 with the automatic path, for callers that must not
 * allocate: an engine that reserves all of its device memory up front and
 * cannot have a library grow it, or code that may not call cudaMalloc and
 * friends (no counterpart in the reference). The tensor-core path's scratch
 * (the quantized activations) and the kernels' status word live in a fixed
 * __device__ array of this library (9 MiB + 256 bytes, created with the
 * module): n * cols may be at most 8 Mi (8388608), else DN_ERR_TOO_LARGE and
 * nothing is launched. The first call on each device looks up that array's
 * address (make it before capturing a stream). The scratch starts undefined
 * and need not be cleared: every call quantizes its activations into it
 * before reading them. Calls that overlap in time on one device share the
 * scratch and race (one stream, or calls ordered by events, is safe). A
 * bounded wait that ran out (a broken device, never an input) is recorded in
 * the array's status word, which dn_linear_noalloc_status reads (not
 * dn_device_status). Results equal dn_linear's with DN_PATH_AUTO and mode 1. */
int64_t dn_linear_noalloc(int64_t format, const void* qs, const void* scales, const float* xs,
                          float* ys, int64_t rows, int64_t cols, int64_t n, int64_t ldy,
                          int64_t flags, void* stream);
/* The status word of dn_linear_noalloc's fixed array on the current device:
 * the same bits as dn_device_status (0 when every bounded wait completed),
 * cleared when `clear` is non-zero. A synchronous copy of four bytes, no
 * allocation: call it after synchronizing the streams of the calls it
 * covers. No counterpart in the reference. */
int64_t dn_linear_noalloc_status(int64_t clear);

/* Measurement only: the tensor-core GEMM's drain step by itself - per block
 * a TMEM load of the 128 x 64 int32 tile, the exact int -> float
 * conversion, the rank-1 scale product and the f32x2 accumulate, the
 * per-32-block work that exact reference semantics put on the CUDA cores
 * (lab_native.c:456-466, 987-1002) - with no MMA, copy or barrier: `ctas`
 * CTAs (one per SM) each run `stages` stages of 4 blocks of 128 x 64
 * elements; out receives ctas x 576 floats. Timing it gives the element-
 * blocks per clock an SM can drain, the GEMM's own ceiling. */
int64_t dn_drain_probe(int64_t ctas, int64_t stages, float* out, void* stream);

/* The calling thread's last error from a lab_* call (DN_OK if none), cleared
 * by reading. */
int64_t dn_last_error(void);

/* Bits the kernels on the current device set when a bounded wait gave up
 * (1: bulk copy, 2: peer flag, 4: tensor-core commit); cleared by reading
 * when `clear` is non-zero. Call after synchronizing. */
int64_t dn_device_status(int64_t clear);

/* Sets how long every bounded wait of the kernels launched afterwards on the
 * current device spins before it records a timeout in the status word and
 * returns (ns > 0; 0 restores the default of 2 s). A synchronous copy into
 * each kernel module: call it outside stream capture, with no kernel of the
 * library running on the device. Returns DN_OK. (The reference's GPU layer
 * reports a failed command buffer as commit() == 0, lab_vulkan.c:737-757;
 * this is the knob that lets a test make such a failure happen quickly.) */
int64_t dn_set_wait_limit_ns(int64_t ns);

/* A short English description of a DN_* code. */
const char* dn_error_string(int64_t code);

#ifdef __cplusplus
}
#endif

#endif /* DIANOIA_B200_H_ */
