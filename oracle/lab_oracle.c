/*
 * TEST INFRASTRUCTURE ONLY - not part of the product.
 *
 * A scalar C restatement of dianoia's CPU kernels for the Q4_0 / Q8_0
 * block-quantized linear path (src/c/lab_native.c in Atrac613/dianoia).
 * It is the checker for the CUDA kernels of this repository: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.
 *
 * Every function reproduces the reference's float operations in the
 * reference's order, one rounding per operation (build with
 * -ffp-contract=off -fno-fast-math, as the reference's own build hook does,
 * hook/build.dart:26), so its results equal the reference's bit for bit.
 * That claim is pinned by tests/test_oracle.py against outputs of the
 * reference library itself (oracle/_ref, compiled from lab_native.c) and the
 * committed fixtures in tests/golden/.
 *
 * Layouts (all row-major, "blocks" = cols / 32):
 *   Q8 weights: qs int8[rows * cols], scales f32[rows * blocks]
 *   Q4 weights: qs uint8[rows * cols / 2] (weight k of a block in the low
 *               nibble of byte k, weight k + 16 in the high nibble),
 *               scales fp16 bits uint16[rows * blocks]; weight = d * (q - 8)
 *   activations xs f32[n * cols]; quantized xq int8[n * cols], xsc f32[n * blocks]
 *   outputs ys f32[n * rows], token-major: ys[t * rows + r]
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { BLK = 32 };

/* x86 cvttss2si, which the reference's (int) casts compile to on x86-64:
 * truncation toward zero, and INT32_MIN for NaN or anything outside int32. */
static int32_t trunc_i32(float q) {
  if (q >= -2147483648.0f && q < 2147483648.0f) return (int32_t)q;
  return INT32_MIN;
}

/* IEEE binary16 bits -> binary32, exact (lab_native.c:905-926 uses F16C). */
float orc_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int shifts = 0;
      while (!(man & 0x400u)) {
        man <<= 1;
        shifts++;
      }
      bits = sign | ((uint32_t)(113 - shifts) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* binary32 -> binary16 bits, round to nearest even (F16C with
 * _MM_FROUND_TO_NEAREST_INT, lab_native.c:922-925). NaN keeps its top payload
 * bits and is made quiet, as F16C does. */
uint16_t orc_float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, a = x & 0x7fffffffu;
  if (a >= 0x7f800000u) {
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((a >> 13) & 0x3ffu));
    return (uint16_t)(sign | 0x7c00u);
  }
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to infinity */
  if (a < 0x38800000u) {                                      /* half subnormal or zero */
    if (a <= 0x33000000u) return (uint16_t)sign;             /* <= 2^-25: ties to even 0 */
    const uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
    const int shift = 126 - (int)e;
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t q = (((a >> 23) - 112u) << 10) | ((a & 0x7fffffu) >> 13);
  const uint32_t rem = a & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

/* lab_quantize_q8 (lab_native.c:407-429): per block of 32, amax by strict
 * '>' from 0, scale = amax / 127, inv = 1 / scale (0 when scale is 0),
 * q = x * inv rounded half away from zero by an f32 add of +-0.5 and a
 * truncating cast, clamped to [-127, 127]. */
void orc_quantize_q8(const float* w, int8_t* qs, float* scales, int64_t rows, int64_t cols) {
  const int64_t blocks = cols / BLK;
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t b = 0; b < blocks; b++) {
      const float* src = w + r * cols + b * BLK;
      float amax = 0.0f;
      for (int k = 0; k < BLK; k++) {
        const float a = src[k] < 0 ? -src[k] : src[k];
        if (a > amax) amax = a;
      }
      const float scale = amax / 127.0f;
      const float inv = scale > 0 ? 1.0f / scale : 0.0f;
      scales[r * blocks + b] = scale;
      for (int k = 0; k < BLK; k++) {
        float q = src[k] * inv;
        q = q < 0 ? q - 0.5f : q + 0.5f;
        const int32_t v = trunc_i32(q);
        qs[r * cols + b * BLK + k] = (int8_t)(v > 127 ? 127 : v < -127 ? -127 : v);
      }
    }
  }
}

/* lab_quantize_q4 (lab_native.c:928-955), llama.cpp's quantize_row_q4_0_ref:
 * d = (value of largest magnitude) / -8, q = (int8)(x * (1/d) + 8.5) capped
 * at 15. The int8 cast keeps the low byte of cvttss2si's result. */
void orc_quantize_q4(const float* w, uint8_t* qs, uint16_t* scales, int64_t rows, int64_t cols) {
  const int64_t blocks = cols / BLK;
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t b = 0; b < blocks; b++) {
      const float* src = w + r * cols + b * BLK;
      float amax = 0.0f, max = 0.0f;
      for (int k = 0; k < BLK; k++) {
        const float a = src[k] < 0 ? -src[k] : src[k];
        if (a > amax) {
          amax = a;
          max = src[k];
        }
      }
      const float d = max / -8.0f;
      const float id = d != 0.0f ? 1.0f / d : 0.0f;
      scales[r * blocks + b] = orc_float_to_half(d);
      uint8_t* q = qs + (r * cols + b * BLK) / 2;
      for (int k = 0; k < BLK / 2; k++) {
        const int8_t lo = (int8_t)trunc_i32(src[k] * id + 8.5f);
        const int8_t hi = (int8_t)trunc_i32(src[k + 16] * id + 8.5f);
        q[k] = (uint8_t)((lo > 15 ? 15 : lo) | ((hi > 15 ? 15 : hi) << 4));
      }
    }
  }
}

/* Weight j (0..31) of a block as an int: Q8 byte, or Q4 nibble minus 8. */
static inline int wq8(const int8_t* blk, int j) { return blk[j]; }
static inline int wq4(const uint8_t* blk, int j) {
  return (j < 16 ? (blk[j] & 15) : (blk[j - 16] >> 4)) - 8;
}

/* The four per-lane int32 sums of one block (dot_q8_sdot / dot_q4_sdot,
 * lab_native.c:456-466, 987-1002 and their AVX2 twins :503-512, :1025-1034):
 * lane l sums bytes 4l..4l+3 of the first and of the second 16-byte half. */
static void lane_dots(const void* wblk, int q4, const int8_t* xb, int32_t d[4]) {
  for (int l = 0; l < 4; l++) {
    int32_t s = 0;
    for (int h = 0; h < 32; h += 16) {
      for (int i = 0; i < 4; i++) {
        const int j = h + 4 * l + i;
        const int w = q4 ? wq4((const uint8_t*)wblk, j) : wq8((const int8_t*)wblk, j);
        s += w * xb[j];
      }
    }
    d[l] = s;
  }
}

/* One output of the int8-input path: per block acc_l = fma(f32(d_l),
 * f32(sw * sx), acc_l); the lanes end as (acc0 + acc1) + (acc2 + acc3)
 * (lane_sum, lab_native.c:208-212). */
static float dot_i8(const void* row, const void* row_scales, int q4, const int8_t* xq,
                    const float* xs, int64_t blocks) {
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int64_t b = 0; b < blocks; b++) {
    int32_t d[4];
    const void* blk = q4 ? (const void*)((const uint8_t*)row + b * 16)
                         : (const void*)((const int8_t*)row + b * BLK);
    lane_dots(blk, q4, xq + b * BLK, d);
    const float sw = q4 ? orc_half_to_float(((const uint16_t*)row_scales)[b])
                        : ((const float*)row_scales)[b];
    const float s = sw * xs[b];
    for (int l = 0; l < 4; l++) acc[l] = fmaf((float)d[l], s, acc[l]);
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

/* One output of the float-input path (dot_q8_f32 / dot_q4_f32,
 * lab_native.c:433-451, 959-983 and the AVX2 twins): per block lane l
 * chains fma over elements 4m + l, m = 0..7, then acc_l = fma(s_l, sw, acc_l). */
static float dot_f32(const void* row, const void* row_scales, int q4, const float* x,
                     int64_t blocks) {
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int64_t b = 0; b < blocks; b++) {
    const void* blk = q4 ? (const void*)((const uint8_t*)row + b * 16)
                         : (const void*)((const int8_t*)row + b * BLK);
    const float sw = q4 ? orc_half_to_float(((const uint16_t*)row_scales)[b])
                        : ((const float*)row_scales)[b];
    for (int l = 0; l < 4; l++) {
      float s = 0.0f;
      for (int m = 0; m < 8; m++) {
        const int j = 4 * m + l;
        const int w = q4 ? wq4((const uint8_t*)blk, j) : wq8((const int8_t*)blk, j);
        s = fmaf((float)w, x[b * BLK + j], s);
      }
      acc[l] = fmaf(s, sw, acc[l]);
    }
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

/* lab_gemm_q8 / lab_gemm_q4 (lab_native.c:553-579, 1059-1080) without the
 * thread split, which does not change any result (lab_native.c:550-552).
 * mode 1 quantizes xs into xq / xsc first; mode 0 multiplies float inputs. */
static void gemm(int q4, const void* qs, const void* scales, const float* xs, int8_t* xq,
                 float* xsc, float* ys, int64_t rows, int64_t cols, int64_t n, int64_t mode) {
  const int64_t blocks = cols / BLK;
  if (mode == 1) orc_quantize_q8(xs, xq, xsc, n, cols);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    const void* row = q4 ? (const void*)((const uint8_t*)qs + r * cols / 2)
                         : (const void*)((const int8_t*)qs + r * cols);
    const void* rs = q4 ? (const void*)((const uint16_t*)scales + r * blocks)
                        : (const void*)((const float*)scales + r * blocks);
    for (int64_t t = 0; t < n; t++) {
      ys[t * rows + r] = mode == 1
                             ? dot_i8(row, rs, q4, xq + t * cols, xsc + t * blocks, blocks)
                             : dot_f32(row, rs, q4, xs + t * cols, blocks);
    }
  }
}

void orc_gemm_q8(const int8_t* qs, const float* scales, const float* xs, int8_t* xq, float* xsc,
                 float* ys, int64_t rows, int64_t cols, int64_t n, int64_t mode) {
  gemm(0, qs, scales, xs, xq, xsc, ys, rows, cols, n, mode);
}

void orc_gemm_q4(const uint8_t* qs, const uint16_t* scales, const float* xs, int8_t* xq,
                 float* xsc, float* ys, int64_t rows, int64_t cols, int64_t n, int64_t mode) {
  gemm(1, qs, scales, xs, xq, xsc, ys, rows, cols, n, mode);
}

/* Per-block int32 dot products of the int8 path, dots[(t * rows + r) * blocks
 * + b] = sum over the block of w * xq (the sum of the four lane sums), for
 * checking the int32 stage of a kernel on its own. */
void orc_block_dots(int q4, const void* qs, const int8_t* xq, int32_t* dots, int64_t rows,
                    int64_t cols, int64_t n) {
  const int64_t blocks = cols / BLK;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t t = 0; t < n; t++) {
      for (int64_t b = 0; b < blocks; b++) {
        const void* blk = q4 ? (const void*)((const uint8_t*)qs + r * cols / 2 + b * 16)
                             : (const void*)((const int8_t*)qs + r * cols + b * BLK);
        int32_t d[4];
        lane_dots(blk, q4, xq + t * cols + b * BLK, d);
        dots[(t * rows + r) * blocks + b] = d[0] + d[1] + d[2] + d[3];
      }
    }
  }
}

/* The double-precision check of test/native_kernels_test.dart:146-180 and
 * bin/dianoia.dart's _nativeQ8Check: ref[t*rows+r] = sum_c w(r,c) * x(t,c)
 * and mag = sum_c |w(r,c) * x(t,c)|, with x the inputs as the kernel sees
 * them (dequantized int8 in mode 1, the floats in mode 0). */
void orc_reference_f64(int q4, const void* qs, const void* scales, const float* xs,
                       int64_t rows, int64_t cols, int64_t n, int64_t mode, double* ref,
                       double* mag) {
  const int64_t blocks = cols / BLK;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < n; t++) {
    int8_t xqb[BLK];
    float xsb;
    for (int64_t r = 0; r < rows; r++) {
      double s = 0.0, m = 0.0;
      for (int64_t b = 0; b < blocks; b++) {
        const float* xb = xs + t * cols + b * BLK;
        if (mode == 1) orc_quantize_q8(xb, xqb, &xsb, 1, BLK);
        const double sw =
            q4 ? (double)orc_half_to_float(((const uint16_t*)scales)[r * blocks + b])
               : (double)((const float*)scales)[r * blocks + b];
        for (int j = 0; j < BLK; j++) {
          const int w = q4 ? wq4((const uint8_t*)qs + r * cols / 2 + b * 16, j)
                           : wq8((const int8_t*)qs + r * cols + b * BLK, j);
          const double x = mode == 1 ? (double)xqb[j] * (double)xsb : (double)xb[j];
          const double d = sw * w * x;
          s += d;
          m += fabs(d);
        }
      }
      ref[t * rows + r] = s;
      mag[t * rows + r] = m;
    }
  }
}

/* ------------------------------------------------------------------ the
 * decode path's neighbours, as dianoia's CPU path computes them. Dart's
 * double is an IEEE binary64 and its Float32List stores round to nearest,
 * so these C doubles and (float) casts are the same operations. */

/* lib/src/ops.dart:12-31 rmsNorm, for each of `rows` rows (model.dart:939-944
 * _normRows): sumSquares += v * v left to right in double, r = 1 / sqrt(
 * sumSquares / n + eps) in double, out = (float)(x * r), then
 * out = (float)(weight * out). With accumulate, the result is added into out
 * in f32 afterwards (model.dart:946-950 _addInto). */
void orc_rms_norm(const float* x, const float* w, float* out, int64_t rows, int64_t cols, double eps,
                  int64_t accumulate) {
  for (int64_t t = 0; t < rows; t++) {
    const float* xr = x + t * cols;
    float* o = out + t * cols;
    double s = 0.0;
    for (int64_t j = 0; j < cols; j++) {
      const double v = xr[j];
      s += v * v;
    }
    const double r = 1 / sqrt(s / (double)cols + eps);
    for (int64_t j = 0; j < cols; j++) {
      float v = (float)((double)xr[j] * r);
      v = (float)((double)w[j] * (double)v);
      o[j] = accumulate ? o[j] + v : v;
    }
  }
}

/* lib/src/shard.dart:456-460: g[j] = (float)(g / (1 + exp(-g))) in double,
 * then g[j] = (float)(g[j] * u[j]). */
void orc_swiglu(float* g, const float* u, int64_t count) {
  for (int64_t j = 0; j < count; j++) {
    const double gd = g[j];
    const float s = (float)(gd / (1 + exp(-gd)));
    g[j] = (float)((double)s * (double)u[j]);
  }
}

/* shard.dart:548-557 + ops.dart:62-71: per (token, head) the head's hd values
 * normalised by orc_rms_norm's arithmetic with weights w, then Rope.apply with
 * the token's table [cos(hd/2), sin(hd/2)]: x1 * cos - x2 * sin and
 * x2 * cos + x1 * sin in double, stored to f32. Strides in floats. */
void orc_head_norm_rope(float* x, int64_t x_stride, const float* w, const float* rope,
                        int64_t rope_stride, int64_t heads, int64_t hd, int64_t n, double eps) {
  const int64_t pair = hd / 2;
  for (int64_t t = 0; t < n; t++) {
    const float* c = rope + t * rope_stride;
    for (int64_t h = 0; h < heads; h++) {
      float* v = x + t * x_stride + h * hd;
      orc_rms_norm(v, w, v, 1, hd, eps, 0);
      for (int64_t j = 0; j < pair; j++) {
        const double x1 = v[j], x2 = v[j + pair];
        v[j] = (float)(x1 * (double)c[j] - x2 * (double)c[pair + j]);
        v[j + pair] = (float)(x2 * (double)c[j] + x1 * (double)c[pair + j]);
      }
    }
  }
}

/* shard.dart:589-628: causal grouped-query attention in double. */
void orc_attention(const float* q, const float* keys, const float* values, const float* gate,
                   float* out, int64_t position, int64_t n, int64_t heads, int64_t kv_heads,
                   int64_t hd, int64_t window, double* scores) {
  const int64_t q_dim = heads * hd, kv_dim = kv_heads * hd, group = heads / kv_heads;
  const double scale = 1 / sqrt((double)hd);
  for (int64_t t = 0; t < n; t++) {
    const int64_t pos = position + t;
    const int64_t start = window > 0 && pos - window + 1 > 0 ? pos - window + 1 : 0;
    for (int64_t h = 0; h < heads; h++) {
      const int64_t qo = t * q_dim + h * hd, kvo = (h / group) * hd;
      double max = -INFINITY;
      for (int64_t s = start; s <= pos; s++) {
        double dot = 0.0;
        for (int64_t d = 0; d < hd; d++) dot += (double)q[qo + d] * (double)keys[s * kv_dim + kvo + d];
        const double score = dot * scale;
        scores[s] = score;
        if (score > max) max = score;
      }
      double sum = 0.0;
      for (int64_t s = start; s <= pos; s++) {
        const double e = exp(scores[s] - max);
        scores[s] = e;
        sum += e;
      }
      const double g = gate ? 1 / (1 + exp(-(double)gate[t * heads + h])) : 1.0;
      for (int64_t d = 0; d < hd; d++) {
        double acc = 0.0;
        for (int64_t s = start; s <= pos; s++) acc += scores[s] * (double)values[s * kv_dim + kvo + d];
        out[qo + d] = (float)(acc / sum);
        if (gate) out[qo + d] = (float)((double)out[qo + d] * g);
      }
    }
  }
}

/* shard.dart:476-516: z = B * X (f32), y = C * sum_s kernel[k-1-s] z[t-s]
 * (the sum in double, from 0.0, s = 0 first), history = the last k - 1 z. */
void orc_conv(const float* bcx, const float* weight, float* history, float* y, int64_t width,
              int64_t k, int64_t n, float* z) {
  for (int64_t t = 0; t < n; t++)
    for (int64_t ch = 0; ch < width; ch++)
      z[t * width + ch] = bcx[t * 3 * width + ch] * bcx[t * 3 * width + 2 * width + ch];
  for (int64_t t = 0; t < n; t++)
    for (int64_t ch = 0; ch < width; ch++) {
      double acc = 0.0;
      for (int64_t s = 0; s < k; s++) {
        const int64_t src = t - s;
        const float zz = src >= 0 ? z[src * width + ch] : history[(k - 1 + src) * width + ch];
        acc += (double)weight[ch * k + k - 1 - s] * (double)zz;
      }
      y[t * width + ch] = (float)((double)bcx[t * 3 * width + width + ch] * acc);
    }
  const int64_t keep = k - 1;
  if (n >= keep) {
    memcpy(history, z + (n - keep) * width, (size_t)(keep * width) * sizeof(float));
  } else {
    memmove(history, history + n * width, (size_t)((keep - n) * width) * sizeof(float));
    memcpy(history + (keep - n) * width, z, (size_t)(n * width) * sizeof(float));
  }
}

/* control_vector.dart:176-203: mode 0 adds v (f32); mode 1 subtracts
 * scale * dot * v, the dot and the update in double, stored to f32. */
void orc_steer(float* x, const float* v, int64_t rows, int64_t cols, int64_t mode, double scale) {
  for (int64_t t = 0; t < rows; t++) {
    float* r = x + t * cols;
    if (mode == 0) {
      for (int64_t j = 0; j < cols; j++) r[j] = r[j] + v[j];
      continue;
    }
    double dot = 0.0;
    for (int64_t j = 0; j < cols; j++) dot += (double)r[j] * (double)v[j];
    const double c = scale * dot;
    for (int64_t j = 0; j < cols; j++) r[j] = (float)((double)r[j] - c * (double)v[j]);
  }
}
