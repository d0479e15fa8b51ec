// dianoia's GPU-layer C-ABI (lab_gpu_*: the Vulkan layer in
// src/vulkan/lab_vulkan.c and the Metal one export it; Dart binds it in
// lib/src/gpu.dart:36-312), for the quantized products that GpuLinear and
// GpuForward encode: buffers the host reads and writes in place, one
// process-wide command buffer opened by lab_gpu_begin, products recorded by
// lab_gpu_enc_matmul_q8 / _q4 and submitted by lab_gpu_commit.
//
// On B200 a buffer is device memory plus a pinned host mirror, which is what
// lab_gpu_contents returns. The host may have written any mirror between two
// command buffers, so lab_gpu_commit first copies to the device the input
// ranges of the recorded products (minus what an earlier product of the same
// command buffer writes), runs the products (activations quantized to Q8_0
// per block, then the decode GEMV or the tensor-core GEMM, as dn_linear in
// mode 1) and copies every range a product wrote back to the mirror. A
// buffer used as a weight matrix is copied to the device once, at its first
// product: dianoia writes weights once, before their first use
// (GpuLinear.upload, gpu.dart:1293-1323, and the wrapped model file of
// GpuForward). A command buffer identical to the previous one (a decode loop)
// replays the CUDA graph captured for it.
//
// Inside a command buffer, a decode product whose input is (a 32-value
// aligned part of) the output of the earlier decode product that last wrote
// it reads that output as quantized activations (QA blocks: 32 int8 and
// their f32 scale per 32 values), which the earlier product's epilogue writes
// to an internal buffer beside its f32 outputs; host-written inputs are
// quantized once for all products that read them. QA blocks are exactly what
// quantizing the f32 values gives, so the results are the same; the products
// skip re-quantizing their input in every CTA.
//
// Errors: like the reference, the void functions report nothing;
// lab_gpu_commit returns 0 when a product's arguments or a CUDA call failed.
// Calls are serialized by one mutex (the reference's layer is single-encoder).
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <mutex>
#include <thread>
#include <vector>

#include "dianoia_b200.h"
#include "dn_launch.h"

namespace dn {
bool status_words(uint32_t** dev, volatile uint32_t** host);  // abi.cu
}

namespace {

constexpr int64_t kBlock = 32;  // values per Q4_0 / Q8_0 block

struct Buf {
  uint8_t* dev = nullptr;
  uint8_t* host = nullptr;  // pinned mirror: lab_gpu_contents (null: a device-only buffer)
  int64_t bytes = 0;
  bool live = false;
  bool weights_on_device = false;  // copied once, at its first use as a matrix
};

enum Kind : int { kMatmul = 0, kNorm = 1, kSwiglu = 2, kAdd = 3, kCopy, kSteer, kHeadNormRope, kConv,
                  kAttention };

// One recorded operation. Every kind writes f32 values token-major, n rows
// of `rows` values at byte y_off of buffer y, and reads n rows of `cols`
// values at x_off of buffer x:
//  * kMatmul: weights w (values at qs_off, scales at sc_off), [rows, cols];
//  * kNorm: RMSNorm of n rows of rows == cols values with the weights at
//    qs_off of buffer w, eps, and acc (added into the output, which it then
//    also reads);
//  * kSwiglu: g = y and u = x, both at offset 0, count = rows == cols, n = 1;
//    it also reads g. No weights (w = -1).
//  * kAdd: dst = y at y_off plus src = x at x_off, count = rows == cols,
//    n = 1; it also reads dst. No weights.
// The other kinds keep their own arguments (see their encode functions) and
// list their ranges in reads / all_writes:
//  * kCopy: src = x at x_off, dst = y at y_off, count = rows == cols, n = 1;
//  * kSteer: rows of x = y at y_off (n rows of cols), v = x at x_off,
//    e[0] mode, eps the scale;
//  * kHeadNormRope: x = y at y_off (n tokens, stride e[0] floats, rows heads
//    of cols = hd), weights w at qs_off, rope table x at x_off (stride e[1]);
//  * kConv: bcx = x, y = y (both at 0), weights w at qs_off, history e[0],
//    rows = width, cols = k, n tokens;
//  * kAttention: q = x, out = y (both at 0), keys e[0], values e[1], gate
//    e[2] (-1: none), rows = heads, cols = hd, n tokens, position e[3],
//    kv heads e[4], window e[5].
struct Op {
  int kind;
  bool q4;
  int64_t w, qs_off, sc_off, x, x_off, y, y_off, rows, cols, n;
  double eps;
  bool acc;
  int64_t e[6] = {};  // zero unless a kind above sets them
  bool operator==(const Op& o) const {
    return kind == o.kind && q4 == o.q4 && w == o.w && qs_off == o.qs_off && sc_off == o.sc_off &&
           x == o.x && x_off == o.x_off && y == o.y && y_off == o.y_off && rows == o.rows &&
           cols == o.cols && n == o.n && memcmp(&eps, &o.eps, sizeof eps) == 0 && acc == o.acc &&
           memcmp(e, o.e, sizeof e) == 0;
  }
};

struct Range {
  int64_t buf, lo, hi;  // bytes [lo, hi) of buffer `buf`
};

Range writes(const Op& o) { return Range{o.y, o.y_off, o.y_off + o.n * o.rows * 4}; }

bool overlap(const Range& a, const Range& b) { return a.buf == b.buf && a.lo < b.hi && b.lo < a.hi; }

// The extent in bytes of n rows of `width` floats `stride` floats apart.
int64_t strided(int64_t n, int64_t stride, int64_t width) { return n <= 0 ? 0 : ((n - 1) * stride + width) * 4; }

void reads(const Op& o, std::vector<Range>& r) {
  r.clear();
  switch (o.kind) {
    case kSteer:
      r.push_back(Range{o.x, o.x_off, o.x_off + o.cols * 4});
      r.push_back(Range{o.y, o.y_off, o.y_off + o.n * o.cols * 4});
      return;
    case kHeadNormRope:
      r.push_back(Range{o.y, o.y_off, o.y_off + strided(o.n, o.e[0], o.rows * o.cols)});
      r.push_back(Range{o.x, o.x_off, o.x_off + strided(o.n, o.e[1], o.cols)});
      return;
    case kConv:
      r.push_back(Range{o.x, 0, o.n * 3 * o.rows * 4});
      r.push_back(Range{o.e[0], 0, (o.cols - 1) * o.rows * 4});
      return;
    case kAttention: {
      const int64_t kv = (o.e[3] + o.n) * o.e[4] * o.cols * 4;
      r.push_back(Range{o.x, 0, o.n * o.rows * o.cols * 4});
      r.push_back(Range{o.e[0], 0, kv});
      r.push_back(Range{o.e[1], 0, kv});
      if (o.e[2] >= 0) r.push_back(Range{o.e[2], 0, o.n * o.rows * 4});
      return;
    }
    default:
      break;
  }
  r.push_back(Range{o.x, o.x_off, o.x_off + o.n * o.cols * 4});
  if (o.kind == kSwiglu || o.kind == kAdd || (o.kind == kNorm && o.acc)) r.push_back(writes(o));
}

// Every range an op writes (writes() is the first of them).
void all_writes(const Op& o, std::vector<Range>& w) {
  w.clear();
  switch (o.kind) {
    case kSteer: w.push_back(Range{o.y, o.y_off, o.y_off + o.n * o.cols * 4}); return;
    case kHeadNormRope: w.push_back(Range{o.y, o.y_off, o.y_off + strided(o.n, o.e[0], o.rows * o.cols)}); return;
    case kConv:
      w.push_back(Range{o.y, 0, o.n * o.rows * 4});
      w.push_back(Range{o.e[0], 0, (o.cols - 1) * o.rows * 4});
      return;
    case kAttention: w.push_back(Range{o.y, 0, o.n * o.rows * o.cols * 4}); return;
    default: w.push_back(writes(o));
  }
}

// The buffers an op uses (for the graph's identity and releases).
void op_handles(const Op& o, std::vector<int64_t>& h) {
  h.clear();
  h.push_back(o.w);
  h.push_back(o.x);
  h.push_back(o.y);
  if (o.kind == kConv) h.push_back(o.e[0]);
  if (o.kind == kAttention) {
    h.push_back(o.e[0]);
    h.push_back(o.e[1]);
    h.push_back(o.e[2]);
  }
}

std::recursive_mutex g_mu;
bool g_ready = false;
int g_device = -1;
cudaStream_t g_stream = nullptr;
cudaEvent_t g_ev0 = nullptr, g_ev1 = nullptr;
std::vector<Buf> g_bufs;
std::vector<int64_t> g_free;
int64_t g_live = 0;
std::vector<Op> g_ops;
bool g_bad_op = false;  // an encode call got handles or ranges that do not fit
bool g_pending = false;
double g_last_ms = 0.0;

// Scratch of the tensor-core path: the quantized activations.
int8_t* g_xq = nullptr;
float* g_xsc = nullptr;
int64_t g_xcap = 0;

// QA blocks of the products whose outputs a later product reads.
uint8_t* g_qa = nullptr;
int64_t g_qa_cap = 0;

// Fusions and QA links on (dn_gpu_set_fusion); off, every op runs as its own
// kernel on f32 inputs, as the reference's layer dispatches them.
bool g_fuse = true;

// lab_gpu_set_decode_rows(0): decode products on the generic kernel, a
// same-device numerical reference (as the reference's old int8 GEMM is).
bool g_generic = false;

// Dispatch profiling (lab_gpu_set_profiling / lab_gpu_profile): the kinds, in
// the reference's order (lab_vulkan.c:174-177), and per kind the GPU time and
// dispatches since the last lab_gpu_profile. A profiled command buffer
// records an event after its uploads and after each launch; a launch's share
// runs from the event before it to its own.
enum ProfKind : int {
  kProfGemvQ8, kProfGemmQ8, kProfGemvQ4, kProfGemmQ4, kProfRmsNorm, kProfHeadNormRope, kProfConv,
  kProfAttention, kProfSwiglu, kProfCopy, kProfQuantize, kProfGemmQ8I8, kProfGemmQ4I8,
  kProfGemvQ8I8, kProfGemvQ4I8, kProfGemvQ8I8Vec, kProfSteer, kProfAdd, kProfKinds
};
bool g_profiling = false;
double g_kind_ms[kProfKinds] = {};
int64_t g_kind_count[kProfKinds] = {};
std::vector<cudaEvent_t> g_prof_events;
std::vector<int> g_prof_kinds;  // of the graph's launches, in order

// The graph of the last command buffer, with what it was captured from.
cudaGraphExec_t g_exec = nullptr;
bool g_exec_fuse = true;
bool g_exec_generic = false;
bool g_exec_prof = false;
std::vector<Op> g_exec_ops;
std::vector<uint8_t*> g_exec_ptrs;  // device addresses the graph uses, per op (w, x, y)
int8_t* g_exec_xq = nullptr;
uint8_t* g_exec_qa = nullptr;

void drop_graph() {
  if (g_exec != nullptr) cudaGraphExecDestroy(g_exec);
  g_exec = nullptr;
  g_exec_ops.clear();
  g_exec_ptrs.clear();
}

bool wait_pending() {
  if (!g_pending) return true;
  g_pending = false;
  if (cudaStreamSynchronize(g_stream) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  float ms = 0.0f;
  if (cudaEventElapsedTime(&ms, g_ev0, g_ev1) == cudaSuccess) g_last_ms = ms;
  if (g_exec_prof) {
    for (size_t i = 0; i < g_prof_kinds.size(); i++) {
      if (cudaEventElapsedTime(&ms, g_prof_events[i], g_prof_events[i + 1]) != cudaSuccess) {
        cudaGetLastError();  // not sticky: keep it from a later launch's check
        continue;
      }
      g_kind_ms[g_prof_kinds[i]] += ms;
      g_kind_count[g_prof_kinds[i]]++;
    }
  }
  uint32_t* sd = nullptr;
  volatile uint32_t* sh = nullptr;
  if (dn::status_words(&sd, &sh) && *sh != 0) return false;  // a bounded wait ran out
  return true;
}

bool valid(int64_t h) { return h >= 0 && h < (int64_t)g_bufs.size() && g_bufs[h].live; }

bool fits(int64_t h, int64_t off, int64_t bytes) {
  return valid(h) && off >= 0 && bytes >= 0 && off <= g_bufs[h].bytes - bytes;
}

int64_t add_buffer(const Buf& b) {
  int64_t h;
  if (!g_free.empty()) {
    h = g_free.back();
    g_free.pop_back();
    g_bufs[h] = b;
  } else {
    h = (int64_t)g_bufs.size();
    g_bufs.push_back(b);
  }
  g_live++;
  return h;
}

int64_t new_buffer(int64_t bytes) {
  if (!g_ready || bytes < 0) return -1;
  cudaSetDevice(g_device);
  const size_t n = bytes == 0 ? 16 : (size_t)bytes;
  Buf b;
  if (cudaMalloc(&b.dev, n) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (cudaHostAlloc(&b.host, n, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(b.dev);
    return -1;
  }
  memset(b.host, 0, n);
  if (cudaMemset(b.dev, 0, n) != cudaSuccess) {
    cudaGetLastError();
    cudaFreeHost(b.host);
    cudaFree(b.dev);
    return -1;
  }
  b.bytes = bytes;
  b.live = true;
  return add_buffer(b);
}

constexpr int64_t kMaxSide = int64_t(1) << 30;  // keeps every byte count below 2^63

bool sides_ok(int64_t a, int64_t b) { return a >= 0 && b >= 0 && a < kMaxSide && b < kMaxSide; }

// Copies `bytes` bytes at file offset `offset` to device memory at `dev`
// through two pinned staging chunks: the read of one chunk runs while the
// other is copied to the device. Returns false on a short read or CUDA error.
bool read_slice(int fd, int64_t offset, int64_t bytes, uint8_t* dev) {
  constexpr int64_t kChunk = int64_t(16) << 20;
  uint8_t* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaStream_t copy = nullptr;
  bool ok = cudaStreamCreateWithFlags(&copy, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; i < 2 && ok; i++)
    ok = cudaHostAlloc(&stage[i], (size_t)std::min(kChunk, std::max<int64_t>(bytes, 16)),
                       cudaHostAllocDefault) == cudaSuccess &&
         cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) == cudaSuccess;
  for (int64_t at = 0, k = 0; ok && at < bytes; at += kChunk, k++) {
    const int i = (int)(k & 1);
    const int64_t n = std::min(kChunk, bytes - at);
    if (k >= 2) ok = cudaEventSynchronize(done[i]) == cudaSuccess;  // its previous copy is done
    for (int64_t got = 0; ok && got < n;) {
      const ssize_t r = pread(fd, stage[i] + got, (size_t)(n - got), (off_t)(offset + at + got));
      if (r <= 0) ok = false;
      else got += r;
    }
    ok = ok && cudaMemcpyAsync(dev + at, stage[i], (size_t)n, cudaMemcpyHostToDevice, copy) == cudaSuccess &&
         cudaEventRecord(done[i], copy) == cudaSuccess;
  }
  if (copy != nullptr) ok = cudaStreamSynchronize(copy) == cudaSuccess && ok;
  for (int i = 0; i < 2; i++) {
    if (done[i] != nullptr) cudaEventDestroy(done[i]);
    if (stage[i] != nullptr) cudaFreeHost(stage[i]);
  }
  if (copy != nullptr) cudaStreamDestroy(copy);
  return ok;
}

// Reads [offset, offset + bytes) of the file at `path` into a new device-only
// buffer: contiguous slices of at least 64 MiB, one per host thread (up to
// 8), each through its own staging (a single reader is bound near 7.5 GB/s
// by copying out of the page cache). Returns the handle, or -1.
int64_t wrap_file(const char* path, int64_t offset, int64_t bytes) {
  if (!g_ready || path == nullptr || offset < 0 || bytes < 0) return -1;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return -1;
  struct stat st;
  if (fstat(fd, &st) != 0 || offset > (int64_t)st.st_size - bytes) {
    close(fd);
    return -1;
  }
  cudaSetDevice(g_device);
  Buf b;
  if (cudaMalloc(&b.dev, (size_t)(bytes == 0 ? 16 : bytes)) != cudaSuccess) {
    cudaGetLastError();
    close(fd);
    return -1;
  }
  constexpr int64_t kMinSlice = int64_t(64) << 20;
  const int64_t hw = std::max<int64_t>(1, (int64_t)std::thread::hardware_concurrency());
  const int64_t threads = std::max<int64_t>(1, std::min({int64_t(8), hw, bytes / kMinSlice}));
  const int64_t slice = (bytes + threads - 1) / threads;
  std::vector<char> ok((size_t)threads, 0);
  std::vector<std::thread> pool;
  const int device = g_device;
  for (int64_t t = 0; t < threads; t++) {
    const int64_t lo = std::min(bytes, t * slice), hi = std::min(bytes, lo + slice);
    pool.emplace_back([&, t, lo, hi] {
      cudaSetDevice(device);
      ok[(size_t)t] = read_slice(fd, offset + lo, hi - lo, b.dev + lo) ? 1 : 0;
    });
  }
  for (std::thread& th : pool) th.join();
  close(fd);
  if (std::find(ok.begin(), ok.end(), 0) != ok.end()) {
    cudaGetLastError();
    cudaFree(b.dev);
    return -1;
  }
  b.bytes = bytes;
  b.live = true;
  b.weights_on_device = true;
  return add_buffer(b);
}

void encode(bool q4, int64_t w, int64_t qs_off, int64_t sc_off, int64_t x, int64_t x_off, int64_t y,
            int64_t y_off, int64_t rows, int64_t cols, int64_t n) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  // f32 activations and scales at their natural alignment: the kernels load
  // them as such.
  const bool ok = sides_ok(rows, cols) && sides_ok(n, 0) && cols % kBlock == 0 &&
                  x_off % 4 == 0 && y_off % 4 == 0 && sc_off % (q4 ? 2 : 4) == 0 &&
                  fits(w, qs_off, q4 ? rows * cols / 2 : rows * cols) &&
                  fits(w, sc_off, rows * (cols / kBlock) * (q4 ? 2 : 4)) &&
                  fits(x, x_off, n * cols * 4) && fits(y, y_off, n * rows * 4);
  if (!ok) {
    g_bad_op = true;
    return;
  }
  g_ops.push_back(Op{kMatmul, q4, w, qs_off, sc_off, x, x_off, y, y_off, rows, cols, n, 0.0, false});
}

void encode_norm(int64_t x, int64_t x_off, int64_t w, int64_t w_off, int64_t out, int64_t out_off,
                 int64_t rows, int64_t cols, double eps, int64_t accumulate) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  const bool ok = sides_ok(rows, cols) && x_off % 4 == 0 && w_off % 4 == 0 && out_off % 4 == 0 &&
                  fits(x, x_off, rows * cols * 4) && fits(w, w_off, cols * 4) &&
                  fits(out, out_off, rows * cols * 4);
  if (!ok) {
    g_bad_op = true;
    return;
  }
  g_ops.push_back(Op{kNorm, false, w, w_off, 0, x, x_off, out, out_off, cols, cols, rows, eps,
                     accumulate != 0});
}

void encode_add(int64_t src, int64_t src_off, int64_t dst, int64_t dst_off, int64_t count) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  if (!sides_ok(count, 0) || src_off % 4 != 0 || dst_off % 4 != 0 || !fits(src, src_off, count * 4) ||
      !fits(dst, dst_off, count * 4)) {
    g_bad_op = true;
    return;
  }
  g_ops.push_back(Op{kAdd, false, -1, 0, 0, src, src_off, dst, dst_off, count, count, 1, 0.0, false});
}

void encode_copy(int64_t src, int64_t src_off, int64_t dst, int64_t dst_off, int64_t count) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  if (!sides_ok(count, 0) || src_off % 4 != 0 || dst_off % 4 != 0 || !fits(src, src_off, count * 4) ||
      !fits(dst, dst_off, count * 4)) {
    g_bad_op = true;
    return;
  }
  g_ops.push_back(Op{kCopy, false, -1, 0, 0, src, src_off, dst, dst_off, count, count, 1, 0.0, false});
}

void encode_steer(int64_t x, int64_t x_off, int64_t v, int64_t v_off, int64_t rows, int64_t cols,
                  int64_t mode, double scale) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  if (!sides_ok(rows, cols) || (mode != 0 && mode != 1) || x_off % 4 != 0 || v_off % 4 != 0 ||
      !fits(x, x_off, rows * cols * 4) || !fits(v, v_off, cols * 4)) {
    g_bad_op = true;
    return;
  }
  Op o{kSteer, false, -1, 0, 0, v, v_off, x, x_off, cols, cols, rows, scale, false};
  o.e[0] = mode;
  g_ops.push_back(o);
}

void encode_head_norm_rope(int64_t x, int64_t x_off, int64_t x_stride, int64_t w, int64_t w_off,
                           int64_t rope, int64_t rope_off, int64_t rope_stride, int64_t heads,
                           int64_t hd, int64_t n, double eps) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  const bool ok = sides_ok(heads, n) && n <= 65535 && hd > 0 && hd % 2 == 0 && hd <= 256 &&
                  x_stride >= heads * hd && rope_stride >= hd && x_off % 4 == 0 && w_off % 4 == 0 &&
                  rope_off % 4 == 0 && x_stride < kMaxSide && rope_stride < kMaxSide &&
                  fits(x, x_off, strided(n, x_stride, heads * hd)) && fits(w, w_off, hd * 4) &&
                  fits(rope, rope_off, strided(n, rope_stride, hd));
  if (!ok) {
    g_bad_op = true;
    return;
  }
  Op o{kHeadNormRope, false, w, w_off, 0, rope, rope_off, x, x_off, heads, hd, n, eps, false};
  o.e[0] = x_stride;
  o.e[1] = rope_stride;
  g_ops.push_back(o);
}

void encode_conv(int64_t bcx, int64_t weight, int64_t weight_off, int64_t history, int64_t y,
                 int64_t width, int64_t k, int64_t n) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  const bool ok = sides_ok(width, n) && k >= 1 && k <= dn::kMaxConvTaps && weight_off % 4 == 0 &&
                  fits(bcx, 0, n * 3 * width * 4) && fits(weight, weight_off, width * k * 4) &&
                  fits(history, 0, (k - 1) * width * 4) && fits(y, 0, n * width * 4);
  if (!ok) {
    g_bad_op = true;
    return;
  }
  Op o{kConv, false, weight, weight_off, 0, bcx, 0, y, 0, width, k, n, 0.0, false};
  o.e[0] = history;
  g_ops.push_back(o);
}

void encode_attention(int64_t q, int64_t keys, int64_t values, int64_t gate, int64_t out,
                      int64_t position, int64_t n, int64_t heads, int64_t kv_heads, int64_t hd,
                      int64_t window) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  const int64_t longest = window > 0 ? std::min(window, position + n) : position + n;
  const int64_t kv = (position + n) * kv_heads * hd * 4;
  // hd: a multiple of 4 up to 256 (the kernel loads values four at a time).
  const bool ok = sides_ok(heads, n) && n <= 65535 && kv_heads > 0 && hd > 0 && hd <= 256 && hd % 4 == 0 &&
                  heads % kv_heads == 0 && position >= 0 && position < kMaxSide && window >= 0 &&
                  longest <= dn::kMaxAttnKeys && fits(q, 0, n * heads * hd * 4) && fits(keys, 0, kv) &&
                  fits(values, 0, kv) && (gate < 0 || fits(gate, 0, n * heads * 4)) &&
                  fits(out, 0, n * heads * hd * 4);
  if (!ok) {
    g_bad_op = true;
    return;
  }
  Op o{kAttention, false, -1, 0, 0, q, 0, out, 0, heads, hd, n, 0.0, false};
  o.e[0] = keys;
  o.e[1] = values;
  o.e[2] = gate < 0 ? -1 : gate;
  o.e[3] = position;
  o.e[4] = kv_heads;
  o.e[5] = window;
  g_ops.push_back(o);
}

void encode_swiglu(int64_t g, int64_t u, int64_t count) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  if (!sides_ok(count, 0) || !fits(g, 0, count * 4) || !fits(u, 0, count * 4)) {
    g_bad_op = true;
    return;
  }
  g_ops.push_back(Op{kSwiglu, false, -1, 0, 0, u, 0, g, 0, count, count, 1, 0.0, false});
}

// Adds [lo, hi) of buffer b to a list of ranges, merging overlaps.
void add_range(std::vector<Range>& v, int64_t b, int64_t lo, int64_t hi) {
  if (lo >= hi) return;
  for (Range& r : v) {
    if (r.buf == b && lo <= r.hi && r.lo <= hi) {
      r.lo = std::min(r.lo, lo);
      r.hi = std::max(r.hi, hi);
      // merging may now touch a neighbour: restart with the merged range
      const Range m = r;
      r = v.back();
      v.pop_back();
      add_range(v, m.buf, m.lo, m.hi);
      return;
    }
  }
  v.push_back(Range{b, lo, hi});
}

// The parts of [lo, hi) of buffer b not covered by `written`.
void subtract(const std::vector<Range>& written, int64_t b, int64_t lo, int64_t hi,
              std::vector<Range>& out) {
  std::vector<std::pair<int64_t, int64_t>> cover;
  for (const Range& r : written)
    if (r.buf == b && r.lo < hi && lo < r.hi) cover.push_back({std::max(r.lo, lo), std::min(r.hi, hi)});
  std::sort(cover.begin(), cover.end());
  int64_t at = lo;
  for (auto& c : cover) {
    if (c.first > at) add_range(out, b, at, c.first);
    at = std::max(at, c.second);
  }
  if (at < hi) add_range(out, b, at, hi);
}

// Removes bytes [lo, hi) of buffer b from the ranges v.
void remove_range(std::vector<Range>& v, int64_t b, int64_t lo, int64_t hi) {
  std::vector<Range> out;
  for (const Range& r : v) {
    if (r.buf != b || r.hi <= lo || hi <= r.lo) {
      out.push_back(r);
      continue;
    }
    if (r.lo < lo) out.push_back(Range{b, r.lo, lo});
    if (hi < r.hi) out.push_back(Range{b, hi, r.hi});
  }
  v.swap(out);
}

// Records the command buffer's copies and products on g_stream.
dn::LinearArgs linear_args(const Op& o, uint32_t* status) {
  const Buf &w = g_bufs[o.w], &x = g_bufs[o.x], &y = g_bufs[o.y];
  return dn::LinearArgs{o.q4, w.dev + o.qs_off, w.dev + o.sc_off,
                        reinterpret_cast<const float*>(x.dev + o.x_off), g_xq, g_xsc,
                        reinterpret_cast<float*>(y.dev + o.y_off), o.rows, o.cols, o.n, o.rows,
                        1, status};
}

// How the recorded ops run: fusions and QA links (decode GEMV path only).
//
// SwiGLU fusion: a SwiGLU op right after the two products that wrote its g
// and u (the feed-forward's gate and up, in either order, same tokens and
// rows) runs in the second product's epilogue (glu[i]), and launches nothing
// itself (absorbed). Residual-add fusion: an add right after the product
// that wrote all of its src, into a dst the product does not read, runs in
// that product's epilogue (res[i]) and is absorbed too. Norm fusion: a norm
// (without accumulate) whose output only GEMV products read, each all of it
// (same tokens and width), before anything writes the norm's input, weights
// or output again, runs in the prologue of the first of them (normin[i]: it
// reads the norm's input as f32 and normalizes it in the CTA), which also
// writes the norm's outputs and, when more products read them, their QA
// blocks (xa_out_at[i]) for those products' QA links; the norm is absorbed.
//
// QA links: every op that writes 32-value rows can also write them as QA
// blocks (the GEMV epilogue, the norm and SwiGLU kernels); with rows a
// multiple of 32, its QA blocks lie in the order of its values, block v/32 of
// value v of the written range, whatever the token split. Product i reads its
// input as QA blocks at byte xa_at[i] of g_qa (row stride xa_stride[i]) when
// the input is either
//  * a 32-value-aligned part of the range of the last op that wrote over it,
//    which then also writes its values as QA blocks, at ya_at[j] (a SwiGLU
//    run by a product: that product's QA outputs); or
//  * host data no earlier op wrote: quantized once, before the ops, for
//    every product that reads the same range.
struct HostQA {
  int64_t buf, off, n, cols, at;
};
struct Plan {
  std::vector<int64_t> xa_at, xa_stride, ya_at;
  std::vector<int> glu;         // product i runs SwiGLU op glu[i] in its epilogue, or -1
  std::vector<int> res;         // product i runs add op res[i] in its epilogue, or -1
  std::vector<int> dual;        // product i also runs product dual[i] and their SwiGLU, or -1
  std::vector<int> grp;         // product i runs itself and the grp[i] - 1 products after it (0: none)
  std::vector<int> hnr2;        // head norm i also runs head norm hnr2[i] (the next op), or -1
  std::vector<int> runs_in;     // an absorbed op: the op whose launch runs it
  std::vector<int> normin;      // product i runs norm op normin[i] in its prologue, or -1
  std::vector<int64_t> xa_out_at;  // product i writes its quantized input as QA blocks there, or -1
  std::vector<bool> absorbed;   // a SwiGLU op that a product's epilogue runs
  std::vector<HostQA> host;
  int64_t bytes = 0;
};

int64_t qa_bytes(int64_t n, int64_t values) { return (n * (values / kBlock) * dn::kQABytes + 15) / 16 * 16; }

Plan plan_ops(uint32_t* status) {
  const int n = (int)g_ops.size();
  Plan k;
  k.xa_at.assign(n, -1);
  k.xa_stride.assign(n, 0);
  k.ya_at.assign(n, -1);
  k.glu.assign(n, -1);
  k.res.assign(n, -1);
  k.dual.assign(n, -1);
  k.grp.assign(n, 0);
  k.hnr2.assign(n, -1);
  k.runs_in.assign(n, -1);
  k.normin.assign(n, -1);
  k.xa_out_at.assign(n, -1);
  k.absorbed.assign(n, false);
  if (!g_fuse) return k;
  std::vector<bool> gemv(n, false);
  for (int i = 0; i < n; i++)
    gemv[i] = g_ops[i].kind == kMatmul && !g_generic && dn::path_for(linear_args(g_ops[i], status)) == 0;
  for (int i = 2; i < n; i++) {
    const Op &s = g_ops[i], &a = g_ops[i - 2], &b = g_ops[i - 1];
    if (s.kind != kSwiglu || !gemv[i - 2] || !gemv[i - 1] || s.x == s.y) continue;
    const bool pair = (a.y == s.y && b.y == s.x) || (a.y == s.x && b.y == s.y);
    if (!(pair && a.n == b.n && a.rows == b.rows && a.n * a.rows == s.rows && a.y_off == 0 &&
          b.y_off == 0 && b.x != s.x && b.x != s.y))
      continue;
    if (a.n == 1 && a.cols == b.cols && a.q4 == b.q4 && a.x == b.x && a.x_off == b.x_off) {
      // One token over one input: both products in one dual launch.
      k.dual[i - 2] = i - 1;
      k.absorbed[i - 1] = k.absorbed[i] = true;
      k.runs_in[i - 1] = k.runs_in[i] = i - 2;
    } else {
      k.glu[i - 1] = i;
      k.absorbed[i] = true;
      k.runs_in[i] = i - 1;
    }
  }
  for (int i = 1; i < n; i++) {
    const Op &d = g_ops[i], &p = g_ops[i - 1];
    if (d.kind != kAdd || !gemv[i - 1] || k.glu[i - 1] >= 0 || k.absorbed[i - 1]) continue;
    const Range src{d.x, d.x_off, d.x_off + d.rows * 4}, dst = writes(d), out = writes(p);
    const Range in{p.x, p.x_off, p.x_off + p.n * p.cols * 4};
    if (out.buf == src.buf && out.lo == src.lo && out.hi == src.hi && !overlap(dst, in) && !overlap(dst, out)) {
      k.res[i - 1] = i;
      k.absorbed[i] = true;
      k.runs_in[i] = i - 1;
    }
  }
  // Grouped launches: consecutive one-token GEMV products of the same input
  // (GpuForward's q, k and v), with nothing else fused into them and outputs
  // that neither overlap each other nor the input, run as one launch over all
  // their tiles; the first launches, the others are absorbed.
  for (int i = 0; i < n;) {
    auto plain = [&](int j) {
      const Op& o = g_ops[j];
      return gemv[j] && o.n == 1 && !k.absorbed[j] && k.glu[j] < 0 && k.dual[j] < 0 && k.res[j] < 0;
    };
    if (!plain(i)) {
      i++;
      continue;
    }
    const Op& f = g_ops[i];
    const Range in{f.x, f.x_off, f.x_off + f.cols * 4};
    std::vector<Range> outs{writes(f)};
    int m = 1;
    while (m < dn::kMaxGroups && i + m < n && plain(i + m)) {
      const Op& o = g_ops[i + m];
      if (o.x != f.x || o.x_off != f.x_off || o.cols != f.cols || o.q4 != f.q4) break;
      const Range w = writes(o);
      bool clash = overlap(w, in) || overlap(outs[0], in);
      for (const Range& r : outs) clash = clash || overlap(r, w);
      if (clash) break;
      outs.push_back(w);
      m++;
    }
    if (m >= 2) {
      k.grp[i] = m;
      for (int j = 1; j < m; j++) {
        k.absorbed[i + j] = true;
        k.runs_in[i + j] = i;
      }
    }
    i += m;
  }
  // Two consecutive head norms with one table and shape (GpuForward's q, then
  // k in its cache row) whose ranges do not overlap: one launch.
  for (int i = 0; i + 1 < n; i++) {
    const Op &p = g_ops[i], &q = g_ops[i + 1];
    if (p.kind != kHeadNormRope || q.kind != kHeadNormRope || k.absorbed[i] || k.hnr2[i] >= 0) continue;
    if (p.x != q.x || p.x_off != q.x_off || p.e[1] != q.e[1] || p.cols != q.cols || p.n != q.n ||
        memcmp(&p.eps, &q.eps, sizeof p.eps) != 0)
      continue;
    std::vector<Range> wp, wq;
    all_writes(p, wp);
    all_writes(q, wq);
    if (overlap(wp[0], wq[0])) continue;
    k.hnr2[i] = i + 1;
    k.absorbed[i + 1] = true;
    k.runs_in[i + 1] = i;
  }
  // Everything op i's launch writes: its own outputs and those of the ops it absorbed.
  auto launch_writes = [&](int i, std::vector<Range>& w) {
    all_writes(g_ops[i], w);
    for (int j = 1; j < k.grp[i]; j++) w.push_back(writes(g_ops[i + j]));
    if (k.hnr2[i] >= 0) {
      std::vector<Range> w2;
      all_writes(g_ops[k.hnr2[i]], w2);
      w.insert(w.end(), w2.begin(), w2.end());
    }
    if (k.glu[i] >= 0) w.push_back(writes(g_ops[k.glu[i]]));
    if (k.dual[i] >= 0) w.push_back(writes(g_ops[k.dual[i]]));
    if (k.res[i] >= 0) w.push_back(writes(g_ops[k.res[i]]));
  };
  std::vector<Range> in, wr;
  for (int j = 0; j < n; j++) {
    const Op& m = g_ops[j];
    // f32 inputs and the weights come into the products by bulk copies.
    if (m.kind != kNorm || m.acc || m.x_off % 16 != 0 || m.qs_off % 16 != 0) continue;
    const Range out = writes(m), src{m.x, m.x_off, m.x_off + m.n * m.cols * 4};
    const Range wts{m.w, m.qs_off, m.qs_off + m.cols * 4};
    std::vector<int> readers;
    bool ok = true;
    for (int i = j + 1; i < n && ok; i++) {
      reads(g_ops[i], in);
      bool reads_out = false;
      for (const Range& r : in) reads_out = reads_out || overlap(r, out);
      if (k.absorbed[i]) {  // runs inside its product, whose writes were seen there
        // The second product of a dual launch reads what the first does.
        const bool dual_partner = g_ops[i].kind == kMatmul && k.runs_in[i] >= 0;
        ok = ok && (dual_partner || !reads_out);
        continue;
      }
      launch_writes(i, wr);
      bool ends = false;
      for (const Range& w : wr) ends = ends || overlap(w, out) || overlap(w, src) || overlap(w, wts);
      if (reads_out) {
        // A reader must take all of the norm's rows as its input and must not
        // write what its own prologue reads, nor the norm's outputs.
        const Op& c = g_ops[i];
        ok = gemv[i] && c.x == out.buf && c.x_off == out.lo && c.n == m.n && c.cols == m.rows && !ends;
        readers.push_back(i);
      }
      if (ends) break;
    }
    if (!ok || readers.empty()) continue;
    k.normin[readers[0]] = j;
    k.absorbed[j] = true;
    if (readers.size() > 1) {
      const int64_t at = k.bytes;
      k.bytes += qa_bytes(m.n, m.rows);
      k.xa_out_at[readers[0]] = at;
      for (size_t r = 1; r < readers.size(); r++) {
        k.xa_at[readers[r]] = at;
        k.xa_stride[readers[r]] = m.rows / kBlock * dn::kQABytes;
      }
    }
  }
  // The op whose launch writes the QA blocks of op j's values, or -1.
  std::vector<int> qa_src(n, -1);
  for (int j = 0; j < n; j++) {
    const Op& o = g_ops[j];
    if (o.rows % kBlock != 0) continue;
    // (a product running a SwiGLU writes the SwiGLU's QA blocks, not its own)
    if (o.kind == kMatmul)
      qa_src[j] = gemv[j] && k.glu[j] < 0 && k.dual[j] < 0 && k.grp[j] < 2 && !k.absorbed[j] ? j : -1;
    else if (o.kind == kSwiglu && k.absorbed[j])
      qa_src[j] = g_ops[k.runs_in[j]].rows % kBlock == 0 ? k.runs_in[j] : -1;
    else if ((o.kind == kNorm || o.kind == kSwiglu) && !k.absorbed[j]) qa_src[j] = j;
  }
  for (int i = 0; i < n; i++) {
    const Op& c = g_ops[i];
    if (!gemv[i] || c.cols % kBlock != 0 || k.normin[i] >= 0 || k.xa_at[i] >= 0 || k.absorbed[i]) continue;
    const int64_t lo = c.x_off, hi = c.x_off + c.n * c.cols * 4;
    int j = i - 1;
    std::vector<Range> ws;
    for (; j >= 0; j--) {
      all_writes(g_ops[j], ws);
      bool hit = false;
      for (const Range& w : ws) hit = hit || (w.buf == c.x && w.lo < hi && lo < w.hi);
      if (hit) break;
    }
    if (j >= 0) {
      const Range w = writes(g_ops[j]);  // QA blocks come only from single-range writers
      const int64_t delta = lo - w.lo;
      const int src = qa_src[j];
      if (src < 0 || delta < 0 || hi > w.hi || delta % (kBlock * 4) != 0) continue;
      if (k.ya_at[src] < 0) {
        k.ya_at[src] = k.bytes;
        k.bytes += qa_bytes(g_ops[src].n, g_ops[src].rows);
      }
      k.xa_at[i] = k.ya_at[src] + delta / (kBlock * 4) * dn::kQABytes;
      k.xa_stride[i] = c.cols / kBlock * dn::kQABytes;
    } else {
      size_t h = 0;
      for (; h < k.host.size(); h++) {
        const HostQA& q = k.host[h];
        if (q.buf == c.x && q.off == lo && q.n == c.n && q.cols == c.cols) break;
      }
      if (h == k.host.size()) {
        k.host.push_back(HostQA{c.x, lo, c.n, c.cols, k.bytes});
        k.bytes += qa_bytes(c.n, c.cols);
      }
      k.xa_at[i] = k.host[h].at;
      k.xa_stride[i] = c.cols / kBlock * dn::kQABytes;
    }
  }
  return k;
}

float* f32_at(int64_t buf, int64_t off) { return reinterpret_cast<float*>(g_bufs[buf].dev + off); }

bool record(const std::vector<Range>& uploads, const std::vector<Range>& downloads,
            const Plan& k, uint32_t* status, int zc_op, float* zc_ys) {
  // With profiling, an event node after the uploads and after every launch
  // (external records: timestamps in the graph), and launches without
  // programmatic dependent launch, so that each one's share is its own.
  g_prof_kinds.clear();
  size_t ev = 0;
  const bool pdl = !g_profiling;
  auto mark = [&](int kind) {
    if (!g_profiling) return true;
    if (kind >= 0) g_prof_kinds.push_back(kind);
    return cudaEventRecordWithFlags(g_prof_events[ev++], g_stream, cudaEventRecordExternal) == cudaSuccess;
  };
  for (const Range& r : uploads) {
    const Buf& b = g_bufs[r.buf];
    if (b.host == nullptr) continue;  // device-only: nothing on the host to copy
    if (cudaMemcpyAsync(b.dev + r.lo, b.host + r.lo, (size_t)(r.hi - r.lo), cudaMemcpyHostToDevice,
                        g_stream) != cudaSuccess)
      return false;
  }
  if (!mark(-1)) return false;
  for (const HostQA& q : k.host) {
    if (dn::launch_quantize_qa(reinterpret_cast<const float*>(g_bufs[q.buf].dev + q.off), g_qa + q.at,
                               q.n, q.cols, q.cols / kBlock * dn::kQABytes, g_stream) != cudaSuccess ||
        !mark(kProfQuantize))
      return false;
  }
  for (size_t i = 0; i < g_ops.size(); i++) {
    const Op& o = g_ops[i];
    uint8_t* qa_out = k.ya_at[i] >= 0 ? g_qa + k.ya_at[i] : nullptr;
    if (o.kind == kNorm) {
      if (k.absorbed[i]) continue;
      const dn::NormArgs na{f32_at(o.x, o.x_off), f32_at(o.w, o.qs_off), f32_at(o.y, o.y_off), qa_out,
                            o.rows / kBlock * dn::kQABytes, o.n, o.rows, o.eps, o.acc};
      if (dn::launch_rms_norm(na, g_stream, pdl) != cudaSuccess || !mark(kProfRmsNorm)) return false;
      continue;
    }
    if (o.kind == kAdd) {
      if (k.absorbed[i]) continue;
      if (dn::launch_add(f32_at(o.x, o.x_off), f32_at(o.y, o.y_off), o.rows, g_stream, pdl) != cudaSuccess ||
          !mark(kProfAdd))
        return false;
      continue;
    }
    if (o.kind == kSwiglu) {
      if (k.absorbed[i]) continue;
      const dn::SwigluArgs sa{f32_at(o.y, 0), f32_at(o.x, 0), qa_out, o.rows};
      if (dn::launch_swiglu(sa, g_stream, pdl) != cudaSuccess || !mark(kProfSwiglu)) return false;
      continue;
    }
    if (o.kind == kCopy) {
      if (dn::launch_copy(f32_at(o.x, o.x_off), f32_at(o.y, o.y_off), o.rows, g_stream, pdl) != cudaSuccess ||
          !mark(kProfCopy))
        return false;
      continue;
    }
    if (o.kind == kSteer) {
      const dn::SteerArgs sa{f32_at(o.y, o.y_off), f32_at(o.x, o.x_off), o.n, o.cols, o.e[0], o.eps};
      if (dn::launch_steer(sa, g_stream, pdl) != cudaSuccess || !mark(kProfSteer)) return false;
      continue;
    }
    if (o.kind == kHeadNormRope) {
      if (k.absorbed[i]) continue;  // runs in the head norm before it
      dn::HeadNormRopeArgs ha{f32_at(o.y, o.y_off), f32_at(o.w, o.qs_off), f32_at(o.x, o.x_off),
                              o.e[0], o.e[1], o.rows, o.cols, o.n, o.eps, nullptr, nullptr, 0, 0};
      if (k.hnr2[i] >= 0) {
        const Op& q = g_ops[k.hnr2[i]];
        ha.x2 = f32_at(q.y, q.y_off);
        ha.w2 = f32_at(q.w, q.qs_off);
        ha.x2_stride = q.e[0];
        ha.heads2 = q.rows;
      }
      if (dn::launch_head_norm_rope(ha, g_stream, pdl) != cudaSuccess || !mark(kProfHeadNormRope))
        return false;
      continue;
    }
    if (o.kind == kConv) {
      const dn::ConvArgs ca{f32_at(o.x, 0), f32_at(o.w, o.qs_off), f32_at(o.e[0], 0), f32_at(o.y, 0),
                            o.rows, o.n, (int)o.cols};
      if (dn::launch_conv(ca, g_stream, pdl) != cudaSuccess || !mark(kProfConv)) return false;
      continue;
    }
    if (o.kind == kAttention) {
      const dn::AttentionArgs aa{f32_at(o.x, 0), f32_at(o.e[0], 0), f32_at(o.e[1], 0),
                                 o.e[2] >= 0 ? f32_at(o.e[2], 0) : nullptr, f32_at(o.y, 0),
                                 o.e[3], o.n, o.rows, o.e[4], o.cols, o.e[5]};
      if (dn::launch_attention(aa, g_stream, pdl) != cudaSuccess || !mark(kProfAttention)) return false;
      continue;
    }
    if (k.absorbed[i]) continue;  // the second product of a dual launch
    dn::LinearArgs a = linear_args(o, status);
    if ((int)i == zc_op) a.ys = zc_ys;  // straight into the pinned host mirror
    int64_t rc;
    if (k.xa_at[i] >= 0 || k.ya_at[i] >= 0 || k.glu[i] >= 0 || k.res[i] >= 0 || k.normin[i] >= 0 ||
        k.dual[i] >= 0 || k.grp[i] > 1) {
      // (xa_out_at is set only together with normin.)
      dn::GemvArgs g{};
      g.q4 = o.q4;
      g.qs = a.qs;
      g.scales = a.scales;
      if (k.xa_at[i] >= 0) {
        g.xa = g_qa + k.xa_at[i];
        g.xa_stride = k.xa_stride[i];
      } else {
        g.xs = a.xs;
      }
      g.ys = a.ys;
      g.ldy = o.rows;
      if (k.ya_at[i] >= 0) {
        g.ya = g_qa + k.ya_at[i];
        g.ya_stride = o.rows / kBlock * dn::kQABytes;
      }
      if (k.glu[i] >= 0) {
        const Op& s = g_ops[k.glu[i]];  // g = s.y, u = s.x
        g.glu_self_gate = o.y == s.y;
        g.glu_other = f32_at(g.glu_self_gate ? s.x : s.y, 0);
        g.glu_out = f32_at(s.y, 0);
      }
      if (k.res[i] >= 0) g.res = f32_at(g_ops[k.res[i]].y, g_ops[k.res[i]].y_off);
      if (k.grp[i] > 1) {
        g.groups = k.grp[i];
        g.group_tile0[0] = 0;
        for (int j = 0; j < k.grp[i]; j++) {
          const Op& p = g_ops[i + j];
          g.group_rows[j] = p.rows;
          g.group_qs[j] = g_bufs[p.w].dev + p.qs_off;
          g.group_scales[j] = g_bufs[p.w].dev + p.sc_off;
          g.group_ys[j] = f32_at(p.y, p.y_off);
          g.group_tile0[j + 1] = g.group_tile0[j] + (p.rows + 31) / 32;
        }
      }
      if (k.dual[i] >= 0) {
        // The gate writes the SwiGLU's g buffer (s.y): its weights go first.
        const Op& p = g_ops[k.dual[i]];
        const Op& sw = g_ops[k.dual[i] + 1];
        const Op& gate = o.y == sw.y ? o : p;
        const Op& up = o.y == sw.y ? p : o;
        g.qs = g_bufs[gate.w].dev + gate.qs_off;
        g.scales = g_bufs[gate.w].dev + gate.sc_off;
        g.qs2 = g_bufs[up.w].dev + up.qs_off;
        g.scales2 = g_bufs[up.w].dev + up.sc_off;
        g.ys = f32_at(gate.y, gate.y_off);
        g.ys2 = f32_at(up.y, up.y_off);
      }
      if (k.normin[i] >= 0) {
        const Op& m = g_ops[k.normin[i]];
        g.xs = f32_at(m.x, m.x_off);
        g.norm_w = f32_at(m.w, m.qs_off);
        g.norm_eps = m.eps;
        g.norm_out = f32_at(m.y, m.y_off);
        if (k.xa_out_at[i] >= 0) {
          g.xa_out = g_qa + k.xa_out_at[i];
          g.xa_out_stride = m.rows / kBlock * dn::kQABytes;
        }
      }
      g.rows = o.rows;
      g.cols = o.cols;
      g.n = o.n;
      g.status = status;
      rc = dn::launch_gemv_ex(g, g_stream, pdl);
    } else if (g_generic) {
      rc = dn::launch_generic(a, g_stream);
    } else {
      rc = dn::path_for(a) == 0 ? dn::launch_gemv(a, g_stream, pdl) : dn::launch_linear(a, g_stream);
    }
    const bool tc = !g_generic && dn::path_for(a) == 1;
    if (rc != 0 || !mark(tc ? (o.q4 ? kProfGemmQ4I8 : kProfGemmQ8I8) : (o.q4 ? kProfGemvQ4I8 : kProfGemvQ8I8)))
      return false;
  }
  for (const Range& r : downloads) {
    const Buf& b = g_bufs[r.buf];
    if (b.host == nullptr) continue;
    if (cudaMemcpyAsync(b.host + r.lo, b.dev + r.lo, (size_t)(r.hi - r.lo), cudaMemcpyDeviceToHost,
                        g_stream) != cudaSuccess)
      return false;
  }
  return true;
}

uint8_t* dev_of(int64_t h) { return h >= 0 ? g_bufs[h].dev : nullptr; }

bool same_as_graph() {
  if (g_exec == nullptr || g_exec_xq != g_xq || g_exec_qa != g_qa || g_exec_ops.size() != g_ops.size() ||
      g_exec_fuse != g_fuse || g_exec_generic != g_generic || g_exec_prof != g_profiling)
    return false;
  std::vector<int64_t> hs;
  size_t at = 0;
  for (size_t i = 0; i < g_ops.size(); i++) {
    if (!(g_ops[i] == g_exec_ops[i])) return false;
    op_handles(g_ops[i], hs);
    for (int64_t h : hs)
      if (at >= g_exec_ptrs.size() || g_exec_ptrs[at++] != dev_of(h)) return false;
  }
  return true;
}

int64_t commit(int64_t wait) {
  if (!g_ready) return 0;
  if (g_bad_op) {
    g_bad_op = false;
    g_ops.clear();
    return 0;
  }
  cudaSetDevice(g_device);
  uint32_t* status = nullptr;
  volatile uint32_t* status_host = nullptr;
  if (!dn::status_words(&status, &status_host)) return 0;
  // Weights (matrices and norm weights): once per buffer, outside the graph.
  for (const Op& o : g_ops) {
    if (o.w < 0) continue;
    Buf& b = g_bufs[o.w];
    if (!b.weights_on_device && b.host != nullptr) {
      if (cudaMemcpyAsync(b.dev, b.host, (size_t)b.bytes, cudaMemcpyHostToDevice, g_stream) !=
          cudaSuccess)
        return 0;
      b.weights_on_device = true;
    }
  }
  // Scratch for the tensor-core path.
  int64_t need = 0;
  for (const Op& o : g_ops)
    if (o.kind == kMatmul) need = std::max(need, o.n * o.cols);
  if (need > g_xcap) {
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) return 0;
    drop_graph();
    cudaFree(g_xq);
    cudaFree(g_xsc);
    g_xq = nullptr;
    g_xsc = nullptr;
    g_xcap = 0;
    if (cudaMalloc(&g_xq, (size_t)need) != cudaSuccess ||
        cudaMalloc(&g_xsc, (size_t)(need / kBlock + 1) * 4) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    g_xcap = need;
  }
  if (!same_as_graph()) {
    drop_graph();
    const Plan plan = plan_ops(status);
    const int64_t qa_need = plan.bytes;
    if (qa_need > g_qa_cap) {
      if (cudaStreamSynchronize(g_stream) != cudaSuccess) return 0;
      cudaFree(g_qa);
      g_qa = nullptr;
      g_qa_cap = 0;
      if (cudaMalloc(&g_qa, (size_t)qa_need) != cudaSuccess) {
        cudaGetLastError();
        return 0;
      }
      g_qa_cap = qa_need;
    }
    // Ranges to copy in (host-written inputs) and out (the ops' outputs).
    std::vector<Range> uploads, written, in;
    std::vector<Range> outs;
    for (const Op& o : g_ops) {
      reads(o, in);
      for (const Range& r : in) subtract(written, r.buf, r.lo, r.hi, uploads);
      all_writes(o, outs);
      for (const Range& w : outs) add_range(written, w.buf, w.lo, w.hi);
    }
    if (g_profiling) {  // one event after the uploads, one per launch at most
      const size_t need = 1 + plan.host.size() + g_ops.size();
      while (g_prof_events.size() < need) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreate(&e) != cudaSuccess) return 0;
        g_prof_events.push_back(e);
      }
    }
    cudaGraph_t graph = nullptr;
    // The command buffer's last op, a plain product with a small output in a
    // host-visible buffer (the logits of a decode step): its epilogue stores
    // straight into the pinned host mirror (the device address of the mapped
    // page-locked memory), so the output crosses PCIe while the product runs
    // instead of in a copy after it. Nothing later in the command buffer reads
    // it, and a later commit that reads the buffer copies the mirror in first.
    int zc_op = -1;
    float* zc_ys = nullptr;
    if (!g_profiling && !g_ops.empty()) {
      const int i = (int)g_ops.size() - 1;
      const Op& o = g_ops[i];
      const int64_t bytes = o.n * o.rows * 4;
      void* d = nullptr;
      if (o.kind == kMatmul && !plan.absorbed[i] && plan.grp[i] <= 1 && plan.dual[i] < 0 && plan.glu[i] < 0 &&
          plan.res[i] < 0 && plan.ya_at[i] < 0 && g_bufs[o.y].host != nullptr && bytes <= (8 << 20)) {
        if (cudaHostGetDevicePointer(&d, g_bufs[o.y].host + o.y_off, 0) == cudaSuccess && d != nullptr) {
          zc_op = i;
          zc_ys = static_cast<float*>(d);
          remove_range(written, o.y, o.y_off, o.y_off + bytes);
        } else {
          cudaGetLastError();
        }
      }
    }
    if (cudaStreamBeginCapture(g_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return 0;
    const bool ok = record(uploads, written, plan, status, zc_op, zc_ys);
    const cudaError_t e = cudaStreamEndCapture(g_stream, &graph);
    if (!ok || e != cudaSuccess || graph == nullptr ||
        cudaGraphInstantiate(&g_exec, graph, 0) != cudaSuccess) {
      if (graph != nullptr) cudaGraphDestroy(graph);
      cudaGetLastError();
      g_exec = nullptr;
      return 0;
    }
    cudaGraphDestroy(graph);
    g_exec_ops = g_ops;
    g_exec_fuse = g_fuse;
    g_exec_generic = g_generic;
    g_exec_prof = g_profiling;
    g_exec_xq = g_xq;
    g_exec_qa = g_qa;
    std::vector<int64_t> hs;
    for (const Op& o : g_ops) {
      op_handles(o, hs);
      for (int64_t h : hs) g_exec_ptrs.push_back(dev_of(h));
    }
  }
  if (cudaEventRecord(g_ev0, g_stream) != cudaSuccess ||
      cudaGraphLaunch(g_exec, g_stream) != cudaSuccess ||
      cudaEventRecord(g_ev1, g_stream) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  g_pending = true;
  if (!wait) return 1;
  return wait_pending() ? 1 : 0;
}

}  // namespace

extern "C" {

int64_t lab_gpu_init(void) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  if (g_ready) return 1;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 0;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess || p.major != 10) {
    cudaGetLastError();
    return 0;
  }
  if (cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&g_ev0) != cudaSuccess || cudaEventCreate(&g_ev1) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  g_device = dev;
  g_ready = true;
  return 1;
}

void lab_gpu_device_name(char* out, int64_t capacity) {
  if (out == nullptr || capacity <= 0) return;
  cudaDeviceProp p;
  const int dev = g_ready ? g_device : 0;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) {
    cudaGetLastError();
    out[0] = 0;
    return;
  }
  snprintf(out, (size_t)capacity, "%s", p.name);
}

// One allocation may take all of the device's memory.
int64_t lab_gpu_max_buffer_length(void) {
  size_t free_b = 0, total = 0;
  if (!g_ready || cudaMemGetInfo(&free_b, &total) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return (int64_t)total;
}

// What gpu.dart bounds maxSeq by: the attention kernel's score array, as the
// reference reports it (lab_vulkan.c:513-515: keys * 4 + 128 bytes). Here the
// scores are doubles, kMaxAttnKeys of them.
int64_t lab_gpu_max_shared_memory(void) { return dn::kMaxAttnKeys * 4 + 128; }

int64_t lab_gpu_recommended_working_set(void) { return lab_gpu_max_buffer_length(); }

int64_t lab_gpu_thermal_state(void) { return -1; }  // no such state on CUDA (as on Vulkan)

int64_t lab_gpu_physical_memory(void) {
  return (int64_t)sysconf(_SC_PHYS_PAGES) * (int64_t)sysconf(_SC_PAGESIZE);
}

// The reference's decode-GEMV shapes (rows per subgroup 1, 2, 4) are one
// kernel here, so those and negative values keep it; 0 selects the generic
// kernel for decode products, a same-device numerical reference.
void lab_gpu_set_decode_rows(int64_t rows) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  g_generic = rows == 0;
}

// Vulkan workgroup sizes and a vectorized Q8 head: not modes of this
// library, so the calls report them unavailable (0), as the reference does
// where they are not.
int64_t lab_gpu_set_q8_group(int64_t invocations) {
  (void)invocations;
  return 0;
}
int64_t lab_gpu_set_q8_vector(int64_t on) {
  (void)on;
  return 0;
}
int64_t lab_gpu_register_q8_head(int64_t w, int64_t qs, int64_t rows, int64_t cols, int64_t q4Body) {
  (void)w, (void)qs, (void)rows, (void)cols, (void)q4Body;
  return 0;
}

void lab_gpu_set_profiling(int64_t on) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  g_profiling = on != 0;
}

int64_t lab_gpu_profile(double* ms, int64_t* counts, int64_t kinds) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  for (int64_t k = 0; k < kinds && k < kProfKinds; k++) {
    if (ms != nullptr) ms[k] = g_kind_ms[k];
    if (counts != nullptr) counts[k] = g_kind_count[k];
    g_kind_ms[k] = 0.0;
    g_kind_count[k] = 0;
  }
  return kProfKinds;
}

int64_t lab_gpu_buffer(int64_t bytes) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return new_buffer(bytes);
}

int64_t lab_gpu_readback_buffer(int64_t bytes) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return new_buffer(bytes);
}

int64_t lab_gpu_wrap(void* address, int64_t bytes) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  const int64_t h = new_buffer(bytes);
  if (h >= 0 && bytes > 0) memcpy(g_bufs[h].host, address, (size_t)bytes);
  return h;
}

int64_t lab_gpu_wrap_copies(void) { return 1; }

void* lab_gpu_contents(int64_t handle) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return valid(handle) ? g_bufs[handle].host : nullptr;
}

double lab_gpu_last_ms(void) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return g_last_ms;
}

void lab_gpu_release(int64_t handle) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  if (!valid(handle)) return;
  wait_pending();
  cudaSetDevice(g_device);
  Buf& b = g_bufs[handle];
  std::vector<int64_t> hs;
  for (const Op& o : g_exec_ops) {
    op_handles(o, hs);
    if (std::find(hs.begin(), hs.end(), handle) != hs.end()) {
      drop_graph();
      break;
    }
  }
  cudaFree(b.dev);
  cudaFreeHost(b.host);
  b = Buf();
  g_free.push_back(handle);
  g_live--;
}

int64_t lab_gpu_live_buffers(void) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return g_live;
}

void lab_gpu_begin(void) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  wait_pending();
  g_ops.clear();
  g_bad_op = false;
}

int64_t lab_gpu_commit(int64_t wait) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return commit(wait);
}

int64_t lab_gpu_wait(void) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return wait_pending() ? 1 : 0;
}

void lab_gpu_enc_matmul_q8(int64_t w, int64_t qsOffset, int64_t scalesOffset, int64_t x,
                           int64_t xOffset, int64_t y, int64_t yOffset, int64_t rows, int64_t cols,
                           int64_t n) {
  encode(false, w, qsOffset, scalesOffset, x, xOffset, y, yOffset, rows, cols, n);
}

void lab_gpu_enc_matmul_q4(int64_t w, int64_t qsOffset, int64_t scalesOffset, int64_t x,
                           int64_t xOffset, int64_t y, int64_t yOffset, int64_t rows, int64_t cols,
                           int64_t n) {
  encode(true, w, qsOffset, scalesOffset, x, xOffset, y, yOffset, rows, cols, n);
}

void lab_gpu_enc_rms_norm(int64_t x, int64_t xOffset, int64_t w, int64_t wOffset, int64_t out,
                          int64_t outOffset, int64_t rows, int64_t cols, double eps, int64_t accumulate) {
  encode_norm(x, xOffset, w, wOffset, out, outOffset, rows, cols, eps, accumulate);
}

void lab_gpu_enc_swiglu(int64_t g, int64_t u, int64_t count) { encode_swiglu(g, u, count); }

void lab_gpu_enc_add(int64_t src, int64_t srcOffset, int64_t dst, int64_t dstOffset, int64_t count) {
  encode_add(src, srcOffset, dst, dstOffset, count);
}

int64_t dn_gpu_device_buffer(int64_t bytes) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  if (!g_ready || bytes < 0) return -1;
  cudaSetDevice(g_device);
  Buf b;
  const size_t n = bytes == 0 ? 16 : (size_t)bytes;
  if (cudaMalloc(&b.dev, n) != cudaSuccess || cudaMemset(b.dev, 0, n) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(b.dev);
    return -1;
  }
  b.bytes = bytes;
  b.live = true;
  b.weights_on_device = true;  // nothing on the host to copy, ever
  return add_buffer(b);
}

int64_t dn_gpu_wrap_file(const char* path, int64_t offset, int64_t bytes) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  return wrap_file(path, offset, bytes);
}

void lab_gpu_enc_copy(int64_t src, int64_t srcOffset, int64_t dst, int64_t dstOffset, int64_t count) {
  encode_copy(src, srcOffset, dst, dstOffset, count);
}

void lab_gpu_enc_steer(int64_t x, int64_t xOffset, int64_t v, int64_t vOffset, int64_t rows,
                       int64_t cols, int64_t mode, double scale) {
  encode_steer(x, xOffset, v, vOffset, rows, cols, mode, scale);
}

void lab_gpu_enc_head_norm_rope(int64_t x, int64_t xOffset, int64_t xStride, int64_t w, int64_t wOffset,
                                int64_t rope, int64_t ropeOffset, int64_t ropeStride, int64_t heads,
                                int64_t hd, int64_t n, double eps) {
  encode_head_norm_rope(x, xOffset, xStride, w, wOffset, rope, ropeOffset, ropeStride, heads, hd, n, eps);
}

void lab_gpu_enc_conv(int64_t bcx, int64_t weight, int64_t weightOffset, int64_t history, int64_t y,
                      int64_t width, int64_t k, int64_t n) {
  encode_conv(bcx, weight, weightOffset, history, y, width, k, n);
}

void lab_gpu_enc_attention(int64_t q, int64_t keys, int64_t values, int64_t gate, int64_t out,
                           int64_t position, int64_t n, int64_t heads, int64_t kvHeads, int64_t hd,
                           int64_t window) {
  encode_attention(q, keys, values, gate, out, position, n, heads, kvHeads, hd, window);
}

void dn_gpu_set_fusion(int64_t on) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  g_fuse = on != 0;
}

void dn_gpu_enc_batch(const int64_t* table, int64_t count) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  for (int64_t i = 0; i < count && table != nullptr; i++) {
    const int64_t* r = table + 11 * i;
    switch (r[0]) {
      case DN_BATCH_Q8:
      case DN_BATCH_Q4:
        encode(r[0] == DN_BATCH_Q4, r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8], r[9], r[10]);
        break;
      case DN_BATCH_RMS_NORM: {
        double eps;
        memcpy(&eps, &r[9], sizeof eps);
        encode_norm(r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8], eps, r[10]);
        break;
      }
      case DN_BATCH_SWIGLU: encode_swiglu(r[1], r[2], r[3]); break;
      case DN_BATCH_ADD: encode_add(r[1], r[2], r[3], r[4], r[5]); break;
      case DN_BATCH_COPY: encode_copy(r[1], r[2], r[3], r[4], r[5]); break;
      case DN_BATCH_STEER: {
        double scale;
        memcpy(&scale, &r[8], sizeof scale);
        encode_steer(r[1], r[2], r[3], r[4], r[5], r[6], r[7], scale);
        break;
      }
      case DN_BATCH_HEAD_NORM_ROPE: {
        double eps;
        memcpy(&eps, &r[10], sizeof eps);
        const int64_t p = r[9];
        encode_head_norm_rope(r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8], p & 0xffff,
                              (p >> 16) & 0xffff, (p >> 32) & 0xffffffff, eps);
        break;
      }
      case DN_BATCH_CONV: encode_conv(r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8]); break;
      case DN_BATCH_ATTENTION:
        encode_attention(r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8], r[9], r[10] & 0xffffffff,
                         (r[10] >> 32) & 0x7fffffff);
        break;
      default: g_bad_op = true;
    }
  }
}

}  // extern "C"
