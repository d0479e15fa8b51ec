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
#include <string.h>

#include <algorithm>
#include <mutex>
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
  uint8_t* host = nullptr;  // pinned mirror: lab_gpu_contents
  int64_t bytes = 0;
  bool live = false;
  bool weights_on_device = false;  // copied once, at its first use as a matrix
};

struct Op {
  bool q4;
  int64_t w, qs_off, sc_off, x, x_off, y, y_off, rows, cols, n;
  bool operator==(const Op& o) const {
    return q4 == o.q4 && w == o.w && qs_off == o.qs_off && sc_off == o.sc_off && x == o.x &&
           x_off == o.x_off && y == o.y && y_off == o.y_off && rows == o.rows && cols == o.cols &&
           n == o.n;
  }
};

struct Range {
  int64_t buf, lo, hi;  // bytes [lo, hi) of buffer `buf`
};

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

// The graph of the last command buffer, with what it was captured from.
cudaGraphExec_t g_exec = nullptr;
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
  uint32_t* sd = nullptr;
  volatile uint32_t* sh = nullptr;
  if (dn::status_words(&sd, &sh) && *sh != 0) return false;  // a bounded wait ran out
  return true;
}

bool valid(int64_t h) { return h >= 0 && h < (int64_t)g_bufs.size() && g_bufs[h].live; }

bool fits(int64_t h, int64_t off, int64_t bytes) {
  return valid(h) && off >= 0 && bytes >= 0 && off <= g_bufs[h].bytes - bytes;
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

void encode(bool q4, int64_t w, int64_t qs_off, int64_t sc_off, int64_t x, int64_t x_off, int64_t y,
            int64_t y_off, int64_t rows, int64_t cols, int64_t n) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  const bool ok = rows >= 0 && cols >= 0 && n >= 0 && cols % kBlock == 0 &&
                  fits(w, qs_off, q4 ? rows * cols / 2 : rows * cols) &&
                  fits(w, sc_off, rows * (cols / kBlock) * (q4 ? 2 : 4)) &&
                  fits(x, x_off, n * cols * 4) && fits(y, y_off, n * rows * 4);
  if (!ok) {
    g_bad_op = true;
    return;
  }
  g_ops.push_back(Op{q4, w, qs_off, sc_off, x, x_off, y, y_off, rows, cols, n});
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

// Records the command buffer's copies and products on g_stream.
dn::LinearArgs linear_args(const Op& o, uint32_t* status) {
  const Buf &w = g_bufs[o.w], &x = g_bufs[o.x], &y = g_bufs[o.y];
  return dn::LinearArgs{o.q4, w.dev + o.qs_off, w.dev + o.sc_off,
                        reinterpret_cast<const float*>(x.dev + o.x_off), g_xq, g_xsc,
                        reinterpret_cast<float*>(y.dev + o.y_off), o.rows, o.cols, o.n, o.rows,
                        1, status};
}

// QA links of the recorded products (decode GEMV path only). Product i reads
// its input as QA blocks at byte xa_at[i] of g_qa (row stride xa_stride[i])
// when the input is either
//  * a 32-value-aligned part of the output of the last product that wrote
//    over it (all of the output when n > 1, where token strides must agree);
//    that product then also writes its output as QA blocks, at ya_at[j]; or
//  * host data no earlier product wrote: quantized once, before the products,
//    for every product that reads the same range.
struct HostQA {
  int64_t buf, off, n, cols, at;
};
struct Links {
  std::vector<int64_t> xa_at, xa_stride, ya_at;
  std::vector<HostQA> host;
  int64_t bytes = 0;
};

int64_t qa_bytes(int64_t n, int64_t values) { return (n * (values / kBlock) * dn::kQABytes + 15) / 16 * 16; }

Links plan_links(uint32_t* status) {
  const int n = (int)g_ops.size();
  Links k;
  k.xa_at.assign(n, -1);
  k.xa_stride.assign(n, 0);
  k.ya_at.assign(n, -1);
  std::vector<bool> gemv(n);
  for (int i = 0; i < n; i++) gemv[i] = dn::path_for(linear_args(g_ops[i], status)) == 0;
  for (int i = 0; i < n; i++) {
    const Op& c = g_ops[i];
    if (!gemv[i] || c.cols % kBlock != 0) continue;
    const int64_t lo = c.x_off, hi = c.x_off + c.n * c.cols * 4;
    int j = i - 1;
    for (; j >= 0; j--) {
      const Op& p = g_ops[j];
      if (p.y == c.x && p.y_off < hi && lo < p.y_off + p.n * p.rows * 4) break;
    }
    if (j >= 0) {
      const Op& p = g_ops[j];
      const int64_t delta = lo - p.y_off;
      const bool inside = delta >= 0 && hi <= p.y_off + p.n * p.rows * 4 && delta % (kBlock * 4) == 0;
      const bool tokens_agree = (c.n == 1 && p.n == 1) || (delta == 0 && p.n == c.n && p.rows == c.cols);
      if (!gemv[j] || p.rows % kBlock != 0 || !inside || !tokens_agree) continue;
      if (k.ya_at[j] < 0) {
        k.ya_at[j] = k.bytes;
        k.bytes += qa_bytes(p.n, p.rows);
      }
      k.xa_at[i] = k.ya_at[j] + delta / (kBlock * 4) * dn::kQABytes;
      k.xa_stride[i] = p.rows / kBlock * dn::kQABytes;
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

bool record(const std::vector<Range>& uploads, const std::vector<Range>& downloads,
            const Links& k, uint32_t* status) {
  for (const Range& r : uploads) {
    const Buf& b = g_bufs[r.buf];
    if (cudaMemcpyAsync(b.dev + r.lo, b.host + r.lo, (size_t)(r.hi - r.lo), cudaMemcpyHostToDevice,
                        g_stream) != cudaSuccess)
      return false;
  }
  for (const HostQA& q : k.host) {
    if (dn::launch_quantize_qa(reinterpret_cast<const float*>(g_bufs[q.buf].dev + q.off), g_qa + q.at,
                               q.n, q.cols, q.cols / kBlock * dn::kQABytes, g_stream) != cudaSuccess)
      return false;
  }
  for (size_t i = 0; i < g_ops.size(); i++) {
    const Op& o = g_ops[i];
    const dn::LinearArgs a = linear_args(o, status);
    int64_t rc;
    if (k.xa_at[i] >= 0 || k.ya_at[i] >= 0) {
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
      g.rows = o.rows;
      g.cols = o.cols;
      g.n = o.n;
      g.status = status;
      rc = dn::launch_gemv_ex(g, g_stream, true);
    } else {
      rc = dn::path_for(a) == 0 ? dn::launch_gemv(a, g_stream, true) : dn::launch_linear(a, g_stream);
    }
    if (rc != 0) return false;
  }
  for (const Range& r : downloads) {
    const Buf& b = g_bufs[r.buf];
    if (cudaMemcpyAsync(b.host + r.lo, b.dev + r.lo, (size_t)(r.hi - r.lo), cudaMemcpyDeviceToHost,
                        g_stream) != cudaSuccess)
      return false;
  }
  return true;
}

bool same_as_graph() {
  if (g_exec == nullptr || g_exec_xq != g_xq || g_exec_qa != g_qa || g_exec_ops.size() != g_ops.size())
    return false;
  for (size_t i = 0; i < g_ops.size(); i++) {
    const Op &a = g_ops[i], &b = g_exec_ops[i];
    if (!(a == b) || g_exec_ptrs[3 * i] != g_bufs[a.w].dev ||
        g_exec_ptrs[3 * i + 1] != g_bufs[a.x].dev || g_exec_ptrs[3 * i + 2] != g_bufs[a.y].dev)
      return false;
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
  // Weights: once per buffer, outside the graph.
  for (const Op& o : g_ops) {
    Buf& b = g_bufs[o.w];
    if (!b.weights_on_device) {
      if (cudaMemcpyAsync(b.dev, b.host, (size_t)b.bytes, cudaMemcpyHostToDevice, g_stream) !=
          cudaSuccess)
        return 0;
      b.weights_on_device = true;
    }
  }
  // Scratch for the tensor-core path.
  int64_t need = 0;
  for (const Op& o : g_ops) need = std::max(need, o.n * o.cols);
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
    const Links links = plan_links(status);
    const int64_t qa_need = links.bytes;
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
    // Ranges to copy in (host-written inputs) and out (products' outputs).
    std::vector<Range> uploads, written;
    for (const Op& o : g_ops) {
      subtract(written, o.x, o.x_off, o.x_off + o.n * o.cols * 4, uploads);
      add_range(written, o.y, o.y_off, o.y_off + o.n * o.rows * 4);
    }
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(g_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return 0;
    const bool ok = record(uploads, written, links, status);
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
    g_exec_xq = g_xq;
    g_exec_qa = g_qa;
    for (const Op& o : g_ops) {
      g_exec_ptrs.push_back(g_bufs[o.w].dev);
      g_exec_ptrs.push_back(g_bufs[o.x].dev);
      g_exec_ptrs.push_back(g_bufs[o.y].dev);
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
  for (const Op& o : g_exec_ops) {
    if (o.w == handle || o.x == handle || o.y == handle) {
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

void dn_gpu_enc_batch(const int64_t* table, int64_t count) {
  std::lock_guard<std::recursive_mutex> lock(g_mu);
  for (int64_t i = 0; i < count && table != nullptr; i++) {
    const int64_t* r = table + 11 * i;
    encode(r[0] != 0, r[1], r[2], r[3], r[4], r[5], r[6], r[7], r[8], r[9], r[10]);
  }
}

}  // extern "C"
