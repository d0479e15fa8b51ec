// The C-ABI of libdianoia_b200.so: dianoia's lab_* kernel symbols served by
// the GPU, and the library's own device-resident dn_* API. See
// include/dianoia_b200.h for the contract of each function.
//
// Host side of a lab_* call: every pointer is classified once per call
// (cudaPointerGetAttributes). Managed (lab_alloc) and device memory is used
// in place; host memory is staged through per-thread pinned and device
// buffers that grow on demand, so concurrent calls from different threads do
// not share scratch. Each call runs on its thread's own stream and
// synchronizes before it returns, like the reference's CPU kernels.
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <new>
#include <mutex>
#include <vector>

#include "dianoia_b200.h"
#include "dn_launch.h"

using dn::LinearArgs;

namespace dn {

// Every translation unit with bounded waits keeps its own device copy of the
// wait limit (dn_common.cuh) and registers a setter here while the library
// loads; dn_set_wait_limit_ns calls them all for the current device.
using WaitLimitSetter = bool (*)(uint64_t ns);

static std::vector<WaitLimitSetter>& wait_limit_setters() {
  static std::vector<WaitLimitSetter> v;
  return v;
}

bool register_wait_limit_setter(WaitLimitSetter setter) {
  wait_limit_setters().push_back(setter);
  return true;
}

}  // namespace dn

namespace {

thread_local int64_t tl_last_error = DN_OK;

void set_error(int64_t e) {
  if (e != DN_OK && tl_last_error == DN_OK) tl_last_error = e;
}

bool cuda_ok(cudaError_t e) {
  if (e == cudaSuccess) return true;
  static int reported = 0;
  if (reported++ < 8) fprintf(stderr, "dianoia_b200: CUDA error: %s\n", cudaGetErrorString(e));
  set_error(DN_ERR_CUDA);
  return false;
}

// ---------------------------------------------------------------- devices

struct DeviceState {
  bool ready = false;
  uint32_t* status_host = nullptr;  // pinned, mapped: kernels' bounded-wait status
  uint32_t* status_dev = nullptr;
};

std::mutex g_mu;
DeviceState g_devices[64];

int device_count() {
  static int count = -1;
  if (count < 0) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    int usable = 0;
    for (int d = 0; d < n; d++) {
      cudaDeviceProp p;
      if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) usable++;
    }
    count = usable;
  }
  return count;
}

DeviceState* device_state() {
  if (device_count() <= 0) return nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& d = g_devices[dev & 63];
  if (!d.ready) {
    void* h = nullptr;
    if (cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess)
      return nullptr;
    memset(h, 0, 64);
    void* dp = nullptr;
    if (cudaHostGetDevicePointer(&dp, h, 0) != cudaSuccess) {
      cudaFreeHost(h);
      return nullptr;
    }
    d.status_host = static_cast<uint32_t*>(h);
    d.status_dev = static_cast<uint32_t*>(dp);
    d.ready = true;
  }
  return &d;
}

// ---------------------------------------------------------- lab_alloc registry
//
// Allocations from lab_alloc, so that a weight matrix in managed memory is
// prefetched to the GPU once, at its first use, instead of page-faulting in.

struct Alloc {
  size_t bytes;
  int prefetched_to;  // device, or -1
};
std::map<uintptr_t, Alloc> g_allocs;

void prefetch_once(const void* p, int dev, cudaStream_t st) {
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_allocs.upper_bound((uintptr_t)p);
  if (it == g_allocs.begin()) return;
  --it;
  if ((uintptr_t)p >= it->first + it->second.bytes || it->second.prefetched_to == dev) return;
  if (cudaMemPrefetchAsync((void*)it->first, it->second.bytes, dev, st) == cudaSuccess) {
    it->second.prefetched_to = dev;
  } else {
    cudaGetLastError();
  }
}

// ------------------------------------------------------------ call context

struct Buf {
  void* p = nullptr;
  size_t cap = 0;
  bool pinned = false;
  bool grow(size_t bytes) {
    if (bytes <= cap) return true;
    release();
    size_t want = bytes < 4096 ? 4096 : bytes + bytes / 4;
    cudaError_t e = pinned ? cudaHostAlloc(&p, want, cudaHostAllocPortable) : cudaMalloc(&p, want);
    if (!cuda_ok(e)) {
      p = nullptr;
      cap = 0;
      return false;
    }
    cap = want;
    return true;
  }
  void release() {
    if (p != nullptr) {
      if (pinned) cudaFreeHost(p); else cudaFree(p);
    }
    p = nullptr;
    cap = 0;
  }
};

struct CallCtx {
  int device = -1;
  cudaStream_t stream = nullptr;
  Buf dw, ds, dx, dy, dxq, dxsc;  // device staging
  Buf hx, hy, hxq, hxsc;          // pinned staging
  CallCtx() { hx.pinned = hy.pinned = hxq.pinned = hxsc.pinned = true; }
  ~CallCtx() {
    // At process exit the runtime may already be gone; errors are ignored.
    for (Buf* b : {&dw, &ds, &dx, &dy, &dxq, &dxsc, &hx, &hy, &hxq, &hxsc}) b->release();
    if (stream != nullptr) cudaStreamDestroy(stream);
    cudaGetLastError();
  }
};

thread_local CallCtx tl_ctx;

CallCtx* call_ctx() {
  if (device_state() == nullptr) {
    set_error(DN_ERR_NO_DEVICE);
    return nullptr;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  CallCtx& c = tl_ctx;
  if (c.device != dev) {
    // A thread that moved to another device starts over there.
    c.~CallCtx();
    new (&c) CallCtx();
    if (!cuda_ok(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking))) return nullptr;
    c.device = dev;
  }
  return &c;
}

bool on_device(const void* p) {
  if (p == nullptr) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// An input the kernels may read: itself when device-addressable, else a
// device copy on the call's stream.
const void* stage_in(CallCtx* c, Buf& dev, Buf* pinned, const void* p, size_t bytes) {
  if (p == nullptr || bytes == 0) return p;
  if (on_device(p)) {
    prefetch_once(p, c->device, c->stream);
    return p;
  }
  if (!dev.grow(bytes)) return nullptr;
  const void* src = p;
  if (pinned != nullptr) {  // small per-call inputs: pinned copy, asynchronous DMA
    if (!pinned->grow(bytes)) return nullptr;
    memcpy(pinned->p, p, bytes);
    src = pinned->p;
  }
  if (!cuda_ok(cudaMemcpyAsync(dev.p, src, bytes, cudaMemcpyHostToDevice, c->stream))) return nullptr;
  return dev.p;
}

// An output: itself when device-addressable, else device staging that
// finish_out copies back after the kernels.
struct Out {
  void* user = nullptr;
  void* dev = nullptr;
  Buf* pinned = nullptr;
  size_t bytes = 0;
  bool staged = false;
};

// With `preserve`, the staging starts as a copy of the user's buffer, for
// outputs the kernels only partly write (xq when cols % 32 != 0: the
// reference leaves each row's tail untouched).
bool stage_out(CallCtx* c, Buf& dev, Buf& pinned, void* p, size_t bytes, Out& o,
               bool preserve = false) {
  o.user = p;
  o.bytes = bytes;
  o.dev = p;
  if (p == nullptr || bytes == 0 || on_device(p)) return true;
  if (!dev.grow(bytes) || !pinned.grow(bytes)) return false;
  o.dev = dev.p;
  o.pinned = &pinned;
  o.staged = true;
  if (preserve) {
    memcpy(pinned.p, p, bytes);
    if (!cuda_ok(cudaMemcpyAsync(dev.p, pinned.p, bytes, cudaMemcpyHostToDevice, c->stream)))
      return false;
  }
  return true;
}

bool copy_back(CallCtx* c, const Out& o) {
  if (!o.staged) return true;
  return cuda_ok(cudaMemcpyAsync(o.pinned->p, o.dev, o.bytes, cudaMemcpyDeviceToHost, c->stream));
}

void finish_out(const Out& o) {
  if (o.staged) memcpy(o.user, o.pinned->p, o.bytes);
}

bool finish_call(CallCtx* c, DeviceState* d) {
  if (!cuda_ok(cudaStreamSynchronize(c->stream))) return false;
  if (d != nullptr && *(volatile uint32_t*)d->status_host != 0) set_error(DN_ERR_CUDA);
  return true;
}

size_t q4_bytes(int64_t rows, int64_t cols) {
  return rows <= 0 ? 0 : (size_t)(((rows - 1) * cols) / 2 + (cols / 32) * 16);
}

void gemm_entry(bool q4, const void* qs, const void* scales, const float* xs, int8_t* xq,
                float* xsc, float* ys, int64_t rows, int64_t cols, int64_t n, int64_t mode) {
  if (rows < 0 || cols < 0 || n < 0 || (mode != 0 && mode != 1)) {
    set_error(DN_ERR_ARGS);
    return;
  }
  if (n == 0) return;
  CallCtx* c = call_ctx();
  DeviceState* d = device_state();
  if (c == nullptr || d == nullptr) return;
  const int64_t blocks = cols / 32;
  const size_t qbytes = q4 ? q4_bytes(rows, cols) : (size_t)(rows * cols);
  const size_t sbytes = (size_t)(rows * blocks * (q4 ? 2 : 4));
  const size_t xbytes = (size_t)(n * cols) * 4, ybytes = (size_t)(n * rows) * 4;
  const size_t xqbytes = (size_t)(n * cols), xscbytes = (size_t)(n * blocks) * 4;

  const void* dqs = rows > 0 && blocks > 0 ? stage_in(c, c->dw, nullptr, qs, qbytes) : qs;
  const void* dsc = rows > 0 && blocks > 0 ? stage_in(c, c->ds, nullptr, scales, sbytes) : scales;
  const float* dxs = static_cast<const float*>(stage_in(c, c->dx, &c->hx, xs, xbytes));
  Out oy, oxq, oxsc;
  bool ok = (dqs != nullptr || qbytes == 0) && (dsc != nullptr || sbytes == 0) &&
            (dxs != nullptr || xbytes == 0);
  ok = ok && stage_out(c, c->dy, c->hy, ys, ybytes, oy);
  if (mode == 1) {
    ok = ok && stage_out(c, c->dxq, c->hxq, xq, xqbytes, oxq, cols % 32 != 0) &&
         stage_out(c, c->dxsc, c->hxsc, xsc, xscbytes, oxsc);
  }
  if (!ok) return;
  LinearArgs a{q4,
               dqs,
               dsc,
               dxs,
               static_cast<int8_t*>(oxq.dev),
               static_cast<float*>(oxsc.dev),
               static_cast<float*>(oy.dev),
               rows,
               cols,
               n,
               rows,
               mode,
               d->status_dev};
  int64_t r = DN_OK;
  if (rows == 0) {
    // No rows to multiply; mode 1 still leaves the quantized inputs behind.
    if (mode == 1 && !cuda_ok(dn::launch_quantize_q8(dxs, a.xq, a.xsc, n, cols, c->stream))) return;
  } else {
    r = dn::launch_linear(a, c->stream);
  }
  if (r != DN_OK) {
    set_error(r);
    return;
  }
  if (!copy_back(c, oy) || !copy_back(c, oxq) || !copy_back(c, oxsc)) return;
  if (!finish_call(c, d)) return;
  finish_out(oy);
  finish_out(oxq);
  finish_out(oxsc);
}

template <typename QT, typename ST>
void quantize_entry(bool q4, const float* w, QT* qs, ST* scales, int64_t rows, int64_t cols) {
  if (rows < 0 || cols < 0) {
    set_error(DN_ERR_ARGS);
    return;
  }
  const int64_t blocks = cols / 32;
  if (rows == 0 || blocks == 0) return;
  CallCtx* c = call_ctx();
  DeviceState* d = device_state();
  if (c == nullptr || d == nullptr) return;
  const size_t wbytes = (size_t)(rows * cols) * 4;
  const size_t qbytes = q4 ? q4_bytes(rows, cols) : (size_t)(rows * cols);
  const size_t sbytes = (size_t)(rows * blocks) * (q4 ? 2 : 4);
  const float* dw = static_cast<const float*>(stage_in(c, c->dx, nullptr, w, wbytes));
  Out oq, os;
  if (dw == nullptr || !stage_out(c, c->dxq, c->hxq, qs, qbytes, oq, cols % 32 != 0) ||
      !stage_out(c, c->dxsc, c->hxsc, scales, sbytes, os))
    return;
  cudaError_t e =
      q4 ? dn::launch_quantize_q4(dw, static_cast<uint8_t*>(oq.dev), static_cast<uint16_t*>(os.dev),
                                  rows, cols, c->stream)
         : dn::launch_quantize_q8(dw, static_cast<int8_t*>(oq.dev), static_cast<float*>(os.dev),
                                  rows, cols, c->stream);
  if (!cuda_ok(e) || !copy_back(c, oq) || !copy_back(c, os) || !finish_call(c, d)) return;
  finish_out(oq);
  finish_out(os);
}

}  // namespace

namespace dn {
// The current device's bounded-wait status word (device address for the
// kernels, host address to read it), for the other C-ABI files.
bool status_words(uint32_t** dev, volatile uint32_t** host) {
  DeviceState* d = device_state();
  if (d == nullptr) return false;
  *dev = d->status_dev;
  *host = d->status_host;
  return true;
}
}  // namespace dn

// ======================================================================= lab_*

extern "C" {

void* lab_alloc(int64_t bytes) {
  if (bytes < 0 || device_state() == nullptr) return nullptr;
  void* p = nullptr;
  const size_t n = bytes == 0 ? 1 : (size_t)bytes;
  if (cudaMallocManaged(&p, n, cudaMemAttachGlobal) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  memset(p, 0, n);
  std::lock_guard<std::mutex> lock(g_mu);
  g_allocs[(uintptr_t)p] = Alloc{n, -1};
  return p;
}

void lab_free(void* p) {
  if (p == nullptr) return;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_allocs.erase((uintptr_t)p) == 0) return;  // not ours
  }
  cudaFree(p);
  cudaGetLastError();
}

int64_t lab_cpu_supported(void) { return device_count() > 0 ? 1 : 0; }

// Read-only private mapping of a whole file (dianoia's MappedFile, the Q8
// cache); NULL when it cannot be opened, is empty or cannot be mapped.
void* lab_map_file(const char* path, int64_t* size) {
  if (path == nullptr || size == nullptr) return nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return nullptr;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    return nullptr;
  }
  void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);  // the mapping keeps the file
  if (p == MAP_FAILED) return nullptr;
  *size = (int64_t)st.st_size;
  return p;
}

void lab_unmap_file(void* p, int64_t size) {
  if (p != nullptr && size > 0) munmap(p, (size_t)size);
}

// Gives the mapping's resident pages back to the OS (a copy lives in GPU
// memory); a later read faults them back in from the file.
void lab_evict_file(void* p, int64_t size) {
  if (p != nullptr && size > 0) madvise(p, (size_t)size, MADV_DONTNEED);
}

// The process's resident set in bytes (/proc/self/statm), -1 if unknown.
int64_t lab_phys_footprint(void) {
  FILE* f = fopen("/proc/self/statm", "r");
  if (f == nullptr) return -1;
  long long total = 0, resident = 0;
  const int got = fscanf(f, "%lld %lld", &total, &resident);
  fclose(f);
  return got == 2 ? (int64_t)resident * (int64_t)sysconf(_SC_PAGESIZE) : -1;
}

void lab_quantize_q8(const float* w, int8_t* qs, float* scales, int64_t rows, int64_t cols) {
  quantize_entry<int8_t, float>(false, w, qs, scales, rows, cols);
}

void lab_quantize_q4(const float* w, uint8_t* qs, uint16_t* scales, int64_t rows, int64_t cols) {
  quantize_entry<uint8_t, uint16_t>(true, w, qs, scales, rows, cols);
}

void lab_gemm_q8(const int8_t* qs, const float* scales, const float* xs, int8_t* xq, float* xsc,
                 float* ys, int64_t rows, int64_t cols, int64_t n, int64_t threads, int64_t mode) {
  (void)threads;
  gemm_entry(false, qs, scales, xs, xq, xsc, ys, rows, cols, n, mode);
}

void lab_gemm_q4(const uint8_t* qs, const uint16_t* scales, const float* xs, int8_t* xq,
                 float* xsc, float* ys, int64_t rows, int64_t cols, int64_t n, int64_t threads,
                 int64_t mode) {
  (void)threads;
  gemm_entry(true, qs, scales, xs, xq, xsc, ys, rows, cols, n, mode);
}

void lab_gemv_q8(const int8_t* qs, const float* scales, const float* x, int8_t* xq, float* xs,
                 float* y, int64_t rows, int64_t cols, int64_t threads, int64_t mode) {
  lab_gemm_q8(qs, scales, x, xq, xs, y, rows, cols, 1, threads, mode);
}

// ======================================================================= dn_*

int64_t dn_linear(int64_t format, const void* qs, const void* scales, const float* xs, int8_t* xq,
                  float* xsc, float* ys, int64_t rows, int64_t cols, int64_t n, int64_t ldy,
                  int64_t mode, int64_t path, int64_t flags, void* stream) {
  if (format != DN_Q8 && format != DN_Q4) return DN_ERR_ARGS;
  if (rows < 0 || cols < 0 || n < 0 || ldy < rows || (mode != 0 && mode != 1)) return DN_ERR_ARGS;
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  LinearArgs a{format == DN_Q4, qs, scales, xs, xq, xsc, ys, rows, cols, n, ldy, mode,
               d->status_dev};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (path) {
    case DN_PATH_AUTO:
      if ((flags & DN_FLAG_PDL) && dn::path_for(a) == 0) return dn::launch_gemv(a, st, true);
      return dn::launch_linear(a, st);
    case DN_PATH_GEMV: return dn::launch_gemv(a, st, (flags & DN_FLAG_PDL) != 0);
    case DN_PATH_TC: return dn::launch_gemm_tc(a, st);
    case DN_PATH_GENERIC: return dn::launch_generic(a, st);
    default: return DN_ERR_ARGS;
  }
}

int64_t dn_linear_path(int64_t format, const void* qs, const void* scales, const float* xs,
                       const int8_t* xq, int64_t rows, int64_t cols, int64_t n, int64_t mode) {
  // Null pointers stand for "suitably aligned" in this query.
  const float* x = xs != nullptr ? xs : reinterpret_cast<const float*>(256);
  int8_t* q = xq != nullptr ? const_cast<int8_t*>(xq) : reinterpret_cast<int8_t*>(256);
  LinearArgs a{format == DN_Q4, qs, scales, x, q, reinterpret_cast<float*>(256), nullptr, rows,
               cols, n, rows, mode, nullptr};
  return dn::path_for(a);
}

int64_t dn_quantize_q8(const float* xs, int8_t* xq, float* xsc, int64_t n, int64_t cols,
                       void* stream) {
  if (n < 0 || cols < 0) return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  return dn::launch_quantize_q8(xs, xq, xsc, n, cols, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? DN_OK
             : DN_ERR_CUDA;
}

int64_t dn_quantize_q4(const float* w, uint8_t* qs, uint16_t* scales, int64_t rows, int64_t cols,
                       void* stream) {
  if (rows < 0 || cols < 0) return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  return dn::launch_quantize_q4(w, qs, scales, rows, cols, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? DN_OK
             : DN_ERR_CUDA;
}

int64_t dn_quantize_qa(const float* xs, uint8_t* xa, int64_t n, int64_t cols, int64_t xa_stride,
                       void* stream) {
  if (n < 0 || cols < 0 || xa_stride < (cols / 32) * dn::kQABytes) return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  return dn::launch_quantize_qa(xs, xa, n, cols, xa_stride, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? DN_OK
             : DN_ERR_CUDA;
}

int64_t dn_gguf_linear_qa(int64_t format, const void* blocks, const uint8_t* xa, float* ys, int64_t rows,
                          int64_t cols, int64_t flags, void* stream) {
  if (format != DN_Q8 && format != DN_Q4) return DN_ERR_ARGS;
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  return dn::launch_gguf_gemv(format == DN_Q4, blocks, xa, ys, rows, cols, d->status_dev,
                              static_cast<cudaStream_t>(stream), (flags & DN_FLAG_PDL) != 0);
}

int64_t dn_gguf_split(int64_t format, const void* blocks, int64_t count, void* qs, void* scales,
                      void* stream) {
  if (format != DN_Q8 && format != DN_Q4) return DN_ERR_ARGS;
  if (count < 0 || (count > 0 && (blocks == nullptr || qs == nullptr || scales == nullptr)))
    return DN_ERR_ARGS;
  if (((uintptr_t)blocks & 1) != 0 || ((uintptr_t)qs & 3) != 0 ||
      ((uintptr_t)scales & (format == DN_Q4 ? 1 : 3)) != 0)
    return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  return dn::launch_gguf_split(format == DN_Q4, blocks, count, qs, scales,
                               static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? DN_OK
             : DN_ERR_CUDA;
}

int64_t dn_rms_norm(const float* x, const float* w, float* out, uint8_t* qa, int64_t qa_stride,
                    int64_t rows, int64_t cols, double eps, int64_t accumulate, int64_t flags,
                    void* stream) {
  if (rows < 0 || cols < 0 || rows > 0x7fffffff) return DN_ERR_ARGS;
  if (rows > 0 && cols > 0 && (x == nullptr || w == nullptr || out == nullptr)) return DN_ERR_ARGS;
  if (((uintptr_t)x & 3) != 0 || ((uintptr_t)w & 3) != 0 || ((uintptr_t)out & 3) != 0) return DN_ERR_ARGS;
  if (qa != nullptr && (cols % 32 != 0 || qa_stride < (cols / 32) * dn::kQABytes ||
                        ((uintptr_t)qa & 3) != 0 || (qa_stride & 3) != 0))
    return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  const dn::NormArgs a{x, w, out, qa, qa_stride, rows, cols, eps, accumulate != 0};
  return dn::launch_rms_norm(a, static_cast<cudaStream_t>(stream), (flags & DN_FLAG_PDL) != 0) ==
                 cudaSuccess
             ? DN_OK
             : DN_ERR_CUDA;
}

int64_t dn_swiglu(float* g, const float* u, uint8_t* qa, int64_t count, int64_t flags, void* stream) {
  if (count < 0 || (count > 0 && (g == nullptr || u == nullptr))) return DN_ERR_ARGS;
  if (((uintptr_t)g & 3) != 0 || ((uintptr_t)u & 3) != 0) return DN_ERR_ARGS;
  if (qa != nullptr && (count % 32 != 0 || ((uintptr_t)qa & 3) != 0)) return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  const dn::SwigluArgs a{g, u, qa, count};
  return dn::launch_swiglu(a, static_cast<cudaStream_t>(stream), (flags & DN_FLAG_PDL) != 0) ==
                 cudaSuccess
             ? DN_OK
             : DN_ERR_CUDA;
}

int64_t dn_linear_qa(int64_t format, const void* qs, const void* scales, const uint8_t* xa,
                     int64_t xa_stride, float* ys, int64_t ldy, uint8_t* ya, int64_t ya_stride,
                     int64_t rows, int64_t cols, int64_t n, int64_t flags, void* stream) {
  if (format != DN_Q8 && format != DN_Q4) return DN_ERR_ARGS;
  if (rows < 0 || cols < 0 || n < 0 || xa == nullptr || xa_stride < (cols / 32) * dn::kQABytes)
    return DN_ERR_ARGS;
  if (ys != nullptr && ldy < rows) return DN_ERR_ARGS;
  if (ya != nullptr && ya_stride < (rows / 32) * dn::kQABytes) return DN_ERR_ARGS;
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  dn::GemvArgs g{};
  g.q4 = format == DN_Q4;
  g.qs = qs;
  g.scales = scales;
  g.xa = xa;
  g.xa_stride = xa_stride;
  g.ys = ys;
  g.ldy = ldy;
  g.ya = ya;
  g.ya_stride = ya_stride;
  g.rows = rows;
  g.cols = cols;
  g.n = n;
  g.status = d->status_dev;
  return dn::launch_gemv_ex(g, static_cast<cudaStream_t>(stream), (flags & DN_FLAG_PDL) != 0);
}

int64_t dn_linear_allgather(int64_t format, const void* qs, const void* scales, const float* xs, int8_t* xq,
                            float* xsc, int64_t rows, int64_t cols, int64_t n, int64_t row0, int64_t total_rows,
                            float* const* ys, int32_t* const* counters, int64_t world, void* stream) {
  if (format != DN_Q8 && format != DN_Q4) return DN_ERR_ARGS;
  if (rows < 0 || cols <= 0 || n < 0 || row0 < 0 || total_rows < row0 + rows || xs == nullptr || ys == nullptr ||
      counters == nullptr || world < 1 || world > dn::kMaxGatherRanks)
    return DN_ERR_ARGS;
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  dn::LinearArgs a{};
  a.q4 = format == DN_Q4;
  a.qs = qs;
  a.scales = scales;
  a.xs = xs;
  a.xq = xq;
  a.xsc = xsc;
  a.ys = nullptr;
  a.rows = rows;
  a.cols = cols;
  a.n = n;
  a.ldy = total_rows;
  a.mode = 1;
  a.status = d->status_dev;
  return dn::launch_gemm_tc_allgather(a, row0, ys, reinterpret_cast<int* const*>(counters), (int)world,
                                      static_cast<cudaStream_t>(stream));
}

int64_t dn_linear_qa_allgather(int64_t format, const void* qs, const void* scales, const uint8_t* xa,
                               int64_t rows, int64_t cols, int64_t row0, float* const* ys,
                               int32_t* const* counters, int64_t world, int64_t flags, void* stream) {
  if (format != DN_Q8 && format != DN_Q4) return DN_ERR_ARGS;
  if (rows < 0 || cols <= 0 || row0 < 0 || xa == nullptr || ys == nullptr || counters == nullptr ||
      world < 1 || world > dn::kMaxGatherRanks)
    return DN_ERR_ARGS;
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  dn::GemvArgs g{};
  g.q4 = format == DN_Q4;
  g.qs = qs;
  g.scales = scales;
  g.xa = xa;
  g.xa_stride = (cols / 32) * dn::kQABytes;
  g.ldy = rows;
  g.rows = rows;
  g.cols = cols;
  g.n = 1;
  g.status = d->status_dev;
  g.gather_n = (int)world;
  g.gather_row0 = row0;
  for (int64_t p = 0; p < world; p++) {
    g.gather_ys[p] = ys[p];
    g.gather_cnt[p] = reinterpret_cast<int*>(counters[p]);
  }
  return dn::launch_gemv_ex(g, static_cast<cudaStream_t>(stream), (flags & DN_FLAG_PDL) != 0);
}

int64_t dn_drain_probe(int64_t ctas, int64_t stages, float* out, void* stream) {
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  return dn::launch_drain_probe(ctas, stages, out, static_cast<cudaStream_t>(stream));
}

int64_t dn_peer_wait(const int32_t* counter, int32_t* expect, int64_t count, void* stream) {
  if (counter == nullptr || expect == nullptr || count < 0 || count > INT32_MAX / 2) return DN_ERR_ARGS;
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  return dn::launch_peer_wait(reinterpret_cast<const int*>(counter), reinterpret_cast<int*>(expect),
                              (int)count, d->status_dev, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? DN_OK
             : DN_ERR_CUDA;
}

int64_t dn_chain_create(int64_t format, const dn_chain_op* ops, int64_t nops, void** chain) {
  if ((format != DN_Q8 && format != DN_Q4) || ops == nullptr || chain == nullptr || nops <= 0)
    return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  static_assert(sizeof(dn_chain_op) == sizeof(dn::ChainOpSpec), "op layouts differ");
  dn::ChainHost* h = nullptr;
  const int64_t rc = dn::chain_create(reinterpret_cast<const dn::ChainOpSpec*>(ops), nops,
                                      format == DN_Q4, &h);
  *chain = rc == DN_OK ? h : nullptr;
  return rc;
}

int64_t dn_chain_create_sharded(int64_t format, const dn_chain_op* ops, const int64_t* row0,
                                const int64_t* total_rows, int64_t nops, int64_t rank,
                                int64_t world, void* const* bases, int64_t region_bytes,
                                int32_t* counters, void** chain) {
  if ((format != DN_Q8 && format != DN_Q4) || ops == nullptr || chain == nullptr || nops <= 0)
    return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  const dn::ChainShard shard{rank, world, reinterpret_cast<const void* const*>(bases),
                             region_bytes, reinterpret_cast<int*>(counters)};
  dn::ChainHost* h = nullptr;
  const int64_t rc = dn::chain_create_sharded(reinterpret_cast<const dn::ChainOpSpec*>(ops), row0,
                                              total_rows, nops, format == DN_Q4, shard, &h);
  *chain = rc == DN_OK ? h : nullptr;
  return rc;
}

int64_t dn_peer_alloc(int64_t bytes, void** ptr, void* handle) {
  if (bytes <= 0 || ptr == nullptr || handle == nullptr) return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  void* p = nullptr;
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == DN_PEER_HANDLE_BYTES, "IPC handle size");
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) {
    cudaGetLastError();
    return DN_ERR_CUDA;
  }
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return DN_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof h);
  *ptr = p;
  return DN_OK;
}

int64_t dn_peer_open(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return DN_ERR_ARGS;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return DN_ERR_CUDA;
  }
  *ptr = p;
  return DN_OK;
}

int64_t dn_peer_close(void* ptr) {
  if (ptr == nullptr) return DN_ERR_ARGS;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? DN_OK : DN_ERR_CUDA;
}

int64_t dn_peer_free(void* ptr) {
  if (ptr == nullptr) return DN_ERR_ARGS;
  return cudaFree(ptr) == cudaSuccess ? DN_OK : DN_ERR_CUDA;
}

int64_t dn_chain_run(void* chain, int64_t flags, void* stream) {
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  if (chain == nullptr) return DN_ERR_ARGS;
  return dn::chain_launch(static_cast<dn::ChainHost*>(chain), d->status_dev,
                          static_cast<cudaStream_t>(stream), (flags & DN_FLAG_PDL) != 0);
}

int64_t dn_chain_reset(void* chain, void* stream) {
  if (chain == nullptr) return DN_ERR_ARGS;
  return dn::chain_reset(static_cast<dn::ChainHost*>(chain), static_cast<cudaStream_t>(stream));
}

int64_t dn_chain_destroy(void* chain) {
  dn::chain_destroy(static_cast<dn::ChainHost*>(chain));
  return DN_OK;
}

int64_t dn_stack_create(int64_t format, const dn_stack_op* ops, int64_t nops, void** stack) {
  if (stack == nullptr) return DN_ERR_ARGS;
  *stack = nullptr;
  if ((format != DN_Q8 && format != DN_Q4) || ops == nullptr || nops <= 0) return DN_ERR_ARGS;
  if (format == DN_Q4) return DN_ERR_UNSUPPORTED;
  if (device_state() == nullptr) return DN_ERR_NO_DEVICE;
  static_assert(sizeof(dn_stack_op) == sizeof(dn::StackOpSpec), "op layouts differ");
  dn::StackHost* h = nullptr;
  const int64_t rc = dn::stack_create(reinterpret_cast<const dn::StackOpSpec*>(ops), nops, &h);
  *stack = rc == DN_OK ? h : nullptr;
  return rc;
}

int64_t dn_stack_run(void* stack, int64_t flags, void* stream) {
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  if (stack == nullptr) return DN_ERR_ARGS;
  return dn::stack_launch(static_cast<dn::StackHost*>(stack), d->status_dev,
                          static_cast<cudaStream_t>(stream), (flags & DN_FLAG_PDL) != 0);
}

int64_t dn_stack_reset(void* stack, void* stream) {
  if (stack == nullptr) return DN_ERR_ARGS;
  return dn::stack_reset(static_cast<dn::StackHost*>(stack), static_cast<cudaStream_t>(stream));
}

int64_t dn_stack_destroy(void* stack) {
  dn::stack_destroy(static_cast<dn::StackHost*>(stack));
  return DN_OK;
}

int64_t dn_last_error(void) {
  const int64_t e = tl_last_error;
  tl_last_error = DN_OK;
  return e;
}

int64_t dn_set_wait_limit_ns(int64_t ns) {
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  if (ns < 0) return DN_ERR_ARGS;
  const uint64_t v = ns == 0 ? 2000000000ull : (uint64_t)ns;
  bool ok = true;
  for (dn::WaitLimitSetter set : dn::wait_limit_setters()) ok = set(v) && ok;
  return ok ? DN_OK : DN_ERR_CUDA;
}

int64_t dn_device_status(int64_t clear) {
  DeviceState* d = device_state();
  if (d == nullptr) return DN_ERR_NO_DEVICE;
  volatile uint32_t* s = d->status_host;
  const int64_t v = *s;
  if (clear) *s = 0;
  return v;
}

const char* dn_error_string(int64_t code) {
  switch (code) {
    case DN_OK: return "ok";
    case DN_ERR_ARGS: return "invalid arguments";
    case DN_ERR_CUDA: return "CUDA runtime error";
    case DN_ERR_NO_DEVICE: return "no usable sm_100 device";
    case DN_ERR_UNSUPPORTED: return "unsupported combination";
    case DN_ERR_TOO_LARGE: return "size beyond the stated maximum";
    default: return "unknown error";
  }
}

}  // extern "C"
