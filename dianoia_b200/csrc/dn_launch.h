// Host-side launchers of the quantized linear kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dn {

// Status codes returned by the launchers and the dn_* entry points.
enum : int64_t {
  kOk = 0,
  kErrArgs = -1,        // a shape, pointer or mode the entry point does not accept
  kErrCuda = -2,        // a CUDA runtime call failed (see dn_last_cuda_error)
  kErrNoDevice = -3,    // no usable sm_100 device
  kErrUnsupported = -4, // a combination this build does not implement
  kErrTooLarge = -5,    // a size beyond a stated maximum
};

struct LinearArgs {
  bool q4;              // Q4_0 (uint8 nibbles + fp16 scales) or Q8_0 (int8 + f32 scales)
  const void* qs;       // weights, [rows, cols] in the reference layout
  const void* scales;   // per-block scales, [rows, cols / 32]
  const float* xs;      // activations [n, cols]
  int8_t* xq;           // quantized activations out [n, cols] (mode 1; may be null on the fast path)
  float* xsc;           // their block scales out [n, cols / 32]
  float* ys;            // outputs, ys[t * ldy + r]
  int64_t rows, cols, n, ldy, mode;
  uint32_t* status;     // device word for bounded-wait timeouts (may be null)
};

// Quantized activations ("QA" blocks): per 32 values, the 32 int8 of
// lab_quantize_q8 followed by their f32 scale, 36 bytes. A decode chain hands
// these from one GEMV's epilogue to the next GEMV's prologue.
constexpr int kQABytes = 36;

constexpr int kMaxGatherRanks = 8;

struct GemvArgs {
  bool q4;
  const void* qs;
  const void* scales;
  const float* xs;        // f32 activations [n, cols] (quantized in the CTA), or null
  const uint8_t* xa;      // QA activations, token t at xa + t * xa_stride, or null
  int64_t xa_stride;
  int8_t* xq;             // with xs: lab_gemm's quantized inputs out (optional)
  float* xsc;
  float* ys;              // f32 outputs ys[t * ldy + r] (optional)
  int64_t ldy;
  uint8_t* ya;            // QA outputs, block r/32 of token t at ya + t * ya_stride (optional)
  int64_t ya_stride;
  int64_t rows, cols, n;
  uint32_t* status;
  // SwiGLU in the epilogue (optional): this product computes one of the
  // feed-forward's g and u, glu_other holds the other (same [n, ldy]
  // layout), and h = silu(g) * u goes to glu_out and, with ya, into the QA
  // outputs. With glu_self_gate this product's outputs are g (ys is then not
  // written: h replaces g); otherwise they are u, written to ys as usual.
  const float* glu_other;
  float* glu_out;
  bool glu_self_gate;
  // Residual add in the epilogue (optional): res[t * ldy + r] += y, after
  // the product's own outputs (the layer's dst += src right after it).
  float* res;
  // RMSNorm in the prologue (optional, with xs): the product's input is
  // token t of xs normalized with the weights norm_w and norm_eps (the norm
  // kernel's arithmetic); CTA 0 also writes those values to norm_out (token t
  // at norm_out + t * cols) unless it is null.
  const float* norm_w;
  float* norm_out;
  double norm_eps;
  // With f32 inputs (optional): CTA 0 also writes the quantized input as QA
  // blocks, token t at xa_out + t * xa_out_stride, for later products.
  uint8_t* xa_out;
  int64_t xa_out_stride;
  // A second matrix of the same shape in the same launch (optional, n = 1):
  // the feed-forward's up projection beside the gate in qs / scales. ys then
  // receives h = silu(gate) * up (and ya its QA blocks), ys2 the up outputs.
  const void* qs2;
  const void* scales2;
  float* ys2;
  // Several products of the same one-token input in one launch (optional,
  // 2 to kMaxGroups): product g has group_rows[g] rows of cols, weights at
  // group_qs[g] / group_scales[g], outputs at group_ys[g]; its 32-row tiles
  // start at tile group_tile0[g] (group_tile0[groups] = all tiles). No QA
  // outputs; qs, scales, ys and rows are then unused.
  int groups;
  int64_t group_rows[4];
  int64_t group_tile0[5];
  const void* group_qs[4];
  const void* group_scales[4];
  float* group_ys[4];
  // The all-gather of a row-sharded output fused into the epilogue
  // (optional; one token, f32 outputs): this product computes rows
  // gather_row0 .. gather_row0 + rows of the whole output, and stores each
  // into every rank's copy of it, gather_ys[p] + gather_row0 + row (rank p's
  // buffer as mapped on this GPU, plain stores over NVLink); then each CTA
  // adds its tile count to every rank's counter gather_cnt[p], after a
  // system-scope fence. 0 ranks: no gather.
  int gather_n;
  int64_t gather_row0;
  float* gather_ys[kMaxGatherRanks];
  int* gather_cnt[kMaxGatherRanks];
};
constexpr int kMaxGroups = 4;

// Waits, on the stream, until *cnt has grown by `count` since the previous
// wait with this `expect` word (device memory holding the value reached last
// time): one thread, bounded, a timeout recorded in the status word.
cudaError_t launch_peer_wait(const int* cnt, int* expect, int count, uint32_t* status, cudaStream_t stream);

// RMSNorm of `rows` rows of `cols` values: out = w * (x * r), r =
// 1 / sqrt(mean(x^2) + eps), added into out with `accumulate`; with qa, the
// results also as QA blocks, row t at qa + t * qa_stride (cols % 32 == 0).
struct NormArgs {
  const float* x;
  const float* w;
  float* out;
  uint8_t* qa;
  int64_t qa_stride;
  int64_t rows, cols;
  double eps;
  bool accumulate;
};
cudaError_t launch_rms_norm(const NormArgs& a, cudaStream_t stream, bool pdl);

// g = silu(g) * u over `count` values; with qa, also the QA blocks of the
// results, block b at qa + b * kQABytes (count % 32 == 0).
struct SwigluArgs {
  float* g;
  const float* u;
  uint8_t* qa;
  int64_t count;
};
cudaError_t launch_swiglu(const SwigluArgs& a, cudaStream_t stream, bool pdl);

// dst += src over `count` f32 values (the residual add).
cudaError_t launch_add(const float* src, float* dst, int64_t count, cudaStream_t stream, bool pdl);

// The rest of the decode layer (mixers.cu).
constexpr int64_t kMaxAttnKeys = 16384;  // keys one token attends to (scores in shared memory)
constexpr int kMaxConvTaps = 16;

cudaError_t launch_copy(const float* src, float* dst, int64_t count, cudaStream_t stream, bool pdl);

// Per (head, token): RMSNorm over hd values with weights w, then the
// half-split RoPE rotation from the token's table [cos(hd/2), sin(hd/2)].
// Head h of token t at x + t * x_stride + h * hd; the table at rope + t * rope_stride.
struct HeadNormRopeArgs {
  float* x;
  const float* w;
  const float* rope;
  int64_t x_stride, rope_stride, heads, hd, n;
  double eps;
  // A second set of heads in the same launch (optional; GpuForward's k after
  // its q): heads2 heads at x2 (stride x2_stride) with weights w2, the same
  // table, head size, tokens and eps.
  float* x2;
  const float* w2;
  int64_t x2_stride, heads2;
};
cudaError_t launch_head_norm_rope(const HeadNormRopeArgs& a, cudaStream_t stream, bool pdl);

// Causal grouped-query attention of n tokens at positions position ..
// position + n - 1 over the KV cache (rows [pos, kv_heads * hd]); q and out
// [n, heads * hd]; gate [n, heads] before the sigmoid, or null; window > 0
// keeps the current key and the window - 1 before it.
struct AttentionArgs {
  const float* q;
  const float* keys;
  const float* values;
  const float* gate;
  float* out;
  int64_t position, n, heads, kv_heads, hd, window;
};
cudaError_t launch_attention(const AttentionArgs& a, cudaStream_t stream, bool pdl);

// The gated short convolution: bcx [n, 3 * width] (B, C, X), weight
// [width, k], history [k - 1, width] (read and updated), y [n, width].
struct ConvArgs {
  const float* bcx;
  const float* weight;
  float* history;
  float* y;
  int64_t width, n;
  int k;
};
cudaError_t launch_conv(const ConvArgs& a, cudaStream_t stream, bool pdl);

// A control vector on `rows` rows of `cols` values: mode 0 adds v, mode 1
// subtracts scale * (x . v) * v.
struct SteerArgs {
  float* x;
  const float* v;
  int64_t rows, cols, mode;
  double scale;
};
cudaError_t launch_steer(const SteerArgs& a, cudaStream_t stream, bool pdl);

// The decode GEMV on either activation form (gemv.cu).
int64_t launch_gemv_ex(const GemvArgs& g, cudaStream_t stream, bool pdl);
bool gemv_ex_supported(const GemvArgs& g);
// The one-token product on QA inputs with plain outputs (gemv1.cu), which
// launch_gemv_ex picks for the products it can take.
bool gemv1_eligible(const GemvArgs& g);
int64_t launch_gemv1(const GemvArgs& g, cudaStream_t stream, bool pdl);
// f32 -> QA blocks (quantize.cu).
cudaError_t launch_quantize_qa(const float* xs, uint8_t* xa, int64_t n, int64_t cols,
                               int64_t xa_stride, cudaStream_t stream);

// Decode chains (chain.cu): the ops of a token run by one persistent kernel.
struct ChainOpSpec {
  const void* qs;
  const void* scales;
  const uint8_t* xa;   // QA input
  float* ys;           // f32 outputs or null
  uint8_t* ya;         // QA outputs or null
  int64_t rows, cols;
  int64_t dep;         // index of the op whose QA output xa is, or -1
};
struct ChainHost;
int64_t chain_create(const ChainOpSpec* specs, int64_t nops, bool q4, ChainHost** out);
// A chain whose ops are split by output rows over `world` GPUs: op i of this
// rank computes rows row0[i] .. row0[i] + rows of total_rows[i], and every
// tile's QA output goes to the same place in every rank's region
// (bases[p]: rank p's region as mapped here; the local one is bases[rank]);
// `counters` (nops + 2 ints) lies in the local region.
struct ChainShard {
  int64_t rank, world;
  const void* const* bases;
  int64_t region_bytes;
  int* counters;
};
int64_t chain_create_sharded(const ChainOpSpec* specs, const int64_t* row0,
                             const int64_t* total_rows, int64_t nops, bool q4,
                             const ChainShard& shard, ChainHost** out);
void chain_destroy(ChainHost* h);
int64_t chain_launch(ChainHost* h, uint32_t* status, cudaStream_t stream, bool pdl);
int64_t chain_reset(ChainHost* h, cudaStream_t stream);

// Decode stacks (stack.cu): a token's one-token Q8_0 products on f32
// activations run by one persistent kernel, each product's rows split evenly
// over every SM.
struct StackOpSpec {
  const void* qs;      // Q8_0 weights [rows, cols], reference layout
  const void* scales;  // f32 block scales [rows, cols / 32]
  const float* x;      // f32 input [cols]
  float* y;            // f32 output [rows]
  int64_t rows, cols;
  int64_t dep;         // index of an earlier op to wait for (its output may be x), or -1
};
struct StackHost;
int64_t stack_create(const StackOpSpec* specs, int64_t nops, StackHost** out);
void stack_destroy(StackHost* h);
int64_t stack_launch(StackHost* h, uint32_t* status, cudaStream_t stream, bool pdl);
int64_t stack_reset(StackHost* h, cudaStream_t stream);

// GGUF Q4_0 / Q8_0 blocks (count of them, 2-byte aligned) -> values (4-byte
// aligned) and scales, the engine's split layout (gguf.cu).
cudaError_t launch_gguf_split(bool q4, const void* blocks, int64_t count, void* qs, void* scales,
                              cudaStream_t stream);

// One token times a matrix of GGUF Q4_0 / Q8_0 blocks, read as stored
// (gguf_gemv.cu): QA input, f32 outputs.
int64_t launch_gguf_gemv(bool q4, const void* blocks, const uint8_t* xa, float* ys, int64_t rows, int64_t cols,
                         uint32_t* status, cudaStream_t stream, bool pdl);

// Quantizes n rows of cols floats to Q8_0 (lab_quantize_q8 semantics).
cudaError_t launch_quantize_q8(const float* xs, int8_t* xq, float* xsc, int64_t n, int64_t cols,
                               cudaStream_t stream);
// Quantizes weights to Q4_0 (lab_quantize_q4 semantics).
cudaError_t launch_quantize_q4(const float* w, uint8_t* qs, uint16_t* scales, int64_t rows,
                               int64_t cols, cudaStream_t stream);

// ys = W xs for all n tokens (lab_gemm_q8 / lab_gemm_q4 semantics). Picks the
// decode GEMV, the tensor-core GEMM or the generic kernel.
int64_t launch_linear(const LinearArgs& a, cudaStream_t stream);

// Individual paths (exposed for tests and benchmarks through dn_* symbols).
int64_t launch_gemv(const LinearArgs& a, cudaStream_t stream, bool pdl);
int64_t launch_generic(const LinearArgs& a, cudaStream_t stream);
int64_t launch_gemm_tc(const LinearArgs& a, cudaStream_t stream);

// The tensor-core GEMM on this GPU's row slice (rows row0 .. row0 + a.rows of
// the whole output, a.ldy values per token) with the all-gather fused into
// its epilogue: every value into every rank's copy ys[p], then, once the
// GEMM is complete, one count in every rank's cnt[p] (gemm_tc.cu).
int64_t launch_gemm_tc_allgather(const LinearArgs& a, int64_t row0, float* const* ys, int* const* cnt, int world,
                                 cudaStream_t stream);

// The tensor-core GEMM's drain step alone, for measuring its ceiling (gemm_tc.cu).
int64_t launch_drain_probe(int64_t ctas, int64_t nst, float* out, cudaStream_t stream);

// Which path launch_linear would pick (0 gemv, 1 tensor-core gemm, 2 generic).
int path_for(const LinearArgs& a);

}  // namespace dn
