// Path selection for ys = W xs (lab_gemm_q8 / lab_gemm_q4 semantics).
//
//   decode GEMV (gemv.cu)        mode 1, aligned, small n: bit-exact with the
//                                reference's f32 outputs
//   tensor-core GEMM (gemm_tc.cu) mode 1, aligned, n above the crossover:
//                                bit-exact int32 block dots, f32 within the
//                                reference's 1e-5 relative bound
//   generic (gemv.cu)            anything else (mode 0, unaligned pointers,
//                                cols not a multiple of 32): bit-exact, slow
#include "dn_common.cuh"
#include "dn_launch.h"

namespace dn {

bool gemv_supported(const LinearArgs& a);
bool gemm_tc_supported(const LinearArgs& a);

// Token count from which the tensor-core GEMM replaces the GEMV: 16, or 5
// for a matrix of at least 32768 rows (the lm_head), where the GEMM's
// narrow-tile kernel streams the weights faster than the n-token GEMV
// (151936 x 2048 Q8 at M = 8: 86 against 124 us; at M = 4 the GEMV still
// wins, 73 against 82 us). DN_GEMM_MIN_N sets one crossover for all shapes.
static int64_t gemm_min_n(int64_t rows) {
  static int64_t v = -2;
  if (v == -2) {
    const char* e = getenv("DN_GEMM_MIN_N");
    v = e ? atoll(e) : -1;
  }
  if (v >= 0) return v;
  return rows >= 32768 ? 5 : 16;
}

int path_for(const LinearArgs& a) {
  if (a.mode == 1 && a.n >= gemm_min_n(a.rows) && gemm_tc_supported(a)) return 1;
  if (gemv_supported(a)) return 0;
  return 2;
}

int64_t launch_linear(const LinearArgs& a, cudaStream_t stream) {
  if (a.rows < 0 || a.cols < 0 || a.n < 0 || (a.mode != 0 && a.mode != 1)) return kErrArgs;
  if (a.ldy < a.rows) return kErrArgs;
  switch (path_for(a)) {
    case 1: return launch_gemm_tc(a, stream);
    case 0: return launch_gemv(a, stream, false);
    default: return launch_generic(a, stream);
  }
}

}  // namespace dn
