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

// Token count from which the tensor-core GEMM replaces the GEMV.
static int64_t gemm_min_n() {
  static int64_t v = -1;
  if (v < 0) {
    const char* e = getenv("DN_GEMM_MIN_N");
    v = e ? atoll(e) : 16;
  }
  return v;
}

int path_for(const LinearArgs& a) {
  if (a.mode == 1 && a.n >= gemm_min_n() && gemm_tc_supported(a)) return 1;
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
