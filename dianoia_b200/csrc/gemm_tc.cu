// Prefill / vision GEMM on the tcgen05 tensor cores: placeholder until the
// kind::i8 kernel lands; launch_linear never selects it while this returns
// false.
#include "dn_common.cuh"
#include "dn_launch.h"

namespace dn {

bool gemm_tc_supported(const LinearArgs&) { return false; }

int64_t launch_gemm_tc(const LinearArgs&, cudaStream_t) { return kErrUnsupported; }

}  // namespace dn
