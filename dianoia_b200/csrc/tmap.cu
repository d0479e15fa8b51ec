// TMA tensor-map encoding (see dn_tmap.h).
#include <cudaTypedefs.h>

#include <mutex>

#include "dn_tmap.h"

namespace dn {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

static bool encode(CUtensorMap* map, const void* base, CUtensorMapDataType type, uint64_t row_elems,
                   uint64_t rows, uint64_t row_bytes, uint32_t box_elems, uint32_t box_rows,
                   CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {row_elems, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_elems, box_rows};
  const cuuint32_t estrides[2] = {1, 1};
  return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estrides,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType type, uint64_t row_elems,
                    uint64_t rows, uint64_t row_bytes, uint32_t box_elems, uint32_t box_rows,
                    bool swizzle128) {
  return encode(map, base, type, row_elems, rows, row_bytes, box_elems, box_rows,
                swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool encode_tmap_row_chunks(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes,
                            uint32_t box_rows, uint32_t chunks) {
  auto fn = encode_fn();
  if (fn == nullptr || row_bytes % 128 != 0) return false;
  // Dimensions innermost first: a 128-byte chunk, the rows, the chunks of a row.
  const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides[2] = {row_bytes, 128};
  const cuuint32_t box[3] = {128, box_rows, chunks};
  const cuuint32_t estrides[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estrides,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tmap_2d_sw64(CUtensorMap* map, const void* base, CUtensorMapDataType type,
                         uint64_t row_elems, uint64_t rows, uint64_t row_bytes, uint32_t box_elems,
                         uint32_t box_rows) {
  return encode(map, base, type, row_elems, rows, row_bytes, box_elems, box_rows,
                CU_TENSOR_MAP_SWIZZLE_64B);
}

}  // namespace dn
