// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry point so the library does not link
// libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dn {

// A 2-D tiled map over a row-major [rows, row_elems] array with `row_bytes`
// between rows: boxes of box_rows x box_elems, 128-byte swizzled when
// `swizzle128` (box_elems * element size must then be 128 bytes). Returns
// false if the driver refuses the map (alignment, sizes).
bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType type, uint64_t row_elems,
                    uint64_t rows, uint64_t row_bytes, uint32_t box_elems, uint32_t box_rows,
                    bool swizzle128);

// The same with a 64-byte swizzle (box_elems * element size must be 64
// bytes): in a box with 64-byte rows, the 16-byte chunk j of row r sits at
// r * 64 + ((j ^ (r / 2)) % 4) * 16.
bool encode_tmap_2d_sw64(CUtensorMap* map, const void* base, CUtensorMapDataType type,
                         uint64_t row_elems, uint64_t rows, uint64_t row_bytes, uint32_t box_elems,
                         uint32_t box_rows);

}  // namespace dn
