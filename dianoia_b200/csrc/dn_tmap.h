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

// A 3-D view of a row-major byte array [rows, row_bytes] (row_bytes a
// multiple of 128) whose box is `chunks` consecutive 128-byte chunks of
// box_rows rows, 128-byte swizzled, landing in shared memory chunk by chunk:
// chunk j of row r at j * box_rows * 128 + r * 128 - the layout of `chunks`
// 2-D boxes of box_rows x 128 bytes, in one copy instead of `chunks`.
// Coordinates (x, y, z) = (byte in the chunk, row, chunk). Returns false if
// the driver refuses the map.
bool encode_tmap_row_chunks(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes,
                            uint32_t box_rows, uint32_t chunks);

}  // namespace dn
