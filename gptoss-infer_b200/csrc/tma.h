// Host-side TMA tensor-map construction (driver entry point resolved through the runtime, no -lcuda needed at
// link time) with a small cache keyed by (pointer, shape), so repeated calls on the same weights reuse the map.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace gpt {

// 2-D uint8 tensor [rows][row_bytes] (row pitch = row_bytes, a multiple of 16), box [box_rows][box_bytes] with the
// 128-byte swizzle (box_bytes <= 128). Out-of-range box parts read as zero.
CUtensorMap make_tmap_u8_sw128(const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                               uint32_t box_rows);

// 3-D uint8 tensor [mats][rows][row_bytes], box [1][box_rows][box_bytes], 128-byte swizzle. Rows past `rows`
// within a matrix read as zero (no spill into the next matrix).
CUtensorMap make_tmap_u8_sw128_3d(const void* base, uint64_t row_bytes, uint64_t rows, uint64_t mats,
                                  uint32_t box_bytes, uint32_t box_rows);

// The same maps with a 64- or 128-byte swizzle (box_bytes <= swizzle_bytes): a 64-byte box of K lands in shared
// memory as 64-byte rows in the 64-byte swizzled K-major layout (8-row atoms of 512 bytes).
CUtensorMap make_tmap_u8_swz(const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                             uint32_t box_rows, uint32_t swizzle_bytes);
CUtensorMap make_tmap_u8_swz_3d(const void* base, uint64_t row_bytes, uint64_t rows, uint64_t mats,
                                uint32_t box_bytes, uint32_t box_rows, uint32_t swizzle_bytes);

}  // namespace gpt
