// tmap.hpp -- host-side creation of TMA tensor maps for packed weights and
// their group metadata (scales / biases).
//
// A row-major matrix of 16-bit elements with `row_bytes` per row is described
// as a 3-D tensor
//   dim0 = 64 elements (one 128-byte piece of a row)
//   dim1 = row            (stride = row pitch)
//   dim2 = 128-byte piece (stride = 128 bytes)
// with the 128-byte swizzle. A box {64, 8, n} then lands in shared memory as
// n atoms of 1024 bytes, atom j holding piece j of 8 consecutive rows, the
// 16-byte unit u of row r stored at unit position (u ^ r). A warp reading
// "row = lane / 4, 4-byte word = lane % 4" of one unit takes one
// conflict-free wavefront, and each TMA request moves whole 128-byte lines.
// Rows whose length is not a multiple of 128 bytes use a plain 2-D box
// {row_bytes / 2, 8} instead (`swizzled == false`).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace b2q {

// box_bytes = bytes of each row the box covers (one reduction chunk).
int make_row_block_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_bytes,
                       bool swizzled);

// Same 3-D swizzled form with a box of `box_rows` rows x the whole row
// (row_bytes / 128 pieces): one copy brings every reduction value of a block
// of rows, landing as [piece][box_rows][128 bytes].
int make_row_tile_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows);

// Plain 2-D map over a row-major matrix of 16-bit elements: box of
// `box_bytes` per row x `box_rows` rows, swizzle 0, 32, 64 or 128 bytes.
int make_2d_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_bytes,
                uint32_t box_rows, int swizzle_bytes);

}  // namespace b2q
