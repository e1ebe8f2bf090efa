// Host helpers shared by the TMA-fed kernels: 2-D tensor maps for bf16 [rows, k] matrices and the
// SM count of the current device.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace ipe {

// A K-contiguous bf16 matrix [rows, k] read in boxes of box_k x box_rows with 128-byte swizzle
// (box_k * 2 must be 128). Returns false if the driver entry point is missing or the encode fails.
bool make_map_2d(CUtensorMap* map, const void* ptr, int rows, int k, int box_rows, int box_k);

// Slices of a K-contiguous bf16 array: `slices` matrices of `rows` rows (of k elements), slice s
// starting slice_rows * s rows in; rows >= `rows` of a slice read as zeros (TMA out-of-bounds fill),
// so a slice can stop short of its allocation. Boxes of box_k x box_rows x 1, 128-byte swizzle.
bool make_map_3d(CUtensorMap* map, const void* ptr, int k, int rows, int slices, int64_t slice_rows, int box_rows,
                 int box_k);

int sm_count();

}  // namespace ipe
