// Host side of the TMA tensor copies: tensor maps encoded through the
// driver entry point the CUDA runtime exposes (no link against the driver
// library).
#pragma once

#include <cuda.h>

namespace vqmoe {

// Row-major [rows][cols] of 2-byte elements (row pitch cols * 2, a multiple
// of 16; base 16-byte aligned): boxes of box_rows rows x 64 columns (128
// bytes) with the 128-byte swizzle; out-of-range elements read as zero.
bool make_tma_map(CUtensorMap *m, const void *base, int rows, int cols, int box_rows);

}  // namespace vqmoe
