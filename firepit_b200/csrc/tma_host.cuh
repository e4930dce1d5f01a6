// Host-side helpers shared by the tensor-core GEMMs (defined in gemm_nvfp4.cu).
#pragma once
#include <cuda.h>
#include <cstdint>

namespace fpb {
// 2-D byte tensor [rows, row_bytes] read in boxes of 128 bytes x box_rows with
// 128-byte swizzle; out-of-range elements read as zero.  FPB status.
int encode_rows_u8(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows);

// Output map for the GEMM epilogues' tiled stores: y [rows, cols] (bf16 or
// f32, row pitch ld elements), boxes of box_cols x box_rows (box_cols 0: 128
// bytes); 128-byte boxes use the 128-byte swizzle, narrower ones none.
// Returns false (no error recorded) when y cannot be stored that way (base or
// pitch not 16-byte aligned); the caller then stores directly.
bool encode_store_map(CUtensorMap *map, void *y, bool bf16, uint64_t rows, uint64_t cols, uint64_t ld,
                      uint32_t box_rows, uint32_t box_cols);
}  // namespace fpb
