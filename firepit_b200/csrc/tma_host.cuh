// Host-side helpers shared by the tensor-core GEMMs (defined in gemm_nvfp4.cu).
#pragma once
#include <cuda.h>
#include <cstdint>

namespace fpb {
// 2-D byte tensor [rows, row_bytes] read in boxes of 128 bytes x box_rows with
// 128-byte swizzle; out-of-range elements read as zero.  FPB status.
int encode_rows_u8(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows);
}  // namespace fpb
