// Host-side helpers shared by the tensor-core GEMMs (defined in gemm_nvfp4.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
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

// A GEMM on bf16 operands through the persistent tcgen05 kernel's bf16 mode:
// y [m, n] = b_globals[n] * sum over passes j of A_{a_sel[j]} . B_{b_sel[j]}^T
// (A [m, k], B [n, k] bf16 row-major, k % 8 == 0; b_globals null = 1).
struct F16Gemm {
  size_t m, n, k;
  const void *a[2];
  const void *b[2];
  int passes;
  int a_sel[3], b_sel[3];
  const float *b_globals;
  void *y;
  int y_bf16;
};
int run_f16_gemm(const F16Gemm &g, cudaStream_t s);
// Activations of the bf16 mode (bf16 x in place; f32 x split into bf16 hi
// and lo in `ws`, `used` bytes) and the workspace that split needs.
int hilo_activations(const void *x, int x_dtype, size_t m, size_t k, uint8_t *ws, const void **hi,
                     const void **lo, size_t *used, cudaStream_t s);
size_t hilo_workspace_bytes(size_t m, size_t k, int x_dtype);
}  // namespace fpb
