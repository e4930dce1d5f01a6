// Device-side storage of an NVFP4 weight matrix (Nvfp4Matrix,
// crates/firepit-kernels/src/weights/nvfp4.rs:11-18).
//
// Layout in HBM, all row-major and owned by the handle:
//   packed      [rows, cols/2]  u8   two e2m1 codes, even column in the low nibble
//   scales      [rows, cols/16] u8   e4m3 block scale per 16 columns
//   row_globals [rows]          f32  per-row global (stacking keeps each part's)
// The GEMM path adds lazily built copies in tcgen05-friendly layouts
// (`extras`), freed with the handle.
#pragma once
#include <cstddef>
#include <cstdint>

namespace fpb {
constexpr int kNvfp4Group = 16;  // NVFP4_GROUP, weights/nvfp4.rs:8
constexpr int kQ8Block = 32;     // Q8_BLOCK, weights/q8_format.rs:3
struct MatrixExtras;
}  // namespace fpb

struct fpb_nvfp4_matrix {
  size_t rows = 0;
  size_t cols = 0;
  int device = 0;
  uint8_t *packed = nullptr;
  uint8_t *scales = nullptr;
  float *row_globals = nullptr;
  fpb::MatrixExtras *extras = nullptr;
};

namespace fpb {
// Frees `m->extras` (defined next to the code that builds them).
void release_matrix_extras(fpb_nvfp4_matrix *m);
}  // namespace fpb
