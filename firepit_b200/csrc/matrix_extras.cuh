// Handle-owned GEMM-side layouts of an NVFP4 matrix (see matrix_extras.cu).
#pragma once
#include <cstddef>
#include <cstdint>

#include "nvfp4_matrix.cuh"

namespace fpb {
struct MatrixExtras {
  // e4m3 block scales rearranged into the tcgen05 scale-factor tile layout.
  uint8_t *sf_tiled = nullptr;
  size_t sf_tiled_bytes = 0;
};
}  // namespace fpb
