// Handle-owned GEMM-side layouts of an NVFP4 matrix (see matrix_extras.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "nvfp4_matrix.cuh"

namespace fpb {
struct MatrixExtras {
  // e4m3 block scales rearranged into the tcgen05 scale-factor tile layout
  // (sign cleared: the tensor cores read them as UE4M3).
  uint8_t *sf_tiled = nullptr;
  size_t sf_tiled_bytes = 0;
  // Codes with the sign of negative block scales folded in; null when no
  // scale is negative (the GEMM then reads the handle's own codes).
  uint8_t *packed_folded = nullptr;
  // TMA descriptor of the codes as read by the GEMM (opaque 128 bytes).
  alignas(64) unsigned char tmap_b[128];
  bool tmap_valid = false;
  // Fused gate/up + SwiGLU GEMM (stacked experts of 2*glu_inter rows, gate
  // rows first): the factors tiled over rows reordered so that each 128-row
  // tile holds gate rows [64b, 64b+64) then up rows [64b, 64b+64) of one
  // expert, and a TMA map of the codes in 64-row boxes (the two halves of a
  // tile are loaded separately, so the codes are not copied).
  uint8_t *sf_tiled_glu = nullptr;
  size_t glu_inter = 0;
  alignas(64) unsigned char tmap_b64[128];
};

// Builds the GEMM-side copies (tiled factors, sign-folded codes when a factor
// is negative, the codes' TMA map) once; allocates and synchronises `s`.
// Called when the matrix handle is created, so GEMM calls allocate nothing.
int prepare_gemm_weights(fpb_nvfp4_matrix *m, cudaStream_t s);
}  // namespace fpb
