// Device-side FP8 weight matrix handle (Fp8Matrix, crates/firepit-kernels/
// src/weights/fp8.rs:14-19), shared by the FP8 GEMM (fp8.cu) and the FP8
// decode GEMV (gemv_fp8.cu).
#pragma once
#include <cstddef>
#include <cstdint>

struct fpb_fp8_matrix {
  size_t rows = 0, cols = 0;
  int block_n = 0, block_k = 0;  // 0, 0: one scale per row
  int device = 0;
  uint8_t *bits = nullptr;
  float *scales = nullptr;
  size_t n_scales = 0;
  alignas(64) unsigned char tmap[128];
  bool tmap_valid = false;
};
