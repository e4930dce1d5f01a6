/*
 * FP8 E4M3 part of the CPU oracle (test infrastructure only; see fp_oracle.h).
 *
 * Weight formats follow kernels src/weights/fp8.rs:8-27 (Fp8Scaling::Blocks
 * with a [rows/block_n, cols/block_k] f32 scale grid, or Fp8Scaling::Rows
 * with one f32 scale per row).  The quantizer has no reference counterpart:
 * its rule is the task's config 1 (scale = block_amax / 448, values rounded
 * to E4M3), the same rule for per-token activation scales.
 */
#include <math.h>
#include <string.h>

#include "fp_oracle.h"

static int fp8_quantize_grid(const float *w, size_t rows, size_t cols, size_t bn, size_t bk,
                             uint8_t *bits, float *scales) {
  int bad = 0;
  size_t gr = rows / bn, gc = cols / bk;
#pragma omp parallel for schedule(static) reduction(| : bad)
  for (size_t b = 0; b < gr * gc; ++b) {
    size_t r0 = (b / gc) * bn, c0 = (b % gc) * bk;
    float amax = 0.0f;
    for (size_t r = r0; r < r0 + bn; ++r)
      for (size_t c = c0; c < c0 + bk; ++c) {
        float v = w[r * cols + c];
        if (!isfinite(v)) bad = 1;
        float a = fabsf(v);
        if (a > amax) amax = a;
      }
    float s = amax / 448.0f;
    scales[b] = s;
    for (size_t r = r0; r < r0 + bn; ++r)
      for (size_t c = c0; c < c0 + bk; ++c)
        bits[r * cols + c] = s > 0.0f ? orc_f32_to_e4m3(w[r * cols + c] / s) : 0;
  }
  return bad ? -1 : 0;
}

int orc_fp8_quantize(const float *w, size_t rows, size_t cols, size_t block_n, size_t block_k,
                     uint8_t *bits, float *scales) {
  if (rows == 0 || cols == 0) return -1;
  if (block_n == 0 && block_k == 0) return fp8_quantize_grid(w, rows, cols, 1, cols, bits, scales);
  if (block_n == 0 || block_k == 0 || rows % block_n || cols % block_k) return -1;
  return fp8_quantize_grid(w, rows, cols, block_n, block_k, bits, scales);
}

void orc_fp8_dequantize(const uint8_t *bits, const float *scales, size_t rows, size_t cols,
                        size_t block_n, size_t block_k, float *out) {
  int row_mode = block_n == 0 && block_k == 0;
  size_t gc = row_mode ? 1 : cols / block_k;
#pragma omp parallel for schedule(static)
  for (size_t r = 0; r < rows; ++r)
    for (size_t c = 0; c < cols; ++c) {
      float s = row_mode ? scales[r] : scales[(r / block_n) * gc + c / block_k];
      out[r * cols + c] = orc_e4m3(bits[r * cols + c]) * s;
    }
}

void orc_fp8_gemm_f64(const uint8_t *a_bits, const float *a_scales, size_t m, const uint8_t *w_bits,
                      const float *w_scales, size_t n, size_t k, size_t block_n, size_t block_k,
                      double *expected, double *magnitude) {
  int row_mode = block_n == 0 && block_k == 0;
  size_t gc = row_mode ? 1 : k / block_k;
  double lut[256];
  for (int i = 0; i < 256; ++i) lut[i] = (double)orc_e4m3((uint8_t)i);
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < m; ++i) {
    for (size_t j = 0; j < n; ++j) {
      double e = 0.0, mag = 0.0;
      for (size_t c = 0; c < k; ++c) {
        double ws = row_mode ? (double)w_scales[j] : (double)w_scales[(j / block_n) * gc + c / block_k];
        double a = lut[a_bits[i * k + c]] * (double)a_scales[i];
        double w = lut[w_bits[j * k + c]] * ws;
        e += a * w;
        mag += fabs(a) * fabs(w);
      }
      expected[i * n + j] = e;
      magnitude[i * n + j] = mag;
    }
  }
}
