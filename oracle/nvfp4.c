/* fp_oracle: NVFP4 quantize / dequantize / validate and the decode GEMV.
 * TEST INFRASTRUCTURE ONLY (see fp_oracle.h). */
#include "fp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define NVFP4_GROUP 16 /* kernels src/weights/nvfp4.rs:8 */
#define Q8_BLOCK 32    /* kernels src/weights/q8_format.rs:3 */
#define GEMV_KT 128    /* DEFAULT_GEMV_TILE.blocks (4) * Q8_BLOCK, kernels src/gemv/mod.rs:22-25 */

static inline uint8_t code_at(const uint8_t *packed, size_t row, size_t cols, size_t col) {
  /* firepit src/checkpoint.rs:414-418: even column in the low nibble. */
  uint8_t pair = packed[row * (cols / 2) + col / 2];
  return (col & 1) ? (uint8_t)(pair >> 4) : (uint8_t)(pair & 0xf);
}

int orc_nvfp4_quantize(const float *w, size_t rows, size_t cols, size_t rows_per_global,
                       uint8_t *packed, uint8_t *scales, float *row_globals) {
  if (rows == 0 || cols == 0 || cols % NVFP4_GROUP || rows_per_global == 0 ||
      rows % rows_per_global)
    return -1;
  size_t blocks = rows / rows_per_global;
  int bad = 0;
  for (size_t b = 0; b < blocks; ++b) {
    const float *wb = w + b * rows_per_global * cols;
    float amax = 0.0f;
    for (size_t i = 0; i < rows_per_global * cols; ++i) {
      if (!isfinite(wb[i])) bad = 1;
      float a = fabsf(wb[i]);
      if (a > amax) amax = a;
    }
    float global = amax / 2688.0f; /* amax / (6 * 448) */
    for (size_t r = b * rows_per_global; r < (b + 1) * rows_per_global; ++r) {
      row_globals[r] = global;
      for (size_t g = 0; g < cols / NVFP4_GROUP; ++g) {
        const float *v = w + r * cols + g * NVFP4_GROUP;
        float bmax = 0.0f;
        for (int i = 0; i < NVFP4_GROUP; ++i) {
          float a = fabsf(v[i]);
          if (a > bmax) bmax = a;
        }
        uint8_t s = 0;
        if (global > 0.0f) {
          float ratio = bmax / 6.0f;
          s = orc_f32_to_e4m3(ratio / global);
        }
        scales[r * (cols / NVFP4_GROUP) + g] = s;
        float denom = orc_e4m3(s) * global;
        for (int i = 0; i < NVFP4_GROUP; i += 2) {
          uint8_t lo = 0, hi = 0;
          if (denom > 0.0f) {
            lo = orc_f32_to_e2m1(v[i] / denom);
            hi = orc_f32_to_e2m1(v[i + 1] / denom);
          }
          packed[r * (cols / 2) + (g * NVFP4_GROUP + i) / 2] = (uint8_t)(lo | (hi << 4));
        }
      }
    }
  }
  return bad ? -1 : 0;
}

void orc_nvfp4_dequantize(const uint8_t *packed, const uint8_t *scales,
                          const float *row_globals, size_t rows, size_t cols, float *out) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    for (size_t c = 0; c < cols; ++c) {
      float s = orc_e4m3(scales[r * (cols / NVFP4_GROUP) + c / NVFP4_GROUP]);
      float sg = s * row_globals[r];
      out[r * cols + c] = orc_e2m1_modelopt(code_at(packed, r, cols, c)) * sg;
    }
  }
}

int orc_nvfp4_validate(size_t packed_len, const uint8_t *scales, size_t scales_len,
                       const float *row_globals, size_t rows, size_t cols) {
  /* kernels src/weights/nvfp4.rs:42-64 (row globals are the per-row form that
   * stack() builds, :84-97). */
  if (rows == 0 || cols == 0 || cols % Q8_BLOCK) return -1;
  if (packed_len != rows * (cols / 2) || scales_len != rows * (cols / NVFP4_GROUP)) return -1;
  for (size_t i = 0; i < scales_len; ++i)
    if ((scales[i] & 0x7f) == 0x7f) return -1;
  for (size_t r = 0; r < rows; ++r)
    if (!isfinite(row_globals[r]) || row_globals[r] < 0.0f) return -1;
  return 0;
}

void orc_nvfp4_gemv_f32(const uint8_t *packed, const uint8_t *scales, const float *row_globals,
                        size_t rows, size_t cols, const float *x, size_t batch, float *y) {
  /* kernels src/gemv/nvfp4.rs:34-59 with KT = 128: for each chunk, per
   * 16-group sum of E2M1*x (f32), times the e4m3 scale, summed over the
   * chunk, added to the accumulator; finally times the row scale.  The
   * reference reduces within a group with a tree; this restatement sums
   * left to right. */
  size_t gpr = cols / NVFP4_GROUP;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    const uint8_t *prow = packed + (size_t)r * (cols / 2);
    const uint8_t *srow = scales + (size_t)r * gpr;
    for (size_t b = 0; b < batch; ++b) {
      const float *xb = x + b * cols;
      float acc = 0.0f;
      for (size_t k0 = 0; k0 < cols; k0 += GEMV_KT) {
        size_t k1 = k0 + GEMV_KT < cols ? k0 + GEMV_KT : cols;
        float chunk = 0.0f;
        for (size_t g = k0 / NVFP4_GROUP; g < k1 / NVFP4_GROUP; ++g) {
          float gsum = 0.0f;
          for (int i = 0; i < NVFP4_GROUP; i += 2) {
            uint8_t pair = prow[(g * NVFP4_GROUP + i) / 2];
            float w0 = orc_e2m1_test(pair & 0xf), w1 = orc_e2m1_test(pair >> 4);
            float p0 = w0 * xb[g * NVFP4_GROUP + i];
            gsum = gsum + p0;
            float p1 = w1 * xb[g * NVFP4_GROUP + i + 1];
            gsum = gsum + p1;
          }
          float sg = gsum * orc_e4m3(srow[g]);
          chunk = chunk + sg;
        }
        acc = acc + chunk;
      }
      y[b * rows + r] = acc * row_globals[r];
    }
  }
}

void orc_nvfp4_gemv_f64(const uint8_t *packed, const uint8_t *scales, const float *row_globals,
                        size_t rows, size_t cols, const float *x, size_t batch,
                        double *expected, double *magnitude) {
  /* kernels tests/nvfp4_oracle.rs:75-101: block_scaled = e2m1(code) *
   * e4m3(scale) in f32 (exact), dot product in f64, then times the global. */
  size_t gpr = cols / NVFP4_GROUP;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    for (size_t b = 0; b < batch; ++b) {
      double e = 0.0, m = 0.0;
      for (size_t c = 0; c < cols; ++c) {
        float w = orc_e2m1_test(code_at(packed, (size_t)r, cols, c)) *
                  orc_e4m3(scales[(size_t)r * gpr + c / NVFP4_GROUP]);
        double xv = (double)x[b * cols + c];
        e += (double)w * xv;
        m += fabs((double)w) * fabs(xv);
      }
      expected[b * rows + r] = e * (double)row_globals[r];
      magnitude[b * rows + r] = m * (double)row_globals[r];
    }
  }
}

void orc_nvfp4_expert_gemv_f32(const uint8_t *packed, const uint8_t *scales,
                               const float *row_globals, size_t cols, const int32_t *ids,
                               size_t slots, size_t rows_per_expert, size_t input_stride,
                               const float *x, float *y) {
  /* kernels src/gemv/nvfp4.rs:62-107: row tile = expert * row_tiles + pid.1,
   * input row = slot * input_stride. */
  for (size_t s = 0; s < slots; ++s) {
    size_t base = (size_t)ids[s] * rows_per_expert;
    orc_nvfp4_gemv_f32(packed + base * (cols / 2), scales + base * (cols / NVFP4_GROUP),
                       row_globals + base, rows_per_expert, cols, x + s * input_stride * cols, 1,
                       y + s * rows_per_expert);
  }
}
