/*
 * MoE part of the CPU oracle (test infrastructure only; see fp_oracle.h).
 * Restates kernels src/moe.rs (top_k_prefill :15-68, PrefillLayout
 * :452-516, combine_prefill_kernel :91-109, combine_add_norm_kernel :111-147)
 * and src/swiglu.rs:16, in f32 in the reference kernels' operation order.
 */
#include <math.h>
#include <string.h>

#include "fp_oracle.h"

void orc_moe_topk(const float *logits, size_t ld, const float *shared_gate, size_t tokens, size_t experts,
                  size_t k, size_t width, int32_t *ids, float *weights) {
  float remaining[4096];
  for (size_t t = 0; t < tokens; ++t) {
    const float *row = logits + t * ld;
    float origin = -INFINITY;
    for (size_t e = 0; e < experts; ++e) {
      remaining[e] = row[e];
      if (row[e] > origin) origin = row[e];
    }
    float total = 0.0f, scores[32];
    int32_t sel[32];
    for (size_t r = 0; r < k; ++r) {
      float peak = -INFINITY;
      for (size_t e = 0; e < experts; ++e)
        if (remaining[e] > peak) peak = remaining[e];
      size_t winner = experts - 1;
      for (size_t e = 0; e < experts; ++e)
        if (remaining[e] == peak) {
          winner = e;
          break;
        }
      float score = expf(peak - origin);
      sel[r] = (int32_t)winner;
      scores[r] = score;
      total = total + score;
      remaining[winner] = -INFINITY;
    }
    for (size_t j = 0; j < width; ++j) {
      int32_t id = 0;
      float w = 0.0f;
      if (j < k) {
        id = sel[j];
        w = scores[j] / total;
      } else if (j == k && shared_gate) {
        id = (int32_t)experts;
        w = 1.0f / (1.0f + expf(shared_gate[t] * -1.0f));
      }
      ids[t * width + j] = id;
      weights[t * width + j] = w;
    }
  }
}

int orc_moe_layout(const int32_t *ids, size_t tokens, size_t width, size_t kk, size_t experts, size_t tile_rows,
                   size_t cap, int32_t *token_rows, int32_t *tile_experts, int32_t *inverse, int64_t *ranges,
                   int32_t *padded) {
  size_t counts[4096];
  if (experts > 4096) return -1;
  memset(counts, 0, sizeof(counts));
  for (size_t t = 0; t < tokens; ++t)
    for (size_t j = 0; j < kk; ++j) {
      int32_t id = ids[t * width + j];
      if (id < 0 || (size_t)id >= experts) return -1;
      counts[id]++;
    }
  size_t start = 0;
  for (size_t e = 0; e < experts; ++e) {
    ranges[2 * e] = (int64_t)start;
    ranges[2 * e + 1] = (int64_t)counts[e];
    start += (counts[e] + tile_rows - 1) / tile_rows * tile_rows;
  }
  if (start > cap) return -1;
  for (size_t r = 0; r < cap; ++r) token_rows[r] = -1;
  for (size_t r = 0; r < cap / tile_rows; ++r) tile_experts[r] = -1;
  for (size_t e = 0; e < experts; ++e) {
    size_t padded_e = (counts[e] + tile_rows - 1) / tile_rows * tile_rows;
    for (size_t r = (size_t)ranges[2 * e]; r < (size_t)ranges[2 * e] + padded_e; r += tile_rows)
      tile_experts[r / tile_rows] = (int32_t)e;
  }
  memset(inverse, 0, tokens * width * sizeof(int32_t));
  size_t cursor[4096];
  for (size_t e = 0; e < experts; ++e) cursor[e] = (size_t)ranges[2 * e];
  for (size_t t = 0; t < tokens; ++t)
    for (size_t j = 0; j < kk; ++j) {
      int32_t id = ids[t * width + j];
      size_t row = cursor[id]++;
      token_rows[row] = (int32_t)t;
      inverse[t * width + j] = (int32_t)row;
    }
  *padded = (int32_t)start;
  return 0;
}

void orc_swiglu(const float *gate_up, size_t rows, size_t inter, float *out) {
  for (size_t r = 0; r < rows; ++r)
    for (size_t c = 0; c < inter; ++c) {
      float g = gate_up[r * 2 * inter + c], u = gate_up[r * 2 * inter + inter + c];
      out[r * inter + c] = g / (1.0f + expf(g * -1.0f)) * u;
    }
}

void orc_moe_combine(const float *routed, size_t cols, const int32_t *inverse, const float *weights, size_t tokens,
                     size_t width, size_t slots, const float *residual, const float *gamma, float eps, float *out,
                     float *normed) {
  for (size_t t = 0; t < tokens; ++t) {
    double ss = 0.0;
    for (size_t c = 0; c < cols; ++c) {
      float sum = 0.0f;
      for (size_t s = 0; s < slots; ++s)
        sum = sum + routed[(size_t)inverse[t * width + s] * cols + c] * weights[t * width + s];
      if (residual) {
        sum = residual[t * cols + c] + sum;
        ss += (double)sum * (double)sum;
      }
      out[t * cols + c] = sum;
    }
    if (residual) {
      float scale = 1.0f / sqrtf((float)ss * (1.0f / (float)cols) + eps);
      for (size_t c = 0; c < cols; ++c) normed[t * cols + c] = out[t * cols + c] * scale * gamma[c];
    }
  }
}
