// Host-side MoE bookkeeping: dimension validation, selection validation and
// the expert-sorted prefill layout (crates/firepit-kernels/src/moe.rs).
// Pure host code; needs no GPU.
#include <climits>
#include <cmath>
#include <vector>

#include "common.cuh"

namespace fpb {

static bool is_pow2(size_t v) { return v && !(v & (v - 1)); }

static bool next_pow2_checked(size_t v, size_t *out) {
  size_t p = 1;
  while (p < v) {
    if (p > ((size_t)1 << 62)) return false;
    p <<= 1;
  }
  *out = p;
  return true;
}

}  // namespace fpb

using namespace fpb;

extern "C" {

// MoeDims::new (moe.rs:172-225).
int fpb_moe_dims_validate(size_t hidden, size_t intermediate, size_t shared_intermediate,
                          size_t experts, size_t top_k) {
  const size_t imax = (size_t)INT_MAX;
  size_t p;
  bool bad = hidden == 0 || intermediate == 0 || shared_intermediate != intermediate ||
             experts == 0 || top_k == 0 || top_k > experts || hidden % 32 || intermediate % 32 ||
             shared_intermediate % 32 || !is_pow2(hidden) || !is_pow2(intermediate) ||
             !is_pow2(shared_intermediate) || shared_intermediate > imax / 2 ||
             !next_pow2_checked(experts + 1, &p) || p > imax ||
             !next_pow2_checked(top_k + 1, &p) || p > imax ||
             hidden > imax / (experts + 1) || intermediate * 2 > imax / (experts + 1);
  if (bad)
    return fail(FPB_ERR_SHAPE, "invalid MoE dimensions (hidden=%zu intermediate=%zu shared=%zu experts=%zu top_k=%zu)",
                hidden, intermediate, shared_intermediate, experts, top_k);
  return FPB_OK;
}

// ExpertSelection::parse checks (moe.rs:327-351): exactly top_k entries,
// ids in range and distinct, weights finite, non-negative, positive sum.
int fpb_expert_selection_validate(const int32_t *indices, const float *weights, size_t count,
                                  size_t experts, size_t top_k) {
  if (!indices || !weights) return fail(FPB_ERR_INVALID_ARGUMENT, "null pointer");
  if (count != top_k) return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  std::vector<char> seen(experts, 0);
  for (size_t i = 0; i < count; ++i) {
    int32_t id = indices[i];
    if (id < 0 || (size_t)id >= experts) return fail(FPB_ERR_SELECTION, "invalid expert selection: Index");
    if (seen[id]) return fail(FPB_ERR_SELECTION, "invalid expert selection: Duplicate");
    seen[id] = 1;
  }
  float total = 0.0f;
  for (size_t i = 0; i < count; ++i) total += weights[i];
  for (size_t i = 0; i < count; ++i)
    if (!std::isfinite(weights[i]) || weights[i] < 0.0f)
      return fail(FPB_ERR_SELECTION, "invalid expert selection: Weight");
  if (!std::isfinite(total) || total <= 0.0f)
    return fail(FPB_ERR_SELECTION, "invalid expert selection: Weight");
  return FPB_OK;
}

// PrefillLayout::max_padded_rows (moe.rs:408-428).
int fpb_prefill_layout_max_padded_rows(size_t tokens, size_t experts, size_t top_k,
                                       size_t tile_rows, size_t *out) {
  if (!out) return fail(FPB_ERR_INVALID_ARGUMENT, "null pointer");
  if (tokens == 0 || tile_rows == 0 || !is_pow2(tile_rows))
    return fail(FPB_ERR_SELECTION, "invalid expert selection: Tile");
  if (top_k && tokens > SIZE_MAX / top_k) return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  size_t routes = tokens * top_k;
  size_t occupied = experts < routes ? experts : routes;
  if (occupied && (tile_rows - 1) > SIZE_MAX / occupied)
    return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  size_t pad = occupied * (tile_rows - 1);
  if (routes > SIZE_MAX - pad || routes + pad > (size_t)INT_MAX)
    return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  *out = routes + pad;
  return FPB_OK;
}

// PrefillLayout::parse + from_indices (moe.rs:430-516): a counting sort of
// the flattened [tokens, top_k] expert ids by expert, each expert's range
// padded to a multiple of tile_rows.  Outputs (caller-allocated):
//   token_rows   [padded_rows]   source token of each sorted row, -1 = padding
//   tile_experts [padded_rows / tile_rows]  expert of each row tile
//   inverse      [count]         sorted row of each (token, slot) entry
//   ranges       [2 * experts]   (start, count) per expert
// `weights` may be null (from_indices skips the weight checks).
int fpb_prefill_layout_host(const int32_t *indices, const float *weights, size_t count,
                            size_t experts, size_t top_k, size_t tile_rows, int32_t *token_rows,
                            size_t token_rows_cap, size_t *padded_rows, int32_t *tile_experts,
                            size_t tile_cap, size_t *n_tiles, int32_t *inverse, size_t *ranges) {
  if (top_k == 0 || experts == 0) return fail(FPB_ERR_SHAPE, "invalid MoE dimensions");
  if (count == 0 || count % top_k != 0) return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  if (!indices || !token_rows || !padded_rows || !tile_experts || !n_tiles || !inverse || !ranges)
    return fail(FPB_ERR_INVALID_ARGUMENT, "null pointer");
  if (weights) {
    for (size_t t = 0; t < count / top_k; ++t) {
      float total = 0.0f;
      bool bad = false;
      for (size_t j = 0; j < top_k; ++j) {
        float w = weights[t * top_k + j];
        total += w;
        if (!std::isfinite(w) || w < 0.0f) bad = true;
      }
      if (bad || !std::isfinite(total) || total <= 0.0f)
        return fail(FPB_ERR_SELECTION, "invalid expert selection: Weight");
    }
  }
  if (count > (size_t)INT_MAX) return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  if (tile_rows == 0 || tile_rows > (size_t)INT_MAX || !is_pow2(tile_rows))
    return fail(FPB_ERR_SELECTION, "invalid expert selection: Tile");
  size_t tokens = count / top_k;
  size_t width;
  if (!next_pow2_checked(top_k, &width) || tokens > (size_t)INT_MAX / width)
    return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  std::vector<size_t> last(experts, SIZE_MAX), counts(experts, 0);
  for (size_t t = 0; t < tokens; ++t) {
    for (size_t j = 0; j < top_k; ++j) {
      int32_t id = indices[t * top_k + j];
      if (id < 0 || (size_t)id >= experts) return fail(FPB_ERR_SELECTION, "invalid expert selection: Index");
      if (last[id] == t) return fail(FPB_ERR_SELECTION, "invalid expert selection: Duplicate");
      last[id] = t;
      counts[id]++;
    }
  }
  size_t start = 0, tiles = 0;
  for (size_t e = 0; e < experts; ++e) {
    ranges[2 * e] = start;
    ranges[2 * e + 1] = counts[e];
    size_t padded = (counts[e] + tile_rows - 1) / tile_rows * tile_rows;
    for (size_t t = 0; t < padded / tile_rows; ++t) {
      if (tiles >= tile_cap) return fail(FPB_ERR_WORKSPACE, "tile_experts capacity %zu too small", tile_cap);
      tile_experts[tiles++] = (int32_t)e;
    }
    start += padded;
    if (start > (size_t)INT_MAX) return fail(FPB_ERR_SELECTION, "invalid expert selection: Count");
  }
  if (start > token_rows_cap) return fail(FPB_ERR_WORKSPACE, "token_rows capacity %zu too small", token_rows_cap);
  for (size_t r = 0; r < start; ++r) token_rows[r] = -1;
  std::vector<size_t> cursor(experts);
  for (size_t e = 0; e < experts; ++e) cursor[e] = ranges[2 * e];
  for (size_t entry = 0; entry < count; ++entry) {
    int32_t id = indices[entry];
    size_t row = cursor[id]++;
    token_rows[row] = (int32_t)(entry / top_k);
    inverse[entry] = (int32_t)row;
  }
  *padded_rows = start;
  *n_tiles = tiles;
  return FPB_OK;
}

}  // extern "C"
