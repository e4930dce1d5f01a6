// MoE routing, layout, gather, SwiGLU and combine on the device
// (crates/firepit-kernels/src/moe.rs:15-147, 397-859; src/swiglu.rs).
//
// The reference computes the router's top-k on the GPU, downloads the ids,
// builds the expert-sorted layout on the host (a counting sort) and uploads it
// again (PrefillPlan::top_k, moe.rs:545-585).  Here every step stays on the
// device, so a prefill MoE is one stream of launches with no host round trip:
//   top-k (one warp per token) -> layout (stable counting sort over CTAs) ->
//   gather + NVFP4 quantize -> grouped gate/up GEMM -> SwiGLU + NVFP4
//   quantize -> grouped down GEMM -> combine (+ residual + RMSNorm).
// The layout is written into buffers sized for the largest possible padding
// (PrefillLayout::max_padded_rows); row tiles past the actual end carry
// expert id -1, which the grouped GEMMs skip.
#include <algorithm>
#include <mutex>
#include <vector>

#include "act_quant.cuh"
#include <type_traits>

#include "common.cuh"
#include "nvfp4_matrix.cuh"

namespace fpb {

// ---- router top-k (moe.rs:15-68) -------------------------------------------------------
// One warp per token; lane l holds logits l, l + 32, ...  Each of the k
// rounds takes the largest remaining logit, the lowest expert id among equal
// ones; scores exp(l - max) are normalised by their sum over the k winners
// (softmax restricted to the top k).  With a shared-expert gate, slot k is
// expert `experts` with weight sigmoid(gate).  Slots past that are id 0,
// weight 0.
// Float -> unsigned key with the same order (-inf lowest); NaN is never
// offered (the loads below turn it into -inf, so it is never chosen, as with
// the comparisons of the reference's loop).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Top-k of one token's logits `row` by one warp (lane l: logits l, l + 32,
// ...); `gate`: the token's shared-expert gate logit or null.
template <int PER_LANE>
__device__ __forceinline__ void topk_warp(const float *row, const float *gate, int experts, int k, int width,
                                          int32_t *ids_row, float *weights_row) {
  const int lane = threadIdx.x & 31;
  float v[PER_LANE];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int p = lane + 32 * i;
    v[i] = p < experts ? row[p] : -INFINITY;
    if (v[i] != v[i]) v[i] = -INFINITY;  // NaN never wins a comparison
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float origin = m;
  float total = 0.0f, my_score = 0.0f;
  int my_id = 0;
  for (int rank = 0; rank < k; ++rank) {
    float bv = -INFINITY;
    int bp = experts - 1;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int p = lane + 32 * i;
      if (p < experts && (v[i] > bv || (v[i] == bv && p < bp))) {
        bv = v[i];
        bp = p;
      }
    }
    // Warp arg-max in two hardware reductions: the largest value (as an
    // order-preserving unsigned key), then the lowest id holding it.
    const uint32_t key = order_key(bv);
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
    bp = (int)__reduce_min_sync(0xffffffffu, key == kmax ? (uint32_t)bp : 0xffffffffu);
    bv = order_key_value(kmax);
    const float score = expf(bv - origin);
    total = total + score;
    if (lane == rank) {
      my_score = score;
      my_id = bp;
    }
    if ((bp & 31) == lane) {
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i)
        if (lane + 32 * i == bp) v[i] = -INFINITY;
    }
  }
  if (lane < width) {
    int id = 0;
    float w = 0.0f;
    if (lane < k) {
      id = my_id;
      w = my_score / total;
    } else if (lane == k && gate) {
      id = experts;
      const float g = *gate;
      w = 1.0f / (1.0f + expf(g * -1.0f));
    }
    ids_row[lane] = id;
    weights_row[lane] = w;
  }
}

template <int PER_LANE>
__global__ void moe_topk_kernel(const float *logits, long long ld, const float *shared_gate, int tokens,
                                int experts, int k, int width, int32_t *ids, float *weights) {
  pdl_enter();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (warp >= tokens) return;
  topk_warp<PER_LANE>(logits + (long long)warp * ld, shared_gate ? shared_gate + warp : nullptr, experts, k, width,
                      ids + (long long)warp * width, weights + (long long)warp * width);
}

// ---- layout: stable counting sort (moe.rs:452-516) -------------------------------------
// Multi-CTA: CTA g owns the contiguous route range [g * kLayoutChunk, ...).
//  1. count: per-CTA histogram of expert ids (shared-memory atomics) -> cnt[g][e];
//  2. scan (one CTA): per expert, cnt[g][e] -> the CTA's first row within the
//     expert (exclusive over g); padded expert ranges (exclusive over e); tile
//     experts; the row count;
//  3. place: per CTA, ranks that keep the routes' order (per-warp counts over
//     contiguous warp segments, __match_any_sync within a batch), so every
//     expert's rows follow the (token, slot) order: the reference's stable sort.
// The fills (token_rows = -1, tile_experts = -1, inverse = 0, or -1 in a
// masked layout) are memsets.
constexpr int kLayoutChunk = 1024;  // routes per CTA
constexpr int kLayoutWarpsPerCta = 8;

// The route's expert, -1 for an id outside [0, experts) (a device error), or
// -2 for the id -1 in a masked layout (a route that is not there: the
// expert-parallel receiver marks the slots it does not own that way).
__device__ __forceinline__ int layout_id(const int32_t *ids, int e, int kk, int width, int experts, bool masked) {
  const int id = ids[(long long)(e / kk) * width + e % kk];
  if (id >= 0 && id < experts) return id;
  return (masked && id == -1) ? -2 : -1;
}

__global__ void __launch_bounds__(256) moe_layout_count_kernel(const int32_t *ids, int n, int kk, int width,
                                                               int experts, int *cnt, int *error, bool masked) {
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int lo = blockIdx.x * kLayoutChunk, hi = min(n, lo + kLayoutChunk);
  for (int e = lo + threadIdx.x; e < hi; e += blockDim.x) {
    const int id = layout_id(ids, e, kk, width, experts, masked);
    if (id >= 0)
      atomicAdd(&hist[id], 1);
    else if (id == -1 && error)
      atomicCAS(error, 0, 401);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < experts; e += blockDim.x) cnt[(size_t)blockIdx.x * experts + e] = hist[e];
}

__global__ void __launch_bounds__(1024) moe_layout_scan_kernel(int *cnt, int groups, int experts, int tile_rows,
                                                               int cap, int32_t *tile_experts, int64_t *ranges,
                                                               int32_t *padded_out, int *error) {
  extern __shared__ int totals[];  // [experts]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int x = tid; x < experts; x += blockDim.x) {
    int run = 0, g = 0;
    for (; g + 8 <= groups; g += 8) {  // eight independent loads in flight
      int c[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) c[u] = cnt[(size_t)(g + u) * experts + x];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        cnt[(size_t)(g + u) * experts + x] = run;
        run += c[u];
      }
    }
    for (; g < groups; ++g) {
      const int c = cnt[(size_t)g * experts + x];
      cnt[(size_t)g * experts + x] = run;
      run += c;
    }
    totals[x] = run;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < experts; base += 32) {
      const int x = base + lane;
      const int total = x < experts ? totals[x] : 0;
      const int padded = (total + tile_rows - 1) / tile_rows * tile_rows;
      int incl = padded;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (x < experts) {
        ranges[2 * x] = carry + incl - padded;
        ranges[2 * x + 1] = total;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      *padded_out = carry;
      if (carry > cap && error) atomicCAS(error, 0, 402);
    }
  }
  __syncthreads();
  for (int x = tid; x < experts; x += blockDim.x) {
    const int start = (int)ranges[2 * x], count = totals[x];
    const int padded = (count + tile_rows - 1) / tile_rows * tile_rows;
    for (int t = start / tile_rows; t < (start + padded) / tile_rows && t < cap / tile_rows; ++t)
      tile_experts[t] = x;
  }
}

__global__ void __launch_bounds__(kLayoutWarpsPerCta * 32) moe_layout_place_kernel(
    const int32_t *ids, int n, int kk, int width, int experts, int cap, const int *cnt, const int64_t *ranges,
    int32_t *token_rows, int32_t *inverse, bool masked) {
  extern __shared__ int wcount[];  // [kLayoutWarpsPerCta][experts]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kLayoutWarpsPerCta * experts; i += blockDim.x) wcount[i] = 0;
  __syncthreads();
  const int lo = blockIdx.x * kLayoutChunk, hi = min(n, lo + kLayoutChunk);
  constexpr int kWarpSpan = kLayoutChunk / kLayoutWarpsPerCta;
  const int w_lo = min(hi, lo + warp * kWarpSpan), w_hi = min(hi, w_lo + kWarpSpan);
  for (int b = w_lo; b < w_hi; b += 32) {
    const int e = b + lane;
    const int id = e < w_hi ? layout_id(ids, e, kk, width, experts, masked) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, id);
    if (id >= 0 && lane == __ffs(grp) - 1) wcount[warp * experts + id] += __popc(grp);
    __syncwarp();
  }
  __syncthreads();
  // each warp's first row per expert: expert start + earlier CTAs' rows + earlier warps'
  for (int x = tid; x < experts; x += blockDim.x) {
    int run = (int)ranges[2 * x] + cnt[(size_t)blockIdx.x * experts + x];
    for (int w = 0; w < kLayoutWarpsPerCta; ++w) {
      const int c = wcount[w * experts + x];
      wcount[w * experts + x] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int b = w_lo; b < w_hi; b += 32) {
    const int e = b + lane;
    const int id = e < w_hi ? layout_id(ids, e, kk, width, experts, masked) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, id);
    const int rank = __popc(grp & ((1u << lane) - 1));
    int pos = -1;
    if (id >= 0) pos = wcount[warp * experts + id] + rank;
    __syncwarp();
    if (id >= 0 && lane == __ffs(grp) - 1) wcount[warp * experts + id] += __popc(grp);
    if (id >= 0 && pos < cap) {
      token_rows[pos] = e / kk;
      inverse[(long long)(e / kk) * width + e % kk] = pos;
    }
    __syncwarp();
  }
}

// Single-CTA layout for launches of at most kLayoutChunk routes (decode-size
// batches): the fills, the per-warp counts, both scans and the stable
// placement of the three kernels above in one launch (one graph node instead
// of three memsets and three kernels).  Same outputs and device errors.
constexpr int kLayoutSmallThreads = 1024;
__global__ void __launch_bounds__(kLayoutSmallThreads) moe_layout_small_kernel(
    const int32_t *ids, int n, int kk, int width, int tokens, int experts, int tile_rows, int cap,
    int32_t *token_rows, int32_t *tile_experts, int32_t *inverse, int64_t *ranges, int32_t *padded_out, int *error,
    bool masked) {
  pdl_enter();
  extern __shared__ int sm_small[];
  constexpr int kWarps = kLayoutSmallThreads / 32;
  int *wcount = sm_small;                     // [kWarps][experts]
  int *totals = sm_small + kWarps * experts;  // [experts]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // fills (token_rows = -1, tile_experts = -1, inverse = 0) and zeroed counts;
  // token_rows (cap is a multiple of the tile rows) in 16-byte stores when aligned
  if ((reinterpret_cast<uintptr_t>(token_rows) & 15) == 0 && (cap & 3) == 0) {
    int4 *t4 = reinterpret_cast<int4 *>(token_rows);
    for (int i = tid; i < cap / 4; i += blockDim.x) t4[i] = make_int4(-1, -1, -1, -1);
  } else {
    for (int i = tid; i < cap; i += blockDim.x) token_rows[i] = -1;
  }
  for (int i = tid; i < cap / tile_rows; i += blockDim.x) tile_experts[i] = -1;
  const int inv_fill = masked ? -1 : 0;
  for (int i = tid; i < tokens * width; i += blockDim.x) inverse[i] = inv_fill;
  for (int i = tid; i < kWarps * experts; i += blockDim.x) wcount[i] = 0;
  __syncthreads();
  // each warp counts a contiguous segment of the routes
  const int span = (n + kWarps - 1) / kWarps;
  const int w_lo = min(n, warp * span), w_hi = min(n, w_lo + span);
  for (int b = w_lo; b < w_hi; b += 32) {
    const int e = b + lane;
    const int id = e < w_hi ? layout_id(ids, e, kk, width, experts, masked) : -1;
    if (e < w_hi && id == -1 && error) atomicCAS(error, 0, 401);
    const unsigned grp = __match_any_sync(0xffffffffu, id);
    if (id >= 0 && lane == __ffs(grp) - 1) wcount[warp * experts + id] += __popc(grp);
    __syncwarp();
  }
  __syncthreads();
  // per expert: each warp's first row within the expert, and the total
  for (int x = tid; x < experts; x += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kWarps; ++w) {
      const int c = wcount[w * experts + x];
      wcount[w * experts + x] = run;
      run += c;
    }
    totals[x] = run;
  }
  __syncthreads();
  // padded expert ranges (exclusive over experts), the row count
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < experts; base += 32) {
      const int x = base + lane;
      const int total = x < experts ? totals[x] : 0;
      const int padded = (total + tile_rows - 1) / tile_rows * tile_rows;
      int incl = padded;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (x < experts) {
        ranges[2 * x] = carry + incl - padded;
        ranges[2 * x + 1] = total;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      *padded_out = carry;
      if (carry > cap && error) atomicCAS(error, 0, 402);
    }
  }
  __syncthreads();
  for (int x = tid; x < experts; x += blockDim.x) {
    const int start = (int)ranges[2 * x], count = totals[x];
    const int padded = (count + tile_rows - 1) / tile_rows * tile_rows;
    for (int t = start / tile_rows; t < (start + padded) / tile_rows && t < cap / tile_rows; ++t) tile_experts[t] = x;
    for (int w = 0; w < kWarps; ++w) wcount[w * experts + x] += start;
  }
  __syncthreads();
  // stable placement: (token, slot) order within each expert
  for (int b = w_lo; b < w_hi; b += 32) {
    const int e = b + lane;
    const int id = e < w_hi ? layout_id(ids, e, kk, width, experts, masked) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, id);
    const int rank = __popc(grp & ((1u << lane) - 1));
    int pos = -1;
    if (id >= 0) pos = wcount[warp * experts + id] + rank;
    __syncwarp();
    if (id >= 0 && lane == __ffs(grp) - 1) wcount[warp * experts + id] += __popc(grp);
    if (id >= 0 && pos < cap) {
      token_rows[pos] = e / kk;
      inverse[(long long)(e / kk) * width + e % kk] = pos;
    }
    __syncwarp();
  }
}

// ---- row loaders for the NVFP4 activation encode ----------------------------------------
// 16 consecutive values as f32 with 16-byte loads (p 16-byte aligned: rows of
// a multiple of 32 columns, groups of 16).
__device__ __forceinline__ void load16_vec(const float *p, float v[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 f = reinterpret_cast<const float4 *>(p)[q];
    v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
  }
}
__device__ __forceinline__ void load16_vec(const uint16_t *p, float v[16]) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 u = reinterpret_cast<const uint4 *>(p)[q];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[8 * q + 2 * t] = __uint_as_float(w[t] << 16);
      v[8 * q + 2 * t + 1] = __uint_as_float(w[t] & 0xffff0000u);
    }
  }
}

// Gathered rows (moe.rs:71-89): sorted row r is token token_rows[r], or zeros.
template <typename T>
// Row loaders: row(r) resolves row r once (64-bit address arithmetic), then
// load16(row, g, v) reads its 16-column group g.
struct GatherRows {
  const T *x;
  const int32_t *token_rows;
  size_t cols;
  int tokens;
  using Row = const T *;  // null: a zero row
  __device__ __forceinline__ Row row(size_t r) const {
    const int t = token_rows[r];
    return (t < 0 || t >= tokens) ? nullptr : x + (size_t)t * cols;  // padding (or an id outside x)
  }
  __device__ __forceinline__ void load16(Row p, int g, float v[16]) const {
    if (!p) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.0f;
      return;
    }
    load16_vec(p + g * 16, v);
  }
};

// Plain rows [rows, cols] (e.g. the fused gate/up GEMM's SwiGLU output).
template <typename T>
struct PlainRows {
  const T *x;
  size_t cols;
  using Row = const T *;
  __device__ __forceinline__ Row row(size_t r) const { return x + r * cols; }
  __device__ __forceinline__ void load16(Row p, int g, float v[16]) const { load16_vec(p + g * 16, v); }
};

// SwiGLU rows (swiglu.rs:16): gate = first `cols` columns, up = next `cols`.

template <typename T>
struct SwigluRows {
  const T *gu;
  size_t cols;  // intermediate size
  using Row = const T *;
  __device__ __forceinline__ Row row(size_t r) const { return gu + r * 2 * cols; }
  __device__ __forceinline__ void load16(Row p, int g, float v[16]) const {
    const T *gate = p + g * 16;
    float gv[16], uv[16];
    load16_vec(gate, gv);
    load16_vec(gate + cols, uv);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = silu_mul(gv[i], uv[i]);
  }
};

// `valid` (nullable, device): rows at or past *valid are neither read nor
// written (row tiles past a device layout's end, which the GEMMs skip).
__device__ __forceinline__ size_t valid_rows(size_t rows, const int32_t *valid) {
  return valid ? min(rows, (size_t)max(*valid, 0)) : rows;
}

// Calls f(r, skip_r) for every row r < n of this warp's grid-stride share
// (rows w, w + W, w + 2W, ... for warp w of W) whose skip entry is >= 0 (every
// row when skip is null; skip_r is then 0).  With skip, the entries of 32 of
// the warp's rows are read in one load per lane and only the live rows are
// visited, so a sparse layout (decode-size batches, where most rows are
// padding) costs one load latency per 32 rows instead of one per row.
template <class Fn>
__device__ __forceinline__ void for_live_rows(size_t n, const int32_t *skip, Fn &&f) {
  const int lane = threadIdx.x & 31;
  const size_t warps = (size_t)gridDim.x * (blockDim.x / 32);
  const size_t w = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (!skip) {
    for (size_t r = w; r < n; r += warps) f(r, 0);
    return;
  }
  for (size_t base = w; base < n; base += 32 * warps) {
    const size_t r_l = base + (size_t)lane * warps;
    const int s_l = r_l < n ? skip[r_l] : -1;
    unsigned live = __ballot_sync(0xffffffffu, s_l >= 0);
    while (live) {
      const int i = __ffs(live) - 1;
      live &= live - 1;
      f(base + (size_t)i * warps, __shfl_sync(0xffffffffu, s_l, i));
    }
  }
}

// Both row kernels: one warp per row (grid-stride over rows), lane l encodes
// the 16-column groups l, l + 32, ... of the row.  skip (nullable): rows r
// with skip[r] < 0 (a layout's padding rows) are neither read nor written.
template <class Rows>
__global__ void rows_amax_kernel(Rows rows_src, size_t rows, const int32_t *valid, const int32_t *skip, size_t cols,
                                 uint32_t *amax_bits) {
  pdl_enter();
  const int gpr = (int)(cols / 16), lane = threadIdx.x & 31;
  const size_t n = valid_rows(rows, valid);
  uint32_t m = 0;
  for_live_rows(n, skip, [&](size_t r, int) {
    const auto src = rows_src.row(r);
    for (int g = lane; g < gpr; g += 32) {
      float v[16];
      rows_src.load16(src, g, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) m = max(m, __float_as_uint(v[i]) & 0x7fffffffu);
    }
  });
  block_amax_to(m, amax_bits);
}

// kRowMajorSf: factors to sf[rows, cols/16] (row-major) instead of the tiled layout.
template <class Rows, bool kRowMajorSf = false>
__global__ void rows_encode_kernel(Rows rows_src, size_t rows, const int32_t *valid, const int32_t *skip, size_t cols,
                                   const uint32_t *amax_bits, uint8_t *packed, uint8_t *sf_tiled, float *global_out) {
  pdl_enter();
  const float global = __fdiv_rn(__uint_as_float(*amax_bits), 2688.0f);
  if (blockIdx.x == 0 && threadIdx.x == 0) *global_out = global;
  const int gpr = (int)(cols / 16), lane = threadIdx.x & 31;
  const size_t n = valid_rows(rows, valid);
  for_live_rows(n, skip, [&](size_t r, int) {
    const auto src = rows_src.row(r);
    uint8_t *prow = packed + r * (cols / 2);
    uint8_t *srow = sf_tiled + (kRowMajorSf ? r * gpr : sf_tiled_row_offset(r, cols));
    for (int g = lane; g < gpr; g += 32) {
      float v[16];
      rows_src.load16(src, g, v);
      encode_group16(v, global, prow + g * 8, srow + (kRowMajorSf ? (uint32_t)g : sf_tiled_group_offset(g)));
    }
  });
}

// Gathered NVFP4 rows from token rows quantized once (token t's codes at
// tok_packed + t * code_stride, its row-major factors at tok_sf + t *
// sf_stride; cols % 64 == 0): one warp per layout row copies the token's
// codes (16-byte vectors) and its factors, four groups (one 4-byte word) at a
// time, into the tiled layout; padding rows get zeros, or nothing with
// `skip`.  NVFP4 encoding is row-local and every gathered row shares the one
// global, so the copies equal encoding the gathered rows.
__global__ void gather_codes_kernel(const uint8_t *tok_packed, const uint8_t *tok_sf, size_t code_stride,
                                    size_t sf_stride, int tokens, const int32_t *token_rows, size_t rows,
                                    const int32_t *valid, const int32_t *skip, size_t cols, uint8_t *packed,
                                    uint8_t *sf_tiled) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int code_vecs = (int)(cols / 32), sf_words = (int)(cols / 64);
  const size_t n = valid_rows(rows, valid);
  for_live_rows(n, skip, [&](size_t r, int) {
    const int t = token_rows[r];
    const bool zero = t < 0 || t >= tokens;
    const uint4 *csrc = reinterpret_cast<const uint4 *>(tok_packed + (size_t)max(t, 0) * code_stride);
    uint4 *cdst = reinterpret_cast<uint4 *>(packed + r * (cols / 2));
    for (int i = lane; i < code_vecs; i += 32) cdst[i] = zero ? make_uint4(0, 0, 0, 0) : csrc[i];
    const uint32_t *ssrc = reinterpret_cast<const uint32_t *>(tok_sf + (size_t)max(t, 0) * sf_stride);
    uint8_t *srow = sf_tiled + sf_tiled_row_offset(r, cols);
    for (int j = lane; j < sf_words; j += 32)
      *reinterpret_cast<uint32_t *>(srow + (size_t)j * kSfChunk) = zero ? 0u : ssrc[j];
  });
}

// Plain gather (gather_prefill_view, moe.rs:71-89, 673-733): f32 or bf16 out.
template <typename T, typename O>
__global__ void gather_rows_kernel(const T *x, int tokens, const int32_t *token_rows, size_t rows, size_t cols,
                                   O *out) {
  size_t n = rows * cols, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const size_t r = i / cols, c = i % cols;
    const int t = token_rows[r];
    const float v = (t < 0 || t >= tokens) ? 0.0f : act_load(x, (size_t)t * cols + c);
    if constexpr (sizeof(O) == 4)
      out[i] = v;
    else
      out[i] = __float2bfloat16_rn(v);
  }
}

template <typename T, typename O>
__global__ void swiglu_kernel(const T *gu, size_t rows, size_t cols, O *out) {
  size_t n = rows * cols, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const size_t r = i / cols, c = i % cols;
    const float v = silu_mul(act_load(gu, r * 2 * cols + c), act_load(gu, r * 2 * cols + cols + c));
    if constexpr (sizeof(O) == 4)
      out[i] = v;
    else
      out[i] = __float2bfloat16_rn(v);
  }
}

// ---- combine (moe.rs:91-147) -------------------------------------------------------------
// One CTA per token: sum over slots (in slot order) of weight * routed row;
// with a residual, out = residual + sum and normed = out * rsqrt(mean(out^2) +
// eps) * gamma (combine_add_norm_kernel).  Each thread owns 8 consecutive
// columns (16-byte vectors; cols is a multiple of 32).
template <typename R, typename O>
__global__ void combine_kernel(const R *routed, int routed_rows, size_t cols, const int32_t *inverse,
                               const float *weights, int width, int slots, const float *residual, const float *gamma,
                               float inv_h, float eps, O *out, float *normed, void *const *out_chunks,
                               int chunk_rows) {
  pdl_enter();
  extern __shared__ float red[];
  const int t = blockIdx.x;
  // out_chunks (device table, nullable): token t's row is row t % chunk_rows
  // of chunk t / chunk_rows, e.g. in another GPU's memory (plain peer stores)
  O *orow = out_chunks ? static_cast<O *>(out_chunks[t / chunk_rows]) + (size_t)(t % chunk_rows) * cols
                       : out + (size_t)t * cols;
  float ss = 0.0f;
  for (size_t c8 = threadIdx.x; c8 < cols / 8; c8 += blockDim.x) {
    const size_t c = c8 * 8;
    float sum[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) sum[j] = 0.0f;
    for (int s = 0; s < slots; ++s) {
      const int row = inverse[(size_t)t * width + s];
      if (row < 0 || row >= routed_rows) continue;  // a slot outside routed adds nothing
      const float w = weights[(size_t)t * width + s];
      float v[8];
      if constexpr (sizeof(R) == 4) {
        const float4 a = *reinterpret_cast<const float4 *>(routed + (size_t)row * cols + c);
        const float4 b = *reinterpret_cast<const float4 *>(routed + (size_t)row * cols + c + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 u = *reinterpret_cast<const uint4 *>(routed + (size_t)row * cols + c);
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] = __uint_as_float(q[j] << 16);
          v[2 * j + 1] = __uint_as_float(q[j] & 0xffff0000u);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) sum[j] = sum[j] + v[j] * w;
    }
    if (residual) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sum[j] = residual[(size_t)t * cols + c + j] + sum[j];
        ss = fmaf(sum[j], sum[j], ss);
      }
    }
    if constexpr (sizeof(O) == 4) {
      float4 *o = reinterpret_cast<float4 *>(orow + c);
      o[0] = make_float4(sum[0], sum[1], sum[2], sum[3]);
      o[1] = make_float4(sum[4], sum[5], sum[6], sum[7]);
    } else {
      *reinterpret_cast<uint4 *>(orow + c) =
          make_uint4(pack_bf16x2(sum[0], sum[1]), pack_bf16x2(sum[2], sum[3]), pack_bf16x2(sum[4], sum[5]),
                     pack_bf16x2(sum[6], sum[7]));
    }
  }
  if (!residual) {
    if (out_chunks) __threadfence_system();  // the stores reach the peer before the host-ordered barrier
    return;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float scale = rsqrtf(red[0] * inv_h + eps);
  for (size_t c = threadIdx.x; c < cols; c += blockDim.x) {
    float x;
    if constexpr (sizeof(O) == 4)
      x = orow[c];
    else
      x = __bfloat162float(orow[c]);
    normed[(size_t)t * cols + c] = x * scale * gamma[c];
  }
}

// Expert-parallel dispatch: the local expert id of every send row.  The send
// order is the layout of the routes by destination rank (fpb_moe_layout with
// ranks as "experts" and one-row tiles), so route (t, s) sits at row
// inverse[t, s] and goes to rank ids[t, s] / per_rank.
__global__ void moe_route_meta_kernel(const int32_t *ids, const int32_t *inverse, int tokens, int width, int slots,
                                      int per_rank, int rows, int32_t *send_expert) {
  const int n = tokens * slots;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int t = i / slots, s = i % slots;
    const int id = ids[(size_t)t * width + s], row = inverse[(size_t)t * width + s];
    if (row >= 0 && row < rows) send_expert[row] = id % per_rank;
  }
}

// Destination rank of every route: dest[t, s] = ids[t, s] / per_rank (slots
// past `slots` copy 0).
__global__ void moe_route_dest_kernel(const int32_t *ids, int tokens, int width, int slots, int per_rank,
                                      int32_t *dest) {
  const int n = tokens * width;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dest[i] = (i % width) < slots ? ids[i] / per_rank : 0;
}

// ---- expert parallel with fixed capacity ------------------------------------------------
// A rank's tokens go to the ranks that own their experts as fixed-size
// records, one per (token, destination) pair, never one per route: chunk d of
// the send buffer holds `tokens` records for rank d, the first count_d of
// them the tokens that route to rank d in token order, the rest marked empty.
// Every chunk has the same size, so the all-to-all needs no host-read counts
// and the whole layer is one CUDA graph.  A record is the token's NVFP4 row
// (codes, then row-major factors, encoded with the global of the all-reduced
// amax: the single-GPU encoding) and its routes as the receiver needs them:
// receiver-local expert ids (-1 for a slot owned by another rank) and the
// routing weights.
struct EpRecord {
  size_t sf, ids, weights, bytes;  // byte offsets in a record (codes at 0), record size
};

__host__ __device__ inline EpRecord ep_record(size_t cols, size_t width) {
  auto a16 = [](size_t v) { return (v + 15) / 16 * 16; };
  EpRecord r;
  r.sf = a16(cols / 2);
  r.ids = r.sf + a16(cols / 16);
  r.weights = r.ids + 4 * width;
  r.bytes = a16(r.weights + 4 * width);
  return r;
}

// positions[t * nranks + d] = d * tokens + (t's index among the tokens that
// route to rank d), or -1; positions[tokens * nranks + d] = count_d.  One CTA:
// per 1024-token chunk, one ballot per destination gives each warp's counts,
// one thread per destination scans the 32 warps, a second ballot places.
// With `staged` (tokens * 4 bytes of dynamic shared memory), every token's
// destination mask comes from ep_mask_kernel (many CTAs, one warp per token)
// through positions[0, tokens); otherwise each thread reads its token's ids
// chunk by chunk (one CTA's loads in flight: slower).
constexpr int kEpPlanThreads = 1024;
constexpr int kEpPlanStagedTokens = 10240;  // 40 KB of masks (+ 4.3 KB static: under the 48 KB default)

__device__ __forceinline__ uint32_t ep_token_mask(const int32_t *ids, int t, int width, int slots, int experts,
                                                  int per_rank, int *error) {
  uint32_t mask = 0;
  const int32_t *row = ids + (size_t)t * width;
#pragma unroll 4
  for (int s = 0; s < slots; ++s) {
    const int id = row[s];
    if (id >= 0 && id < experts)
      mask |= 1u << (id / per_rank);
    else if (error)
      atomicCAS(error, 0, 403);
  }
  return mask;
}

// Destination mask of every token (bit d: a route to rank d), one warp per
// token, into masks[t].
__global__ void ep_mask_kernel(const int32_t *ids, int tokens, int width, int slots, int experts, int per_rank,
                               uint32_t *masks, int *error) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x / 32);
  for (int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < tokens; t += warps) {
    uint32_t bit = 0;
    if (lane < slots) {
      const int id = ids[(size_t)t * width + lane];
      if (id >= 0 && id < experts)
        bit = 1u << (id / per_rank);
      else if (error)
        atomicCAS(error, 0, 403);
    }
    const uint32_t mask = __reduce_or_sync(0xffffffffu, bit);
    if (lane == 0) masks[t] = mask;
  }
}

__global__ void __launch_bounds__(kEpPlanThreads) ep_plan_kernel(const int32_t *ids, int tokens, int width,
                                                                 int slots, int experts, int per_rank, int nranks,
                                                                 int32_t *positions, int *error, bool staged) {
  pdl_enter();
  extern __shared__ uint32_t masks[];
  __shared__ int wtot[32][33];
  __shared__ int carry[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < nranks) carry[tid] = 0;
  if (staged) {  // the masks ep_mask_kernel left in positions[0, tokens), read before any write
    const uint32_t *src = reinterpret_cast<const uint32_t *>(positions);
    for (int t = tid; t < tokens; t += kEpPlanThreads) masks[t] = src[t];
  }
  __syncthreads();
  for (int base = 0; base < tokens; base += kEpPlanThreads) {
    const int t = base + tid;
    uint32_t mask = 0;
    if (t < tokens) mask = staged ? masks[t] : ep_token_mask(ids, t, width, slots, experts, per_rank, error);
    for (int d = 0; d < nranks; ++d) {
      const unsigned b = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
      if (lane == 0) wtot[warp][d] = __popc(b);
    }
    __syncthreads();
    if (tid < nranks) {
      int run = carry[tid];
      for (int w = 0; w < kEpPlanThreads / 32; ++w) {
        const int c = wtot[w][tid];
        wtot[w][tid] = run;
        run += c;
      }
      carry[tid] = run;
    }
    __syncthreads();
    for (int d = 0; d < nranks; ++d) {
      const bool on = (mask >> d) & 1u;
      const unsigned b = __ballot_sync(0xffffffffu, on);
      if (t < tokens)
        positions[(size_t)t * nranks + d] =
            on ? d * tokens + wtot[warp][d] + __popc(b & ((1u << lane) - 1u)) : -1;
    }
    __syncthreads();
  }
  if (tid < nranks) positions[(size_t)tokens * nranks + tid] = carry[tid];
}

// Record p (= chunk p / tokens, index p % tokens): in `records`, or, with a
// chunk table, at chunks[chunk] + index * record bytes (another GPU's
// receive buffer: plain peer stores over NVLink).
__device__ __forceinline__ uint8_t *ep_rec(uint8_t *records, void *const *chunks, int tokens, size_t p,
                                           size_t bytes) {
  return chunks ? static_cast<uint8_t *>(chunks[p / tokens]) + (p % tokens) * bytes : records + p * bytes;
}

// One warp per token: the routes' metadata into each destination's record,
// the empty marks of record t in every chunk past its count, and the NVFP4
// row encoded once into one destination's record (this rank's own when the
// token routes here, so that the copies read local memory) and copied
// (16-byte vectors, after __syncwarp) into the others.
template <typename T>
__global__ void ep_pack_kernel(const T *x, int tokens, int cols, const int32_t *ids, const float *weights, int width,
                               int slots, int experts, int per_rank, int nranks, const int32_t *positions,
                               const uint32_t *amax_bits, uint8_t *records, void *const *chunks, int self,
                               EpRecord rec, float *global_out) {
  pdl_enter();
  const float global = __fdiv_rn(__uint_as_float(*amax_bits), 2688.0f);
  if (blockIdx.x == 0 && threadIdx.x == 0) *global_out = global;
  const int lane = threadIdx.x & 31, gpr = cols / 16;
  const int warps = gridDim.x * (blockDim.x / 32);
  const int32_t *counts = positions + (size_t)tokens * nranks;
  for (int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < tokens; t += warps) {
    const int pos_l = lane < nranks ? positions[(size_t)t * nranks + lane] : -1;
    const unsigned live = __ballot_sync(0xffffffffu, pos_l >= 0);
    int id_l = -1;
    float w_l = 0.0f;
    if (lane < slots) {
      id_l = ids[(size_t)t * width + lane];
      w_l = weights[(size_t)t * width + lane];
    }
    for (int d = 0; d < nranks; ++d) {
      const int p = __shfl_sync(0xffffffffu, pos_l, d);
      if (p >= 0 && lane < width) {
        uint8_t *r = ep_rec(records, chunks, tokens, (size_t)p, rec.bytes);
        const bool mine = id_l >= 0 && id_l < experts && id_l / per_rank == d;
        reinterpret_cast<int32_t *>(r + rec.ids)[lane] = mine ? id_l % per_rank : -1;
        reinterpret_cast<float *>(r + rec.weights)[lane] = w_l;
      }
      if (t >= counts[d] && lane < width)
        reinterpret_cast<int32_t *>(ep_rec(records, chunks, tokens, (size_t)d * tokens + t, rec.bytes) +
                                    rec.ids)[lane] = -1;
    }
    if (!live) continue;
    const int d0 = (self >= 0 && ((live >> self) & 1u)) ? self : __ffs(live) - 1;
    uint8_t *first = ep_rec(records, chunks, tokens, (size_t)__shfl_sync(0xffffffffu, pos_l, d0), rec.bytes);
    const T *src = x + (size_t)t * cols;
    for (int g = lane; g < gpr; g += 32) {
      float v[16];
      load16_vec(src + (size_t)g * 16, v);
      uint2 c;
      first[rec.sf + g] = encode_group16_regs(v, global, c);
      *reinterpret_cast<uint2 *>(first + (size_t)g * 8) = c;
    }
    __syncwarp();
    const int vecs = (int)((rec.sf + (size_t)gpr + 15) / 16);
    unsigned rest = live & ~(1u << d0);
    while (rest) {
      const int d = __ffs(rest) - 1;
      rest &= rest - 1;
      uint8_t *r = ep_rec(records, chunks, tokens, (size_t)__shfl_sync(0xffffffffu, pos_l, d), rec.bytes);
      for (int i = lane; i < vecs; i += 32)
        reinterpret_cast<uint4 *>(r)[i] = reinterpret_cast<const uint4 *>(first)[i];
    }
  }
  if (chunks) __threadfence_system();  // the peer stores land before the host-ordered barrier
}

// The received records' routes as dense tables: ids [rows, width] (-1 where
// the slot is another rank's, or the record is empty) and weights.
__global__ void ep_unpack_kernel(const uint8_t *records, int rows, EpRecord rec, int width, int32_t *ids_out,
                                 float *w_out) {
  pdl_enter();
  const int n = rows * width;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint8_t *r = records + (size_t)(i / width) * rec.bytes;
    ids_out[i] = reinterpret_cast<const int32_t *>(r + rec.ids)[i % width];
    w_out[i] = reinterpret_cast<const float *>(r + rec.weights)[i % width];
  }
}

static unsigned stride_grid(size_t n) {
  size_t g = (n + 255) / 256, cap = (size_t)sm_count() * 8;
  return (unsigned)std::max<size_t>(1, std::min(g, cap));
}

// Row kernels: one warp per row, 8 rows per 256-thread block, at most 8
// blocks per SM resident (grid-stride beyond).
static unsigned row_grid(size_t rows) {
  size_t g = (rows + 7) / 8, cap = (size_t)sm_count() * 8;
  return (unsigned)std::max<size_t>(1, std::min(g, cap));
}

// The row encode (one warp per row).
template <class Rows>
static void launch_rows_encode(const Rows &src, size_t rows, const int32_t *valid, const int32_t *skip, size_t cols,
                               const uint32_t *amax, uint8_t *packed, uint8_t *sf_tiled, float *global_out,
                               cudaStream_t s) {
  launch_pdl(rows_encode_kernel<Rows>, row_grid(rows), 256, 0, s, src, rows, valid, skip, cols, amax, packed, sf_tiled, global_out);
}

// ---- decode: distinct experts of a batch's routes ------------------------------------------------
// For a decode batch (a few tokens) the MoE GEMVs run over the distinct
// experts the routes name, each expert's weights read once for every token:
// experts[0, count) are those ids in ascending order (-1 up to cap) and
// map[t * slots + s] is the index of ids[t, s] among them.  One CTA: a
// shared-memory bitmap of the experts, popcount prefix sums over its words.
// Device error 107 (and map -1) for an id outside [0, experts).
constexpr int kPlanThreads = 256;
// The plan by one CTA (any multiple of 32 threads up to 1024); `plan_sm`:
// 2 * ceil(n_experts / 32) words of shared memory.
__device__ __forceinline__ void plan_block(const int32_t *ids, int tokens, int width, int slots, int n_experts,
                                           int cap, int32_t *experts, int32_t *count, int32_t *map, int *error,
                                           uint32_t *plan_sm) {
  __shared__ int wsum[32];
  const int words = (n_experts + 31) / 32;
  uint32_t *bits = plan_sm, *base = plan_sm + words;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthreads = blockDim.x, nwarps = nthreads >> 5;
  for (int w = tid; w < words; w += nthreads) bits[w] = 0;
  __syncthreads();
  const int n = tokens * slots;
  for (int i = tid; i < n; i += nthreads) {
    const int e = ids[(size_t)(i / slots) * width + i % slots];
    if (e >= 0 && e < n_experts)
      atomicOr(&bits[e >> 5], 1u << (e & 31));
    else if (error)
      atomicCAS(error, 0, 107);
  }
  __syncthreads();
  // exclusive prefix of the words' popcounts: contiguous words per thread
  const int per = (words + nthreads - 1) / nthreads;
  const int w0 = min(words, tid * per), w1 = min(words, w0 + per);
  int local = 0;
  for (int w = w0; w < w1; ++w) local += __popc(bits[w]);
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int before = 0, total = 0;
  for (int w = 0; w < nwarps; ++w) {
    before += w < warp ? wsum[w] : 0;
    total += wsum[w];
  }
  int run = before + incl - local;
  for (int w = w0; w < w1; ++w) {
    base[w] = run;
    run += __popc(bits[w]);
  }
  __syncthreads();
  for (int w = tid; w < words; w += nthreads) {
    uint32_t b = bits[w];
    int idx = base[w];
    while (b) {
      const int bit = __ffs(b) - 1;
      b &= b - 1;
      if (idx < cap) experts[idx] = w * 32 + bit;
      ++idx;
    }
  }
  for (int i = total + tid; i < cap; i += nthreads) experts[i] = -1;
  if (tid == 0) *count = min(total, cap);
  for (int i = tid; i < n; i += nthreads) {
    const int e = ids[(size_t)(i / slots) * width + i % slots];
    int m = -1;
    if (e >= 0 && e < n_experts) m = (int)base[e >> 5] + __popc(bits[e >> 5] & ((1u << (e & 31)) - 1u));
    map[i] = m < cap ? m : -1;
  }
}

__global__ void __launch_bounds__(kPlanThreads) moe_decode_plan_kernel(const int32_t *ids, int tokens, int width,
                                                                       int slots, int n_experts, int cap,
                                                                       int32_t *experts, int32_t *count,
                                                                       int32_t *map, int *error) {
  pdl_enter();
  extern __shared__ uint32_t plan_sm[];
  plan_block(ids, tokens, width, slots, n_experts, cap, experts, count, map, error, plan_sm);
}

// Router top-k and the plan in one launch for decode-size batches: warp t
// takes token t's top-k (the shared-expert gate logit, when gate_col >= 0,
// is column gate_col of the same logits row; the shared expert is id
// `experts`), then the CTA builds the plan over the k (+1) slots.
template <int PER_LANE>
__global__ void __launch_bounds__(1024) moe_decode_route_kernel(const float *logits, long long ld, int gate_col,
                                                                 int tokens, int experts, int k, int width,
                                                                 int32_t *ids, float *weights, int cap,
                                                                 int32_t *distinct, int32_t *count, int32_t *map,
                                                                 int *error) {
  pdl_enter();
  extern __shared__ uint32_t plan_sm[];
  const int warp = threadIdx.x >> 5;
  if (warp < tokens) {
    const float *row = logits + (long long)warp * ld;
    topk_warp<PER_LANE>(row, gate_col >= 0 ? row + gate_col : nullptr, experts, k, width,
                        ids + (long long)warp * width, weights + (long long)warp * width);
  }
  __syncthreads();  // the ids written above are read by the whole CTA below (same CTA: visible after the barrier)
  const int slots = k + (gate_col >= 0 ? 1 : 0);
  plan_block(ids, tokens, width, slots, experts + (gate_col >= 0 ? 1 : 0), cap, distinct, count, map, error, plan_sm);
}

}  // namespace fpb

// ---- host side -------------------------------------------------------------------------
using namespace fpb;

namespace {
template <typename F>
int with_dtype(int dtype, F &&f) {
  if (dtype == FPB_F32) return f(static_cast<const float *>(nullptr));
  if (dtype == FPB_BF16) return f(static_cast<const uint16_t *>(nullptr));
  return fail(FPB_ERR_INVALID_ARGUMENT, "dtype %d", dtype);
}
}  // namespace

extern "C" int fpb_moe_topk(const float *logits, size_t ld, const float *shared_gate, size_t tokens, size_t experts,
                            size_t top_k, size_t width, int32_t *ids, float *weights, void *stream) {
  if (!logits || !ids || !weights) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_topk: null pointer");
  const size_t need = top_k + (shared_gate ? 1 : 0);
  if (tokens == 0 || experts == 0 || top_k == 0 || top_k > experts || width < need || width > 32 || ld < experts ||
      experts > 2048 || tokens > 0x7fffffffu / 32)
    return fail(FPB_ERR_SHAPE, "fpb_moe_topk: tokens %zu experts %zu top_k %zu width %zu ld %zu", tokens, experts,
                top_k, width, ld);
  cudaStream_t s = as_stream(stream);
  const unsigned grid = (unsigned)((tokens * 32 + 255) / 256);
  const int per = (int)((experts + 31) / 32);
  auto go = [&](auto kernel) {
    launch_pdl(kernel, grid, 256, 0, s, logits, (long long)ld, shared_gate, (int)tokens, (int)experts, (int)top_k,
                                (int)width, ids, weights);
  };
  if (per <= 4)
    go(moe_topk_kernel<4>);
  else if (per <= 8)
    go(moe_topk_kernel<8>);
  else if (per <= 16)
    go(moe_topk_kernel<16>);
  else if (per <= 32)
    go(moe_topk_kernel<32>);
  else
    go(moe_topk_kernel<64>);
  FPB_LAUNCH_CHECK("moe_topk_kernel");
  return FPB_OK;
}

extern "C" size_t fpb_moe_layout_scratch_bytes(size_t tokens, size_t slots, size_t experts) {
  const size_t groups = (tokens * slots + kLayoutChunk - 1) / kLayoutChunk;
  return std::max<size_t>(1, groups) * experts * sizeof(int);
}

static int layout_impl(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts,
                       size_t tile_rows, size_t cap, int32_t *token_rows, int32_t *tile_experts, int32_t *inverse,
                       size_t *ranges, int32_t *padded_rows, void *scratch, size_t scratch_bytes, bool masked,
                       void *stream) {
  if (!ids || !token_rows || !tile_experts || !inverse || !ranges || !padded_rows || !scratch)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_layout: null pointer");
  if (tokens == 0 || slots == 0 || slots > width || experts == 0 || tile_rows == 0 || (tile_rows & (tile_rows - 1)))
    return fail(FPB_ERR_SELECTION, "invalid expert selection: shape");
  size_t max_rows = 0;
  int st = fpb_prefill_layout_max_padded_rows(tokens, experts, slots, tile_rows, &max_rows);
  if (st) return st;
  if (cap < max_rows || cap % tile_rows || cap > 0x7fffffffu || tokens * width > 0x7fffffffu)
    return fail(FPB_ERR_WORKSPACE, "fpb_moe_layout: capacity %zu below %zu (or not a multiple of tile_rows)", cap,
                max_rows);
  if (scratch_bytes < fpb_moe_layout_scratch_bytes(tokens, slots, experts))
    return fail(FPB_ERR_WORKSPACE, "fpb_moe_layout: scratch of %zu bytes needed",
                fpb_moe_layout_scratch_bytes(tokens, slots, experts));
  const size_t wsmem = (size_t)kLayoutWarpsPerCta * experts * sizeof(int);
  if (wsmem > 200 * 1024) return fail(FPB_ERR_UNSUPPORTED, "fpb_moe_layout: %zu experts", experts);
  {
    static std::mutex mu;
    static std::vector<int> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (std::find(done.begin(), done.end(), dev) == done.end()) {
      FPB_CUDA_TRY(cudaFuncSetAttribute(moe_layout_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        200 * 1024));
      FPB_CUDA_TRY(cudaFuncSetAttribute(moe_layout_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        200 * 1024));
      FPB_CUDA_TRY(cudaFuncSetAttribute(moe_layout_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        200 * 1024));
      done.push_back(dev);
    }
  }
  cudaStream_t s = as_stream(stream);
  const int n = (int)(tokens * slots);
  const int groups = (n + kLayoutChunk - 1) / kLayoutChunk;
  int *cnt = static_cast<int *>(scratch);
  int *err = device_error_ptr();
  const size_t small_smem = (size_t)(kLayoutSmallThreads / 32 + 1) * experts * sizeof(int);
  if (groups == 1 && small_smem <= 200 * 1024) {
    static std::mutex mu_small;
    static std::vector<int> done_small;
    {
      int dev = 0;
      cudaGetDevice(&dev);
      std::lock_guard<std::mutex> lock(mu_small);
      if (std::find(done_small.begin(), done_small.end(), dev) == done_small.end()) {
        FPB_CUDA_TRY(cudaFuncSetAttribute(moe_layout_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          200 * 1024));
        done_small.push_back(dev);
      }
    }
    launch_pdl(moe_layout_small_kernel, 1, kLayoutSmallThreads, small_smem, s,
        ids, n, (int)slots, (int)width, (int)tokens, (int)experts, (int)tile_rows, (int)cap, token_rows,
        tile_experts, inverse, reinterpret_cast<int64_t *>(ranges), padded_rows, err, masked);
    FPB_LAUNCH_CHECK("moe_layout_small_kernel");
    return FPB_OK;
  }
  FPB_CUDA_TRY(cudaMemsetAsync(token_rows, 0xff, cap * sizeof(int32_t), s));
  FPB_CUDA_TRY(cudaMemsetAsync(tile_experts, 0xff, cap / tile_rows * sizeof(int32_t), s));
  FPB_CUDA_TRY(cudaMemsetAsync(inverse, masked ? 0xff : 0, tokens * width * sizeof(int32_t), s));
  moe_layout_count_kernel<<<groups, 256, experts * sizeof(int), s>>>(ids, n, (int)slots, (int)width, (int)experts,
                                                                     cnt, err, masked);
  FPB_LAUNCH_CHECK("moe_layout_count_kernel");
  moe_layout_scan_kernel<<<1, 1024, experts * sizeof(int), s>>>(cnt, groups, (int)experts, (int)tile_rows, (int)cap,
                                                                tile_experts, reinterpret_cast<int64_t *>(ranges),
                                                                padded_rows, err);
  FPB_LAUNCH_CHECK("moe_layout_scan_kernel");
  moe_layout_place_kernel<<<groups, kLayoutWarpsPerCta * 32, wsmem, s>>>(
      ids, n, (int)slots, (int)width, (int)experts, (int)cap, cnt, reinterpret_cast<const int64_t *>(ranges),
      token_rows, inverse, masked);
  FPB_LAUNCH_CHECK("moe_layout_place_kernel");
  return FPB_OK;
}

extern "C" int fpb_moe_layout(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts,
                              size_t tile_rows, size_t cap, int32_t *token_rows, int32_t *tile_experts,
                              int32_t *inverse, size_t *ranges, int32_t *padded_rows, void *scratch,
                              size_t scratch_bytes, void *stream) {
  return layout_impl(ids, tokens, width, slots, experts, tile_rows, cap, token_rows, tile_experts, inverse, ranges,
                     padded_rows, scratch, scratch_bytes, false, stream);
}

extern "C" int fpb_moe_layout_masked(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts,
                                     size_t tile_rows, size_t cap, int32_t *token_rows, int32_t *tile_experts,
                                     int32_t *inverse, size_t *ranges, int32_t *padded_rows, void *scratch,
                                     size_t scratch_bytes, void *stream) {
  return layout_impl(ids, tokens, width, slots, experts, tile_rows, cap, token_rows, tile_experts, inverse, ranges,
                     padded_rows, scratch, scratch_bytes, true, stream);
}

extern "C" int fpb_moe_gather(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *token_rows,
                              size_t rows, void *out, int out_dtype, void *stream) {
  if (!x || !token_rows || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_gather: null pointer");
  if (tokens == 0 || cols == 0 || rows == 0) return fail(FPB_ERR_SHAPE, "fpb_moe_gather: empty");
  cudaStream_t s = as_stream(stream);
  const unsigned grid = stride_grid(rows * cols);
  return with_dtype(x_dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    const T *xs = static_cast<const T *>(x);
    if (out_dtype == FPB_F32)
      gather_rows_kernel<T, float><<<grid, 256, 0, s>>>(xs, (int)tokens, token_rows, rows, cols,
                                                         static_cast<float *>(out));
    else if (out_dtype == FPB_BF16)
      gather_rows_kernel<T, __nv_bfloat16><<<grid, 256, 0, s>>>(xs, (int)tokens, token_rows, rows, cols,
                                                                 static_cast<__nv_bfloat16 *>(out));
    else
      return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_gather: out dtype");
    FPB_LAUNCH_CHECK("gather_rows_kernel");
    return (int)FPB_OK;
  });
}

static size_t align256_sz(size_t n) { return (n + 255) / 256 * 256; }

extern "C" size_t fpb_moe_gather_quantize_workspace_bytes(size_t tokens, size_t cols) {
  return align256_sz(tokens * cols / 2) + tokens * cols / 16;
}

extern "C" int fpb_moe_gather_quantize(const void *x, int x_dtype, size_t tokens, size_t cols,
                                       const int32_t *token_rows, size_t rows, const int32_t *valid_rows,
                                       uint8_t *packed, uint8_t *sf_tiled, float *global_out, float *amax_scratch,
                                       int flags, void *workspace, size_t workspace_bytes, void *stream) {
  if (!x || !token_rows || !packed || !sf_tiled || !global_out || !amax_scratch)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_gather_quantize: null pointer");
  if (tokens == 0 || rows == 0 || cols == 0 || cols % 32) return fail(FPB_ERR_SHAPE, "fpb_moe_gather_quantize: shape");
  if (reinterpret_cast<uintptr_t>(x) & 15)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_gather_quantize: x must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  uint32_t *amax = reinterpret_cast<uint32_t *>(amax_scratch);
  const bool given = flags & FPB_QUANT_AMAX_GIVEN;
  if (!given) FPB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(uint32_t), s));
  // Factors of the K padding up to a multiple of 256 columns are read by the
  // tensor cores (times zero codes) and must be zero, not stale bytes.
  if (cols % 256) FPB_CUDA_TRY(cudaMemsetAsync(sf_tiled, 0, sf_tiled_bytes(rows, cols), s));
  return with_dtype(x_dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    const T *xs = static_cast<const T *>(x);
    if (!given) {
      launch_pdl(act_amax_kernel<T>, stride_grid(tokens * cols), 256, 0, s, xs, tokens * cols, amax);
      FPB_LAUNCH_CHECK("act_amax_kernel");
    }
    GatherRows<T> src{xs, token_rows, cols, (int)tokens};
    const int32_t *skip = (flags & FPB_QUANT_SKIP_PADDING) ? token_rows : nullptr;
    const bool via_tokens = workspace && workspace_bytes >= fpb_moe_gather_quantize_workspace_bytes(tokens, cols) &&
                            cols % 64 == 0 && tokens <= 0x7fffffffu &&
                            !(reinterpret_cast<uintptr_t>(workspace) & 255) &&
                            !(reinterpret_cast<uintptr_t>(packed) & 15);
    if (!via_tokens) {
      launch_rows_encode(src, rows, valid_rows, skip, cols, amax, packed, sf_tiled, global_out, s);
      FPB_LAUNCH_CHECK("rows_encode_kernel(gather)");
      return (int)FPB_OK;
    }
    // each token once, then copies into the layout's rows
    uint8_t *tok_packed = static_cast<uint8_t *>(workspace);
    uint8_t *tok_sf = tok_packed + align256_sz(tokens * cols / 2);
    PlainRows<T> tok{xs, cols};
    launch_pdl(rows_encode_kernel<PlainRows<T>, true>, row_grid(tokens), 256, 0, s, tok, tokens, nullptr, nullptr, cols, amax,
                                                                             tok_packed, tok_sf, global_out);
    FPB_LAUNCH_CHECK("rows_encode_kernel(tokens)");
    launch_pdl(gather_codes_kernel, row_grid(rows), 256, 0, s, tok_packed, tok_sf, cols / 2, cols / 16, (int)tokens,
               token_rows, rows, valid_rows, skip, cols, packed, sf_tiled);
    FPB_LAUNCH_CHECK("gather_codes_kernel");
    return (int)FPB_OK;
  });
}

extern "C" int fpb_swiglu(const void *gate_up, int dtype, size_t rows, size_t inter, void *out, int out_dtype,
                          void *stream) {
  if (!gate_up || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_swiglu: null pointer");
  if (rows == 0 || inter == 0) return fail(FPB_ERR_SHAPE, "fpb_swiglu: empty");
  cudaStream_t s = as_stream(stream);
  const unsigned grid = stride_grid(rows * inter);
  return with_dtype(dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    const T *g = static_cast<const T *>(gate_up);
    if (out_dtype == FPB_F32)
      swiglu_kernel<T, float><<<grid, 256, 0, s>>>(g, rows, inter, static_cast<float *>(out));
    else if (out_dtype == FPB_BF16)
      swiglu_kernel<T, __nv_bfloat16><<<grid, 256, 0, s>>>(g, rows, inter, static_cast<__nv_bfloat16 *>(out));
    else
      return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_swiglu: out dtype");
    FPB_LAUNCH_CHECK("swiglu_kernel");
    return (int)FPB_OK;
  });
}

extern "C" int fpb_swiglu_quantize(const void *gate_up, int dtype, size_t rows, const int32_t *valid_rows,
                                   size_t inter, uint8_t *packed, uint8_t *sf_tiled, float *global_out,
                                   float *amax_scratch, int flags, void *stream) {
  if (!gate_up || !packed || !sf_tiled || !global_out || !amax_scratch)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_swiglu_quantize: null pointer");
  if (rows == 0 || inter == 0 || inter % 32) return fail(FPB_ERR_SHAPE, "fpb_swiglu_quantize: shape");
  if (reinterpret_cast<uintptr_t>(gate_up) & 15)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_swiglu_quantize: gate_up must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  uint32_t *amax = reinterpret_cast<uint32_t *>(amax_scratch);
  const bool given = flags & FPB_QUANT_AMAX_GIVEN;
  if (!given) FPB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(uint32_t), s));
  if (inter % 256) FPB_CUDA_TRY(cudaMemsetAsync(sf_tiled, 0, sf_tiled_bytes(rows, inter), s));
  return with_dtype(dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    SwigluRows<T> src{static_cast<const T *>(gate_up), inter};
    const unsigned grid = row_grid(rows);
    if (!given) {
      launch_pdl(rows_amax_kernel<std::decay_t<decltype(src)>>, grid, 256, 0, s, src, rows, valid_rows, nullptr, inter, amax);
      FPB_LAUNCH_CHECK("rows_amax_kernel(swiglu)");
    }
    launch_rows_encode(src, rows, valid_rows, nullptr, inter, amax, packed, sf_tiled, global_out, s);
    FPB_LAUNCH_CHECK("rows_encode_kernel(swiglu)");
    return (int)FPB_OK;
  });
}

extern "C" int fpb_rows_quantize(const void *x, int dtype, size_t rows, const int32_t *valid_rows,
                                 const int32_t *token_rows, size_t cols, uint8_t *packed, uint8_t *sf_tiled,
                                 float *global_out, float *amax_scratch, int flags, void *stream) {
  if (!x || !packed || !sf_tiled || !global_out || !amax_scratch)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_rows_quantize: null pointer");
  if (rows == 0 || cols == 0 || cols % 32) return fail(FPB_ERR_SHAPE, "fpb_rows_quantize: shape");
  if ((flags & FPB_QUANT_SKIP_PADDING) && !token_rows)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_rows_quantize: FPB_QUANT_SKIP_PADDING needs token_rows");
  if (reinterpret_cast<uintptr_t>(x) & 15)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_rows_quantize: x must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  uint32_t *amax = reinterpret_cast<uint32_t *>(amax_scratch);
  const bool given = flags & FPB_QUANT_AMAX_GIVEN;
  if (!given) FPB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(uint32_t), s));
  if (cols % 256) FPB_CUDA_TRY(cudaMemsetAsync(sf_tiled, 0, sf_tiled_bytes(rows, cols), s));
  return with_dtype(dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    PlainRows<T> src{static_cast<const T *>(x), cols};
    const int32_t *skip = (flags & FPB_QUANT_SKIP_PADDING) ? token_rows : nullptr;
    const unsigned grid = row_grid(rows);
    if (!given) {
      launch_pdl(rows_amax_kernel<std::decay_t<decltype(src)>>, grid, 256, 0, s, src, rows, valid_rows, skip, cols, amax);
      FPB_LAUNCH_CHECK("rows_amax_kernel(rows)");
    }
    launch_rows_encode(src, rows, valid_rows, skip, cols, amax, packed, sf_tiled, global_out, s);
    FPB_LAUNCH_CHECK("rows_encode_kernel(rows)");
    return (int)FPB_OK;
  });
}

static int combine_impl(const void *routed, int r_dtype, size_t routed_rows, size_t cols, const int32_t *inverse,
                        const float *weights, size_t tokens, size_t width, size_t slots, const float *residual,
                        const float *gamma, float eps, void *out, int out_dtype, float *normed, cudaStream_t s,
                        void *const *out_chunks = nullptr, size_t chunk_rows = 0) {
  if (!routed || !inverse || !weights || (!out && !out_chunks))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_combine: null pointer");
  if (out_chunks && (chunk_rows == 0 || chunk_rows > 0x7fffffffu))
    return fail(FPB_ERR_SHAPE, "fpb_moe_combine_chunks: chunk_rows %zu", chunk_rows);
  if (tokens == 0 || cols == 0 || cols % 32 || slots == 0 || slots > width || tokens > 0x7fffffffu ||
      routed_rows > 0x7fffffffu)
    return fail(FPB_ERR_SHAPE, "fpb_moe_combine: shape");
  if ((reinterpret_cast<uintptr_t>(routed) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_combine: routed and out must be 16-byte aligned");
  const int threads = std::min<int>(256, std::max<int>(32, (int)(cols / 8 + 31) / 32 * 32));
  const float inv_h = 1.0f / (float)cols;
  return with_dtype(r_dtype, [&](auto tp) {
    using R = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    const R *rs = static_cast<const R *>(routed);
    if (out_dtype == FPB_F32)
      launch_pdl(combine_kernel<R, float>, (unsigned)tokens, threads, 32 * sizeof(float), s,
          rs, (int)routed_rows, cols, inverse, weights, (int)width, (int)slots, residual, gamma, inv_h, eps,
          static_cast<float *>(out), normed, out_chunks, (int)chunk_rows);
    else if (out_dtype == FPB_BF16)
      launch_pdl(combine_kernel<R, __nv_bfloat16>, (unsigned)tokens, threads, 32 * sizeof(float), s,
          rs, (int)routed_rows, cols, inverse, weights, (int)width, (int)slots, residual, gamma, inv_h, eps,
          static_cast<__nv_bfloat16 *>(out), normed, out_chunks, (int)chunk_rows);
    else
      return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_combine: out dtype");
    FPB_LAUNCH_CHECK("combine_kernel");
    return (int)FPB_OK;
  });
}

extern "C" int fpb_moe_combine(const void *routed, int r_dtype, size_t routed_rows, size_t cols,
                               const int32_t *inverse, const float *weights, size_t tokens, size_t width,
                               size_t slots, void *out, int out_dtype, void *stream) {
  return combine_impl(routed, r_dtype, routed_rows, cols, inverse, weights, tokens, width, slots, nullptr, nullptr,
                      0.0f, out, out_dtype, nullptr, as_stream(stream));
}

extern "C" int fpb_moe_combine_chunks(const void *routed, int r_dtype, size_t routed_rows, size_t cols,
                                      const int32_t *inverse, const float *weights, size_t tokens, size_t width,
                                      size_t slots, void *const *out_chunks, size_t chunk_rows, int out_dtype,
                                      void *stream) {
  if (!out_chunks) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_combine_chunks: null chunk table");
  return combine_impl(routed, r_dtype, routed_rows, cols, inverse, weights, tokens, width, slots, nullptr, nullptr,
                      0.0f, nullptr, out_dtype, nullptr, as_stream(stream), out_chunks, chunk_rows);
}

extern "C" int fpb_moe_combine_add_norm(const void *routed, int r_dtype, size_t routed_rows, size_t cols,
                                        const int32_t *inverse, const float *weights, size_t tokens, size_t width,
                                        size_t slots, const float *residual, const float *gamma, float eps,
                                        float *out, float *normed, void *stream) {
  if (!residual || !gamma || !normed) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_combine_add_norm: null pointer");
  return combine_impl(routed, r_dtype, routed_rows, cols, inverse, weights, tokens, width, slots, residual, gamma,
                      eps, out, FPB_F32, normed, as_stream(stream));
}

extern "C" int fpb_moe_route_meta(const int32_t *ids, const int32_t *inverse, size_t tokens, size_t width,
                                  size_t slots, size_t experts_per_rank, size_t rows, int32_t *send_expert,
                                  void *stream) {
  if (!ids || !inverse || !send_expert) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_route_meta: null pointer");
  if (tokens == 0 || slots == 0 || slots > width || experts_per_rank == 0 || tokens * width > 0x7fffffffu ||
      rows > 0x7fffffffu)
    return fail(FPB_ERR_SHAPE, "fpb_moe_route_meta: shape");
  moe_route_meta_kernel<<<stride_grid(tokens * slots), 256, 0, as_stream(stream)>>>(
      ids, inverse, (int)tokens, (int)width, (int)slots, (int)experts_per_rank, (int)rows, send_expert);
  FPB_LAUNCH_CHECK("moe_route_meta_kernel");
  return FPB_OK;
}

extern "C" int fpb_moe_route_dest(const int32_t *ids, size_t tokens, size_t width, size_t slots,
                                  size_t experts_per_rank, int32_t *dest, void *stream) {
  if (!ids || !dest) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_route_dest: null pointer");
  if (tokens == 0 || slots == 0 || slots > width || experts_per_rank == 0 || tokens * width > 0x7fffffffu)
    return fail(FPB_ERR_SHAPE, "fpb_moe_route_dest: shape");
  moe_route_dest_kernel<<<stride_grid(tokens * width), 256, 0, as_stream(stream)>>>(
      ids, (int)tokens, (int)width, (int)slots, (int)experts_per_rank, dest);
  FPB_LAUNCH_CHECK("moe_route_dest_kernel");
  return FPB_OK;
}

extern "C" size_t fpb_ep_record_bytes(size_t cols, size_t width) { return ep_record(cols, width).bytes; }

static int ep_dispatch_impl(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *ids,
                            const float *weights, size_t width, size_t slots, size_t experts, size_t nranks,
                            const float *amax, void *records, void *const *chunks, int self, int32_t *positions,
                            float *global_out, void *stream) {
  if (!x || !ids || !weights || !amax || (!records && !chunks) || !positions || !global_out)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ep_dispatch: null pointer");
  if (tokens == 0 || cols == 0 || cols % 64 || slots == 0 || slots > width || width > 32 || nranks == 0 ||
      nranks > 32 || experts == 0 || experts % nranks || tokens * nranks > 0x7fffffffu ||
      tokens * width > 0x7fffffffu)
    return fail(FPB_ERR_SHAPE, "fpb_ep_dispatch: tokens %zu cols %zu slots %zu width %zu experts %zu nranks %zu",
                tokens, cols, slots, width, experts, nranks);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(records) & 15))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ep_dispatch: x and records must be 16-byte aligned");
  if (self > 31) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ep_dispatch: self rank");
  cudaStream_t s = as_stream(stream);
  const int per_rank = (int)(experts / nranks);
  const bool staged = tokens <= (size_t)kEpPlanStagedTokens;
  if (staged) {
    launch_pdl(ep_mask_kernel, row_grid(tokens), 256, 0, s, ids, (int)tokens, (int)width, (int)slots, (int)experts,
               per_rank, reinterpret_cast<uint32_t *>(positions), device_error_ptr());
    FPB_LAUNCH_CHECK("ep_mask_kernel");
  }
  launch_pdl(ep_plan_kernel, 1, kEpPlanThreads, staged ? tokens * sizeof(uint32_t) : 0, s, ids, (int)tokens,
             (int)width, (int)slots, (int)experts, per_rank, (int)nranks, positions, device_error_ptr(), staged);
  FPB_LAUNCH_CHECK("ep_plan_kernel");
  const EpRecord rec = ep_record(cols, width);
  return with_dtype(x_dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    launch_pdl(ep_pack_kernel<T>, row_grid(tokens), 256, 0, s, static_cast<const T *>(x), (int)tokens, (int)cols,
               ids, weights, (int)width, (int)slots, (int)experts, per_rank, (int)nranks,
               (const int32_t *)positions, reinterpret_cast<const uint32_t *>(amax), static_cast<uint8_t *>(records),
               chunks, self, rec, global_out);
    FPB_LAUNCH_CHECK("ep_pack_kernel");
    return (int)FPB_OK;
  });
}

extern "C" int fpb_ep_dispatch(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *ids,
                               const float *weights, size_t width, size_t slots, size_t experts, size_t nranks,
                               const float *amax, void *records, int32_t *positions, float *global_out,
                               void *stream) {
  return ep_dispatch_impl(x, x_dtype, tokens, cols, ids, weights, width, slots, experts, nranks, amax, records,
                          nullptr, -1, positions, global_out, stream);
}

extern "C" int fpb_ep_dispatch_chunks(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *ids,
                                      const float *weights, size_t width, size_t slots, size_t experts,
                                      size_t nranks, const float *amax, void *const *chunks, int self_rank,
                                      int32_t *positions, float *global_out, void *stream) {
  if (!chunks) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ep_dispatch_chunks: null chunk table");
  if (self_rank < -1 || self_rank >= (int)std::min<size_t>(nranks, 32))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ep_dispatch_chunks: self_rank %d", self_rank);
  return ep_dispatch_impl(x, x_dtype, tokens, cols, ids, weights, width, slots, experts, nranks, amax, nullptr,
                          chunks, self_rank, positions, global_out, stream);
}

extern "C" int fpb_ep_unpack(const void *records, size_t rows, size_t cols, size_t width, int32_t *ids,
                             float *weights, void *stream) {
  if (!records || !ids || !weights) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_ep_unpack: null pointer");
  if (rows == 0 || cols == 0 || cols % 64 || width == 0 || width > 32 || rows * width > 0x7fffffffu)
    return fail(FPB_ERR_SHAPE, "fpb_ep_unpack: rows %zu cols %zu width %zu", rows, cols, width);
  launch_pdl(ep_unpack_kernel, stride_grid(rows * width), 256, 0, as_stream(stream),
             static_cast<const uint8_t *>(records), (int)rows, ep_record(cols, width), (int)width, ids, weights);
  FPB_LAUNCH_CHECK("ep_unpack_kernel");
  return FPB_OK;
}

extern "C" int fpb_moe_gather_codes(const uint8_t *codes, size_t code_stride, const uint8_t *sf, size_t sf_stride,
                                    size_t tokens, size_t cols, const int32_t *token_rows, size_t rows,
                                    const int32_t *valid_rows, int flags, uint8_t *packed, uint8_t *sf_tiled,
                                    void *stream) {
  if (!codes || !sf || !token_rows || !packed || !sf_tiled)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_gather_codes: null pointer");
  if (tokens == 0 || tokens > 0x7fffffffu || rows == 0 || cols == 0 || cols % 64 || code_stride < cols / 2 ||
      sf_stride < cols / 16)
    return fail(FPB_ERR_SHAPE, "fpb_moe_gather_codes: shape");
  if ((reinterpret_cast<uintptr_t>(codes) & 15) || code_stride % 16 || (reinterpret_cast<uintptr_t>(sf) & 3) ||
      sf_stride % 4 || (reinterpret_cast<uintptr_t>(packed) & 15) || (reinterpret_cast<uintptr_t>(sf_tiled) & 3))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_gather_codes: alignment (codes 16 B, factors 4 B)");
  cudaStream_t s = as_stream(stream);
  if (cols % 256) FPB_CUDA_TRY(cudaMemsetAsync(sf_tiled, 0, sf_tiled_bytes(rows, cols), s));
  const int32_t *skip = (flags & FPB_QUANT_SKIP_PADDING) ? token_rows : nullptr;
  launch_pdl(gather_codes_kernel, row_grid(rows), 256, 0, s, codes, sf, code_stride, sf_stride, (int)tokens,
             token_rows, rows, valid_rows, skip, cols, packed, sf_tiled);
  FPB_LAUNCH_CHECK("gather_codes_kernel");
  return FPB_OK;
}

extern "C" int fpb_act_amax(const void *x, int dtype, size_t n, float *amax_scratch, int accumulate, void *stream) {
  if (!x || !amax_scratch) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_act_amax: null pointer");
  cudaStream_t s = as_stream(stream);
  uint32_t *amax = reinterpret_cast<uint32_t *>(amax_scratch);
  if (!accumulate) FPB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(uint32_t), s));
  if (n == 0) return FPB_OK;
  return with_dtype(dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    launch_pdl(act_amax_kernel<T>, stride_grid(n), 256, 0, s, static_cast<const T *>(x), n, amax);
    FPB_LAUNCH_CHECK("act_amax_kernel");
    return (int)FPB_OK;
  });
}

extern "C" int fpb_swiglu_amax(const void *gate_up, int dtype, size_t rows, const int32_t *valid_rows, size_t inter,
                               float *amax_scratch, int accumulate, void *stream) {
  if (!gate_up || !amax_scratch) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_swiglu_amax: null pointer");
  if (inter == 0 || inter % 32) return fail(FPB_ERR_SHAPE, "fpb_swiglu_amax: shape");
  if (reinterpret_cast<uintptr_t>(gate_up) & 15)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_swiglu_amax: gate_up must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  uint32_t *amax = reinterpret_cast<uint32_t *>(amax_scratch);
  if (!accumulate) FPB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(uint32_t), s));
  if (rows == 0) return FPB_OK;
  return with_dtype(dtype, [&](auto tp) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
    SwigluRows<T> src{static_cast<const T *>(gate_up), inter};
    launch_pdl(rows_amax_kernel<std::decay_t<decltype(src)>>, row_grid(rows), 256, 0, s, src, rows, valid_rows, nullptr, inter, amax);
    FPB_LAUNCH_CHECK("rows_amax_kernel(swiglu)");
    return (int)FPB_OK;
  });
}

extern "C" int fpb_moe_decode_plan(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts,
                                   int32_t *distinct, int32_t *count, size_t cap, int32_t *map, void *stream) {
  if (!ids || !distinct || !count || !map) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_decode_plan: null pointer");
  if (tokens == 0 || slots == 0 || slots > width || experts == 0 || experts > 65536 || tokens * slots > 0x7fffffff ||
      cap < tokens * slots || cap > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_moe_decode_plan: tokens %zu slots %zu width %zu experts %zu cap %zu", tokens,
                slots, width, experts, cap);
  const size_t words = (experts + 31) / 32;
  cudaError_t e = launch_pdl(moe_decode_plan_kernel, 1, kPlanThreads, 2 * words * sizeof(uint32_t), as_stream(stream),
                             ids, (int)tokens, (int)width, (int)slots, (int)experts, (int)cap, distinct, count, map,
                             device_error_ptr());
  if (e != cudaSuccess) return cuda_fail(e, "moe_decode_plan_kernel");
  FPB_LAUNCH_CHECK("moe_decode_plan_kernel");
  return FPB_OK;
}

extern "C" int fpb_moe_decode_route(const float *logits, size_t ld, long long gate_col, size_t tokens,
                                    size_t experts, size_t top_k, size_t width, int32_t *ids, float *weights,
                                    int32_t *distinct, int32_t *count, size_t cap, int32_t *map, void *stream) {
  if (!logits || !ids || !weights || !distinct || !count || !map)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_decode_route: null pointer");
  const size_t slots = top_k + (gate_col >= 0 ? 1 : 0);
  // up to 512 experts: a warp's logits stay in registers under the 1024-thread
  // launch bound (64 registers a thread); larger routers use fpb_moe_topk +
  // fpb_moe_decode_plan
  if (tokens == 0 || tokens > 32 || experts == 0 || experts > 512 || top_k == 0 || top_k > experts ||
      width < slots || width > 32 || ld < experts || (gate_col >= 0 && (size_t)gate_col >= ld) ||
      cap < tokens * slots || cap > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_moe_decode_route: tokens %zu (at most 32) experts %zu (at most 512) top_k %zu width %zu "
                "ld %zu cap %zu", tokens, experts, top_k, width, ld, cap);
  const size_t words = (experts + 1 + 31) / 32;
  const int per = (int)((experts + 31) / 32);
  const unsigned threads = (unsigned)std::max<size_t>(64, tokens * 32);
  const size_t smem = 2 * words * sizeof(uint32_t);
  cudaStream_t s = as_stream(stream);
  auto go = [&](auto kernel) {
    return launch_pdl(kernel, 1, threads, smem, s, logits, (long long)ld, (int)gate_col, (int)tokens,
                      (int)experts, (int)top_k, (int)width, ids, weights, (int)cap, distinct, count, map,
                      device_error_ptr());
  };
  cudaError_t e;
  if (per <= 4)
    e = go(moe_decode_route_kernel<4>);
  else if (per <= 8)
    e = go(moe_decode_route_kernel<8>);
  else
    e = go(moe_decode_route_kernel<16>);
  if (e != cudaSuccess) return cuda_fail(e, "moe_decode_route_kernel");
  FPB_LAUNCH_CHECK("moe_decode_route_kernel");
  return FPB_OK;
}
