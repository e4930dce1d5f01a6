// Decode-step kernels of the hybrid MoE decoder around the quantized-matmul
// path: embedding, RMSNorm, the full-attention layer's
// head norms + RoPE + KV-cache append and split-position GQA decode
// attention with the output gate, the gated-delta-net layer's causal conv,
// delta-rule step and gated norm, the decode MoE combine + residual + norm,
// and greedy sampling.  The linear layers are the library's NVFP4 GEMVs.
//
// Each kernel restates one firepit-kernels operation (crate src/ paths):
//   embedding        embedding.rs            rms_norm / add_norm   norm.rs
//   attn_prepare     norm.rs (q/k head norms), rope.rs:6-22, attention.rs:6-30
//   attn_decode      attention.rs:128-168 (online_attention), :170-190 (output_gate)
//   gdn_conv         gdn.rs:6-63 (conv1d_silu)
//   gdn_delta        gdn.rs:206-263 (delta_step)
//   gdn_gated_norm   norm.rs rms_norm over each value head, gdn.rs:266-278 (gated_silu)
//   combine_add_norm moe.rs:111-147 (combine_add_norm_view), normed in bf16
//   argmax           firepit src/generation.rs:34-42 (greedy)
// Every kernel starts with pdl_enter() (programmatic dependent launch: it waits
// for the previous kernel before reading anything).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace fpb {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ float load_f(const T *p, size_t i);
template <>
__device__ __forceinline__ float load_f<float>(const float *p, size_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16 *p, size_t i) {
  return __bfloat162float(p[i]);
}

__device__ __forceinline__ void store_f(void *p, int bf16, size_t i, float v) {
  if (bf16)
    reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float *>(p)[i] = v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// ---- embedding ----------------------------------------------------------------------------
__global__ void embedding_kernel(const __nv_bfloat16 *table, const int32_t *ids, int rows, int hidden, int vocab,
                                 float *out, int *error) {
  pdl_enter();
  const int r = blockIdx.y;
  const int id = ids[r];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && error) atomicCAS(error, 0, 501);
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < hidden; c += gridDim.x * blockDim.x)
      out[(size_t)r * hidden + c] = 0.0f;
    return;
  }
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < hidden; c += gridDim.x * blockDim.x)
    out[(size_t)r * hidden + c] = __bfloat162float(table[(size_t)id * hidden + c]);
}

// ---- RMSNorm (norm.rs): out = x * rsqrt(mean(x^2) + eps) * gamma -------------------------------
// Minimum over the CTA (every thread gets it); `red` holds 32 floats.
__device__ __forceinline__ float block_min(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
  for (int i = 1; i < warps; ++i) t = fminf(t, red[i]);
  return t;
}

// Sum over the CTA (every thread gets it); `red` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < warps; ++w) t += red[w];
  return t;
}

// One CTA per row (a decode batch has a few rows, each a few thousand
// columns: the row's loads spread over the CTA's threads); with `delta`,
// x = residual + delta is also stored to `sum_out`.
template <typename T>
__global__ void rms_norm_kernel(const T *x, size_t x_pitch, const float *delta, float *sum_out, int rows,
                                int width, const float *gamma, float inv_w, float eps, void *out, int out_bf16,
                                size_t out_pitch) {
  pdl_enter();
  __shared__ float red[32];
  const int r = blockIdx.x;
  const T *xr = x + (size_t)r * x_pitch;
  float ss = 0.0f;
#pragma unroll 4
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float v = load_f(xr, c);
    if (delta) {
      v += delta[(size_t)r * width + c];
      sum_out[(size_t)r * width + c] = v;
    }
    ss = fmaf(v, v, ss);
  }
  const float scale = __frsqrt_rn(fmaf(block_sum(ss, red), inv_w, eps));
#pragma unroll 4
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    const float v = delta ? sum_out[(size_t)r * width + c] : load_f(xr, c);
    store_f(out, out_bf16, (size_t)r * out_pitch + c, v * scale * gamma[c]);
  }
}

// Row norms over a thread-block cluster: a decode batch has a few rows of a
// few thousand columns, so each row is spread over the `n` CTAs of one
// cluster (CTA rank r owns columns [r * per, (r + 1) * per), each thread up
// to kClusterVals of them, held in registers); the CTAs' sums of squares
// meet through distributed shared memory, added in rank order on every CTA.
constexpr int kClusterVals = 4, kClusterThreads = 256, kClusterMax = 8;

// Sum over the cluster of one value per CTA (every thread gets it).  `slot`
// is a shared float of this CTA that other CTAs read: the caller ends with
// cluster_sync() so that no CTA leaves while its slot may still be read.
__device__ __forceinline__ float cluster_total(float cta_value, float *slot) {
  if (threadIdx.x == 0) *slot = cta_value;
  cluster_sync();
  const unsigned n = cluster_nctarank();
  float t = 0.0f;
  for (unsigned r = 0; r < n; ++r) t += dsmem_load(slot, r);
  return t;
}

template <typename T>
__global__ void __launch_bounds__(kClusterThreads) rms_norm_cluster_kernel(
    const T *x, size_t x_pitch, const float *delta, float *sum_out, int width, const float *gamma, float inv_w,
    float eps, void *out, int out_bf16, size_t out_pitch) {
  pdl_enter();
  __shared__ float red[32];
  __shared__ float slot;
  const int r = blockIdx.y;
  const int n = (int)cluster_nctarank(), per = (width + n - 1) / n;
  const int c0 = (int)cluster_ctarank() * per, c1 = min(width, c0 + per);
  const T *xr = x + (size_t)r * x_pitch;
  float v[kClusterVals];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kClusterVals; ++k) {
    const int c = c0 + threadIdx.x + k * kClusterThreads;
    float e = 0.0f;
    if (c < c1) {
      e = load_f(xr, c);
      if (delta) {
        e += delta[(size_t)r * width + c];
        sum_out[(size_t)r * width + c] = e;
      }
    }
    v[k] = e;
    ss = fmaf(e, e, ss);
  }
  const float tot = cluster_total(block_sum(ss, red), &slot);
  const float scale = __frsqrt_rn(fmaf(tot, inv_w, eps));
#pragma unroll
  for (int k = 0; k < kClusterVals; ++k) {
    const int c = c0 + threadIdx.x + k * kClusterThreads;
    if (c < c1) store_f(out, out_bf16, (size_t)r * out_pitch + c, v[k] * scale * gamma[c]);
  }
  cluster_sync();
}

// Cluster size for rows of `width` columns, or 0 when a row needs more than
// kClusterMax CTAs' registers (the one-CTA-per-row kernels then run).
int cluster_for(size_t width) {
  const size_t n = (width + kClusterThreads - 1) / kClusterThreads;
  const size_t c = std::min<size_t>(kClusterMax, std::max<size_t>(1, n));
  return (width + c - 1) / c <= (size_t)kClusterVals * kClusterThreads ? (int)c : 0;
}

// ---- full attention: head norms, RoPE, cache append --------------------------------------------
struct AttnPrepArgs {
  const float *q_gate;  // [B, q_heads * 2 * head_dim]: per head q then gate
  const float *k;       // [B, k_pitch]: kv_heads * head_dim keys
  const float *v;       // [B, v_pitch]
  long long k_pitch, v_pitch, qg_pitch;
  const float *q_gamma, *k_gamma;
  const int32_t *positions;  // [B] position of this token
  float *q_out;              // [B, q_heads, head_dim]
  float *k_cache, *v_cache;  // [B, max_seq, kv_heads, head_dim]
  int batch, q_heads, kv_heads, head_dim, rotary_dim, max_seq;
  float inv_d, eps;
  float inv_freq[64];  // 1 / theta^(i / half), i < rotary_dim / 2
  int *error;
};

// One warp per (b, head) of q (heads [0, q_heads)) and k (heads [q_heads,
// q_heads + kv_heads)); the k warps also append v.
__global__ void attn_prepare_kernel(const __grid_constant__ AttnPrepArgs a) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int per_b = a.q_heads + a.kv_heads;
  if (item >= a.batch * per_b) return;
  const int b = item / per_b, h = item % per_b;
  const bool is_q = h < a.q_heads;
  const int D = a.head_dim;
  const float *src = is_q ? a.q_gate + (size_t)b * a.qg_pitch + (size_t)h * 2 * D
                          : a.k + (size_t)b * a.k_pitch + (size_t)(h - a.q_heads) * D;
  const float *gamma = is_q ? a.q_gamma : a.k_gamma;
  const int pos = a.positions[b];
  if (pos < 0 || pos >= a.max_seq) {
    if (lane == 0 && a.error) atomicCAS(a.error, 0, 502);
    return;
  }
  float ss = 0.0f;
  for (int c = lane; c < D; c += 32) ss = fmaf(src[c], src[c], ss);
  ss = warp_sum(ss);
  const float scale = __frsqrt_rn(fmaf(ss, a.inv_d, a.eps));
  float *dst = is_q ? a.q_out + ((size_t)b * a.q_heads + h) * D
                    : a.k_cache + (((size_t)b * a.max_seq + pos) * a.kv_heads + (h - a.q_heads)) * D;
  const int half = a.rotary_dim / 2;
  for (int c = lane; c < D; c += 32) {
    const float x = src[c] * scale * gamma[c];
    float y = x;
    if (c < a.rotary_dim) {
      // rotate_half over the rotary dims: cat(-x1, x0) (rope.rs:17-20)
      const int i = c < half ? c : c - half;
      const int pair = c < half ? c + half : c - half;
      const float xp = src[pair] * scale * gamma[pair];
      float sn, cs;
      sincosf((float)pos * a.inv_freq[i], &sn, &cs);
      y = x * cs + (c < half ? -xp : xp) * sn;
    }
    dst[c] = y;
  }
  if (!is_q) {
    const int kvh = h - a.q_heads;
    const float *vs = a.v + (size_t)b * a.v_pitch + (size_t)kvh * D;
    float *vd = a.v_cache + (((size_t)b * a.max_seq + pos) * a.kv_heads + kvh) * D;
    for (int c = lane; c < D; c += 32) vd[c] = vs[c];
  }
}

// ---- split-position GQA decode attention --------------------------------------------------------
// Block (b, kv head, chunk): one warp per query head of the group, positions
// [chunk * chunk_len, min(+chunk_len, pos + 1)), online softmax per warp
// (attention.rs:128-168), partial (max, sum, numerator) to the workspace.
constexpr int kAttnMaxD = 256;

__global__ void attn_decode_partial_kernel(const float *q, const float *k_cache, const float *v_cache,
                                           const int32_t *positions, int batch, int q_heads, int kv_heads, int D,
                                           int max_seq, int chunk_len, int chunks, float scale, float *part) {
  pdl_enter();
  const int group = q_heads / kv_heads;
  const int lane = threadIdx.x & 31, w = threadIdx.x / 32;
  const int bk = blockIdx.x, chunk = blockIdx.y;
  const int b = bk / kv_heads, kvh = bk % kv_heads;
  const int qh = kvh * group + w;
  if (w >= group) return;
  const int limit = min(positions[b], max_seq - 1) + 1;  // positions 0 .. pos
  const int t0 = chunk * chunk_len, t1 = min(limit, t0 + chunk_len);
  float *out = part + (((size_t)b * q_heads + qh) * chunks + chunk) * (D + 2);
  constexpr int kPer = kAttnMaxD / 32;
  float qv[kPer], acc[kPer];
  const float *qr = q + ((size_t)b * q_heads + qh) * D;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int c = lane + 32 * i;
    qv[i] = c < D ? qr[c] : 0.0f;
    acc[i] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  for (int t = t0; t < t1; ++t) {
    const float *kr = k_cache + (((size_t)b * max_seq + t) * kv_heads + kvh) * D;
    float dot = 0.0f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = lane + 32 * i;
      if (c < D) dot = fmaf(qv[i], kr[c], dot);
    }
    const float score = warp_sum(dot) * scale;
    const float mn = fmaxf(m, score);
    const float old_w = expf(m - mn), new_w = expf(score - mn);
    const float *vr = v_cache + (((size_t)b * max_seq + t) * kv_heads + kvh) * D;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = lane + 32 * i;
      if (c < D) acc[i] = acc[i] * old_w + vr[c] * new_w;
    }
    l = l * old_w + new_w;
    m = mn;
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int c = lane + 32 * i;
    if (c < D) out[c] = acc[i];
  }
  if (lane == 0) {
    out[D] = m;
    out[D + 1] = l;
  }
}

// The same partials from a shared-memory tile: block (b, kv head, chunk of
// kAttnTile positions); the tile's K and V rows are loaded by all threads as
// 16-byte pieces (each row 1 KB contiguous) into rows padded to 260 floats
// (a warp's 16-byte reads of 32 rows fall on distinct banks), with the
// group's q vectors.  Warp h scores query head h against the tile (lane t:
// position t), takes the tile's max and sum of exponentials with warp
// shuffles, and accumulates p . V with lanes over the head dimension.
constexpr int kAttnTile = 32, kAttnPitch = kAttnMaxD + 4, kAttnTileThreads = 256;

__global__ void __launch_bounds__(kAttnTileThreads) attn_decode_tile_kernel(
    const float *q, const float *k_cache, const float *v_cache, const int32_t *positions, int q_heads, int kv_heads,
    int D, int max_seq, int chunks, float scale, float *part) {
  pdl_enter();
  extern __shared__ float4 attn_sm[];
  float *ks = reinterpret_cast<float *>(attn_sm);  // [kAttnTile][kAttnPitch]
  float *vs = ks + kAttnTile * kAttnPitch;         // [kAttnTile][kAttnPitch]
  float *qs = vs + kAttnTile * kAttnPitch;         // [group][D]
  const int group = q_heads / kv_heads;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int bk = blockIdx.x, chunk = blockIdx.y;
  const int b = bk / kv_heads, kvh = bk % kv_heads;
  const int limit = min(positions[b], max_seq - 1) + 1;  // positions 0 .. pos
  const int t0 = chunk * kAttnTile, n = min(limit - t0, kAttnTile);
  if (n <= 0) return;  // past this row's position: not read by the merge
  const int d4 = D / 4;
  for (int i = tid; i < n * d4; i += kAttnTileThreads) {
    const int r = i / d4, c = i % d4;
    const size_t g = (((size_t)b * max_seq + t0 + r) * kv_heads + kvh) * D + 4 * c;
    reinterpret_cast<float4 *>(ks + r * kAttnPitch)[c] = __ldg(reinterpret_cast<const float4 *>(k_cache + g));
    reinterpret_cast<float4 *>(vs + r * kAttnPitch)[c] = __ldg(reinterpret_cast<const float4 *>(v_cache + g));
  }
  for (int i = tid; i < group * d4; i += kAttnTileThreads) {
    const int h = i / d4, c = i % d4;
    reinterpret_cast<float4 *>(qs + h * D)[c] =
        __ldg(reinterpret_cast<const float4 *>(q + ((size_t)b * q_heads + kvh * group + h) * D) + c);
  }
  __syncthreads();
  for (int h = w; h < group; h += kAttnTileThreads / 32) {
    const int qh = kvh * group + h;
    float sc = 0.0f;
    if (lane < n) {
      const float4 *kr = reinterpret_cast<const float4 *>(ks + lane * kAttnPitch);
      const float4 *qr = reinterpret_cast<const float4 *>(qs + h * D);
      for (int c = 0; c < d4; ++c) {
        const float4 kv = kr[c], qv = qr[c];
        sc = fmaf(qv.x, kv.x, sc);
        sc = fmaf(qv.y, kv.y, sc);
        sc = fmaf(qv.z, kv.z, sc);
        sc = fmaf(qv.w, kv.w, sc);
      }
      sc *= scale;
    }
    float m = lane < n ? sc : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float p = lane < n ? expf(sc - m) : 0.0f;
    const float l = warp_sum(p);
    constexpr int kPer = kAttnMaxD / 32;
    float acc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
    for (int t = 0; t < n; ++t) {
      const float pt = __shfl_sync(0xffffffffu, p, t);
      const float *vr = vs + t * kAttnPitch;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (lane + 32 * i < D) acc[i] = fmaf(pt, vr[lane + 32 * i], acc[i]);
    }
    float *out = part + (((size_t)b * q_heads + qh) * chunks + chunk) * (D + 2);
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i < D) out[lane + 32 * i] = acc[i];
    if (lane == 0) {
      out[D] = m;
      out[D + 1] = l;
    }
  }
}

// The same partials with K and V rows read straight from global memory (no
// shared-memory tile): block (b, kv head, chunk of kAttnTile positions), 8
// warps, D = 32 * DPL.  Lane l holds columns [l * DPL, (l + 1) * DPL) of
// every query head of the group in registers (group * DPL <= 64).
//  1. scores: warp w takes positions w, w + 8, ...; it reads each K row once
//     (a coalesced row per warp) and reduces each head's dot product over
//     the lanes;
//  2. softmax: warp w takes heads w, w + 8, ... (lane t: position t), the
//     tile's max and sum of exponentials;
//  3. p . V: warp w owns 32 columns (slice w % DPL) of the heads w / DPL,
//     + 8 / DPL, ...; it reads each V row's slice once.
// Each K and V element crosses the SM once.  The tile kernel above staged
// the rows in shared memory and had each of the group's warps read all of
// them: shared-memory bound at 3 CTAs per SM.
template <int DPL>
__global__ void __launch_bounds__(256) attn_decode_rows_kernel(const float *q, const float *k_cache,
                                                               const float *v_cache, const int32_t *positions,
                                                               int q_heads, int kv_heads, int max_seq, int chunks,
                                                               float scale, float *part) {
  pdl_enter();
  constexpr int D = 32 * DPL, kMaxHeads = 64 / DPL, kSlicesPerHead = DPL, kHeadStride = 8 / DPL;
  constexpr int kAccHeads = kMaxHeads / kHeadStride;  // heads a warp accumulates in step 3
  __shared__ float sc[32][kAttnTile + 1];             // [head][position]: scores, then probabilities
  const int group = q_heads / kv_heads;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int bk = blockIdx.x, chunk = blockIdx.y;
  const int b = bk / kv_heads, kvh = bk % kv_heads;
  const int limit = min(positions[b], max_seq - 1) + 1;
  const int t0 = chunk * kAttnTile, n = min(limit - t0, kAttnTile);
  if (n <= 0) return;  // past this row's position: not read by the merge
  auto load_slice = [&](const float *src, float (&dst)[DPL]) {
    if constexpr (DPL % 4 == 0) {
#pragma unroll
      for (int j = 0; j < DPL / 4; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(src) + j);
        dst[4 * j] = v.x; dst[4 * j + 1] = v.y; dst[4 * j + 2] = v.z; dst[4 * j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < DPL / 2; ++j) {
        const float2 v = __ldg(reinterpret_cast<const float2 *>(src) + j);
        dst[2 * j] = v.x; dst[2 * j + 1] = v.y;
      }
    }
  };
  float qv[kMaxHeads][DPL];
#pragma unroll
  for (int h = 0; h < kMaxHeads; ++h) {
    if (h < group) {
      load_slice(q + ((size_t)b * q_heads + kvh * group + h) * D + lane * DPL, qv[h]);
    } else {
#pragma unroll
      for (int j = 0; j < DPL; ++j) qv[h][j] = 0.0f;
    }
  }
  // 1. scores: the warp's (up to) four K rows requested together
  constexpr int kRowsPerWarp = kAttnTile / 8;
  float kx[kRowsPerWarp][DPL];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int t = w + 8 * i;
    if (t < n) load_slice(k_cache + (((size_t)b * max_seq + t0 + t) * kv_heads + kvh) * D + lane * DPL, kx[i]);
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int t = w + 8 * i;
    if (t >= n) break;  // warp-uniform
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h < group) {
        float sdot = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) sdot = fmaf(qv[h][j], kx[i][j], sdot);
        sdot = warp_sum(sdot);
        if (lane == 0) sc[h][t] = sdot * scale;
      }
    }
  }
  __syncthreads();
  // 2. softmax of each head over the tile
  for (int h = w; h < group; h += 8) {
    const float sv = lane < n ? sc[h][lane] : -INFINITY;
    float m = sv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float p = lane < n ? expf(sv - m) : 0.0f;
    const float l = warp_sum(p);
    sc[h][lane] = p;
    if (lane == 0) {
      float *out = part + (((size_t)b * q_heads + kvh * group + h) * chunks + chunk) * (D + 2);
      out[D] = m;
      out[D + 1] = l;
    }
  }
  __syncthreads();
  // 3. p . V: column d = slice * 32 + lane of heads h0, h0 + kHeadStride, ...
  const int slice = w % kSlicesPerHead, h0 = w / kSlicesPerHead;
  const int d = slice * 32 + lane;
  float acc[kAccHeads];
#pragma unroll
  for (int i = 0; i < kAccHeads; ++i) acc[i] = 0.0f;
  const float *vcol = v_cache + ((size_t)b * max_seq + t0) * kv_heads * D + (size_t)kvh * D + d;
  const size_t vstride = (size_t)kv_heads * D;
  float vv[kAttnTile];  // the column's tile, all requested before use
#pragma unroll
  for (int t = 0; t < kAttnTile; ++t) vv[t] = t < n ? __ldg(vcol + (size_t)t * vstride) : 0.0f;
#pragma unroll
  for (int t = 0; t < kAttnTile; ++t) {
#pragma unroll
    for (int i = 0; i < kAccHeads; ++i) {
      const int h = h0 + i * kHeadStride;
      if (h < group && t < n) acc[i] = fmaf(sc[h][t], vv[t], acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < kAccHeads; ++i) {
    const int h = h0 + i * kHeadStride;
    if (h < group) part[(((size_t)b * q_heads + kvh * group + h) * chunks + chunk) * (D + 2) + d] = acc[i];
  }
}

// Merge of the tile kernel's chunks with the output gate: one block per
// (b, q head); the chunk weights exp(m_c - m) in shared memory, threads over
// the head dimension.
__global__ void attn_decode_merge_kernel(const float *part, const float *q_gate, long long qg_pitch,
                                         const int32_t *positions, int q_heads, int D, int max_seq, int chunk_len,
                                         int chunks, void *out, int out_bf16) {
  pdl_enter();
  extern __shared__ float wsm[];  // [chunks]
  __shared__ float red[32];
  const int item = blockIdx.x, b = item / q_heads, h = item % q_heads;
  const int limit = min(positions[b], max_seq - 1) + 1;
  const int used = (limit + chunk_len - 1) / chunk_len;
  const float *pp = part + (size_t)item * chunks * (D + 2);
  float m = -INFINITY;
  for (int c = threadIdx.x; c < used; c += blockDim.x) m = fmaxf(m, pp[(size_t)c * (D + 2) + D]);
  m = -block_min(-m, red);
  float l = 0.0f;
  for (int c = threadIdx.x; c < used; c += blockDim.x) {
    const float wc = expf(pp[(size_t)c * (D + 2) + D] - m);
    wsm[c] = wc;
    l += pp[(size_t)c * (D + 2) + D + 1] * wc;
  }
  const float inv_l = 1.0f / block_sum(l, red);  // its barriers also publish wsm
  const float *gate = q_gate + (size_t)b * qg_pitch + (size_t)h * 2 * D + D;
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    // four independent partial sums, eight chunks' loads in flight
    float num[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int c = 0;
    for (; c + 8 <= used; c += 8) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = pp[(size_t)(c + i) * (D + 2) + j];
#pragma unroll
      for (int i = 0; i < 8; ++i) num[i & 3] = fmaf(v[i], wsm[c + i], num[i & 3]);
    }
    for (; c < used; ++c) num[c & 3] = fmaf(pp[(size_t)c * (D + 2) + j], wsm[c], num[c & 3]);
    const float total = (num[0] + num[1]) + (num[2] + num[3]);
    store_f(out, out_bf16, (size_t)b * q_heads * D + (size_t)h * D + j, total * inv_l * sigmoidf_(gate[j]));
  }
}

// Merges the chunks of each (b, q head) and applies the output gate
// out = attn * sigmoid(gate) (attention.rs:170-190); one warp per (b, head).
__global__ void attn_decode_combine_kernel(const float *part, const float *q_gate, long long qg_pitch,
                                           const int32_t *positions, int batch, int q_heads, int D, int max_seq,
                                           int chunk_len, int chunks, void *out, int out_bf16) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (item >= batch * q_heads) return;
  const int b = item / q_heads, h = item % q_heads;
  const int limit = min(positions[b], max_seq - 1) + 1;
  const int used = (limit + chunk_len - 1) / chunk_len;
  const float *pp = part + (size_t)item * chunks * (D + 2);
  float m = -INFINITY;
  for (int c = 0; c < used; ++c) m = fmaxf(m, pp[(size_t)c * (D + 2) + D]);
  float l = 0.0f;
  for (int c = 0; c < used; ++c) l += pp[(size_t)c * (D + 2) + D + 1] * expf(pp[(size_t)c * (D + 2) + D] - m);
  const float inv_l = 1.0f / l;
  const float *gate = q_gate + (size_t)b * qg_pitch + (size_t)h * 2 * D + D;
  for (int j = lane; j < D; j += 32) {
    float num = 0.0f;
    for (int c = 0; c < used; ++c)
      num += pp[(size_t)c * (D + 2) + j] * expf(pp[(size_t)c * (D + 2) + D] - m);
    const float attn = num * inv_l;
    store_f(out, out_bf16, (size_t)b * q_heads * D + (size_t)h * D + j, attn * sigmoidf_(gate[j]));
  }
}

// ---- gated delta net -----------------------------------------------------------------------------
// Causal depthwise conv over the last `kernel` inputs of each channel, SiLU
// (gdn.rs:6-63); state [B, channels, kernel - 1] holds the previous inputs.
__global__ void gdn_conv_kernel(const float *x, long long x_pitch, float *state, const float *weight, int batch,
                                int channels, int kernel, float *out) {
  pdl_enter();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)batch * channels) return;
  const int b = (int)(i / channels), c = (int)(i % channels);
  float *st = state + i * (kernel - 1);
  const float *wr = weight + (size_t)c * kernel;
  const float cur = x[(size_t)b * x_pitch + c];
  float sum = 0.0f;
  for (int j = 0; j < kernel - 1; ++j) sum = fmaf(st[j], wr[j], sum);
  sum = fmaf(cur, wr[kernel - 1], sum);
  out[i] = sum / (1.0f + expf(-sum));
  for (int j = 0; j + 1 < kernel - 1; ++j) st[j] = st[j + 1];
  st[kernel - 2] = cur;
}

// The delta rule for one token (gdn.rs:206-263): memory_j = decay * sum_i
// S[i][j] k_i, delta_j = (v_j - memory_j) * beta, S[i][j] = S[i][j] * decay +
// k_i delta_j, out_j = sum_i S[i][j] q_i, with q, k L2-normalised (q also by
// 1/sqrt(dk)).  Block (b * value_heads + h, column group).  With dk = 128
// and 64-column groups (the config's heads), 256 threads each hold 32 rows of
// one column in registers: the state is read once and written once, and the
// four row groups' partial sums meet in shared memory (fixed order).  Other
// shapes: one thread per column, two passes over the state.
constexpr int kDeltaRows = 32, kDeltaRowGroups = 4, kDeltaCols = 64, kDeltaThreads = 256;
__global__ void gdn_delta_kernel(const float *conv_out, int conv_dim, const float *a, const float *bgate,
                                 long long ab_pitch, const float *a_log, const float *dt_bias, float *state,
                                 int batch, int key_heads, int value_heads, int dk, int dv, float eps,
                                 float inv_sqrt_dk, float *out) {
  pdl_enter();
  extern __shared__ float sh[];  // q[dk], k[dk], reduction scratch [2 * warps], partial sums
  float *qs = sh, *ks = sh + dk, *red = sh + 2 * dk;
  const int b = blockIdx.x / value_heads, h = blockIdx.x % value_heads;
  const int kh = h / (value_heads / key_heads);
  const float *x = conv_out + (size_t)b * conv_dim;
  const int key_dim = key_heads * dk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid / 32, warps = blockDim.x / 32;
  float sq = 0.0f, sk = 0.0f;
  for (int i = tid; i < dk; i += blockDim.x) {
    const float qv = x[kh * dk + i], kv = x[key_dim + kh * dk + i];
    qs[i] = qv;
    ks[i] = kv;
    sq = fmaf(qv, qv, sq);
    sk = fmaf(kv, kv, sk);
  }
  sq = warp_sum(sq);
  sk = warp_sum(sk);
  if (lane == 0) {
    red[warp] = sq;
    red[warps + warp] = sk;
  }
  __syncthreads();
  float tq = 0.0f, tk = 0.0f;
  for (int w = 0; w < warps; ++w) {
    tq += red[w];
    tk += red[warps + w];
  }
  const float q_scale = __frsqrt_rn(tq + eps) * inv_sqrt_dk, k_scale = __frsqrt_rn(tk + eps);
  const float bv = bgate[(size_t)b * ab_pitch + h], av = a[(size_t)b * ab_pitch + h];
  const float beta = 1.0f / (1.0f + expf(-bv));
  const float xs = av + dt_bias[h];
  const float tiny = expf(fminf(xs, 0.0f));
  const float series = tiny - tiny * tiny * 0.5f + tiny * tiny * tiny * 0.33333334f;
  const float ordinary = fmaxf(xs, 0.0f) + logf(1.0f + expf(-fabsf(xs)));
  const float softplus = xs < -8.0f ? series : ordinary;
  const float decay = expf(-(expf(a_log[h]) * softplus));
  float *S = state + ((size_t)b * value_heads + h) * dk * dv;
  const float *v = x + 2 * key_dim + (size_t)h * dv;
  if (dk == kDeltaRowGroups * kDeltaRows && dv == kDeltaCols * (int)gridDim.y && blockDim.x == kDeltaThreads) {
    // Thread (group, column): rows [group * 32, +32) of one state column,
    // held in registers between the two products (one read, one write).
    float *part = red + 2 * warps;  // [2][groups][cols]
    const int col = tid % kDeltaCols, grp = tid / kDeltaCols;
    const int j = blockIdx.y * kDeltaCols + col, i0 = grp * kDeltaRows;
    float sv[kDeltaRows];
#pragma unroll
    for (int r = 0; r < kDeltaRows; ++r) sv[r] = S[(size_t)(i0 + r) * dv + j];
    float mem = 0.0f;
#pragma unroll
    for (int r = 0; r < kDeltaRows; ++r) mem = fmaf(sv[r], ks[i0 + r] * k_scale, mem);
    part[grp * kDeltaCols + col] = mem;
    __syncthreads();
    mem = 0.0f;
#pragma unroll
    for (int g2 = 0; g2 < kDeltaRowGroups; ++g2) mem += part[g2 * kDeltaCols + col];
    mem *= decay;
    const float delta = (v[j] - mem) * beta;
    float o = 0.0f;
#pragma unroll
    for (int r = 0; r < kDeltaRows; ++r) {
      const float nxt = fmaf(sv[r], decay, ks[i0 + r] * k_scale * delta);
      S[(size_t)(i0 + r) * dv + j] = nxt;
      o = fmaf(nxt, qs[i0 + r] * q_scale, o);
    }
    float *part2 = part + kDeltaRowGroups * kDeltaCols;
    part2[grp * kDeltaCols + col] = o;
    __syncthreads();
    if (grp == 0) {
      o = 0.0f;
#pragma unroll
      for (int g2 = 0; g2 < kDeltaRowGroups; ++g2) o += part2[g2 * kDeltaCols + col];
      out[((size_t)b * value_heads + h) * dv + j] = o;
    }
    return;
  }
  for (int j = blockIdx.y * blockDim.x + tid; j < dv; j += blockDim.x * gridDim.y) {
    float mem = 0.0f;
    for (int i = 0; i < dk; ++i) mem = fmaf(S[(size_t)i * dv + j], ks[i] * k_scale, mem);
    mem *= decay;
    const float delta = (v[j] - mem) * beta;
    float o = 0.0f;
    for (int i = 0; i < dk; ++i) {
      const float nxt = fmaf(S[(size_t)i * dv + j], decay, ks[i] * k_scale * delta);
      S[(size_t)i * dv + j] = nxt;
      o = fmaf(nxt, qs[i] * q_scale, o);
    }
    out[((size_t)b * value_heads + h) * dv + j] = o;
  }
}

// The whole GDN mixer step after the projections in one launch, for the
// config's heads (dk = dv = 128, two value heads per key head, conv kernel
// <= 8): block (b, key head) of 512 threads.
//  1. conv1d_silu (gdn.rs:6-63) of the block's 512 channels (the key head's
//     q and k channels, its two value heads' v channels), one per thread,
//     state shifted in place;
//  2. q, k L2 norms (block reductions);
//  3. delta_step (gdn.rs:206-263) for both value heads: thread (row half,
//     column) holds 64 state rows of one column in registers;
//  4. gated RMSNorm times SiLU(z) (gdn.rs:266-278), out [B, value_dim].
constexpr int kGdnThreads = 512, kGdnD = 128, kGdnRows = 64;
__global__ void __launch_bounds__(kGdnThreads, 1) gdn_step_kernel(
    const float *x, long long x_pitch, float *conv_state, const float *conv_w, int conv_kernel, const float *a,
    const float *bgate, long long ab_pitch, const float *a_log, const float *dt_bias, float *state, const float *z,
    long long z_pitch, const float *gamma, int key_heads, float eps, float inv_sqrt_dk, void *out, int out_bf16) {
  pdl_enter();
  __shared__ float qs[kGdnD], ks[kGdnD], vs[2 * kGdnD];
  __shared__ float part[2][2 * kGdnD], part2[2][2 * kGdnD];
  __shared__ float red[32];
  const int b = blockIdx.x / key_heads, kh = blockIdx.x % key_heads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int key_dim = key_heads * kGdnD, value_heads = 2 * key_heads;
  const int conv_dim = 2 * key_dim + value_heads * kGdnD;
  // 1. conv + SiLU
  {
    const int c = tid < kGdnD ? kh * kGdnD + tid
                : tid < 2 * kGdnD ? key_dim + kh * kGdnD + (tid - kGdnD)
                                  : 2 * key_dim + kh * 2 * kGdnD + (tid - 2 * kGdnD);
    float *st = conv_state + ((size_t)b * conv_dim + c) * (conv_kernel - 1);
    const float *wr = conv_w + (size_t)c * conv_kernel;
    const float cur = x[(size_t)b * x_pitch + c];
    float hist[8];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 7; ++j)
      if (j < conv_kernel - 1) {
        hist[j] = st[j];
        sum = fmaf(hist[j], wr[j], sum);
      }
    sum = fmaf(cur, wr[conv_kernel - 1], sum);
    const float o = sum / (1.0f + expf(-sum));
#pragma unroll
    for (int j = 0; j < 6; ++j)
      if (j + 1 < conv_kernel - 1) st[j] = hist[j + 1];
    st[conv_kernel - 2] = cur;
    if (tid < kGdnD)
      qs[tid] = o;
    else if (tid < 2 * kGdnD)
      ks[tid - kGdnD] = o;
    else
      vs[tid - 2 * kGdnD] = o;
  }
  __syncthreads();
  // 2. L2 norms: warps 0-3 hold q, warps 4-7 k
  {
    float v2 = 0.0f;
    if (tid < kGdnD)
      v2 = qs[tid] * qs[tid];
    else if (tid < 2 * kGdnD)
      v2 = ks[tid - kGdnD] * ks[tid - kGdnD];
    v2 = warp_sum(v2);
    if (lane == 0 && warp < 8) red[warp] = v2;
  }
  __syncthreads();
  const float q_scale = __frsqrt_rn(red[0] + red[1] + red[2] + red[3] + eps) * inv_sqrt_dk;
  const float k_scale = __frsqrt_rn(red[4] + red[5] + red[6] + red[7] + eps);
  // 3. gates and the delta rule; thread (rg, col): head j = col / 128, column jc
  const int col = tid & (2 * kGdnD - 1), rg = tid >> 8;
  const int j = col >> 7, jc = col & (kGdnD - 1), h = 2 * kh + j;
  const float bv = bgate[(size_t)b * ab_pitch + h], av = a[(size_t)b * ab_pitch + h];
  const float beta = 1.0f / (1.0f + expf(-bv));
  const float xs = av + dt_bias[h];
  const float tiny = expf(fminf(xs, 0.0f));
  const float series = tiny - tiny * tiny * 0.5f + tiny * tiny * tiny * 0.33333334f;
  const float ordinary = fmaxf(xs, 0.0f) + logf(1.0f + expf(-fabsf(xs)));
  const float softplus = xs < -8.0f ? series : ordinary;
  const float decay = expf(-(expf(a_log[h]) * softplus));
  float *S = state + ((size_t)b * value_heads + h) * kGdnD * kGdnD;
  const int i0 = rg * kGdnRows;
  float sv[kGdnRows];
#pragma unroll
  for (int r = 0; r < kGdnRows; ++r) sv[r] = S[(size_t)(i0 + r) * kGdnD + jc];
  float mem = 0.0f;
#pragma unroll
  for (int r = 0; r < kGdnRows; ++r) mem = fmaf(sv[r], ks[i0 + r] * k_scale, mem);
  part[rg][col] = mem;
  __syncthreads();
  mem = (part[0][col] + part[1][col]) * decay;
  const float delta = (vs[col] - mem) * beta;
  float o = 0.0f;
#pragma unroll
  for (int r = 0; r < kGdnRows; ++r) {
    const float nxt = fmaf(sv[r], decay, ks[i0 + r] * k_scale * delta);
    S[(size_t)(i0 + r) * kGdnD + jc] = nxt;
    o = fmaf(nxt, qs[i0 + r] * q_scale, o);
  }
  part2[rg][col] = o;
  __syncthreads();
  // 4. gated norm: threads of row half 0 hold the 256 outputs (warps 0-3:
  // head 0, warps 4-7: head 1)
  o = part2[0][col] + part2[1][col];
  float o2 = warp_sum(rg == 0 ? o * o : 0.0f);
  if (lane == 0 && rg == 0) red[8 + warp] = o2;
  __syncthreads();
  if (rg == 0) {
    const float ss = red[8 + 4 * j] + red[9 + 4 * j] + red[10 + 4 * j] + red[11 + 4 * j];
    const float scale = __frsqrt_rn(fmaf(ss, 1.0f / kGdnD, eps));
    const float zz = z[(size_t)b * z_pitch + (size_t)h * kGdnD + jc];
    store_f(out, out_bf16, (size_t)b * value_heads * kGdnD + (size_t)h * kGdnD + jc,
            o * scale * gamma[jc] * zz / (1.0f + expf(-zz)));
  }
}

// RMSNorm of each value head's output (gated_norm gamma [dv]) times SiLU(z)
// (gdn.rs:266-278); one warp per (b, head); out [B, value_heads * dv].
__global__ void gdn_gated_norm_kernel(const float *x, const float *z, long long z_pitch, const float *gamma,
                                      int batch, int heads, int dv, float inv_dv, float eps, void *out,
                                      int out_bf16) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (item >= batch * heads) return;
  const int b = item / heads, h = item % heads;
  const float *xr = x + (size_t)item * dv;
  float ss = 0.0f;
  for (int c = lane; c < dv; c += 32) ss = fmaf(xr[c], xr[c], ss);
  ss = warp_sum(ss);
  const float scale = __frsqrt_rn(fmaf(ss, inv_dv, eps));
  const float *zr = z + (size_t)b * z_pitch + (size_t)h * dv;
  for (int c = lane; c < dv; c += 32) {
    const float n = xr[c] * scale * gamma[c];
    const float zz = zr[c];
    store_f(out, out_bf16, (size_t)b * heads * dv + (size_t)h * dv + c, n * zz / (1.0f + expf(-zz)));
  }
}

// ---- decode MoE combine + residual + RMSNorm ------------------------------------------------------
// out[t] = residual[t] + sum_s w[t, s] * routed[row(t, s)] (slots in order,
// moe.rs:111-147); normed = RMSNorm(out) * gamma.  row(t, s) = t * slots + s,
// or with `map` (the distinct-expert MoE GEMV's output [cap, tokens, hidden])
// map[t * slots + s] * tokens + t.  One block per token; the slots' rows and
// weights are read once into registers / shared memory per column group.
constexpr int kCombineMaxSlots = 32;
__global__ void decode_combine_add_norm_kernel(const float *routed, const int32_t *map, const float *weights,
                                               int width, int slots, int tokens, const float *residual,
                                               const float *gamma, int hidden, float inv_h, float eps, float *out,
                                               void *normed, int normed_bf16) {
  pdl_enter();
  __shared__ float red[32];
  __shared__ float w_s[kCombineMaxSlots];
  __shared__ const float *row_s[kCombineMaxSlots];
  const int t = blockIdx.x;
  if (threadIdx.x < slots) {
    const int s = threadIdx.x;
    w_s[s] = weights[(size_t)t * width + s];
    const long long row = map ? (long long)max(map[(size_t)t * slots + s], 0) * tokens + t : (long long)t * slots + s;
    row_s[s] = routed + row * hidden;
  }
  __syncthreads();
  float ss = 0.0f;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    float acc = 0.0f;
    for (int s = 0; s < slots; ++s) acc = fmaf(w_s[s], row_s[s][c], acc);
    const float v = residual[(size_t)t * hidden + c] + acc;
    out[(size_t)t * hidden + c] = v;
    ss = fmaf(v, v, ss);
  }
  const float scale = __frsqrt_rn(fmaf(block_sum(ss, red), inv_h, eps));
  for (int c = threadIdx.x; c < hidden; c += blockDim.x)
    store_f(normed, normed_bf16, (size_t)t * hidden + c, out[(size_t)t * hidden + c] * scale * gamma[c]);
}

// The same over a cluster per token (see rms_norm_cluster_kernel).
__global__ void __launch_bounds__(kClusterThreads) decode_combine_add_norm_cluster_kernel(
    const float *routed, const int32_t *map, const float *weights, int width, int slots, int tokens,
    const float *residual, const float *gamma, int hidden, float inv_h, float eps, float *out, void *normed,
    int normed_bf16) {
  pdl_enter();
  __shared__ float red[32];
  __shared__ float slot;
  __shared__ float w_s[kCombineMaxSlots];
  __shared__ const float *row_s[kCombineMaxSlots];
  const int t = blockIdx.y;
  if (threadIdx.x < slots) {
    const int s = threadIdx.x;
    w_s[s] = weights[(size_t)t * width + s];
    const long long row = map ? (long long)max(map[(size_t)t * slots + s], 0) * tokens + t : (long long)t * slots + s;
    row_s[s] = routed + row * hidden;
  }
  __syncthreads();
  const int n = (int)cluster_nctarank(), per = (hidden + n - 1) / n;
  const int c0 = (int)cluster_ctarank() * per, c1 = min(hidden, c0 + per);
  float v[kClusterVals];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kClusterVals; ++k) {
    const int c = c0 + threadIdx.x + k * kClusterThreads;
    float e = 0.0f;
    if (c < c1) {
      float acc = 0.0f;
      for (int s = 0; s < slots; ++s) acc = fmaf(w_s[s], row_s[s][c], acc);
      e = residual[(size_t)t * hidden + c] + acc;
      out[(size_t)t * hidden + c] = e;
    }
    v[k] = e;
    ss = fmaf(e, e, ss);
  }
  const float tot = cluster_total(block_sum(ss, red), &slot);
  const float scale = __frsqrt_rn(fmaf(tot, inv_h, eps));
#pragma unroll
  for (int k = 0; k < kClusterVals; ++k) {
    const int c = c0 + threadIdx.x + k * kClusterThreads;
    if (c < c1) store_f(normed, normed_bf16, (size_t)t * hidden + c, v[k] * scale * gamma[c]);
  }
  cluster_sync();
}

// ---- greedy sampling ----------------------------------------------------------------------------------
// Largest finite logit of each row, lowest index among equals (greedy,
// generation.rs:34-42); the token becomes the next input, its position
// advances by one and it is appended to the history.
__global__ void argmax_advance_kernel(const float *logits, int vocab, int32_t *tokens, int32_t *positions,
                                      int32_t *history, int history_len, int32_t *step) {
  pdl_enter();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int b = blockIdx.x;
  const float *row = logits + (size_t)b * vocab;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int c = threadIdx.x; c < vocab; c += blockDim.x) {
    const float v = row[c];
    if (isfinite(v) && (v > best || (v == best && c < idx))) {
      best = v;
      idx = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x / 32;
  if (lane == 0) {
    bv[w] = best;
    bi[w] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x / 32); ++i)
      if (bv[i] > best || (bv[i] == best && bi[i] < idx)) {
        best = bv[i];
        idx = bi[i];
      }
    if (idx == 0x7fffffff) idx = 0;  // no finite logit
    tokens[b] = idx;
    positions[b] += 1;
    if (history) {
      const int s = *step;
      if (s < history_len) history[(size_t)b * history_len + s] = idx;
    }
  }
  // the step counter advances once every row has read it: the last block does it
  if (step && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(step + 1, 1) == (int)gridDim.x - 1) {
      step[1] = 0;
      step[0] += 1;
    }
  }
}

unsigned blocks_for(size_t n, int per_block) { return (unsigned)((n + per_block - 1) / per_block); }

}  // namespace
}  // namespace fpb

using namespace fpb;

#define FPB_LAUNCH(kernel, grid, block, smem, s, ...)                            \
  do {                                                                          \
    cudaError_t e_ = launch_pdl(kernel, grid, block, smem, s, __VA_ARGS__);     \
    if (e_ != cudaSuccess) return cuda_fail(e_, #kernel);                       \
    FPB_LAUNCH_CHECK(#kernel);                                                  \
  } while (0)

extern "C" int fpb_embedding(const void *table_bf16, size_t vocab, size_t hidden, const int32_t *ids, size_t rows,
                             float *out, void *stream) {
  if (!table_bf16 || !ids || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_embedding: null pointer");
  if (rows == 0 || rows > 65535 || hidden == 0 || vocab == 0 || vocab > 0x7fffffff || hidden > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_embedding: shape");
  FPB_LAUNCH(embedding_kernel, dim3((unsigned)std::min<size_t>(8, (hidden + 255) / 256), (unsigned)rows), 256, 0,
             as_stream(stream), static_cast<const __nv_bfloat16 *>(table_bf16), ids, (int)rows, (int)hidden,
             (int)vocab, out, device_error_ptr());
  return FPB_OK;
}

extern "C" int fpb_rms_norm(const void *x, int x_dtype, size_t x_pitch, const float *residual_delta,
                            float *sum_out, size_t rows, size_t width, const float *gamma, float eps, void *out,
                            int out_dtype, size_t out_pitch, void *stream) {
  if (!x || !gamma || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_rms_norm: null pointer");
  if ((residual_delta != nullptr) != (sum_out != nullptr) || (residual_delta && x_dtype != FPB_F32))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_rms_norm: delta and sum_out go together, with f32 x");
  if (rows == 0 || width == 0 || rows > 0x7fffffff || width > 0x7fffffff || x_pitch < width || out_pitch < width)
    return fail(FPB_ERR_SHAPE, "fpb_rms_norm: shape");
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (out_dtype != FPB_F32 && out_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_rms_norm: dtype");
  const float inv_w = 1.0f / (float)width;
  cudaStream_t s = as_stream(stream);
  if (const int cl = cluster_for(width); cl > 0 && rows <= 65535) {
    const dim3 grid((unsigned)cl, (unsigned)rows);
    cudaError_t e = x_dtype == FPB_F32
        ? launch_pdl_cluster(rms_norm_cluster_kernel<float>, grid, kClusterThreads, 0, s, (unsigned)cl,
                             static_cast<const float *>(x), x_pitch, residual_delta, sum_out, (int)width, gamma,
                             inv_w, eps, out, out_dtype == FPB_BF16, out_pitch)
        : launch_pdl_cluster(rms_norm_cluster_kernel<__nv_bfloat16>, grid, kClusterThreads, 0, s, (unsigned)cl,
                             static_cast<const __nv_bfloat16 *>(x), x_pitch, residual_delta, sum_out, (int)width,
                             gamma, inv_w, eps, out, out_dtype == FPB_BF16, out_pitch);
    if (e != cudaSuccess) return cuda_fail(e, "rms_norm_cluster_kernel");
    FPB_LAUNCH_CHECK("rms_norm_cluster_kernel");
    return FPB_OK;
  }
  if (x_dtype == FPB_F32)
    FPB_LAUNCH(rms_norm_kernel<float>, (unsigned)rows, 256, 0, s, static_cast<const float *>(x), x_pitch,
               residual_delta, sum_out, (int)rows, (int)width, gamma, inv_w, eps, out, out_dtype == FPB_BF16,
               out_pitch);
  else
    FPB_LAUNCH(rms_norm_kernel<__nv_bfloat16>, (unsigned)rows, 256, 0, s,
               static_cast<const __nv_bfloat16 *>(x), x_pitch, residual_delta, sum_out, (int)rows, (int)width,
               gamma, inv_w, eps, out, out_dtype == FPB_BF16, out_pitch);
  return FPB_OK;
}

extern "C" int fpb_attn_prepare(const float *q_gate, size_t qg_pitch, const float *k, size_t k_pitch, const float *v,
                                size_t v_pitch, const float *q_gamma, const float *k_gamma, const int32_t *positions,
                                size_t batch, size_t q_heads, size_t kv_heads, size_t head_dim, size_t rotary_dim,
                                float theta, float eps, size_t max_seq, float *q_out, float *k_cache, float *v_cache,
                                void *stream) {
  if (!q_gate || !k || !v || !q_gamma || !k_gamma || !positions || !q_out || !k_cache || !v_cache)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_attn_prepare: null pointer");
  if (batch == 0 || q_heads == 0 || kv_heads == 0 || q_heads % kv_heads || head_dim == 0 ||
      rotary_dim > head_dim || rotary_dim % 2 || rotary_dim / 2 > 64 || max_seq == 0 ||
      batch * (q_heads + kv_heads) > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_attn_prepare: shape");
  AttnPrepArgs a{};
  a.q_gate = q_gate;
  a.k = k;
  a.v = v;
  a.qg_pitch = (long long)qg_pitch;
  a.k_pitch = (long long)k_pitch;
  a.v_pitch = (long long)v_pitch;
  a.q_gamma = q_gamma;
  a.k_gamma = k_gamma;
  a.positions = positions;
  a.q_out = q_out;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.batch = (int)batch;
  a.q_heads = (int)q_heads;
  a.kv_heads = (int)kv_heads;
  a.head_dim = (int)head_dim;
  a.rotary_dim = (int)rotary_dim;
  a.max_seq = (int)max_seq;
  a.inv_d = 1.0f / (float)head_dim;
  a.eps = eps;
  const int half = (int)rotary_dim / 2;
  for (int i = 0; i < half; ++i) a.inv_freq[i] = 1.0f / powf(theta, (float)i / (float)half);  // rope.rs:110-113
  a.error = device_error_ptr();
  FPB_LAUNCH(attn_prepare_kernel, blocks_for(batch * (q_heads + kv_heads), 8), 256, 0, as_stream(stream), a);
  return FPB_OK;
}

extern "C" size_t fpb_attn_decode_workspace_bytes(size_t batch, size_t q_heads, size_t head_dim, size_t max_seq,
                                                 size_t chunk_len) {
  if (chunk_len == 0) chunk_len = 64;
  const size_t chunks = (max_seq + chunk_len - 1) / chunk_len;
  return batch * q_heads * chunks * (head_dim + 2) * sizeof(float);
}

extern "C" int fpb_attn_decode(const float *q, const float *k_cache, const float *v_cache, const int32_t *positions,
                               const float *q_gate, size_t qg_pitch, size_t batch, size_t q_heads, size_t kv_heads,
                               size_t head_dim, size_t max_seq, size_t chunk_len, float scale, void *workspace,
                               size_t workspace_bytes, void *out, int out_dtype, void *stream) {
  if (!q || !k_cache || !v_cache || !positions || !q_gate || !workspace || !out)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_attn_decode: null pointer");
  if (chunk_len == 0) chunk_len = 64;
  if (batch == 0 || q_heads == 0 || kv_heads == 0 || q_heads % kv_heads || q_heads / kv_heads > 32 ||
      head_dim == 0 || head_dim > (size_t)kAttnMaxD || max_seq == 0 || batch * kv_heads > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_attn_decode: shape (group <= 32, head_dim <= %d)", kAttnMaxD);
  if (out_dtype != FPB_F32 && out_dtype != FPB_BF16)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_attn_decode: dtype");
  const size_t need = fpb_attn_decode_workspace_bytes(batch, q_heads, head_dim, max_seq, chunk_len);
  if (workspace_bytes < need)
    return fail(FPB_ERR_WORKSPACE, "fpb_attn_decode: workspace %zu < %zu bytes", workspace_bytes, need);
  const int chunks = (int)((max_seq + chunk_len - 1) / chunk_len);
  cudaStream_t s = as_stream(stream);
  float *part = static_cast<float *>(workspace);
  const size_t group = q_heads / kv_heads;
  if (chunk_len == (size_t)kAttnTile && chunks <= 65535 && (head_dim == 64 || head_dim == 128 || head_dim == 256) &&
      group * (head_dim / 32) <= 64) {
    const dim3 grid((unsigned)(batch * kv_heads), (unsigned)chunks);
    auto go = [&](auto kernel) {
      FPB_LAUNCH(kernel, grid, 256, 0, s, q, k_cache, v_cache, positions, (int)q_heads, (int)kv_heads, (int)max_seq,
                 chunks, scale, part);
      return (int)FPB_OK;
    };
    const int st = head_dim == 64    ? go(attn_decode_rows_kernel<2>)
                   : head_dim == 128 ? go(attn_decode_rows_kernel<4>)
                                     : go(attn_decode_rows_kernel<8>);
    if (st) return st;
    FPB_LAUNCH(attn_decode_merge_kernel, (unsigned)(batch * q_heads), 256, chunks * sizeof(float), s, part, q_gate,
               (long long)qg_pitch, positions, (int)q_heads, (int)head_dim, (int)max_seq, (int)chunk_len, chunks, out,
               out_dtype == FPB_BF16);
    return FPB_OK;
  }
  if (chunk_len == (size_t)kAttnTile && head_dim % 4 == 0 && chunks <= 8192) {
    const size_t smem = (2 * kAttnTile * kAttnPitch + group * head_dim) * sizeof(float);
    {
      static std::mutex mu;
      static std::vector<int> done;
      int dev = 0;
      cudaGetDevice(&dev);
      std::lock_guard<std::mutex> lock(mu);
      if (std::find(done.begin(), done.end(), dev) == done.end()) {
        FPB_CUDA_TRY(cudaFuncSetAttribute(attn_decode_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)((2 * kAttnTile * kAttnPitch + 32 * kAttnMaxD) * sizeof(float))));
        done.push_back(dev);
      }
    }
    FPB_LAUNCH(attn_decode_tile_kernel, dim3((unsigned)(batch * kv_heads), (unsigned)chunks), kAttnTileThreads, smem,
               s, q, k_cache, v_cache, positions, (int)q_heads, (int)kv_heads, (int)head_dim, (int)max_seq, chunks,
               scale, part);
    FPB_LAUNCH(attn_decode_merge_kernel, (unsigned)(batch * q_heads), 256, chunks * sizeof(float), s, part, q_gate,
               (long long)qg_pitch, positions, (int)q_heads, (int)head_dim, (int)max_seq, (int)chunk_len, chunks, out,
               out_dtype == FPB_BF16);
    return FPB_OK;
  }
  // Chunks past a row's position write nothing and are not read.
  FPB_LAUNCH(attn_decode_partial_kernel, dim3((unsigned)(batch * kv_heads), (unsigned)chunks),
             (unsigned)(32 * (q_heads / kv_heads)), 0, s, q, k_cache, v_cache, positions, (int)batch, (int)q_heads,
             (int)kv_heads, (int)head_dim, (int)max_seq, (int)chunk_len, chunks, scale, part);
  FPB_LAUNCH(attn_decode_combine_kernel, blocks_for(batch * q_heads, 8), 256, 0, s, part, q_gate,
             (long long)qg_pitch, positions, (int)batch, (int)q_heads, (int)head_dim, (int)max_seq, (int)chunk_len,
             chunks, out, out_dtype == FPB_BF16);
  return FPB_OK;
}

extern "C" int fpb_gdn_conv(const float *x, size_t x_pitch, float *state, const float *weight, size_t batch,
                            size_t channels, size_t kernel, float *out, void *stream) {
  if (!x || !state || !weight || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_gdn_conv: null pointer");
  if (batch == 0 || channels == 0 || kernel < 2 || kernel > 16 || x_pitch < channels ||
      batch * channels > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_gdn_conv: shape");
  FPB_LAUNCH(gdn_conv_kernel, blocks_for(batch * channels, 256), 256, 0, as_stream(stream), x, (long long)x_pitch,
             state, weight, (int)batch, (int)channels, (int)kernel, out);
  return FPB_OK;
}

extern "C" int fpb_gdn_delta(const float *conv_out, const float *a, const float *b, size_t ab_pitch,
                             const float *a_log, const float *dt_bias, float *state, size_t batch, size_t key_heads,
                             size_t value_heads, size_t dk, size_t dv, float eps, float *out, void *stream) {
  if (!conv_out || !a || !b || !a_log || !dt_bias || !state || !out)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_gdn_delta: null pointer");
  if (batch == 0 || key_heads == 0 || value_heads % key_heads || dk == 0 || dv == 0 || dk > 1024 ||
      batch * value_heads > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_gdn_delta: shape");
  const int conv_dim = (int)(2 * key_heads * dk + value_heads * dv);
  const bool tiled = dk == (size_t)kDeltaRowGroups * kDeltaRows && dv % kDeltaCols == 0 && dv / kDeltaCols <= 65535;
  const dim3 grid((unsigned)(batch * value_heads), tiled ? (unsigned)(dv / kDeltaCols) : 1u);
  const int threads = tiled ? kDeltaThreads : 128;
  const size_t smem = (2 * dk + 2 * (threads / 32) + (tiled ? 2 * kDeltaRowGroups * kDeltaCols : 0)) * sizeof(float);
  FPB_LAUNCH(gdn_delta_kernel, grid, threads, smem, as_stream(stream), conv_out, conv_dim, a, b, (long long)ab_pitch, a_log, dt_bias, state, (int)batch,
             (int)key_heads, (int)value_heads, (int)dk, (int)dv, eps, 1.0f / sqrtf((float)dk), out);
  return FPB_OK;
}

extern "C" int fpb_gdn_gated_norm(const float *x, const float *z, size_t z_pitch, const float *gamma, size_t batch,
                                  size_t heads, size_t dv, float eps, void *out, int out_dtype, void *stream) {
  if (!x || !z || !gamma || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_gdn_gated_norm: null pointer");
  if (batch == 0 || heads == 0 || dv == 0 || batch * heads > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_gdn_gated_norm: shape");
  if (out_dtype != FPB_F32 && out_dtype != FPB_BF16)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_gdn_gated_norm: dtype");
  FPB_LAUNCH(gdn_gated_norm_kernel, blocks_for(batch * heads, 8), 256, 0, as_stream(stream), x, z,
             (long long)z_pitch, gamma, (int)batch, (int)heads, (int)dv, 1.0f / (float)dv, eps, out,
             out_dtype == FPB_BF16);
  return FPB_OK;
}

static int combine_add_norm(const char *name, const float *routed, const int32_t *map, const float *weights,
                            size_t width, size_t slots, const float *residual, const float *gamma, size_t tokens,
                            size_t hidden, float eps, float *out, void *normed, int normed_dtype, void *stream) {
  if (!routed || !weights || !residual || !gamma || !out || !normed)
    return fail(FPB_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (tokens == 0 || tokens > 0x7fffffff || hidden == 0 || hidden > 0x7fffffff || slots == 0 || slots > width ||
      slots > (size_t)kCombineMaxSlots)
    return fail(FPB_ERR_SHAPE, "%s: shape (at most %d slots)", name, kCombineMaxSlots);
  if (normed_dtype != FPB_F32 && normed_dtype != FPB_BF16) return fail(FPB_ERR_INVALID_ARGUMENT, "%s: dtype", name);
  if (const int cl = cluster_for(hidden); cl > 0 && tokens <= 65535) {
    cudaError_t e = launch_pdl_cluster(decode_combine_add_norm_cluster_kernel, dim3((unsigned)cl, (unsigned)tokens),
                                       kClusterThreads, 0, as_stream(stream), (unsigned)cl, routed, map, weights,
                                       (int)width, (int)slots, (int)tokens, residual, gamma, (int)hidden,
                                       1.0f / (float)hidden, eps, out, normed, normed_dtype == FPB_BF16);
    if (e != cudaSuccess) return cuda_fail(e, "decode_combine_add_norm_cluster_kernel");
    FPB_LAUNCH_CHECK("decode_combine_add_norm_cluster_kernel");
    return FPB_OK;
  }
  FPB_LAUNCH(decode_combine_add_norm_kernel, (unsigned)tokens, 256, 0, as_stream(stream), routed, map, weights,
             (int)width, (int)slots, (int)tokens, residual, gamma, (int)hidden, 1.0f / (float)hidden, eps, out, normed,
             normed_dtype == FPB_BF16);
  return FPB_OK;
}

extern "C" int fpb_decode_combine_add_norm(const float *routed, const float *weights, size_t width, size_t slots,
                                           const float *residual, const float *gamma, size_t tokens, size_t hidden,
                                           float eps, float *out, void *normed, int normed_dtype, void *stream) {
  return combine_add_norm("fpb_decode_combine_add_norm", routed, nullptr, weights, width, slots, residual, gamma,
                          tokens, hidden, eps, out, normed, normed_dtype, stream);
}

extern "C" int fpb_moe_decode_combine_add_norm(const float *routed, const int32_t *map, const float *weights,
                                               size_t width, size_t slots, const float *residual, const float *gamma,
                                               size_t tokens, size_t hidden, float eps, float *out, void *normed,
                                               int normed_dtype, void *stream) {
  if (!map) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_moe_decode_combine_add_norm: null map");
  return combine_add_norm("fpb_moe_decode_combine_add_norm", routed, map, weights, width, slots, residual, gamma,
                          tokens, hidden, eps, out, normed, normed_dtype, stream);
}

extern "C" int fpb_argmax_advance(const float *logits, size_t rows, size_t vocab, int32_t *tokens,
                                  int32_t *positions, int32_t *history, size_t history_len, int32_t *step,
                                  void *stream) {
  if (!logits || !tokens || !positions) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_argmax_advance: null pointer");
  if (rows == 0 || rows > 65535 || vocab == 0 || vocab > 0x7fffffff || (history && !step))
    return fail(FPB_ERR_SHAPE, "fpb_argmax_advance: shape");
  FPB_LAUNCH(argmax_advance_kernel, (unsigned)rows, 1024, 0, as_stream(stream), logits, (int)vocab, tokens, positions,
             history, (int)history_len, step);
  return FPB_OK;
}

extern "C" int fpb_gdn_step(const float *x, size_t x_pitch, float *conv_state, const float *conv_weight,
                            size_t conv_kernel, const float *a, const float *b, size_t ab_pitch, const float *a_log,
                            const float *dt_bias, float *state, const float *z, size_t z_pitch, const float *gamma,
                            size_t batch, size_t key_heads, size_t value_heads, size_t dk, size_t dv, float eps,
                            void *out, int out_dtype, void *stream) {
  if (!x || !conv_state || !conv_weight || !a || !b || !a_log || !dt_bias || !state || !z || !gamma || !out)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_gdn_step: null pointer");
  if (out_dtype != FPB_F32 && out_dtype != FPB_BF16) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_gdn_step: dtype");
  if (batch == 0 || key_heads == 0 || batch * key_heads > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_gdn_step: shape");
  if (dk != (size_t)kGdnD || dv != (size_t)kGdnD || value_heads != 2 * key_heads || conv_kernel < 2 ||
      conv_kernel > 8)
    return fail(FPB_ERR_UNSUPPORTED, "fpb_gdn_step: dk = dv = 128, value_heads = 2 * key_heads and a conv kernel "
                "of 2..8 only (other shapes: fpb_gdn_conv, fpb_gdn_delta, fpb_gdn_gated_norm)");
  if (x_pitch < 2 * key_heads * dk + value_heads * dv || z_pitch < value_heads * dv)
    return fail(FPB_ERR_SHAPE, "fpb_gdn_step: pitches");
  FPB_LAUNCH(gdn_step_kernel, (unsigned)(batch * key_heads), kGdnThreads, 0, as_stream(stream), x,
             (long long)x_pitch, conv_state, conv_weight, (int)conv_kernel, a, b, (long long)ab_pitch, a_log,
             dt_bias, state, z, (long long)z_pitch, gamma, (int)key_heads, eps, 1.0f / sqrtf((float)dk), out,
             out_dtype == FPB_BF16);
  return FPB_OK;
}
