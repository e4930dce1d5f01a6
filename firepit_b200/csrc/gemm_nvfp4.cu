// NVFP4 prefill GEMM on the 5th-generation tensor cores
// (crates/firepit-kernels/src/gemm/nvfp4.rs: nvfp4_gemm / nvfp4_gemm_view).
//
//   y[m, n] = ga * g[n] * sum_k E2M1[a(m,k)] e4m3(sa(m,k/16)) E2M1[w(n,k)] e4m3(sw(n,k/16))
//
// Both operands are NVFP4: the weights as stored in the handle, the
// activations quantized on the fly (fpb_nvfp4_quantize_act, per-tensor
// global ga).  One CTA computes a 128 x 128 tile of y:
//   warp 0      TMA producer: per 256-column K block, A and B tiles (128 rows
//               x 128 bytes, 128-byte swizzle) and the four 512-byte scale
//               factor chunks of each operand, into a 4-stage ring;
//   warp 1      allocates TMEM, copies the stage's scale factors to TMEM
//               (tcgen05.cp) and issues four
//               tcgen05.mma.kind::mxf4nvf4.block_scale.block16 (K = 64 each)
//               accumulating in TMEM; tcgen05.commit frees the stage;
//   warps 2-9   epilogue, two per TMEM lane quadrant (64 columns each):
//               tcgen05.ld of the f32 accumulator, times ga * g[n], staged
//               as bf16 or f32 in shared memory (128-byte swizzle) and
//               written by TMA tiled stores, so each row segment leaves as
//               whole 128-byte lines.
// Every TMA load lands in the issuing CTA alone.
//
// Scale factors live in the tensor cores' tiled layout: for each 128-row
// block and each 64-column block, 512 bytes with the factor of row r,
// 16-column group s at byte (r % 32) * 16 + (r / 32) * 4 + s.  The K blocks
// are padded to a multiple of four (256 columns) with zero factors.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "act_quant.cuh"
#include "common.cuh"
#include "matrix_extras.cuh"
#include "nvfp4_matrix.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace fpb {

__device__ int g_device_error;  // first failing kernel's error code (0 = none)

constexpr int kBM = 128, kBN = 128, kBKBytes = 128;  // K block = 256 fp4 columns
constexpr int kStages = 5;

// Row-major e4m3 scales [rows, cols/16] -> tiled, sign cleared (UE4M3).
// Padding entries are written as zero.  One thread per output byte.  With
// glu_inter > 0 tiled row v holds source row glu_source_row(v, glu_inter).
__host__ __device__ inline size_t glu_source_row(size_t v, size_t inter) {
  const size_t e = v / (2 * inter), w = v % (2 * inter);
  return e * 2 * inter + ((w % 128) / 64) * inter + (w / 128) * 64 + w % 64;
}

__global__ void sf_tile_kernel(const uint8_t *scales, size_t rows, size_t cols, uint8_t *tiled,
                               size_t total, size_t glu_inter) {
  size_t kb64_per_rb = (cols + 255) / 256 * 4;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    size_t chunk = i / kSfChunk, b = i % kSfChunk;
    size_t rb = chunk / kb64_per_rb, kb64 = chunk % kb64_per_rb;
    size_t r = (b / 16) + 32 * ((b % 16) / 4), s = b % 4;
    size_t row = rb * 128 + r, group = kb64 * 4 + s;
    uint8_t v = 0;
    if (row < rows && group < cols / 16) {
      const size_t src = glu_inter ? glu_source_row(row, glu_inter) : row;
      v = scales[src * (cols / 16) + group] & 0x7f;
    }
    tiled[i] = v;
  }
}

// Codes of groups whose e4m3 scale is negative get their sign bits flipped,
// so that (code, |scale|) decodes to the same value.
__global__ void sign_fold_kernel(const uint8_t *packed, const uint8_t *scales, size_t rows, size_t cols,
                                 uint8_t *out) {
  size_t n = rows * cols / 2;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    size_t row = (2 * i) / cols, col = (2 * i) % cols;
    uint8_t s = scales[row * (cols / 16) + col / 16];
    uint8_t p = packed[i];
    if (s & 0x80) p ^= 0x88;
    out[i] = p;
  }
}

__global__ void any_negative_kernel(const uint8_t *scales, size_t n, int *flag) {
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    if (scales[i] & 0x80) atomicOr(flag, 1);
}

// ---- activation quantize: amax, then codes + tiled factors --------------------------
// One thread per 16-column group: same arithmetic as fpb_nvfp4_quantize, the
// factor written to the tiled layout and the global to *global_out.
template <typename T>
__global__ void act_encode_kernel(const T *x, size_t rows, size_t cols, const uint32_t *amax_bits,
                                  uint8_t *packed, uint8_t *sf_tiled, float *global_out) {
  pdl_enter();
  const float global = __fdiv_rn(__uint_as_float(*amax_bits), 2688.0f);
  if (blockIdx.x == 0 && threadIdx.x == 0) *global_out = global;
  // One warp per row (grid-stride over rows); lane l takes groups l, l + 32, ...
  const int gpr = (int)(cols / kNvfp4Group), lane = threadIdx.x & 31;
  const size_t warps = (size_t)gridDim.x * (blockDim.x / 32);
  for (size_t r = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps) {
    const T *xrow = x + r * cols;
    uint8_t *prow = packed + r * (cols / 2);
    uint8_t *srow = sf_tiled + sf_tiled_row_offset(r, cols);
    for (int g = lane; g < gpr; g += 32) {
      float v[kNvfp4Group];
      const T *src = xrow + g * kNvfp4Group;
#pragma unroll
      for (int i = 0; i < kNvfp4Group; ++i) v[i] = act_load(src, i);
      encode_group16(v, global, prow + g * (kNvfp4Group / 2), srow + sf_tiled_group_offset(g));
    }
  }
}

// One matrix of a prepared tensor-core GEMV batch (device table, built at
// load time): weight rows [row_begin, row_begin + rows) of one handle times
// its own x [batch, K], into y [batch, rows].  The tensor map lives in
// global memory (64-byte aligned), which TMA reads like a parameter.
constexpr int kMaxPeerCopies = 8;
struct alignas(64) PlaneSeg {
  CUtensorMap tmap_b;       // the handle's codes (box 128 rows x 128 bytes)
  CUtensorMap tmap_y;       // W4A4 batch: y [m, rows] for TMA stores (valid when the batch stores that way)
  const uint8_t *b_sf;      // the handle's tiled factors
  const float *b_globals;   // the handle's row globals, row 0
  const void *x;
  void *y;
  int row_begin, rows;
  int item_begin;           // first item (128-row tile) of this segment
  int a_group;              // A row group of its x: the first segment with the same x (encoded once)
  // Planes batch with peer copies: y goes to these n_peer rows instead (e.g.
  // this rank's slice in every rank's gathered buffer: plain stores over
  // NVLink, the all-gather of an N-split GEMV done by the epilogue).
  int n_peer;
  void *y_peer[kMaxPeerCopies];
};

// ---- x as NVFP4 digit planes (tensor-core GEMV) ----------------------------------------
// Row t of x (K values) becomes kPlanes NVFP4 rows: plane 0 encodes x with
// the config-0 rule (global g0 = amax / 2688, e4m3 factors per 16 values,
// e2m1 codes), plane p encodes the residual x - (planes < p) with global
// g0 / 4^p.  An e2m1 code is off by at most one unit (its factor times its
// global), so a residual block never needs a factor above 4 / 6 of the
// previous one: no factor saturates, and 8 planes reproduce x to about
// 5e-9 of its norm.  With the globals fixed up front every 16-value group
// runs its 8 planes independently (one thread, in registers).  Token slot j
// of group g owns A rows g * 128 + j * kPlanes + p, their factors in the
// tiled layout and their globals in ga[row].  GLU: x rows are f32
// [gate (K) | up (K)] and the input is silu(gate) * up (swiglu.rs:16, in f32).
constexpr int kPlanes = 8, kPlaneThreads = 256, kPlaneMaxK = 4096;
template <typename T, bool GLU>
__device__ __forceinline__ float plane_in(const T *xr, int K, int i) {
  if (GLU) {
    const float *f = reinterpret_cast<const float *>(xr);
    return silu_mul(f[i], f[K + i]);
  }
  return act_load(xr, i);
}

template <typename T, bool GLU>
__global__ void __launch_bounds__(kPlaneThreads) planes_encode_kernel(const T *x, long long x_group_stride,
                                                                      int tokens, int K, const int32_t *live_groups,
                                                                      uint8_t *packed, uint8_t *sf_tiled,
                                                                      float *ga, const PlaneSeg *segs) {
  pdl_enter();
  __shared__ uint32_t red[32];
  const int g = blockIdx.x / tokens, t = blockIdx.x % tokens;
  if (live_groups && g >= *live_groups) return;  // a group nothing reads (uniform)
  if (segs && segs[g].a_group != g) return;      // its x is encoded by an earlier segment (uniform)
  const T *xg = segs ? static_cast<const T *>(segs[g].x) : x + (long long)g * x_group_stride;
  const T *xr = xg + (long long)t * K * (GLU ? 2 : 1);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int groups = K / kNvfp4Group;
  uint32_t m = 0;
  for (int i = tid; i < K; i += kPlaneThreads) m = max(m, __float_as_uint(plane_in<T, GLU>(xr, K, i)) & 0x7fffffffu);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = 0;
  for (int w = 0; w < kPlaneThreads / 32; ++w) m = max(m, red[w]);
  const float g0 = __fdiv_rn(__uint_as_float(m), 2688.0f);
  const size_t row0 = (size_t)g * 128 + (size_t)t * kPlanes;
  if (tid < kPlanes) ga[row0 + tid] = g0 * __uint_as_float((uint32_t)(127 - 2 * tid) << 23);  // g0 / 4^p
  for (int q = tid; q < groups; q += kPlaneThreads) {
    float r[kNvfp4Group];
#pragma unroll
    for (int i = 0; i < kNvfp4Group; ++i) r[i] = plane_in<T, GLU>(xr, K, q * kNvfp4Group + i);
    float gp = g0;
#pragma unroll 1
    for (int p = 0; p < kPlanes; ++p, gp *= 0.25f) {
      const size_t row = row0 + p;
      uint8_t *cdst = packed + row * (K / 2) + q * (kNvfp4Group / 2);
      uint8_t *sdst = sf_tiled + sf_tiled_row_offset(row, K) + sf_tiled_group_offset(q);
      float bmax = 0.0f;
#pragma unroll
      for (int i = 0; i < kNvfp4Group; ++i) bmax = fmaxf(bmax, fabsf(r[i]));
      const uint8_t sb = gp > 0.0f ? f32_to_e4m3(bmax * (1.0f / 6.0f) / gp) : (uint8_t)0;
      const float unit = e4m3_to_f32(sb) * gp;
      uint32_t lo = 0, hi = 0;
      if (unit > 0.0f) {
        const float inv = 1.0f / unit;
        float qv[kNvfp4Group];
#pragma unroll
        for (int i = 0; i < kNvfp4Group; ++i) qv[i] = r[i] * inv;
        lo = f32x8_to_e2m1x8(qv);
        hi = f32x8_to_e2m1x8(qv + 8);
#pragma unroll
        for (int i = 0; i < kNvfp4Group; ++i)
          r[i] -= e2m1_to_f32(((i < 8 ? lo : hi) >> (4 * (i & 7))) & 0xf) * unit;
      }
      *reinterpret_cast<uint2 *>(cdst) = make_uint2(lo, hi);
      *sdst = sb;
    }
  }
}

// ---- W4A4 batch: each member's x [m, K] quantized to NVFP4 (config 2's rule) -----------
// The prepared batch's W4A4 form (fpb_nvfp4_gemm_batch_create): every distinct
// x gets the per-tensor quantization of fpb_nvfp4_quantize_act (global = amax
// / 2688 over that x, e4m3 factors per 16 values, e2m1 codes), into A row
// group a_group (rows a_group * 128 + r), each row's global in ga[row].
// Pass 1: amax per group (blockIdx.y), atomicMax of each CTA's maximum
// (amax zeroed by the caller).
template <typename T>
__global__ void batch_amax_kernel(const PlaneSeg *segs, int m, int K, uint32_t *amax) {
  pdl_enter();
  const int g = blockIdx.y;
  if (segs[g].a_group != g) return;  // encoded with an earlier segment (uniform)
  const T *x = static_cast<const T *>(segs[g].x);
  const size_t n = (size_t)m * K;
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  constexpr size_t kVec = 16 / sizeof(T);
  uint32_t mx = 0;
  size_t head = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {  // 16-byte loads, four in flight
    const uint4 *xv = reinterpret_cast<const uint4 *>(x);
    const size_t nv = n / kVec;
#pragma unroll 4
    for (size_t i = tid; i < nv; i += stride) {
      const uint4 u = xv[i];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (sizeof(T) == 4)
          mx = max(mx, w[k] & 0x7fffffffu);
        else
          mx = max(mx, max((w[k] << 16) & 0x7fffffffu, w[k] & 0x7fff0000u));
      }
    }
    head = nv * kVec;
  }
  for (size_t i = head + tid; i < n; i += stride) mx = max(mx, __float_as_uint(act_load(x, i)) & 0x7fffffffu);
  block_amax_to(mx, &amax[g]);
}

// Pass 2: one warp per (row, 32 groups) of each group: lane l encodes group
// 32 c + l of the row (the encode of act_encode_kernel).
template <typename T>
__global__ void batch_encode_kernel(const PlaneSeg *segs, int m, int K, const uint32_t *amax, uint8_t *packed,
                                    uint8_t *sf_tiled, float *ga) {
  pdl_enter();
  const int g = blockIdx.y;
  if (segs[g].a_group != g) return;
  const float global = __fdiv_rn(__uint_as_float(amax[g]), 2688.0f);
  const T *x = static_cast<const T *>(segs[g].x);
  const int gpr = K / kNvfp4Group, lane = threadIdx.x & 31;
  const int chunks = (gpr + 31) / 32;
  const int warps = gridDim.x * (blockDim.x / 32);
  for (int w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; w < m * chunks; w += warps) {
    const int r = w / chunks, q = (w % chunks) * 32 + lane;
    const size_t row = (size_t)g * 128 + r;
    if (lane == 0 && w % chunks == 0) ga[row] = global;
    if (q >= gpr) continue;
    float v[kNvfp4Group];
    const T *src = x + (size_t)r * K + q * kNvfp4Group;
#pragma unroll
    for (int i = 0; i < kNvfp4Group; ++i) v[i] = act_load(src, i);
    encode_group16(v, global, packed + row * (K / 2) + q * (kNvfp4Group / 2),
                   sf_tiled + sf_tiled_row_offset(row, K) + sf_tiled_group_offset(q));
  }
}

}  // namespace fpb

namespace fpb {

struct GemmParams {
  const uint8_t *a_sf;     // activations' tiled scale factors
  const uint8_t *b_sf;     // weights' tiled scale factors (whole matrix)
  const float *a_global;   // device scalar
  const float *b_globals;  // per weight row, row 0 of the matrix
  void *y;
  long long ldy;  // elements between output rows
  int y_bf16;
  int M;         // activation rows
  int N;         // weight rows of the view
  int n_base;    // first weight row of the view (multiple of 128)
  int kb_count;  // ceil(K / 256)
  int *error;    // device error word
  // Grouped (MoE) mode, crates/firepit-kernels/src/gemm/nvfp4.rs:57-105: row
  // tile m of A belongs to expert tile_experts[m], whose weights are rows
  // [e * rows_per_expert, (e + 1) * rows_per_expert); N = rows_per_expert.
  const int32_t *tile_experts;  // null for a dense GEMM
  int n_experts;
  int tma_store;  // y through tmap_y (else direct per-row stores: unaligned y)
  // Fused SwiGLU (grouped mode only): N = 2 * inter rows per expert, gate rows
  // first; B tiles are gate rows [64b, 64b+64) + up rows [64b, 64b+64) (two
  // 64-row loads through tmap_b64, factors from the interleaved tiled copy)
  // and the epilogue writes h = silu(gate) * up [M, inter] through tmap_y,
  // with max |h| (as stored) into *amax_bits.
  int glu;
  uint32_t *amax_bits;
  // Grouped mode, nullable: the layout's token of each row (-1 = padding row).
  // Padding rows' outputs are not needed: a warp whose 32 rows are all padding
  // stores nothing, and padding rows are left out of the amax (so their
  // activations may hold anything, e.g. rows an encoder skipped).
  const int32_t *row_tokens;
  // bf16 mode (tcgen05 kind::f16, the reference's hi/lo activations): tiles
  // hold 64 bf16 per 128-byte row; each K block runs `passes` (A, B) pairs,
  // A from tmap_a (a_sel 0) or tmap_a2 (1), B from tmap_b (b_sel 0) or
  // tmap_b64 (1), all accumulated in the same TMEM accumulator; no scale
  // factors, ga = 1, and b_globals may be null (factor 1).
  int f16;
  int passes;
  int a_sel[3], b_sel[3];
  // Planes mode (the tensor-core GEMV): A row group g (128 rows) holds up to
  // 16 tokens' 8 digit planes each (row j * 8 + p), with per-row globals
  // a_globals[g * 128 + row]; the epilogue adds each token's 8 plane rows and
  // stores y[g * y_group_stride + j * ldy + n] for j < tokens.  Items are
  // (group, n tile): with moe_ids, group u < *moe_count uses expert
  // moe_ids[u]'s rows (N = rows per expert) and A group u * a_group_step
  // (0: one x for every expert); without, one group (a dense GEMV).
  int planes;
  int tokens;
  const float *a_globals;
  const int32_t *moe_ids;
  const int32_t *moe_count;
  int moe_cap;
  int a_group_step;
  long long y_group_stride;
  // Planes mode over a prepared batch: items are the segments' 128-row tiles
  // in order (segment s from segs[s].item_begin), A group s = segment s.
  const PlaneSeg *segs;
  int nseg;
  int total_items;
  int peer_stores;  // some segment stores to peer copies: a system-scope fence ends the epilogue
  // Rows of each A box tmap_a loads (planes: the tokens' 8 * tokens plane
  // rows; the tile's other rows keep whatever the stage held and only feed
  // accumulator rows nothing reads).  128 otherwise.
  int a_box_rows;
};

constexpr int kTileBytes = kBM * kBKBytes;   // 16 KB per operand per stage
constexpr int kSfStageBytes = 4 * kSfChunk;  // 2 KB per operand per stage
// TMEM: two 128-column accumulators (tiles alternate), then per stage 16
// columns of A factors (256..) and 16 of B factors (after the A ones).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemSfa = 256, kTmemSfb = 256 + 16 * kStages;
static_assert(kTmemSfb + 16 * kStages <= kTmemCols, "TMEM columns");
// Epilogue staging: one 32-row x 128-byte box per epilogue warp (bf16: its
// 64 columns; f32: 32 columns at a time), two per TMEM lane quadrant.
constexpr int kOutBoxBytes = 32 * 128;
constexpr int kOutWarpBytes = 2 * kOutBoxBytes;  // per TMEM lane quadrant
constexpr int kEpiWarps = 8;                      // two per quadrant
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr size_t kGemmSmem = 1024 + kStages * (2 * kTileBytes + 2 * kSfStageBytes) + 4 * kOutWarpBytes + 256;

__device__ __forceinline__ void report(int *error, volatile int *abort, int code) {
  *abort = 1;
  if (error) atomicCAS(error, 0, code);
}

// Tile t of the launch: m-major over (m_tiles, n_tiles); false when it is a
// grouped row tile past the layout's end (expert -1), which every role skips.
// A malformed expert id records device error 106 and is skipped too.
// Planes + MoE mode: the live count and the first kMoeIdsCached expert ids,
// read once per CTA after the dependency wait (a global load per tile and
// role put two dependent round trips in front of every tile's first copy).
constexpr int kMoeIdsCached = 1024;
struct MoeIdsCache {
  int count;
  int ids[kMoeIdsCached];
};

__device__ __forceinline__ bool gemm_tile(const GemmParams &p, int t, int n_tiles, int &m_tile, int &n_tile,
                                          int &n_base, const MoeIdsCache *moe = nullptr,
                                          const PlaneSeg **seg = nullptr) {
  if (p.segs) {
    // the segment whose items hold t (item starts cached in moe->ids)
    int lo = 0, hi = p.nseg - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (moe->ids[mid] <= t)
        lo = mid;
      else
        hi = mid - 1;
    }
    if (seg) *seg = p.segs + lo;
    m_tile = p.segs[lo].a_group;
    n_tile = t - moe->ids[lo];
    n_base = p.segs[lo].row_begin;
    return true;
  }
  m_tile = t / n_tiles;
  n_tile = t - m_tile * n_tiles;
  n_base = p.n_base;
  if (p.planes && p.moe_ids) {
    // m_tile is the group u: skipped past the live count; its expert's rows
    const int u = m_tile;
    if (u >= moe->count) return false;
    const int e = u < kMoeIdsCached ? moe->ids[u] : p.moe_ids[u];
    if (e < 0 || e >= p.n_experts) {
      if (threadIdx.x == 0 && p.error) atomicCAS(p.error, 0, 106);
      return false;
    }
    n_base = e * p.N;
    m_tile = u * p.a_group_step;  // the A row group this item reads
    return true;
  }
  if (p.tile_experts) {
    const int e = p.tile_experts[m_tile];
    if (e == -1) return false;
    if (e < 0 || e >= p.n_experts) {
      if (threadIdx.x == 0 && p.error) atomicCAS(p.error, 0, 106);
      return false;
    }
    n_base = e * p.N;
  }
  return true;
}

// Persistent: one CTA per SM walks the tiles t = blockIdx.x, + gridDim.x, ...
// The producer and the MMA issuer share one ring counter across tiles; the
// accumulator alternates between two TMEM buffers, so the epilogue of one
// tile overlaps the main loop of the next.
__global__ void __launch_bounds__(kGemmThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ CUtensorMap tmap_b64,
                      const __grid_constant__ CUtensorMap tmap_a2, GemmParams p) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = base;
  uint8_t *sB = sA + kStages * kTileBytes;
  uint8_t *sSFA = sB + kStages * kTileBytes;
  uint8_t *sSFB = sSFA + kStages * kSfStageBytes;
  uint8_t *sOut = sSFB + kStages * kSfStageBytes;  // 1024-byte aligned
  uint64_t *full = reinterpret_cast<uint64_t *>(sOut + 4 * kOutWarpBytes);
  uint64_t *empty = full + kStages;
  uint64_t *acc_full = empty + kStages;  // [2]
  uint64_t *acc_empty = acc_full + 2;    // [2]
  uint32_t *tmem_base_s = reinterpret_cast<uint32_t *>(acc_empty + 2);
  volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_base_s + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (p.N + kBN - 1) / kBN;
  const int m_tiles = p.planes ? (p.moe_ids ? p.moe_cap : 1) : (p.M + kBM - 1) / kBM;
  const int total = p.segs ? p.total_items : n_tiles * m_tiles;
  const int kb64_per_rb = p.kb_count * 4;
  // K blocks as the producer and the MMA issuer walk them (bf16 mode: each
  // block once per (A, B) pass).
  const int vblocks = p.f16 ? p.kb_count * p.passes : p.kb_count;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    *abort_s = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
    if (p.tma_store && !p.segs) prefetch_tensormap(&tmap_y);
    if (p.glu || p.f16) prefetch_tensormap(&tmap_b64);
    if (p.f16) prefetch_tensormap(&tmap_a2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  // Programmatic dependent launch: the set-up above overlaps the previous
  // kernel in the stream; nothing it wrote is read before this wait.
  pdl_enter();
  __shared__ MoeIdsCache moe_cache;
  if (p.planes && p.moe_ids) {
    const int live = min(max(*p.moe_count, 0), p.moe_cap);
    for (int i = threadIdx.x; i < min(live, kMoeIdsCached); i += blockDim.x) moe_cache.ids[i] = p.moe_ids[i];
    if (threadIdx.x == 0) moe_cache.count = live;
    __syncthreads();
  } else if (p.segs) {  // the segments' first items (nseg <= kMoeIdsCached, checked by the host)
    for (int i = threadIdx.x; i < p.nseg; i += blockDim.x) moe_cache.ids[i] = p.segs[i].item_begin;
    __syncthreads();
  }

  if (warp == 0) {
    // ---- TMA producer ----------------------------------------------------------
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int m_tile, n_tile, n_base;
        const PlaneSeg *sg = nullptr;
        if (!gemm_tile(p, t, n_tiles, m_tile, n_tile, n_base, &moe_cache, &sg)) continue;
        const int nb_global = n_base / 128 + n_tile;
        const CUtensorMap *tb = sg ? &sg->tmap_b : &tmap_b;
        const uint8_t *bsf = sg ? sg->b_sf : p.b_sf;
        for (int vb = 0; vb < vblocks; ++vb, ++it) {
          const int s = it % kStages;
          if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, abort_s)) {
            report(p.error, abort_s, 101);
            ok = false;
            break;
          }
          if (p.f16) {
            const int kb = vb / p.passes, j = vb - kb * p.passes;
            mbar_arrive_expect_tx(&full[s], 2 * kTileBytes);
            tma_load_2d(sA + s * kTileBytes, p.a_sel[j] ? &tmap_a2 : &tmap_a, kb * kBKBytes, m_tile * kBM,
                        &full[s]);
            tma_load_2d(sB + s * kTileBytes, p.b_sel[j] ? &tmap_b64 : &tmap_b, kb * kBKBytes,
                        n_base + n_tile * kBN, &full[s]);
            continue;
          }
          const int kb = vb;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(p.a_box_rows * kBKBytes + kTileBytes + 2 * kSfStageBytes));
          tma_load_2d(sA + s * kTileBytes, &tmap_a, kb * kBKBytes, m_tile * kBM, &full[s]);
          if (p.glu) {
            const int row_gate = n_base + n_tile * 64;
            tma_load_2d(sB + s * kTileBytes, &tmap_b64, kb * kBKBytes, row_gate, &full[s]);
            tma_load_2d(sB + s * kTileBytes + kTileBytes / 2, &tmap_b64, kb * kBKBytes, row_gate + p.N / 2,
                        &full[s]);
          } else {
            tma_load_2d(sB + s * kTileBytes, tb, kb * kBKBytes, n_base + n_tile * kBN, &full[s]);
          }
          bulk_load(sSFA + s * kSfStageBytes, p.a_sf + ((size_t)m_tile * kb64_per_rb + kb * 4) * kSfChunk,
                    kSfStageBytes, &full[s]);
          bulk_load(sSFB + s * kSfStageBytes, bsf + ((size_t)nb_global * kb64_per_rb + kb * 4) * kSfChunk,
                    kSfStageBytes, &full[s]);
        }
      }
      // Our own copies must have landed before the CTA may exit.
      const uint32_t issued = it;
      for (uint32_t j = (issued > kStages ? issued - kStages : 0); j < issued; ++j)
        if (!mbar_wait(&full[j % kStages], (j / kStages) & 1, abort_s)) report(p.error, abort_s, 102);
    }
  } else if (warp == 1) {
    // ---- MMA issuer -------------------------------------------------------------
    if (elect_one()) {
      const uint32_t idesc = p.f16 ? idesc_bf16(kBM, kBN) : idesc_nvf4(kBM, kBN);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int m_tile, n_tile, n_base;
        if (!gemm_tile(p, t, n_tiles, m_tile, n_tile, n_base, &moe_cache)) continue;
        const uint32_t buf = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) - 1) & 1, abort_s)) {
          report(p.error, abort_s, 107);
          break;
        }
        tc_fence_after();
        const uint32_t tmem_acc = tmem + buf * kBN;
        for (int vb = 0; vb < vblocks; ++vb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, abort_s)) {
            report(p.error, abort_s, 103);
            ok = false;
            break;
          }
          tc_fence_after();
          if (p.f16) {
            // four K = 16 steps of bf16 over the stage's 64 columns
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t a_desc = smem_desc(smem_u32(sA + s * kTileBytes) + kk * 32, 16, 1024, 2);
              const uint64_t b_desc = smem_desc(smem_u32(sB + s * kTileBytes) + kk * 32, 16, 1024, 2);
              mma_bf16(tmem_acc, a_desc, b_desc, idesc, (vb | kk) != 0);
            }
            tc_commit(&empty[s]);
            continue;
          }
          const int kb = vb;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            tmem_cp_sf(tmem + kTmemSfa + s * 16 + kk * 4,
                       smem_desc(smem_u32(sSFA + s * kSfStageBytes + kk * kSfChunk), 0, 128, 0));
            tmem_cp_sf(tmem + kTmemSfb + s * 16 + kk * 4,
                       smem_desc(smem_u32(sSFB + s * kSfStageBytes + kk * kSfChunk), 0, 128, 0));
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a_desc = smem_desc(smem_u32(sA + s * kTileBytes) + kk * 32, 16, 1024, 2);
            const uint64_t b_desc = smem_desc(smem_u32(sB + s * kTileBytes) + kk * 32, 16, 1024, 2);
            mma_nvf4(tmem_acc, a_desc, b_desc, idesc, tmem + kTmemSfa + s * 16 + kk * 4,
                     tmem + kTmemSfb + s * 16 + kk * 4, (kb | kk) != 0);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
        ++lt;
      }
    }
  } else {
    // ---- epilogue: warps 2..9, two per TMEM lane quadrant (warp % 4) ---------
    // Warp (quadrant qw, half ch) owns rows qw*32 .. +31 of the tile and
    // accumulator columns ch*64 .. +63 (glu: gate and up columns of h
    // columns ch*32 .. +31); each warp stages and stores its own boxes.
    const int qw = warp & 3, ch = (warp - 2) >> 2;
    const uint32_t lane_base = (uint32_t)(qw * 32) << 16;
    // W4A4 batch (segments without planes): each row's global from a_globals
    const float ga = (p.f16 || p.planes || p.segs) ? 1.0f : __ldg(p.a_global);
    uint8_t *stage = sOut + qw * kOutWarpBytes;
    uint8_t *row_s = stage + lane * 128;
    uint32_t lt = 0;
    uint32_t glu_max = 0;  // glu: this lane's max |h| bits over its live rows and tiles
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int m_tile, n_tile, n_base;
      const PlaneSeg *sg = nullptr;
      if (!gemm_tile(p, t, n_tiles, m_tile, n_tile, n_base, &moe_cache, &sg)) continue;
      const uint32_t buf = lt & 1;
      const int n_lim = sg ? sg->rows : p.N;                        // rows of this item's view
      const float *bglob = sg ? sg->b_globals : p.b_globals;
      // What the tile's epilogue reads from memory besides the accumulator
      // (the rows' tokens, the weight rows' globals) is loaded before the
      // wait, so its latency hides behind the main loop.
      const int row0 = m_tile * kBM + qw * 32;
      const int n0 = n_tile * kBN;
      const bool row_live = p.planes ? qw * 32 + lane < p.tokens * 8
                            : p.segs ? qw * 32 + lane < p.tokens
                                     : row0 + lane < p.M && (!p.row_tokens || p.row_tokens[row0 + lane] >= 0);
      const float ga_row = (p.planes || p.segs) && row_live ? __ldg(p.a_globals + row0 + lane) : 0.0f;
      float gl[2];
      if (p.glu) {
        const int j0 = n_tile * 64;
        gl[0] = __ldg(p.b_globals + n_base + j0 + ch * 32 + lane);                // gate rows
        gl[1] = __ldg(p.b_globals + n_base + p.N / 2 + j0 + ch * 32 + lane);  // up rows
      } else {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int n = n0 + ch * 64 + c * 32 + lane;
          gl[c] = n < n_lim ? (bglob ? __ldg(bglob + n_base + n) : 1.0f) : 0.0f;
        }
      }
      if (!mbar_wait(&acc_full[buf], (lt >> 1) & 1, abort_s)) {
        report(p.error, abort_s, 105);
        break;
      }
      __syncwarp();  // the TMEM loads below are warp-collective
      tc_fence_after();
      // Drain this warp's 64 accumulator columns (glu: 32 gate + the 32 up
      // columns of the same h columns), then free the buffer.
      uint32_t r[2][32];
      const uint32_t tacc = tmem + lane_base + buf * kBN;
      if (p.glu) {
        tmem_ld32(tacc + ch * 32, r[0]);
        tmem_ld32(tacc + 64 + ch * 32, r[1]);
      } else {
        tmem_ld32(tacc + ch * 64, r[0]);
        tmem_ld32(tacc + ch * 64 + 32, r[1]);
      }
      tmem_ld_wait(r[0]);
      tmem_ld_wait(r[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      ++lt;
      if (p.planes) {
        // Each token's 8 plane rows are 8 consecutive lanes.  Each value is
        // scaled by its row's plane global, then the 8 lanes reduce-scatter
        // (recursive halving over xor 4, 2, 1: 28 shuffles for 32 columns) so
        // that lane p of the token holds the sums of columns p, p + 8,
        // p + 16, p + 24, which it scales by their weight globals and stores.
        if (qw * 32 >= p.tokens * 8) continue;  // no token in this quadrant (uniform)
        const int token = (qw * 32 + lane) >> 3, pl = lane & 7;
        const bool b2 = pl & 4, b1 = pl & 2, b0 = pl & 1;
        const int item_group = t / n_tiles;  // the item's group: y block
        const int nw = n0 + ch * 64;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[c][j]) * ga_row;
          // column j = 8 i + q; step 1 keeps q with bit 2 == b2
          float w1[4][4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int ql = 0; ql < 4; ++ql) {
              const float lo = v[8 * i + ql], hi = v[8 * i + 4 + ql];
              w1[i][ql] = (b2 ? hi : lo) + __shfl_xor_sync(0xffffffffu, b2 ? lo : hi, 4);
            }
          float w2[4][2];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int q0 = 0; q0 < 2; ++q0) {
              const float lo = w1[i][q0], hi = w1[i][2 + q0];
              w2[i][q0] = (b1 ? hi : lo) + __shfl_xor_sync(0xffffffffu, b1 ? lo : hi, 2);
            }
          float keep[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float lo = w2[i][0], hi = w2[i][1];
            keep[i] = ((b0 ? hi : lo) + __shfl_xor_sync(0xffffffffu, b0 ? lo : hi, 1)) *
                      __shfl_sync(0xffffffffu, gl[c], 8 * i + pl);
          }
          if (token < p.tokens) {
            void *ydst = sg ? sg->y : p.y;
            const long long ybase = sg ? (long long)token * sg->rows
                                       : (long long)item_group * p.y_group_stride + (long long)token * p.ldy;
            // peer copies: the count read once per tile, the addresses through
            // the read-only path (the stores cannot alias the segment table)
            const int n_peer = sg ? __ldg(&sg->n_peer) : 0;
            if (n_peer == 0) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int n = nw + c * 32 + i * 8 + pl;
                if (n < n_lim) {
                  if (p.y_bf16)
                    reinterpret_cast<__nv_bfloat16 *>(ydst)[ybase + n] = __float2bfloat16_rn(keep[i]);
                  else
                    reinterpret_cast<float *>(ydst)[ybase + n] = keep[i];
                }
              }
            } else {
              for (int k = 0; k < n_peer; ++k) {
                void *dst = reinterpret_cast<void *>(
                    __ldg(reinterpret_cast<const unsigned long long *>(&sg->y_peer[k])));
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const int n = nw + c * 32 + i * 8 + pl;
                  if (n < n_lim) {
                    if (p.y_bf16)
                      reinterpret_cast<__nv_bfloat16 *>(dst)[ybase + n] = __float2bfloat16_rn(keep[i]);
                    else
                      reinterpret_cast<float *>(dst)[ybase + n] = keep[i];
                  }
                }
              }
            }
          }
        }
        continue;
      }
      if (row0 >= p.M) continue;  // the warp's rows are all past the end
      if (!__any_sync(0xffffffffu, row_live)) continue;  // nothing of these 32 rows is needed (both warps agree)
      if (p.glu) {
        // h columns j0 + ch*32 + i: silu(gate) * up, gate / up scaled by ga
        // and their weight rows' globals.  exp2 and reciprocal approximations
        // (no branches, so the 32 evaluations interleave): relative error
        // about 1e-6 against the exact formula, far below the NVFP4 encode
        // that follows.
        const int j0 = n_tile * 64;
        const float g_gate = gl[0], g_up = gl[1];
        float v[32];
        uint32_t mx = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float gate = (__uint_as_float(r[0][j]) * ga) * __shfl_sync(0xffffffffu, g_gate, j);
          const float up = (__uint_as_float(r[1][j]) * ga) * __shfl_sync(0xffffffffu, g_up, j);
          v[j] = __fdividef(gate, 1.0f + __expf(-gate)) * up;
        }
        if (lane == 0) bulk_wait_read_all();  // this warp's previous store has left its box
        __syncwarp();
        if (p.y_bf16) {
          // the warp's own box: 32 rows x 64 bytes, unswizzled (tmap_y's box
          // is 32 x 32 bf16 in this mode)
          uint8_t *row64 = stage + ch * kOutBoxBytes + lane * 64;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 pk;
            pk.x = pack_bf16x2(v[8 * q], v[8 * q + 1]);
            pk.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
            pk.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
            pk.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
            const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) mx = max(mx, max((w4[i] << 16) & 0x7fffffffu, w4[i] & 0x7fff0000u));
            *reinterpret_cast<uint4 *>(row64 + q * 16) = pk;
          }
        } else {
          // f32: the warp's 32 columns are one 128-byte-swizzled box
#pragma unroll
          for (int j = 0; j < 32; ++j) mx = max(mx, __float_as_uint(v[j]) & 0x7fffffffu);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4 *>(row_s + ch * kOutBoxBytes + ((q ^ (lane & 7)) * 16)) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_y, stage + ch * kOutBoxBytes, j0 + ch * 32, row0);
          bulk_commit_group();
        }
        if (row_live) glu_max = max(glu_max, mx);
        continue;
      }
      // Lane l holds the weight global of column n0 + ch*64 + 32c + l; the
      // products are scaled in place by every lane (shuffles are warp-wide).
      const int nw = n0 + ch * 64;
      const float gax = p.segs ? ga_row : ga;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int j = 0; j < 32; ++j)
          r[c][j] = __float_as_uint((__uint_as_float(r[c][j]) * gax) * __shfl_sync(0xffffffffu, gl[c], j));
      if (p.tma_store) {
        // a W4A4 batch member's own map: its y [m, rows], rows local to the member
        const CUtensorMap *ymap = sg ? &sg->tmap_y : &tmap_y;
        const int yrow = sg ? qw * 32 : row0;
        if (lane == 0) bulk_wait_read_all();  // this warp's previous stores have left its box
        __syncwarp();
        if (p.y_bf16) {
          // box ch: this warp's 64 columns
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(r[c][8 * q]), __uint_as_float(r[c][8 * q + 1]));
              pk.y = pack_bf16x2(__uint_as_float(r[c][8 * q + 2]), __uint_as_float(r[c][8 * q + 3]));
              pk.z = pack_bf16x2(__uint_as_float(r[c][8 * q + 4]), __uint_as_float(r[c][8 * q + 5]));
              pk.w = pack_bf16x2(__uint_as_float(r[c][8 * q + 6]), __uint_as_float(r[c][8 * q + 7]));
              *reinterpret_cast<uint4 *>(row_s + ch * kOutBoxBytes + (((c * 4 + q) ^ (lane & 7)) * 16)) = pk;
            }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (nw < n_lim) tma_store_2d(ymap, stage + ch * kOutBoxBytes, nw, yrow);
            bulk_commit_group();
          }
        } else {
          // f32: the warp's box takes 32 columns at a time
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if (c) {
              if (lane == 0) bulk_wait_read_all();
              __syncwarp();
            }
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<uint4 *>(row_s + ch * kOutBoxBytes + ((q ^ (lane & 7)) * 16)) =
                  make_uint4(r[c][4 * q], r[c][4 * q + 1], r[c][4 * q + 2], r[c][4 * q + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (nw + c * 32 < n_lim) tma_store_2d(ymap, stage + ch * kOutBoxBytes, nw + c * 32, yrow);
              bulk_commit_group();
            }
          }
        }
        continue;
      }
      // Direct stores (y not addressable by a tensor map; a W4A4 batch
      // member's y [m, rows]).
      const int row = sg ? qw * 32 + lane : row0 + lane;
      if (!row_live) continue;  // no warp-collective operation follows in this iteration
      void *ydst = sg ? sg->y : p.y;
      const long long ldy = sg ? (long long)sg->rows : p.ldy;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int nc = nw + c * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[c][j]);
        const long long off = (long long)row * ldy + nc;
        const bool full_cols = nc + 32 <= n_lim;
        if (p.y_bf16) {
          __nv_bfloat16 *yp = reinterpret_cast<__nv_bfloat16 *>(ydst) + off;
          if (full_cols && (reinterpret_cast<uintptr_t>(yp) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 pk;
              pk.x = pack_bf16x2(v[j], v[j + 1]);
              pk.y = pack_bf16x2(v[j + 2], v[j + 3]);
              pk.z = pack_bf16x2(v[j + 4], v[j + 5]);
              pk.w = pack_bf16x2(v[j + 6], v[j + 7]);
              *reinterpret_cast<uint4 *>(yp + j) = pk;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nc + j < n_lim) yp[j] = __float2bfloat16_rn(v[j]);
          }
        } else {
          float *yp = reinterpret_cast<float *>(ydst) + off;
          if (full_cols && (reinterpret_cast<uintptr_t>(yp) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4 *>(yp + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nc + j < n_lim) yp[j] = v[j];
          }
        }
      }
    }
    if (p.glu) {  // one atomicMax per warp and launch (per tile made same-address atomics pile up in L2)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) glu_max = max(glu_max, __shfl_xor_sync(0xffffffffu, glu_max, o));
      if (lane == 0 && glu_max) atomicMax(p.amax_bits, glu_max);
    }
    // Stores in flight read this CTA's shared memory: complete them before exit.
    if (lane == 0 && p.tma_store) bulk_wait_all();
    if (p.peer_stores) __threadfence_system();  // peer copies land before the caller's barrier
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace fpb

// ---- host side -------------------------------------------------------------------------
namespace fpb {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
static EncodeTiledFn encode_fn() {
  static std::mutex mu;
  static EncodeTiledFn fn = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    cudaDriverEntryPointQueryResult q{};
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D byte tensor [rows, row_bytes] read in boxes of 128 bytes x box_rows with
// 128-byte swizzle; out-of-range elements read as zero.
int encode_rows_u8(CUtensorMap *map, const void *base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FPB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15))
    return fail(FPB_ERR_INVALID_ARGUMENT, "TMA operand must be 16-byte aligned with 16-byte row pitch");
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FPB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FPB_OK;
}

bool encode_store_map(CUtensorMap *map, void *y, bool bf16, uint64_t rows, uint64_t cols, uint64_t ld,
                      uint32_t box_rows, uint32_t box_cols) {
  EncodeTiledFn fn = encode_fn();
  const uint64_t esize = bf16 ? 2 : 4;
  if (!fn || (reinterpret_cast<uintptr_t>(y) & 15) || ((ld * esize) & 15) || ld < cols || rows == 0 || cols == 0)
    return false;
  if (box_cols == 0) box_cols = (uint32_t)(128 / esize);
  // 128-byte boxes are stored from 128-byte-swizzled staging; narrower boxes unswizzled
  const bool swz = box_cols * esize == 128;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, y, dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static unsigned grid_for(size_t n) {
  size_t g = (n + 255) / 256, cap = (size_t)sm_count() * 16;
  return (unsigned)std::max<size_t>(1, std::min(g, cap));
}

// Raises the GEMM kernel's dynamic shared-memory limit once per device (at
// matrix creation, so that no GEMM call makes the runtime call during a
// stream capture).
static int ensure_gemm_attr() {
  static std::mutex mu;
  static std::vector<int> attr_devs;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (std::find(attr_devs.begin(), attr_devs.end(), dev) == attr_devs.end()) {
    FPB_CUDA_TRY(cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem));
    attr_devs.push_back(dev);
  }
  return FPB_OK;
}

// A handle from fpb_nvfp4_matrix_create(_device) always has its GEMM-side
// copies; this guards against handles built some other way.
static int require_prepared(const fpb_nvfp4_matrix *m, const char *fn) {
  if (!m->extras || !m->extras->tmap_valid)
    return fail(FPB_ERR_INVALID_ARGUMENT, "%s: matrix has no GEMM-side copies (fpb_nvfp4_matrix_prepare_gemm)", fn);
  return FPB_OK;
}

// Builds the GEMM-side copies of a weight matrix once: tiled UE4M3 factors,
// sign-folded codes when any factor is negative, and the codes' TMA map.
int prepare_gemm_weights(fpb_nvfp4_matrix *m, cudaStream_t s) {
  if (int st = ensure_gemm_attr()) return st;
  if (m->extras && m->extras->tmap_valid) return FPB_OK;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (m->extras && m->extras->tmap_valid) return FPB_OK;
  if (!m->extras) m->extras = new MatrixExtras();
  MatrixExtras *x = m->extras;
  const size_t bytes = sf_tiled_bytes(m->rows, m->cols);
  if (!x->sf_tiled) {
    FPB_CUDA_TRY(cudaMalloc(&x->sf_tiled, bytes));
    x->sf_tiled_bytes = bytes;
  }
  sf_tile_kernel<<<grid_for(bytes), 256, 0, s>>>(m->scales, m->rows, m->cols, x->sf_tiled, bytes, 0);
  FPB_LAUNCH_CHECK("sf_tile_kernel");
  int *flag = nullptr;
  int neg = 0;
  FPB_CUDA_TRY(cudaMalloc(&flag, sizeof(int)));
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), s);
  if (e == cudaSuccess) {
    any_negative_kernel<<<grid_for(m->rows * m->cols / 16), 256, 0, s>>>(m->scales, m->rows * m->cols / 16, flag);
    e = cudaGetLastError();
    count_launch();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(&neg, flag, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(flag);
  if (e != cudaSuccess) return cuda_fail(e, "prepare_gemm_weights");
  const uint8_t *codes = m->packed;
  if (neg) {
    if (!x->packed_folded) FPB_CUDA_TRY(cudaMalloc(&x->packed_folded, m->rows * m->cols / 2));
    sign_fold_kernel<<<grid_for(m->rows * m->cols / 2), 256, 0, s>>>(m->packed, m->scales, m->rows, m->cols,
                                                                      x->packed_folded);
    FPB_LAUNCH_CHECK("sign_fold_kernel");
    codes = x->packed_folded;
  }
  int st = encode_rows_u8(reinterpret_cast<CUtensorMap *>(x->tmap_b), codes, m->rows, m->cols / 2, kBN);
  if (st) return st;
  FPB_CUDA_TRY(cudaStreamSynchronize(s));
  x->tmap_valid = true;
  return FPB_OK;
}

template <typename T>
static int quantize_act_impl(const T *x, size_t rows, size_t cols, uint8_t *packed, uint8_t *sf_tiled,
                             float *global_out, float *amax_scratch, cudaStream_t s) {
  FPB_CUDA_TRY(cudaMemsetAsync(amax_scratch, 0, sizeof(uint32_t), s));
  FPB_CUDA_TRY(cudaMemsetAsync(sf_tiled, 0, sf_tiled_bytes(rows, cols), s));
  uint32_t *amax = reinterpret_cast<uint32_t *>(amax_scratch);
  launch_pdl(act_amax_kernel<T>, grid_for(rows * cols), 256, 0, s, x, rows * cols, amax);
  FPB_LAUNCH_CHECK("act_amax_kernel");
  launch_pdl(act_encode_kernel<T>, grid_for(rows * 32), 256, 0, s, x, rows, cols, amax, packed, sf_tiled,
             global_out);
  FPB_LAUNCH_CHECK("act_encode_kernel");
  return FPB_OK;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_nvfp4_act_sf_bytes(size_t m, size_t k) { return sf_tiled_bytes(m, k); }

extern "C" size_t fpb_nvfp4_gemv_planes_workspace_bytes(size_t groups, size_t k);

extern "C" size_t fpb_nvfp4_gemm_workspace_bytes(size_t m, size_t k) {
  const size_t quantized = align256(m * k / 2) + align256(sf_tiled_bytes(m, k)) + 256;
  // m <= 16 runs as the tensor-core GEMV (x as digit planes): its workspace
  return m <= 16 ? std::max(quantized, fpb_nvfp4_gemv_planes_workspace_bytes(1, k)) : quantized;
}

extern "C" int fpb_nvfp4_quantize_act(const void *x, int x_dtype, size_t m, size_t k, uint8_t *packed,
                                      uint8_t *sf_tiled, float *global_out, float *amax_scratch, void *stream) {
  if (!x || !packed || !sf_tiled || !global_out || !amax_scratch)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_quantize_act: null pointer");
  if (m == 0 || k == 0 || k % kQ8Block) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_quantize_act: bad shape");
  cudaStream_t s = as_stream(stream);
  if (x_dtype == FPB_F32)
    return quantize_act_impl(static_cast<const float *>(x), m, k, packed, sf_tiled, global_out, amax_scratch, s);
  if (x_dtype == FPB_BF16)
    return quantize_act_impl(static_cast<const uint16_t *>(x), m, k, packed, sf_tiled, global_out, amax_scratch,
                             s);
  return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_quantize_act: dtype %d", x_dtype);
}

static int prepare_glu_weights(fpb_nvfp4_matrix *m, size_t inter, cudaStream_t s);

extern "C" int fpb_nvfp4_matrix_prepare_gemm(fpb_nvfp4_matrix *w, void *stream) {
  if (!w) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_matrix_prepare_gemm: null handle");
  return prepare_gemm_weights(w, as_stream(stream));
}

extern "C" int fpb_nvfp4_matrix_prepare_glu(fpb_nvfp4_matrix *w, size_t inter, void *stream) {
  if (!w) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_matrix_prepare_glu: null handle");
  if (inter == 0 || inter % 64 || w->rows % (2 * inter))
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_matrix_prepare_glu: inter %zu must be a multiple of 64 with 2*inter "
                "dividing %zu", inter, w->rows);
  return prepare_glu_weights(w, inter, as_stream(stream));
}

extern "C" int fpb_nvfp4_gemm_q(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const uint8_t *a_packed,
                                const uint8_t *a_sf_tiled, const float *a_global, size_t m, void *y, int y_dtype,
                                void *stream) {
  if (!w || !a_packed || !a_sf_tiled || !a_global || !y)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemm_q: null pointer");
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemm_q: row range [%zu, %zu) outside %zu rows", row_begin, row_end,
                w->rows);
  if (row_begin % 128)
    return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemm_q: row_begin %zu is not a multiple of 128", row_begin);
  if (m == 0 || m > (size_t)65535 * kBM) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemm_q: m = %zu", m);
  if (y_dtype != FPB_F32 && y_dtype != FPB_BF16) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemm_q: dtype");
  cudaStream_t s = as_stream(stream);
  int st = require_prepared(w, "fpb_nvfp4_gemm_q");
  if (st) return st;
  CUtensorMap tmap_a;
  if ((st = encode_rows_u8(&tmap_a, a_packed, m, w->cols / 2, kBM))) return st;
  {
    static std::mutex mu;
    static std::vector<int> attr_devs;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (std::find(attr_devs.begin(), attr_devs.end(), dev) == attr_devs.end()) {
      FPB_CUDA_TRY(
          cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem));
      attr_devs.push_back(dev);
    }
  }
  int *err = nullptr;
  FPB_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_device_error));
  GemmParams p{};
  p.a_box_rows = kBM;
  p.a_sf = a_sf_tiled;
  p.b_sf = w->extras->sf_tiled;
  p.a_global = a_global;
  p.b_globals = w->row_globals;
  p.y = y;
  p.N = (int)(row_end - row_begin);
  p.ldy = p.N;
  p.y_bf16 = y_dtype == FPB_BF16;
  p.M = (int)m;
  p.n_base = (int)row_begin;
  p.kb_count = (int)((w->cols + 255) / 256);
  p.error = err;
  CUtensorMap tmap_y{};
  p.tma_store = encode_store_map(&tmap_y, y, p.y_bf16, m, p.N, p.ldy, 32, 0);
  const size_t tiles = (size_t)((p.N + kBN - 1) / kBN) * ((m + kBM - 1) / kBM);
  const unsigned grid = (unsigned)std::min<size_t>(tiles, (size_t)std::max(1, sm_count()));
  launch_pdl(nvfp4_gemm_kernel, grid, kGemmThreads, kGemmSmem, s, tmap_a, *reinterpret_cast<const CUtensorMap *>(w->extras->tmap_b),
                                                 tmap_y, *reinterpret_cast<const CUtensorMap *>(w->extras->tmap_b), tmap_a, p);
  FPB_LAUNCH_CHECK("nvfp4_gemm_kernel");
  return FPB_OK;
}

namespace fpb {
static int run_planes(const char *fn, fpb_nvfp4_matrix *w, size_t n_base, size_t n_rows, const void *x, int x_dtype,
                      bool glu, size_t x_group_stride, int tokens, size_t groups, const int32_t *moe_ids,
                      const int32_t *moe_count, int moe_cap, int n_experts, void *y, int y_dtype,
                      long long y_group_stride, long long ldy, void *workspace, size_t workspace_bytes,
                      cudaStream_t s);
}  // namespace fpb

extern "C" int fpb_nvfp4_gemm(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                              size_t m, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                              void *stream) {
  if (!w || !x || !y || !workspace) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemm: null pointer");
  if (workspace_bytes < fpb_nvfp4_gemm_workspace_bytes(m, w->cols))
    return fail(FPB_ERR_WORKSPACE, "fpb_nvfp4_gemm: workspace %zu < %zu bytes", workspace_bytes,
                fpb_nvfp4_gemm_workspace_bytes(m, w->cols));
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemm: workspace must be 256-byte aligned");
  if (row_end == 0) row_end = w->rows;
  // Decode-size M (BASELINE config 2 keeps activations in bf16 below 128
  // rows; the reference keeps them in f32): the tensor-core GEMV, x as 8
  // NVFP4 digit planes, no activation quantization.
  if (m <= 16 && w->cols % 256 == 0 && w->cols <= (size_t)kPlaneMaxK && row_begin % kBN == 0 &&
      row_begin < row_end && row_end <= w->rows)
    return run_planes("fpb_nvfp4_gemm", w, row_begin, row_end - row_begin, x, x_dtype, false, 0, (int)m, 1, nullptr,
                      nullptr, 0, 0, y, y_dtype, 0, (long long)(row_end - row_begin), workspace, workspace_bytes,
                      as_stream(stream));
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  uint8_t *packed = ws;
  uint8_t *sf = packed + align256(m * w->cols / 2);
  float *scalars = reinterpret_cast<float *>(sf + align256(sf_tiled_bytes(m, w->cols)));
  int st = fpb_nvfp4_quantize_act(x, x_dtype, m, w->cols, packed, sf, scalars, scalars + 1, stream);
  if (st) return st;
  return fpb_nvfp4_gemm_q(w, row_begin, row_end, packed, sf, scalars, m, y, y_dtype, stream);
}

// ---- tensor-core GEMV: x as digit planes (fpb_nvfp4_gemv_planes, fpb_nvfp4_moe_gemv_planes)
extern "C" size_t fpb_nvfp4_gemv_planes_workspace_bytes(size_t groups, size_t k) {
  const size_t rows = groups * kBM;
  return align256(rows * k / 2) + align256(sf_tiled_bytes(rows, k)) + align256(rows * sizeof(float)) + 256;
}

namespace fpb {
// Encodes x's planes into the workspace and runs the GEMM kernel in planes
// mode.  groups: A row groups (1, or cap with per-expert x); moe: device ids.
static int run_planes(const char *fn, fpb_nvfp4_matrix *w, size_t n_base, size_t n_rows, const void *x, int x_dtype,
                      bool glu, size_t x_group_stride, int tokens, size_t groups, const int32_t *moe_ids,
                      const int32_t *moe_count, int moe_cap, int n_experts, void *y, int y_dtype,
                      long long y_group_stride, long long ldy, void *workspace, size_t workspace_bytes,
                      cudaStream_t s) {
  const size_t K = w->cols;
  if (tokens < 1 || tokens > 16) return fail(FPB_ERR_SHAPE, "%s: tokens %d not in [1, 16]", fn, tokens);
  if (K % 256 || K > (size_t)kPlaneMaxK)
    return fail(FPB_ERR_UNSUPPORTED, "%s: cols %zu must be a multiple of 256 and at most %d", fn, K, kPlaneMaxK);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "%s: dtype", fn);
  if (workspace_bytes < fpb_nvfp4_gemv_planes_workspace_bytes(groups, K))
    return fail(FPB_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", fn, workspace_bytes,
                fpb_nvfp4_gemv_planes_workspace_bytes(groups, K));
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(FPB_ERR_INVALID_ARGUMENT, "%s: workspace must be 256-byte aligned", fn);
  if (int st = require_prepared(w, fn)) return st;
  if (int st = ensure_gemm_attr()) return st;
  const size_t rows = groups * kBM;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  uint8_t *packed = ws;
  uint8_t *sf = packed + align256(rows * K / 2);
  float *ga = reinterpret_cast<float *>(sf + align256(sf_tiled_bytes(rows, K)));
  const unsigned enc_grid = (unsigned)(groups * tokens);
  const int32_t *live = moe_ids ? moe_count : nullptr;
  cudaError_t e =
      glu ? launch_pdl(planes_encode_kernel<float, true>, enc_grid, kPlaneThreads, 0, s, static_cast<const float *>(x),
                       (long long)x_group_stride, tokens, (int)K, live, packed, sf, ga, nullptr)
      : x_dtype == FPB_F32
          ? launch_pdl(planes_encode_kernel<float, false>, enc_grid, kPlaneThreads, 0, s,
                       static_cast<const float *>(x), (long long)x_group_stride, tokens, (int)K, live, packed, sf, ga, nullptr)
          : launch_pdl(planes_encode_kernel<uint16_t, false>, enc_grid, kPlaneThreads, 0, s,
                       static_cast<const uint16_t *>(x), (long long)x_group_stride, tokens, (int)K, live, packed, sf,
                       ga, nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "planes_encode_kernel");
  FPB_LAUNCH_CHECK("planes_encode_kernel");
  CUtensorMap tmap_a;
  if (int st = encode_rows_u8(&tmap_a, packed, rows, K / 2, (uint32_t)(tokens * kPlanes))) return st;
  int *err = nullptr;
  FPB_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_device_error));
  GemmParams p{};
  p.a_box_rows = kBM;
  p.a_sf = sf;
  p.b_sf = w->extras->sf_tiled;
  p.b_globals = w->row_globals;
  p.y = y;
  p.N = (int)n_rows;
  p.ldy = ldy;
  p.y_bf16 = y_dtype == FPB_BF16;
  p.M = (int)rows;
  p.n_base = (int)n_base;
  p.kb_count = (int)(K / 256);
  p.error = err;
  p.planes = 1;
  p.tokens = tokens;
  p.a_box_rows = tokens * kPlanes;
  p.a_globals = ga;
  p.moe_ids = moe_ids;
  p.moe_count = moe_count;
  p.moe_cap = moe_cap;
  p.n_experts = n_experts;
  p.a_group_step = groups > 1 ? 1 : 0;
  p.y_group_stride = y_group_stride;
  const size_t items = (size_t)((n_rows + kBN - 1) / kBN) * (moe_ids ? (size_t)moe_cap : 1);
  const unsigned grid = (unsigned)std::min<size_t>(items, (size_t)std::max(1, sm_count()));
  const CUtensorMap &tb = *reinterpret_cast<const CUtensorMap *>(w->extras->tmap_b);
  e = launch_pdl(nvfp4_gemm_kernel, grid, kGemmThreads, kGemmSmem, s, tmap_a, tb, tmap_a, tb, tmap_a, p);
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4_gemm_kernel (planes)");
  FPB_LAUNCH_CHECK("nvfp4_gemm_kernel");
  return FPB_OK;
}
}  // namespace fpb

extern "C" int fpb_nvfp4_gemv_planes(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const void *x,
                                     int x_dtype, int tokens, void *y, int y_dtype, void *workspace,
                                     size_t workspace_bytes, void *stream) {
  if (!w || !x || !y || !workspace) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_planes: null pointer");
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv_planes: row range [%zu, %zu) outside %zu rows", row_begin, row_end,
                w->rows);
  if (row_begin % kBN)
    return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemv_planes: row_begin %zu is not a multiple of %d", row_begin, kBN);
  const size_t n = row_end - row_begin;
  return run_planes("fpb_nvfp4_gemv_planes", w, row_begin, n, x, x_dtype, false, 0, tokens, 1, nullptr, nullptr, 0, 0, y,
                    y_dtype, 0, (long long)n, workspace, workspace_bytes, as_stream(stream));
}

extern "C" int fpb_nvfp4_moe_gemv_planes(fpb_nvfp4_matrix *w, size_t rows_per_expert, const int32_t *distinct,
                                         const int32_t *count, int cap, const void *x, int x_dtype, size_t x_stride,
                                         int tokens, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                                         void *stream) {
  if (!w || !distinct || !count || !x || !y || !workspace)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_moe_gemv_planes: null pointer");
  if (cap < 1 || cap > 65535) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv_planes: cap %d", cap);
  if (rows_per_expert == 0 || rows_per_expert % kBN || w->rows % rows_per_expert || rows_per_expert > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv_planes: rows_per_expert %zu must be a multiple of %d dividing %zu",
                rows_per_expert, kBN, w->rows);
  if (x_stride != 0 && x_stride < (size_t)tokens * w->cols)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv_planes: x_stride %zu below tokens x cols", x_stride);
  const size_t groups = x_stride ? (size_t)cap : 1;
  return run_planes("fpb_nvfp4_moe_gemv_planes", w, 0, rows_per_expert, x, x_dtype, false, x_stride, tokens, groups,
                    distinct, count, cap, (int)(w->rows / rows_per_expert), y, y_dtype,
                    (long long)tokens * (long long)rows_per_expert, (long long)rows_per_expert, workspace,
                    workspace_bytes, as_stream(stream));
}

extern "C" int fpb_nvfp4_moe_gemv_planes_glu(fpb_nvfp4_matrix *w, size_t rows_per_expert, const int32_t *distinct,
                                             const int32_t *count, int cap, const float *gate_up,
                                             size_t gate_up_stride, int tokens, void *y, int y_dtype,
                                             void *workspace, size_t workspace_bytes, void *stream) {
  if (!w || !distinct || !count || !gate_up || !y || !workspace)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_moe_gemv_planes_glu: null pointer");
  if (cap < 1 || cap > 65535) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv_planes_glu: cap %d", cap);
  if (rows_per_expert == 0 || rows_per_expert % kBN || w->rows % rows_per_expert || rows_per_expert > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv_planes_glu: rows_per_expert %zu must be a multiple of %d "
                "dividing %zu", rows_per_expert, kBN, w->rows);
  if (gate_up_stride < (size_t)tokens * 2 * w->cols)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv_planes_glu: gate_up_stride %zu below tokens x 2 x cols",
                gate_up_stride);
  return run_planes("fpb_nvfp4_moe_gemv_planes_glu", w, 0, rows_per_expert, gate_up, FPB_F32, true, gate_up_stride,
                    tokens, (size_t)cap, distinct, count, cap, (int)(w->rows / rows_per_expert), y, y_dtype,
                    (long long)tokens * (long long)rows_per_expert, (long long)rows_per_expert, workspace,
                    workspace_bytes, as_stream(stream));
}

// ---- prepared tensor-core GEMV batch (fpb_nvfp4_gemv_batch_*) ------------------------
struct fpb_gemv_batch {
  fpb::PlaneSeg *segs = nullptr;  // device table
  CUtensorMap tmap_a{};           // the planes' codes
  CUtensorMap tmap_b0{};          // segment 0's weights (a valid map for the unused parameter)
  void *ws = nullptr;             // planes (or W4A4 activations) workspace
  int count = 0, batch = 0, K = 0, x_dtype = 0, y_dtype = 0, total_items = 0;
  int w4a4 = 0;                   // fpb_nvfp4_gemm_batch_create: x quantized to NVFP4, batch = m <= 128
  int tma_store = 0;              // W4A4: every member's y takes TMA stores (16-byte aligned base and pitch)
  int n_peer = 0;                 // peer copies of every member's y
};

static int batch_create_impl(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype, int batch,
                             bool w4a4, void *stream, fpb_gemv_batch **out, const void *const *y_peers = nullptr,
                             int n_peer = 0) {
  if (!segs || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batch_create: null pointer");
  *out = nullptr;
  if (count < 1 || count > kMoeIdsCached)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv_batch_create: count %d not in [1, %d]", count, kMoeIdsCached);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batch_create: dtype");
  if (n_peer < 0 || n_peer > kMaxPeerCopies || (n_peer && (!y_peers || w4a4)))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batch_create_peers: %d peer copies (at most %d)", n_peer,
                kMaxPeerCopies);
  const int max_batch = w4a4 ? kBM : 16;
  if (batch < 1 || batch > max_batch)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_%s_batch_create: %s %d not in [1, %d]", w4a4 ? "gemm" : "gemv",
                w4a4 ? "m" : "batch", batch, max_batch);
  if (!segs[0].w) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batch_create: null matrix");
  const size_t K = segs[0].w->cols;
  if (K % 256 || (!w4a4 && K > (size_t)kPlaneMaxK))
    return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemv_batch_create: cols %zu must be a multiple of 256%s", K,
                w4a4 ? "" : " and at most 4096");
  std::vector<PlaneSeg> host((size_t)count);
  int items = 0;
  bool all_tma = w4a4;
  for (int i = 0; i < count; ++i) {
    const fpb_gemv_segment &sg = segs[i];
    if (!sg.w || !sg.x || !sg.y)
      return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batch_create: null pointer in segment %d", i);
    if (sg.w->cols != K)
      return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv_batch_create: segment %d has %zu columns, segment 0 has %zu", i,
                  sg.w->cols, K);
    const size_t end = sg.row_end ? sg.row_end : sg.w->rows;
    if (sg.row_begin >= end || end > sg.w->rows || end - sg.row_begin > 0x7fffffff)
      return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv_batch_create: segment %d row range [%zu, %zu) outside %zu rows", i,
                  sg.row_begin, end, sg.w->rows);
    if (sg.row_begin % kBN)
      return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemv_batch_create: segment %d row_begin %zu not a multiple of %d",
                  i, sg.row_begin, kBN);
    if (int st = require_prepared(sg.w, "fpb_nvfp4_gemv_batch_create")) return st;
    PlaneSeg &d = host[(size_t)i];
    std::memcpy(&d.tmap_b, sg.w->extras->tmap_b, sizeof(CUtensorMap));
    d.b_sf = sg.w->extras->sf_tiled;
    d.b_globals = sg.w->row_globals;
    d.x = sg.x;
    d.y = sg.y;
    d.row_begin = (int)sg.row_begin;
    d.rows = (int)(end - sg.row_begin);
    d.item_begin = items;
    items += (d.rows + kBN - 1) / kBN;
    if (w4a4 && !encode_store_map(&d.tmap_y, sg.y, y_dtype == FPB_BF16, (uint64_t)batch, (uint64_t)d.rows,
                                  (uint64_t)d.rows, 32, 0))
      all_tma = false;
    d.n_peer = n_peer;
    for (int k = 0; k < n_peer; ++k) {
      const void *yp = y_peers[(size_t)i * n_peer + k];
      if (!yp || (reinterpret_cast<uintptr_t>(yp) & (y_dtype == FPB_BF16 ? 1 : 3)))
        return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batch_create_peers: segment %d copy %d null or unaligned",
                    i, k);
      d.y_peer[k] = const_cast<void *>(yp);
    }
    d.a_group = i;
    for (int j = 0; j < i; ++j)
      if (segs[j].x == sg.x) {
        d.a_group = j;
        break;
      }
  }
  if (int st = ensure_gemm_attr()) return st;
  fpb_gemv_batch *b = new fpb_gemv_batch();
  b->count = count;
  b->batch = batch;
  b->K = (int)K;
  b->x_dtype = x_dtype;
  b->y_dtype = y_dtype;
  b->total_items = items;
  b->w4a4 = w4a4 ? 1 : 0;
  b->n_peer = n_peer;
  b->tma_store = all_tma ? 1 : 0;
  std::memcpy(&b->tmap_b0, segs[0].w->extras->tmap_b, sizeof(CUtensorMap));
  cudaStream_t s = as_stream(stream);
  // W4A4: the same layout (codes, tiled factors, row globals) plus one amax
  // word per group; zeroed once, so rows past m stay zero codes and factors
  const size_t ws_bytes =
      fpb_nvfp4_gemv_planes_workspace_bytes((size_t)count, K) + (w4a4 ? 256 + (size_t)count * 4 : 0);
  cudaError_t e = cudaMalloc(reinterpret_cast<void **>(&b->segs), sizeof(PlaneSeg) * (size_t)count);
  if (e == cudaSuccess) e = cudaMalloc(&b->ws, ws_bytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(b->ws, 0, ws_bytes, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(b->segs, host.data(), sizeof(PlaneSeg) * (size_t)count, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    cudaFree(b->segs);
    cudaFree(b->ws);
    delete b;
    return cuda_fail(e, "fpb_nvfp4_gemv_batch_create");
  }
  const uint32_t a_box = w4a4 ? (uint32_t)((batch + 7) / 8 * 8) : (uint32_t)(batch * kPlanes);
  if (int st = encode_rows_u8(&b->tmap_a, b->ws, (uint64_t)count * kBM, K / 2, a_box)) {
    cudaFree(b->segs);
    cudaFree(b->ws);
    delete b;
    return st;
  }
  *out = b;
  return FPB_OK;
}

extern "C" int fpb_nvfp4_gemv_batch_create(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype,
                                           int batch, void *stream, fpb_gemv_batch **out) {
  return batch_create_impl(segs, count, x_dtype, y_dtype, batch, false, stream, out);
}

extern "C" int fpb_nvfp4_gemv_batch_create_peers(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype,
                                                 int batch, const void *const *y_peers, int n_peer, void *stream,
                                                 fpb_gemv_batch **out) {
  return batch_create_impl(segs, count, x_dtype, y_dtype, batch, false, stream, out, y_peers, n_peer);
}

extern "C" int fpb_nvfp4_gemm_batch_create(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype, int m,
                                           void *stream, fpb_gemv_batch **out) {
  return batch_create_impl(segs, count, x_dtype, y_dtype, m, true, stream, out);
}

// The W4A4 form of a batch: every distinct x quantized (amax, then encode),
// then the GEMM kernel over all members' tiles with per-row globals.
static int run_w4a4_batch(const fpb_gemv_batch *b, cudaStream_t s) {
  const size_t K = (size_t)b->K, rows = (size_t)b->count * kBM;
  uint8_t *packed = static_cast<uint8_t *>(b->ws);
  uint8_t *sf = packed + align256(rows * K / 2);
  float *ga = reinterpret_cast<float *>(sf + align256(sf_tiled_bytes(rows, K)));
  uint32_t *amax = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(b->ws) +
                                                align256(fpb_nvfp4_gemv_planes_workspace_bytes((size_t)b->count, K)));
  FPB_CUDA_TRY(cudaMemsetAsync(amax, 0, (size_t)b->count * sizeof(uint32_t), s));
  const size_t n = (size_t)b->batch * K;
  const dim3 agrid((unsigned)std::min<size_t>(128, (n + 8191) / 8192), (unsigned)b->count);
  const size_t warp_items = (size_t)b->batch * ((K / kNvfp4Group + 31) / 32);
  const dim3 egrid((unsigned)std::min<size_t>(256, (warp_items + 7) / 8), (unsigned)b->count);
  cudaError_t e;
  if (b->x_dtype == FPB_F32) {
    e = launch_pdl(batch_amax_kernel<float>, agrid, 256, 0, s, (const PlaneSeg *)b->segs, b->batch, b->K, amax);
    if (e == cudaSuccess)
      e = launch_pdl(batch_encode_kernel<float>, egrid, 256, 0, s, (const PlaneSeg *)b->segs, b->batch, b->K,
                     (const uint32_t *)amax, packed, sf, ga);
  } else {
    e = launch_pdl(batch_amax_kernel<uint16_t>, agrid, 256, 0, s, (const PlaneSeg *)b->segs, b->batch, b->K, amax);
    if (e == cudaSuccess)
      e = launch_pdl(batch_encode_kernel<uint16_t>, egrid, 256, 0, s, (const PlaneSeg *)b->segs, b->batch, b->K,
                     (const uint32_t *)amax, packed, sf, ga);
  }
  if (e != cudaSuccess) return cuda_fail(e, "batch_encode_kernel");
  FPB_LAUNCH_CHECK("batch_encode_kernel");
  GemmParams p{};
  p.a_box_rows = (b->batch + 7) / 8 * 8;
  p.a_sf = sf;
  p.y_bf16 = b->y_dtype == FPB_BF16;
  p.M = (int)rows;
  p.N = kBN;  // per segment in the kernel
  p.kb_count = b->K / 256;
  p.error = device_error_ptr();
  p.tokens = b->batch;
  p.a_globals = ga;
  p.segs = b->segs;
  p.nseg = b->count;
  p.total_items = b->total_items;
  p.tma_store = b->tma_store;
  const unsigned grid = (unsigned)std::min<size_t>((size_t)b->total_items, (size_t)std::max(1, sm_count()));
  // tmap_y (unused with segments: each member's map is in the table) gets a valid map
  e = launch_pdl(nvfp4_gemm_kernel, grid, kGemmThreads, kGemmSmem, s, b->tmap_a, b->tmap_b0, b->tmap_a, b->tmap_b0,
                 b->tmap_a, p);
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4_gemm_kernel (W4A4 batch)");
  FPB_LAUNCH_CHECK("nvfp4_gemm_kernel");
  return FPB_OK;
}

extern "C" int fpb_nvfp4_gemv_batch_run(const fpb_gemv_batch *b, void *stream) {
  if (!b) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batch_run: null handle");
  cudaStream_t s = as_stream(stream);
  if (b->w4a4) return run_w4a4_batch(b, s);
  const size_t K = (size_t)b->K, rows = (size_t)b->count * kBM;
  uint8_t *packed = static_cast<uint8_t *>(b->ws);
  uint8_t *sf = packed + align256(rows * K / 2);
  float *ga = reinterpret_cast<float *>(sf + align256(sf_tiled_bytes(rows, K)));
  const unsigned enc_grid = (unsigned)(b->count * b->batch);
  cudaError_t e = b->x_dtype == FPB_F32
      ? launch_pdl(planes_encode_kernel<float, false>, enc_grid, kPlaneThreads, 0, s, static_cast<const float *>(nullptr),
                   0LL, b->batch, b->K, static_cast<const int32_t *>(nullptr), packed, sf, ga,
                   static_cast<const PlaneSeg *>(b->segs))
      : launch_pdl(planes_encode_kernel<uint16_t, false>, enc_grid, kPlaneThreads, 0, s,
                   static_cast<const uint16_t *>(nullptr), 0LL, b->batch, b->K, static_cast<const int32_t *>(nullptr),
                   packed, sf, ga, static_cast<const PlaneSeg *>(b->segs));
  if (e != cudaSuccess) return cuda_fail(e, "planes_encode_kernel");
  FPB_LAUNCH_CHECK("planes_encode_kernel");
  GemmParams p{};
  p.a_box_rows = b->batch * kPlanes;
  p.a_sf = sf;
  p.y_bf16 = b->y_dtype == FPB_BF16;
  p.M = (int)rows;
  p.N = kBN;  // per segment in the kernel
  p.kb_count = b->K / 256;
  p.error = device_error_ptr();
  p.planes = 1;
  p.tokens = b->batch;
  p.a_globals = ga;
  p.segs = b->segs;
  p.nseg = b->count;
  p.total_items = b->total_items;
  p.peer_stores = b->n_peer > 0;
  const unsigned grid = (unsigned)std::min<size_t>((size_t)b->total_items, (size_t)std::max(1, sm_count()));
  e = launch_pdl(nvfp4_gemm_kernel, grid, kGemmThreads, kGemmSmem, s, b->tmap_a, b->tmap_b0, b->tmap_a, b->tmap_b0,
                 b->tmap_a, p);
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4_gemm_kernel (batch)");
  FPB_LAUNCH_CHECK("nvfp4_gemm_kernel");
  return FPB_OK;
}

extern "C" int fpb_nvfp4_gemv_batch_destroy(fpb_gemv_batch *b) {
  if (!b) return FPB_OK;
  cudaFree(b->segs);
  cudaFree(b->ws);
  delete b;
  return FPB_OK;
}

extern "C" int fpb_nvfp4_grouped_gemm_q(fpb_nvfp4_matrix *w, const uint8_t *a_packed, const uint8_t *a_sf_tiled,
                                        const float *a_global, size_t padded_rows, const int32_t *tile_experts,
                                        const int32_t *token_rows, size_t rows_per_expert, void *y, int y_dtype,
                                        void *stream) {
  if (!w || !a_packed || !a_sf_tiled || !a_global || !tile_experts || !y)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_grouped_gemm_q: null pointer");
  if (padded_rows == 0 || padded_rows % kBM || padded_rows / kBM > 65535)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_grouped_gemm_q: padded_rows %zu must be a positive multiple of %d",
                padded_rows, kBM);
  if (rows_per_expert == 0 || rows_per_expert % kBN || w->rows % rows_per_expert)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_grouped_gemm_q: rows_per_expert %zu must be a multiple of %d dividing %zu",
                rows_per_expert, kBN, w->rows);
  if (y_dtype != FPB_F32 && y_dtype != FPB_BF16)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_grouped_gemm_q: dtype");
  cudaStream_t s = as_stream(stream);
  int st = require_prepared(w, "fpb_nvfp4_grouped_gemm_q");
  if (st) return st;
  CUtensorMap tmap_a;
  if ((st = encode_rows_u8(&tmap_a, a_packed, padded_rows, w->cols / 2, kBM))) return st;
  {
    static std::mutex mu;
    static std::vector<int> attr_devs;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (std::find(attr_devs.begin(), attr_devs.end(), dev) == attr_devs.end()) {
      FPB_CUDA_TRY(
          cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem));
      attr_devs.push_back(dev);
    }
  }
  int *err = nullptr;
  FPB_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_device_error));
  GemmParams p{};
  p.a_box_rows = kBM;
  p.a_sf = a_sf_tiled;
  p.b_sf = w->extras->sf_tiled;
  p.a_global = a_global;
  p.b_globals = w->row_globals;
  p.y = y;
  p.N = (int)rows_per_expert;
  p.ldy = p.N;
  p.y_bf16 = y_dtype == FPB_BF16;
  p.M = (int)padded_rows;
  p.n_base = 0;
  p.kb_count = (int)((w->cols + 255) / 256);
  p.error = err;
  p.tile_experts = tile_experts;
  p.row_tokens = token_rows;
  p.n_experts = (int)(w->rows / rows_per_expert);
  CUtensorMap tmap_y{};
  p.tma_store = encode_store_map(&tmap_y, y, p.y_bf16, padded_rows, p.N, p.ldy, 32, 0);
  const size_t tiles = (rows_per_expert / kBN) * (padded_rows / kBM);
  const unsigned grid = (unsigned)std::min<size_t>(tiles, (size_t)std::max(1, sm_count()));
  launch_pdl(nvfp4_gemm_kernel, grid, kGemmThreads, kGemmSmem, s, tmap_a, *reinterpret_cast<const CUtensorMap *>(w->extras->tmap_b),
                                                 tmap_y, *reinterpret_cast<const CUtensorMap *>(w->extras->tmap_b), tmap_a, p);
  FPB_LAUNCH_CHECK("nvfp4_gemm_kernel(grouped)");
  return FPB_OK;
}

// Fused gate/up copies (interleaved factors, 64-row code map) for an
// intermediate size `inter`; built once per matrix (fpb_nvfp4_matrix_prepare_glu,
// at load time), allocates and synchronises `s`.
static int prepare_glu_weights(fpb_nvfp4_matrix *m, size_t inter, cudaStream_t s) {
  int st = prepare_gemm_weights(m, s);
  if (st) return st;
  MatrixExtras *x = m->extras;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (x->sf_tiled_glu && x->glu_inter == inter) return FPB_OK;
  const size_t bytes = sf_tiled_bytes(m->rows, m->cols);
  if (!x->sf_tiled_glu) FPB_CUDA_TRY(cudaMalloc(&x->sf_tiled_glu, bytes));
  x->glu_inter = 0;
  sf_tile_kernel<<<grid_for(bytes), 256, 0, s>>>(m->scales, m->rows, m->cols, x->sf_tiled_glu, bytes, inter);
  FPB_LAUNCH_CHECK("sf_tile_kernel(glu)");
  const uint8_t *codes = x->packed_folded ? x->packed_folded : m->packed;
  if ((st = encode_rows_u8(reinterpret_cast<CUtensorMap *>(x->tmap_b64), codes, m->rows, m->cols / 2, 64))) return st;
  FPB_CUDA_TRY(cudaStreamSynchronize(s));
  x->glu_inter = inter;
  return FPB_OK;
}

extern "C" int fpb_nvfp4_grouped_gemm_swiglu_q(fpb_nvfp4_matrix *w, const uint8_t *a_packed,
                                               const uint8_t *a_sf_tiled, const float *a_global, size_t padded_rows,
                                               const int32_t *tile_experts, const int32_t *token_rows, size_t inter,
                                               void *h, int h_dtype, uint32_t *amax_bits, void *stream) {
  if (!w || !a_packed || !a_sf_tiled || !a_global || !tile_experts || !h || !amax_bits)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_grouped_gemm_swiglu_q: null pointer");
  if (padded_rows == 0 || padded_rows % kBM || padded_rows / kBM > 65535)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_grouped_gemm_swiglu_q: padded_rows %zu must be a positive multiple of %d",
                padded_rows, kBM);
  if (inter == 0 || inter % 64 || w->rows % (2 * inter))
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_grouped_gemm_swiglu_q: inter %zu must be a multiple of 64 with 2*inter "
                "dividing %zu", inter, w->rows);
  if (h_dtype != FPB_F32 && h_dtype != FPB_BF16)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_grouped_gemm_swiglu_q: dtype");
  if (reinterpret_cast<uintptr_t>(h) & 15)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_grouped_gemm_swiglu_q: h must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  int st = require_prepared(w, "fpb_nvfp4_grouped_gemm_swiglu_q");
  if (st) return st;
  if (!w->extras->sf_tiled_glu || w->extras->glu_inter != inter)
    return fail(FPB_ERR_INVALID_ARGUMENT,
                "fpb_nvfp4_grouped_gemm_swiglu_q: call fpb_nvfp4_matrix_prepare_glu(w, %zu) at load time", inter);
  CUtensorMap tmap_a, tmap_y{};
  if ((st = encode_rows_u8(&tmap_a, a_packed, padded_rows, w->cols / 2, kBM))) return st;
  // h boxes: 32 rows x 32 columns per epilogue warp (bf16 unswizzled, f32
  // with 128-byte swizzle)
  if (!encode_store_map(&tmap_y, h, h_dtype == FPB_BF16, padded_rows, inter, inter, 32, 32))
    return fail(FPB_ERR_CUDA, "fpb_nvfp4_grouped_gemm_swiglu_q: cannot encode the output map");
  {
    static std::mutex mu;
    static std::vector<int> attr_devs;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (std::find(attr_devs.begin(), attr_devs.end(), dev) == attr_devs.end()) {
      FPB_CUDA_TRY(
          cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem));
      attr_devs.push_back(dev);
    }
  }
  FPB_CUDA_TRY(cudaMemsetAsync(amax_bits, 0, sizeof(uint32_t), s));
  GemmParams p{};
  p.a_box_rows = kBM;
  p.a_sf = a_sf_tiled;
  p.b_sf = w->extras->sf_tiled_glu;
  p.a_global = a_global;
  p.b_globals = w->row_globals;
  p.y = h;
  p.N = (int)(2 * inter);
  p.ldy = (long long)inter;
  p.y_bf16 = h_dtype == FPB_BF16;
  p.M = (int)padded_rows;
  p.n_base = 0;
  p.kb_count = (int)((w->cols + 255) / 256);
  p.error = device_error_ptr();
  p.tile_experts = tile_experts;
  p.row_tokens = token_rows;
  p.n_experts = (int)(w->rows / (2 * inter));
  p.tma_store = 1;
  p.glu = 1;
  p.amax_bits = amax_bits;
  const size_t tiles = (2 * inter / kBN) * (padded_rows / kBM);
  const unsigned grid = (unsigned)std::min<size_t>(tiles, (size_t)std::max(1, sm_count()));
  launch_pdl(nvfp4_gemm_kernel, grid, kGemmThreads, kGemmSmem, s, tmap_a, *reinterpret_cast<const CUtensorMap *>(w->extras->tmap_b),
                                                 tmap_y, *reinterpret_cast<const CUtensorMap *>(w->extras->tmap_b64),
                                                 tmap_a, p);
  FPB_LAUNCH_CHECK("nvfp4_gemm_kernel(grouped swiglu)");
  return FPB_OK;
}

// Device address of g_device_error on the current device, cached per device
// (kernels of other translation units record their errors there).
int *fpb::device_error_ptr() {
  static std::mutex mu;
  static std::vector<std::pair<int, int *>> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  for (auto &e : cache)
    if (e.first == dev) return e.second;
  int *p = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_device_error) != cudaSuccess) return nullptr;
  cache.push_back({dev, p});
  return p;
}

extern "C" int fpb_device_error(int *out, int reset) {
  if (!out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_device_error: null pointer");
  FPB_CUDA_TRY(cudaDeviceSynchronize());
  FPB_CUDA_TRY(cudaMemcpyFromSymbol(out, g_device_error, sizeof(int)));
  if (reset) {
    int zero = 0;
    FPB_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  }
  return FPB_OK;
}

// ---- the reference's activation semantics: bf16 hi + lo on bf16 weights ----------------
// gemm/nvfp4.rs:33-50 keeps the activations in f32 and multiplies their bf16
// hi and lo halves (hi = bf16(x), lo = bf16(x - hi)) by the weights
// dequantized to bf16 (E2M1 * e4m3 scale, exact in bf16), accumulating in
// f32, then scales by the row global.  Here: the split and the dequantized
// weights go to the caller's workspace (two element-wise launches), then the
// persistent GEMM kernel runs in its bf16 mode (tcgen05 kind::f16), one pass
// per (A, B) pair of each K block.
namespace fpb {

// hi = bf16(x) (round to nearest even), lo = bf16(x - hi), x f32 [n].
__global__ void split_hilo_kernel(const float *x, size_t n, __nv_bfloat16 *hi, __nv_bfloat16 *lo) {
  pdl_enter();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    if (lo) lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

// Rows of an NVFP4 matrix as bf16 E2M1 * e4m3 scale (exact; no row global),
// one thread per code byte.
__global__ void nvfp4_to_bf16_kernel(const uint8_t *packed, const uint8_t *scales, size_t rows, size_t cols,
                                     __nv_bfloat162 *out) {
  pdl_enter();
  const size_t n = rows * cols / 2, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const size_t r = (2 * i) / cols, c = (2 * i) % cols;
    const float s = e4m3_to_f32(scales[r * (cols / 16) + c / 16]);
    const uint8_t b = packed[i];
    out[i] = __floats2bfloat162_rn(e2m1_to_f32(b & 0xf) * s, e2m1_to_f32(b >> 4) * s);
  }
}

int run_f16_gemm(const F16Gemm &g, cudaStream_t s) {
  if (int st = ensure_gemm_attr()) return st;
  CUtensorMap ta, ta2, tb, tb2, ty{};
  int st;
  if ((st = encode_rows_u8(&ta, g.a[0], g.m, g.k * 2, kBM))) return st;
  if ((st = encode_rows_u8(&ta2, g.a[1] ? g.a[1] : g.a[0], g.m, g.k * 2, kBM))) return st;
  if ((st = encode_rows_u8(&tb, g.b[0], g.n, g.k * 2, kBN))) return st;
  if ((st = encode_rows_u8(&tb2, g.b[1] ? g.b[1] : g.b[0], g.n, g.k * 2, kBN))) return st;
  int *err = nullptr;
  FPB_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_device_error));
  GemmParams p{};
  p.a_box_rows = kBM;
  p.b_globals = g.b_globals;
  p.y = g.y;
  p.N = (int)g.n;
  p.ldy = p.N;
  p.y_bf16 = g.y_bf16;
  p.M = (int)g.m;
  p.n_base = 0;
  p.kb_count = (int)((g.k + 63) / 64);
  p.error = err;
  p.f16 = 1;
  p.passes = g.passes;
  for (int j = 0; j < 3; ++j) {
    p.a_sel[j] = g.a_sel[j];
    p.b_sel[j] = g.b_sel[j];
  }
  p.tma_store = encode_store_map(&ty, g.y, p.y_bf16, g.m, p.N, p.ldy, 32, 0);
  const size_t tiles = (size_t)((p.N + kBN - 1) / kBN) * ((g.m + kBM - 1) / kBM);
  const unsigned grid = (unsigned)std::min<size_t>(tiles, (size_t)std::max(1, sm_count()));
  launch_pdl(nvfp4_gemm_kernel, grid, kGemmThreads, kGemmSmem, s, ta, tb, ty, tb2, ta2, p);
  FPB_LAUNCH_CHECK("nvfp4_gemm_kernel(bf16)");
  return FPB_OK;
}

// Activations for the bf16 mode: bf16 x is read in place (lo = 0: one
// pass); f32 x is split into hi and lo in the workspace.  Returns the bytes
// of workspace used.
int hilo_activations(const void *x, int x_dtype, size_t m, size_t k, uint8_t *ws, const void **hi,
                     const void **lo, size_t *used, cudaStream_t s) {
  *used = 0;
  if (x_dtype == FPB_BF16) {
    *hi = x;
    *lo = nullptr;
    return FPB_OK;
  }
  __nv_bfloat16 *h = reinterpret_cast<__nv_bfloat16 *>(ws);
  __nv_bfloat16 *l = reinterpret_cast<__nv_bfloat16 *>(ws + align256(m * k * 2));
  launch_pdl(split_hilo_kernel, grid_for(m * k), 256, 0, s, static_cast<const float *>(x), m * k, h, l);
  FPB_LAUNCH_CHECK("split_hilo_kernel");
  *hi = h;
  *lo = l;
  *used = 2 * align256(m * k * 2);
  return FPB_OK;
}

size_t hilo_workspace_bytes(size_t m, size_t k, int x_dtype) {
  return x_dtype == FPB_BF16 ? 0 : 2 * align256(m * k * 2);
}

}  // namespace fpb

extern "C" size_t fpb_nvfp4_gemm_hilo_workspace_bytes(size_t m, size_t rows, size_t k, int x_dtype) {
  return hilo_workspace_bytes(m, k, x_dtype) + align256(rows * k * 2) + 256;
}

extern "C" int fpb_nvfp4_gemm_hilo(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const void *x,
                                   int x_dtype, size_t m, void *y, int y_dtype, void *workspace,
                                   size_t workspace_bytes, void *stream) {
  if (!w || !x || !y || !workspace) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemm_hilo: null pointer");
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemm_hilo: row range [%zu, %zu) outside %zu rows", row_begin, row_end,
                w->rows);
  if (m == 0 || m > (size_t)65535 * kBM) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemm_hilo: m = %zu", m);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemm_hilo: dtype");
  const size_t rows = row_end - row_begin, k = w->cols;
  const size_t need = fpb_nvfp4_gemm_hilo_workspace_bytes(m, rows, k, x_dtype);
  if (workspace_bytes < need)
    return fail(FPB_ERR_WORKSPACE, "fpb_nvfp4_gemm_hilo: workspace %zu < %zu bytes", workspace_bytes, need);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) || (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemm_hilo: workspace 256-byte and x 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const void *hi, *lo;
  size_t used = 0;
  int st = hilo_activations(x, x_dtype, m, k, ws, &hi, &lo, &used, s);
  if (st) return st;
  __nv_bfloat162 *wb = reinterpret_cast<__nv_bfloat162 *>(ws + used);
  launch_pdl(nvfp4_to_bf16_kernel, grid_for(rows * k / 2), 256, 0, s, w->packed + row_begin * (k / 2),
             w->scales + row_begin * (k / 16), rows, k, wb);
  FPB_LAUNCH_CHECK("nvfp4_to_bf16_kernel");
  F16Gemm g{};
  g.m = m;
  g.n = rows;
  g.k = k;
  g.a[0] = hi;
  g.a[1] = lo;
  g.b[0] = wb;
  g.b[1] = nullptr;
  g.passes = lo ? 2 : 1;  // hi x W, then lo x W (gemm/nvfp4.rs:47-48)
  g.a_sel[0] = 0, g.b_sel[0] = 0;
  g.a_sel[1] = 1, g.b_sel[1] = 0;
  g.b_globals = w->row_globals + row_begin;
  g.y = y;
  g.y_bf16 = y_dtype == FPB_BF16;
  return run_f16_gemm(g, s);
}
