// FP8 E4M3 weights, quantizers and the prefill FP8 GEMM on the tcgen05 tensor
// cores (crates/firepit-kernels/src/weights/fp8.rs, src/gemm/mod.rs:67-206,
// 417-697).
//
// Formats (weights/fp8.rs:8-27): bits [rows, cols] e4m3 row-major; scales f32
// either a [rows/block_n, cols/block_k] grid (Fp8Scaling::Blocks) or one per
// row (Fp8Scaling::Rows, block_n = block_k = 0 at this ABI).
//
// Quantizers (no reference counterpart; the rule of the task's config 1):
// scale = amax/448 over each block (or row, or activation token), bits =
// RN_e4m3_satfinite(w / scale), 0 when the scale is 0.  Every step is a single
// IEEE operation, so the result equals the CPU oracle bit for bit.
//
// GEMM.  y[m, n] = sum_kb (w_s[n / block_n, kb] a_s[m]) * sum_{k in kb} a[m,k] w[n,k]
// (blocks) or (a_s[m] w_s[n]) * sum_k a[m,k] w[n,k] (rows), activations
// quantized to e4m3 with a per-token scale (the config's W8A8 setting; the
// reference keeps f32 activations split into bf16 hi/lo).  One CTA per
// 128 x 256 output tile (operand bytes per MMA flop are what bound a
// 128 x 128 tile: both operands stream from L2 for every K block):
//  * warp 0: TMA producer, 4-stage ring of a 128 x 128-byte A tile and a
//    256 x 128-byte B tile per 128-wide K block (128-byte swizzle);
//  * warp 1: TMEM allocation and MMA issue, four
//    tcgen05.mma.cta_group::1.kind::f8f6f4 (M 128, N 256, K 32) per K block;
//  * warps 4..11: epilogue, two warps per 32-lane TMEM quadrant (128 columns
//    each), with the registers of warpgroup 0 (setmaxnreg) so that each TMEM
//    load overlaps the previous chunk's scale-and-add.
// Block scales vary along K every 128 columns, so with block scaling each K
// block's product goes to one of two TMEM accumulators (double-buffered): the
// epilogue warps read it, multiply it by that block's scale and add it to
// their register accumulators while the tensor cores fill the other buffer
// (the promotion of per-block partial sums in f32, as in the reference's
// per-part scale).  With row scales the tensor cores accumulate the whole K
// range in TMEM.  Every mbarrier wait is bounded; a wait that gives up records
// an error code (fpb_device_error) and ends its role.  Every TMA load lands in
// the issuing CTA alone.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "common.cuh"
#include "fp8_matrix.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"


namespace fpb {

// ---- quantizer ---------------------------------------------------------------------
__device__ __forceinline__ float load_as_f32(const float *p, size_t i) { return p[i]; }
__device__ __forceinline__ float load_as_f32(const __nv_bfloat16 *p, size_t i) { return __bfloat162float(p[i]); }

// One CTA per scale block of bn rows x bk columns (bk a multiple of 4).
template <typename T>
__global__ void __launch_bounds__(256) fp8_quantize_kernel(const T *w, size_t cols, int bn, int bk, uint8_t *bits,
                                                           float *scales) {
  __shared__ uint32_t wmax[8];
  const size_t gc = cols / (size_t)bk;
  const size_t b = blockIdx.x;
  const size_t r0 = (b / gc) * (size_t)bn, c0 = (b % gc) * (size_t)bk;
  const int q4 = bk / 4;
  const int n4 = bn * q4;
  uint32_t m = 0;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const size_t base = (r0 + i / q4) * cols + c0 + (size_t)(i % q4) * 4;
#pragma unroll
    for (int t = 0; t < 4; ++t) m = max(m, __float_as_uint(load_as_f32(w, base + t)) & 0x7fffffffu);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  m = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = max(m, wmax[i]);
  const float s = __fdiv_rn(__uint_as_float(m), 448.0f);
  if (threadIdx.x == 0) scales[b] = s;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const size_t base = (r0 + i / q4) * cols + c0 + (size_t)(i % q4) * 4;
    uint32_t packed = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t q = s > 0.0f ? f32_to_e4m3(__fdiv_rn(load_as_f32(w, base + t), s)) : 0u;
      packed |= q << (8 * t);
    }
    *reinterpret_cast<uint32_t *>(bits + base) = packed;
  }
}

// ---- GEMM kernel ---------------------------------------------------------------------
constexpr int kF8Tile = 128;                      // M and K-block (bytes) of a tile
constexpr int kF8BN = 256;                        // N of a tile
constexpr int kF8Stages = 4;
constexpr int kF8ABytes = kF8Tile * kF8Tile;      // 16 KB of A per stage
constexpr int kF8BBytes = kF8BN * kF8Tile;        // 32 KB of B per stage
constexpr int kF8EpiWarps = 8;                    // warpgroups 1 and 2
constexpr int kF8Threads = 128 + 32 * kF8EpiWarps;  // warpgroup 0: producer, MMA, two idle warps
// Register split (setmaxnreg): the launch gives every thread 168; warpgroup 0
// drops to 56 and the epilogue warpgroups take the rest (128*56 + 256*224 =
// 384*168), enough for a row's 128 f32 sums plus two 32-register TMEM buffers.
constexpr int kF8CtrlRegs = 56, kF8EpiRegs = 224;
static_assert(128 * kF8CtrlRegs + 32 * kF8EpiWarps * kF8EpiRegs <= kF8Threads * 168, "register split");
constexpr uint32_t kF8TmemCols = 512;             // two 256-column accumulators
// Epilogue staging: one 32-row x 128-byte box per epilogue warp (128-byte
// swizzle), stored by TMA while the warp goes on with the next tile.
constexpr int kF8OutBoxBytes = 32 * 128;
constexpr size_t kF8Smem = 1024 + kF8Stages * (kF8ABytes + kF8BBytes) + kF8EpiWarps * kF8OutBoxBytes + 256;
static_assert(kF8Smem <= 232448, "shared memory per CTA");

struct Fp8GemmParams {
  const float *a_scale;  // [M] per token
  const float *w_scale;  // blocks: [rows/bn, ws_cols]; rows: [rows]
  void *y;
  long long ldy;
  int y_bf16;
  int M;
  int N;           // weight rows of the view (grouped: rows per expert)
  int n_base;      // first weight row of the view (multiple of 128)
  int kb_count;    // ceil(K / 128)
  int bn, bk;      // block scaling: multiples of 128
  int ws_cols;     // columns of the scale grid
  int *error;
  int tma_store;                // y through tmap_y (else direct per-row stores: unaligned y)
  const int32_t *tile_experts;  // grouped mode (gemm/mod.rs:103-140), else null
  int n_experts;
  // Schedule.  Tile t = n_tile * m_tiles + m_tile (neighbouring CTAs share a
  // weight tile).  CTA c first runs whole tiles c, c + G, ... below
  // whole_tiles (G = grid), then the K blocks [c*T/G, (c+1)*T/G) of the
  // concatenation of the remaining tiles' K blocks (T = total_kb): whole
  // tiles, or a tile's K range split between consecutive CTAs (stream-K
  // over the last, partial wave).  A CTA with part of a tile writes its f32
  // partial sums to `partials`; the last of the tile's parts to finish (per
  // epilogue warp, a counter per tile and warp) adds them in part order and
  // stores the tile.  No CTA waits for another.
  int m_tiles, tiles;
  int whole_tiles;      // tiles [0, whole_tiles) run whole, strided over the CTAs
  long long total_kb;   // K blocks of the remaining (split) tiles
  int ctas, max_seg;
  float *partials;      // [split tiles][max_seg][kF8EpiWarps][32][32 lanes] float4; null: no split
  int *tile_counters;   // [split tiles][kF8EpiWarps], zero at launch, left zero
};

__device__ __forceinline__ void f8_report(int *error, volatile int *abort, int code) {
  *abort = 1;
  if (error) atomicCAS(error, 0, code);
}

// The CTA whose K-block range holds global K block x.
__host__ __device__ __forceinline__ long long f8_cta_of(long long x, long long total, long long ctas) {
  return ((x + 1) * ctas - 1) / total;
}

// One tile's part in a CTA's range: K blocks [kb0, kb1) of tile `tile`,
// part `seg` of `nseg`.
struct F8Seg {
  int tile, kb0, kb1, seg, nseg;
};

// Iterates the CTA's parts.  Without partial-sum storage every part is a
// whole tile: tiles blockIdx.x, blockIdx.x + ctas, ... (persistent CTAs, so a
// tile's loads and MMAs start while the previous tile's epilogue runs).
struct F8Sched {
  long long gk, end;
  int t;
  __device__ __forceinline__ F8Sched(const Fp8GemmParams &p) {
    t = blockIdx.x;
    gk = p.partials ? (long long)blockIdx.x * p.total_kb / p.ctas : 0;
    end = p.partials ? ((long long)blockIdx.x + 1) * p.total_kb / p.ctas : 0;
  }
  __device__ __forceinline__ bool next(const Fp8GemmParams &p, F8Seg &g) {
    if (t < p.whole_tiles) {
      g.tile = t;
      g.kb0 = 0;
      g.kb1 = p.kb_count;
      g.seg = 0;
      g.nseg = 1;
      t += p.ctas;
      return true;
    }
    if (gk >= end) return false;
    g.tile = p.whole_tiles + (int)(gk / p.kb_count);
    g.kb0 = (int)(gk - (long long)(g.tile - p.whole_tiles) * p.kb_count);
    g.kb1 = (int)min((long long)p.kb_count, g.kb0 + (end - gk));
    const long long t0 = (long long)(g.tile - p.whole_tiles) * p.kb_count;
    const long long first = f8_cta_of(t0, p.total_kb, p.ctas);
    const long long last = f8_cta_of(t0 + p.kb_count - 1, p.total_kb, p.ctas);
    g.seg = (int)(blockIdx.x - first);
    g.nseg = (int)(last - first + 1);
    gk += g.kb1 - g.kb0;
    return true;
  }
};

template <bool kBlocks>
__global__ void __launch_bounds__(kF8Threads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_y, Fp8GemmParams p) {
  using namespace sm100;
  pdl_enter();  // programmatic dependent launch: nothing is read before the previous kernel is done
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = base;
  uint8_t *sB = sA + kF8Stages * kF8ABytes;
  uint8_t *sOut = sB + kF8Stages * kF8BBytes;  // [kF8EpiWarps][32 rows][128 bytes]
  uint64_t *full = reinterpret_cast<uint64_t *>(sOut + kF8EpiWarps * kF8OutBoxBytes);
  uint64_t *empty = full + kF8Stages;
  // Accumulator barriers per (buffer, column half): [b * 2 + h].
  uint64_t *acc_full = empty + kF8Stages;  // [4]
  uint64_t *acc_empty = acc_full + 4;      // [4]
  uint32_t *tmem_base_s = reinterpret_cast<uint32_t *>(acc_empty + 4);
  volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_base_s + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Weight row base of a tile (grouped: its expert's rows); false for a row
  // tile past the end of a device-built layout (expert -1) or a bad id.
  auto tile_rows = [&](int tile, int &m0, int &n0, int &n_base) -> bool {
    const int m_tile = tile % p.m_tiles, n_tile = tile / p.m_tiles;
    m0 = m_tile * kF8Tile;
    n0 = n_tile * kF8BN;
    n_base = p.n_base;
    if (p.tile_experts) {
      const int e = p.tile_experts[m_tile];
      if (e == -1) return false;
      if (e < 0 || e >= p.n_experts) {
        if (threadIdx.x == 0 && p.error) atomicCAS(p.error, 0, 306);
        return false;
      }
      n_base = e * p.N;
    }
    return true;
  };
  if (p.tile_experts) {  // grouped: one whole tile per CTA; a dead tile's CTA leaves at once
    int m0, n0, nb;
    if (!tile_rows((int)blockIdx.x, m0, n0, nb)) return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kF8Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kF8EpiWarps / 2);  // the four warps of a column half
    }
    *abort_s = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
    if (p.tma_store) prefetch_tensormap(&tmap_y);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_s, kF8TmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kF8CtrlRegs));
  if (warp == 0) {
    // ---- TMA producer: the CTA's K blocks, one ring across parts ----------------
    if (elect_one()) {
      uint32_t g = 0;
      bool ok = true;
      F8Sched sched(p);
      F8Seg sg;
      while (ok && sched.next(p, sg)) {
        int m0, n0, n_base;
        tile_rows(sg.tile, m0, n0, n_base);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++g) {
          const uint32_t s = g % kF8Stages;
          if (g >= kF8Stages && !mbar_wait(&empty[s], ((g / kF8Stages) - 1) & 1, abort_s)) {
            f8_report(p.error, abort_s, 301);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kF8ABytes + kF8BBytes);
          tma_load_2d(sA + s * kF8ABytes, &tmap_a, kb * kF8Tile, m0, &full[s]);
          tma_load_2d(sB + s * kF8BBytes, &tmap_b, kb * kF8Tile, n_base + n0, &full[s]);
        }
      }
      // Our own copies must have landed before the CTA may exit.
      for (uint32_t j = (g > kF8Stages ? g - kF8Stages : 0); j < g; ++j)
        if (!mbar_wait(&full[j % kF8Stages], (j / kF8Stages) & 1, abort_s)) f8_report(p.error, abort_s, 302);
    }
  } else if (warp == 1) {
    // ---- MMA issuer -------------------------------------------------------------
    // Blocks: each K block into TMEM buffer (g & 1); rows: each part into
    // buffer (part & 1), accumulated over its K blocks.  Each K block runs as
    // two N = 128 halves (B rows 0-127, then 128-255) with their own
    // barriers, so the epilogue warps of a column half take their columns as
    // soon as those are done, and hand them back independently: the half
    // has one and a half K blocks of MMA time to be read and released.
    if (elect_one()) {
      constexpr int kHalf = kF8BN / 2;
      const uint32_t idesc = idesc_f8(kF8Tile, kHalf);
      uint32_t g = 0, part = 0;
      bool ok = true;
      F8Sched sched(p);
      F8Seg sg;
      while (ok && sched.next(p, sg)) {
        const uint32_t pb = part & 1;
        if (!kBlocks && part >= 2)
          for (int h = 0; h < 2 && ok; ++h)
            if (!mbar_wait(&acc_empty[pb * 2 + h], ((part >> 1) - 1) & 1, abort_s)) {
              f8_report(p.error, abort_s, 304);
              ok = false;
            }
        if (!ok) break;
        for (int kb = sg.kb0; kb < sg.kb1 && ok; ++kb, ++g) {
          const uint32_t s = g % kF8Stages;
          if (!mbar_wait(&full[s], (g / kF8Stages) & 1, abort_s)) {
            f8_report(p.error, abort_s, 303);
            ok = false;
            break;
          }
          const uint32_t b = kBlocks ? (g & 1) : pb;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (kBlocks && g >= 2 && !mbar_wait(&acc_empty[b * 2 + h], ((g >> 1) - 1) & 1, abort_s)) {
              f8_report(p.error, abort_s, 304);
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t a_desc = smem_desc(smem_u32(sA + s * kF8ABytes) + kk * 32, 16, 1024, 2);
              const uint64_t b_desc =
                  smem_desc(smem_u32(sB + s * kF8BBytes + h * (kHalf * kF8Tile)) + kk * 32, 16, 1024, 2);
              const uint32_t acc = kBlocks ? (kk != 0) : (kb != sg.kb0 || kk != 0);
              mma_f8(tmem + b * kF8BN + h * kHalf, a_desc, b_desc, idesc, acc);
            }
            if (kBlocks) tc_commit(&acc_full[b * 2 + h]);
          }
          if (!ok) break;
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        if (!kBlocks) {
          tc_commit(&acc_full[pb * 2]);
          tc_commit(&acc_full[pb * 2 + 1]);
        }
        ++part;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kF8EpiRegs));
    // ---- epilogue: quadrant (warp % 4), column part (warp - 4) / 4 -------------
    constexpr int kParts = kF8EpiWarps / 4;
    constexpr int kCols = kF8BN / kParts;  // columns per epilogue warp
    static_assert(kCols == 128, "four 32-column chunks per epilogue warp");
    const int qd = warp & 3, half = (warp - 4) >> 2;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const int c_base = half * kCols;
    uint32_t g = 0, part = 0;
    bool ok = true;
    F8Sched sched(p);
    F8Seg sg;
    while (ok && sched.next(p, sg)) {
      int m0, n0, n_base;
      tile_rows(sg.tile, m0, n0, n_base);
      const int row = m0 + qd * 32 + lane;
      float acc[kCols];
#pragma unroll
      for (int j = 0; j < kCols; ++j) acc[j] = 0.0f;
      // The token scale is folded into each block scale before it meets the
      // partial sums, so that extreme but finite scale pairs (one tiny, one
      // huge) do not overflow or underflow in between.
      const float as = row < p.M ? __ldg(p.a_scale + row) : 0.0f;
      if (kBlocks) {
        // A part's columns lie in one block of bn (a multiple of 128) rows.
        const int nb = (n_base + n0 + c_base) / p.bn;
        const float *ws_row = p.w_scale + (size_t)nb * p.ws_cols;
        // The next K block's scale is loaded before this block's wait, so its
        // latency hides behind the wait and the promotion (the FMAs need it).
        float ws_next = __ldg(ws_row + (sg.kb0 * kF8Tile) / p.bk);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++g) {
          const uint32_t b = g & 1;
          const float ws = ws_next * as;
          if (kb + 1 < sg.kb1) ws_next = __ldg(ws_row + ((kb + 1) * kF8Tile) / p.bk);
          if (!mbar_wait(&acc_full[b * 2 + half], (g >> 1) & 1, abort_s)) {
            f8_report(p.error, abort_s, 305);
            ok = false;
            break;
          }
          __syncwarp();  // the TMEM loads below are warp-collective
          tc_fence_after();
          const uint32_t taddr = tmem + lane_base + b * kF8BN + c_base;
          // Two TMEM loads per wait (a wait covers every load in flight, and a
          // TMEM round trip costs more than 64 FMAs): two round trips per K
          // block instead of four.
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t ra[32], rb[32];
            tmem_ld32(taddr + h * 64, ra);
            tmem_ld32(taddr + h * 64 + 32, rb);
            tmem_ld_wait(ra);
            tmem_ld_wait(rb);
            if (h == 1) {
              // The whole buffer is in registers: hand it back to the tensor
              // cores before the last 64 FMAs, which then overlap the next MMA.
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[b * 2 + half]);
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[h * 64 + j] = fmaf(__uint_as_float(ra[j]), ws, acc[h * 64 + j]);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              acc[h * 64 + 32 + j] = fmaf(__uint_as_float(rb[j]), ws, acc[h * 64 + 32 + j]);
          }
        }
        if (!ok) break;
      } else {
        const uint32_t pb = part & 1;
        if (!mbar_wait(&acc_full[pb * 2 + half], (part >> 1) & 1, abort_s)) {
          f8_report(p.error, abort_s, 305);
          break;
        }
        __syncwarp();
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kCols / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + pb * kF8BN + c_base + c * 32, r);
          tmem_ld_wait(r);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c * 32 + j] = __uint_as_float(r[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[pb * 2 + half]);
        ++part;
      }
      const int nc = n0 + c_base;
      if (sg.nseg > 1) {
        // Part of a split tile: publish this warp's 32 x 128 partial sums; the
        // warp that completes the tile's count adds all parts in order.  The
        // layout is private to this kernel and lane-major (float4 j of lane l
        // at [j][l]), so every store and load of a warp is 512 contiguous
        // bytes; the warp of the same role reads it back.
        const int st = sg.tile - p.whole_tiles;
        auto slot = [&](int q) {
          return reinterpret_cast<float4 *>(p.partials) +
                 (((size_t)st * p.max_seg + q) * kF8EpiWarps + (warp - 4)) * (kCols / 4) * 32 + lane;
        };
        float4 *mine = slot(sg.seg);
#pragma unroll
        for (int j = 0; j < kCols / 4; ++j)
          mine[j * 32] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        __threadfence();
        __syncwarp();
        int done = 0;
        int *counter = p.tile_counters + (size_t)st * kF8EpiWarps + (warp - 4);
        if (lane == 0) done = atomicAdd(counter, 1);
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done != sg.nseg - 1) continue;  // another part finishes this tile
        __threadfence();
#pragma unroll
        for (int j = 0; j < kCols; ++j) acc[j] = 0.0f;
        for (int q = 0; q < sg.nseg; ++q) {
          const float4 *src = slot(q);
#pragma unroll
          for (int j = 0; j < kCols / 4; ++j) {
            const float4 v = __ldcg(src + j * 32);
            acc[4 * j] += v.x;
            acc[4 * j + 1] += v.y;
            acc[4 * j + 2] += v.z;
            acc[4 * j + 3] += v.w;
          }
        }
        if (lane == 0) *counter = 0;  // ready for the next launch
      }
      // Final scale in place (rows mode: token x weight-row scale; rows past
      // M have a zero token scale and are not stored).
      if (!kBlocks) {
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          const float ws = (nc + j < p.N) ? __ldg(p.w_scale + n_base + nc + j) : 0.0f;
          acc[j] = acc[j] * (as * ws);
        }
      }
      if (p.tma_store) {
        // The warp's 32 rows x 128 columns leave as 128-byte-wide boxes (64
        // bf16 or 32 f32 columns) through its own staging box: each lane
        // writes its row (16-byte chunks XOR-swizzled by row, the 128-byte
        // swizzle), then one lane issues the tiled store, which clips rows
        // past M and columns past N.  Every lane takes every step.
        const int row0 = m0 + qd * 32;
        if (row0 >= p.M) continue;  // warp-uniform
        uint8_t *box = sOut + (warp - 4) * kF8OutBoxBytes;
        uint8_t *row_s = box + lane * 128;
        auto store_box = [&](int col) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (col < p.N) tma_store_2d(&tmap_y, box, col, row0);
            bulk_commit_group();
          }
        };
        if (p.y_bf16) {
#pragma unroll
          for (int bx = 0; bx < 2; ++bx) {  // 64 columns per box
            if (lane == 0) bulk_wait_read_all();  // the previous box has left the staging
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const int j = bx * 64 + 8 * q;
              uint4 pk;
              pk.x = pack_bf16x2(acc[j], acc[j + 1]);
              pk.y = pack_bf16x2(acc[j + 2], acc[j + 3]);
              pk.z = pack_bf16x2(acc[j + 4], acc[j + 5]);
              pk.w = pack_bf16x2(acc[j + 6], acc[j + 7]);
              *reinterpret_cast<uint4 *>(row_s + ((q ^ (lane & 7)) * 16)) = pk;
            }
            store_box(nc + bx * 64);
          }
        } else {
#pragma unroll
          for (int bx = 0; bx < 4; ++bx) {  // 32 columns per box
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const int j = bx * 32 + 4 * q;
              *reinterpret_cast<float4 *>(row_s + ((q ^ (lane & 7)) * 16)) =
                  make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
            }
            store_box(nc + bx * 32);
          }
        }
        continue;
      }
      if (row >= p.M) continue;  // direct stores only below: no warp-collective step follows
      const long long off = (long long)row * p.ldy + nc;
      const bool full_cols = nc + kCols <= p.N;
      if (p.y_bf16) {
        __nv_bfloat16 *yp = reinterpret_cast<__nv_bfloat16 *>(p.y) + off;
        if (full_cols && (reinterpret_cast<uintptr_t>(yp) & 15) == 0) {
#pragma unroll
          for (int j = 0; j < kCols; j += 8) {
            uint4 pk;
            pk.x = pack_bf16x2(acc[j], acc[j + 1]);
            pk.y = pack_bf16x2(acc[j + 2], acc[j + 3]);
            pk.z = pack_bf16x2(acc[j + 4], acc[j + 5]);
            pk.w = pack_bf16x2(acc[j + 6], acc[j + 7]);
            *reinterpret_cast<uint4 *>(yp + j) = pk;
          }
        } else {
#pragma unroll
          for (int j = 0; j < kCols; ++j)
            if (nc + j < p.N) yp[j] = __float2bfloat16_rn(acc[j]);
        }
      } else {
        float *yp = reinterpret_cast<float *>(p.y) + off;
        if (full_cols && (reinterpret_cast<uintptr_t>(yp) & 15) == 0) {
#pragma unroll
          for (int j = 0; j < kCols; j += 4)
            *reinterpret_cast<float4 *>(yp + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < kCols; ++j)
            if (nc + j < p.N) yp[j] = acc[j];
        }
      }
    }
    // Stores in flight read this CTA's shared memory: complete them before exit.
    if (lane == 0 && p.tma_store) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kF8TmemCols);
  }
}

}  // namespace fpb

// ---- host side -------------------------------------------------------------------------
namespace fpb {

static int fp8_check_layout(size_t rows, size_t cols, size_t block_n, size_t block_k, size_t *n_scales) {
  if (block_n == 0 && block_k == 0) {
    *n_scales = rows;
  } else {
    if (block_n == 0 || block_k == 0 || rows % block_n != 0 || cols % block_k != 0)
      return fail(FPB_ERR_FORMAT, "invalid FP8 scale grid");  // weights/fp8.rs:39-46
    *n_scales = (rows / block_n) * (cols / block_k);
  }
  if (rows == 0 || cols == 0 || cols % 32 != 0)
    return fail(FPB_ERR_FORMAT, "invalid FP8 matrix or scales");  // weights/fp8.rs:91-98
  if (block_n > 0x7fffffff || block_k > 0x7fffffff) return fail(FPB_ERR_UNSUPPORTED, "FP8 block too large");
  return FPB_OK;
}

static int fp8_check_scales_host(const float *scales, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(scales[i])) return fail(FPB_ERR_FORMAT, "invalid FP8 matrix or scales");
  return FPB_OK;
}

static int fp8_alloc(size_t rows, size_t cols, size_t bn, size_t bk, size_t n_scales, fpb_fp8_matrix **out) {
  auto *m = new (std::nothrow) fpb_fp8_matrix();
  if (!m) return fail(FPB_ERR_INVALID_ARGUMENT, "out of host memory");
  m->rows = rows;
  m->cols = cols;
  m->block_n = (int)bn;
  m->block_k = (int)bk;
  m->n_scales = n_scales;
  cudaGetDevice(&m->device);
  cudaError_t e = cudaMalloc(&m->bits, rows * cols);
  if (e == cudaSuccess) e = cudaMalloc(&m->scales, n_scales * sizeof(float));
  if (e != cudaSuccess) {
    cudaFree(m->bits);
    cudaFree(m->scales);
    delete m;
    return cuda_fail(e, "cudaMalloc(FP8 matrix)");
  }
  *out = m;
  return FPB_OK;
}

// Raises a kernel's dynamic shared-memory limit once per device.
template <typename K>
static int raise_smem_once(K kernel, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<int, const void *>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  const void *key = reinterpret_cast<const void *>(kernel);
  if (std::find(done.begin(), done.end(), std::make_pair(dev, key)) != done.end()) return FPB_OK;
  FPB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.push_back({dev, key});
  return FPB_OK;
}

static int fp8_quantize_impl(const void *w, int dtype, size_t rows, size_t cols, size_t bn, size_t bk,
                             uint8_t *bits, float *scales, cudaStream_t s) {
  size_t n_scales = 0;
  int st = fp8_check_layout(rows, cols, bn, bk, &n_scales);
  if (st) return st;
  if (dtype != FPB_F32 && dtype != FPB_BF16) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_quantize: dtype");
  const bool row_mode = bn == 0 && bk == 0;
  const int ibn = row_mode ? 1 : (int)bn, ibk = row_mode ? (int)cols : (int)bk;
  if (ibk % 4 != 0) return fail(FPB_ERR_SHAPE, "fpb_fp8_quantize: block_k %d not a multiple of 4", ibk);
  if ((size_t)ibn * ibk > 0x7fffffffu || n_scales > 0x7fffffffu)
    return fail(FPB_ERR_UNSUPPORTED, "fpb_fp8_quantize: too many elements per block or blocks");
  if (dtype == FPB_F32)
    fp8_quantize_kernel<float><<<(unsigned)n_scales, 256, 0, s>>>(static_cast<const float *>(w), cols, ibn, ibk,
                                                                  bits, scales);
  else
    fp8_quantize_kernel<__nv_bfloat16><<<(unsigned)n_scales, 256, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(w), cols, ibn, ibk, bits, scales);
  FPB_LAUNCH_CHECK("fp8_quantize_kernel");
  return FPB_OK;
}

static int fp8_prepare(fpb_fp8_matrix *w) {
  if (w->tmap_valid) return FPB_OK;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (w->tmap_valid) return FPB_OK;
  int st = encode_rows_u8(reinterpret_cast<CUtensorMap *>(w->tmap), w->bits, w->rows, w->cols, kF8BN);
  if (st) return st;
  w->tmap_valid = true;
  return FPB_OK;
}

// Stream-K schedule of a dense GEMM: grid, parts per tile at most, bytes of
// partial sums and counters.
struct F8Split {
  int ctas, whole, max_seg;
  long long tail_kb;
  bool split;
  size_t partial_bytes, counter_bytes;
};
// Whole tiles in waves over the SMs.  A GEMM of less than one wave of tiles
// has its K blocks split evenly over the SMs instead (stream-K).  Splitting
// only the last partial wave of a larger GEMM is supported by the kernel
// (whole_tiles > 0) but not planned: the promotion epilogue makes each
// partial tile's fix-up cost more than the wave tail it removes (config 1,
// 224 tiles: 46.1 us whole, 51.9 us with the 76-tile tail split).
static F8Split fp8_split_plan(size_t m, size_t n_rows, size_t k) {
  const size_t tiles = ((m + kF8Tile - 1) / kF8Tile) * ((n_rows + kF8BN - 1) / kF8BN);
  const size_t kb = (k + kF8Tile - 1) / kF8Tile;
  const size_t sms = (size_t)std::max(1, sm_count());
  F8Split sp{};
  sp.ctas = (int)std::max<size_t>(1, std::min(tiles, sms));
  sp.whole = (int)tiles;
  const size_t whole = tiles >= sms ? (tiles / sms) * sms : 0;
  const size_t tail = tiles - whole, tail_kb = tail * kb;
  if (whole || tail_kb < 2) return sp;
  const size_t ctas = std::min(sms, tail_kb);
  const size_t range = tail_kb / ctas;  // shortest CTA range
  sp.ctas = (int)ctas;
  sp.whole = (int)whole;
  sp.tail_kb = (long long)tail_kb;
  sp.split = true;
  sp.max_seg = (int)std::min<size_t>((kb + range - 1) / range + 1, kb);
  sp.partial_bytes = tail * (size_t)sp.max_seg * kF8Tile * kF8BN * sizeof(float);
  sp.counter_bytes = tail * kF8EpiWarps * sizeof(int);
  return sp;
}

static int fp8_gemm_launch(fpb_fp8_matrix *w, const uint8_t *a_bits, const float *a_scale, size_t m,
                           size_t n_base, size_t n_rows, const int32_t *tile_experts, void *y, int y_dtype,
                           cudaStream_t s, void *split_ws = nullptr, size_t split_bytes = 0) {
  if (y_dtype != FPB_F32 && y_dtype != FPB_BF16) return fail(FPB_ERR_INVALID_ARGUMENT, "FP8 GEMM: dtype");
  const bool blocks = !(w->block_n == 0 && w->block_k == 0);
  if (blocks && (w->block_n % kF8Tile != 0 || w->block_k % kF8Tile != 0))
    return fail(FPB_ERR_UNSUPPORTED, "FP8 GEMM: block scales of %dx%d (need multiples of 128)", w->block_n,
                w->block_k);
  if (w->cols % 16 != 0) return fail(FPB_ERR_SHAPE, "FP8 GEMM: cols %zu not a multiple of 16", w->cols);
  if (m == 0 || m > (size_t)65535 * kF8Tile || w->rows > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "FP8 GEMM: m = %zu", m);
  int st = fp8_prepare(w);
  if (st) return st;
  CUtensorMap tmap_a;
  if ((st = encode_rows_u8(&tmap_a, a_bits, m, w->cols, kF8Tile))) return st;
  auto kernel = blocks ? fp8_gemm_kernel<true> : fp8_gemm_kernel<false>;
  if ((st = raise_smem_once(kernel, (int)kF8Smem))) return st;
  Fp8GemmParams p{};
  p.a_scale = a_scale;
  p.w_scale = w->scales;
  p.y = y;
  p.ldy = (long long)n_rows;
  p.y_bf16 = y_dtype == FPB_BF16;
  p.M = (int)m;
  p.N = (int)n_rows;
  p.n_base = (int)n_base;
  p.kb_count = (int)((w->cols + kF8Tile - 1) / kF8Tile);
  p.bn = w->block_n;
  p.bk = w->block_k;
  p.ws_cols = blocks ? (int)(w->cols / w->block_k) : 0;
  p.error = device_error_ptr();
  p.tile_experts = tile_experts;
  p.n_experts = tile_experts ? (int)(w->rows / n_rows) : 0;
  p.m_tiles = (int)((m + kF8Tile - 1) / kF8Tile);
  p.tiles = p.m_tiles * (int)((n_rows + kF8BN - 1) / kF8BN);
  // Whole tiles, one persistent CTA per SM (grouped: one CTA per tile, so
  // that a CTA whose row tile is dead can leave at once).
  p.ctas = tile_experts ? p.tiles : std::min(p.tiles, std::max(1, sm_count()));
  p.whole_tiles = p.tiles;
  p.total_kb = 0;
  p.max_seg = 1;
  const F8Split sp = fp8_split_plan(m, n_rows, w->cols);
  // With a workspace, the last partial wave of tiles is split along K.
  if (!tile_experts && sp.split && split_ws && split_bytes >= sp.partial_bytes + sp.counter_bytes) {
    p.ctas = sp.ctas;
    p.whole_tiles = sp.whole;
    p.total_kb = sp.tail_kb;
    p.max_seg = sp.max_seg;
    p.partials = static_cast<float *>(split_ws);
    p.tile_counters = reinterpret_cast<int *>(static_cast<uint8_t *>(split_ws) + sp.partial_bytes);
    FPB_CUDA_TRY(cudaMemsetAsync(p.tile_counters, 0, sp.counter_bytes, s));
  }
  CUtensorMap tmap_y;
  std::memset(&tmap_y, 0, sizeof(tmap_y));
  p.tma_store = encode_store_map(&tmap_y, y, p.y_bf16, m, n_rows, (uint64_t)p.ldy, 32, 0);
  launch_pdl(kernel, p.ctas, kF8Threads, kF8Smem, s, tmap_a, *reinterpret_cast<const CUtensorMap *>(w->tmap), tmap_y, p);
  FPB_LAUNCH_CHECK("fp8_gemm_kernel");
  return FPB_OK;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace fpb

using namespace fpb;

extern "C" int fpb_fp8_validate(size_t bits_len, const float *scales, size_t scales_len, size_t rows, size_t cols,
                                size_t block_n, size_t block_k) {
  size_t n_scales = 0;
  if (block_n == 0 && block_k == 0 && scales_len != rows)
    return fail(FPB_ERR_FORMAT, "FP8 row scales must have one value per row");  // weights/fp8.rs:63-65
  int st = fp8_check_layout(rows, cols, block_n, block_k, &n_scales);
  if (st) return st;
  if (scales_len != n_scales) return fail(FPB_ERR_FORMAT, "invalid FP8 scale grid");
  if (bits_len != rows * cols) return fail(FPB_ERR_FORMAT, "invalid FP8 matrix or scales");
  if (!scales && n_scales) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_validate: null scales");
  return fp8_check_scales_host(scales, n_scales);
}

extern "C" int fpb_fp8_matrix_create(const uint8_t *bits, const float *scales, size_t rows, size_t cols,
                                     size_t block_n, size_t block_k, void *stream, fpb_fp8_matrix **out) {
  if (!bits || !scales || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_matrix_create: null pointer");
  *out = nullptr;
  size_t n_scales = 0;
  int st = fp8_check_layout(rows, cols, block_n, block_k, &n_scales);
  if (st) return st;
  if ((st = fp8_check_scales_host(scales, n_scales))) return st;
  fpb_fp8_matrix *m = nullptr;
  if ((st = fp8_alloc(rows, cols, block_n, block_k, n_scales, &m))) return st;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(m->bits, bits, rows * cols, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->scales, scales, n_scales * sizeof(float), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    fpb_fp8_matrix_destroy(m);
    return cuda_fail(e, "fpb_fp8_matrix_create upload");
  }
  *out = m;
  return FPB_OK;
}

extern "C" int fpb_fp8_matrix_create_device(const uint8_t *bits, const float *scales, size_t rows, size_t cols,
                                            size_t block_n, size_t block_k, void *stream, fpb_fp8_matrix **out) {
  if (!bits || !scales || !out)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_matrix_create_device: null pointer");
  *out = nullptr;
  size_t n_scales = 0;
  int st = fp8_check_layout(rows, cols, block_n, block_k, &n_scales);
  if (st) return st;
  std::vector<float> host(n_scales);
  cudaStream_t s = as_stream(stream);
  FPB_CUDA_TRY(cudaMemcpyAsync(host.data(), scales, n_scales * sizeof(float), cudaMemcpyDeviceToHost, s));
  FPB_CUDA_TRY(cudaStreamSynchronize(s));
  if ((st = fp8_check_scales_host(host.data(), n_scales))) return st;
  fpb_fp8_matrix *m = nullptr;
  if ((st = fp8_alloc(rows, cols, block_n, block_k, n_scales, &m))) return st;
  cudaError_t e = cudaMemcpyAsync(m->bits, bits, rows * cols, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->scales, scales, n_scales * sizeof(float), cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    fpb_fp8_matrix_destroy(m);
    return cuda_fail(e, "fpb_fp8_matrix_create_device copy");
  }
  *out = m;
  return FPB_OK;
}

extern "C" int fpb_fp8_matrix_destroy(fpb_fp8_matrix *m) {
  if (!m) return FPB_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != m->device) cudaSetDevice(m->device);
  cudaFree(m->bits);
  cudaFree(m->scales);
  if (prev != m->device) cudaSetDevice(prev);
  delete m;
  return FPB_OK;
}

extern "C" int fpb_fp8_matrix_shape(const fpb_fp8_matrix *m, size_t *rows, size_t *cols, size_t *block_n,
                                    size_t *block_k) {
  if (!m) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_matrix_shape: null matrix");
  if (rows) *rows = m->rows;
  if (cols) *cols = m->cols;
  if (block_n) *block_n = (size_t)m->block_n;
  if (block_k) *block_k = (size_t)m->block_k;
  return FPB_OK;
}

extern "C" int fpb_fp8_matrix_download(const fpb_fp8_matrix *m, uint8_t *bits, float *scales, void *stream) {
  if (!m || !bits || !scales) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_matrix_download: null pointer");
  cudaStream_t s = as_stream(stream);
  FPB_CUDA_TRY(cudaMemcpyAsync(bits, m->bits, m->rows * m->cols, cudaMemcpyDeviceToHost, s));
  FPB_CUDA_TRY(cudaMemcpyAsync(scales, m->scales, m->n_scales * sizeof(float), cudaMemcpyDeviceToHost, s));
  FPB_CUDA_TRY(cudaStreamSynchronize(s));
  return FPB_OK;
}

extern "C" int fpb_fp8_quantize(const void *w, int dtype, size_t rows, size_t cols, size_t block_n, size_t block_k,
                                uint8_t *bits, float *scales, void *stream) {
  if (!w || !bits || !scales) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_quantize: null pointer");
  return fp8_quantize_impl(w, dtype, rows, cols, block_n, block_k, bits, scales, as_stream(stream));
}

extern "C" size_t fpb_fp8_gemm_workspace_bytes(size_t m, size_t k) { return align256(m * k) + align256(4 * m); }

extern "C" size_t fpb_fp8_gemm_split_bytes(size_t m, size_t k, size_t n) {
  const F8Split sp = fp8_split_plan(m, n, k);
  return align256(sp.partial_bytes + sp.counter_bytes);
}

extern "C" int fpb_fp8_gemm_q(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const uint8_t *a_bits,
                              const float *a_scales, size_t m, void *y, int y_dtype, void *stream) {
  if (!w || !a_bits || !a_scales || !y) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_gemm_q: null pointer");
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_gemm_q: row range [%zu, %zu) outside %zu rows", row_begin, row_end, w->rows);
  if (row_begin % kF8Tile != 0)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_gemm_q: first row %zu not a multiple of 128", row_begin);
  if (w->block_n && (row_begin % w->block_n || row_end % w->block_n))  // gemm/mod.rs:596-599
    return fail(FPB_ERR_SHAPE, "fpb_fp8_gemm_q: rows [%zu, %zu) not aligned to block_n %d", row_begin, row_end,
                w->block_n);
  return fp8_gemm_launch(w, a_bits, a_scales, m, row_begin, row_end - row_begin, nullptr, y, y_dtype,
                         as_stream(stream));
}

extern "C" int fpb_fp8_gemm_q_split(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const uint8_t *a_bits,
                                    const float *a_scales, size_t m, void *y, int y_dtype, void *split_ws,
                                    size_t split_bytes, void *stream) {
  if (!w || !a_bits || !a_scales || !y) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_gemm_q_split: null pointer");
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows || row_begin % kF8Tile ||
      (w->block_n && (row_begin % w->block_n || row_end % w->block_n)))
    return fpb_fp8_gemm_q(w, row_begin, row_end, a_bits, a_scales, m, y, y_dtype, stream);  // its errors
  if (split_ws && (reinterpret_cast<uintptr_t>(split_ws) & 255))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_gemm_q_split: workspace must be 256-byte aligned");
  return fp8_gemm_launch(w, a_bits, a_scales, m, row_begin, row_end - row_begin, nullptr, y, y_dtype,
                         as_stream(stream), split_ws, split_bytes);
}

extern "C" int fpb_fp8_gemm(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                            size_t m, void *y, int y_dtype, void *workspace, size_t workspace_bytes, void *stream) {
  if (!w || !x || !y || !workspace) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_gemm: null pointer");
  if (workspace_bytes < fpb_fp8_gemm_workspace_bytes(m, w->cols) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FPB_ERR_WORKSPACE, "fpb_fp8_gemm: workspace must be 256-byte aligned and %zu bytes",
                fpb_fp8_gemm_workspace_bytes(m, w->cols));
  uint8_t *a_bits = static_cast<uint8_t *>(workspace);
  float *a_scales = reinterpret_cast<float *>(a_bits + align256(m * w->cols));
  cudaStream_t s = as_stream(stream);
  int st = fp8_quantize_impl(x, x_dtype, m, w->cols, 0, 0, a_bits, a_scales, s);
  if (st) return st;
  // Room past the activations (fpb_fp8_gemm_split_bytes): the stream-K partial sums.
  const size_t base = fpb_fp8_gemm_workspace_bytes(m, w->cols);
  return fpb_fp8_gemm_q_split(w, row_begin, row_end, a_bits, a_scales, m, y, y_dtype,
                              static_cast<uint8_t *>(workspace) + base, workspace_bytes - base, stream);
}

extern "C" int fpb_fp8_grouped_gemm_q(fpb_fp8_matrix *w, const uint8_t *a_bits, const float *a_scales,
                                      size_t padded_rows, const int32_t *tile_experts, size_t rows_per_expert,
                                      void *y, int y_dtype, void *stream) {
  if (!w || !a_bits || !a_scales || !tile_experts || !y)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_grouped_gemm_q: null pointer");
  if (padded_rows == 0 || padded_rows % kF8Tile)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_grouped_gemm_q: padded_rows %zu not a positive multiple of 128", padded_rows);
  if (rows_per_expert == 0 || rows_per_expert % kF8Tile || w->rows % rows_per_expert)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_grouped_gemm_q: rows_per_expert %zu must be a multiple of 128 dividing %zu",
                rows_per_expert, w->rows);
  if (w->block_n && rows_per_expert % w->block_n)  // gemm/mod.rs:675-677
    return fail(FPB_ERR_SHAPE, "fpb_fp8_grouped_gemm_q: rows_per_expert not a multiple of block_n");
  return fp8_gemm_launch(w, a_bits, a_scales, padded_rows, 0, rows_per_expert, tile_experts, y, y_dtype,
                         as_stream(stream));
}

// ---- the reference's activation semantics (gemm/mod.rs:87-100, 155-168) -----------------
// fp8_gemm_kernel multiplies the f32 activations by the weight block scale,
// splits them into bf16 hi + lo and multiplies both by the e4m3 weights as
// bf16 (exact); fp8_rows_gemm_kernel does the same without the scale and
// multiplies the f32 sums by the row scale.  Here the weights go to bf16 in
// the caller's workspace: with row scales the exact e4m3 values (the row
// scale is applied in the epilogue); with block scales w * s split into hi
// and lo (the scale folded into the weights instead of the activations: the
// same product to within the bf16 hi + lo precision, about 2^-16 relative).
// The GEMM is the tcgen05 bf16 mode of the NVFP4 kernel, one pass per (A, B)
// pair: hi.W (+ lo.W) with row scales; hi.Whi + hi.Wlo + lo.Whi with blocks.
namespace fpb {
__global__ void fp8_to_bf16_kernel(const uint8_t *bits, const float *scales, size_t rows, size_t cols, int block_n,
                                   int block_k, size_t scale_cols, __nv_bfloat16 *hi, __nv_bfloat16 *lo) {
  pdl_enter();
  const size_t n = rows * cols, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = e4m3_to_f32(bits[i]);
    if (!lo) {
      hi[i] = __float2bfloat16_rn(v);  // exact: e4m3 values are bf16 values
      continue;
    }
    const size_t r = i / cols, c = i % cols;
    const float w = v * scales[(r / block_n) * scale_cols + c / block_k];
    const __nv_bfloat16 h = __float2bfloat16_rn(w);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(w - __bfloat162float(h));
  }
}

static unsigned f8_grid_for(size_t n) {
  size_t g = (n + 255) / 256, cap = (size_t)sm_count() * 16;
  return (unsigned)std::max<size_t>(1, std::min(g, cap));
}
}  // namespace fpb

extern "C" size_t fpb_fp8_gemm_hilo_workspace_bytes(size_t m, size_t rows, size_t k, int x_dtype, int blocks) {
  return hilo_workspace_bytes(m, k, x_dtype) + (blocks ? 2 : 1) * align256(rows * k * 2) + 256;
}

extern "C" int fpb_fp8_gemm_hilo(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                                 size_t m, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                                 void *stream) {
  if (!w || !x || !y || !workspace) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_gemm_hilo: null pointer");
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_gemm_hilo: row range [%zu, %zu) outside %zu rows", row_begin, row_end,
                w->rows);
  const bool blocks = w->block_n != 0;
  if (blocks && row_begin % (size_t)w->block_n)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_gemm_hilo: row_begin %zu not a multiple of block_n %d", row_begin,
                w->block_n);
  if (m == 0 || m > (size_t)65535 * 128) return fail(FPB_ERR_SHAPE, "fpb_fp8_gemm_hilo: m = %zu", m);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_gemm_hilo: dtype");
  if (w->cols % 8) return fail(FPB_ERR_SHAPE, "fpb_fp8_gemm_hilo: cols %zu not a multiple of 8", w->cols);
  const size_t rows = row_end - row_begin, k = w->cols;
  const size_t need = fpb_fp8_gemm_hilo_workspace_bytes(m, rows, k, x_dtype, blocks);
  if (workspace_bytes < need)
    return fail(FPB_ERR_WORKSPACE, "fpb_fp8_gemm_hilo: workspace %zu < %zu bytes", workspace_bytes, need);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) || (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_gemm_hilo: workspace 256-byte and x 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const void *hi, *lo;
  size_t used = 0;
  int st = hilo_activations(x, x_dtype, m, k, ws, &hi, &lo, &used, s);
  if (st) return st;
  __nv_bfloat16 *whi = reinterpret_cast<__nv_bfloat16 *>(ws + used);
  __nv_bfloat16 *wlo = blocks ? reinterpret_cast<__nv_bfloat16 *>(ws + used + align256(rows * k * 2)) : nullptr;
  const float *sc = blocks ? w->scales + (row_begin / w->block_n) * (k / w->block_k) : w->scales;
  launch_pdl(fp8_to_bf16_kernel, f8_grid_for(rows * k), 256, 0, s, w->bits + row_begin * k, sc, rows, k,
             w->block_n, w->block_k, blocks ? k / w->block_k : 0, whi, wlo);
  FPB_LAUNCH_CHECK("fp8_to_bf16_kernel");
  F16Gemm g{};
  g.m = m;
  g.n = rows;
  g.k = k;
  g.a[0] = hi;
  g.a[1] = lo;
  g.b[0] = whi;
  g.b[1] = wlo;
  if (blocks) {
    // hi.Whi, hi.Wlo, then lo.Whi (lo.Wlo is below f32 rounding of the sum)
    g.passes = lo ? 3 : 2;
    g.a_sel[0] = 0, g.b_sel[0] = 0;
    g.a_sel[1] = 0, g.b_sel[1] = 1;
    g.a_sel[2] = 1, g.b_sel[2] = 0;
    g.b_globals = nullptr;
  } else {
    g.passes = lo ? 2 : 1;
    g.a_sel[0] = 0, g.b_sel[0] = 0;
    g.a_sel[1] = 1, g.b_sel[1] = 0;
    g.b_globals = w->scales + row_begin;
  }
  g.y = y;
  g.y_bf16 = y_dtype == FPB_BF16;
  return run_f16_gemm(g, s);
}
