// NVFP4 decode GEMV, dense and expert (crates/firepit-kernels/src/gemv/nvfp4.rs).
//
// y[b, r] = g[r] * sum_k E2M1[w[r,k]] * e4m3(s[r,k/16]) * x[b,k]
//
// Design.  The path is HBM-bound (3.5 FLOP/B); the per-element arithmetic
// must stay below the time the element takes to arrive, and the kernel has no
// phase that waits on anything but its own loads.
//  * A CTA has up to 16 warps.  Every warp owns a fixed slice of K (C chunks
//    of 128 columns) for the whole kernel, so its share of x is loaded once,
//    straight into registers as ready-made MMA B fragments; there is no
//    shared-memory staging and no barrier before the first MMA.
//  * Weights stream with 128-bit non-coherent loads that do not allocate in
//    L1: per chunk a warp covers 16 rows x 128 columns, lanes 4g..4g+3 reading
//    rows g and g+8.  The next row block's loads are issued before the current
//    one is computed.
//  * Codes become f16 with `cvt.rn.f16x2.e2m1x2` and are multiplied by their
//    e4m3 block scale in f16.  e2m1 * e4m3 is exact in f16 (at most six
//    significant bits, magnitude in [2^-10, 2688]), so the dequantized weight
//    equals the reference's E2M1 * scale exactly.
//  * The dot products run on the tensor cores as m16n8k16 MMAs with f32
//    accumulation (two independent accumulator chains): weights are the A
//    operand, up to 8 input rows per MMA the B operand.  The MMA's k order is
//    a permutation of the physical columns shared by A and B, which a dot
//    product does not see.
//  * To keep x exact in f16, each warp scales its slice of each input row by
//    a power of two that puts the slice's largest magnitude in [2^14, 2^15)
//    and removes it (exactly) from its partial sums.  bf16 inputs are then
//    exact, except elements below amax * 2^-29, which round to f16 subnormals
//    (absolute error < amax * 2^-40).  f32 inputs are split into f16 hi and
//    lo parts (22 significant bits) and take two MMAs, the f16 counterpart of
//    the reference's bf16 hi/lo split (gemm/nvfp4.rs:33-36).
//  * The warps sharing a row block add their partials in shared memory (one
//    barrier per row block, double-buffered), then the sum times the row
//    global is stored as f32 or bf16.
//  * Programmatic dependent launch: the register variant waits for the
//    previous kernel before it reads anything (x, and in expert mode the
//    expert ids that pick the weight rows).  The streaming variant (dense
//    only) issues its weight copies before the wait: weights are immutable
//    once their handle exists (handle creation synchronises its stream).
#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "nvfp4_matrix.cuh"
#include "sm100.cuh"

namespace fpb {

struct GemvArgs {
  const uint8_t *packed;  // row 0 of the addressed rows
  const uint8_t *scales;
  const float *globals;
  const void *x;
  void *y;
  const int32_t *expert_ids;  // null for dense
  long long x_slot_stride;    // elements between the input rows of consecutive slots (or slot groups)
  int x_div;                  // slots per input row: slot s reads input row s / x_div (1: one row per slot)
  long long y_slot_stride;    // elements between the output rows of consecutive slots
  long long y_batch_stride;   // elements between output rows of consecutive batch rows
  int rows;                   // rows per slot
  int K;                      // columns this launch covers (a slice of k_pitch when K > 4096)
  int k_pitch;                // columns of a full weight row and of an x row
  int accumulate;             // 1: y (f32) += this slice's sums
  int batch;
  int n_experts;  // expert mode: valid ids are [0, n_experts)
  int chunks;     // ceil(K / 128)
  int nrb;        // ceil(rows / 16)
  int wk;         // warps per row block (K slices)
  int g;          // row blocks per CTA iteration
  int y_bf16;
};

__device__ __forceinline__ uint4 ldg_stream_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ldg_u16(const void *p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Power-of-two exponent F for a slice whose largest magnitude has the given
// float bits: amax * 2^F lies in [2^14, 2^15).  Clamped so that 2^F and 2^-F
// are both normal floats.
__device__ __forceinline__ int prescale_exponent(uint32_t amax_bits) {
  int ef = (int)(amax_bits >> 23) & 0xff;
  int F = 141 - ef;
  return max(-126, min(126, F));
}

// Loads 4 consecutive input values (bf16 or f32) as floats.
template <bool F32>
__device__ __forceinline__ void load_x4(const void *x, long long off, float v[4]) {
  if (F32) {
    float4 f = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + off);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else {
    uint2 b = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(x) + off);
    v[0] = __uint_as_float(b.x << 16); v[1] = __uint_as_float(b.x & 0xffff0000u);
    v[2] = __uint_as_float(b.y << 16); v[3] = __uint_as_float(b.y & 0xffff0000u);
  }
}

template <int C, int NG, bool XLO>
__global__ void __launch_bounds__(512, 1) gemv_nvfp4_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  float4 *red = reinterpret_cast<float4 *>(smem);  // [2][g][wk][NG][32]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int K = a.K, kb2 = a.k_pitch >> 1, kb16 = a.k_pitch >> 4;  // kb2 / kb16: row pitches
  const int chunks = a.chunks, batch = a.batch;
  const int wk_count = a.wk, g_count = a.g;
  const int wk = warp % wk_count, gi = warp / wk_count;
  const int c_begin = wk * C;
  const int slot = blockIdx.y;
  // The host launches exactly wk * g warps; any other block size would index
  // past the reduction buffer, so it does nothing (uniform for the CTA).
  if ((int)blockDim.x != wk_count * g_count * 32) return;
  // Register double-buffering of the next row block, except where the f32
  // hi/lo fragments already fill the register budget.
  constexpr bool kPrefetch = !(XLO && C >= 2);

  // Programmatic dependent launch: nothing this kernel reads may be written
  // by the previous kernel before this wait, and that includes the expert
  // ids (a router top-k launched just before writes them).
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  long long base_row = 0;
  bool slot_ok = true;
  if (a.expert_ids) {
    int e = a.expert_ids[slot];
    slot_ok = (e >= 0 && e < a.n_experts);
    base_row = (long long)(slot_ok ? e : 0) * a.rows;
  }
  const uint8_t *packed = a.packed + base_row * kb2;
  const uint8_t *scales = a.scales + base_row * kb16;
  const float *globals = a.globals + base_row;
  const long long x_off = (long long)(slot / a.x_div) * a.x_slot_stride;

  // Contiguous, balanced range of row-block groups for this CTA.
  const int total_groups = (a.nrb + g_count - 1) / g_count;
  const int grp_begin = (int)((long long)blockIdx.x * total_groups / gridDim.x);
  const int grp_end = (int)((long long)(blockIdx.x + 1) * total_groups / gridDim.x);
  const int iters = grp_end - grp_begin;

  // Loads one row block's codes and scales, and (for the warp that writes
  // the outputs) the row globals the epilogue multiplies by.
  auto load = [&](int it, uint4 (&w)[2][C], uint16_t (&s)[2][C], float (&gl)[2]) {
    int rb = (grp_begin + it) * g_count + gi;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int r = rb * 16 + g + 8 * h;
      bool row_ok = slot_ok && rb < a.nrb && r < a.rows;
      gl[h] = (row_ok && wk == 0) ? __ldg(globals + r) : 0.0f;
#pragma unroll
      for (int cc = 0; cc < C; ++cc) {
        int c = c_begin + cc;
        if (row_ok && c < chunks && (c * 128 + q * 32) < K) {
          w[h][cc] = ldg_stream_v4(packed + (long long)r * kb2 + c * 64 + q * 16);
          s[h][cc] = ldg_u16(scales + (long long)r * kb16 + c * 8 + 2 * q);
        } else {
          w[h][cc] = make_uint4(0, 0, 0, 0);
          s[h][cc] = 0;
        }
      }
    }
  };

  // ---- this warp's slice of x as B fragments, in registers -------------------
  // Lane (g, q) feeds batch rows n = ng*8 + g; for chunk cc and MMA j it holds
  // x[n][k0 + 4j .. k0 + 4j + 3] with k0 = c*128 + q*32.  The lane's 32
  // consecutive inputs of each chunk are loaded once with 16-byte loads (4
  // for bf16, 8 for f32), issued before the weight loads so that they are not
  // queued behind them.
  constexpr int kVec = XLO ? 8 : 4;
  uint4 raw[NG][C][kVec];
#pragma unroll
  for (int ng = 0; ng < NG; ++ng) {
    const int n = ng * 8 + g;
#pragma unroll
    for (int cc = 0; cc < C; ++cc) {
      const int k0 = (c_begin + cc) * 128 + q * 32;
      const bool ok = n < batch && k0 < K;
      const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const char *>(a.x) +
                                                         (x_off + (long long)n * a.k_pitch + k0) * (XLO ? 4 : 2));
#pragma unroll
      for (int v = 0; v < kVec; ++v) raw[ng][cc][v] = ok ? src[v] : make_uint4(0, 0, 0, 0);
    }
  }

  uint4 wcur[2][C];
  uint16_t scur[2][C];
  float gcur[2];
  if (iters > 0) load(0, wcur, scur, gcur);

  uint32_t xb[C][8][NG][2];
  uint32_t xl[XLO ? C : 1][8][NG][2];
  float unscale[NG];
#pragma unroll
  for (int ng = 0; ng < NG; ++ng) {
    const int n = ng * 8 + g;
    const bool n_ok = n < batch;
    uint32_t m = 0;
#pragma unroll
    for (int cc = 0; cc < C; ++cc) {
#pragma unroll
      for (int v = 0; v < kVec; ++v) {
        const uint4 r = raw[ng][cc][v];
        const uint32_t wv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (XLO) {
            m = max(m, wv[t] & 0x7fffffffu);
          } else {
            const uint32_t mag = wv[t] & 0x7fff7fffu;  // bf16 magnitudes order like their floats
            m = max(m, max(mag << 16, mag & 0xffff0000u));
          }
        }
      }
    }
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int F = prescale_exponent(m);
    const float up = __uint_as_float((uint32_t)(127 + F) << 23);
    unscale[ng] = __uint_as_float((uint32_t)(127 - F) << 23);
#pragma unroll
    for (int cc = 0; cc < C; ++cc) {
      const int k0 = (c_begin + cc) * 128 + q * 32;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
        if (n_ok && k0 < K) {
          float v[4];
          if (XLO) {
            const uint4 r4 = raw[ng][cc][j];
            v[0] = __uint_as_float(r4.x); v[1] = __uint_as_float(r4.y);
            v[2] = __uint_as_float(r4.z); v[3] = __uint_as_float(r4.w);
          } else {
            const uint4 r4 = raw[ng][cc][j >> 1];
            const uint32_t b0 = (j & 1) ? r4.z : r4.x, b1 = (j & 1) ? r4.w : r4.y;
            v[0] = __uint_as_float(b0 << 16); v[1] = __uint_as_float(b0 & 0xffff0000u);
            v[2] = __uint_as_float(b1 << 16); v[3] = __uint_as_float(b1 & 0xffff0000u);
          }
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = v[t] * up;
          h0 = pack_half2(v[0], v[1]);
          h1 = pack_half2(v[2], v[3]);
          if (XLO) {
            float2 f01 = __half22float2(*reinterpret_cast<__half2 *>(&h0));
            float2 f23 = __half22float2(*reinterpret_cast<__half2 *>(&h1));
            l0 = pack_half2(v[0] - f01.x, v[1] - f01.y);
            l1 = pack_half2(v[2] - f23.x, v[3] - f23.y);
          }
        }
        xb[cc][j][ng][0] = h0;
        xb[cc][j][ng][1] = h1;
        if (XLO) {
          xl[XLO ? cc : 0][j][ng][0] = l0;
          xl[XLO ? cc : 0][j][ng][1] = l1;
        }
      }
    }
  }
  // Unscale factors of the accumulator columns n = ng*8 + 2q (+1), held by
  // lanes 4*(2q) and 4*(2q+1).
  float us[NG][2];
#pragma unroll
  for (int ng = 0; ng < NG; ++ng) {
    us[ng][0] = __shfl_sync(0xffffffffu, unscale[ng], (2 * q) * 4);
    us[ng][1] = __shfl_sync(0xffffffffu, unscale[ng], (2 * q + 1) * 4);
  }

  // ---- stream the row blocks ---------------------------------------------------
  for (int it = 0; it < iters; ++it) {
    uint4 wnext[2][C];
    uint16_t snext[2][C];
    float gnext[2];
    if (kPrefetch && it + 1 < iters) load(it + 1, wnext, snext, gnext);

    float acc2[2][NG][4];
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
#pragma unroll
        for (int t = 0; t < 4; ++t) acc2[p][ng][t] = 0.0f;

#pragma unroll
    for (int cc = 0; cc < C; ++cc) {
      if (c_begin + cc >= chunks) continue;
      uint32_t s_lo[2], s_hi[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t sc = e4m3x2_to_f16x2(scur[hh][cc]);
        s_lo[hh] = __byte_perm(sc, sc, 0x1010);
        s_hi[hh] = __byte_perm(sc, sc, 0x3232);
      }
      const uint32_t w0[4] = {wcur[0][cc].x, wcur[0][cc].y, wcur[0][cc].z, wcur[0][cc].w};
      const uint32_t w1[4] = {wcur[1][cc].x, wcur[1][cc].y, wcur[1][cc].z, wcur[1][cc].w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        // word wi holds columns 8wi..8wi+7 of the lane's 32: MMAs 2wi, 2wi+1
        uint32_t f0[4], f1[4];
        e2m1x8_to_f16x8(w0[wi], f0);
        e2m1x8_to_f16x8(w1[wi], f1);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          f0[t] = hmul2(f0[t], wi < 2 ? s_lo[0] : s_hi[0]);
          f1[t] = hmul2(f1[t], wi < 2 ? s_lo[1] : s_hi[1]);
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * wi + jj;
#pragma unroll
          for (int ng = 0; ng < NG; ++ng) {
            mma_f16(acc2[jj][ng], f0[2 * jj], f1[2 * jj], f0[2 * jj + 1], f1[2 * jj + 1], xb[cc][j][ng][0],
                    xb[cc][j][ng][1]);
            if (XLO)
              mma_f16(acc2[jj][ng], f0[2 * jj], f1[2 * jj], f0[2 * jj + 1], f1[2 * jj + 1],
                      xl[XLO ? cc : 0][j][ng][0], xl[XLO ? cc : 0][j][ng][1]);
          }
        }
      }
    }

    // ---- cross-warp reduction and epilogue -----------------------------------
    const int buf = it & 1;
    float4 *rb_red = red + (size_t)buf * g_count * wk_count * NG * 32;
#pragma unroll
    for (int ng = 0; ng < NG; ++ng)
      rb_red[((gi * wk_count + wk) * NG + ng) * 32 + lane] =
          make_float4((acc2[0][ng][0] + acc2[1][ng][0]) * us[ng][0], (acc2[0][ng][1] + acc2[1][ng][1]) * us[ng][1],
                      (acc2[0][ng][2] + acc2[1][ng][2]) * us[ng][0], (acc2[0][ng][3] + acc2[1][ng][3]) * us[ng][1]);
    __syncthreads();
    const int rb = (grp_begin + it) * g_count + gi;
    if (wk == 0 && rb < a.nrb) {
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) {
        // All partial loads are independent (unrolled with predication).
        float4 part[16];
#pragma unroll
        for (int w = 0; w < 16; ++w)
          part[w] = w < wk_count ? rb_red[((gi * wk_count + w) * NG + ng) * 32 + lane]
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 sum = part[0];
#pragma unroll
        for (int w = 1; w < 16; ++w) {
          sum.x += part[w].x; sum.y += part[w].y; sum.z += part[w].z; sum.w += part[w].w;
        }
        const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          int r = rb * 16 + g + ((t >> 1) << 3);
          int n = ng * 8 + 2 * q + (t & 1);
          if (r < a.rows && n < batch) {
            float v = slot_ok ? vals[t] * gcur[t >> 1] : 0.0f;
            long long off = (long long)slot * a.y_slot_stride + (long long)n * a.y_batch_stride + r;
            if (a.accumulate) v += reinterpret_cast<const float *>(a.y)[off];  // f32 y: later K slices
            if (a.y_bf16)
              reinterpret_cast<__nv_bfloat16 *>(a.y)[off] = __float2bfloat16_rn(v);
            else
              reinterpret_cast<float *>(a.y)[off] = v;
          }
        }
      }
    }
    if (it + 1 < iters) {
      if (kPrefetch) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int cc = 0; cc < C; ++cc) {
            wcur[hh][cc] = wnext[hh][cc];
            scur[hh][cc] = snext[hh][cc];
          }
        gcur[0] = gnext[0];
        gcur[1] = gnext[1];
      } else {
        load(it + 1, wcur, scur, gcur);
      }
    }
  }
}

// ---- streaming variant: weights staged in shared memory ahead of the wait ----
//
// Dense GEMV with K % 128 == 0, K <= 4096, batch <= 8, over one or several
// matrices ("segments": each a row range of one matrix with its own x and y,
// all with the same K), or over device-indirect expert segments (MOE, see
// StreamMoe).  The segments' rows are laid end to end in a virtual row space;
// CTA c owns the contiguous virtual rows [c*rpc, (c+1)*rpc) (rpc a multiple
// of 4) and walks them in units of at most UR rows (16 or 32: one or two MMA
// row blocks, independent chains that share each x fragment) that never
// cross a segment.  Warp 0 issues the bulk copies of the CTA's first units
// (codes, factors and row globals, one contiguous copy each) into a ring of
// shared-memory stages before griddepcontrol.wait, so with dense segments the
// weights of launch i+1 stream from HBM while launch i computes (two CTAs fit
// on an SM).  After the wait each warp stages its K slice of the unit's x
// (f16, prescaled as in the register variant; again only when the segment's
// x changes; rows 16 mod 128 bytes apart, 16-byte slots swizzled so that the
// MMA's x reads are conflict-free) and runs the cvt / mul.f16x2 / m16n8k16
// arithmetic on every unit.  Partial sums of the 8 K slices meet in shared
// memory; the last warp to finish a unit (a shared counter) adds them, stores
// y and refills the stage with the unit S stages ahead.  Every warp walks the
// CTA's units itself (one iterator for the unit it computes, one S units
// ahead for refills), so no unit table is shared.  What bounds it: the
// per-unit chain of each warp (wait, decode, MMAs, partial sums, reduction,
// refill), not DRAM: per-row copies (two bulk copies a row) made the copy
// issue rate the limit, 8-row units were 1.43x slower than 16-row ones and
// one 16-warp CTA per SM 1.65x slower than two 8-warp CTAs.
struct StreamSeg {
  const uint8_t *packed;  // first addressed row
  const uint8_t *scales;
  const float *globals;
  const void *x;   // [batch, K]
  void *y;         // [batch, rows]
  long long vbeg;  // first virtual row
  int rows;
  int pad_;
};

constexpr int kStreamMaxSegs = 128;

// Device-indirect segments (the decode MoE GEMV): segment i is expert
// ids[i]'s rows_per_expert rows, for i < *count, read after the dependency
// wait.  seg[0] then holds the base pointers: expert 0's first row, x of
// segment 0 and y of segment 0.
struct StreamMoe {
  const int32_t *ids;    // [cap] expert ids of the segments
  const int32_t *count;  // live segments (device)
  int cap;
  int rpe;               // rows per expert = rows of every segment
  int n_experts;
  long long x_stride;    // input elements between consecutive segments' x
  long long y_stride;    // output elements between consecutive segments' y
};

template <int NSEG>
struct StreamArgs {
  StreamSeg seg[NSEG];
  StreamMoe moe;
  int nseg;
  int rpc;  // virtual rows per CTA (multiple of 4)
  long long total_rows;
  int *error;
  int K, batch;
  int stages;       // ring depth
  int wpitch;       // shared bytes per staged code row (64 mod 128)
  int spitch;       // shared bytes per staged factor row
  int scale_rows;   // 1: one copy per factor row; 0: one contiguous copy per unit
  int contig;       // 1: a unit's codes also arrive as one contiguous copy (pitch K/2)
  int stage_bytes;  // UR * wpitch + UR * spitch + max(64, 4 * UR)
  int xpitch;       // f16 elements per staged input row (16 mod 128 bytes)
  int y_bf16;
};

constexpr int kStreamWarps = 8;

// Position of input element k in its staged row.  Lane (g, q) of an MMA
// reads the 16 bytes at k = c*128 + q*32 + 8*wi of row g; with rows 16 mod
// 128 bytes apart and bit 4 of k flipped where bit 6 is set (q = 2, 3), the
// 8 lanes of each quarter-warp phase (rows g, g + 1, q = 0..3) read 8
// distinct 16-byte bank groups.
__device__ __forceinline__ int xswz(int k) { return k ^ (((k >> 6) & 1) << 4); }

__device__ __forceinline__ uint4 lds128(const void *p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(sm100::smem_u32(p)));
  return v;
}

__device__ __forceinline__ uint16_t lds16(const void *p) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(sm100::smem_u32(p)));
  return v;
}

// Position of the next unit of a CTA's virtual row range.  The segment's row
// count is cached so that the segment table (kernel parameters, read with a
// computed index) is consulted only when a unit starts a new segment.
struct UnitIter {
  int seg;       // segment of the next unit
  int row;       // its first row within the segment
  int seg_rows;  // rows of that segment
  long long v;   // its virtual row
};

struct Unit {
  int seg, row0, nrows;
};

// Takes the next unit (at most UR rows, within one segment and below v_hi);
// false once the range is exhausted.
template <int UR, bool MOE, int NSEG>
__device__ __forceinline__ bool next_unit(const StreamArgs<NSEG> &a, UnitIter &it, long long v_hi, Unit &u) {
  if (it.v >= v_hi) return false;
  while (it.row >= it.seg_rows) {
    ++it.seg;
    it.row = 0;
    it.seg_rows = MOE ? a.moe.rpe : a.seg[it.seg].rows;
  }
  u.seg = it.seg;
  u.row0 = it.row;
  u.nrows = (int)min((long long)min(UR, it.seg_rows - it.row), v_hi - it.v);
  it.row += u.nrows;
  it.v += u.nrows;
  return true;
}

// Smallest piece a unit's contiguous code copy is split into.
constexpr uint32_t kCopyPiece = 16384;

// Expert ids of device-indirect segments held in shared memory (the refill
// of a stage is on the warps' critical path; a global load there cost a
// round trip per unit).
constexpr int kMoeIdsShared = 1024;

// Issues (one warp) the copies of one unit of `u.nrows` rows (a multiple of
// 4, at most UR) into `stage`.
template <int UR, bool MOE, int NSEG>
__device__ __forceinline__ void stream_issue(const StreamArgs<NSEG> &a, uint8_t *stage, uint64_t *bar,
                                             const Unit &u, int lane, const int *ids_shared) {
  const uint32_t kb2 = (uint32_t)a.K >> 1, kb16 = (uint32_t)a.K >> 4;
  const uint8_t *packed, *scales;
  const float *globals;
  if (MOE) {
    int e = u.seg < kMoeIdsShared ? ids_shared[u.seg] : a.moe.ids[u.seg];
    if (e < 0 || e >= a.moe.n_experts) {  // a bad id reads expert 0 and is recorded
      if (lane == 0 && a.error) atomicCAS(a.error, 0, 203);
      e = 0;
    }
    const size_t r = (size_t)e * a.moe.rpe;
    packed = a.seg[0].packed + r * kb2;
    scales = a.seg[0].scales + r * kb16;
    globals = a.seg[0].globals + r;
  } else {
    const StreamSeg &sg = a.seg[u.seg];
    packed = sg.packed;
    scales = sg.scales;
    globals = sg.globals;
  }
  const int nrows = u.nrows, row0 = u.row0;
  if (lane == 0) sm100::mbar_arrive_expect_tx(bar, (uint32_t)nrows * (kb2 + kb16 + 4));
  __syncwarp();
  if (a.contig) {
    // a few row-aligned pieces of at least kCopyPiece bytes, issued by
    // different lanes: few copies a row, but more than one in flight
    const int pieces = max(1, min(8, (int)((uint32_t)nrows * kb2 / kCopyPiece)));
    const int rpp = (nrows + pieces - 1) / pieces;
    if (lane < pieces) {
      const int r0 = lane * rpp, r1 = min(nrows, r0 + rpp);
      if (r1 > r0)
        sm100::bulk_load(stage + (size_t)r0 * kb2, packed + (size_t)(row0 + r0) * kb2, (uint32_t)(r1 - r0) * kb2,
                         bar);
    }
  } else {
    for (int r = lane; r < nrows; r += 32)
      sm100::bulk_load(stage + r * a.wpitch, packed + (size_t)(row0 + r) * kb2, kb2, bar);
  }
  uint8_t *sc = stage + UR * a.wpitch;
  if (a.scale_rows) {
    for (int r = (lane + 16) & 31; r < nrows; r += 32)  // lanes 16.. start, spreading the issue
      sm100::bulk_load(sc + r * a.spitch, scales + (size_t)(row0 + r) * kb16, kb16, bar);
  } else if (lane == 16) {
    sm100::bulk_load(sc, scales + (size_t)row0 * kb16, (uint32_t)nrows * kb16, bar);
  }
  if (lane == 31) sm100::bulk_load(sc + UR * a.spitch, globals + row0, (uint32_t)nrows * 4, bar);
}

// MOE: the segments are device-indirect (StreamMoe): the expert ids and their
// count come from the previous kernel, so nothing is copied before the
// dependency wait, and each CTA's share of the rows is computed from the
// count after it.
template <bool XLO, int NSEG, int UR, bool MOE>
__global__ void __launch_bounds__(kStreamWarps * 32, 2)
    gemv_nvfp4_stream_kernel(const __grid_constant__ StreamArgs<NSEG> a) {
  constexpr int W = kStreamWarps;
  extern __shared__ __align__(16) unsigned char smem[];
  const int S = a.stages;
  uint8_t *stages = smem;
  __half *xh = reinterpret_cast<__half *>(smem + (size_t)S * a.stage_bytes);
  __half *xl = xh + (size_t)a.batch * a.xpitch;
  // Row blocks of 16 per unit (UR = 8: one block whose rows 8-15 are zero).
  constexpr int RB = UR >= 16 ? UR / 16 : 1;
  constexpr bool HALF = UR < 16;
  float4 *red = reinterpret_cast<float4 *>(xh + (size_t)a.batch * a.xpitch * (XLO ? 2 : 1));
  uint64_t *full = reinterpret_cast<uint64_t *>(red + (size_t)S * W * RB * 32);
  int *count = reinterpret_cast<int *>(full + S);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  if (blockDim.x != W * 32) return;  // the layout below assumes W warps
  long long total = a.total_rows, rpc = a.rpc;
  __shared__ int ids_shared[MOE ? kMoeIdsShared : 1];
  if (MOE) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int live = min(max(*a.moe.count, 0), a.moe.cap);
    total = (long long)live * a.moe.rpe;
    rpc = ((total + gridDim.x - 1) / gridDim.x + 15) / 16 * 16;
    for (int i = tid; i < min(live, kMoeIdsShared); i += blockDim.x) ids_shared[i] = a.moe.ids[i];
    __syncthreads();
  }
  const long long v_lo = (long long)blockIdx.x * rpc;
  const long long v_hi = min(total, v_lo + rpc);
  if (v_lo >= v_hi) return;
  // The segment holding v_lo (segments are in virtual-row order).
  UnitIter it_c{0, 0, 0, v_lo};
  if (MOE) {
    it_c.seg = (int)(v_lo / a.moe.rpe);
    it_c.row = (int)(v_lo % a.moe.rpe);
    it_c.seg_rows = a.moe.rpe;
  } else {
    while (it_c.seg + 1 < a.nseg && a.seg[it_c.seg + 1].vbeg <= v_lo) ++it_c.seg;
    it_c.row = (int)(v_lo - a.seg[it_c.seg].vbeg);
    it_c.seg_rows = a.seg[it_c.seg].rows;
  }
  UnitIter it_a = it_c;  // S units ahead of it_c once the ring is primed

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(&full[s], 1);
      count[s] = 0;
    }
    sm100::fence_barrier_init();
  }
  __syncthreads();
  // Weights are immutable while their handle exists: copy them before the
  // wait (dense segments; device-indirect ones are known only after it).
  for (int s = 0; s < S; ++s) {
    Unit u;
    if (!next_unit<UR, MOE>(a, it_a, v_hi, u)) break;
    if (warp == 0) stream_issue<UR, MOE>(a, stages + (size_t)s * a.stage_bytes, &full[s], u, lane, ids_shared);
  }
  if (!MOE) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }

  const int chunks = a.K >> 7;
  const int cpw = (chunks + W - 1) / W;
  const int c_lo = min(chunks, warp * cpw), c_hi = min(chunks, c_lo + cpw);
  const int k_lo = c_lo * 128, pieces = (c_hi - c_lo) * 16;  // 8-element pieces
  const bool n_ok = g < a.batch;
  const __half *xrow = xh + (size_t)(n_ok ? g : 0) * a.xpitch;
  const __half *xrow_lo = xl + (size_t)(n_ok ? g : 0) * a.xpitch;
  const void *staged_x = nullptr;
  float us0 = 1.0f, us1 = 1.0f;
  int cur_seg = -1;
  const void *seg_x = nullptr;  // input, output and row count of segment cur_seg
  void *y_seg = nullptr;
  int y_rows = 0;

  // ---- units -------------------------------------------------------------------
  Unit u;
  for (int i = 0; next_unit<UR, MOE>(a, it_c, v_hi, u); ++i) {
    if (u.seg != cur_seg) {
      cur_seg = u.seg;
      if (MOE) {
        seg_x = static_cast<const char *>(a.seg[0].x) + (size_t)u.seg * a.moe.x_stride * (XLO ? 4 : 2);
        y_seg = static_cast<char *>(a.seg[0].y) + (size_t)u.seg * a.moe.y_stride * (a.y_bf16 ? 2 : 4);
      } else {
        seg_x = a.seg[u.seg].x;
        y_seg = a.seg[u.seg].y;
      }
      y_rows = it_c.seg_rows;
    }
    if (seg_x != staged_x) {
      // ---- this warp's K slice of the segment's x, prescaled to f16 ----------
      staged_x = seg_x;
      float my_unscale = 1.0f;  // lane b: batch row b
      // Rows in groups of G = 4, every load of a group
      // issued before the first reduction: the rows' latencies overlap.
      constexpr int G = 4, NV = XLO ? 2 : 1;
      for (int b0 = 0; b0 < a.batch; b0 += G) {
        uint4 raw[G][2][NV];
#pragma unroll
        for (int bb = 0; bb < G; ++bb)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int b = b0 + bb, p = lane + 32 * h;
            const bool ok = b < a.batch && p < pieces;
            const long long off = (long long)b * a.K + k_lo + p * 8;
#pragma unroll
            for (int j = 0; j < NV; ++j)
              raw[bb][h][j] = !ok ? make_uint4(0, 0, 0, 0)
                              : XLO ? *reinterpret_cast<const uint4 *>(reinterpret_cast<const float *>(seg_x) +
                                                                       off + 4 * j)
                                    : *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(seg_x) +
                                                                       off);
          }
#pragma unroll
        for (int bb = 0; bb < G; ++bb) {
          const int b = b0 + bb;
          if (b >= a.batch) break;  // uniform over the warp
          float v[2][8];
          uint32_t m = 0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (XLO) {
#pragma unroll
              for (int j = 0; j < NV; ++j) {
                const uint4 r = raw[bb][h][j];
                v[h][4 * j + 0] = __uint_as_float(r.x); v[h][4 * j + 1] = __uint_as_float(r.y);
                v[h][4 * j + 2] = __uint_as_float(r.z); v[h][4 * j + 3] = __uint_as_float(r.w);
              }
            } else {
              const uint4 r = raw[bb][h][0];
              const uint32_t wv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                v[h][2 * t] = __uint_as_float(wv[t] << 16);
                v[h][2 * t + 1] = __uint_as_float(wv[t] & 0xffff0000u);
              }
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) m = max(m, __float_as_uint(v[h][t]) & 0x7fffffffu);
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
          const int F = prescale_exponent(m);
          const float up = __uint_as_float((uint32_t)(127 + F) << 23);
          if (lane == b) my_unscale = __uint_as_float((uint32_t)(127 - F) << 23);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int p = lane + 32 * h;
            if (p >= pieces) continue;
            uint32_t hv[4], lv[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const float v0 = v[h][2 * t] * up, v1 = v[h][2 * t + 1] * up;
              hv[t] = pack_half2(v0, v1);
              if (XLO) {
                const float2 f = __half22float2(*reinterpret_cast<__half2 *>(&hv[t]));
                lv[t] = pack_half2(v0 - f.x, v1 - f.y);
              }
            }
            const size_t o = (size_t)b * a.xpitch + xswz(k_lo + p * 8);
            *reinterpret_cast<uint4 *>(xh + o) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
            if (XLO) *reinterpret_cast<uint4 *>(xl + o) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
          }
        }
      }
      __syncwarp();
      // Unscale of accumulator columns n = 2q, 2q + 1.
      us0 = __shfl_sync(0xffffffffu, my_unscale, 2 * q);
      us1 = __shfl_sync(0xffffffffu, my_unscale, 2 * q + 1);
    }

    const int s = i % S;
    const uint32_t parity = (uint32_t)(i / S) & 1u;
    uint8_t *st = stages + (size_t)s * a.stage_bytes;
    bool ready = false;
    for (uint32_t t = 0; t < sm100::kSpinLimit && !ready; ++t) ready = sm100::mbar_try_wait(&full[s], parity);
    if (!ready) {  // copies that never landed: record it and leave
      if (lane == 0 && a.error) atomicCAS(a.error, 0, 201);
      return;
    }
    // RB row blocks, each with NCH independent accumulators (four chains for
    // one block, two for several: the blocks are independent chains too).
    constexpr int NCH = RB == 1 ? 4 : 2;
    float acc[RB][NCH][4];
#pragma unroll
    for (int rb = 0; rb < RB; ++rb)
#pragma unroll
      for (int c4 = 0; c4 < NCH; ++c4)
#pragma unroll
        for (int t = 0; t < 4; ++t) acc[rb][c4][t] = 0.0f;

    const uint8_t *sc = st + UR * a.wpitch;
    const int live_rb = min(RB, (u.nrows + 15) >> 4);  // blocks holding rows of this unit
    for (int c = c_lo; c < c_hi; ++c) {
      uint4 wa[RB], wb[RB];
      uint32_t s_lo[RB][2], s_hi[RB][2];
#pragma unroll
      for (int rb = 0; rb < RB; ++rb) {
        const int r0 = rb * 16 + g;
        wa[rb] = lds128(st + r0 * a.wpitch + c * 64 + q * 16);
        wb[rb] = HALF ? make_uint4(0, 0, 0, 0) : lds128(st + (r0 + 8) * a.wpitch + c * 64 + q * 16);
        const uint32_t fa = e4m3x2_to_f16x2(lds16(sc + r0 * a.spitch + c * 8 + 2 * q));
        s_lo[rb][0] = __byte_perm(fa, fa, 0x1010);
        s_hi[rb][0] = __byte_perm(fa, fa, 0x3232);
        if (!HALF) {
          const uint32_t fb = e4m3x2_to_f16x2(lds16(sc + (r0 + 8) * a.spitch + c * 8 + 2 * q));
          s_lo[rb][1] = __byte_perm(fb, fb, 0x1010);
          s_hi[rb][1] = __byte_perm(fb, fb, 0x3232);
        } else {
          s_lo[rb][1] = s_hi[rb][1] = 0;
        }
      }
      const int k0 = c * 128 + q * 32;
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        uint4 xv = make_uint4(0, 0, 0, 0), xlv = make_uint4(0, 0, 0, 0);
        if (n_ok) {
          const int kx = xswz(k0 + 8 * wi);
          xv = lds128(xrow + kx);
          if (XLO) xlv = lds128(xrow_lo + kx);
        }
#pragma unroll
        for (int rb = 0; rb < RB; ++rb) {
          if (rb >= live_rb) break;  // uniform over the warp
          const uint32_t w0 = wi == 0 ? wa[rb].x : wi == 1 ? wa[rb].y : wi == 2 ? wa[rb].z : wa[rb].w;
          const uint32_t w1 = wi == 0 ? wb[rb].x : wi == 1 ? wb[rb].y : wi == 2 ? wb[rb].z : wb[rb].w;
          uint32_t f0[4], f1[4] = {0, 0, 0, 0};
          e2m1x8_to_f16x8(w0, f0);
          if (!HALF) e2m1x8_to_f16x8(w1, f1);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            f0[t] = hmul2(f0[t], wi < 2 ? s_lo[rb][0] : s_hi[rb][0]);
            if (!HALF) f1[t] = hmul2(f1[t], wi < 2 ? s_lo[rb][1] : s_hi[rb][1]);
          }
          // MMA 2wi + jj takes codes 4jj..4jj+3 of this word and x words 2jj, 2jj+1.
          const int ch = NCH == 4 ? (wi & 1) * 2 : 0;
          mma_f16(acc[rb][ch], f0[0], f1[0], f0[1], f1[1], xv.x, xv.y);
          mma_f16(acc[rb][ch + 1], f0[2], f1[2], f0[3], f1[3], xv.z, xv.w);
          if (XLO) {
            mma_f16(acc[rb][ch], f0[0], f1[0], f0[1], f1[1], xlv.x, xlv.y);
            mma_f16(acc[rb][ch + 1], f0[2], f1[2], f0[3], f1[3], xlv.z, xlv.w);
          }
        }
      }
    }
    float4 *slot = red + (size_t)s * W * RB * 32;
#pragma unroll
    for (int rb = 0; rb < RB; ++rb) {
      float v4[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float sum = acc[rb][0][t];
#pragma unroll
        for (int c4 = 1; c4 < NCH; ++c4) sum += acc[rb][c4][t];
        v4[t] = sum * ((t & 1) ? us1 : us0);
      }
      slot[(warp * RB + rb) * 32 + lane] = make_float4(v4[0], v4[1], v4[2], v4[3]);
    }
    // The unit S ahead, which the last warp to finish this one copies into
    // its stage (every warp advances its look-ahead iterator in step).
    Unit ahead;
    const bool has_ahead = next_unit<UR, MOE>(a, it_a, v_hi, ahead);
    // The last of the W warps to finish this unit reduces it, stores y and
    // refills the stage (the counter only grows: last = W-th arrival).
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = (atomicAdd(&count[s], 1) % W) == W - 1;
      __threadfence_block();
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    if (!last) continue;
    const float *gl = reinterpret_cast<const float *>(sc + UR * a.spitch);
#pragma unroll
    for (int rb = 0; rb < RB; ++rb) {
      if (rb >= live_rb) break;
      float4 sum = slot[rb * 32 + lane];
#pragma unroll
      for (int w = 1; w < W; ++w) {
        const float4 p = slot[(w * RB + rb) * 32 + lane];
        sum.x += p.x; sum.y += p.y; sum.z += p.z; sum.w += p.w;
      }
      const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int rl = rb * 16 + g + ((t >> 1) << 3), n = 2 * q + (t & 1);
        if (rl < u.nrows && n < a.batch) {
          const float v = vals[t] * gl[rl];
          const size_t off = (size_t)n * y_rows + u.row0 + rl;
          if (a.y_bf16)
            reinterpret_cast<__nv_bfloat16 *>(y_seg)[off] = __float2bfloat16_rn(v);
          else
            reinterpret_cast<float *>(y_seg)[off] = v;
        }
      }
    }
    if (has_ahead) {
      __syncwarp();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      stream_issue<UR, MOE>(a, st, &full[s], ahead, lane, ids_shared);
    }
  }
}

// ---- host dispatch -----------------------------------------------------------
struct GemvConfig {
  int C, wk, g, threads;
};

// Up to 16 warps per CTA, each covering 16 rows x 128*C columns; C = 2 only
// when K needs more than 16 warps (K <= 4096).
static GemvConfig pick_config(int K) {
  int chunks = (K + 127) / 128;
  int C = 1;
  while ((chunks + C - 1) / C > 16 && C < 2) C *= 2;
  int wk = (chunks + C - 1) / C;
  if (wk > 16) return {0, 0, 0, 0};
  int g = std::max(1, 16 / wk);
  return {C, wk, g, wk * g * 32};
}

// Largest batch rows per launch: x fragments live in registers, so f32 input
// (hi and lo fragments) or more than one group of 8 rows are limited by the
// chunks a warp holds.
static int gemv_max_batch(int K, bool x_f32) {
  GemvConfig cfg = pick_config(K);
  return (cfg.C == 1 && !x_f32) ? 16 : 8;  // two 8-row groups only where they fit
}

static size_t gemv_smem_bytes(const GemvConfig &cfg, int NG) {
  return 2 * (size_t)cfg.g * cfg.wk * NG * 32 * sizeof(float4);
}

using GemvKernel = void (*)(GemvArgs);

template <int C, int NG, bool XLO>
static GemvKernel kernel_for() {
  return gemv_nvfp4_kernel<C, NG, XLO>;
}

static GemvKernel select_kernel(int C, int NG, bool xlo) {
  // Instantiated variants are exactly those that fit in registers without
  // spilling: 16 input rows only with bf16 input and K <= 2048.
  if (C == 1 && NG == 1) return xlo ? kernel_for<1, 1, true>() : kernel_for<1, 1, false>();
  if (C == 1 && NG == 2 && !xlo) return kernel_for<1, 2, false>();
  if (C == 2 && NG == 1) return xlo ? kernel_for<2, 1, true>() : kernel_for<2, 1, false>();
  return nullptr;
}

static int run_gemv_slice(GemvArgs args, int slots, bool x_f32, cudaStream_t stream);

// Rows longer than 4096 columns run as consecutive launches over 4096-column
// slices of K, the later ones adding their sums to y (f32; every slice's sum
// times the row global).
static int run_gemv(GemvArgs args, int slots, bool x_f32, cudaStream_t stream) {
  constexpr int kSlice = 4096;
  args.k_pitch = args.K;
  if (args.K <= kSlice) return run_gemv_slice(args, slots, x_f32, stream);
  if (args.y_bf16)
    return fail(FPB_ERR_UNSUPPORTED, "NVFP4 GEMV: K=%d > 4096 needs an f32 y (the sums of the K slices add there)",
                args.K);
  const int K = args.K;
  for (int k0 = 0; k0 < K; k0 += kSlice) {
    GemvArgs part = args;
    part.K = std::min(kSlice, K - k0);
    part.packed = args.packed + k0 / 2;
    part.scales = args.scales + k0 / kNvfp4Group;
    part.x = static_cast<const char *>(args.x) + (size_t)k0 * (x_f32 ? 4 : 2);
    part.accumulate = k0 > 0;
    int st = run_gemv_slice(part, slots, x_f32, stream);
    if (st) return st;
  }
  return FPB_OK;
}

static int run_gemv_slice(GemvArgs args, int slots, bool x_f32, cudaStream_t stream) {
  GemvConfig cfg = pick_config(args.K);
  if (!cfg.C) return fail(FPB_ERR_UNSUPPORTED, "NVFP4 GEMV: K=%d exceeds 4096", args.K);
  args.chunks = (args.K + 127) / 128;
  args.nrb = (args.rows + 15) / 16;
  args.wk = cfg.wk;
  args.g = cfg.g;
  const int NG = args.batch > 8 ? 2 : 1;
  const size_t smem = gemv_smem_bytes(cfg, NG);
  GemvKernel k = select_kernel(cfg.C, NG, x_f32);
  if (!k) return fail(FPB_ERR_UNSUPPORTED, "NVFP4 GEMV: no kernel for C=%d", cfg.C);

  // Kernel attributes and occupancy are queried once per (device, kernel,
  // block size, shared memory), so that repeated calls, including calls made
  // while a stream is captured into a CUDA graph, make no extra runtime calls.
  struct OccEntry {
    int dev;
    GemvKernel k;
    int threads;
    size_t smem;
    int occ;
  };
  static std::mutex mu;
  static std::vector<OccEntry> occ_cache;
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (auto &o : occ_cache)
      if (o.dev == dev && o.k == k && o.threads == cfg.threads && o.smem == smem) occ = o.occ;
    if (occ == 0) {
      // The reduction buffer is at most 32 KB, below the default 48 KB limit
      // of dynamic shared memory, so the kernel attribute is never touched
      // (lowering it for one launch would cap every later, larger launch).
      static_assert(2 * 16 * 2 * 32 * sizeof(float4) <= 48 * 1024, "GEMV reduction buffer");
      cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, cfg.threads, smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      if (occ < 1) occ = 1;
      occ_cache.push_back({dev, k, cfg.threads, smem, occ});
    }
  }
  const int groups = (args.nrb + cfg.g - 1) / cfg.g;
  const long long resident = (long long)occ * sm_count();
  const long long per_slot = std::max(1LL, resident / std::max(1, slots));
  const int grid_x = (int)std::min<long long>(groups, per_slot);
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(grid_x, slots);
  lc.blockDim = dim3(cfg.threads);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&lc, k, args);
  if (le == cudaErrorInvalidValue) {
    // A runtime that refuses the programmatic-serialization attribute for
    // this launch gets a plain stream-ordered launch instead.
    cudaGetLastError();
    lc.numAttrs = 0;
    le = cudaLaunchKernelEx(&lc, k, args);
  }
  if (le != cudaSuccess) {
    // Report what the runtime knows about the kernel and this launch.
    cudaGetLastError();
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, k);
    int occ_now = -1;
    cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_now, k, cfg.threads, smem);
    cudaGetLastError();
    return fail(FPB_ERR_CUDA,
                "cudaLaunchKernelEx(gemv_nvfp4_kernel): %s; grid (%d,%d) block %d smem %zu; kernel regs %d "
                "local %zu maxThreads %d maxDynSmem %d; occupancy now %d (%s), cached %d",
                cudaGetErrorName(le), grid_x, slots, cfg.threads, smem, fa.numRegs, fa.localSizeBytes,
                fa.maxThreadsPerBlock, fa.maxDynamicSharedSizeBytes, occ_now, cudaGetErrorName(oe), occ);
  }
  FPB_LAUNCH_CHECK("gemv_nvfp4_kernel");
  return FPB_OK;
}


// Shared memory one streaming CTA may use: two CTAs (and their 1 KB system
// reservations) fit in the 228 KB of an SM.
constexpr int kStreamSmemBudget = 110 * 1024;

// A unit's codes, factors and row globals each arrive as one contiguous bulk
// copy (rows are contiguous in HBM).  Copies of single rows would pad the
// shared-memory row pitch against bank conflicts, but cost two copies per
// row, and the copy issue rate, not the bytes, then bounded the kernel (a
// 512-column expert GEMV ran 1.9x slower, 4096-column rows 1.15x).
#ifndef FPB_STREAM_CONTIG
#define FPB_STREAM_CONTIG 1
#endif

// Ring and staging geometry of the streaming kernel for (K, batch, x dtype,
// unit rows); false when the streaming kernel cannot serve that shape.
template <int NSEG>
static bool stream_geometry(int K, int batch, bool x_f32, int unit_rows, long long max_units_per_cta,
                            StreamArgs<NSEG> *a, size_t *smem) {
  if (K % 128 != 0 || K > 4096 || batch < 1 || batch > 8) return false;
  a->K = K;
  a->batch = batch;
  const int kb2 = K / 2, kb16 = K / 16;
  a->contig = FPB_STREAM_CONTIG;
  a->wpitch = a->contig ? kb2 : kb2 + ((kb2 % 128 == 0) ? 64 : 0);  // 64 mod 128 when per row
  a->scale_rows = !a->contig && kb16 % 16 == 0;
  a->spitch = a->scale_rows ? kb16 + (16 - kb16 % 128 + 128) % 128 : kb16;  // 16 mod 128 when per row
  a->stage_bytes = unit_rows * a->wpitch + unit_rows * a->spitch + std::max(64, unit_rows * 4);  // + row globals
  a->xpitch = K + 8;
  const size_t x_bytes = (size_t)batch * a->xpitch * 2 * (x_f32 ? 2 : 1);
  const int row_blocks = unit_rows >= 16 ? unit_rows / 16 : 1;
  const size_t per_stage = (size_t)a->stage_bytes + (size_t)kStreamWarps * row_blocks * 32 * sizeof(float4) + 12;
  if (x_bytes + per_stage + 16 > (size_t)kStreamSmemBudget) return false;
  long long S = (long long)((kStreamSmemBudget - x_bytes - 16) / per_stage);
  S = std::max(1LL, std::min({S, 8LL, max_units_per_cta}));
  a->stages = (int)S;
  *smem = (size_t)S * per_stage + x_bytes + 16;
  return true;
}

#ifndef FPB_STREAM_UNIT_ROWS_MAX
#define FPB_STREAM_UNIT_ROWS_MAX 32  // 64-row units need more than 128 registers a thread (spills)
#endif

// Rows per unit for a launch whose CTAs own about `rows_per_cta` rows: a
// unit's row blocks are independent MMA chains sharing each x fragment, and
// the per-unit protocol (wait, partial sums, reduction, refill) is paid once
// per unit, so the largest size up to FPB_STREAM_UNIT_ROWS_MAX that fits the
// CTA's share and a ring of two stages, else 16.  0 when the kernel cannot
// take the shape.
template <int NSEG>
static int stream_plan(int K, int batch, bool x_f32, long long rows_per_cta, long long extra_units,
                       StreamArgs<NSEG> *a, size_t *smem) {
  for (int ur = FPB_STREAM_UNIT_ROWS_MAX; ur > 16; ur /= 2) {
    if (ur > rows_per_cta) continue;
    if (stream_geometry(K, batch, x_f32, ur, (rows_per_cta + ur - 1) / ur + extra_units, a, smem) && a->stages >= 2)
      return ur;
  }
  return stream_geometry(K, batch, x_f32, 16, (rows_per_cta + 15) / 16 + extra_units, a, smem) ? 16 : 0;
}

template <int NSEG, bool MOE = false>
static int launch_stream_ur(int ur, const StreamArgs<NSEG> &a, int grid, size_t smem, bool x_f32,
                            cudaStream_t stream);

// A segment the streaming kernel can read with 16-byte bulk copies: rows and
// the first row a multiple of 4 (so every unit's factor and global copies are
// whole 16-byte pieces) and aligned row pointers.
static bool stream_segment_ok(const uint8_t *packed, const uint8_t *scales, const float *globals, long long rows) {
  return rows > 0 && rows % 4 == 0 && rows <= 0x7fffffff && reinterpret_cast<uintptr_t>(packed) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(scales) % 16 == 0 && reinterpret_cast<uintptr_t>(globals) % 16 == 0;
}

template <int NSEG, int UR, bool MOE = false>
static int launch_stream(const StreamArgs<NSEG> &a, int grid, size_t smem, bool x_f32, cudaStream_t stream) {
  auto k = x_f32 ? gemv_nvfp4_stream_kernel<true, NSEG, UR, MOE> : gemv_nvfp4_stream_kernel<false, NSEG, UR, MOE>;
  {
    // Raised once per device and kernel to the budget, never lowered.
    static std::mutex mu;
    static std::vector<std::pair<int, const void *>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    const void *key = reinterpret_cast<const void *>(k);
    if (std::find(done.begin(), done.end(), std::make_pair(dev, key)) == done.end()) {
      FPB_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kStreamSmemBudget));
      done.push_back({dev, key});
    }
  }
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(kStreamWarps * 32);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&lc, k, a);
  if (le == cudaErrorInvalidValue) {
    cudaGetLastError();
    lc.numAttrs = 0;
    le = cudaLaunchKernelEx(&lc, k, a);
  }
  if (le != cudaSuccess) {
    cudaGetLastError();
    return fail(FPB_ERR_CUDA,
                "cudaLaunchKernelEx(gemv_nvfp4_stream_kernel): %s; grid %d smem %zu stages %d segments %d",
                cudaGetErrorName(le), grid, smem, a.stages, a.nseg);
  }
  FPB_LAUNCH_CHECK("gemv_nvfp4_stream_kernel");
  return FPB_OK;
}

// One matrix: one CTA per SM, each owning ceil(rows / SMs) rows rounded up to
// 4, so that a CTA of the next launch in the stream fits beside it and
// streams its weights while this launch computes.
static int try_stream_single(const uint8_t *packed, const uint8_t *scales, const float *globals, int rows, int K,
                             const void *x, bool x_f32, void *y, bool y_bf16, int batch, cudaStream_t stream,
                             bool *served) {
  *served = false;
  if (!stream_segment_ok(packed, scales, globals, rows)) return FPB_OK;
  StreamArgs<1> a{};
  const int nsm = std::max(1, sm_count());
  int rpc = (rows + nsm - 1) / nsm;
  rpc = (rpc + 3) / 4 * 4;
  size_t smem = 0;
  const int ur = stream_plan(K, batch, x_f32, rpc, 0, &a, &smem);
  if (!ur) return FPB_OK;
  a.seg[0] = StreamSeg{packed, scales, globals, x, y, 0, rows, 0};
  a.nseg = 1;
  a.rpc = rpc;
  a.total_rows = rows;
  a.error = device_error_ptr();
  a.y_bf16 = y_bf16;
  *served = true;
  return launch_stream_ur<1>(ur, a, (rows + rpc - 1) / rpc, smem, x_f32, stream);
}

template <int NSEG, bool MOE>
static int launch_stream_ur(int ur, const StreamArgs<NSEG> &a, int grid, size_t smem, bool x_f32,
                            cudaStream_t stream) {
  switch (ur) {
    case 16: return launch_stream<NSEG, 16, MOE>(a, grid, smem, x_f32, stream);
    case 32: return launch_stream<NSEG, 32, MOE>(a, grid, smem, x_f32, stream);
#if FPB_STREAM_UNIT_ROWS_MAX >= 64
    case 64: return launch_stream<NSEG, 64, MOE>(a, grid, smem, x_f32, stream);
#endif
    default: return fail(FPB_ERR_UNSUPPORTED, "streaming GEMV: unit rows %d", ur);
  }
}

}  // namespace fpb

using namespace fpb;

extern "C" int fpb_nvfp4_gemv(const fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end,
                              const void *x, int x_dtype, void *y, int y_dtype, int batch,
                              void *stream) {
  if (!w || !x || !y) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv: null pointer");
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv: row range [%zu, %zu) outside %zu rows", row_begin,
                row_end, w->rows);
  if (batch < 1 || batch > 16) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv: batch %d not in [1, 16]", batch);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv: dtype");
  if ((size_t)(row_end - row_begin) > 0x7fffffff)
    return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemv: too many rows");
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv: x must be 16-byte aligned");
  GemvArgs a{};
  a.x_div = 1;
  a.packed = w->packed + row_begin * (w->cols / 2);
  a.scales = w->scales + row_begin * (w->cols / kNvfp4Group);
  a.globals = w->row_globals + row_begin;
  a.expert_ids = nullptr;
  a.rows = (int)(row_end - row_begin);
  a.K = (int)w->cols;
  a.y_bf16 = y_dtype == FPB_BF16;
  a.y_batch_stride = a.rows;
  const bool x_f32 = x_dtype == FPB_F32;
  bool served = false;
  int st0 = try_stream_single(a.packed, a.scales, a.globals, a.rows, a.K, x, x_f32, y, a.y_bf16 != 0, batch,
                              as_stream(stream), &served);
  if (served || st0) return st0;
  // More input rows than one launch holds in registers run as several
  // launches over row groups of x (each re-reads W).
  const int step = std::min(batch, gemv_max_batch((int)w->cols, x_f32));
  for (int b0 = 0; b0 < batch; b0 += step) {
    GemvArgs part = a;
    part.batch = std::min(step, batch - b0);
    part.x = static_cast<const char *>(x) + (size_t)b0 * w->cols * (x_f32 ? 4 : 2);
    part.y = static_cast<char *>(y) + (size_t)b0 * a.rows * (a.y_bf16 ? 2 : 4);
    int st = run_gemv(part, 1, x_f32, as_stream(stream));
    if (st) return st;
  }
  return FPB_OK;
}

extern "C" int fpb_nvfp4_expert_gemv(const fpb_nvfp4_matrix *w, const void *x, int x_dtype,
                                     const int32_t *expert_ids, int slots, size_t rows_per_expert,
                                     int input_stride, void *y, int y_dtype, void *stream) {
  if (!w || !x || !y || !expert_ids)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_expert_gemv: null pointer");
  if (slots < 1 || slots > 65535) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_expert_gemv: slots %d", slots);
  if (rows_per_expert == 0 || w->rows % rows_per_expert != 0)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_expert_gemv: rows %zu not a multiple of rows_per_expert %zu",
                w->rows, rows_per_expert);
  if (input_stride < 0) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_expert_gemv: input_stride < 0");
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_expert_gemv: dtype");
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_expert_gemv: x must be 16-byte aligned");
  GemvArgs a{};
  a.packed = w->packed;
  a.scales = w->scales;
  a.globals = w->row_globals;
  a.x = x;
  a.y = y;
  a.expert_ids = expert_ids;
  a.n_experts = (int)(w->rows / rows_per_expert);
  a.rows = (int)rows_per_expert;
  a.K = (int)w->cols;
  a.batch = 1;
  a.y_bf16 = y_dtype == FPB_BF16;
  a.y_batch_stride = 0;
  a.x_slot_stride = (long long)input_stride * (long long)w->cols;
  a.x_div = 1;
  a.y_slot_stride = (long long)rows_per_expert;
  return run_gemv(a, slots, x_dtype == FPB_F32, as_stream(stream));
}

// The expert GEMV of several tokens at once (decode of a batch of sessions):
// token t's slots t*slots_per_token .. +slots_per_token-1 use x row t.
extern "C" int fpb_nvfp4_expert_gemv_tokens(const fpb_nvfp4_matrix *w, const void *x, int x_dtype,
                                            const int32_t *expert_ids, int tokens, int slots_per_token,
                                            size_t rows_per_expert, void *y, int y_dtype, void *stream) {
  if (!w || !x || !y || !expert_ids)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_expert_gemv_tokens: null pointer");
  if (tokens < 1 || slots_per_token < 1 || (long long)tokens * slots_per_token > 65535)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_expert_gemv_tokens: %d tokens x %d slots", tokens, slots_per_token);
  if (rows_per_expert == 0 || w->rows % rows_per_expert != 0)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_expert_gemv_tokens: rows %zu not a multiple of rows_per_expert %zu",
                w->rows, rows_per_expert);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_expert_gemv_tokens: dtype");
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_expert_gemv_tokens: x must be 16-byte aligned");
  GemvArgs a{};
  a.packed = w->packed;
  a.scales = w->scales;
  a.globals = w->row_globals;
  a.x = x;
  a.y = y;
  a.expert_ids = expert_ids;
  a.n_experts = (int)(w->rows / rows_per_expert);
  a.rows = (int)rows_per_expert;
  a.K = (int)w->cols;
  a.batch = 1;
  a.y_bf16 = y_dtype == FPB_BF16;
  a.y_batch_stride = 0;
  a.x_slot_stride = (long long)w->cols;
  a.x_div = slots_per_token;
  a.y_slot_stride = (long long)rows_per_expert;
  return run_gemv(a, tokens * slots_per_token, x_dtype == FPB_F32, as_stream(stream));
}

// The decode MoE GEMV over distinct experts (see fpb_nvfp4_moe_gemv in the
// header): the streaming kernel with device-indirect segments when it can
// take the shape, else the register kernel in expert mode over all `cap`
// slots (ids past the count are -1 there and give zero rows).
extern "C" int fpb_nvfp4_moe_gemv(const fpb_nvfp4_matrix *w, size_t rows_per_expert, const int32_t *experts,
                                  const int32_t *count, int cap, const void *x, int x_dtype, size_t x_stride,
                                  int tokens, void *y, int y_dtype, void *stream) {
  if (!w || !experts || !count || !x || !y) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_moe_gemv: null pointer");
  if (cap < 1 || cap > 65535) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv: cap %d", cap);
  if (tokens < 1 || tokens > 16) return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv: tokens %d not in [1, 16]", tokens);
  if (rows_per_expert == 0 || w->rows % rows_per_expert != 0 || rows_per_expert > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv: rows %zu not a multiple of rows_per_expert %zu", w->rows,
                rows_per_expert);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_moe_gemv: dtype");
  const bool x_f32 = x_dtype == FPB_F32, y_bf16 = y_dtype == FPB_BF16;
  const size_t xe = x_f32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || (x_stride * xe) % 16 != 0)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_moe_gemv: x and x_stride must keep 16-byte alignment");
  if (x_stride != 0 && x_stride < (size_t)tokens * w->cols)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_moe_gemv: x_stride %zu below tokens x cols", x_stride);
  const int K = (int)w->cols, rpe = (int)rows_per_expert;
  cudaStream_t s = as_stream(stream);
  StreamArgs<1> a{};
  size_t smem = 0;
  const int grid = 2 * std::max(1, sm_count());
  // rows per CTA when every slot holds a distinct expert (the most there can be)
  const long long share = ((long long)cap * rpe + grid - 1) / grid;
  int ur = 0;
  if (tokens <= 8 && rpe % 4 == 0 && stream_segment_ok(w->packed, w->scales, w->row_globals, rpe) &&
      (ur = stream_plan(K, tokens, x_f32, share, 2, &a, &smem)) != 0) {
    a.seg[0] = StreamSeg{w->packed, w->scales, w->row_globals, x, y, 0, rpe, 0};
    a.nseg = 1;
    a.moe = StreamMoe{experts, count, cap, rpe, (int)(w->rows / rows_per_expert), (long long)x_stride,
                      (long long)tokens * rpe};
    a.error = device_error_ptr();
    a.y_bf16 = y_bf16;
    return launch_stream_ur<1, true>(ur, a, grid, smem, x_f32, s);
  }
  GemvArgs g{};
  g.packed = w->packed;
  g.scales = w->scales;
  g.globals = w->row_globals;
  g.x = x;
  g.y = y;
  g.expert_ids = experts;
  g.n_experts = (int)(w->rows / rows_per_expert);
  g.rows = rpe;
  g.K = K;
  g.batch = tokens;
  g.y_bf16 = y_bf16;
  g.y_batch_stride = rpe;
  g.x_slot_stride = (long long)x_stride;
  g.x_div = 1;
  g.y_slot_stride = (long long)tokens * rpe;
  return run_gemv(g, cap, x_f32, s);
}

// Several dense GEMVs in one launch (see fpb_nvfp4_gemv_batched in the
// header).  Served by the streaming kernel over up to kStreamMaxSegs
// segments, two CTAs per SM, each owning an equal share of the segments'
// rows laid end to end; shapes it cannot take run as one fpb_nvfp4_gemv per
// segment.
extern "C" int fpb_nvfp4_gemv_batched(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype,
                                      int batch, void *stream) {
  if (!segs || count < 1) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batched: no segments");
  if (count > kStreamMaxSegs)
    return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemv_batched: %d segments exceed %d", count, kStreamMaxSegs);
  if ((x_dtype != FPB_F32 && x_dtype != FPB_BF16) || (y_dtype != FPB_F32 && y_dtype != FPB_BF16))
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batched: dtype");
  if (batch < 1 || batch > 16)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv_batched: batch %d not in [1, 16]", batch);
  if (!segs[0].w) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batched: null matrix in segment 0");
  const size_t K = segs[0].w->cols;
  for (int i = 0; i < count; ++i) {
    const fpb_gemv_segment &sg = segs[i];
    if (!sg.w || !sg.x || !sg.y)
      return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batched: null pointer in segment %d", i);
    if (sg.w->cols != K)
      return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv_batched: segment %d has %zu columns, segment 0 has %zu", i,
                  sg.w->cols, K);
    const size_t end = sg.row_end ? sg.row_end : sg.w->rows;
    if (sg.row_begin >= end || end > sg.w->rows)
      return fail(FPB_ERR_SHAPE, "fpb_nvfp4_gemv_batched: segment %d row range [%zu, %zu) outside %zu rows", i,
                  sg.row_begin, end, sg.w->rows);
    if (reinterpret_cast<uintptr_t>(sg.x) % 16 != 0)
      return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv_batched: x of segment %d not 16-byte aligned", i);
  }
  const bool x_f32 = x_dtype == FPB_F32;
  cudaStream_t s = as_stream(stream);

  // Segments the streaming kernel can read go into one launch; any other
  // segment (a row count or first row not a multiple of 4, an unaligned
  // row) runs as its own fpb_nvfp4_gemv.
  StreamArgs<kStreamMaxSegs> a{};
  bool alone[kStreamMaxSegs] = {};
  int nstream = 0;
  long long total = 0;
  for (int i = 0; i < count; ++i) {
    const fpb_gemv_segment &sg = segs[i];
    const size_t end = sg.row_end ? sg.row_end : sg.w->rows;
    const long long rows = (long long)(end - sg.row_begin);
    const uint8_t *packed = sg.w->packed + sg.row_begin * (K / 2);
    const uint8_t *scales = sg.w->scales + sg.row_begin * (K / kNvfp4Group);
    const float *globals = sg.w->row_globals + sg.row_begin;
    alone[i] = K > 4096 || !stream_segment_ok(packed, scales, globals, rows);
    if (alone[i]) continue;
    a.seg[nstream++] = StreamSeg{packed, scales, globals, sg.x, sg.y, total, (int)rows, 0};
    total += rows;
  }
  bool streamed = false;
  if (nstream > 0) {
    const int grid_target = 2 * std::max(1, sm_count());
    long long rpc = (total + grid_target - 1) / grid_target;
    rpc = (rpc + 3) / 4 * 4;
    size_t smem = 0;
    // A CTA's rows split into at most one more unit per segment they touch;
    // its ring never needs more stages than units.
    int unit_rows = 0;
    if (rpc <= 0x7fffffff && (unit_rows = stream_plan((int)K, batch, x_f32, rpc, nstream, &a, &smem)) != 0) {
      a.nseg = nstream;
      a.rpc = (int)rpc;
      a.total_rows = total;
      a.error = device_error_ptr();
      a.y_bf16 = y_dtype == FPB_BF16;
      const int grid = (int)((total + rpc - 1) / rpc);
      int st = launch_stream_ur<kStreamMaxSegs>(unit_rows, a, grid, smem, x_f32, s);
      if (st) return st;
      streamed = true;
    }
  }
  for (int i = 0; i < count; ++i) {
    if (streamed && !alone[i]) continue;
    const fpb_gemv_segment &sg = segs[i];
    int st = fpb_nvfp4_gemv(sg.w, sg.row_begin, sg.row_end, sg.x, x_dtype, sg.y, y_dtype, batch, stream);
    if (st) return st;
  }
  return FPB_OK;
}
