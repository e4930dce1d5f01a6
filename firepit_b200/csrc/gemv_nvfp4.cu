// NVFP4 decode GEMV, dense and expert (crates/firepit-kernels/src/gemv/nvfp4.rs).
//
// y[b, r] = g[r] * sum_k E2M1[w[r,k]] * e4m3(s[r,k/16]) * x[b,k]
//
// Design (HBM-bound; the instruction budget per weight element at full HBM
// bandwidth is about three thread-instructions, so arithmetic must be cheap):
//  * Each lane streams 16 bytes (32 codes) of one weight row per load
//    (128-bit, non-coherent, no L1 allocation).  A warp covers 16 rows x
//    128 columns per chunk: lanes 4g..4g+3 read rows g and g+8.
//  * Codes become f16 with `cvt.rn.f16x2.e2m1x2` and are multiplied by their
//    e4m3 block scale in f16.  e2m1 * e4m3 is exact in f16 (at most six
//    significant bits, magnitude in [2^-10, 2688]), so the dequantized weight
//    equals the reference's E2M1 * scale exactly.
//  * The dot products run on the tensor cores as m16n8k16 MMAs with f32
//    accumulation: weights are the A operand, the (up to 8 per MMA) input
//    vectors the B operand.  The MMA's k order is a permutation of the
//    physical columns that A and B share, which is free for a dot product.
//  * x is staged once per CTA in shared memory as ready-made B fragments.  To
//    keep them exact in f16, each input row is scaled by a power of two so
//    that its largest magnitude lands in [2^14, 2^15); bf16 inputs are then
//    exact (elements below amax * 2^-29 round to f16 subnormals, absolute
//    error < amax * 2^-40).  f32 inputs are split into an f16 hi and lo part
//    (22 significant bits) and take two MMAs, the f16 counterpart of the
//    reference's bf16 hi/lo split (gemm/nvfp4.rs:33-36).
//  * The per-lane partial sums of the warps that share a row block are added
//    in shared memory; the result is unscaled (exact power of two), times the
//    row global, and stored as f32 or bf16.
#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "nvfp4_matrix.cuh"

namespace fpb {

struct GemvArgs {
  const uint8_t *packed;  // row 0 of the addressed rows
  const uint8_t *scales;
  const float *globals;
  const void *x;
  void *y;
  const int32_t *expert_ids;  // null for dense
  long long x_slot_stride;    // elements between the input rows of consecutive slots
  long long y_slot_stride;    // elements between the output rows of consecutive slots
  long long y_batch_stride;   // elements between output rows of consecutive batch rows
  int rows;                   // rows per slot
  int K;
  int batch;
  int n_experts;  // expert mode: valid ids are [0, n_experts)
  int chunks;     // ceil(K / 128)
  int nrb;        // ceil(rows / 16)
  int iters;      // row-block iterations per CTA
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

// Power-of-two exponent F for a row whose largest magnitude has biased
// exponent `ef`: amax * 2^F lies in [2^14, 2^15).  Clamped so that 2^F and
// 2^-F are both normal floats.
__device__ __forceinline__ int prescale_exponent(uint32_t amax_bits) {
  int ef = (int)(amax_bits >> 23) & 0xff;
  int F = 141 - ef;
  return max(-126, min(126, F));
}

template <int C, int NG, bool XLO>
__global__ void __launch_bounds__(256, (C >= 4 ? 1 : 2)) gemv_nvfp4_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int chunks = a.chunks;
  const int batch = a.batch;
  // Compact B-fragment store: entry ((c*8 + j)*batch + n)*4 + q holds
  // x[n][c*128 + q*32 + 4j .. +3] as two f16x2 words, i.e. exactly what lane
  // (g = n % 8, q) feeds MMA j of chunk c.  Rows n >= batch are not stored:
  // their fragments are zero.
  const int n_entries = chunks * 8 * batch * 4;
  uint2 *xs_hi = reinterpret_cast<uint2 *>(smem);
  uint2 *xs_lo = xs_hi + (XLO ? n_entries : 0);
  const int wk_count = (chunks + C - 1) / C;
  const int g_count = max(1, (int)(blockDim.x / 32) / wk_count);
  float4 *red = reinterpret_cast<float4 *>(xs_hi + (XLO ? 2 : 1) * n_entries);
  __shared__ uint32_t amax_s[16];
  __shared__ float unscale_s[16];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int slot = blockIdx.y;
  const int K = a.K;
  const int kb2 = K >> 1, kb16 = K >> 4;

  // Which weight rows and which input/output rows this CTA serves.
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
  const long long x_off = (long long)slot * a.x_slot_stride;

  // ---- weight-row streaming; the first loads are issued before x is staged
  // so that their HBM latency overlaps the staging work.
  const int wk = warp % wk_count, gi = warp / wk_count;
  const bool warp_active = gi < g_count;
  const int c_begin = wk * C;
  const int g = lane >> 2, q = lane & 3;


  auto load = [&](int it, uint4 (&w)[2][C], uint16_t (&s)[2][C]) {
    int rb = (it * gridDim.x + blockIdx.x) * g_count + gi;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int r = rb * 16 + g + 8 * h;
      bool row_ok = warp_active && slot_ok && rb < a.nrb && r < a.rows;
#pragma unroll
      for (int cc = 0; cc < C; ++cc) {
        int c = c_begin + cc;
        bool ok = row_ok && c < chunks && (c * 128 + q * 32) < K;
        if (ok) {
          w[h][cc] = ldg_stream_v4(packed + (long long)r * kb2 + c * 64 + q * 16);
          s[h][cc] = ldg_u16(scales + (long long)r * kb16 + c * 8 + 2 * q);
        } else {
          w[h][cc] = make_uint4(0, 0, 0, 0);
          s[h][cc] = 0;
        }
      }
    }
  };

  uint4 wcur[2][C];
  uint16_t scur[2][C];
  load(0, wcur, scur);

  // Programmatic dependent launch: weights are immutable once their handle
  // exists (handle creation synchronises its stream), so their loads are
  // issued before waiting on the preceding kernel; x and y are touched only
  // after griddepcontrol.wait, which returns once the preceding grid has
  // completed and its writes are visible.  The next kernel in the stream may
  // start launching now.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- stage x as B fragments ----------------------------------------------
  // Pass 1: per-row amax, 8 elements per vector load, all loads of a thread
  // independent of each other so that they are in flight together.
  if (tid < 16) amax_s[tid] = 0;
  __syncthreads();
  {
    const int vec_per_row = K >> 3;
    const int total_vec = batch * vec_per_row;
    uint32_t m = 0;
    int cur_n = -1;
#pragma unroll 2
    for (int v = tid; v < total_vec; v += blockDim.x) {
      int n = v / vec_per_row;
      long long base = x_off + (long long)n * K + (long long)(v - n * vec_per_row) * 8;
      uint32_t vm;
      if (XLO) {
        const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + base);
        float4 f0 = p[0], f1 = p[1];
        vm = max(max(max(__float_as_uint(f0.x) & 0x7fffffffu, __float_as_uint(f0.y) & 0x7fffffffu),
                     max(__float_as_uint(f0.z) & 0x7fffffffu, __float_as_uint(f0.w) & 0x7fffffffu)),
                 max(max(__float_as_uint(f1.x) & 0x7fffffffu, __float_as_uint(f1.y) & 0x7fffffffu),
                     max(__float_as_uint(f1.z) & 0x7fffffffu, __float_as_uint(f1.w) & 0x7fffffffu)));
      } else {
        uint4 b = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(a.x) + base);
        // bf16 magnitude bits order like the floats they widen to
        uint32_t w0 = b.x & 0x7fff7fffu, w1 = b.y & 0x7fff7fffu, w2 = b.z & 0x7fff7fffu,
                 w3 = b.w & 0x7fff7fffu;
        vm = max(max(max(w0 & 0xffffu, w0 >> 16), max(w1 & 0xffffu, w1 >> 16)),
                 max(max(w2 & 0xffffu, w2 >> 16), max(w3 & 0xffffu, w3 >> 16))) << 16;
      }
      if (n != cur_n) {
        if (cur_n >= 0) atomicMax(&amax_s[cur_n], m);
        m = 0;
        cur_n = n;
      }
      m = max(m, vm);
    }
    if (cur_n >= 0) atomicMax(&amax_s[cur_n], m);
  }
  __syncthreads();
  if (tid < 16) {
    int F = prescale_exponent(amax_s[tid]);
    unscale_s[tid] = __uint_as_float((uint32_t)(127 - F) << 23);
  }
  // Pass 2: scale by 2^F (exact), convert to f16 (hi, and lo for f32 input).
#pragma unroll 2
  for (int e = tid; e < n_entries; e += blockDim.x) {
    int q = e & 3;
    int t = e >> 2;
    int n = t % batch;
    int cj = t / batch;  // c * 8 + j
    int c = cj >> 3, j = cj & 7;
    int k = c * 128 + q * 32 + 4 * j;
    uint2 hi = make_uint2(0, 0), lo = make_uint2(0, 0);
    if (k < K) {
      float up = __uint_as_float((uint32_t)(127 + prescale_exponent(amax_s[n])) << 23);
      float v[4];
      if (XLO) {
        float4 f = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + x_off +
                                                     (long long)n * K + k);
        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
      } else {
        uint2 b = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(a.x) + x_off +
                                                   (long long)n * K + k);
        v[0] = __uint_as_float(b.x << 16); v[1] = __uint_as_float(b.x & 0xffff0000u);
        v[2] = __uint_as_float(b.y << 16); v[3] = __uint_as_float(b.y & 0xffff0000u);
      }
#pragma unroll
      for (int t2 = 0; t2 < 4; ++t2) v[t2] = v[t2] * up;
      hi.x = pack_half2(v[0], v[1]);
      hi.y = pack_half2(v[2], v[3]);
      if (XLO) {
        __half2 h01 = *reinterpret_cast<__half2 *>(&hi.x), h23 = *reinterpret_cast<__half2 *>(&hi.y);
        float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        lo.x = pack_half2(v[0] - f01.x, v[1] - f01.y);
        lo.y = pack_half2(v[2] - f23.x, v[3] - f23.y);
      }
    }
    xs_hi[e] = hi;
    if (XLO) xs_lo[e] = lo;
  }
  __syncthreads();

  for (int it = 0; it < a.iters; ++it) {
    uint4 wnext[2][C];
    uint16_t snext[2][C];
    if (it + 1 < a.iters) load(it + 1, wnext, snext);

    float acc[NG][4];
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) acc[ng][0] = acc[ng][1] = acc[ng][2] = acc[ng][3] = 0.0f;

#pragma unroll
    for (int cc = 0; cc < C; ++cc) {
      const int c = c_begin + cc;
      if (!(warp_active && c < chunks)) continue;
      uint32_t h[2][16];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t sc = e4m3x2_to_f16x2(scur[hh][cc]);
        uint32_t s_lo = __byte_perm(sc, sc, 0x1010), s_hi = __byte_perm(sc, sc, 0x3232);
        uint32_t words[4] = {wcur[hh][cc].x, wcur[hh][cc].y, wcur[hh][cc].z, wcur[hh][cc].w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          uint32_t f[4];
          e2m1x8_to_f16x8(words[wi], f);
#pragma unroll
          for (int t = 0; t < 4; ++t) h[hh][wi * 4 + t] = hmul2(f[t], wi < 2 ? s_lo : s_hi);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
          const int n = ng * 8 + g;
          const int idx = ((c * 8 + j) * batch + n) * 4 + q;
          uint2 b = n < batch ? xs_hi[idx] : make_uint2(0, 0);
          mma_f16(acc[ng], h[0][2 * j], h[1][2 * j], h[0][2 * j + 1], h[1][2 * j + 1], b.x, b.y);
          if (XLO) {
            uint2 bb = n < batch ? xs_lo[idx] : make_uint2(0, 0);
            mma_f16(acc[ng], h[0][2 * j], h[1][2 * j], h[0][2 * j + 1], h[1][2 * j + 1], bb.x, bb.y);
          }
        }
      }
    }

    // ---- cross-warp reduction and epilogue ---------------------------------
    if (warp_active) {
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
        red[((gi * wk_count + wk) * NG + ng) * 32 + lane] =
            make_float4(acc[ng][0], acc[ng][1], acc[ng][2], acc[ng][3]);
    }
    __syncthreads();
    const int rb = (it * gridDim.x + blockIdx.x) * g_count + gi;
    if (warp_active && wk == 0 && rb < a.nrb) {
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) {
        float4 sum = red[((gi * wk_count) * NG + ng) * 32 + lane];
        for (int w = 1; w < wk_count; ++w) {
          float4 p = red[((gi * wk_count + w) * NG + ng) * 32 + lane];
          sum.x += p.x; sum.y += p.y; sum.z += p.z; sum.w += p.w;
        }
        const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          int r = rb * 16 + g + ((t >> 1) << 3);
          int n = ng * 8 + 2 * q + (t & 1);
          if (r < a.rows && n < a.batch) {
            float v = slot_ok ? (vals[t] * unscale_s[n]) * globals[r] : 0.0f;
            long long off = (long long)slot * a.y_slot_stride + (long long)n * a.y_batch_stride + r;
            if (a.y_bf16)
              reinterpret_cast<__nv_bfloat16 *>(a.y)[off] = __float2bfloat16_rn(v);
            else
              reinterpret_cast<float *>(a.y)[off] = v;
          }
        }
      }
    }
    __syncthreads();
    if (it + 1 < a.iters) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int cc = 0; cc < C; ++cc) {
          wcur[hh][cc] = wnext[hh][cc];
          scur[hh][cc] = snext[hh][cc];
        }
    }
  }
}

// ---- host dispatch -----------------------------------------------------------
struct GemvConfig {
  int C, wk, g, threads;
};

constexpr size_t kGemvSmemLimit = 200 * 1024;

static GemvConfig pick_config(int K);

// Dynamic shared memory of one launch: the compact B fragments (2 bytes per
// element of x, twice for f32 input) and the cross-warp reduction buffer.
static size_t gemv_smem_bytes(int K, int batch, bool x_f32) {
  GemvConfig cfg = pick_config(K);
  size_t chunks = (size_t)(K + 127) / 128;
  size_t frag = chunks * 8 * (size_t)batch * 4 * sizeof(uint2) * (x_f32 ? 2 : 1);
  size_t red = (size_t)cfg.wk * cfg.g * (batch > 8 ? 2 : 1) * 32 * sizeof(float4);
  return frag + red;
}

// Largest batch per launch whose staging fits in shared memory.
static int gemv_max_batch(int K, bool x_f32) {
  int b = 16;
  while (b > 1 && gemv_smem_bytes(K, b, x_f32) > kGemvSmemLimit) --b;
  return b;
}

static GemvConfig pick_config(int K) {
  int chunks = (K + 127) / 128;
  int C = 1;
  while ((chunks + C - 1) / C > 8 && C < 8) C *= 2;
  int wk = (chunks + C - 1) / C;
  if (wk > 8) return {0, 0, 0, 0};
  int g = wk <= 8 ? std::max(1, 8 / wk) : 1;
  return {C, wk, g, wk * g * 32};
}

using GemvKernel = void (*)(GemvArgs);

template <int C, int NG, bool XLO>
static GemvKernel kernel_for() {
  return gemv_nvfp4_kernel<C, NG, XLO>;
}

static GemvKernel select_kernel(int C, int NG, bool xlo) {
#define FPB_GEMV_CASE(c)                                                     \
  if (C == c) {                                                              \
    if (NG == 1) return xlo ? kernel_for<c, 1, true>() : kernel_for<c, 1, false>(); \
    return xlo ? kernel_for<c, 2, true>() : kernel_for<c, 2, false>();       \
  }
  FPB_GEMV_CASE(1)
  FPB_GEMV_CASE(2)
  FPB_GEMV_CASE(4)
  FPB_GEMV_CASE(8)
#undef FPB_GEMV_CASE
  return nullptr;
}

static int run_gemv(GemvArgs args, int slots, bool x_f32, cudaStream_t stream) {
  GemvConfig cfg = pick_config(args.K);
  if (!cfg.C) return fail(FPB_ERR_UNSUPPORTED, "NVFP4 GEMV: K=%d exceeds 8192", args.K);
  args.chunks = (args.K + 127) / 128;
  args.nrb = (args.rows + 15) / 16;
  int NG = args.batch > 8 ? 2 : 1;
  size_t smem = gemv_smem_bytes(args.K, args.batch, x_f32);
  if (smem > kGemvSmemLimit)
    return fail(FPB_ERR_UNSUPPORTED, "NVFP4 GEMV: x staging needs %zu bytes", smem);
  GemvKernel k = select_kernel(cfg.C, NG, x_f32);
  if (!k) return fail(FPB_ERR_UNSUPPORTED, "NVFP4 GEMV: no kernel for C=%d", cfg.C);

  // Kernel attributes and occupancy are queried once per (device, kernel,
  // block size, shared memory) so that repeated calls, including calls made
  // while a stream is being captured into a CUDA graph, issue no extra
  // runtime calls.
  struct OccKey {
    int dev;
    GemvKernel k;
    int threads;
    size_t smem;
  };
  struct OccEntry {
    OccKey key;
    int occ;
  };
  static std::mutex mu;
  static std::vector<OccEntry> occ_cache;
  static std::vector<std::pair<std::pair<int, GemvKernel>, size_t>> smem_set;
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    size_t have = 0;
    for (auto &p : smem_set)
      if (p.first.first == dev && p.first.second == k) have = p.second;
    if (have < smem) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
      smem_set.push_back({{dev, k}, smem});
    }
    for (auto &o : occ_cache)
      if (o.key.dev == dev && o.key.k == k && o.key.threads == cfg.threads && o.key.smem == smem) occ = o.occ;
    if (occ == 0) {
      cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, cfg.threads, smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      if (occ < 1) occ = 1;
      occ_cache.push_back({{dev, k, cfg.threads, smem}, occ});
    }
  }
  int groups = (args.nrb + cfg.g - 1) / cfg.g;
  long long resident = (long long)occ * sm_count();
  long long per_slot = std::max(1LL, resident / std::max(1, slots));
  int grid_x = (int)std::min<long long>(groups, per_slot);
  args.iters = (groups + grid_x - 1) / grid_x;
  dim3 grid(grid_x, slots);
  cudaLaunchConfig_t lc{};
  lc.gridDim = grid;
  lc.blockDim = dim3(cfg.threads);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&lc, k, args);
  if (le != cudaSuccess) return cuda_fail(le, "cudaLaunchKernelEx(gemv_nvfp4_kernel)");
  FPB_LAUNCH_CHECK("gemv_nvfp4_kernel");
  return FPB_OK;
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
  GemvArgs a{};
  a.packed = w->packed + row_begin * (w->cols / 2);
  a.scales = w->scales + row_begin * (w->cols / kNvfp4Group);
  a.globals = w->row_globals + row_begin;
  a.x = x;
  a.y = y;
  a.expert_ids = nullptr;
  a.rows = (int)(row_end - row_begin);
  a.K = (int)w->cols;
  a.y_bf16 = y_dtype == FPB_BF16;
  a.y_batch_stride = a.rows;
  a.x_slot_stride = 0;
  a.y_slot_stride = 0;
  bool x_f32 = x_dtype == FPB_F32;
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_gemv: x must be 16-byte aligned");
  if (w->cols > 8192) return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemv: cols %zu > 8192", w->cols);
  // x is staged whole in shared memory; batches whose staging does not fit
  // run as several launches over row groups of x (each re-reads W).
  int step = std::min(batch, gemv_max_batch((int)w->cols, x_f32));
  if (gemv_smem_bytes((int)w->cols, 1, x_f32) > kGemvSmemLimit)
    return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_gemv: cols %zu too large for x staging", w->cols);
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
  if (w->cols > 8192) return fail(FPB_ERR_UNSUPPORTED, "fpb_nvfp4_expert_gemv: cols %zu > 8192", w->cols);
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
  a.y_slot_stride = (long long)rows_per_expert;
  return run_gemv(a, slots, x_dtype == FPB_F32, as_stream(stream));
}
