// Decode GEMV on FP8 E4M3 weights (crates/firepit-kernels/src/gemv/fp8.rs):
// dense (dense_fp8_kernel / dense_fp8_rows_kernel, :13-54 and :108-132) and
// expert (expert_fp8_kernel / expert_fp8_rows_kernel, :56-106 and :134-160)
// over the FP8 matrix handle of fp8.cu, with 128x128-style block scales or
// one scale per row.
//
//   blocks: y[b, r] = sum_kb s[r / bn, kb] * sum_{k in kb} w[r, k] * x[b, k]
//   rows:   y[b, r] = s[r] * sum_k w[r, k] * x[b, k]
//
// Memory-bound: a warp owns one weight row and streams it with 16-byte loads
// (lane l takes the 16-column chunks l, l + 32, ...; four chunks in flight
// per lane), converts e4m3 pairs to f16x2 (exact) and then to f32, and
// accumulates in f32.  With block scales each lane multiplies the partial sum
// of a chunk by its block's scale before the cross-lane reduction (a chunk
// never straddles a block: block_k % 16 == 0), so the scale distributes over
// the block's sum as in the reference, in a different f32 order.  x is read
// through L1 (every warp of a CTA reads the same x).
#include <cuda_bf16.h>

#include "common.cuh"
#include "fp8_matrix.cuh"

namespace fpb {
namespace {

constexpr int kFp8GemvWarps = 8;   // rows per CTA (one per warp)
constexpr int kFp8GemvUnroll = 4;  // 16-byte chunks in flight per lane

struct Fp8GemvArgs {
  const uint8_t *bits;
  const float *scales;
  size_t cols;
  int block_n, block_k;       // 0, 0: one scale per row
  size_t ws_cols;             // scale-grid columns (blocks)
  const void *x;
  long long x_batch_stride;   // elements between batch rows
  void *y;
  long long y_batch_stride;   // elements between y rows
  int batch;
  int nrows;                  // rows per slot (expert) or of the view (dense)
  long long row_begin;        // dense: first matrix row
  const int32_t *expert_ids;
  int n_experts;
  long long x_slot_stride;    // expert: x row of slot s = s * x_slot_stride
};

__device__ __forceinline__ void load16_x(const float *p, float v[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 f = __ldg(reinterpret_cast<const float4 *>(p) + q);
    v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
  }
}
__device__ __forceinline__ void load16_x(const __nv_bfloat16 *p, float v[16]) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p) + q);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[8 * q + 2 * t] = __uint_as_float(w[t] << 16);
      v[8 * q + 2 * t + 1] = __uint_as_float(w[t] & 0xffff0000u);
    }
  }
}

// 16 e4m3 bytes -> 16 f32 (via f16x2, exact).
__device__ __forceinline__ void decode16(const uint4 w, float f[16]) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t p = e4m3x2_to_f16x2((uint16_t)(words[i] >> (16 * h)));
      const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&p));
      f[4 * i + 2 * h] = v.x;
      f[4 * i + 2 * h + 1] = v.y;
    }
  }
}

template <typename XT, typename YT, int B>
__global__ void __launch_bounds__(kFp8GemvWarps * 32, B == 1 ? 4 : 1) fp8_gemv_kernel(Fp8GemvArgs a) {
  const int lane = threadIdx.x & 31;
  const int r_local = blockIdx.x * kFp8GemvWarps + (threadIdx.x >> 5);
  if (r_local >= a.nrows) {  // warp-uniform; still releases the next launch
    asm volatile("griddepcontrol.launch_dependents;");
    return;
  }
  const int slot = blockIdx.y;
  // In expert mode the ids that pick the weight rows may come from the
  // previous kernel in the stream (the router top-k), so they are read only
  // after griddepcontrol.wait; the dense path requests its first weight
  // chunks before the wait (weights are immutable while their handle exists).
  const bool dense = a.expert_ids == nullptr;
  if (!dense) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }
  long long row;
  bool ok = true;
  if (!dense) {
    const int e = a.expert_ids[slot];
    ok = e >= 0 && e < a.n_experts;  // a bad id yields zeros, as the NVFP4 expert GEMV
    row = (long long)(ok ? e : 0) * a.nrows + r_local;
  } else {
    row = a.row_begin + r_local;
  }
  const XT *x = static_cast<const XT *>(a.x) + (long long)slot * a.x_slot_stride;
  const uint8_t *wrow = a.bits + (size_t)row * a.cols;
  const bool blocks = a.block_n != 0;
  const float *srow = blocks ? a.scales + (size_t)(row / a.block_n) * a.ws_cols : nullptr;
  const int chunks = (int)(a.cols / 16);

  float acc[B];
#pragma unroll
  for (int b = 0; b < B; ++b) acc[b] = 0.0f;
  // Programmatic dependent launch (dense): the weights (and scales) are
  // immutable while their handle exists, so the first chunks are requested
  // before waiting for the previous kernel in the stream; x is read and y
  // written only after it.
  uint4 w[kFp8GemvUnroll];
  auto load_w = [&](int c0) {
#pragma unroll
    for (int u = 0; u < kFp8GemvUnroll; ++u) {
      const int c = c0 + 32 * u;
      w[u] = c < chunks ? __ldg(reinterpret_cast<const uint4 *>(wrow) + c) : make_uint4(0, 0, 0, 0);
    }
  };
  load_w(lane);
  if (dense) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }
  for (int c0 = lane; c0 < chunks; c0 += 32 * kFp8GemvUnroll) {
    if (c0 != lane) load_w(c0);
#pragma unroll
    for (int u = 0; u < kFp8GemvUnroll; ++u) {
      const int c = c0 + 32 * u;
      if (c >= chunks) break;
      float f[16];
      decode16(w[u], f);
      const float s = blocks ? __ldg(srow + (size_t)(c * 16) / a.block_k) : 1.0f;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b >= a.batch) break;
        float xv[16];
        load16_x(x + (long long)b * a.x_batch_stride + (long long)c * 16, xv);
        float p = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) p = fmaf(f[i], xv[i], p);
        acc[b] = fmaf(p, s, acc[b]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
  }
  if (lane == 0) {
    const float rs = blocks ? 1.0f : a.scales[row];
    YT *y = static_cast<YT *>(a.y) + (long long)slot * a.y_batch_stride;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (b >= a.batch) break;
      const float v = ok ? acc[b] * rs : 0.0f;
      if constexpr (sizeof(YT) == 4)
        y[(long long)b * a.y_batch_stride + r_local] = v;
      else
        y[(long long)b * a.y_batch_stride + r_local] = __float2bfloat16_rn(v);
    }
  }
}

template <typename XT, typename YT>
int launch_b(const Fp8GemvArgs &a, int slots, cudaStream_t s) {
  void (*k)(Fp8GemvArgs) = a.batch <= 1   ? fp8_gemv_kernel<XT, YT, 1>
                           : a.batch <= 2 ? fp8_gemv_kernel<XT, YT, 2>
                           : a.batch <= 4 ? fp8_gemv_kernel<XT, YT, 4>
                           : a.batch <= 8 ? fp8_gemv_kernel<XT, YT, 8>
                                          : fp8_gemv_kernel<XT, YT, 16>;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3((unsigned)((a.nrows + kFp8GemvWarps - 1) / kFp8GemvWarps), (unsigned)slots);
  lc.blockDim = dim3(kFp8GemvWarps * 32);
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&lc, k, a);
  if (le == cudaErrorInvalidValue) {  // no programmatic launch here: a plain launch
    cudaGetLastError();
    lc.numAttrs = 0;
    le = cudaLaunchKernelEx(&lc, k, a);
  }
  if (le != cudaSuccess) {
    cudaGetLastError();
    return fail(FPB_ERR_CUDA, "cudaLaunchKernelEx(fp8_gemv_kernel): %s", cudaGetErrorName(le));
  }
  FPB_LAUNCH_CHECK("fp8_gemv_kernel");
  return FPB_OK;
}

int launch(const Fp8GemvArgs &a, int x_dtype, int y_dtype, int slots, cudaStream_t s) {
  if (x_dtype == FPB_F32 && y_dtype == FPB_F32) return launch_b<float, float>(a, slots, s);
  if (x_dtype == FPB_F32 && y_dtype == FPB_BF16) return launch_b<float, __nv_bfloat16>(a, slots, s);
  if (x_dtype == FPB_BF16 && y_dtype == FPB_F32) return launch_b<__nv_bfloat16, float>(a, slots, s);
  if (x_dtype == FPB_BF16 && y_dtype == FPB_BF16) return launch_b<__nv_bfloat16, __nv_bfloat16>(a, slots, s);
  return fail(FPB_ERR_INVALID_ARGUMENT, "FP8 GEMV: dtype");
}

int common_checks(const fpb_fp8_matrix *w, const void *x, const void *y, const char *what) {
  if (!w || !x || !y) return fail(FPB_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  if (w->cols % 32 != 0) return fail(FPB_ERR_SHAPE, "%s: cols %zu not a multiple of 32", what, w->cols);
  if (w->block_n != 0 && w->block_k % 16 != 0)
    return fail(FPB_ERR_UNSUPPORTED, "%s: block_k %d not a multiple of 16", what, w->block_k);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w->bits) & 15))
    return fail(FPB_ERR_INVALID_ARGUMENT, "%s: x and the weights must be 16-byte aligned", what);
  return FPB_OK;
}

Fp8GemvArgs base_args(const fpb_fp8_matrix *w) {
  Fp8GemvArgs a{};
  a.bits = w->bits;
  a.scales = w->scales;
  a.cols = w->cols;
  a.block_n = w->block_n;
  a.block_k = w->block_k;
  a.ws_cols = w->block_n ? w->cols / (size_t)w->block_k : 0;
  return a;
}

}  // namespace
}  // namespace fpb

using namespace fpb;

extern "C" int fpb_fp8_gemv(const fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                            void *y, int y_dtype, int batch, void *stream) {
  int st = common_checks(w, x, y, "fpb_fp8_gemv");
  if (st) return st;
  if (row_end == 0) row_end = w->rows;
  if (row_begin >= row_end || row_end > w->rows || row_end - row_begin > 0x7fffffff)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_gemv: rows [%zu, %zu) of %zu", row_begin, row_end, w->rows);
  if (batch < 1 || batch > 16) return fail(FPB_ERR_SHAPE, "fpb_fp8_gemv: batch %d (1..16)", batch);
  Fp8GemvArgs a = base_args(w);
  a.x = x;
  a.x_batch_stride = (long long)w->cols;
  a.y = y;
  a.y_batch_stride = (long long)(row_end - row_begin);
  a.batch = batch;
  a.nrows = (int)(row_end - row_begin);
  a.row_begin = (long long)row_begin;
  return launch(a, x_dtype, y_dtype, 1, as_stream(stream));
}

extern "C" int fpb_fp8_expert_gemv(const fpb_fp8_matrix *w, const void *x, int x_dtype, const int32_t *expert_ids,
                                   int slots, size_t rows_per_expert, int input_stride, void *y, int y_dtype,
                                   void *stream) {
  int st = common_checks(w, x, y, "fpb_fp8_expert_gemv");
  if (st) return st;
  if (!expert_ids) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_fp8_expert_gemv: null expert ids");
  if (slots < 1 || slots > 65535 || rows_per_expert == 0 || w->rows % rows_per_expert != 0 ||
      rows_per_expert > 0x7fffffff || input_stride < 0)
    return fail(FPB_ERR_SHAPE, "fpb_fp8_expert_gemv: %d slots, %zu rows per expert of %zu", slots, rows_per_expert,
                w->rows);
  if (w->block_n != 0 && rows_per_expert % (size_t)w->block_n != 0)  // gemv/fp8.rs:264
    return fail(FPB_ERR_SHAPE, "fpb_fp8_expert_gemv: rows per expert %zu not a multiple of block_n %d",
                rows_per_expert, w->block_n);
  Fp8GemvArgs a = base_args(w);
  a.x = x;
  a.x_batch_stride = 0;
  a.x_slot_stride = (long long)input_stride * (long long)w->cols;
  a.y = y;
  a.y_batch_stride = (long long)rows_per_expert;
  a.batch = 1;
  a.nrows = (int)rows_per_expert;
  a.expert_ids = expert_ids;
  a.n_experts = (int)(w->rows / rows_per_expert);
  return launch(a, x_dtype, y_dtype, slots, as_stream(stream));
}
