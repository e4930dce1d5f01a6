// NVFP4 quantize and dequantize.
//
// The reference receives NVFP4 weights already quantized (ModelOpt
// checkpoints) and has no quantizer; the rule implemented here is the one the
// task's configs state: per block of rows a global g = amax / (6*448); per 16
// columns s = RN_e4m3_satfinite((block_amax / 6) / g); each value
// RN_e2m1_satfinite(w / (e4m3(s) * g)).  Every step is one IEEE binary32
// operation, so the CPU oracle reproduces the codes bit for bit.
//
// Dequantize follows ModelOpt's order E2M1[c] * (e4m3(s) * g), with code 0x8
// decoding to +0 (crates/firepit/src/checkpoint.rs:386-420).
#include "common.cuh"
#include "nvfp4_matrix.cuh"

namespace fpb {

template <typename T>
__device__ __forceinline__ float load_as_f32(const T *p, size_t i);
template <>
__device__ __forceinline__ float load_as_f32<float>(const float *p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_as_f32<uint16_t>(const uint16_t *p, size_t i) {
  return bf16_bits_to_f32(p[i]);
}

// amax over each block of `block_elems` consecutive elements.  |x| is
// compared as unsigned bits, which orders non-negative floats and puts Inf
// and NaN above every finite value (so a non-finite input poisons the global).
template <typename T>
__global__ void amax_kernel(const T *w, size_t block_elems, size_t chunk, size_t chunks_per_block,
                            uint32_t *amax_bits) {
  size_t cta = blockIdx.x;
  size_t blk = cta / chunks_per_block;
  size_t begin = blk * block_elems + (cta % chunks_per_block) * chunk;
  size_t end = begin + chunk;
  size_t block_end = (blk + 1) * block_elems;
  if (end > block_end) end = block_end;
  uint32_t m = 0;
  for (size_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
    uint32_t b = __float_as_uint(load_as_f32(w, i)) & 0x7fffffffu;
    m = max(m, b);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ uint32_t warp_max_s[32];
  if ((threadIdx.x & 31) == 0) warp_max_s[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t r = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = max(r, warp_max_s[i]);
    atomicMax(amax_bits + blk, r);
  }
}

// One thread per 16-column group.
template <typename T>
__global__ void nvfp4_encode_kernel(const T *w, size_t rows, size_t cols, size_t rows_per_global,
                                    const uint32_t *amax_bits, uint8_t *packed, uint8_t *scales,
                                    float *row_globals) {
  size_t groups_per_row = cols / kNvfp4Group;
  size_t n_groups = rows * groups_per_row;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t gi = (size_t)blockIdx.x * blockDim.x + threadIdx.x; gi < n_groups; gi += stride) {
    size_t r = gi / groups_per_row;
    size_t g = gi - r * groups_per_row;
    float amax = __uint_as_float(amax_bits[r / rows_per_global]);
    float global = __fdiv_rn(amax, 2688.0f);  // amax / (6 * 448)
    float v[kNvfp4Group];
    const T *src = w + r * cols + g * kNvfp4Group;
#pragma unroll
    for (int i = 0; i < kNvfp4Group; ++i) v[i] = load_as_f32(src, i);
    float bmax = 0.0f;
#pragma unroll
    for (int i = 0; i < kNvfp4Group; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
    uint8_t s = 0;
    if (global > 0.0f) s = f32_to_e4m3(__fdiv_rn(__fdiv_rn(bmax, 6.0f), global));
    float denom = __fmul_rn(e4m3_to_f32(s), global);
    uint32_t lo = 0, hi = 0;
    if (denom > 0.0f) {
      float q[kNvfp4Group];
  #pragma unroll
    for (int i = 0; i < 16; ++i) q[i] = __fdiv_rn(v[i], denom);
      lo = f32x8_to_e2m1x8(q);
      hi = f32x8_to_e2m1x8(q + 8);
    }
    *reinterpret_cast<uint2 *>(packed + r * (cols / 2) + g * (kNvfp4Group / 2)) = make_uint2(lo, hi);
    scales[gi] = s;
    if (g == 0) row_globals[r] = global;
  }
}

__global__ void nvfp4_dequant_kernel(const uint8_t *packed, const uint8_t *scales,
                                     const float *row_globals, size_t rows, size_t cols,
                                     float *out) {
  size_t n = rows * cols / 2;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    size_t r = (2 * i) / cols;
    size_t c = 2 * i - r * cols;
    float sg = __fmul_rn(e4m3_to_f32(scales[r * (cols / kNvfp4Group) + c / kNvfp4Group]),
                         row_globals[r]);
    uint32_t byte = packed[i];
    uint32_t lo = byte & 0xf, hi = byte >> 4;
    float wl = (lo == 8) ? 0.0f : e2m1_to_f32(lo);
    float wh = (hi == 8) ? 0.0f : e2m1_to_f32(hi);
    out[r * cols + c] = __fmul_rn(wl, sg);
    out[r * cols + c + 1] = __fmul_rn(wh, sg);
  }
}

template <typename T>
static int quantize_impl(const T *w, size_t rows, size_t cols, size_t rpg, uint8_t *packed,
                         uint8_t *scales, float *row_globals, float *amax_scratch, cudaStream_t s) {
  size_t n_blocks = rows / rpg;
  uint32_t *amax_bits = reinterpret_cast<uint32_t *>(amax_scratch);
  FPB_CUDA_TRY(cudaMemsetAsync(amax_bits, 0, n_blocks * sizeof(uint32_t), s));
  size_t block_elems = rpg * cols;
  size_t chunk = 16384;
  size_t chunks_per_block = (block_elems + chunk - 1) / chunk;
  size_t ctas = n_blocks * chunks_per_block;
  if (ctas > 0x7fffffffu) return fail(FPB_ERR_UNSUPPORTED, "quantize: matrix too large");
  amax_kernel<T><<<(unsigned)ctas, 256, 0, s>>>(w, block_elems, chunk, chunks_per_block, amax_bits);
  FPB_LAUNCH_CHECK("amax_kernel");
  size_t groups = rows * cols / kNvfp4Group;
  size_t grid = (groups + 255) / 256;
  size_t cap = (size_t)sm_count() * 32;
  if (grid > cap) grid = cap;
  nvfp4_encode_kernel<T><<<(unsigned)grid, 256, 0, s>>>(w, rows, cols, rpg, amax_bits, packed,
                                                        scales, row_globals);
  FPB_LAUNCH_CHECK("nvfp4_encode_kernel");
  return FPB_OK;
}

}  // namespace fpb

using namespace fpb;

extern "C" int fpb_nvfp4_quantize(const void *w, int w_dtype, size_t rows, size_t cols,
                                  size_t rows_per_global, uint8_t *packed, uint8_t *scales,
                                  float *row_globals, float *amax_scratch, void *stream) {
  if (!w || !packed || !scales || !row_globals || !amax_scratch)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_quantize: null pointer");
  if (rows == 0 || cols == 0 || cols % kQ8Block != 0)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_quantize: cols must be a positive multiple of %d", kQ8Block);
  if (rows_per_global == 0 || rows % rows_per_global != 0)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_quantize: rows_per_global must divide rows");
  cudaStream_t s = as_stream(stream);
  if (w_dtype == FPB_F32)
    return quantize_impl(static_cast<const float *>(w), rows, cols, rows_per_global, packed, scales,
                         row_globals, amax_scratch, s);
  if (w_dtype == FPB_BF16)
    return quantize_impl(static_cast<const uint16_t *>(w), rows, cols, rows_per_global, packed,
                         scales, row_globals, amax_scratch, s);
  return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_quantize: dtype %d", w_dtype);
}

extern "C" int fpb_nvfp4_dequantize(const fpb_nvfp4_matrix *m, float *out, void *stream) {
  if (!m || !out) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_dequantize: null pointer");
  size_t n = m->rows * m->cols / 2;
  size_t grid = (n + 255) / 256, cap = (size_t)sm_count() * 32;
  if (grid > cap) grid = cap;
  nvfp4_dequant_kernel<<<(unsigned)grid, 256, 0, as_stream(stream)>>>(
      m->packed, m->scales, m->row_globals, m->rows, m->cols, out);
  FPB_LAUNCH_CHECK("nvfp4_dequant_kernel");
  return FPB_OK;
}

// ---- quantize without allocating ------------------------------------------------------
// fpb_nvfp4_quantize needs a caller-provided scratch buffer for its per-block
// amax.  Some callers cannot allocate one: an engine that carves all device
// memory out of a single arena reserved at start-up and forbids any further
// cudaMalloc, or a serving loop where an allocation would synchronise the
// device mid-step.  For them the same quantizer runs on a fixed scratch array
// compiled into this library: kNoAllocMaxBlocks words, 64 KiB, which every
// GPU that loads the library keeps until the process exits.
#include <cuda.h>

#include <mutex>
#include <utility>
#include <vector>

namespace fpb {

constexpr size_t kNoAllocMaxBlocks = 16384;  // row blocks (one global each) per call
static __device__ __align__(256) uint32_t g_noalloc_amax[kNoAllocMaxBlocks];

// The array's device address in the current context.  In host code the
// array's name only stands in for it, so the address is looked up with
// cudaGetSymbolAddress (the device current) and cached per context: the key
// is the driver's unique context id (cuCtxGetId, never reused within a
// process), so a context re-created after cudaDeviceReset gets a fresh
// lookup instead of a stale address.
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

static int current_context_id(unsigned long long *id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return fail(FPB_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return fail(FPB_ERR_CUDA, "no current CUDA context");
  if (get_id(ctx, id) != CUDA_SUCCESS) return fail(FPB_ERR_CUDA, "cuCtxGetId failed");
  return FPB_OK;
}

static int noalloc_scratch(float **out) {
  static std::mutex mu;
  static std::vector<std::pair<unsigned long long, float *>> by_context;
  // cudaSetDevice makes the device's primary context current (initialising
  // it if needed), so the driver's current context is the runtime's.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  unsigned long long ctx = 0;
  int st = current_context_id(&ctx);
  if (st) return st;
  std::lock_guard<std::mutex> lock(mu);
  for (auto &entry : by_context)
    if (entry.first == ctx) {
      *out = entry.second;
      return FPB_OK;
    }
  void *p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_amax);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc quantize scratch)");
  by_context.push_back({ctx, static_cast<float *>(p)});
  *out = static_cast<float *>(p);
  return FPB_OK;
}

}  // namespace fpb

extern "C" int fpb_nvfp4_quantize_noalloc(const void *w, int w_dtype, size_t rows, size_t cols,
                                          size_t rows_per_global, uint8_t *packed, uint8_t *scales,
                                          float *row_globals, void *stream) {
  if (!w || !packed || !scales || !row_globals)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_quantize_noalloc: null pointer");
  if (rows == 0 || cols == 0 || cols % kQ8Block != 0)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_quantize_noalloc: cols must be a positive multiple of %d", kQ8Block);
  if (rows_per_global == 0 || rows % rows_per_global != 0)
    return fail(FPB_ERR_SHAPE, "fpb_nvfp4_quantize_noalloc: rows_per_global must divide rows");
  if (rows / rows_per_global > kNoAllocMaxBlocks)
    return fail(FPB_ERR_UNSUPPORTED,
                "fpb_nvfp4_quantize_noalloc: %zu row blocks exceed the built-in scratch of %zu; "
                "use fpb_nvfp4_quantize with a scratch buffer",
                rows / rows_per_global, kNoAllocMaxBlocks);
  if (w_dtype != FPB_F32 && w_dtype != FPB_BF16)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_quantize_noalloc: dtype %d", w_dtype);
  float *scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st) return st;
  // quantize_impl zeroes the amax words it uses before its first launch.
  cudaStream_t s = as_stream(stream);
  if (w_dtype == FPB_F32)
    return quantize_impl(static_cast<const float *>(w), rows, cols, rows_per_global, packed, scales,
                         row_globals, scratch, s);
  return quantize_impl(static_cast<const uint16_t *>(w), rows, cols, rows_per_global, packed, scales,
                       row_globals, scratch, s);
}
