// Library core: status/error plumbing, scalar codecs on the host, and the
// NVFP4 weight-matrix handle (HostNvfp4Matrix / Nvfp4Matrix of
// crates/firepit-kernels/src/weights/nvfp4.rs).
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "matrix_extras.cuh"
#include "nvfp4_matrix.cuh"

namespace fpb {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

int fail(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t err, const char *what) {
  cudaGetLastError();  // clear a non-sticky error so later calls can proceed
  return fail(err == cudaErrorNoDevice ? FPB_ERR_NO_DEVICE : FPB_ERR_CUDA, "%s: %s (%s)", what,
              cudaGetErrorString(err), cudaGetErrorName(err));
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// ---- host codecs (same arithmetic as the device conversions) ---------------
static const float kE2m1Mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float host_e2m1(uint8_t code) {
  float m = kE2m1Mag[code & 7];
  return (code & 8) ? -m : m;
}

float host_e4m3(uint8_t bits) {
  float sign = (bits & 0x80) ? -1.0f : 1.0f;
  int e = (bits >> 3) & 0xf;
  float f = (float)(bits & 7);
  if (e == 0) return sign * f * ldexpf(1.0f, -9);
  return sign * (1.0f + f / 8.0f) * ldexpf(1.0f, e - 7);
}

static int round_to_quantum(float a, int q_exp) { return (int)nearbyintf(ldexpf(a, -q_exp)); }

uint8_t host_f32_to_e2m1(float v) {
  uint8_t sign = std::signbit(v) ? 8 : 0;
  float a = fabsf(v);
  if (std::isnan(v) || a >= 6.0f) return sign | 7;
  int e2 = 0;
  frexpf(a, &e2);
  int ex = (a == 0.0f) ? 0 : e2 - 1;
  if (ex < 0) ex = 0;
  int n = round_to_quantum(a, ex - 1);
  if (n == 0) return sign;
  if (ex == 0 && n < 2) return sign | (uint8_t)n;
  if (n == 4) { ex += 1; n = 2; }
  if (ex + 1 > 3) return sign | 7;
  return sign | (uint8_t)(((ex + 1) << 1) | (n - 2));
}

uint8_t host_f32_to_e4m3(float v) {
  uint8_t sign = std::signbit(v) ? 0x80 : 0;
  float a = fabsf(v);
  if (std::isnan(v)) return sign | 0x7f;
  if (a > 448.0f) return sign | 0x7e;
  int e2 = 0;
  frexpf(a, &e2);
  int ex = (a == 0.0f) ? -6 : e2 - 1;
  if (ex < -6) ex = -6;
  int n = round_to_quantum(a, ex - 3);
  if (n == 0) return sign;
  if (ex == -6 && n < 8) return sign | (uint8_t)n;
  if (n == 16) { ex += 1; n = 8; }
  int ef = ex + 7;
  if (ef > 15 || (ef == 15 && n > 14)) return sign | 0x7e;
  return sign | (uint8_t)((ef << 3) | (n - 8));
}

// ---- NVFP4 handle ----------------------------------------------------------
static bool is_nan_e4m3(uint8_t s) { return (s & 0x7f) == 0x7f; }  // weights/nvfp4.rs:42-44

int validate_nvfp4_host(size_t packed_len, const uint8_t *scales, size_t scales_len,
                        const float *row_globals, size_t rows, size_t cols) {
  // weights/nvfp4.rs:53-64
  if (rows == 0 || cols == 0 || cols % kQ8Block != 0)
    return fail(FPB_ERR_FORMAT, "invalid NVFP4 matrix: rows=%zu cols=%zu (cols must be a multiple of %d)",
                rows, cols, kQ8Block);
  if (packed_len != rows * (cols / 2) || scales_len != rows * (cols / kNvfp4Group))
    return fail(FPB_ERR_FORMAT, "invalid NVFP4 matrix: storage lengths do not match %zux%zu", rows,
                cols);
  for (size_t i = 0; i < scales_len; ++i)
    if (is_nan_e4m3(scales[i]))
      return fail(FPB_ERR_FORMAT, "invalid NVFP4 block scale: NaN e4m3 at index %zu", i);
  for (size_t r = 0; r < rows; ++r)
    if (!std::isfinite(row_globals[r]) || row_globals[r] < 0.0f)
      return fail(FPB_ERR_FORMAT, "invalid NVFP4 global scale %g at row %zu", (double)row_globals[r],
                  r);
  return FPB_OK;
}

__global__ void validate_nvfp4_kernel(const uint8_t *scales, size_t n_scales, const float *globals,
                                      size_t rows, int *bad) {
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_scales; i += stride)
    if ((scales[i] & 0x7f) == 0x7f) atomicOr(bad, 1);
  for (size_t r = (size_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += stride) {
    float g = globals[r];
    if (!(g >= 0.0f) || isinf(g)) atomicOr(bad, 2);
  }
}

static int alloc_matrix(size_t rows, size_t cols, fpb_nvfp4_matrix **out) {
  auto *m = new (std::nothrow) fpb_nvfp4_matrix();
  if (!m) return fail(FPB_ERR_INVALID_ARGUMENT, "out of host memory");
  m->rows = rows;
  m->cols = cols;
  cudaGetDevice(&m->device);
  cudaError_t e = cudaMalloc(&m->packed, rows * cols / 2);
  if (e == cudaSuccess) e = cudaMalloc(&m->scales, rows * cols / kNvfp4Group);
  if (e == cudaSuccess) e = cudaMalloc(&m->row_globals, rows * sizeof(float));
  if (e != cudaSuccess) {
    cudaFree(m->packed);
    cudaFree(m->scales);
    cudaFree(m->row_globals);
    delete m;
    return cuda_fail(e, "cudaMalloc(NVFP4 matrix)");
  }
  *out = m;
  return FPB_OK;
}

}  // namespace fpb

using namespace fpb;

extern "C" {

const char *fpb_version(void) { return "firepit_b200 0.1 (sm_100a)"; }

const char *fpb_status_string(int s) {
  switch (s) {
    case FPB_OK: return "ok";
    case FPB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FPB_ERR_SHAPE: return "shape mismatch";
    case FPB_ERR_FORMAT: return "invalid format";
    case FPB_ERR_CUDA: return "CUDA error";
    case FPB_ERR_UNSUPPORTED: return "unsupported shape";
    case FPB_ERR_SELECTION: return "invalid expert selection";
    case FPB_ERR_WORKSPACE: return "workspace too small";
    case FPB_ERR_NO_DEVICE: return "no CUDA device";
    case FPB_ERR_IO: return "I/O error";
    case FPB_ERR_COMM: return "communication error";
    default: return "unknown status";
  }
}

const char *fpb_last_error(void) { return g_last_error.c_str(); }
uint64_t fpb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

float fpb_e2m1_to_f32(uint8_t code) { return host_e2m1(code); }
float fpb_e4m3_to_f32(uint8_t bits) { return host_e4m3(bits); }
uint8_t fpb_f32_to_e2m1(float v) { return host_f32_to_e2m1(v); }
uint8_t fpb_f32_to_e4m3(float v) { return host_f32_to_e4m3(v); }

int fpb_nvfp4_validate(const uint8_t *packed, size_t packed_len, const uint8_t *scales,
                       size_t scales_len, const float *row_globals, size_t rows, size_t cols) {
  if (!packed || !scales || !row_globals)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_validate: null pointer");
  return validate_nvfp4_host(packed_len, scales, scales_len, row_globals, rows, cols);
}

int fpb_nvfp4_matrix_create(const uint8_t *packed, const uint8_t *scales, const float *row_globals,
                            size_t rows, size_t cols, void *stream, fpb_nvfp4_matrix **out) {
  if (!packed || !scales || !row_globals || !out)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_matrix_create: null pointer");
  *out = nullptr;
  if (rows == 0 || cols == 0 || cols % kQ8Block != 0)
    return fail(FPB_ERR_FORMAT, "invalid NVFP4 matrix: rows=%zu cols=%zu", rows, cols);
  int st = validate_nvfp4_host(rows * (cols / 2), scales, rows * (cols / kNvfp4Group), row_globals,
                               rows, cols);
  if (st) return st;
  fpb_nvfp4_matrix *m = nullptr;
  if ((st = alloc_matrix(rows, cols, &m))) return st;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(m->packed, packed, rows * cols / 2, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(m->scales, scales, rows * cols / kNvfp4Group, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(m->row_globals, row_globals, rows * sizeof(float), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    fpb_nvfp4_matrix_destroy(m);
    return cuda_fail(e, "fpb_nvfp4_matrix_create upload");
  }
  // The GEMM-side copies are built here, at load time, so that no GEMM call
  // allocates or synchronises (the calls can then be recorded into a graph).
  if ((st = prepare_gemm_weights(m, s))) {
    fpb_nvfp4_matrix_destroy(m);
    return st;
  }
  *out = m;
  return FPB_OK;
}

int fpb_nvfp4_matrix_create_device(const uint8_t *packed, const uint8_t *scales,
                                   const float *row_globals, size_t rows, size_t cols, void *stream,
                                   fpb_nvfp4_matrix **out) {
  if (!packed || !scales || !row_globals || !out)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_matrix_create_device: null pointer");
  *out = nullptr;
  if (rows == 0 || cols == 0 || cols % kQ8Block != 0)
    return fail(FPB_ERR_FORMAT, "invalid NVFP4 matrix: rows=%zu cols=%zu", rows, cols);
  fpb_nvfp4_matrix *m = nullptr;
  int st = alloc_matrix(rows, cols, &m);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  int *bad = nullptr;
  int host_bad = 0;
  cudaError_t e = cudaMalloc(&bad, sizeof(int));
  if (e == cudaSuccess) e = cudaMemsetAsync(bad, 0, sizeof(int), s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(m->packed, packed, rows * cols / 2, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(m->scales, scales, rows * cols / kNvfp4Group, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(m->row_globals, row_globals, rows * sizeof(float), cudaMemcpyDeviceToDevice,
                        s);
  if (e == cudaSuccess) {
    validate_nvfp4_kernel<<<2 * sm_count(), 256, 0, s>>>(m->scales, rows * cols / kNvfp4Group,
                                                         m->row_globals, rows, bad);
    e = cudaGetLastError();
    count_launch();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host_bad, bad, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(bad);
  if (e != cudaSuccess) {
    fpb_nvfp4_matrix_destroy(m);
    return cuda_fail(e, "fpb_nvfp4_matrix_create_device");
  }
  if (host_bad) {
    fpb_nvfp4_matrix_destroy(m);
    return fail(FPB_ERR_FORMAT, "invalid NVFP4 matrix, block scales, or global scale (%s)",
                (host_bad & 1) ? "NaN e4m3 block scale" : "global scale not finite and >= 0");
  }
  if ((st = prepare_gemm_weights(m, s))) {  // load time: GEMM calls allocate nothing
    fpb_nvfp4_matrix_destroy(m);
    return st;
  }
  *out = m;
  return FPB_OK;
}

int fpb_nvfp4_matrix_destroy(fpb_nvfp4_matrix *m) {
  if (!m) return FPB_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != m->device) cudaSetDevice(m->device);
  cudaFree(m->packed);
  cudaFree(m->scales);
  cudaFree(m->row_globals);
  release_matrix_extras(m);
  if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
  delete m;
  return FPB_OK;
}

int fpb_nvfp4_matrix_shape(const fpb_nvfp4_matrix *m, size_t *rows, size_t *cols) {
  if (!m || !rows || !cols) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_matrix_shape: null pointer");
  *rows = m->rows;
  *cols = m->cols;
  return FPB_OK;
}

int fpb_nvfp4_matrix_device_ptrs(const fpb_nvfp4_matrix *m, const uint8_t **packed,
                                 const uint8_t **scales, const float **row_globals) {
  if (!m) return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_matrix_device_ptrs: null handle");
  if (packed) *packed = m->packed;
  if (scales) *scales = m->scales;
  if (row_globals) *row_globals = m->row_globals;
  return FPB_OK;
}

int fpb_nvfp4_matrix_download(const fpb_nvfp4_matrix *m, uint8_t *packed, uint8_t *scales,
                              float *row_globals, void *stream) {
  if (!m || !packed || !scales || !row_globals)
    return fail(FPB_ERR_INVALID_ARGUMENT, "fpb_nvfp4_matrix_download: null pointer");
  cudaStream_t s = as_stream(stream);
  FPB_CUDA_TRY(cudaMemcpyAsync(packed, m->packed, m->rows * m->cols / 2, cudaMemcpyDeviceToHost, s));
  FPB_CUDA_TRY(cudaMemcpyAsync(scales, m->scales, m->rows * m->cols / kNvfp4Group,
                               cudaMemcpyDeviceToHost, s));
  FPB_CUDA_TRY(cudaMemcpyAsync(row_globals, m->row_globals, m->rows * sizeof(float),
                               cudaMemcpyDeviceToHost, s));
  FPB_CUDA_TRY(cudaStreamSynchronize(s));
  return FPB_OK;
}

}  // extern "C"
