// Shared helpers of the firepit_b200 CUDA library: status plumbing, the
// per-thread error message, the launch counter and small device utilities.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <string>

#include "../../include/firepit_b200.h"

namespace fpb {

// Records `msg` as the calling thread's last error and returns `status`.
int fail(int status, const char *fmt, ...);
// Converts a CUDA error into FPB_ERR_CUDA with a message naming `what`.
int cuda_fail(cudaError_t err, const char *what);
void count_launch(uint64_t n = 1);
// Streaming multiprocessor count of the current device (cached per device).
int sm_count();
// Device address of the library's device-side error word on the current
// device (first error code a kernel recorded; read by fpb_device_error).
int *device_error_ptr();

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace fpb

#define FPB_CUDA_TRY(expr)                                  \
  do {                                                      \
    cudaError_t fpb_err_ = (expr);                          \
    if (fpb_err_ != cudaSuccess) return fpb::cuda_fail(fpb_err_, #expr); \
  } while (0)

// Checks the launch that was just issued on this thread.
// Programmatic dependent launch for short kernels that follow one another in
// a stream.  pdl_enter(), first in such a kernel, waits until the previous
// kernel in the stream has completed and its writes are visible (a no-op when
// the kernel was launched without the attribute), then lets the next kernel
// start launching; so nothing is read before its producer is done, and only
// the launch latency overlaps the previous kernel.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
}

// Launches a kernel whose body starts with pdl_enter() with the
// programmatic-serialization attribute (a plain launch where the attribute is
// refused).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
  cudaLaunchConfig_t lc{};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&lc, kernel, args...);
  if (e == cudaErrorInvalidValue) {
    cudaGetLastError();
    lc.numAttrs = 0;
    e = cudaLaunchKernelEx(&lc, kernel, args...);
  }
  return e;
}

// launch_pdl with a thread-block cluster of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                      unsigned cluster_x, Args &&...args) {
  cudaLaunchConfig_t lc{};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&lc, kernel, args...);
  if (e == cudaErrorInvalidValue) {
    cudaGetLastError();
    lc.numAttrs = 1;
    e = cudaLaunchKernelEx(&lc, kernel, args...);
  }
  return e;
}

// ---- thread-block clusters (distributed shared memory) ----------------------------
__device__ __forceinline__ unsigned cluster_ctarank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ unsigned cluster_nctarank() {
  unsigned n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}

// Every thread of every CTA of the cluster arrives; writes before it are
// visible to the cluster after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The float at this CTA's shared-memory address `p`, read from the same
// address in cluster CTA `rank`.
__device__ __forceinline__ float dsmem_load(const float *p, unsigned rank) {
  unsigned local = (unsigned)__cvta_generic_to_shared(p), remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

#define FPB_LAUNCH_CHECK(name)                                   \
  do {                                                           \
    cudaError_t fpb_err_ = cudaGetLastError();                   \
    if (fpb_err_ != cudaSuccess) return fpb::cuda_fail(fpb_err_, name); \
    fpb::count_launch();                                         \
  } while (0)

// ---- device helpers ---------------------------------------------------------
namespace fpb {

// Two e4m3 bytes (low byte = first) -> f16x2 (low half = first), exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t out;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(v));
  return out;
}

// One byte of two e2m1 codes (low nibble = first) -> f16x2 (low half = first).
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
      : "=r"(out)
      : "r"(byte));
  return out;
}

// Four bytes (eight e2m1 codes, first code in the lowest nibble) -> four
// f16x2 words, out[i] holding codes 2i (low half) and 2i+1 (high half).
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t out[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
      : "r"(w));
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
  uint32_t h2 = e4m3x2_to_f16x2((uint16_t)v);
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffff)));
}

__device__ __forceinline__ float e2m1_to_f32(uint32_t code) {
  uint32_t h2 = e2m1x2_to_f16x2(code & 0xf);
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffff)));
}

// Eight f32 values -> eight e2m1 codes packed in 32 bits, v[0] in the lowest
// nibble; round-to-nearest-even, satfinite.  (cvt's first source operand goes
// to the upper nibble of each byte.)
__device__ __forceinline__ uint32_t f32x8_to_e2m1x8(const float v[8]) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

// f32 -> e4m3 byte, RNE satfinite.
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(0.0f), "f"(v));
  return (uint8_t)(out & 0xff);
}

// Two floats -> bf16x2 (RNE), first value in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace fpb
