// NVFP4 activation encoding shared by the GEMM's quantizer and the MoE
// gather / SwiGLU quantizers: the tensor cores' tiled scale-factor layout and
// the per-16-column group encode (same arithmetic as fpb_nvfp4_quantize).
//
// Tiled factor layout: for each 128-row block and each 64-column block, 512
// bytes holding the factor of row r, 16-column group s at byte
// (r % 32) * 16 + (r / 32) * 4 + s; K blocks are padded to a multiple of four
// (256 columns) with zero factors.
#pragma once
#include <cstddef>
#include <cstdint>

#include "common.cuh"
#include "nvfp4_matrix.cuh"

namespace fpb {

constexpr int kSfChunk = 512;  // bytes per (128 rows, 64 columns)

__host__ __device__ inline size_t sf_tiled_bytes(size_t rows, size_t cols) {
  size_t rb = (rows + 127) / 128, kb = (cols + 255) / 256;
  return rb * kb * 4 * kSfChunk;
}

// Byte offset of the factor of (row, group) in the tiled layout.
__host__ __device__ inline size_t sf_tiled_offset(size_t row, size_t group, size_t cols) {
  size_t kb64_per_rb = (cols + 255) / 256 * 4;
  size_t rb = row / 128, r = row % 128, kb64 = group / 4, s = group % 4;
  return (rb * kb64_per_rb + kb64) * kSfChunk + (r % 32) * 16 + (r / 32) * 4 + s;
}

// sf_tiled_offset split into its row part (64-bit, once per row) and its
// group part (32-bit): offset = row part + group part.
__host__ __device__ inline size_t sf_tiled_row_offset(size_t row, size_t cols) {
  const size_t r = row % 128;
  return (row / 128) * ((cols + 255) / 256 * 4) * kSfChunk + (r % 32) * 16 + (r / 32) * 4;
}
__host__ __device__ inline uint32_t sf_tiled_group_offset(uint32_t group) {
  return (group / 4) * kSfChunk + group % 4;
}

template <typename T>
__device__ __forceinline__ float act_load(const T *p, size_t i);
template <>
__device__ __forceinline__ float act_load<float>(const float *p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float act_load<uint16_t>(const uint16_t *p, size_t i) {
  return bf16_bits_to_f32(p[i]);
}

// Reduces each thread's |x| maximum over the CTA and adds it to *amax_bits
// with one atomicMax per CTA (one per warp made thousands of atomics on a
// single address, which the L2 serialises).  Every thread of the CTA calls it.
__device__ __forceinline__ void block_amax_to(uint32_t m, uint32_t *amax_bits) {
  __shared__ uint32_t warp_max[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_max[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)((blockDim.x + 31) >> 5) ? warp_max[lane] : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0 && m) atomicMax(amax_bits, m);
  }
}

// atomicMax of |x| bits over x[0, n) (amax_bits zeroed by the caller).
// 16-byte loads when x is 16-byte aligned, element loads for the tail.
template <typename T>
__global__ void act_amax_kernel(const T *x, size_t n, uint32_t *amax_bits) {
  pdl_enter();
  uint32_t m = 0;
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  constexpr size_t kVec = 16 / sizeof(T);
  size_t head = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const size_t nv = n / kVec;
    const uint4 *xv = reinterpret_cast<const uint4 *>(x);
#pragma unroll 4
    for (size_t i = tid; i < nv; i += stride) {
      const uint4 u = xv[i];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (sizeof(T) == 4)
          m = max(m, w[k] & 0x7fffffffu);
        else
          m = max(m, max((w[k] << 16) & 0x7fffffffu, w[k] & 0x7fff0000u));
      }
    }
    head = nv * kVec;
  }
  for (size_t i = head + tid; i < n; i += stride) m = max(m, __float_as_uint(act_load(x, i)) & 0x7fffffffu);
  block_amax_to(m, amax_bits);
}

// SwiGLU of one element in the reference's order (swiglu.rs:16):
// gate / (1 + exp(gate * -1)) * up, IEEE division and CUDA's expf (the
// unfused SwiGLU kernels; the fused GEMM epilogue uses exp2 / reciprocal
// approximations).
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(g * -1.0f)) * u; }

// One 16-value group: s = RN_e4m3((bmax / 6) / global), codes =
// RN_e2m1(v / (e4m3(s) * global)); returns the factor, the 8 code bytes in
// `codes` (values 0-7 in .x, 8-15 in .y).
__device__ __forceinline__ uint8_t encode_group16_regs(const float v[16], float global, uint2 &codes) {
  float bmax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
  uint8_t s = 0;
  if (global > 0.0f) s = f32_to_e4m3(__fdiv_rn(__fdiv_rn(bmax, 6.0f), global));
  const float denom = __fmul_rn(e4m3_to_f32(s), global);
  uint32_t lo = 0, hi = 0;
  if (denom > 0.0f) {
    float q[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) q[i] = __fdiv_rn(v[i], denom);
    lo = f32x8_to_e2m1x8(q);
    hi = f32x8_to_e2m1x8(q + 8);
  }
  codes = make_uint2(lo, hi);
  return s;
}

// The same group written out: 8 code bytes and the factor.
__device__ __forceinline__ void encode_group16(const float v[16], float global, uint8_t *packed_dst,
                                               uint8_t *sf_dst) {
  uint2 codes;
  *sf_dst = encode_group16_regs(v, global, codes);
  *reinterpret_cast<uint2 *>(packed_dst) = codes;
}

}  // namespace fpb
