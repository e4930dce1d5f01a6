// Seeded synthetic data on the device (random-init weights and activations).
//
// Philox4x32-10 (Salmon et al., SC'11) gives four 32-bit words per counter;
// Box-Muller turns pairs of them into normals.  log/sin/cos are this file's
// own series evaluations, written as single IEEE binary32 operations
// (_rn intrinsics, so nvcc cannot contract them into FMAs), which makes every
// value reproducible bit for bit by a CPU implementation that performs the
// same operations in the same order.  Element i of (seed, stream) depends on
// nothing else, so any slice can be regenerated independently.
#include "common.cuh"

namespace fpb {

__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
    uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
    uint32_t n0 = hi1 ^ c[1] ^ k0;
    uint32_t n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

__device__ __forceinline__ float det_log(float x) {
  uint32_t u = __float_as_uint(x);
  int e = (int)((u >> 23) & 0xff) - 127;
  uint32_t mant = u & 0x7fffffu;
  if (mant > 0x3504f3u) {
    e += 1;
    mant |= (126u << 23);
  } else {
    mant |= (127u << 23);
  }
  float m = __uint_as_float(mant);
  float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  float s2 = __fmul_rn(s, s);
  float p = 0.0769230798f;
  p = __fmul_rn(p, s2); p = __fadd_rn(p, 0.0909090936f);
  p = __fmul_rn(p, s2); p = __fadd_rn(p, 0.111111112f);
  p = __fmul_rn(p, s2); p = __fadd_rn(p, 0.142857149f);
  p = __fmul_rn(p, s2); p = __fadd_rn(p, 0.200000003f);
  p = __fmul_rn(p, s2); p = __fadd_rn(p, 0.333333343f);
  p = __fmul_rn(p, s2);
  float t = __fmul_rn(s, p);
  t = __fadd_rn(t, s);
  t = __fadd_rn(t, t);
  float r = __fmul_rn((float)e, 0.693147182f);
  return __fadd_rn(r, t);
}

__device__ __forceinline__ void det_sincos_quarter(float a, float &s_out, float &c_out) {
  float a2 = __fmul_rn(a, a);
  float c = -1.14707456e-11f;
  c = __fmul_rn(c, a2); c = __fadd_rn(c, 2.08767570e-09f);
  c = __fmul_rn(c, a2); c = __fsub_rn(c, 2.75573192e-07f);
  c = __fmul_rn(c, a2); c = __fadd_rn(c, 2.48015876e-05f);
  c = __fmul_rn(c, a2); c = __fsub_rn(c, 1.38888892e-03f);
  c = __fmul_rn(c, a2); c = __fadd_rn(c, 4.16666679e-02f);
  c = __fmul_rn(c, a2); c = __fsub_rn(c, 0.5f);
  c = __fmul_rn(c, a2); c = __fadd_rn(c, 1.0f);
  float s = 1.60590444e-10f;
  s = __fmul_rn(s, a2); s = __fsub_rn(s, 2.50521079e-08f);
  s = __fmul_rn(s, a2); s = __fadd_rn(s, 2.75573188e-06f);
  s = __fmul_rn(s, a2); s = __fsub_rn(s, 1.98412701e-04f);
  s = __fmul_rn(s, a2); s = __fadd_rn(s, 8.33333377e-03f);
  s = __fmul_rn(s, a2); s = __fsub_rn(s, 0.166666672f);
  s = __fmul_rn(s, a2);
  s = __fmul_rn(s, a);
  s = __fadd_rn(s, a);
  s_out = s;
  c_out = c;
}

__device__ __forceinline__ float synth_normal_one(uint64_t seed, uint32_t stream, uint64_t index) {
  uint64_t block = index >> 2;
  uint32_t c[4] = {(uint32_t)block, (uint32_t)(block >> 32), stream, 0x46495245u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  int pair = (int)((index >> 1) & 1);
  uint32_t r1 = pair ? c[2] : c[0];
  uint32_t r2 = pair ? c[3] : c[1];
  float u1 = __fmul_rn((float)((r1 >> 8) + 1u), 5.96046448e-08f);
  float u2 = __fmul_rn((float)(r2 >> 8), 5.96046448e-08f);
  float l = det_log(u1);
  float radius = __fsqrt_rn(__fmul_rn(-2.0f, l));
  float t = __fmul_rn(u2, 4.0f);
  int q = (int)t;
  float f = __fsub_rn(t, (float)q);
  float a = __fmul_rn(f, 1.57079637f);
  float s, co;
  det_sincos_quarter(a, s, co);
  float cs, sn;
  switch (q & 3) {
    case 0: cs = co; sn = s; break;
    case 1: cs = -s; sn = co; break;
    case 2: cs = -co; sn = -s; break;
    default: cs = s; sn = -co; break;
  }
  return __fmul_rn(radius, (index & 1) ? sn : cs);
}

__global__ void synth_normal_kernel(uint64_t seed, uint32_t stream, uint64_t offset, size_t count,
                                    float mean, float stddev, int dtype, void *out) {
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
    float z = synth_normal_one(seed, stream, offset + i);
    float v = __fadd_rn(__fmul_rn(stddev, z), mean);
    if (dtype == FPB_BF16)
      reinterpret_cast<__nv_bfloat16 *>(out)[i] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<float *>(out)[i] = v;
  }
}

}  // namespace fpb

extern "C" int fpb_synth_normal(uint64_t seed, uint32_t stream_id, uint64_t offset, size_t count,
                                float mean, float stddev, int dtype, void *out, void *stream) {
  if (!out) return fpb::fail(FPB_ERR_INVALID_ARGUMENT, "fpb_synth_normal: null output");
  if (dtype != FPB_F32 && dtype != FPB_BF16)
    return fpb::fail(FPB_ERR_INVALID_ARGUMENT, "fpb_synth_normal: dtype %d", dtype);
  if (count == 0) return FPB_OK;
  size_t blocks = (count + 255) / 256;
  size_t cap = (size_t)fpb::sm_count() * 16;
  if (blocks > cap) blocks = cap;
  fpb::synth_normal_kernel<<<(unsigned)blocks, 256, 0, fpb::as_stream(stream)>>>(
      seed, stream_id, offset, count, mean, stddev, dtype, out);
  FPB_LAUNCH_CHECK("synth_normal_kernel");
  return FPB_OK;
}
