/* fp_oracle: scalar codecs, synthetic data and the error model.
 * TEST INFRASTRUCTURE ONLY (see fp_oracle.h). */
#include "fp_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* kernels tests/nvfp4_oracle.rs:21 */
static const float E2M1_MAG[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float orc_e2m1_test(uint8_t code) {
  /* kernels tests/nvfp4_oracle.rs:24-31: magnitude from the low three bits,
   * negated when bit 3 is set (so 0x8 is -0.0). */
  float m = E2M1_MAG[code & 0x7];
  return (code & 0x8) ? -m : m;
}

float orc_e2m1_modelopt(uint8_t code) {
  /* firepit src/checkpoint.rs:386-390: ModelOpt's e2m1_values table, where
   * 0b1000 is +0. */
  code &= 0xf;
  if (code == 0x8) return 0.0f;
  return orc_e2m1_test(code);
}

float orc_e4m3(uint8_t bits) {
  /* kernels tests/nvfp4_oracle.rs:33-42: sign, 4-bit exponent (bias 7),
   * 3-bit fraction, exponent 0 is subnormal fraction*2^-9.  The formula has
   * no NaN case; 0x7f/0xff are rejected by the validators instead. */
  float sign = (bits & 0x80) ? -1.0f : 1.0f;
  int exponent = (bits >> 3) & 0x0f;
  float fraction = (float)(bits & 0x07);
  if (exponent == 0) return sign * fraction * ldexpf(1.0f, -9);
  return sign * (1.0f + fraction / 8.0f) * ldexpf(1.0f, exponent - 7);
}

/* Round |v| to the nearest multiple of 2^q_exp, ties to even.  |v|/2^q_exp is
 * exact (power-of-two scaling of a normal float), and nearbyintf uses the
 * default round-to-nearest-even mode. */
static float rne_multiple(float a, int q_exp, int *n_out) {
  float n = nearbyintf(ldexpf(a, -q_exp));
  *n_out = (int)n;
  return n;
}

uint8_t orc_f32_to_e2m1(float v) {
  /* E2M1: 1 sign, 2 exponent bits (bias 1), 1 mantissa bit; largest 6.0. */
  uint8_t sign = signbit(v) ? 0x8 : 0x0;
  float a = fabsf(v);
  if (isnan(v)) return sign | 0x7; /* no NaN code in e2m1: satfinite */
  if (a >= 6.0f) return sign | 0x7;
  int e2;
  frexpf(a, &e2); /* a in [2^(e2-1), 2^e2) */
  int ex = (a == 0.0f) ? 0 : e2 - 1;
  if (ex < 0) ex = 0; /* subnormal binade shares the quantum 0.5 */
  int n;
  rne_multiple(a, ex - 1, &n); /* quantum 2^(ex-1) */
  if (n == 0) return sign;
  if (ex == 0 && n < 2) return sign | (uint8_t)n; /* 0.5 */
  if (n == 4) { ex += 1; n = 2; }
  int e_field = ex + 1;
  if (e_field > 3) return sign | 0x7;
  return sign | (uint8_t)((e_field << 1) | (n - 2));
}

uint8_t orc_f32_to_e4m3(float v) {
  /* E4M3 (fn): 1 sign, 4 exponent bits (bias 7), 3 mantissa bits; largest
   * finite 448 (0x7e); 0x7f is NaN.  satfinite clamps to 448. */
  uint8_t sign = signbit(v) ? 0x80 : 0x00;
  float a = fabsf(v);
  if (isnan(v)) return sign | 0x7f;
  if (a > 448.0f) return sign | 0x7e;
  int e2;
  frexpf(a, &e2);
  int ex = (a == 0.0f) ? -6 : e2 - 1;
  if (ex < -6) ex = -6; /* subnormals share the quantum 2^-9 */
  int n;
  rne_multiple(a, ex - 3, &n); /* quantum 2^(ex-3) */
  if (n == 0) return sign;
  if (ex == -6 && n < 8) return sign | (uint8_t)n;
  if (n == 16) { ex += 1; n = 8; }
  int e_field = ex + 7;
  if (e_field > 15 || (e_field == 15 && n > 14)) return sign | 0x7e;
  return sign | (uint8_t)((e_field << 3) | (n - 8));
}

uint16_t orc_f32_to_bf16(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ---- Philox4x32-10 --------------------------------------------------------- */
static inline void mulhilo(uint32_t a, uint32_t b, uint32_t *hi, uint32_t *lo) {
  uint64_t p = (uint64_t)a * (uint64_t)b;
  *hi = (uint32_t)(p >> 32);
  *lo = (uint32_t)p;
}

void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
  uint32_t k0 = key[0], k1 = key[1];
  for (int round = 0; round < 10; ++round) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(0xD2511F53u, c0, &hi0, &lo0);
    mulhilo(0xCD9E8D57u, c2, &hi1, &lo1);
    uint32_t n0 = hi1 ^ c1 ^ k0;
    uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* The generator's transcendental pieces.  Written from the series
 * definitions; every step is a single IEEE binary32 operation, in the same
 * order as firepit_b200/csrc/synth.cu (compiled there with _rn intrinsics). */
static float det_log(float x) {
  /* x = m * 2^e with m in [sqrt(1/2), sqrt(2)); ln m = 2 atanh(s),
   * s = (m-1)/(m+1), atanh(s) = s + s^3/3 + s^5/5 + ... */
  uint32_t u;
  memcpy(&u, &x, 4);
  int e = (int)((u >> 23) & 0xff) - 127;
  uint32_t mant = u & 0x7fffffu;
  if (mant > 0x3504f3u) { /* m > sqrt(2) */
    e += 1;
    mant |= (126u << 23);
  } else {
    mant |= (127u << 23);
  }
  float m;
  memcpy(&m, &mant, 4);
  float s = (m - 1.0f) / (m + 1.0f);
  float s2 = s * s;
  float p = 0.0769230798f;            /* 1/13 */
  p = p * s2; p = p + 0.0909090936f;  /* 1/11 */
  p = p * s2; p = p + 0.111111112f;   /* 1/9 */
  p = p * s2; p = p + 0.142857149f;   /* 1/7 */
  p = p * s2; p = p + 0.200000003f;   /* 1/5 */
  p = p * s2; p = p + 0.333333343f;   /* 1/3 */
  p = p * s2;
  float t = s * p;
  t = t + s;
  t = t + t; /* 2 atanh(s) */
  float ef = (float)e;
  float r = ef * 0.693147182f; /* ln 2 */
  return r + t;
}

static void det_sincos_quarter(float a, float *s_out, float *c_out) {
  /* a in [0, pi/2): Taylor series of sin and cos to degree 13 / 14. */
  float a2 = a * a;
  float c = -1.14707456e-11f;          /* -1/14! */
  c = c * a2; c = c + 2.08767570e-09f; /* 1/12! */
  c = c * a2; c = c - 2.75573192e-07f; /* 1/10! */
  c = c * a2; c = c + 2.48015876e-05f; /* 1/8! */
  c = c * a2; c = c - 1.38888892e-03f; /* 1/6! */
  c = c * a2; c = c + 4.16666679e-02f; /* 1/4! */
  c = c * a2; c = c - 0.5f;
  c = c * a2; c = c + 1.0f;
  float s = 1.60590444e-10f;           /* 1/13! */
  s = s * a2; s = s - 2.50521079e-08f; /* 1/11! */
  s = s * a2; s = s + 2.75573188e-06f; /* 1/9! */
  s = s * a2; s = s - 1.98412701e-04f; /* 1/7! */
  s = s * a2; s = s + 8.33333377e-03f; /* 1/5! */
  s = s * a2; s = s - 0.166666672f;    /* 1/3! */
  s = s * a2;
  s = s * a;
  s = s + a;
  *s_out = s;
  *c_out = c;
}

float orc_synth_normal_one(uint64_t seed, uint32_t stream, uint64_t index) {
  uint64_t block = index >> 2;
  uint32_t ctr[4] = {(uint32_t)block, (uint32_t)(block >> 32), stream, 0x46495245u};
  uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t r[4];
  orc_philox4x32_10(ctr, key, r);
  int pair = (int)((index >> 1) & 1);
  uint32_t r1 = r[2 * pair], r2 = r[2 * pair + 1];
  float u1 = (float)((r1 >> 8) + 1u) * 5.96046448e-08f; /* (0, 1] */
  float u2 = (float)(r2 >> 8) * 5.96046448e-08f;        /* [0, 1) */
  float l = det_log(u1);
  float radius = sqrtf(-2.0f * l);
  float t = u2 * 4.0f;
  int q = (int)t;
  float f = t - (float)q;
  float a = f * 1.57079637f;
  float s, c;
  det_sincos_quarter(a, &s, &c);
  float cs, sn;
  switch (q & 3) {
    case 0: cs = c; sn = s; break;
    case 1: cs = -s; sn = c; break;
    case 2: cs = -c; sn = -s; break;
    default: cs = s; sn = -c; break;
  }
  return radius * ((index & 1) ? sn : cs);
}

void orc_synth_normal(uint64_t seed, uint32_t stream, uint64_t offset, size_t count,
                      float mean, float stddev, float *out) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)count; ++i) {
    float z = orc_synth_normal_one(seed, stream, offset + (uint64_t)i);
    float v = stddev * z;
    out[i] = v + mean;
  }
}

/* ---- error model ------------------------------------------------------------ */
double orc_gamma_tilde(size_t n) {
  /* kernels tests/common/check.rs:19-26: Higham & Mary (2019) Thm 3.1 with
   * lambda = 8 and u = 2^-24. */
  const double u = 5.9604644775390625e-08, lambda = 8.0;
  double nn = (double)n;
  return expm1(lambda * sqrt(nn) * u + nn * u * u / (1.0 - u));
}

double orc_inner_product_excess(const float *actual, const double *expected,
                                const double *magnitude, size_t len, size_t n) {
  /* kernels tests/common/check.rs:28-38 */
  double bound = orc_gamma_tilde(n), worst = 0.0;
  for (size_t i = 0; i < len; ++i) {
    double allowed = bound * magnitude[i];
    if (allowed < 2.2250738585072014e-308) allowed = 2.2250738585072014e-308;
    double r = fabs((double)actual[i] - expected[i]) / allowed;
    if (r > worst || isnan(r)) worst = isnan(r) ? INFINITY : r;
  }
  return worst;
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Sets the OpenMP thread count of the oracle's parallel loops (a launcher
 * such as torch.distributed.run sets OMP_NUM_THREADS=1 for every rank). */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
