/*
 * fp_oracle — CPU restatement of firepit's quantized-matmul arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  The product (firepit_b200) never links, loads or
 * calls this library; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py use it, as the checker and as the timed CPU
 * baseline.
 *
 * Every function names the reference item it restates, as `path:line` in
 * almightychang/firepit (crate-relative: kernels = crates/firepit-kernels,
 * firepit = crates/firepit).  The reference's own kernels are cuTile DSL
 * code with no CPU form; its tests hold the f64 oracle restated here.
 *
 * Parity pins (see tests/test_oracle_pins.py): the e2m1/e4m3 decode tables
 * against the reference formulas, every e4m3 byte against an independent
 * decoder, the ModelOpt dequant fixture's internal structure, and the MoE
 * layout against a stable sort (kernels src/moe.rs:865-941).  The quantizer
 * has no reference counterpart (its rule comes from the task's config) and is
 * "parity unpinned"; it is pinned by round-trip properties instead.
 *
 * Build: oracle/Makefile (gcc, -ffp-contract=off so that the synthetic data
 * generator matches the GPU generator bit for bit).
 */
#ifndef FP_ORACLE_H
#define FP_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- codecs --------------------------------------------------------------- */
/* kernels tests/nvfp4_oracle.rs:24-31: 0x8 decodes to -0.0 */
float orc_e2m1_test(uint8_t code);
/* firepit src/checkpoint.rs:386-390 (ModelOpt table): 0x8 decodes to +0.0 */
float orc_e2m1_modelopt(uint8_t code);
/* kernels tests/nvfp4_oracle.rs:33-42, firepit src/checkpoint.rs:338-347 */
float orc_e4m3(uint8_t bits);
/* round-to-nearest-even, satfinite (max 6 / 448); sign kept for -0 */
uint8_t orc_f32_to_e2m1(float v);
uint8_t orc_f32_to_e4m3(float v);
/* bfloat16 <-> f32, RNE (NaN kept quiet) */
uint16_t orc_f32_to_bf16(float v);
float orc_bf16_to_f32(uint16_t b);

/* ---- synthetic data --------------------------------------------------------
 * Philox4x32-10 (Salmon et al., SC'11) counter-based stream + Box-Muller with
 * this file's own log/sin/cos polynomials, evaluated with plain IEEE binary32
 * operations in a fixed order, so that the device generator in
 * firepit_b200/csrc/synth.cu reproduces every value bit for bit.
 * Element i of (seed, stream) is independent of every other element. */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
float orc_synth_normal_one(uint64_t seed, uint32_t stream, uint64_t index);
void orc_synth_normal(uint64_t seed, uint32_t stream, uint64_t offset, size_t count,
                      float mean, float stddev, float *out);

/* ---- NVFP4 ---------------------------------------------------------------- */
/* Quantize rule (no reference counterpart): global = amax/(6*448) per block of
 * rows_per_global rows, s = RN_e4m3((block_amax/6)/global),
 * code = RN_e2m1(w / (e4m3(s)*global)).  packed low nibble = even column
 * (firepit src/checkpoint.rs:414-418). Returns 0, or -1 on a non-finite input. */
int orc_nvfp4_quantize(const float *w, size_t rows, size_t cols, size_t rows_per_global,
                       uint8_t *packed, uint8_t *scales, float *row_globals);
/* ModelOpt dequant order E2M1[c] * (e4m3(s) * g) (firepit src/checkpoint.rs:401-420) */
void orc_nvfp4_dequantize(const uint8_t *packed, const uint8_t *scales,
                          const float *row_globals, size_t rows, size_t cols, float *out);
/* Host validation of HostNvfp4Matrix::from_parts (kernels src/weights/nvfp4.rs:47-64). */
int orc_nvfp4_validate(size_t packed_len, const uint8_t *scales, size_t scales_len,
                       const float *row_globals, size_t rows, size_t cols);

/* Decode GEMV in the reference kernel's f32 order (kernels src/gemv/nvfp4.rs:34-59):
 * per 128-column chunk, per 16-group f32 sum of E2M1*x, times e4m3 scale, summed
 * over the chunk's groups, added to the row accumulator; times the row global.
 * x [batch, cols] f32, y [batch, rows].  OpenMP over rows. */
void orc_nvfp4_gemv_f32(const uint8_t *packed, const uint8_t *scales, const float *row_globals,
                        size_t rows, size_t cols, const float *x, size_t batch, float *y);
/* f64 oracle (kernels tests/nvfp4_oracle.rs:75-101 with tests/common/oracle.rs:3-19):
 * expected = g * sum f64(E2M1*e4m3) * f64(x); magnitude = g * sum |.|*|x|. */
void orc_nvfp4_gemv_f64(const uint8_t *packed, const uint8_t *scales, const float *row_globals,
                        size_t rows, size_t cols, const float *x, size_t batch,
                        double *expected, double *magnitude);
/* Expert GEMV (kernels src/gemv/nvfp4.rs:62-107): slot s uses weight rows
 * ids[s]*rows_per_expert + [0, rows_per_expert) and input row s*input_stride. */
void orc_nvfp4_expert_gemv_f32(const uint8_t *packed, const uint8_t *scales,
                               const float *row_globals, size_t cols, const int32_t *ids,
                               size_t slots, size_t rows_per_expert, size_t input_stride,
                               const float *x, float *y);

/* ---- FP8 E4M3 (oracle/fp8.c) --------------------------------------------
 * Formats of kernels src/weights/fp8.rs:8-27.  block_n = block_k = 0 selects
 * per-row scales (Fp8Scaling::Rows), otherwise a [rows/block_n, cols/block_k]
 * grid.  Quantize (no reference counterpart; task config 1): scale =
 * amax/448 per block or row, bits = RN_e4m3_satfinite(w / scale), 0 when the
 * scale is 0.  Per-token activation scales are the row mode.  Returns 0, or
 * -1 on a bad shape or a non-finite input. */
int orc_fp8_quantize(const float *w, size_t rows, size_t cols, size_t block_n, size_t block_k,
                     uint8_t *bits, float *scales);
void orc_fp8_dequantize(const uint8_t *bits, const float *scales, size_t rows, size_t cols,
                        size_t block_n, size_t block_k, float *out);
/* f64 product of the dequantized operands (kernels tests/fp8_oracle.rs:139-170
 * with tests/common/oracle.rs): a [m, k] with per-row scales, w [n, k];
 * expected = sum (e4m3(a) a_s)(e4m3(w) w_s), magnitude = sum |.||.|. */
void orc_fp8_gemm_f64(const uint8_t *a_bits, const float *a_scales, size_t m, const uint8_t *w_bits,
                      const float *w_scales, size_t n, size_t k, size_t block_n, size_t block_k,
                      double *expected, double *magnitude);

/* ---- MoE (oracle/moe.c) ---------------------------------------------------
 * top_k_prefill (kernels src/moe.rs:15-68): per token, k rounds of "largest
 * remaining logit, lowest id among equals"; weight exp(l - max) / sum over
 * the k winners; slot k = expert `experts` with sigmoid(gate) when
 * shared_gate is given; other slots id 0 weight 0.  ids/weights [tokens, width]. */
void orc_moe_topk(const float *logits, size_t ld, const float *shared_gate, size_t tokens, size_t experts,
                  size_t k, size_t width, int32_t *ids, float *weights);
/* PrefillLayout::from_indices (kernels src/moe.rs:452-516) over the first kk
 * slots of each row of ids [tokens, width]: stable counting sort by expert,
 * each expert padded to tile_rows; token_rows [cap] (-1 padding), tile_experts
 * [cap / tile_rows] (-1 past the end), inverse [tokens, width] (0 padding),
 * ranges [experts][2] (start, count).  Returns 0, or -1 on a bad id/capacity. */
int orc_moe_layout(const int32_t *ids, size_t tokens, size_t width, size_t kk, size_t experts, size_t tile_rows,
                   size_t cap, int32_t *token_rows, int32_t *tile_experts, int32_t *inverse, int64_t *ranges,
                   int32_t *padded);
/* swiglu (kernels src/swiglu.rs:16): gate / (1 + exp(-gate)) * up. */
void orc_swiglu(const float *gate_up, size_t rows, size_t inter, float *out);
/* combine_prefill_kernel (moe.rs:91-109); with residual, combine_add_norm_kernel
 * (moe.rs:111-147): out = residual + sum, normed = out * rsqrt(mean(out^2) + eps) * gamma. */
void orc_moe_combine(const float *routed, size_t cols, const int32_t *inverse, const float *weights, size_t tokens,
                     size_t width, size_t slots, const float *residual, const float *gamma, float eps, float *out,
                     float *normed);

/* ---- error model (kernels tests/common/check.rs:19-38) ------------------- */
double orc_gamma_tilde(size_t n);
double orc_inner_product_excess(const float *actual, const double *expected,
                                const double *magnitude, size_t len, size_t n);

/* ---- CPU baseline helpers ------------------------------------------------- */
int orc_num_threads(void);
void orc_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
