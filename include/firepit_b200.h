/*
 * firepit_b200 — C ABI of the B200-native (sm_100a) quantized-matmul hot path.
 *
 * These entry points sit behind firepit-kernels' Rust API (crate
 * `firepit-kernels` of almightychang/firepit).  Each declaration names the
 * reference item it replaces as `path:line`, relative to that crate's
 * `src/` directory unless stated otherwise.
 *
 * Conventions
 *  - Every function returns an `int` status (`FPB_OK` == 0).  Nothing aborts
 *    and nothing throws across this boundary.  `fpb_last_error()` gives the
 *    calling thread's message for the last non-zero status.
 *  - The reference panics (`assert!`) on shape or tile mismatches and returns
 *    `Err(&'static str)` on bad formats.  Here those cases return
 *    `FPB_ERR_SHAPE` and `FPB_ERR_FORMAT`.
 *  - Device pointers are plain `void*` or typed pointers.  The caller owns
 *    them.  Handles (`fpb_nvfp4_matrix`, `fpb_fp8_matrix`) own the device
 *    copies they were created with and free them in `*_destroy`.
 *  - Every launch takes an explicit `cudaStream_t` (passed as `void*`; NULL
 *    is the legacy default stream).  No call synchronises the stream unless
 *    its comment says so.  Calls that take a `workspace` allocate nothing.
 *  - Dtype codes: FPB_F32 (IEEE binary32) and FPB_BF16 (bfloat16).
 */
#ifndef FIREPIT_B200_H
#define FIREPIT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
  FPB_OK = 0,
  FPB_ERR_INVALID_ARGUMENT = 1, /* null pointer, zero size, bad enum        */
  FPB_ERR_SHAPE = 2,            /* the reference's assert! on shapes/tiles  */
  FPB_ERR_FORMAT = 3,           /* the reference's Err(..) on bad formats   */
  FPB_ERR_CUDA = 4,             /* a CUDA runtime call failed               */
  FPB_ERR_UNSUPPORTED = 5,      /* shape outside this build's kernels       */
  FPB_ERR_SELECTION = 6,        /* ExpertSelectionError (moe.rs:262-269)    */
  FPB_ERR_WORKSPACE = 7,        /* workspace too small                      */
  FPB_ERR_NO_DEVICE = 8,        /* no CUDA device visible                   */
  FPB_ERR_IO = 9,               /* a checkpoint file could not be read      */
  FPB_ERR_COMM = 10             /* NCCL missing or a collective failed      */
};

enum { FPB_F32 = 0, FPB_BF16 = 1 };

/* Quantizer flags: FPB_QUANT_AMAX_GIVEN = the amax scratch already holds the
 * |x| maximum (float bits) to derive the global from, e.g. reduced over ranks
 * (fpb_act_amax / fpb_swiglu_amax, then an all-reduce MAX), so that every
 * rank encodes with the same global. */
enum { FPB_QUANT_AMAX_GIVEN = 1 };
/* FPB_QUANT_SKIP_PADDING: rows of a MoE layout whose token is -1 (padding)
 * are neither read nor written nor counted in the amax; for activations
 * whose GEMM gets the same token_rows (fpb_nvfp4_grouped_gemm_q), which
 * then ignores those rows. */
enum { FPB_QUANT_SKIP_PADDING = 2 };

/* Library / error reporting ------------------------------------------------ */
const char *fpb_version(void);
const char *fpb_status_string(int status);
/* Message for the calling thread's last non-zero status ("" if none). */
const char *fpb_last_error(void);
/* Number of kernel launches this process made through the library. */
uint64_t fpb_launch_count(void);

/* ---- formats: scalar codecs (host, no GPU needed) -------------------------
 * e2m1 / e4m3 decode follow tests/nvfp4_oracle.rs:24-42 (crate tests/) and
 * src/checkpoint.rs:338-349 of crate `firepit`; the quantize rule
 * (RNE, satfinite) has no counterpart in the reference.                    */
float fpb_e2m1_to_f32(uint8_t code);
float fpb_e4m3_to_f32(uint8_t bits);
uint8_t fpb_f32_to_e2m1(float value);
uint8_t fpb_f32_to_e4m3(float value);

/* ---- seeded synthetic data (random-init weights and inputs) ---------------
 * Replaces the role of Model::random_from_config's LCG (firepit
 * src/testing.rs:15-151) for the quantized formats: element i of
 * (seed, stream_id) is mean + stddev * N(0,1) from Philox4x32-10 +
 * Box-Muller, independent of every other element; out is f32 or bf16
 * (RNE) [count], starting at element `offset`. */
int fpb_synth_normal(uint64_t seed, uint32_t stream_id, uint64_t offset, size_t count,
                     float mean, float stddev, int dtype, void *out, void *stream);

/* ---- NVFP4 weight matrix ------------------------------------------------- */
typedef struct fpb_nvfp4_matrix fpb_nvfp4_matrix;

/* HostNvfp4Matrix::from_parts validation (weights/nvfp4.rs:47-64), host side:
 * rows>0, cols>0, cols%32==0, lengths match, no NaN e4m3 scale (0x7f/0xff),
 * globals finite and >= 0.  `row_globals` has `rows` entries (stacked
 * matrices keep one global per source matrix, weights/nvfp4.rs:84-97). */
int fpb_nvfp4_validate(const uint8_t *packed, size_t packed_len,
                       const uint8_t *scales, size_t scales_len,
                       const float *row_globals, size_t rows, size_t cols);

/* HostNvfp4Matrix::{from_parts,stack} + upload (weights/nvfp4.rs:47-120).
 * Host arrays: packed [rows, cols/2] (even column in the low nibble),
 * scales [rows, cols/16] e4m3, row_globals [rows] f32.  Copies to device,
 * builds the GEMM-side copies (the factors in the tensor cores' tiled
 * layout: cols/16 more bytes per row; codes with negative factors' signs
 * folded in, only if a factor is negative) and synchronises `stream`.
 * Building them here, at load time, is what lets every later GEMV and GEMM
 * call run without allocating or synchronising. */
int fpb_nvfp4_matrix_create(const uint8_t *packed, const uint8_t *scales,
                            const float *row_globals, size_t rows, size_t cols,
                            void *stream, fpb_nvfp4_matrix **out);
/* Same, from device arrays in the same layout (device-to-device copy). The
 * format is validated on the device; synchronises `stream`. */
int fpb_nvfp4_matrix_create_device(const uint8_t *packed, const uint8_t *scales,
                                   const float *row_globals, size_t rows,
                                   size_t cols, void *stream,
                                   fpb_nvfp4_matrix **out);
int fpb_nvfp4_matrix_destroy(fpb_nvfp4_matrix *m);
int fpb_nvfp4_matrix_shape(const fpb_nvfp4_matrix *m, size_t *rows,
                           size_t *cols);
/* Device pointers of the handle's storage (row-major, as uploaded). */
int fpb_nvfp4_matrix_device_ptrs(const fpb_nvfp4_matrix *m, const uint8_t **packed,
                                 const uint8_t **scales, const float **row_globals);

/* Copies the handle's storage to host arrays (same layout as create);
 * synchronises `stream`. */
int fpb_nvfp4_matrix_download(const fpb_nvfp4_matrix *m, uint8_t *packed, uint8_t *scales,
                              float *row_globals, void *stream);

/* ---- quantize (no reference counterpart: BASELINE's rule) ---------------
 * global = amax / (6*448) per block of `rows_per_global` rows; block scale
 * s = RN_e4m3_satfinite((block_amax / 6) / global); code =
 * RN_e2m1_satfinite(w / (e4m3(s) * global)).  Two launches (amax, encode).
 * `amax_scratch` is rows/rows_per_global floats of device scratch.  Outputs
 * packed [rows, cols/2], scales [rows, cols/16], row_globals [rows]. */
int fpb_nvfp4_quantize(const void *w, int w_dtype, size_t rows, size_t cols,
                       size_t rows_per_global, uint8_t *packed, uint8_t *scales,
                       float *row_globals, float *amax_scratch, void *stream);
/* fpb_nvfp4_quantize without the caller's scratch buffer.  No counterpart in
 * the reference: it is for callers that cannot allocate device memory (an
 * engine whose device memory is one arena reserved up front, a serving loop
 * that must not call cudaMalloc).  The per-block amax scratch is a fixed
 * array inside the library (64 KiB on every GPU that loads it, kept until
 * exit), so rows / rows_per_global may be at most 16384; larger requests
 * return FPB_ERR_UNSUPPORTED.  Allocates nothing.  The first call in a CUDA
 * context looks up the array's device address (cached per context, so a
 * context re-created after cudaDeviceReset looks it up again), so make that
 * first call before any stream capture.  All calls share the array: calls
 * that overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller. */
int fpb_nvfp4_quantize_noalloc(const void *w, int w_dtype, size_t rows, size_t cols,
                               size_t rows_per_global, uint8_t *packed, uint8_t *scales,
                               float *row_globals, void *stream);
/* Dequantize to f32 [rows, cols] with the ModelOpt order
 * E2M1[c] * (e4m3(s) * g) (firepit src/checkpoint.rs:401-420). */
int fpb_nvfp4_dequantize(const fpb_nvfp4_matrix *m, float *out, void *stream);

/* ---- decode GEMV -----------------------------------------------------------
 * gemv(&Weight::Nvfp4, x, y, tile).submit(sink)
 *   (gemv/mod.rs:74-123 -> gemv/nvfp4.rs:120-149, kernel :13-60).
 * y[b, r] = g[r] * sum_k E2M1[w[r,k]] * e4m3(s[r,k/16]) * x[b,k]
 * for rows r in [row_begin, row_end) of the matrix (row_end == 0 means all
 * rows).  x: [batch, cols] (x_dtype), y: [batch, row_end-row_begin]
 * (y_dtype), both contiguous.  1 <= batch <= 16.  Any cols % 32 == 0: rows
 * longer than 4096 columns run as consecutive launches over 4096-column
 * slices that add their sums into y, which must then be f32. */
int fpb_nvfp4_gemv(const fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end,
                   const void *x, int x_dtype, void *y, int y_dtype, int batch,
                   void *stream);

/* Several dense NVFP4 GEMVs in one launch.  Replaces what the reference does
 * at load time to save launches on decode: it stacks projections that read
 * the same input into one matrix (stack_group, firepit src/model.rs:407-444;
 * measured in docs/research/measurements/gemv-probe-gb10.md:98-102, which
 * also notes that independent GEMVs could not run concurrently there).  Here
 * the matrices stay separate handles: segment i computes
 *   segs[i].y[b, r - row_begin] = GEMV of rows [row_begin, row_end) of
 *   segs[i].w with segs[i].x[b, :]
 * as fpb_nvfp4_gemv does, with its own x [batch, cols] and y [batch,
 * row_end - row_begin] (x may be shared).  All segments have the same cols;
 * 1 <= count <= 128, 1 <= batch <= 16.  When cols % 128 == 0, cols <= 4096
 * and batch <= 8, the segments whose row_begin and row count are multiples
 * of 4 run in one launch and each other segment in its own fpb_nvfp4_gemv
 * launch; other shapes run one fpb_nvfp4_gemv launch per segment.  `segs` is
 * read on the host during the call only. */
typedef struct fpb_gemv_segment {
  const fpb_nvfp4_matrix *w;
  size_t row_begin, row_end; /* row_end == 0: all rows */
  const void *x;
  void *y;
} fpb_gemv_segment;
int fpb_nvfp4_gemv_batched(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype, int batch,
                           void *stream);

/* expert_gemv_weight_view(&Weight::Nvfp4, x, selection, y, rows_per_expert,
 * input_stride, tile) (gemv/mod.rs:137-206 -> gemv/nvfp4.rs:151-182,
 * kernel :62-107).  For slot s in [0, slots):
 *   y[s, r] = sum over K of W[expert_ids[s]*rows_per_expert + r, :] . x[s*input_stride, :]
 * expert_ids: device int32 [slots] (ExpertSelection::indices, padding
 * entries beyond `slots` are not read).  x: [*, cols], y: [slots,
 * rows_per_expert].  cols > 4096 as fpb_nvfp4_gemv (f32 y). */
int fpb_nvfp4_expert_gemv(const fpb_nvfp4_matrix *w, const void *x, int x_dtype,
                          const int32_t *expert_ids, int slots,
                          size_t rows_per_expert, int input_stride, void *y,
                          int y_dtype, void *stream);

/* gemv(&Weight::Fp8, x, y, tile).submit(sink) (gemv/mod.rs:74-123 ->
 * gemv/fp8.rs:186-246, kernels dense_fp8_kernel :13-54 and
 * dense_fp8_rows_kernel :108-132), over an FP8 matrix handle (declared
 * below with the FP8 GEMM).  Block scales:
 *   y[b, r] = sum_kb s[r / block_n, kb] * sum_{k in kb} w[r, k] * x[b, k];
 * row scales: y[b, r] = s[r] * sum_k w[r, k] * x[b, k].  Rows [row_begin,
 * row_end) (row_end == 0: all), x [batch, cols], y [batch, row_end -
 * row_begin], contiguous, 1 <= batch <= 16; cols % 32 == 0 (the reference's
 * GemvTile::fits), block_k % 16 == 0. */
struct fpb_fp8_matrix;
int fpb_fp8_gemv(const struct fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                 void *y, int y_dtype, int batch, void *stream);
/* expert_gemv_weight_view(&Weight::Fp8, ...) (gemv/mod.rs:137-206 ->
 * gemv/fp8.rs:248-281, kernels expert_fp8_kernel :56-106 and
 * expert_fp8_rows_kernel :134-160): for slot s, y[s, r] = the GEMV of rows
 * expert_ids[s] * rows_per_expert + r with x row s * input_stride.  Block
 * scales need rows_per_expert % block_n == 0 (gemv/fp8.rs:264).  An id
 * outside [0, rows / rows_per_expert) gives a zero row. */
int fpb_fp8_expert_gemv(const struct fpb_fp8_matrix *w, const void *x, int x_dtype, const int32_t *expert_ids,
                        int slots, size_t rows_per_expert, int input_stride, void *y, int y_dtype, void *stream);

/* ---- prefill NVFP4 GEMM (tcgen05, NVFP4 x NVFP4 -> f32 accumulate) --------
 * Replaces nvfp4_gemm / nvfp4_gemm_view (gemm/nvfp4.rs:119-207, kernel
 * :12-55).  The reference keeps activations in f32 (bf16 hi/lo MMAs); this
 * path quantizes them to NVFP4 (per-tensor global ga = amax/(6*448), E4M3
 * factor per 16 columns) and multiplies on the block-scaled tensor cores:
 *   y[m, n] = ga * g[n] * sum_k a(m,k) * w(n,k)
 * for weight rows n in [row_begin, row_end); row_begin must be a multiple
 * of 128.  y: [m, row_end - row_begin] row-major. */

/* Bytes of the tensor-core tiled scale factors of an [m, k] operand. */
size_t fpb_nvfp4_act_sf_bytes(size_t m, size_t k);
/* Workspace of fpb_nvfp4_gemm (quantized activations + factors + scalars). */
size_t fpb_nvfp4_gemm_workspace_bytes(size_t m, size_t k);
/* Quantizes activations x [m, k] (f32 or bf16) to NVFP4: packed [m, k/2],
 * tiled factors (fpb_nvfp4_act_sf_bytes), global (1 float, device), with
 * amax_scratch one float of device scratch.  Two launches plus two memsets. */
int fpb_nvfp4_quantize_act(const void *x, int x_dtype, size_t m, size_t k, uint8_t *packed,
                           uint8_t *sf_tiled, float *global_out, float *amax_scratch, void *stream);
/* Builds the matrix's GEMM-side copies (tiled factors, TMA map) if they are
 * missing; matrix creation already builds them, so this is a no-op on every
 * handle from fpb_nvfp4_matrix_create(_device).  The GEMM calls below never
 * build anything: they allocate nothing and do not synchronise. */
int fpb_nvfp4_matrix_prepare_gemm(fpb_nvfp4_matrix *w, void *stream);
/* Builds the interleaved factor copy the fused gate/up + SwiGLU GEMM needs
 * for experts of 2*inter rows (fpb_nvfp4_grouped_gemm_swiglu_q); allocates
 * and synchronises `stream`: call it at load time, outside any capture.  A
 * no-op when already built for `inter`. */
int fpb_nvfp4_matrix_prepare_glu(fpb_nvfp4_matrix *w, size_t inter, void *stream);
/* GEMM on already quantized activations. */
int fpb_nvfp4_gemm_q(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const uint8_t *a_packed,
                     const uint8_t *a_sf_tiled, const float *a_global, size_t m, void *y, int y_dtype,
                     void *stream);
/* Quantize x into `workspace` (256-byte aligned, fpb_nvfp4_gemm_workspace_bytes)
 * and run the GEMM (BASELINE config 2's rule for M >= 128).  m <= 16 with
 * cols % 256 == 0, cols <= 4096 and row_begin % 128 == 0 runs as
 * fpb_nvfp4_gemv_planes instead (x not quantized: config 2 keeps decode-size
 * activations in bf16, the reference keeps them in f32). */
int fpb_nvfp4_gemm(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                   size_t m, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                   void *stream);
/* nvfp4_gemm / nvfp4_gemm_view with the reference's activation semantics
 * (gemm/nvfp4.rs:33-50): x stays f32 (or bf16) and is split into bf16
 * hi = bf16(x) and lo = bf16(x - hi); both multiply the weights dequantized
 * to bf16 (E2M1 * e4m3, exact) with f32 accumulation on the tensor cores
 * (tcgen05 kind::f16), then y[m, n] = g[n] * acc.  bf16 x has lo = 0 (one
 * pass).  Any row_begin; x [m, K] 16-byte aligned; workspace 256-byte
 * aligned, fpb_nvfp4_gemm_hilo_workspace_bytes(m, rows, K, x_dtype) bytes
 * (the split activations and the rows' bf16 weights). */
size_t fpb_nvfp4_gemm_hilo_workspace_bytes(size_t m, size_t rows, size_t k, int x_dtype);
int fpb_nvfp4_gemm_hilo(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                        size_t m, void *y, int y_dtype, void *workspace, size_t workspace_bytes, void *stream);
/* The NVFP4 GEMV on the tensor cores (no reference counterpart for the
 * method; same results as gemv() up to f32 rounding): each row of x
 * (`tokens` of them, 1..16) becomes 8 NVFP4 digit planes (plane 0 = x with
 * the config-0 quantize rule, plane p = the residual of the planes before
 * it, each with its own global: x to about 2^-27 of its magnitude), the
 * planes of up to 16 tokens are the 128-row A operand of tcgen05
 * kind::mxf4nvf4 against the weight rows (the hardware decodes e2m1 / e4m3),
 * and the epilogue adds each token's 8 plane rows times their globals.
 * y [tokens, row_end - row_begin].  cols % 256 == 0, cols <= 4096,
 * row_begin % 128 == 0; workspace 256-byte aligned,
 * fpb_nvfp4_gemv_planes_workspace_bytes(1, cols) bytes.
 * fpb_nvfp4_moe_gemv_planes: fpb_nvfp4_moe_gemv (distinct experts, device
 * count) the same way; rows_per_expert % 128 == 0; x_stride 0 (one x for
 * every expert: workspace for 1 group) or per distinct expert (cap groups). */
size_t fpb_nvfp4_gemv_planes_workspace_bytes(size_t groups, size_t k);
int fpb_nvfp4_gemv_planes(fpb_nvfp4_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype,
                          int tokens, void *y, int y_dtype, void *workspace, size_t workspace_bytes, void *stream);
int fpb_nvfp4_moe_gemv_planes(fpb_nvfp4_matrix *w, size_t rows_per_expert, const int32_t *distinct,
                              const int32_t *count, int cap, const void *x, int x_dtype, size_t x_stride, int tokens,
                              void *y, int y_dtype, void *workspace, size_t workspace_bytes, void *stream);
/* A prepared tensor-core GEMV batch: the segments of fpb_nvfp4_gemv_batched
 * (each its own matrix rows, x [batch, cols] and y [batch, rows]) with every
 * pointer fixed at creation, run as one plane encode + one tcgen05 launch
 * (fpb_nvfp4_gemv_planes per segment, in one kernel).  create validates,
 * allocates the segment table and the planes workspace and synchronises
 * `stream` (load time); run allocates nothing and reads nothing on the host
 * (graph-capturable).  cols % 256 == 0, cols <= 4096, every row_begin a
 * multiple of 128, 1 <= batch <= 16, at most 1024 segments
 * (FPB_ERR_UNSUPPORTED for other shapes: use fpb_nvfp4_gemv_batched). */
typedef struct fpb_gemv_batch fpb_gemv_batch;
int fpb_nvfp4_gemv_batch_create(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype, int batch,
                                void *stream, fpb_gemv_batch **out);
/* The prepared batch under BASELINE config 2's W4A4 rule: members as above
 * but each x is [m, K] (f32/bf16, m <= 128, K % 256 == 0) and y [m, rows];
 * every distinct x is quantized to NVFP4 per tensor (global = amax / 2688,
 * the codes of fpb_nvfp4_quantize_act) and y = fpb_nvfp4_gemm's W4A4 result
 * (bit for bit).  One amax launch, one encode launch and one tcgen05 launch
 * over all members' 128-row weight tiles per fpb_nvfp4_gemv_batch_run, so
 * that a few tokens against many matrices keep every SM busy; the handle is
 * run and destroyed with fpb_nvfp4_gemv_batch_run / _destroy. */
int fpb_nvfp4_gemm_batch_create(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype, int m,
                                void *stream, fpb_gemv_batch **out);
/* fpb_nvfp4_gemv_batch_create whose members' results go, instead of to y, to
 * n_peer copies each: y_peers [count * n_peer] host array of device
 * pointers (member i's copies at y_peers[i * n_peer .. + n_peer), each laid
 * out like its y, 2-byte (bf16) or 4-byte (f32) aligned, n_peer <= 8).  For
 * an N-split GEMV the copies are this rank's slice in every rank's gathered
 * output (buffers of the other GPUs opened with fpb_ipc_open): the epilogue
 * does the all-gather with plain stores over NVLink and ends with a
 * system-scope fence; the caller orders the readers after it with a barrier
 * on the stream (e.g. a one-word fpb_comm_all_reduce), and the next run's
 * stores after the readers. */
int fpb_nvfp4_gemv_batch_create_peers(const fpb_gemv_segment *segs, int count, int x_dtype, int y_dtype, int batch,
                                      const void *const *y_peers, int n_peer, void *stream, fpb_gemv_batch **out);
int fpb_nvfp4_gemv_batch_run(const fpb_gemv_batch *b, void *stream);
int fpb_nvfp4_gemv_batch_destroy(fpb_gemv_batch *b);
/* The down projection after the gate/up one: gate_up [cap][tokens][2 * cols]
 * f32 (distinct expert u's block at gate_up + u * gate_up_stride, gate
 * columns first) and the GEMV input is silu(gate) * up (swiglu.rs:16) in f32,
 * encoded straight into planes (no SwiGLU launch, no rounding of h). */
int fpb_nvfp4_moe_gemv_planes_glu(fpb_nvfp4_matrix *w, size_t rows_per_expert, const int32_t *distinct,
                                  const int32_t *count, int cap, const float *gate_up, size_t gate_up_stride,
                                  int tokens, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                                  void *stream);
/* Grouped (MoE) GEMM on quantized activations; replaces
 * nvfp4_grouped_gemm_view (gemm/nvfp4.rs:209-264, kernel :56-107).  A holds
 * the prefill layout's padded_rows gathered rows (a multiple of 128: the
 * layout is built with tile_rows = 128); row tile t (128 rows) belongs to
 * expert tile_experts[t] (device int32 [padded_rows / 128]) and is
 * multiplied by that expert's rows [e*rows_per_expert, (e+1)*rows_per_expert)
 * of w:  y[t*128 + i, n] = ga * g[e*rpe + n] * sum_k a(t*128+i, k) w(e*rpe+n, k).
 * y: [padded_rows, rows_per_expert]; rows_per_expert % 128 == 0.  An expert
 * id outside [0, w.rows / rows_per_expert) leaves that tile unwritten and
 * records device error 106 (fpb_device_error).  token_rows (nullable, the
 * layout's token of each row, -1 = padding): padding rows' outputs are then
 * not needed (rows of a 32-row group that is all padding are not written,
 * the others hold unspecified values), so their activations may be anything
 * (see FPB_QUANT_SKIP_PADDING). */
int fpb_nvfp4_grouped_gemm_q(fpb_nvfp4_matrix *w, const uint8_t *a_packed, const uint8_t *a_sf_tiled,
                             const float *a_global, size_t padded_rows, const int32_t *tile_experts,
                             const int32_t *token_rows, size_t rows_per_expert, void *y, int y_dtype,
                             void *stream);
/* First error code a tensor-core kernel recorded (0: none; bounded waits
 * that gave up); synchronises the device; reset != 0 clears it. */
int fpb_device_error(int *out, int reset);

/* ---- FP8 E4M3 weights and the prefill FP8 GEMM (tcgen05 kind::f8f6f4) ----
 * Replaces HostFp8Matrix / Fp8Matrix (weights/fp8.rs:8-132) and fp8_gemm /
 * fp8_gemm_view / fp8_grouped_gemm_view (gemm/mod.rs:67-206, 417-697).
 * bits: e4m3 [rows, cols] row-major; scales f32: a [rows/block_n, cols/block_k]
 * grid (Fp8Scaling::Blocks), or one per row when block_n = block_k = 0
 * (Fp8Scaling::Rows).  The reference keeps f32 activations (bf16 hi/lo MMAs);
 * this path quantizes them to e4m3 with one f32 scale per token
 * (amax/448), the W8A8 setting of the task's config 1:
 *   y[m, n] = a_s[m] * sum_kb w_s[n/block_n, kb] * sum_{k in kb} a[m,k] w[n,k]
 * (rows mode: a_s[m] * w_s[n] * sum_k a[m,k] w[n,k]).  The GEMM needs block
 * sizes that are multiples of 128 (FPB_ERR_UNSUPPORTED otherwise). */
typedef struct fpb_fp8_matrix fpb_fp8_matrix;
/* HostFp8Matrix::from_parts / with_row_scales validation (weights/fp8.rs:30-99):
 * FPB_ERR_FORMAT with the reference's messages. */
int fpb_fp8_validate(size_t bits_len, const float *scales, size_t scales_len, size_t rows, size_t cols,
                     size_t block_n, size_t block_k);
/* HostFp8Matrix::upload (weights/fp8.rs:114-131) from host buffers. */
int fpb_fp8_matrix_create(const uint8_t *bits, const float *scales, size_t rows, size_t cols,
                          size_t block_n, size_t block_k, void *stream, fpb_fp8_matrix **out);
/* Same from device buffers (copied; the scales are checked finite). */
int fpb_fp8_matrix_create_device(const uint8_t *bits, const float *scales, size_t rows, size_t cols,
                                 size_t block_n, size_t block_k, void *stream, fpb_fp8_matrix **out);
int fpb_fp8_matrix_destroy(fpb_fp8_matrix *m);
int fpb_fp8_matrix_shape(const fpb_fp8_matrix *m, size_t *rows, size_t *cols, size_t *block_n,
                         size_t *block_k);
int fpb_fp8_matrix_download(const fpb_fp8_matrix *m, uint8_t *bits, float *scales, void *stream);
/* Quantizes w [rows, cols] (f32 or bf16, device) to e4m3: scale = amax/448
 * per block_n x block_k block (block_n = block_k = 0: per row, which is also
 * the per-token activation rule), bits = RN_e4m3_satfinite(w / scale). */
int fpb_fp8_quantize(const void *w, int dtype, size_t rows, size_t cols, size_t block_n, size_t block_k,
                     uint8_t *bits, float *scales, void *stream);
/* Workspace of fpb_fp8_gemm (quantized activations and their scales). */
size_t fpb_fp8_gemm_workspace_bytes(size_t m, size_t k);
/* GEMM on quantized activations a_bits [m, K] with per-token a_scales [m];
 * weight rows [row_begin, row_end) (row_end 0 = all), row_begin a multiple of
 * 128 and of block_n; y [m, row_end - row_begin]. */
int fpb_fp8_gemm_q(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const uint8_t *a_bits,
                   const float *a_scales, size_t m, void *y, int y_dtype, void *stream);
/* The same with a stream-K schedule when `split_ws` (256-byte aligned, at
 * least fpb_fp8_gemm_split_bytes(m, K, rows) bytes) is given and the GEMM has
 * fewer 128 x 256 tiles than the GPU has SMs: one CTA per SM, each taking an
 * equal share of all tiles' 128-wide K blocks; a tile split between CTAs is
 * finished by the last of them from f32 partial sums in the workspace (no CTA
 * waits for another; the parts are added in a fixed order).  Otherwise, or
 * with a too small or null workspace: as fpb_fp8_gemm_q. */
int fpb_fp8_gemm_q_split(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const uint8_t *a_bits,
                         const float *a_scales, size_t m, void *y, int y_dtype, void *split_ws,
                         size_t split_bytes, void *stream);
size_t fpb_fp8_gemm_split_bytes(size_t m, size_t k, size_t n);
/* Quantize x [m, K] (f32 or bf16) into `workspace` and run the GEMM; a
 * workspace of fpb_fp8_gemm_workspace_bytes(m, K) + fpb_fp8_gemm_split_bytes(m,
 * K, rows) bytes also gets the stream-K schedule. */
int fpb_fp8_gemm(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype, size_t m,
                 void *y, int y_dtype, void *workspace, size_t workspace_bytes, void *stream);
/* fp8_gemm / fp8_gemm_view with the reference's activation semantics
 * (gemm/mod.rs:87-100 blocks, 155-168 rows): f32 (or bf16) x as bf16 hi + lo
 * times the e4m3 weights in bf16, f32 accumulation on the tensor cores.  Row
 * scales multiply the sums (y = s[n] * acc); block scales (any block_n,
 * block_k dividing the matrix) are folded into the weights, w * s split into
 * bf16 hi + lo (the same product to about 2^-16).  row_begin a multiple of
 * block_n; cols % 8 == 0; workspace 256-byte aligned,
 * fpb_fp8_gemm_hilo_workspace_bytes(m, rows, K, x_dtype, blocks != 0). */
size_t fpb_fp8_gemm_hilo_workspace_bytes(size_t m, size_t rows, size_t k, int x_dtype, int blocks);
int fpb_fp8_gemm_hilo(fpb_fp8_matrix *w, size_t row_begin, size_t row_end, const void *x, int x_dtype, size_t m,
                      void *y, int y_dtype, void *workspace, size_t workspace_bytes, void *stream);
/* Grouped (MoE) GEMM, as fpb_nvfp4_grouped_gemm_q: row tile t (128 rows) of
 * a_bits [padded_rows, K] uses expert tile_experts[t]'s rows
 * [e*rows_per_expert, (e+1)*rows_per_expert); device error 306 on a bad id. */
int fpb_fp8_grouped_gemm_q(fpb_fp8_matrix *w, const uint8_t *a_bits, const float *a_scales,
                           size_t padded_rows, const int32_t *tile_experts, size_t rows_per_expert,
                           void *y, int y_dtype, void *stream);

/* ---- MoE on the device ----------------------------------------------------
 * The reference runs the router top-k on the GPU but builds the sorted layout
 * on the host (PrefillPlan::top_k, moe.rs:545-585); here it stays on the
 * device.  Layout arrays are sized `cap` >= fpb_prefill_layout_max_padded_rows
 * (a multiple of tile_rows); row tiles past the real end get expert id -1,
 * which fpb_nvfp4_grouped_gemm_q / fpb_fp8_grouped_gemm_q skip. */
/* top_k_prefill (moe.rs:15-68): logits f32 [tokens, ld >= experts] ->
 * ids int32 / weights f32 [tokens, width]: k rounds of the largest remaining
 * logit (lowest id among equals), weight exp(l - max) / sum over the k; with
 * shared_gate (f32 [tokens]) slot k is expert `experts`, weight sigmoid(gate).
 * width <= 32, experts <= 2048.  One warp per token. */
int fpb_moe_topk(const float *logits, size_t ld, const float *shared_gate, size_t tokens, size_t experts,
                 size_t top_k, size_t width, int32_t *ids, float *weights, void *stream);
/* PrefillLayout::from_indices (moe.rs:452-516) on the device, over the first
 * `slots` entries of each row of ids [tokens, width]: stable counting sort by
 * expert (experts ids in [0, experts)), each padded to tile_rows (a power of
 * two).  Outputs: token_rows [cap] (-1 = padding), tile_experts [cap/tile_rows]
 * (-1 past the end), inverse [tokens, width] (0 in unused slots), ranges
 * [experts][2] (start, count), padded_rows (device int32).  Three launches
 * and three memsets, no host synchronisation; device error 401 on an id out
 * of range. */
int fpb_moe_layout(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts,
                   size_t tile_rows, size_t cap, int32_t *token_rows, int32_t *tile_experts,
                   int32_t *inverse, size_t *ranges, int32_t *padded_rows, void *scratch,
                   size_t scratch_bytes, void *stream);
/* Device scratch fpb_moe_layout needs (per-CTA expert counts). */
size_t fpb_moe_layout_scratch_bytes(size_t tokens, size_t slots, size_t experts);
/* fpb_moe_layout where an id of -1 is a route that is not there (the
 * expert-parallel receiver's slots owned by other ranks): it takes no row, its
 * inverse entry is -1 (every unused slot's is) and it is no error; other ids
 * outside [0, experts) are device error 401 as above.  fpb_moe_combine skips
 * slots whose inverse is negative. */
int fpb_moe_layout_masked(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts,
                          size_t tile_rows, size_t cap, int32_t *token_rows, int32_t *tile_experts,
                          int32_t *inverse, size_t *ranges, int32_t *padded_rows, void *scratch,
                          size_t scratch_bytes, void *stream);
/* gather_prefill_view (moe.rs:71-89, 705-733): out [rows, cols] (f32/bf16),
 * row r = x[token_rows[r]] or zeros. */
int fpb_moe_gather(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *token_rows,
                   size_t rows, void *out, int out_dtype, void *stream);
/* The gather fused with the NVFP4 activation quantize of fpb_nvfp4_quantize_act
 * (global from amax over x): packed [rows, cols/2], tiled factors, global.
 * valid_rows (nullable device int32, e.g. fpb_moe_layout's padded_rows):
 * rows at or past it are not written (their row tiles are skipped); with
 * FPB_QUANT_SKIP_PADDING neither are padding rows (token -1).  workspace
 * (nullable, 256-byte aligned, fpb_moe_gather_quantize_workspace_bytes):
 * when given and cols % 64 == 0, each token row is encoded once and its codes
 * and factors are copied to every layout row that routes it (same bytes:
 * the encode is row-local with one global), instead of encoding each
 * gathered row. */
int fpb_moe_gather_quantize(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *token_rows,
                            size_t rows, const int32_t *valid_rows, uint8_t *packed, uint8_t *sf_tiled,
                            float *global_out, float *amax_scratch, int flags, void *workspace,
                            size_t workspace_bytes, void *stream);
size_t fpb_moe_gather_quantize_workspace_bytes(size_t tokens, size_t cols);
/* swiglu (swiglu.rs:5-20): out [rows, inter] = gate / (1 + exp(-gate)) * up,
 * gate = gate_up[:, :inter], up = gate_up[:, inter:]. */
int fpb_swiglu(const void *gate_up, int dtype, size_t rows, size_t inter, void *out, int out_dtype,
               void *stream);
/* SwiGLU fused with the NVFP4 activation quantize (input of the down GEMM);
 * global from amax over the first valid_rows rows (nullable: all rows). */
int fpb_swiglu_quantize(const void *gate_up, int dtype, size_t rows, const int32_t *valid_rows, size_t inter,
                        uint8_t *packed, uint8_t *sf_tiled, float *global_out, float *amax_scratch, int flags,
                        void *stream);
/* The gate/up GEMM fused with SwiGLU (gemm/nvfp4.rs:57-105 grouped GEMM, then
 * swiglu.rs:16 on its f32 output): w holds experts of 2*inter rows each
 * (gate rows, then up rows); h [padded_rows, inter] (f32/bf16, 16-byte
 * aligned) = silu(gate) * up computed from the f32 accumulators (no rounding
 * of gate/up, as the reference's f32 swiglu input; exp and the division by
 * hardware approximations, relative error about 1e-6); *amax_bits = max |h| as
 * stored (float bits; zeroed first).  inter % 64 == 0.  Needs the matrix's
 * interleaved factor copy from fpb_nvfp4_matrix_prepare_glu(w, inter)
 * (FPB_ERR_INVALID_ARGUMENT otherwise); allocates nothing.
 * token_rows as in fpb_nvfp4_grouped_gemm_q; padding rows are also left out
 * of the amax. */
int fpb_nvfp4_grouped_gemm_swiglu_q(fpb_nvfp4_matrix *w, const uint8_t *a_packed, const uint8_t *a_sf_tiled,
                                    const float *a_global, size_t padded_rows, const int32_t *tile_experts,
                                    const int32_t *token_rows, size_t inter, void *h, int h_dtype,
                                    uint32_t *amax_bits, void *stream);
/* NVFP4 activation quantize of rows x [rows, cols] (f32/bf16, 16-byte
 * aligned) as fpb_swiglu_quantize without the SwiGLU: with
 * FPB_QUANT_AMAX_GIVEN the global comes from *amax_scratch (e.g. the fused
 * GEMM's amax_bits); rows at or past *valid_rows are not written, nor (with
 * FPB_QUANT_SKIP_PADDING) rows whose token_rows entry is -1. */
int fpb_rows_quantize(const void *x, int dtype, size_t rows, const int32_t *valid_rows,
                      const int32_t *token_rows, size_t cols, uint8_t *packed, uint8_t *sf_tiled,
                      float *global_out, float *amax_scratch, int flags, void *stream);
/* |x| maximum over x[0, n) (f32/bf16) or over SwiGLU(gate_up) rows, as float
 * bits in *amax_scratch (zeroed first unless accumulate != 0). */
int fpb_act_amax(const void *x, int dtype, size_t n, float *amax_scratch, int accumulate, void *stream);
int fpb_swiglu_amax(const void *gate_up, int dtype, size_t rows, const int32_t *valid_rows, size_t inter,
                    float *amax_scratch, int accumulate, void *stream);
/* combine / combine_prefill (moe.rs:91-109, 779-822): out [tokens, cols] =
 * sum over the first `slots` slots of weights[t, s] * routed[inverse[t, s]]
 * (routed [routed_rows, cols]; a row index outside it adds nothing). */
int fpb_moe_combine(const void *routed, int r_dtype, size_t routed_rows, size_t cols, const int32_t *inverse,
                    const float *weights, size_t tokens, size_t width, size_t slots, void *out, int out_dtype,
                    void *stream);
/* combine_add_norm_{view,prefill} (moe.rs:111-147, 824-859): out = residual +
 * combine, normed = out * rsqrt(mean(out^2) + eps) * gamma (f32). */
/* fpb_moe_combine with token t's output row at row t % chunk_rows of
 * out_chunks[t / chunk_rows] (a device table of pointers, each 16-byte
 * aligned; e.g. other GPUs' buffers, written with plain peer stores and a
 * system-scope fence at the end, as fpb_ep_dispatch_chunks). */
int fpb_moe_combine_chunks(const void *routed, int r_dtype, size_t routed_rows, size_t cols,
                           const int32_t *inverse, const float *weights, size_t tokens, size_t width, size_t slots,
                           void *const *out_chunks, size_t chunk_rows, int out_dtype, void *stream);
int fpb_moe_combine_add_norm(const void *routed, int r_dtype, size_t routed_rows, size_t cols,
                             const int32_t *inverse, const float *weights, size_t tokens, size_t width,
                             size_t slots, const float *residual, const float *gamma, float eps, float *out,
                             float *normed, void *stream);

/* Expert-parallel dispatch (no reference counterpart: the reference runs on
 * one GPU).  Experts are sharded `experts_per_rank` per rank.
 * fpb_moe_route_dest: dest [tokens, width] = ids / experts_per_rank (first
 * `slots` slots, 0 after).  Laying dest out with fpb_moe_layout (ranks as
 * experts, tile_rows 1) gives the send order and its `inverse`; then
 * fpb_moe_route_meta writes send_expert[inverse[t, s]] = ids[t, s] %
 * experts_per_rank (the receiver's local expert id; rows >= `rows` skipped). */
int fpb_moe_route_dest(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts_per_rank,
                       int32_t *dest, void *stream);
int fpb_moe_route_meta(const int32_t *ids, const int32_t *inverse, size_t tokens, size_t width, size_t slots,
                       size_t experts_per_rank, size_t rows, int32_t *send_expert, void *stream);

/* Expert parallel with fixed capacity: one record per (token, destination
 * rank), never one per route, in chunks of equal size, so the all-to-alls
 * need no host-read counts and a layer is one CUDA graph.
 * A record (fpb_ep_record_bytes(cols, width) bytes, a multiple of 16) holds
 * the token's NVFP4 row - codes [cols/2] at offset 0, row-major e4m3 factors
 * [cols/16] at offset cols/2 - then int32 ids [width] (receiver-local expert
 * of each slot, -1 where another rank owns it or the record is empty) and f32
 * routing weights [width], each region 16-byte aligned.
 * fpb_ep_dispatch: ids / weights [tokens, width] (fpb_moe_topk's output, the
 * first `slots` used), experts split evenly over nranks (<= 32) ranks, cols %
 * 64 == 0, x [tokens, cols] (f32/bf16, 16-byte aligned), amax = the amax
 * word all-reduced (MAX) over the ranks (fpb_act_amax + fpb_comm_all_reduce),
 * so the global (amax / 2688, written to global_out) is the single-GPU
 * layer's.  Writes records [nranks][tokens] (chunk d for rank d: the tokens
 * that route to d in token order, then empty records) and positions
 * [tokens * nranks + nranks] int32: positions[t * nranks + d] = d * tokens +
 * the token's record index in chunk d, or -1; the last nranks entries are the
 * chunk counts.  Three launches (two above 10240 tokens); device error 403 on
 * an id outside [0, experts).
 * The receiver turns the records it got (nranks chunks) into dense route
 * tables with fpb_ep_unpack, lays them out with fpb_moe_layout_masked and
 * gathers the NVFP4 rows with fpb_moe_gather_codes (code_stride = sf_stride =
 * the record size, factors at records + cols/2); after the expert GEMMs,
 * fpb_moe_combine with f32 output gives each record's partial sum (its
 * routes in slot order), which goes back in the same fixed chunks; the source
 * sums the partials in rank order with fpb_moe_combine over `positions`
 * (width = slots = nranks, weights 1). */
size_t fpb_ep_record_bytes(size_t cols, size_t width);
int fpb_ep_dispatch(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *ids,
                    const float *weights, size_t width, size_t slots, size_t experts, size_t nranks,
                    const float *amax, void *records, int32_t *positions, float *global_out, void *stream);
/* fpb_ep_dispatch writing through a device table of nranks chunk pointers
 * (chunks[d] = where chunk d's `tokens` records go, each 16-byte aligned),
 * e.g. straight into each destination GPU's receive buffer (its chunk for
 * this rank, opened with fpb_ipc_open): plain peer stores over NVLink, no
 * all-to-all.  The kernel ends with a system-scope fence; the caller orders
 * the receivers' reads after it with a barrier on the stream (e.g. a
 * one-word fpb_comm_all_reduce).  self_rank (-1 if none): the chunk in this
 * GPU's memory, where each row is encoded before being copied to the others. */
int fpb_ep_dispatch_chunks(const void *x, int x_dtype, size_t tokens, size_t cols, const int32_t *ids,
                           const float *weights, size_t width, size_t slots, size_t experts, size_t nranks,
                           const float *amax, void *const *chunks, int self_rank, int32_t *positions,
                           float *global_out, void *stream);
/* ids / weights [rows, width] from `rows` records (rows = nranks * tokens). */
int fpb_ep_unpack(const void *records, size_t rows, size_t cols, size_t width, int32_t *ids, float *weights,
                  void *stream);
/* The layout rows' NVFP4 codes from rows encoded once: row r of the layout
 * copies token token_rows[r]'s codes (codes + t * code_stride, cols/2 bytes)
 * and factors (sf + t * sf_stride, cols/16 bytes) into packed [rows, cols/2]
 * and the tiled factor layout; token -1 rows are zeros (skipped with
 * FPB_QUANT_SKIP_PADDING in flags).  cols % 64 == 0; codes and code_stride
 * 16-byte aligned, sf and sf_stride 4-byte aligned. */
int fpb_moe_gather_codes(const uint8_t *codes, size_t code_stride, const uint8_t *sf, size_t sf_stride,
                         size_t tokens, size_t cols, const int32_t *token_rows, size_t rows,
                         const int32_t *valid_rows, int flags, uint8_t *packed, uint8_t *sf_tiled, void *stream);

/* ---- decode step of the hybrid MoE decoder -----------------
 * The operations around the quantized matmuls in firepit's decode step
 * (firepit src/plan.rs:283-420, src/execute.rs:334-716); the linear layers
 * are the NVFP4 GEMVs above.  All activations f32 unless a dtype says so;
 * `pitch` arguments are elements between rows.  Positions are device int32
 * [batch] (the token's index in its session). */
/* embedding.rs: out [rows, hidden] f32 = table_bf16[ids[r]] (device error
 * 501 on an id outside [0, vocab); that row is zeroed). */
int fpb_embedding(const void *table_bf16, size_t vocab, size_t hidden, const int32_t *ids, size_t rows,
                  float *out, void *stream);
/* norm.rs rms_norm / add_norm: out = x * rsqrt(mean(x^2) + eps) * gamma over
 * `width` columns of each row; with residual_delta, x = x + residual_delta
 * is first stored to sum_out (f32, [rows, width] contiguous). */
int fpb_rms_norm(const void *x, int x_dtype, size_t x_pitch, const float *residual_delta, float *sum_out,
                 size_t rows, size_t width, const float *gamma, float eps, void *out, int out_dtype,
                 size_t out_pitch, void *stream);
/* The full-attention layer's per-head RMSNorms of q (the first head_dim of
 * each 2*head_dim pitch of q_gate) and k, RoPE over the first rotary_dim
 * dims (rope.rs:6-22, inverse frequencies 1 / theta^(i / half) as
 * rope.rs:110-113, angles pos * inv_freq), q to q_out [batch, q_heads,
 * head_dim], k and v appended to the caches [batch, max_seq, kv_heads,
 * head_dim] at each row's position (attention.rs:6-30).  Device error 502 on
 * a position outside [0, max_seq). */
int fpb_attn_prepare(const float *q_gate, size_t qg_pitch, const float *k, size_t k_pitch, const float *v,
                     size_t v_pitch, const float *q_gamma, const float *k_gamma, const int32_t *positions,
                     size_t batch, size_t q_heads, size_t kv_heads, size_t head_dim, size_t rotary_dim, float theta,
                     float eps, size_t max_seq, float *q_out, float *k_cache, float *v_cache, void *stream);
/* online_attention + output_gate (attention.rs:128-190): each query head
 * attends over cache positions 0 .. position of its row (GQA: q head h reads
 * kv head h / (q_heads / kv_heads)), scores * scale, softmax, times the
 * values; out [batch, q_heads * head_dim] = attn * sigmoid(gate) (gate: the
 * second head_dim of each head's q_gate pitch).  Positions are split into
 * chunks of chunk_len (0: 64) on separate blocks and merged.  head_dim <=
 * 256, q_heads / kv_heads <= 32; workspace fpb_attn_decode_workspace_bytes. */
size_t fpb_attn_decode_workspace_bytes(size_t batch, size_t q_heads, size_t head_dim, size_t max_seq,
                                       size_t chunk_len);
int fpb_attn_decode(const float *q, const float *k_cache, const float *v_cache, const int32_t *positions,
                    const float *q_gate, size_t qg_pitch, size_t batch, size_t q_heads, size_t kv_heads,
                    size_t head_dim, size_t max_seq, size_t chunk_len, float scale, void *workspace,
                    size_t workspace_bytes, void *out, int out_dtype, void *stream);
/* conv1d_silu (gdn.rs:6-63): per channel, SiLU of the causal conv of the
 * last `kernel` inputs; state [batch, channels, kernel - 1] keeps the
 * previous inputs and is shifted. */
int fpb_gdn_conv(const float *x, size_t x_pitch, float *state, const float *weight, size_t batch,
                 size_t channels, size_t kernel, float *out, void *stream);
/* delta_step (gdn.rs:206-263) on conv_out [batch, 2*key_heads*dk +
 * value_heads*dv] (q, k, v), gates a, b [batch, ab_pitch] (value_heads
 * used): beta = sigmoid(b), decay = exp(-exp(a_log) * softplus(a + dt_bias))
 * with the reference's series below -8; q, k L2-normalised (+ eps, q also
 * / sqrt(dk)); state [batch, value_heads, dk, dv] updated in place; out
 * [batch, value_heads, dv]. */
int fpb_gdn_delta(const float *conv_out, const float *a, const float *b, size_t ab_pitch, const float *a_log,
                  const float *dt_bias, float *state, size_t batch, size_t key_heads, size_t value_heads, size_t dk,
                  size_t dv, float eps, float *out, void *stream);
/* RMSNorm of each value head (gamma [dv]) times SiLU(z) (gdn.rs:266-278):
 * out [batch, heads * dv]. */
int fpb_gdn_gated_norm(const float *x, const float *z, size_t z_pitch, const float *gamma, size_t batch, size_t heads,
                       size_t dv, float eps, void *out, int out_dtype, void *stream);
/* fpb_gdn_conv + fpb_gdn_delta + fpb_gdn_gated_norm in one launch (the GDN
 * mixer after its projections): x [batch, x_pitch] the q/k/v projection,
 * conv_state / conv_weight as fpb_gdn_conv, a / b / a_log / dt_bias / state
 * as fpb_gdn_delta, z [batch, z_pitch] and gamma [dv] as fpb_gdn_gated_norm;
 * out [batch, value_heads * dv].  dk = dv = 128, value_heads = 2 *
 * key_heads and a conv kernel of 2..8 only (FPB_ERR_UNSUPPORTED otherwise:
 * use the three calls).  Same results up to f32 summation order. */
int fpb_gdn_step(const float *x, size_t x_pitch, float *conv_state, const float *conv_weight, size_t conv_kernel,
                 const float *a, const float *b, size_t ab_pitch, const float *a_log, const float *dt_bias,
                 float *state, const float *z, size_t z_pitch, const float *gamma, size_t batch, size_t key_heads,
                 size_t value_heads, size_t dk, size_t dv, float eps, void *out, int out_dtype, void *stream);
/* combine_add_norm_view (moe.rs:111-147) for decode: out[t] = residual[t] +
 * sum over slots s of weights[t, s] * routed[t * slots + s], normed =
 * RMSNorm(out) * gamma (f32 or bf16); slots <= 32. */
int fpb_decode_combine_add_norm(const float *routed, const float *weights, size_t width, size_t slots,
                                const float *residual, const float *gamma, size_t tokens, size_t hidden, float eps,
                                float *out, void *normed, int normed_dtype, void *stream);
/* greedy (firepit src/generation.rs:34-42): tokens[r] = index of the largest
 * finite logit of row r (lowest index among equals), positions[r] += 1, and
 * (history non-null) history[r * history_len + step[0]] = token, after which
 * step[0] advances (step: device int32 [2], the second word for the blocks'
 * arrivals, zero at start). */
int fpb_argmax_advance(const float *logits, size_t rows, size_t vocab, int32_t *tokens, int32_t *positions,
                       int32_t *history, size_t history_len, int32_t *step, void *stream);
/* The expert GEMV of several tokens (a decode batch): slot s = t *
 * slots_per_token + j of expert_ids [tokens, slots_per_token] reads x row t;
 * y [tokens * slots_per_token, rows_per_expert].  Otherwise as
 * fpb_nvfp4_expert_gemv. */
int fpb_nvfp4_expert_gemv_tokens(const fpb_nvfp4_matrix *w, const void *x, int x_dtype, const int32_t *expert_ids,
                                 int tokens, int slots_per_token, size_t rows_per_expert, void *y, int y_dtype,
                                 void *stream);
/* The decode MoE over distinct experts instead of (token, slot) pairs (no
 * reference counterpart: the reference runs expert_gemv_weight_view per
 * slot, gemv/mod.rs:137-206, reading a routed expert once per token).
 * fpb_moe_decode_plan: distinct[0, *count) = the distinct ids of ids
 * [tokens, width] (first `slots` of each row) in ascending order, -1 up to
 * cap (cap >= tokens * slots); map[t * slots + s] = index of ids[t, s] in
 * distinct.  Device error 107 (map -1) for an id outside [0, experts).
 * fpb_nvfp4_moe_gemv: for u < *count (device), y[u] [tokens, rows_per_expert]
 * (at y + u * tokens * rows_per_expert) = W[distinct[u]] x[u], x[u] =
 * [tokens, cols] at x + u * x_stride elements (x_stride 0: one x for all);
 * tokens <= 16.  K % 128 == 0, K <= 4096, tokens <= 8: one streaming launch
 * whose CTAs share the live rows (device error 203 on an id outside the
 * experts); other shapes: the register kernel over all cap slots (rows of
 * slots past the count are zero).  Each token's result equals the per-slot
 * expert GEMV's up to f32 summation order.
 * fpb_moe_decode_combine_add_norm: fpb_decode_combine_add_norm reading the
 * routed row of (t, s) at map[t * slots + s] * tokens + t of routed
 * [cap, tokens, hidden] (the moe GEMV's output layout); slots <= 32. */
int fpb_moe_decode_plan(const int32_t *ids, size_t tokens, size_t width, size_t slots, size_t experts,
                        int32_t *distinct, int32_t *count, size_t cap, int32_t *map, void *stream);
/* fpb_moe_topk followed by fpb_moe_decode_plan in one launch (decode-size
 * batches: tokens <= 32, experts <= 512): the shared-expert gate logit, when
 * gate_col >= 0, is column gate_col of each logits row (a router matrix with
 * the gate row stacked under the experts' rows); the plan covers the top_k
 * (+ 1 shared) slots with the shared expert as id `experts`. */
int fpb_moe_decode_route(const float *logits, size_t ld, long long gate_col, size_t tokens, size_t experts,
                         size_t top_k, size_t width, int32_t *ids, float *weights, int32_t *distinct,
                         int32_t *count, size_t cap, int32_t *map, void *stream);
int fpb_nvfp4_moe_gemv(const fpb_nvfp4_matrix *w, size_t rows_per_expert, const int32_t *distinct,
                       const int32_t *count, int cap, const void *x, int x_dtype, size_t x_stride, int tokens, void *y,
                       int y_dtype, void *stream);
int fpb_moe_decode_combine_add_norm(const float *routed, const int32_t *map, const float *weights, size_t width,
                                    size_t slots, const float *residual, const float *gamma, size_t tokens,
                                    size_t hidden, float eps, float *out, void *normed, int normed_dtype,
                                    void *stream);

/* ---- collectives (NCCL) ------------------------------------------------------
 * The reference runs on one GPU and has no collectives.  These are the
 * exchange steps of the multi-GPU paths: the all-gather of each rank's output
 * columns after an N-split GEMV/GEMM, and the all-to-all dispatch/combine and
 * amax MAX all-reduce of the expert-parallel MoE layer.  One communicator per
 * (process, GPU); rank 0 makes the unique id and the caller hands it to the
 * other ranks (a TCP store, MPI, a file).  NCCL is opened at run time
 * (libnccl.so.2); FPB_ERR_COMM when it is missing or a call fails.  The
 * collectives are enqueued on `stream` (asynchronous, capturable like any
 * NCCL call); every rank must make the same calls in the same order. */
#define FPB_COMM_ID_BYTES 128
/* Peer memory for kernels that store into another GPU's buffers (the
 * expert-parallel chunks): fpb_ipc_alloc makes a device buffer of its own
 * allocation, fpb_ipc_get_handle names it for other processes of the node,
 * fpb_ipc_open maps a peer's buffer (peer access enabled lazily),
 * fpb_ipc_close unmaps it, fpb_ipc_free frees an fpb_ipc_alloc buffer. */
#define FPB_IPC_HANDLE_BYTES 64
int fpb_ipc_alloc(size_t bytes, void **ptr);
int fpb_ipc_free(void *ptr);
int fpb_ipc_get_handle(const void *ptr, uint8_t handle[FPB_IPC_HANDLE_BYTES]);
int fpb_ipc_open(const uint8_t handle[FPB_IPC_HANDLE_BYTES], void **ptr);
int fpb_ipc_close(void *ptr);
/* Barrier of nranks GPUs over peer memory, one 32-thread launch on the
 * stream: flags = this rank's nranks uint32 words in a buffer every rank
 * maps (zeroed before first use), peer_flags = device table of every rank's
 * flags as this process maps them (fpb_ipc_open), counter = this rank's
 * device uint32 epoch counter (zeroed; the same number of barriers on every
 * rank).  Each rank stores the new epoch into every rank's flag word for it
 * (system-scope release) and waits for every rank's (acquire), so the stores
 * each rank made before its barrier - e.g. peer copies of
 * fpb_nvfp4_gemv_batch_create_peers or fpb_ep_dispatch_chunks - are visible
 * to all ranks after theirs.  A wait gives up after timeout_ms of global time
 * with device error 601 (fpb_device_error) and the kernel returns.  Cheaper
 * than a one-word NCCL all-reduce; graph-capturable. */
int fpb_peer_barrier(uint32_t *counter, const uint32_t *flags, uint32_t *const *peer_flags, int nranks, int rank,
                     int timeout_ms, void *stream);
/* The same barrier carrying one uint32 word: *value (device, in/out) becomes
 * the maximum of every rank's *value (e.g. activation amax float bits, as
 * fpb_comm_all_reduce MAX).  The flag buffer then needs 96 words (the flags
 * and two banks of slots, by epoch parity). */
int fpb_peer_all_reduce_max(uint32_t *counter, const uint32_t *flags, uint32_t *const *peer_flags, int nranks,
                            int rank, uint32_t *value, int timeout_ms, void *stream);
typedef struct fpb_comm fpb_comm;
/* Extra element types of the collectives (besides FPB_F32, FPB_BF16). */
enum { FPB_COMM_U32 = 2, FPB_COMM_I32 = 3, FPB_COMM_BYTES = 4 };
enum { FPB_COMM_SUM = 0, FPB_COMM_MAX = 1 };
/* 1 if NCCL could be loaded, else 0. */
int fpb_comm_available(void);
int fpb_comm_version(int *version);
int fpb_comm_unique_id(uint8_t id[FPB_COMM_ID_BYTES]);
/* Joins the communicator of `nranks` ranks named by `id` as `rank`, on CUDA
 * device `device` (blocks until every rank has joined). */
int fpb_comm_init(const uint8_t id[FPB_COMM_ID_BYTES], int nranks, int rank, int device, fpb_comm **out);
int fpb_comm_destroy(fpb_comm *c);
/* Aborts pending operations and frees the communicator: the way out for a
 * host watchdog when a peer died (no GPU-side wait is left behind). */
int fpb_comm_abort(fpb_comm *c);
/* FPB_ERR_COMM when the communicator recorded an asynchronous error. */
int fpb_comm_status(const fpb_comm *c);
int fpb_comm_size(const fpb_comm *c, int *nranks, int *rank);
/* recv [nranks][count] = every rank's send [count] in rank order. */
int fpb_comm_all_gather(fpb_comm *c, const void *send, void *recv, size_t count, int dtype, void *stream);
/* recv [count] = SUM or MAX over ranks of send [count] (MAX of FPB_COMM_U32
 * float bits of non-negative values is the float maximum). */
int fpb_comm_all_reduce(fpb_comm *c, const void *send, void *recv, size_t count, int dtype, int op,
                        void *stream);
/* Variable all-to-all: to each rank p, send_counts[p] elements from
 * send + send_offsets[p]; from each rank p, recv_counts[p] elements into
 * recv + recv_offsets[p] (host arrays of nranks entries, in elements). */
int fpb_comm_all_to_all(fpb_comm *c, const void *send, const size_t *send_counts, const size_t *send_offsets,
                        void *recv, const size_t *recv_counts, const size_t *recv_offsets, int dtype,
                        void *stream);

/* ---- MoE host bookkeeping (no GPU needed) -------------------------------- */
/* MoeDims::new (moe.rs:172-225): FPB_ERR_SHAPE on invalid dimensions. */
int fpb_moe_dims_validate(size_t hidden, size_t intermediate, size_t shared_intermediate,
                          size_t experts, size_t top_k);
/* ExpertSelection::parse checks (moe.rs:327-351): FPB_ERR_SELECTION. */
int fpb_expert_selection_validate(const int32_t *indices, const float *weights, size_t count,
                                  size_t experts, size_t top_k);
/* PrefillLayout::max_padded_rows (moe.rs:408-428). */
int fpb_prefill_layout_max_padded_rows(size_t tokens, size_t experts, size_t top_k,
                                       size_t tile_rows, size_t *out);
/* PrefillLayout::parse / from_indices (moe.rs:430-516), host counting sort.
 * weights may be NULL (from_indices).  See moe_host.cu for the outputs. */
int fpb_prefill_layout_host(const int32_t *indices, const float *weights, size_t count,
                            size_t experts, size_t top_k, size_t tile_rows, int32_t *token_rows,
                            size_t token_rows_cap, size_t *padded_rows, int32_t *tile_experts,
                            size_t tile_cap, size_t *n_tiles, int32_t *inverse, size_t *ranges);

/* ---- checkpoint files (crates/firepit/src/checkpoint.rs) -------------------
 * Safetensors reader: the on-disk format the reference loads NVFP4 / FP8
 * weights from (ModelOpt NVFP4: U8 [N, K/2] codes low nibble first, F8_E4M3
 * [N, K/16] scales, F32 scalar weight_scale_2; Qwen FP8: F8_E4M3 [N, K]
 * with BF16 [N/bn, K/bk] weight_scale_inv).  Host only; reads with pread.
 * The handle is read-only after open and may be shared between threads. */
typedef struct fpb_safetensors fpb_safetensors;

/* Stored dtypes (safetensors' Dtype names). */
enum {
  FPB_ST_BOOL = 0, FPB_ST_U8 = 1, FPB_ST_I8 = 2, FPB_ST_F8_E5M2 = 3, FPB_ST_F8_E4M3 = 4,
  FPB_ST_I16 = 5, FPB_ST_U16 = 6, FPB_ST_F16 = 7, FPB_ST_BF16 = 8, FPB_ST_I32 = 9,
  FPB_ST_U32 = 10, FPB_ST_F32 = 11, FPB_ST_F64 = 12, FPB_ST_I64 = 13, FPB_ST_U64 = 14
};

/* SafetensorsFile::open (checkpoint.rs:63-76): parses and validates the
 * header (every tensor's byte range against its dtype, shape and the file
 * size).  FPB_ERR_IO if the file cannot be opened, FPB_ERR_FORMAT if the
 * header is malformed. */
int fpb_safetensors_open(const char *path, fpb_safetensors **out);
void fpb_safetensors_close(fpb_safetensors *f);
/* Tensor names in data-offset order. */
size_t fpb_safetensors_count(const fpb_safetensors *f);
const char *fpb_safetensors_name(const fpb_safetensors *f, size_t i);
/* SafetensorsFile::has_tensor (checkpoint.rs:86-88): 1 or 0. */
int fpb_safetensors_has(const fpb_safetensors *f, const char *name);
/* SafetensorsFile::metadata (checkpoint.rs:78-84): NULL when absent. */
const char *fpb_safetensors_metadata(const fpb_safetensors *f, const char *key);
const char *fpb_safetensors_dtype_name(int dtype);
/* TensorInfo (checkpoint.rs:187-191): dtype code, shape (up to max_dims),
 * number of dimensions and byte size.  FPB_ERR_FORMAT "unknown tensor". */
int fpb_safetensors_info(const fpb_safetensors *f, const char *name, int *dtype, int64_t *shape,
                         int max_dims, int *ndim, size_t *nbytes);
/* SafetensorsFile::bytes (checkpoint.rs:158-167): `bytes` raw bytes of the
 * tensor from byte `byte_begin` of its range into host memory, after checking
 * that it is stored as `dtype` (FPB_ERR_FORMAT "expected X, got Y"). */
int fpb_safetensors_read(const fpb_safetensors *f, const char *name, int dtype, size_t byte_begin, void *dst,
                         size_t bytes);

#ifdef __cplusplus
}
#endif
#endif /* FIREPIT_B200_H */
