/*
 * synapse_oracle.h -- CPU restatement of eren23/synapse's quantized-matmul
 * arithmetic. TEST INFRASTRUCTURE ONLY: used by tests/, by the smoke check and
 * by the CPU-baseline legs of bench.py as the checker. Nothing in the shipped
 * CUDA path links or calls this code.
 *
 * Every function cites the reference file:line whose arithmetic it restates
 * (paths relative to the reference's `synapse/` workspace root).
 *
 * Parity status: partially pinned. The reference (Zig + Rust) cannot be built
 * in this container, so the restatement is pinned against the known-answer
 * tests of the reference's own test suites (tests/golden/kat.json). Q4_K and
 * Q6_K dequantisation have no reference test: for those the restatement of
 * weight_loading/gguf.rs:375-487 is the only pin ("parity unpinned").
 */
#ifndef SYNAPSE_ORACLE_H
#define SYNAPSE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: same values as synapse.h:27-35. */
#define ORC_OK 0
#define ORC_ERR_NULL_PTR 1
#define ORC_ERR_INVALID_ARG 2
#define ORC_ERR_SHAPE_MISMATCH 4

/* Weight formats (same numbering as include/synapse_cuda.h syn_qformat_t). */
#define ORC_FMT_INT8_KN 0
#define ORC_FMT_Q4_0 1
#define ORC_FMT_Q8_0 2
#define ORC_FMT_Q4_K 3
#define ORC_FMT_Q6_K 4

/* f16 bits -> f32, Zig version (zig/src/ops/qmatmul.zig:346-371). Exact. */
float orc_f16_zig(uint16_t bits);
/* f16 bits -> f32, Rust loader version (weight_loading/converter.rs:12-40).
 * Differs from the Zig one on subnormals: the normalisation counter starts at
 * 1 instead of 0, so every subnormal comes out at half its IEEE value. */
float orc_f16_rust(uint16_t bits);

/* zig/src/ops/quantize.zig:12-47 via syn_quantize_per_channel_int8
 * (zig/src/ffi/exports.zig:1275-1289). */
int orc_quantize_per_channel_int8(const float *data, size_t channels,
                                  size_t channel_size, int8_t *out,
                                  float *scales);

/* MinMaxCalibration::compute_scales (quantization/primitives/calibration.rs:11-24)
 * then QuantizedLinear::from_f32_with_scales + transpose_i8
 * (quantization/primitives/int8_linear.rs:21-70). w is [n,k] row-major; the
 * output is the reference's GEMM layout [k,n] plus [n] scales. */
void orc_quantize_weights_int8(const float *w, size_t n, size_t k,
                               int8_t *out_kn, float *scales);

/* syn_qgemm_int8 (zig/src/ffi/exports.zig:1313-1350) -> int8GemmTiled
 * (zig/src/ops/qmatmul.zig:37-99, 171-256, 442-549). */
int orc_qgemm_int8(size_t m, size_t n, size_t k, const int8_t *a, size_t lda,
                   const int8_t *b, size_t ldb, float *c, size_t ldc,
                   const float *scales_a, const float *scales_b);

/* naiveInt8Gemm (zig/src/ops/qmatmul.zig:106-128): one int32 accumulator
 * over all of K, used by the reference's own tiled-vs-naive test. */
void orc_naive_int8_gemm(size_t m, size_t n, size_t k, const int8_t *a,
                         size_t lda, const int8_t *b, size_t ldb, float *c,
                         size_t ldc, const float *scales_a,
                         const float *scales_b);

/* syn_q4_0_gemv (zig/src/ffi/exports.zig:1614-1628) -> q4_0GemvRow
 * (zig/src/ops/qmatmul.zig:276-343). */
int orc_q4_0_gemv(size_t n, size_t k, const float *a, const uint8_t *b_q4,
                  float *c);

/* Bytes of one row of K elements in a block format (0 if K is not a
 * multiple of the block). */
size_t orc_row_bytes(int fmt, size_t k);

/* GGUF block dequantisation (weight_loading/gguf.rs:255-288 Q8_0,
 * :294-330 Q4_0, :375-431 Q4_K, :440-487 Q6_K), f16 via orc_f16_rust. */
int orc_dequant(int fmt, const uint8_t *blocks, size_t numel, float *out);

/* matmul_t (ops/matmul.rs:55-79): out zeroed, then syn_sgemm(trans_a=0,
 * trans_b=1) (zig/src/ffi/exports.zig:725-763) -> sgemmTiled / f32GemvRow
 * (zig/src/ops/matmul.zig:125-347, 355-515). b is [n,k] row-major. */
int orc_sgemm_nt(size_t m, size_t n, size_t k, const float *a, size_t lda,
                 const float *b, size_t ldb, float *c, size_t ldc);

/* The reference's route for block formats on the LM path: dequantise at load
 * (orc_dequant) and run matmul_t. Convenience wrapper; w_f32 is scratch of
 * n*k floats provided by the caller. */
int orc_block_matmul(int fmt, size_t m, size_t n, size_t k, const float *x,
                     const uint8_t *w_blocks, float *w_f32, float *y);

/* ---- language-model epilogues (synapse_oracle_lm.c) ---- */

/* exp evaluated in double, rounded once to float (stand-in for the
 * reference's f32 exp on both sides of every parity check). */
float orc_exp(float x);
/* ops/norm.rs:8-37 with vecHsum (zig/src/ffi/exports.zig:503-514). */
void orc_rmsnorm(const float *x, const float *w, size_t rows, size_t h, float eps,
                 float *out);
/* models/lm/builder.rs:88-133 (no RoPE scaling). */
void orc_rope_tables(double base, size_t max_pos, size_t hd, float *cos_t, float *sin_t);
/* ops/rope.rs:13-60, RotateHalf. */
void orc_rope_inplace(float *qk, const float *cos_t, const float *sin_t, size_t seq,
                      size_t heads, size_t hd, size_t pos_off);
/* ops/activation.rs:117-130. */
void orc_softmax(float *x, size_t n);
/* matmul_nn (ops/matmul.rs:82-101) -> sgemmTiled(trans_b=0). */
int orc_sgemm_nn(size_t m, size_t n, size_t k, const float *a, size_t lda, const float *b,
                 size_t ldb, float *c, size_t ldc);
/* ops/attention.rs:70-147 (after the cache append); window 0 = none. */
void orc_attention_decode(const float *q, const float *kc, const float *vc, size_t len,
                          size_t n_heads, size_t n_kv, size_t hd, size_t window, float *out);
/* syn_fused_attention (zig/src/ffi/exports.zig:1364-1478). */
int orc_fused_attention(size_t seq_q, size_t seq_k, size_t hd, const float *q, const float *k,
                        const float *v, float *out);
/* quantization/lm/int8.rs:500-503. */
void orc_silu_mul(const float *g, const float *u, size_t n, float *out);
/* zig/src/ops/silu.zig:85-114. */
void orc_swiglu(const float *g, const float *u, size_t n, float *out);
/* generation/sampler.rs:217-224. */
uint32_t orc_argmax(const float *x, size_t n);

#ifdef __cplusplus
}
#endif
#endif
