/*
 * synapse_cuda.h -- C ABI of the B200 (sm_100a) backend for Synapse's
 * quantized-matmul hot path.
 *
 * Conventions follow synapse.h (reference: synapse/synapse.h:25-35 and
 * zig/src/ffi/exports.zig:1-3,55-63): every function returns a syn_status_t,
 * no exception crosses the boundary, null pointers are checked first, and a
 * zero-sized call returns SYN_OK without touching memory. Unlike the CPU
 * library, compute entry points take DEVICE pointers and a cudaStream_t
 * (passed as void*, NULL = legacy default stream); they are stream-ordered
 * and never synchronise. Handles (context, weights) are library-owned.
 *
 * Paths cited below are relative to the reference's `synapse/` root.
 */
#ifndef SYNAPSE_CUDA_H
#define SYNAPSE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* Status codes: 0-8 are synapse.h:27-35; 9-12 are new for the GPU.    */
/* ------------------------------------------------------------------ */
typedef int32_t syn_status_t;

#define SYN_OK                     0
#define SYN_ERR_NULL_PTR           1
#define SYN_ERR_INVALID_ARG        2
#define SYN_ERR_OUT_OF_MEMORY      3
#define SYN_ERR_SHAPE_MISMATCH     4
#define SYN_ERR_NOT_CONTIGUOUS     5
#define SYN_ERR_INVALID_AXIS       6
#define SYN_ERR_INVALID_DIMENSIONS 7
#define SYN_ERR_INTERNAL           8
#define SYN_ERR_CUDA               9
#define SYN_ERR_NCCL               10
#define SYN_ERR_TIMEOUT            11
#define SYN_ERR_UNSUPPORTED        12

/* Capability report: same struct as synapse.h (syn_capability_summary_t,
 * zig/src/ffi/exports.zig:98-106) with a new backend id. */
#ifndef SYN_CAPABILITY_SUMMARY_DEFINED
#define SYN_CAPABILITY_SUMMARY_DEFINED
typedef struct syn_capability_summary_t {
    uint32_t abi_version;
    uint32_t target_arch;
    uint32_t target_os;
    uint32_t simd_backend;
    uint32_t runtime_profile;
    uint32_t support_level;
    uint64_t feature_bits;
} syn_capability_summary_t;
#endif

#define SYN_BACKEND_CUDA_SM100 3
#define SYN_CUDA_FEATURE_INT8_QUANT (1ULL << 4)  /* = SYN_FEATURE_INT8_QUANT */
#define SYN_CUDA_FEATURE_Q4_0_GEMV  (1ULL << 5)  /* = SYN_FEATURE_Q4_0_GEMV */
#define SYN_CUDA_FEATURE_QMATMUL    (1ULL << 16) /* format-generic weight handles */

/* Weight formats accepted by syn_cuda_weight_upload. */
typedef enum syn_qformat_t {
    SYN_QFMT_INT8_KN = 0, /* reference GEMM layout: int8 [K,N] + f32 scales [N]
                             (quantization/primitives/int8_linear.rs:10-18) */
    SYN_QFMT_Q4_0 = 1,    /* GGUF blocks, 18 B / 32 (weight_loading/gguf.rs:294-330) */
    SYN_QFMT_Q8_0 = 2,    /* GGUF blocks, 34 B / 32 (gguf.rs:255-288) */
    SYN_QFMT_Q4_K = 3,    /* GGUF super-blocks, 144 B / 256 (gguf.rs:375-431) */
    SYN_QFMT_Q6_K = 4     /* GGUF super-blocks, 210 B / 256 (gguf.rs:440-487) */
} syn_qformat_t;

/* Element types of safetensors tensors (weight_loading/safetensors.rs:233-290). */
typedef enum syn_dtype_t {
    SYN_DTYPE_F32 = 0,
    SYN_DTYPE_F16 = 1,  /* IEEE half; converted like converter.rs:12-40 */
    SYN_DTYPE_BF16 = 2, /* upper 16 bits of an f32 (converter.rs:43-48) */
    SYN_DTYPE_I64 = 3,
    SYN_DTYPE_I32 = 4,
    SYN_DTYPE_U8 = 5
} syn_dtype_t;

typedef struct syn_cuda_ctx_s syn_cuda_ctx_t;
typedef struct syn_cuda_weight_s syn_cuda_weight_t;

/* ------------------------------------------------------------------ */
/* Context and capability                                              */
/* ------------------------------------------------------------------ */

/* Binds a device and creates the library state for it. New (the CPU
 * library has no context); replaces the implicit global state of
 * zig/src/ffi/exports.zig:47-49. */
syn_status_t syn_cuda_context_create(int device, syn_cuda_ctx_t **out);
syn_status_t syn_cuda_context_destroy(syn_cuda_ctx_t *ctx);

/* Reads and clears the context's device-side error word, where kernels
 * record asynchronous failures such as SYN_ERR_TIMEOUT. New (the CPU
 * library has no asynchronous errors). Synchronous. */
syn_status_t syn_cuda_context_get_error(syn_cuda_ctx_t *ctx, int32_t *status);

/* Replaces syn_capability_summary (zig/src/ffi/exports.zig:230-290). */
syn_status_t syn_cuda_capability_summary(syn_capability_summary_t *out);

/* Text of a status code, and of the last CUDA error seen on this thread. */
const char *syn_cuda_status_string(syn_status_t status);
const char *syn_cuda_last_error(void);

/* ------------------------------------------------------------------ */
/* Reference-mirroring entry points (device pointers, stream-ordered)  */
/* ------------------------------------------------------------------ */

/* Replaces syn_quantize_per_channel_int8 (synapse.h:341-350,
 * zig/src/ffi/exports.zig:1275-1289, zig/src/ops/quantize.zig:12-47).
 * Bit-exact with the reference. channels==0 or channel_size==0 ->
 * SYN_ERR_INVALID_ARG, as in the reference. */
syn_status_t syn_cuda_quantize_per_channel_int8(const float *data,
                                                size_t channels,
                                                size_t channel_size,
                                                int8_t *out, float *scales,
                                                void *stream);

/* Load-time weight quantisation on the device: replaces
 * MinMaxCalibration::compute_scales (quantization/primitives/calibration.rs:11-24)
 * + QuantizedLinear::from_f32_with_scales + transpose_i8
 * (quantization/primitives/int8_linear.rs:21-70). w: f32 [n,k] row-major;
 * out_kn: int8 [k,n] (the reference's GEMM layout); scales: f32 [n].
 * Bit-exact with the reference. */
syn_status_t syn_cuda_quantize_weights_int8(const float *w, size_t n, size_t k,
                                            int8_t *out_kn, float *scales,
                                            void *stream);

/* Replaces syn_qgemm_int8 (synapse.h:359-368,
 * zig/src/ffi/exports.zig:1313-1350, zig/src/ops/qmatmul.zig:37-99).
 * C = diag(scales_a) (A_i8 B_i8) diag(scales_b), B in the reference's
 * [K,N] layout with row stride ldb. C is fully overwritten. Bit-exact with
 * the reference, including the M>16 per-512-K-chunk float epilogue. */
syn_status_t syn_cuda_qgemm_int8(size_t m, size_t n, size_t k,
                                 const int8_t *a, size_t lda,
                                 const int8_t *b, size_t ldb,
                                 float *c, size_t ldc,
                                 const float *scales_a,
                                 const float *scales_b, void *stream);

/* Replaces syn_q4_0_gemv (zig/src/ffi/exports.zig:1614-1628, bound at
 * crates/synapse-sys/src/lib.rs:413-420; qmatmul.zig:276-343). b_q4 holds
 * the raw 18-byte Q4_0 blocks of an [N,K] matrix. k % 32 != 0 ->
 * SYN_ERR_SHAPE_MISMATCH. Matches within 1e-3 relative error. */
syn_status_t syn_cuda_q4_0_gemv(size_t n, size_t k, const float *a,
                                const uint8_t *b_q4, float *c, void *stream);

/* ------------------------------------------------------------------ */
/* Weight handles: one-time repack into the coalesced HBM layout       */
/* ------------------------------------------------------------------ */

/* Uploads one linear layer's weights (host memory) and repacks them on the
 * device. Replaces the load-time step of QuantizedLinear::from_f32
 * (int8_linear.rs:35-70, INT8_KN: host = int8 [K,N], scales = f32 [N]) and
 * of the GGUF loader (weight_loading/gguf.rs:156-248, block formats:
 * host = raw blocks of an [N,K] row-major matrix, scales = NULL).
 * Block formats need k % 32 (Q4_0, Q8_0) or k % 256 (Q4_K, Q6_K) == 0,
 * else SYN_ERR_SHAPE_MISMATCH. Synchronous. */
syn_status_t syn_cuda_weight_upload(syn_cuda_ctx_t *ctx, syn_qformat_t fmt,
                                    const void *host, size_t n, size_t k,
                                    const float *scales_or_null,
                                    syn_cuda_weight_t **out);
syn_status_t syn_cuda_weight_destroy(syn_cuda_weight_t *w);

/* Device bytes held by the repacked weight (HBM footprint). */
syn_status_t syn_cuda_weight_bytes(const syn_cuda_weight_t *w, size_t *bytes);

/* Debug hook: writes the dequantised [N,K] f32 matrix to host memory with
 * the reference's own formulas (gguf.rs:255-487 for block formats,
 * dequantizePerChannelInt8 quantize.zig:90-106 for INT8), bit-exact. */
syn_status_t syn_cuda_weight_dequant(const syn_cuda_weight_t *w,
                                     float *host_out);

/* Format-generic fused dequant matmul: y[m,N] = x[m,K] * W^T on device
 * pointers. INT8: quantises each x row (quantize.zig:12-47) and applies the
 * W8A8 product bit-exactly like QuantizedLinear::forward
 * (int8_linear.rs:87-117). Block formats follow the reference's route
 * "dequantise to f32, then matmul_t" (gguf.rs + ops/matmul.rs:55-79)
 * within 1e-3 relative error (normwise per output row: max|y - ref| /
 * max|ref|); Q4_K and Q6_K above 32 rows to about 1e-7.
 * Scratch: the context's buffers grow the first time a call needs more
 * (a larger m or weight). That growth calls cudaDeviceSynchronize, then
 * cudaFree / cudaMalloc, and is refused (SYN_ERR_UNSUPPORTED) while the
 * stream is being captured; warm a context up with its largest shapes
 * before capturing or timing. Calls at sizes already seen never
 * synchronise. The same holds for syn_cuda_qmatmul_int8_prequant and
 * syn_cuda_qmatmul_rmsnorm. */
syn_status_t syn_cuda_qmatmul(syn_cuda_ctx_t *ctx, const syn_cuda_weight_t *w,
                              const float *x, size_t m, float *y,
                              void *stream);

/* INT8 weight handle with activations already quantised (x_i8 [m,K],
 * scales_x [m]); mirrors QuantizedLinear::forward_pre_quantized
 * (int8_linear.rs:124-165). Bit-exact. */
syn_status_t syn_cuda_qmatmul_int8_prequant(syn_cuda_ctx_t *ctx,
                                            const syn_cuda_weight_t *w,
                                            const int8_t *x_i8,
                                            const float *scales_x, size_t m,
                                            float *y, void *stream);

/* One decode row through RMSNorm and a matmul in one launch:
 * x = rmsnorm(residual (+ delta), norm_weight) (ops/norm.rs:8-37, same
 * arithmetic as syn_cuda_add_rmsnorm; parallel_sum != 0 sums the squares in a
 * parallel order instead of vecHsum's), then y[1,N] = x * W^T as
 * syn_cuda_qmatmul. residual_out (optional, must not alias residual)
 * receives residual + delta. delta may be NULL. M = 1. */
syn_status_t syn_cuda_qmatmul_rmsnorm(syn_cuda_ctx_t *ctx, const syn_cuda_weight_t *w,
                                      const float *residual, const float *delta,
                                      const float *norm_weight, float eps,
                                      float *residual_out, int parallel_sum, float *y,
                                      void *stream);

/* Allocation-free variant of syn_cuda_qmatmul. It has no counterpart in the
 * reference: it is for callers that must not allocate device memory while
 * they run (latency-critical decode loops, processes whose device memory is
 * owned by an external pool or budget, hosts that forbid the CUDA
 * allocator). Same inputs and outputs as syn_cuda_qmatmul, and results
 * within the same tolerances: it always runs the GEMV, so INT8 is bit-exact
 * either way, while block formats from the tensor-core GEMM's row threshold
 * on differ from syn_cuda_qmatmul's values within 1e-3. No context is
 * needed, and the weight's device must be current.
 * Its scratch (split-K partial sums and arrival counters) is a fixed device
 * array of SYN_CUDA_NOALLOC_SCRATCH_BYTES that every GPU loading the library
 * keeps until exit. A call needing more returns SYN_ERR_OUT_OF_MEMORY without
 * launching anything. The first call on a device looks the array up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the one array and each resets its counters first: calls
 * whose execution overlaps on the GPU (other streams, other threads) race
 * and must be serialised by the caller. */
#define SYN_CUDA_NOALLOC_SCRATCH_BYTES (4u << 20)
syn_status_t syn_cuda_qmatmul_noalloc(const syn_cuda_weight_t *w,
                                      const float *x, size_t m, float *y,
                                      void *stream);

/* ------------------------------------------------------------------ */
/* Decoder-layer kernels around the matmuls (device pointers, stream-  */
/* ordered). Reductions follow the reference's order so that greedy    */
/* decoding reproduces its token ids.                                  */
/* ------------------------------------------------------------------ */

/* RoPE tables [max_pos, head_dim/2] on the host, as
 * precompute_rope_tables (models/lm/builder.rs:88-133, no scaling). */
syn_status_t syn_cuda_rope_tables(double base, size_t max_pos, size_t head_dim,
                                  float *cos_out, float *sin_out);

/* rmsnorm (ops/norm.rs:8-37; sum of squares in vecHsum order,
 * zig/src/ffi/exports.zig:503-514): out = (x * w) * 1/sqrt(ms + eps). */
syn_status_t syn_cuda_rmsnorm(const float *x, const float *weight, size_t rows,
                              size_t hidden, float eps, float *out, void *stream);
/* residual += delta (add_vecs, ops/vector.rs:1-9), then out = rmsnorm(residual). */
syn_status_t syn_cuda_add_rmsnorm(float *residual, const float *delta,
                                  const float *weight, size_t rows, size_t hidden,
                                  float eps, float *out, void *stream);
/* Embedding lookup (ids >= vocab give zeros, int8.rs:566-574) into x_out
 * (optional), then out = rmsnorm(x). ids: device int32 [rows]. */
syn_status_t syn_cuda_embed_rmsnorm(const float *table, size_t vocab,
                                    const int32_t *ids, size_t rows, size_t hidden,
                                    const float *weight, float eps, float *x_out,
                                    float *out, void *stream);

/* KV cache in HBM (zig/src/ops/kvcache.zig:13-170, syn_kvcache_* at
 * exports.zig:1879-1940): per layer and sequence, K and V [max_seq,
 * n_kv_heads*head_dim] f32. The length is per sequence and shared by all
 * layers (LayerCaches). Appends write at the current length; _advance
 * commits them. A call that would pass max_seq returns SYN_ERR_INVALID_ARG
 * (CacheFull, mapError exports.zig:122-136). */
typedef struct syn_cuda_kvcache_s syn_cuda_kvcache_t;
syn_status_t syn_cuda_kvcache_create(syn_cuda_ctx_t *ctx, size_t max_seq,
                                     size_t n_kv_heads, size_t head_dim,
                                     size_t num_layers, size_t batch,
                                     syn_cuda_kvcache_t **out);
/* Paged variant (no counterpart in the reference, whose cache is one
 * contiguous buffer per layer, kv_cache/cache.rs:26-340): every layer holds
 * a pool of n_pages pages of `page` positions; a sequence takes pages as it
 * grows (append, advance and the attention entry points) and returns them
 * on truncate / reset. No free page -> SYN_ERR_OUT_OF_MEMORY. page = 0 is
 * the contiguous cache. _view is unsupported on a paged cache. */
syn_status_t syn_cuda_kvcache_create_paged(syn_cuda_ctx_t *ctx, size_t max_seq,
                                           size_t n_kv_heads, size_t head_dim,
                                           size_t num_layers, size_t batch, size_t page,
                                           size_t n_pages, syn_cuda_kvcache_t **out);
/* Free pages of a paged cache (0 for a contiguous one). */
syn_status_t syn_cuda_kvcache_pages_free(const syn_cuda_kvcache_t *cache, size_t *n);
syn_status_t syn_cuda_kvcache_destroy(syn_cuda_kvcache_t *cache);
syn_status_t syn_cuda_kvcache_len(const syn_cuda_kvcache_t *cache, size_t seq,
                                  size_t *len);
/* Device pointers of one layer's K and V arrays of one sequence. */
syn_status_t syn_cuda_kvcache_view(const syn_cuda_kvcache_t *cache, size_t layer,
                                   size_t seq, float **k, float **v);
syn_status_t syn_cuda_kvcache_append(syn_cuda_kvcache_t *cache, size_t layer,
                                     size_t seq, const float *k, const float *v,
                                     size_t n_tokens, void *stream);
syn_status_t syn_cuda_kvcache_advance(syn_cuda_kvcache_t *cache, size_t seq,
                                      size_t n_tokens, void *stream);
/* truncateTo (kvcache.zig:109-113): only shortens. */
syn_status_t syn_cuda_kvcache_truncate(syn_cuda_kvcache_t *cache, size_t seq,
                                       size_t new_len, void *stream);
syn_status_t syn_cuda_kvcache_reset(syn_cuda_kvcache_t *cache, size_t seq,
                                    void *stream);

/* cached_attention_decode (ops/attention.rs:24-147) for sequences
 * [0, batch), one new token each: headwise RMSNorm of q and k (q_norm /
 * k_norm may be NULL = identity), RoPE at position len, K and raw V
 * appended at len, GQA attention over the last `window` positions (0 =
 * all). Rows: q/k/v of sequence b at q + b*ld etc.; out + b*ldo. The cache
 * length is not advanced. */
syn_status_t syn_cuda_attention_decode(syn_cuda_kvcache_t *cache, size_t layer,
                                       size_t batch, float *q, const float *k,
                                       const float *v, size_t ld, size_t n_heads,
                                       const float *q_norm, const float *k_norm,
                                       float eps, const float *rope_cos,
                                       const float *rope_sin, size_t window,
                                       float *out, size_t ldo, void *stream);
/* The first half of cached_attention_prefill (ops/attention.rs:153-210):
 * headwise norms and RoPE (offsets 0..n-1) of q in place and of k, K and
 * raw V appended at the sequence's length. */
syn_status_t syn_cuda_qk_norm_rope_kv_append(
    syn_cuda_kvcache_t *cache, size_t layer, size_t seq, size_t n_tokens, float *q,
    const float *k, const float *v, size_t ld, size_t n_heads, const float *q_norm,
    const float *k_norm, float eps, const float *rope_cos, const float *rope_sin,
    void *stream);
/* cached_attention_prefill (ops/attention.rs:153-247): the above, then
 * syn_fused_attention per head (exports.zig:1364-1478) over the prompt. */
syn_status_t syn_cuda_attention_prefill(
    syn_cuda_kvcache_t *cache, size_t layer, size_t seq, size_t n_tokens, float *q,
    const float *k, const float *v, size_t ld, size_t n_heads, const float *q_norm,
    const float *k_norm, float eps, const float *rope_cos, const float *rope_sin,
    float *out, size_t ldo, void *stream);

/* The same two attention operations with a parallel reduction order (split
 * over positions with max/sum rescaling; flash-style tiles for the prefill):
 * identical inputs, outputs and cache effects, results within f32
 * reassociation of the reference order. The runner uses them for
 * block-format models, whose matmuls carry a 1e-3 tolerance; head_dim 32,
 * 64 or 128 (prefill: 64 or 128; other sizes fall back to the exact order). */
syn_status_t syn_cuda_attention_decode_flash(syn_cuda_kvcache_t *cache, size_t layer,
                                             size_t batch, float *q, const float *k,
                                             const float *v, size_t ld, size_t n_heads,
                                             const float *q_norm, const float *k_norm,
                                             float eps, const float *rope_cos,
                                             const float *rope_sin, size_t window,
                                             float *out, size_t ldo, void *stream);
syn_status_t syn_cuda_attention_prefill_flash(
    syn_cuda_kvcache_t *cache, size_t layer, size_t seq, size_t n_tokens, float *q,
    const float *k, const float *v, size_t ld, size_t n_heads, const float *q_norm,
    const float *k_norm, float eps, const float *rope_cos, const float *rope_sin,
    float *out, size_t ldo, void *stream);

/* SwiGLU. variant 0: silu(g)*u of the INT8 model (int8.rs:500-503);
 * variant 1: syn_swiglu / swigluFused (zig/src/ops/silu.zig:85-114). */
syn_status_t syn_cuda_swiglu(const float *gate, const float *up, size_t ld_in,
                             size_t rows, size_t n, int variant, float *out,
                             size_t ldo, void *stream);
/* Greedy argmax per row (generation/sampler.rs:217-224): last maximal index
 * wins ties; NaN compares Equal. out_idx: device int32 [rows]. */
syn_status_t syn_cuda_argmax(const float *logits, size_t rows, size_t n,
                             int32_t *out_idx, void *stream);

/* ------------------------------------------------------------------ */
/* Model runner: QuantizedCausalLM / CausalLM on the GPU               */
/* (quantization/lm/int8.rs:171-709, models/lm/causal_lm.rs:195-280).  */
/* ------------------------------------------------------------------ */
typedef struct syn_cuda_model_s syn_cuda_model_t;

/* config_json: a model config in the reference's format (configs/<name>.json:
 * architecture / attention / norm / ffn / position). max_seq: KV capacity
 * per sequence; max_batch: sequences decoded together. */
syn_status_t syn_cuda_model_create(syn_cuda_ctx_t *ctx, const char *config_json,
                                   size_t max_seq, size_t max_batch,
                                   syn_cuda_model_t **out);
/* f32 tensors by Hugging Face name: model.embed_tokens.weight, model.norm.weight,
 * model.layers.{i}.{input_layernorm,post_attention_layernorm}.weight,
 * model.layers.{i}.self_attn.{q_norm,k_norm}.weight (optional). Host memory. */
syn_status_t syn_cuda_model_set_tensor(syn_cuda_model_t *m, const char *name,
                                       const float *host, size_t numel);
/* Linear weights: model.layers.{i}.self_attn.{q,k,v,o}_proj.weight,
 * model.layers.{i}.mlp.{gate,up,down}_proj.weight, lm_head.weight, in any
 * syn_qformat_t (as syn_cuda_weight_upload). INT8 weights make the layer
 * run the reference's W8A8 QuantizedDecoderLayer; block formats run the f32
 * DecoderLayer semantics. */
syn_status_t syn_cuda_model_set_linear(syn_cuda_model_t *m, const char *name,
                                       syn_qformat_t fmt, const void *host, size_t n,
                                       size_t k, const float *scales_or_null);
/* Uploads and repacks everything (Q/K/V and gate/up fused along N) and
 * allocates the KV cache. Synchronous. */
syn_status_t syn_cuda_model_finalize(syn_cuda_model_t *m);
/* forward_prefill (int8.rs:593-634) of sequence `seq` (must be empty):
 * host tokens [n]; writes the greedy next token and, when logits_host is
 * non-NULL, the last token's logits [vocab]. Synchronous. */
syn_status_t syn_cuda_prefill(syn_cuda_model_t *m, size_t seq,
                              const int32_t *tokens, size_t n,
                              float *logits_host, int32_t *next_token);
/* forward_one (int8.rs:637-709) of sequences [0, batch), one token each
 * (host last_tokens[batch]); writes the greedy tokens and optionally the
 * logits [batch, vocab]. Replays a CUDA graph of the whole step after the
 * first call for a batch size. Synchronous. */
syn_status_t syn_cuda_decode_step(syn_cuda_model_t *m, size_t batch,
                                  const int32_t *last_tokens, int32_t *out_tokens,
                                  float *logits_host);
/* Greedy generation of n_steps further tokens for sequences [0, batch)
 * entirely on the device: each step's input is the previous step's argmax
 * (the last token produced by syn_cuda_prefill / syn_cuda_decode_step /
 * syn_cuda_generate), one captured CUDA graph replayed n_steps times, one
 * synchronisation at the end. out_tokens: host [batch][n_steps]. */
syn_status_t syn_cuda_generate(syn_cuda_model_t *m, size_t batch, size_t n_steps,
                               int32_t *out_tokens);
/* Continuous batching (the reference decodes one sequence at a time,
 * generation/pipeline.rs:197-280). syn_cuda_model_set_kv_paging, before
 * finalize, gives the model a paged KV cache of n_pages pages of `page`
 * positions shared by all its max_batch sequence slots, so memory follows
 * the live contexts rather than max_batch * max_seq.
 * syn_cuda_decode_step_slots runs one decode step for an arbitrary set of
 * started sequences (slots[i], distinct) -- sequences join with
 * syn_cuda_prefill into a free slot and leave with syn_cuda_model_reset,
 * between steps -- and returns each row's greedy token (and optionally its
 * logits [n, vocab]); each sequence advances by one position. */
syn_status_t syn_cuda_model_set_kv_paging(syn_cuda_model_t *m, size_t page, size_t n_pages);
syn_status_t syn_cuda_model_kv_pages_free(const syn_cuda_model_t *m, size_t *n);
syn_status_t syn_cuda_decode_step_slots(syn_cuda_model_t *m, size_t n, const int32_t *slots,
                                        const int32_t *last_tokens, int32_t *out_tokens,
                                        float *logits_host);

/* Speculative decoding support. syn_cuda_decode_span runs n (<= 16)
 * tokens of sequence seq at positions len .. len+n-1 (each attending to the
 * cache up to itself, RoPE at its position) through the first n_layers
 * layers (0 = all), and returns every row's greedy token (and optionally
 * its logits [n, vocab]); the cache length is NOT advanced, so the caller
 * commits or rolls back with syn_cuda_model_truncate. Not for TP models. */
syn_status_t syn_cuda_decode_span(syn_cuda_model_t *m, size_t seq, const int32_t *tokens,
                                  size_t n, size_t n_layers, int32_t *out_tokens,
                                  float *logits_host);
/* Self-speculative greedy generation of n_steps tokens after last_token
 * for sequence seq (generation/pipeline.rs:281-396): k (<= 15) draft tokens
 * from the first draft_layers layers, KV rollback on the device, one
 * full-model span step to verify them. Every draft token is checked (the
 * reference accepts all), so the tokens are the plain greedy ones; drafted /
 * accepted (optional) count the draft tokens made and kept. */
syn_status_t syn_cuda_generate_speculative(syn_cuda_model_t *m, size_t seq, int32_t last_token,
                                           size_t n_steps, size_t k, size_t draft_layers,
                                           int32_t *out_tokens, size_t *drafted,
                                           size_t *accepted);
syn_status_t syn_cuda_model_seq_len(const syn_cuda_model_t *m, size_t seq, size_t *len);
syn_status_t syn_cuda_model_reset(syn_cuda_model_t *m, size_t seq);
syn_status_t syn_cuda_model_truncate(syn_cuda_model_t *m, size_t seq, size_t new_len);
syn_status_t syn_cuda_model_destroy(syn_cuda_model_t *m);

/* ------------------------------------------------------------------ */
/* Tensor parallelism (Megatron column/row split; the reference has no */
/* multi-GPU code). One process per GPU; every rank passes the full    */
/* weights to its model and keeps its own shard: Q/K/V by heads and    */
/* gate/up by FFN rows (column-parallel), O and down by input columns  */
/* (row-parallel, whole quant blocks) with one sum all-reduce after    */
/* each, the LM head by vocabulary rows with an all-gather of the      */
/* logits. Block formats only (the INT8 W8A8 row-parallel split would  */
/* need the activation scale of the whole row).                        */
/* ------------------------------------------------------------------ */
#define SYN_CUDA_TP_ID_BYTES 128
/* Rank 0 creates the group id (ncclGetUniqueId) and shares it. */
syn_status_t syn_cuda_tp_unique_id(uint8_t *id_out);
/* Joins the TP group: every model created on ctx afterwards is sharded. */
syn_status_t syn_cuda_tp_init(syn_cuda_ctx_t *ctx, int rank, int world, const uint8_t *id);
/* In-place sum all-reduce of device floats over the group. */
syn_status_t syn_cuda_tp_allreduce_sum(syn_cuda_ctx_t *ctx, float *buf, size_t count,
                                       void *stream);
/* Host-side shard of a linear weight in its reference storage format:
 * axis 0 = output rows [rank*n/world, ...), axis 1 = input columns
 * [rank*k/world, ...) (block-aligned). out: n_out*k_out weights in the same
 * format; INT8_KN also slices (axis 0) or copies (axis 1) the scales. */
syn_status_t syn_cuda_tp_shard_linear(syn_qformat_t fmt, const void *host, size_t n,
                                      size_t k, const float *scales, int axis, int rank,
                                      int world, void *out, float *out_scales,
                                      size_t *n_out, size_t *k_out);

/* ------------------------------------------------------------------ */
/* Weight files (host side; the parsers need no GPU).                  */
/* ------------------------------------------------------------------ */
typedef struct syn_gguf_s syn_gguf_t;
typedef struct syn_safetensors_s syn_safetensors_t;

/* GGUF v2/v3 (weight_loading/gguf.rs:71-152 and :156-248): the file is
 * memory-mapped; the header, metadata and tensor infos are parsed as the
 * reference parses them (data section at the 32-byte default alignment, or
 * general.alignment when present). Bad magic, an unsupported version, a
 * truncated header or tensor data beyond the file -> SYN_ERR_INVALID_ARG. */
syn_status_t syn_gguf_open(const char *path, syn_gguf_t **out);
syn_status_t syn_gguf_close(syn_gguf_t *g);
syn_status_t syn_gguf_tensor_count(const syn_gguf_t *g, size_t *count);
/* Tensor i: name, GGML type (0 F32, 1 F16, 2 Q4_0, 3 Q4_1, 8 Q8_0, 12 Q4_K,
 * 14 Q6_K; others report nbytes 0), dims (ne0 = the contiguous one first;
 * unused dims are 1), a pointer to its bytes inside the mapping and their
 * size. Pointers live until syn_gguf_close. */
syn_status_t syn_gguf_tensor_info(const syn_gguf_t *g, size_t i, const char **name,
                                  uint32_t *ggml_type, size_t *n_dims, uint64_t *dims4,
                                  const void **data, size_t *nbytes);
/* Scalar metadata (numbers and bools as double; strings). */
syn_status_t syn_gguf_meta_num(const syn_gguf_t *g, const char *key, double *value);
syn_status_t syn_gguf_meta_str(const syn_gguf_t *g, const char *key, const char **value);
/* llama.cpp tensor names onto the runner's (Hugging Face) names:
 * token_embd / output_norm / output and blk.N.{attn_norm, attn_q, attn_k,
 * attn_v, attn_output, attn_q_norm, attn_k_norm, ffn_norm, ffn_gate,
 * ffn_up, ffn_down}.weight. Other names -> SYN_ERR_INVALID_ARG. The
 * reference's weight map has no such table (weight_map.rs:37-135). */
syn_status_t syn_gguf_runner_name(const char *gguf_name, char *out, size_t cap);
/* The model config (the reference's config-JSON schema, as read by
 * syn_cuda_model_create) from <arch>.* metadata and token_embd's shape.
 * *needed = bytes including the terminator; out may be NULL to query. */
syn_status_t syn_gguf_config_json(const syn_gguf_t *g, char *out, size_t cap, size_t *needed);

/* safetensors (weight_loading/safetensors.rs:176-290): F32, F16, BF16, I64,
 * I32 and U8 tensors; "__metadata__" skipped; another dtype ->
 * SYN_ERR_UNSUPPORTED; a bad header or data beyond the file ->
 * SYN_ERR_INVALID_ARG. */
syn_status_t syn_safetensors_open(const char *path, syn_safetensors_t **out);
syn_status_t syn_safetensors_close(syn_safetensors_t *f);
syn_status_t syn_safetensors_tensor_count(const syn_safetensors_t *f, size_t *count);
syn_status_t syn_safetensors_tensor_info(const syn_safetensors_t *f, size_t i, const char **name,
                                         syn_dtype_t *dtype, size_t *n_dims, uint64_t *dims4,
                                         const void **data, size_t *nbytes);
/* Element conversion of the safetensors loader (converter.rs:12-48; f16
 * subnormals come out at half their value, as there). */
syn_status_t syn_convert_to_f32(syn_dtype_t dtype, const void *src, size_t count, float *dst);

/* Load-time INT8 quantisation from f16 / bf16 weights on the device
 * (syn_cuda_quantize_weights_int8 after the loader's conversion:
 * safetensors.rs + converter.rs, then int8.rs:78-152). w: device bits
 * [n,k]; out_kn: int8 [k,n]; scales: f32 [n]. Bit-exact. */
syn_status_t syn_cuda_quantize_weights_int8_half(const uint16_t *w, syn_dtype_t dtype,
                                                 size_t n, size_t k, int8_t *out_kn,
                                                 float *scales, void *stream);
/* The same from HOST f32 / f16 / bf16 [n,k] into host int8 [k,n] + scales,
 * computed on the context's device. Synchronous. */
syn_status_t syn_cuda_quantize_weights_int8_host(syn_cuda_ctx_t *ctx, syn_dtype_t dtype,
                                                 const void *w, size_t n, size_t k,
                                                 int8_t *out_kn, float *scales);

/* syn_cuda_weight_upload with an on-disk cache of the repacked device
 * bytes: the file <cache_dir>/<hash>.synw is named by a 64-bit hash of the
 * source bytes (and scales, format and shape). When it exists and its
 * header matches, the weight is read from it (*hit = 1); otherwise the
 * weight is uploaded and repacked, and the file written (atomically). */
syn_status_t syn_cuda_weight_upload_cached(syn_cuda_ctx_t *ctx, syn_qformat_t fmt,
                                           const void *host, size_t n, size_t k,
                                           const float *scales_or_null, const char *cache_dir,
                                           syn_cuda_weight_t **out, int *hit);

/* Model weights from files, into a model before syn_cuda_model_finalize.
 * GGUF: quantised linears keep their raw blocks (no f32 copy); norms and
 * F32/F16 embeddings become f32; a quantised token_embd is dequantised
 * with the reference's formulas; no output.weight = tied LM head. For
 * general.architecture "llama" the attn_q / attn_k rows are put back from
 * the GGUF converter's pairwise-RoPE order into rotate-half order.
 * safetensors: the reference's --quantize load (int8.rs:78-152): 2-D
 * *_proj.weight and lm_head.weight are quantised to INT8 on the device,
 * other float tensors become f32, a missing lm_head is tied. */
syn_status_t syn_cuda_model_load_gguf(syn_cuda_model_t *m, const syn_gguf_t *g);
syn_status_t syn_cuda_model_load_safetensors(syn_cuda_model_t *m, const syn_safetensors_t *f);
/* Repacked-weight cache for the model's finalize (NULL or "" = none), and
 * how many of its weights finalize read from the cache. */
syn_status_t syn_cuda_model_set_cache_dir(syn_cuda_model_t *m, const char *dir);
syn_status_t syn_cuda_model_cache_hits(const syn_cuda_model_t *m, int *hits);

#ifdef __cplusplus
}
#endif

#endif /* SYNAPSE_CUDA_H */
