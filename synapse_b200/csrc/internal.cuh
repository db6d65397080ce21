// internal.cuh -- library-private types shared by the .cu files.
#pragma once

#include "common.cuh"

// One context per device and per issuing stream: the scratch buffers are
// reused by every call made through the context, in stream order.
struct syn_cuda_ctx_s {
  int device;
  int sms;
  cudaStream_t upload_stream;
  float* part;       // per-(row, K-split) partial sums of split GEMVs
  size_t part_bytes;
  int* cnt;          // per-row-group arrival counters; zero between launches
  size_t cnt_bytes;
  uint8_t* abuf;     // activations prepared for the tensor-core GEMM
  size_t abuf_bytes;
  int* err;          // device-side error word (e.g. SYN_ERR_TIMEOUT)
  void* nccl;        // tensor-parallel communicator (ncclComm_t) or nullptr
  int tp_rank, tp_world;
  void* tp_peer;     // peer-memory all-reduce state (tp.cu) or nullptr
};

// Repacked weight in HBM. One allocation; the views below point into it.
// Rows are row-interleaved by 32 (see repack.cu for the exact layout):
//   INT8  : q tiles of 32 rows x 32 int8 (kp = K rounded up to 32), sb f32
//   Q4_0  : q tiles of 32 rows x 16 nibble bytes, d f16 bits per row-block
//   Q8_0  : q tiles of 32 rows x 32 int8, d f16 bits per row-block
//   Q4_K  : q tiles of 32 rows x 16 nibble bytes, hdr 16 B per row-superblock
//   Q6_K  : q low-nibble tiles, qh 8 B per row-block (re-arranged high bits),
//           sc 2 int8 scales per row-block, d f16 bits per row-superblock
struct syn_cuda_weight_s {
  int fmt;
  int device;
  size_t n, k, kp;
  void* buf;
  size_t bytes;
  size_t algo_bytes;  // bytes of the source format (roofline accounting)
  uint8_t* q;
  uint16_t* d;
  float* sb;
  uint8_t* hdr;
  uint8_t* qh;
  int8_t* sc;
};

// KV cache in HBM (zig/src/ops/kvcache.zig:13-170, kv_cache/cache.rs:26-340):
// per layer and sequence, K and V rows of n_kv*hd f32 for max_seq positions.
// One length per sequence, shared by all layers (LayerCaches advance, reset
// and truncate together). The device copy of the lengths is what kernels
// read (so that a captured graph replays at the current position); the host
// copy mirrors it for the CacheFull check.
struct syn_cuda_kvcache_s {
  int device;
  size_t max_seq, n_kv, hd, layers, batch;
  float* k;     // [layers][batch][max_seq][n_kv*hd]
  float* v;
  int* d_len;   // [batch]
  size_t* len;  // [batch], host mirror
  float* part;  // split-attention counters + partials (grown on demand)
  size_t part_bytes;
  int part_heads;  // the head count the counters are laid out for
  // Paged layout (page > 0): each layer's K and V are pools of n_pages pages
  // of `page` positions, and position p of sequence s lives in page
  // ptab[s * maxp + p / page]. Pages are taken from a free list as a
  // sequence grows and returned when it is truncated or reset.
  size_t page, n_pages, maxp;
  int* ptab_h;       // pinned host table [batch][maxp], -1 = none
  int* d_ptab;       // device copy
  int* free_pages;   // stack of free page ids (host)
  size_t n_free;
};

namespace syn {

// Makes `dev` current for the scope and restores the previous device.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      ok = false;
      return;
    }
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};


// Scratch of a GEMV over m activation rows: partial sums (0 when K is not
// split across CTAs; planned with the weight's own format, and for m = 1
// with k > 0 also covering the fused-RMSNorm launch) and per-row-group
// arrival counters (zero before the first launch; the kernel leaves them
// zero). Every launch takes the capacity of its partial-sum buffer and
// returns SYN_ERR_INTERNAL, launching nothing, if its plan needs more.
size_t gemv_partial_bytes(int fmt, size_t m, size_t n, size_t kp, size_t k = 0);
// fmt value of the raw-layout Q4_0 GEMV (syn_cuda_q4_0_gemv) for the above
constexpr int GEMV_FMT_Q4_0_RAW = 100;
size_t gemv_counter_bytes(size_t m, size_t n);

// Launches the fused GEMV for rows [0, m) of x (programmatic dependent
// launch). x: f32 [m, k] (row stride ldx; 16-byte aligned rows) or, when
// xq != nullptr (INT8 only), int8 [m, k] (row stride ldx) with per-row
// scales sx. y: f32 [m, n] (row stride ldy). chunked=1 selects the
// reference's M>16 INT8 epilogue (per-512-K chunks). err: device error word
// or nullptr.
syn_status_t launch_qgemv(const syn_cuda_weight_s* w, const float* x, size_t ldx,
                          const int8_t* xq, const float* sx, size_t m, float* y, size_t ldy,
                          int chunked, float* part, size_t part_cap, int* cnt, int* err,
                          cudaStream_t st);

// The GEMV for one activation row x = RMSNorm(res (+ delta)) * w, fused into
// its prologue (same arithmetic as launch_add_rmsnorm; fast = parallel sum of
// squares). The grid's first CTA stores res + delta into res_out, which must
// not alias res. Scratch as launch_qgemv with m = 1.
struct GemvNorm {
  const float* res;
  const float* delta;  // or nullptr
  const float* w;
  float eps;
  float* res_out;      // or nullptr
  int fast;
  // optional SwiGLU epilogue: the weight's rows are gate/up interleaved by
  // 16 (2 * sw_n rows); sw_out[0, sw_n) receives swiglu(gate, up) instead
  // of y (variant as launch_swiglu)
  float* sw_out;
  int sw_n;
  int sw_variant;
};
syn_status_t launch_qgemv_norm(const syn_cuda_weight_s* w, const GemvNorm& nm, float* y,
                               float* part, size_t part_cap, int* cnt, int* err,
                               cudaStream_t st);
// Grows the context's GEMV scratch for m rows of w (refused during capture).
syn_status_t ensure_scratch(syn_cuda_ctx_s* ctx, const syn_cuda_weight_s* w, size_t m,
                            cudaStream_t st);

// Tensor-core GEMM (gemm.cu) for m >= gemm_min_rows(fmt, n) activation rows
// of an n-row weight (fewer rows run the GEMV). abuf: scratch of
// gemm_a_bytes(fmt, m, kp) bytes for the prepared activations.
size_t gemm_min_rows(int fmt, size_t n);
size_t gemm_a_bytes(int fmt, size_t m, size_t kp);
syn_status_t launch_qgemm(const syn_cuda_weight_s* w, const float* x, size_t ldx,
                          const int8_t* xq, const float* sx, size_t m, float* y, size_t ldy,
                          int chunked, uint8_t* abuf, int* err, cudaStream_t st);

// Raw-layout Q4_0 GEMV over the reference's 18-byte blocks (M = 1).
syn_status_t launch_q4_0_raw(size_t n, size_t k, const float* a, const uint8_t* b, float* c,
                             float* part, size_t part_cap, int* cnt, int* err,
                             cudaStream_t st);

// Per-row INT8 quantisation (quantize.zig:12-47).
syn_status_t launch_quantize_rows(const float* x, size_t rows, size_t cols, int8_t* out,
                                  float* scales, cudaStream_t st);

// Load-time per-output-row INT8 weight quantisation into the [K,N] layout.
syn_status_t launch_quantize_weights(const float* w, size_t n, size_t k, int8_t* out_kn,
                                     float* scales, cudaStream_t st);

// The same from f16 / bf16 bit patterns (dtype SYN_DTYPE_F16 / _BF16),
// converted to f32 as weight_loading/converter.rs does.
syn_status_t launch_quantize_weights_half(const uint16_t* w, int dtype, size_t n, size_t k,
                                          int8_t* out_kn, float* scales, cudaStream_t st);

// The context a model was created on (runner.cu).
syn_cuda_ctx_s* model_context(const syn_cuda_model_s* m);

// Byte layout of a repacked weight (capi.cu): sets the array views of `w`
// inside `base` (nullptr: sizes only) and returns the allocation's bytes.
size_t weight_layout(syn_cuda_weight_s* w, uint8_t* base);
size_t weight_src_row_bytes(int fmt, size_t k);

// Repack kernels (repack.cu). ld_src: row stride of an INT8_KN source
// (0 = n); ignored by block formats. w->buf / w->bytes are zero-filled first.
syn_status_t repack_weight(syn_cuda_weight_s* w, const uint8_t* d_src, size_t ld_src,
                           const float* d_scales, cudaStream_t st);
syn_status_t dequant_weight(const syn_cuda_weight_s* w, float* d_out, cudaStream_t st);

// ---- decoder-layer kernels (lm.cu) ----
// Residual add + RMSNorm: row r of out = rmsnorm(src_r (+ delta_r)), where
// src_r is x_r or, when ids != nullptr, the embedding row table[ids[r]]
// (zeros for ids outside the vocabulary). x_out (optional) receives the
// normalised input (the updated residual stream); it may alias x. fast=1
// sums the squares in a parallel order (models with a tolerance).
syn_status_t launch_add_rmsnorm(const float* x, size_t ldx, const float* delta, size_t ldd,
                                const int32_t* ids, const float* table, size_t vocab,
                                float* x_out, size_t ldxo, const float* w, size_t rows, size_t h,
                                float eps, float* out, size_t ldo, cudaStream_t st, int fast = 0);

// Attention over the KV cache. q/k/v rows have stride ld (row b = sequence b
// for decode, token t for prefill); out rows have stride ldo.
struct AttnArgs {
  float* q;
  const float* k;
  const float* v;
  size_t ld;
  size_t n_heads;
  const float* qn;  // headwise norm weights or nullptr
  const float* kn;
  float eps;
  const float* cos_t;
  const float* sin_t;
  size_t window;    // 0 = none
  syn_cuda_kvcache_t* cache;
  size_t layer;
  float* out;
  size_t ldo;
  int flash;        // 1: parallel reduction order (block-format models)
  const int* slots; // decode: device map row -> sequence (nullptr: row b = sequence b)
};
// Paged cache: maps pages for positions [0, new_len) of sequence seq (host
// table, copied to the device on `st`); SYN_ERR_OUT_OF_MEMORY when the pool
// is exhausted. No-op for a contiguous cache.
syn_status_t kv_reserve(syn_cuda_kvcache_t* c, size_t seq, size_t new_len, cudaStream_t st);
// Frees the pages of seq beyond position keep_len (drains `st` first).
syn_status_t kv_release(syn_cuda_kvcache_t* c, size_t seq, size_t keep_len, cudaStream_t st);
// Decode step of sequences [0, batch): norm/RoPE/append of the new token,
// attention over positions [0, len] (the cache lengths are not advanced).
syn_status_t launch_attn_decode_args(const AttnArgs& a, size_t batch, int* err, cudaStream_t st);
// Prefill of ntok prompt tokens of sequence `seq` (appended from its current
// length; RoPE at offsets 0..ntok-1 as the reference's prefill).
syn_status_t launch_attn_prefill_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                      cudaStream_t st);
// ntok new positions of sequence `seq` from its current length, each
// attending to the cache up to itself (speculative verification; RoPE at
// the cache slots). The cache length is not advanced.
syn_status_t launch_attn_span_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                   cudaStream_t st);
// The two halves of the prefill: norm/RoPE/append, then attention.
syn_status_t launch_norm_rope_append_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                          cudaStream_t st);
syn_status_t launch_prefill_attention_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                           cudaStream_t st);
syn_status_t launch_swiglu(const float* gate, const float* up, size_t ld_in, size_t rows, size_t n,
                           int variant, float* out, size_t ldo, cudaStream_t st, int il16 = 0);
// il16 = 1: gate and up interleaved by 16 columns in one buffer (gate at
// gu[r*ld_in + (i/16)*32 + i%16], up 16 further): pass gate = gu, up = gu + 16.
// Greedy argmax per row; when len_adv != nullptr, len_adv[row] += adv after
// and (hist != nullptr) the token is recorded at hist[row*hist_ld + new len].
// scratch: argmax_scratch_bytes(rows, n) bytes, zero before the first launch
// (each launch leaves it reusable).
size_t argmax_scratch_bytes(size_t rows, size_t n);
syn_status_t launch_argmax(const float* x, size_t ldx, size_t rows, size_t n, int32_t* out,
                           int* len_adv, int adv, int max_len, int32_t* hist, int hist_ld,
                           void* scratch, cudaStream_t st);
// Tensor-parallel greedy token: launch_argmax_slice writes each row's argmax
// state over this rank's vocabulary slice (indices offset by idx_off) as 16
// bytes into pairs[row]; after an all-gather of the pairs into [world][rows]
// (rank = vocabulary order), launch_argmax_pairs combines them in rank order
// into the token of one argmax over the whole row (ties: the later index;
// the last NaN wins), with launch_argmax's length advance and history.
syn_status_t launch_argmax_slice(const float* x, size_t ldx, size_t rows, size_t n, int idx_off,
                                 void* pairs, void* scratch, cudaStream_t st);
syn_status_t launch_argmax_pairs(const void* pairs, int world, size_t rows, int32_t* out,
                                 int* len_adv, int adv, int max_len, int32_t* hist, int hist_ld,
                                 cudaStream_t st);
// Device lengths of the sequences slots[0, n) (device array) advanced by one.
syn_status_t launch_kv_advance_slots(syn_cuda_kvcache_t* c, const int* slots, size_t n,
                                     cudaStream_t st);
// Device length of sequence seq: set to value (add=0) or advanced by it.
syn_status_t launch_kv_set(syn_cuda_kvcache_t* c, size_t seq, int value, int add, cudaStream_t st);

// ---- tensor parallelism (tp.cu) ----
// Releases the context's communicator (context destroy).
void tp_release(syn_cuda_ctx_s* ctx);
// Sum all-reduce of count floats in place over the context's TP group.
syn_status_t tp_allreduce_sum(syn_cuda_ctx_s* ctx, float* buf, size_t count, cudaStream_t st);
// All-gather: every rank contributes count floats; recv holds world*count
// in rank order.
syn_status_t tp_allgather(syn_cuda_ctx_s* ctx, const float* send, float* recv, size_t count,
                          cudaStream_t st);

}  // namespace syn
