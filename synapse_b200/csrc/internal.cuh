// internal.cuh -- library-private types shared by the .cu files.
#pragma once

#include "common.cuh"

struct syn_cuda_ctx_s {
  int device;
  int sms;
  cudaStream_t upload_stream;
};

// Repacked weight in HBM. One allocation; the views below point into it.
// Per output row n the arrays hold, in K order (see repack.cu):
//   INT8  : q[N][kp] int8 (kp = K rounded up to 32, zero padded), sb[N] f32
//   Q4_0  : q[N][K/2] nibbles (as in the GGUF block), d[N][K/32] f16 bits
//   Q8_0  : q[N][K] int8, d[N][K/32] f16 bits
//   Q4_K  : q[N][K/2] nibbles, hdr[N][K/256][16] (d, dmin, 12 scale bytes)
//   Q6_K  : q[N][K/2] low nibbles, qh[N][K/32][8] high bits (re-arranged),
//           sc[N][K/16] int8 scales, d[N][K/256] f16 bits
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

namespace syn {

// Launches the fused activation-prologue GEMV for rows [0, m) of x.
// x: f32 [m, k] (row stride ldx) or, when xq != nullptr (INT8 only), int8
// [m, k] (row stride ldx) with per-row scales sx. y: f32 [m, n] (row stride ldy).
// chunked=1 selects the reference's M>16 INT8 epilogue (per-512-K chunks).
syn_status_t launch_qgemv(const syn_cuda_weight_s* w, const float* x, size_t ldx,
                          const int8_t* xq, const float* sx, size_t m, float* y,
                          size_t ldy, int chunked, cudaStream_t st);

// Raw-layout Q4_0 GEMV over the reference's 18-byte blocks (M = 1).
syn_status_t launch_q4_0_raw(size_t n, size_t k, const float* a,
                             const uint8_t* b, float* c, cudaStream_t st);

// Per-row INT8 quantisation (quantize.zig:12-47).
syn_status_t launch_quantize_rows(const float* x, size_t rows, size_t cols,
                                  int8_t* out, float* scales, cudaStream_t st);

// Load-time per-output-row INT8 weight quantisation into the [K,N] layout.
syn_status_t launch_quantize_weights(const float* w, size_t n, size_t k, int8_t* out_kn,
                                     float* scales, cudaStream_t st);

// Repack kernels (repack.cu).
// ld_src: row stride of an INT8_KN source (0 = n); ignored by block formats.
syn_status_t repack_weight(syn_cuda_weight_s* w, const uint8_t* d_src, size_t ld_src,
                           const float* d_scales, cudaStream_t st);
syn_status_t dequant_weight(const syn_cuda_weight_s* w, float* d_out,
                            cudaStream_t st);

}  // namespace syn
