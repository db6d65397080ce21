// repack.cu -- one-time repack of reference weight bytes into the coalesced
// HBM layout read by the GEMV/GEMM kernels, and the bit-exact dequant hook.
//
// Source layouts:
//   INT8_KN: int8 [K,N] + f32 [N]  (quantization/primitives/int8_linear.rs:10-18)
//   Q4_0   : 18 B blocks [f16 d][16 nibble bytes]          (gguf.rs:294-330)
//   Q8_0   : 34 B blocks [f16 d][32 int8]                  (gguf.rs:255-288)
//   Q4_K   : 144 B [f16 d][f16 dmin][12 scale B][128 nib]  (gguf.rs:375-431)
//   Q6_K   : 210 B [128 ql][64 qh][16 int8 sc][f16 d]      (gguf.rs:440-487)
// Each row of an [N,K] matrix is K/block consecutive blocks.
#include "internal.cuh"

namespace syn {
namespace {

__global__ void k_repack_int8_kn(const int8_t* __restrict__ src, size_t ldsrc, size_t n,
                                 size_t k, size_t kp, int8_t* __restrict__ dst) {
  // 32x32 tile transpose: src [k][n] -> dst [n][kp] (zero padded k..kp)
  __shared__ int8_t tile[32][33];
  size_t k0 = (size_t)blockIdx.y * 32, n0 = (size_t)blockIdx.x * 32;
  int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    size_t kk = k0 + r, nn = n0 + tx;
    tile[r][tx] = (kk < k && nn < n) ? src[kk * ldsrc + nn] : (int8_t)0;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    size_t nn = n0 + r, kk = k0 + tx;
    if (nn < n && kk < kp) dst[nn * kp + kk] = tile[tx][r];
  }
}

__global__ void k_repack_q4_0(const uint8_t* __restrict__ src, size_t nblocks,
                              uint8_t* __restrict__ q, uint16_t* __restrict__ d) {
  size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const uint8_t* s = src + b * 18;
  d[b] = (uint16_t)(s[0] | (s[1] << 8));
  for (int i = 0; i < 16; i++) q[b * 16 + i] = s[2 + i];
}

__global__ void k_repack_q8_0(const uint8_t* __restrict__ src, size_t nblocks,
                              uint8_t* __restrict__ q, uint16_t* __restrict__ d) {
  size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const uint8_t* s = src + b * 34;
  d[b] = (uint16_t)(s[0] | (s[1] << 8));
  for (int i = 0; i < 32; i++) q[b * 32 + i] = s[2 + i];
}

__global__ void k_repack_q4_k(const uint8_t* __restrict__ src, size_t nsb,
                              uint8_t* __restrict__ q, uint8_t* __restrict__ hdr) {
  size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nsb) return;
  const uint8_t* s = src + b * 144;
  for (int i = 0; i < 16; i++) hdr[b * 16 + i] = s[i];
  for (int i = 0; i < 128; i++) q[b * 128 + i] = s[16 + i];
}

// Q6_K: the 2 high bits of the 32 elements of chunk c are re-arranged into two
// words (H_A for ql words 0-1, H_B for words 2-3) so that the GEMV rebuilds
// each 6-bit code with one shift and one mask. In byte t of H_A, bit pair f
// holds the high bits of element 8*(f>>1) + 2t + (f&1); H_B likewise for
// elements 16 + 8*(f>>1) + 2t + (f&1). The reference's own order
// (element idx -> qh[idx/4] bits 2*(idx%4), gguf.rs:466-478) is the source.
__global__ void k_repack_q6_k(const uint8_t* __restrict__ src, size_t nsb,
                              uint8_t* __restrict__ ql, uint8_t* __restrict__ qh,
                              int8_t* __restrict__ sc, uint16_t* __restrict__ d) {
  size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nsb) return;
  const uint8_t* s = src + b * 210;
  for (int i = 0; i < 128; i++) ql[b * 128 + i] = s[i];
  for (int i = 0; i < 16; i++) sc[b * 16 + i] = (int8_t)s[192 + i];
  d[b] = (uint16_t)(s[208] | (s[209] << 8));
  const uint8_t* sqh = s + 128;
  for (int c = 0; c < 8; c++) {
    uint32_t hw[2] = {0u, 0u};
    for (int half = 0; half < 2; half++)
      for (int t = 0; t < 4; t++)
        for (int f = 0; f < 4; f++) {
          int e = 32 * c + 16 * half + 8 * (f >> 1) + 2 * t + (f & 1);  // idx in superblock
          uint32_t hi = (sqh[e / 4] >> ((e % 4) * 2)) & 3u;
          hw[half] |= hi << (8 * t + 2 * f);
        }
    uint32_t* o = reinterpret_cast<uint32_t*>(qh + (b * 8 + c) * 8);
    o[0] = hw[0];
    o[1] = hw[1];
  }
}

// ---------------------------------------------------------------------------
// Dequant hook: the reference's formulas, one element per thread, with every
// multiply and subtract rounded separately (no contraction).
// ---------------------------------------------------------------------------
__global__ void k_dequant(syn_cuda_weight_s w, float* __restrict__ out) {
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  size_t n = idx / w.k, kk = idx % w.k;
  if (n >= w.n) return;
  float v = 0.0f;
  switch (w.fmt) {
    case SYN_QFMT_INT8_KN: {  // quantize.zig:90-106
      v = __fmul_rn((float)((const int8_t*)w.q)[n * w.kp + kk], w.sb[n]);
      break;
    }
    case SYN_QFMT_Q4_0: {  // gguf.rs:315-324
      size_t b = kk / 32, e = kk % 32;
      uint8_t byte = w.q[n * (w.k / 2) + b * 16 + e / 2];
      int nib = (e & 1) ? (byte >> 4) : (byte & 15);
      float delta = f16_loader(w.d[n * (w.k / 32) + b]);
      v = __fmul_rn(delta, (float)(nib - 8));
      break;
    }
    case SYN_QFMT_Q8_0: {  // gguf.rs:276-285
      size_t b = kk / 32;
      float scale = f16_loader(w.d[n * (w.k / 32) + b]);
      v = __fmul_rn(scale, (float)(int8_t)w.q[n * w.k + kk]);
      break;
    }
    case SYN_QFMT_Q4_K: {  // gguf.rs:395-427
      size_t j = kk / 256, e = kk % 256, s = e / 32, i = e % 32;
      const uint8_t* h = w.hdr + (n * (w.k / 256) + j) * 16;
      float dd = f16_loader((uint16_t)(h[0] | (h[1] << 8)));
      float dmin = f16_loader((uint16_t)(h[2] | (h[3] << 8)));
      const uint8_t* sb = h + 4;
      uint32_t scv, mnv;
      if (s < 4) {
        scv = sb[s] & 0x3F;
        mnv = (sb[s + 4] >> 4) | ((sb[s + 8] & 0x0F) << 4);
      } else {
        size_t t = s - 4;
        scv = (sb[t + 4] & 0x0F) | ((sb[t] >> 6) << 4);
        mnv = (sb[t + 8] >> 4) | (((sb[t] >> 4) & 0x0C) << 4);
      }
      float scl = __fmul_rn(dd, (float)scv);
      float m = __fmul_rn(dmin, (float)mnv);
      uint8_t byte = w.q[n * (w.k / 2) + j * 128 + s * 16 + i / 2];
      float nib = (float)((i & 1) ? (byte >> 4) : (byte & 15));
      v = __fsub_rn(__fmul_rn(nib, scl), m);
      break;
    }
    case SYN_QFMT_Q6_K: {  // gguf.rs:462-483
      size_t j = kk / 256, e = kk % 256;
      uint8_t qlb = w.q[n * (w.k / 2) + j * 128 + e / 2];
      uint32_t lo = (e & 1) ? (qlb >> 4) : (qlb & 15);
      // invert the re-arrangement of k_repack_q6_k
      size_t c = e / 32, el = e % 32;
      size_t half = el / 16, r = el % 16, f = 2 * (r / 8) + (r & 1), t = (r % 8) / 2;
      const uint32_t* hq = reinterpret_cast<const uint32_t*>(w.qh + ((n * (w.k / 256) + j) * 8 + c) * 8);
      uint32_t hi = (hq[half] >> (8 * t + 2 * f)) & 3u;
      float dd = f16_loader(w.d[n * (w.k / 256) + j]);
      float scale = __fmul_rn((float)w.sc[n * (w.k / 16) + j * 16 + e / 16], dd);
      float qv = (float)((int)(lo | (hi << 4)) - 32);
      v = __fmul_rn(qv, scale);
      break;
    }
  }
  out[n * w.k + kk] = v;
}

}  // namespace

syn_status_t repack_weight(syn_cuda_weight_s* w, const uint8_t* src, size_t ld_src,
                           const float* d_scales, cudaStream_t st) {
  const int T = 256;
  switch (w->fmt) {
    case SYN_QFMT_INT8_KN: {
      dim3 grid((unsigned)((w->n + 31) / 32), (unsigned)((w->kp + 31) / 32));
      k_repack_int8_kn<<<grid, dim3(32, 8), 0, st>>>((const int8_t*)src, ld_src ? ld_src : w->n,
                                                     w->n, w->k, w->kp, (int8_t*)w->q);
      if (d_scales && d_scales != w->sb)
        SYN_CUDA_TRY(cudaMemcpyAsync(w->sb, d_scales, w->n * sizeof(float),
                                     cudaMemcpyDeviceToDevice, st));
      break;
    }
    case SYN_QFMT_Q4_0: {
      size_t nb = w->n * (w->k / 32);
      k_repack_q4_0<<<(unsigned)((nb + T - 1) / T), T, 0, st>>>(src, nb, w->q, w->d);
      break;
    }
    case SYN_QFMT_Q8_0: {
      size_t nb = w->n * (w->k / 32);
      k_repack_q8_0<<<(unsigned)((nb + T - 1) / T), T, 0, st>>>(src, nb, w->q, w->d);
      break;
    }
    case SYN_QFMT_Q4_K: {
      size_t nb = w->n * (w->k / 256);
      k_repack_q4_k<<<(unsigned)((nb + T - 1) / T), T, 0, st>>>(src, nb, w->q, w->hdr);
      break;
    }
    case SYN_QFMT_Q6_K: {
      size_t nb = w->n * (w->k / 256);
      k_repack_q6_k<<<(unsigned)((nb + T - 1) / T), T, 0, st>>>(src, nb, w->q, w->qh, w->sc,
                                                                 w->d);
      break;
    }
    default:
      return SYN_ERR_INVALID_ARG;
  }
  SYN_LAUNCH_CHECK("repack");
  return SYN_OK;
}

syn_status_t dequant_weight(const syn_cuda_weight_s* w, float* d_out, cudaStream_t st) {
  size_t total = w->n * w->k;
  const int T = 256;
  k_dequant<<<(unsigned)((total + T - 1) / T), T, 0, st>>>(*w, d_out);
  SYN_LAUNCH_CHECK("dequant");
  return SYN_OK;
}

}  // namespace syn
