// repack.cu -- one-time repack of reference weight bytes into the coalesced
// HBM layout read by the GEMV kernels, and the bit-exact dequant hook.
//
// Source layouts:
//   INT8_KN: int8 [K,N] + f32 [N]  (quantization/primitives/int8_linear.rs:10-18)
//   Q4_0   : 18 B blocks [f16 d][16 nibble bytes]          (gguf.rs:294-330)
//   Q8_0   : 34 B blocks [f16 d][32 int8]                  (gguf.rs:255-288)
//   Q4_K   : 144 B [f16 d][f16 dmin][12 scale B][128 nib]  (gguf.rs:375-431)
//   Q6_K   : 210 B [128 ql][64 qh][16 int8 sc][f16 d]      (gguf.rs:440-487)
// Each row of an [N,K] matrix is K/block consecutive blocks.
//
// Repacked layout ("row-interleaved by 32"): rows are grouped in 32s (the
// last group zero-padded); for group g and 32-element block b the 32 rows'
// data for that block are stored back to back, so one warp (lane = row)
// reads a tile of 32 rows x one block as one contiguous run:
//   tile index t = g * nblk + b, row-in-group l:
//   q    : (t*32 + l) * 16 bytes      (4-bit formats)
//          t*1024 + h*512 + l*16      (8-bit formats: half h of the block)
//   d    : u16 [t*32 + l]             (Q4_0, Q8_0 block scale bits)
//   hdr  : ((g*nsb + j)*32 + l) * 16  (Q4_K super-block j header: d, dmin,
//                                      12 scale bytes, verbatim)
//   qh   : (t*32 + l) * 8             (Q6_K high bits, re-arranged, below)
//   sc   : u16 [t*32 + l]             (Q6_K: the two int8 scales of block b)
//   d6   : u16 [(g*nsb + j)*32 + l]   (Q6_K super-block scale bits)
//   sb   : f32 [G*32]                 (INT8 per-row scales, pad rows 0)
#include "internal.cuh"

namespace syn {
namespace {

__device__ __forceinline__ size_t tile_row(size_t n, size_t b, size_t nblk) {
  return ((n >> 5) * nblk + b) * 32 + (n & 31);
}

// 8-bit formats: a tile of 32 rows x 32 bytes is stored as two half-planes
// (elements 0-15 of the 32 rows, then elements 16-31), so lane l's 16-byte
// reads are consecutive across lanes in both halves.
__device__ __forceinline__ size_t q8_off(size_t t, size_t e) {
  return (t >> 5) * 1024 + (e >> 4) * 512 + (t & 31) * 16 + (e & 15);
}

__global__ void k_repack_int8_kn(const int8_t* __restrict__ src, size_t ldsrc, size_t n,
                                 size_t k, size_t nblk, int8_t* __restrict__ dst) {
  // 32x32 tile transpose: src [k][n] -> dst tiles (zero padded)
  __shared__ int8_t tile[32][33];
  const size_t k0 = (size_t)blockIdx.y * 32, n0 = (size_t)blockIdx.x * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    const size_t kk = k0 + r, nn = n0 + tx;
    tile[r][tx] = (kk < k && nn < n) ? src[kk * ldsrc + nn] : (int8_t)0;
  }
  __syncthreads();
  // row n0 + r, block blockIdx.y, element tx
  for (int r = ty; r < 32; r += 8) {
    const size_t nn = n0 + r;
    dst[q8_off(tile_row(nn, blockIdx.y, nblk), tx)] = tile[tx][r];
  }
}

__global__ void k_repack_q4_0(const uint8_t* __restrict__ src, size_t n, size_t nblk,
                              uint8_t* __restrict__ q, uint16_t* __restrict__ d) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // row * nblk + b
  if (idx >= n * nblk) return;
  const size_t row = idx / nblk, b = idx % nblk;
  const uint8_t* s = src + idx * 18;
  const size_t t = tile_row(row, b, nblk);
  d[t] = (uint16_t)(s[0] | (s[1] << 8));
  for (int i = 0; i < 16; i++) q[t * 16 + i] = s[2 + i];
}

__global__ void k_repack_q8_0(const uint8_t* __restrict__ src, size_t n, size_t nblk,
                              uint8_t* __restrict__ q, uint16_t* __restrict__ d) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * nblk) return;
  const size_t row = idx / nblk, b = idx % nblk;
  const uint8_t* s = src + idx * 34;
  const size_t t = tile_row(row, b, nblk);
  d[t] = (uint16_t)(s[0] | (s[1] << 8));
  for (int i = 0; i < 32; i++) q[q8_off(t, i)] = s[2 + i];
}

__global__ void k_repack_q4_k(const uint8_t* __restrict__ src, size_t n, size_t nsb,
                              uint8_t* __restrict__ q, uint8_t* __restrict__ hdr) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // row * nsb + j
  if (idx >= n * nsb) return;
  const size_t row = idx / nsb, j = idx % nsb, nblk = nsb * 8;
  const uint8_t* s = src + idx * 144;
  const size_t th = tile_row(row, j, nsb);
  for (int i = 0; i < 16; i++) hdr[th * 16 + i] = s[i];
  for (int c = 0; c < 8; c++) {
    const size_t t = tile_row(row, j * 8 + c, nblk);
    for (int i = 0; i < 16; i++) q[t * 16 + i] = s[16 + c * 16 + i];
  }
}

// Q6_K: the 2 high bits of the 32 elements of block c are re-arranged into
// two words (H_A for ql words 0-1, H_B for words 2-3) so that the GEMV
// rebuilds each 6-bit code with one shift and one mask. In byte t of H_A,
// bit pair f holds the high bits of element 8*(f>>1) + 2t + (f&1); H_B
// likewise for elements 16 + 8*(f>>1) + 2t + (f&1). The reference's own order
// (element idx -> qh[idx/4] bits 2*(idx%4), gguf.rs:466-478) is the source.
__global__ void k_repack_q6_k(const uint8_t* __restrict__ src, size_t n, size_t nsb,
                              uint8_t* __restrict__ ql, uint8_t* __restrict__ qh,
                              uint16_t* __restrict__ sc, uint16_t* __restrict__ d) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * nsb) return;
  const size_t row = idx / nsb, j = idx % nsb, nblk = nsb * 8;
  const uint8_t* s = src + idx * 210;
  d[tile_row(row, j, nsb)] = (uint16_t)(s[208] | (s[209] << 8));
  const uint8_t* sqh = s + 128;
  for (int c = 0; c < 8; c++) {
    const size_t t = tile_row(row, j * 8 + c, nblk);
    for (int i = 0; i < 16; i++) ql[t * 16 + i] = s[c * 16 + i];
    sc[t] = (uint16_t)(s[192 + 2 * c] | (s[192 + 2 * c + 1] << 8));
    uint32_t hw[2] = {0u, 0u};
    for (int half = 0; half < 2; half++)
      for (int tt = 0; tt < 4; tt++)
        for (int f = 0; f < 4; f++) {
          const int e = 32 * c + 16 * half + 8 * (f >> 1) + 2 * tt + (f & 1);
          const uint32_t hi = (sqh[e / 4] >> ((e % 4) * 2)) & 3u;
          hw[half] |= hi << (8 * tt + 2 * f);
        }
    uint32_t* o = reinterpret_cast<uint32_t*>(qh + t * 8);
    o[0] = hw[0];
    o[1] = hw[1];
  }
}

__global__ void k_copy_scales(const float* __restrict__ src, size_t n, float* __restrict__ dst) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i];
}

// ---------------------------------------------------------------------------
// Dequant hook: the reference's formulas, one element per thread, with every
// multiply and subtract rounded separately (no contraction).
// ---------------------------------------------------------------------------
__global__ void k_dequant(syn_cuda_weight_s w, float* __restrict__ out) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t n = idx / w.k, kk = idx % w.k;
  if (n >= w.n) return;
  const size_t nblk = w.kp / 32, nsb = w.k / 256, b = kk / 32, e = kk % 32;
  const size_t t = tile_row(n, b, nblk);
  float v = 0.0f;
  switch (w.fmt) {
    case SYN_QFMT_INT8_KN: {  // quantize.zig:90-106
      v = __fmul_rn((float)((const int8_t*)w.q)[q8_off(t, e)], w.sb[n]);
      break;
    }
    case SYN_QFMT_Q4_0: {  // gguf.rs:315-324
      const uint8_t byte = w.q[t * 16 + e / 2];
      const int nib = (e & 1) ? (byte >> 4) : (byte & 15);
      v = __fmul_rn(f16_loader(w.d[t]), (float)(nib - 8));
      break;
    }
    case SYN_QFMT_Q8_0: {  // gguf.rs:276-285
      v = __fmul_rn(f16_loader(w.d[t]), (float)(int8_t)w.q[q8_off(t, e)]);
      break;
    }
    case SYN_QFMT_Q4_K: {  // gguf.rs:395-427
      const size_t j = kk / 256, s = (kk % 256) / 32;
      const uint8_t* h = w.hdr + tile_row(n, j, nsb) * 16;
      const float dd = f16_loader((uint16_t)(h[0] | (h[1] << 8)));
      const float dmin = f16_loader((uint16_t)(h[2] | (h[3] << 8)));
      const uint8_t* sb = h + 4;
      uint32_t scv, mnv;
      if (s < 4) {
        scv = sb[s] & 0x3F;
        mnv = (sb[s + 4] >> 4) | ((sb[s + 8] & 0x0F) << 4);
      } else {
        const size_t u = s - 4;
        scv = (sb[u + 4] & 0x0F) | ((sb[u] >> 6) << 4);
        mnv = (sb[u + 8] >> 4) | (((sb[u] >> 4) & 0x0C) << 4);
      }
      const float scl = __fmul_rn(dd, (float)scv);
      const float m = __fmul_rn(dmin, (float)mnv);
      const uint8_t byte = w.q[t * 16 + e / 2];
      const float nib = (float)((e & 1) ? (byte >> 4) : (byte & 15));
      v = __fsub_rn(__fmul_rn(nib, scl), m);
      break;
    }
    case SYN_QFMT_Q6_K: {  // gguf.rs:462-483
      const size_t j = kk / 256;
      const uint8_t qlb = w.q[t * 16 + e / 2];
      const uint32_t lo = (e & 1) ? (qlb >> 4) : (qlb & 15);
      // invert the re-arrangement of k_repack_q6_k
      const size_t half = e / 16, r = e % 16, f = 2 * (r / 8) + (r & 1), tt = (r % 8) / 2;
      const uint32_t* hq = reinterpret_cast<const uint32_t*>(w.qh + t * 8);
      const uint32_t hi = (hq[half] >> (8 * tt + 2 * f)) & 3u;
      const float dd = f16_loader(w.d[tile_row(n, j, nsb)]);
      const uint16_t scp = reinterpret_cast<const uint16_t*>(w.sc)[t];
      const int8_t scv = (int8_t)((e < 16) ? (scp & 0xFF) : (scp >> 8));
      const float scale = __fmul_rn((float)scv, dd);
      const float qv = (float)((int)(lo | (hi << 4)) - 32);
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
  const size_t nblk = w->kp / 32, nsb = w->k / 256;
  // padded rows and K tails must read as zero
  SYN_CUDA_TRY(cudaMemsetAsync(w->buf, 0, w->bytes, st));
  switch (w->fmt) {
    case SYN_QFMT_INT8_KN: {
      dim3 grid((unsigned)((w->n + 31) / 32), (unsigned)nblk);
      k_repack_int8_kn<<<grid, dim3(32, 8), 0, st>>>((const int8_t*)src, ld_src ? ld_src : w->n,
                                                     w->n, w->k, nblk, (int8_t*)w->q);
      if (d_scales)
        k_copy_scales<<<(unsigned)((w->n + T - 1) / T), T, 0, st>>>(d_scales, w->n, w->sb);
      break;
    }
    case SYN_QFMT_Q4_0: {
      const size_t cnt = w->n * nblk;
      k_repack_q4_0<<<(unsigned)((cnt + T - 1) / T), T, 0, st>>>(src, w->n, nblk, w->q, w->d);
      break;
    }
    case SYN_QFMT_Q8_0: {
      const size_t cnt = w->n * nblk;
      k_repack_q8_0<<<(unsigned)((cnt + T - 1) / T), T, 0, st>>>(src, w->n, nblk, w->q, w->d);
      break;
    }
    case SYN_QFMT_Q4_K: {
      const size_t cnt = w->n * nsb;
      k_repack_q4_k<<<(unsigned)((cnt + T - 1) / T), T, 0, st>>>(src, w->n, nsb, w->q, w->hdr);
      break;
    }
    case SYN_QFMT_Q6_K: {
      const size_t cnt = w->n * nsb;
      k_repack_q6_k<<<(unsigned)((cnt + T - 1) / T), T, 0, st>>>(
          src, w->n, nsb, w->q, w->qh, reinterpret_cast<uint16_t*>(w->sc), w->d);
      break;
    }
    default:
      return SYN_ERR_INVALID_ARG;
  }
  SYN_LAUNCH_CHECK("repack");
  return SYN_OK;
}

syn_status_t dequant_weight(const syn_cuda_weight_s* w, float* d_out, cudaStream_t st) {
  const size_t total = w->n * w->k;
  const int T = 256;
  k_dequant<<<(unsigned)((total + T - 1) / T), T, 0, st>>>(*w, d_out);
  SYN_LAUNCH_CHECK("dequant");
  return SYN_OK;
}

}  // namespace syn
