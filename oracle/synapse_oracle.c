/*
 * synapse_oracle.c -- CPU restatement of eren23/synapse's quantized-matmul
 * arithmetic (TEST INFRASTRUCTURE ONLY; see synapse_oracle.h).
 *
 * Compiled with -O2 -ffp-contract=off so that every a*b+c that the reference
 * writes as two operations stays two roundings; fmaf() is used exactly where
 * the Zig source uses @mulAdd. Zig's default float mode is strict, so Zig
 * expressions are evaluated left to right with one rounding per operation.
 */
#include "synapse_oracle.h"

#include <math.h>
#include <string.h>

static float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* zig/src/ops/qmatmul.zig:346-371 */
float orc_f16_zig(uint16_t bits) {
  uint32_t sign = ((uint32_t)(bits >> 15)) << 31;
  uint32_t exp5 = (bits >> 10) & 0x1F;
  uint32_t mant = bits & 0x3FF;
  if (exp5 == 0) {
    if (mant == 0) return bits_to_f32(sign);
    uint32_t m = mant, e = 0;
    while ((m & 0x400) == 0) {
      m <<= 1;
      e += 1;
    }
    m &= 0x3FF;
    uint32_t exp32 = (127 - 15 + 1 - e) << 23;
    return bits_to_f32(sign | exp32 | (m << 13));
  } else if (exp5 == 31) {
    return bits_to_f32(sign | 0x7F800000u | (mant << 13));
  }
  return bits_to_f32(sign | ((exp5 + 127 - 15) << 23) | (mant << 13));
}

/* weight_loading/converter.rs:12-40. The subnormal branch starts its counter
 * at e=1 (the Zig version starts at 0), which halves every subnormal. */
float orc_f16_rust(uint16_t h) {
  uint32_t sign = (h >> 15) & 1;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ff;
  if (exp == 0) {
    if (mant == 0) return bits_to_f32(sign << 31);
    uint32_t e = 1, m = mant;
    while ((m & 0x400) == 0) {
      m <<= 1;
      e += 1;
    }
    m = (m & 0x3ff) << 13;
    uint32_t ee = 127 - 15 + 1 - e;
    return bits_to_f32((sign << 31) | (ee << 23) | m);
  } else if (exp == 31) {
    return bits_to_f32((sign << 31) | (0xffu << 23) | (mant << 13));
  }
  return bits_to_f32((sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13));
}

/* zig/src/ops/quantize.zig:12-47; argument checks from
 * zig/src/ffi/exports.zig:1275-1289. */
int orc_quantize_per_channel_int8(const float *data, size_t channels,
                                  size_t channel_size, int8_t *out,
                                  float *scales) {
  if (!data || !out || !scales) return ORC_ERR_NULL_PTR;
  if (channels == 0 || channel_size == 0) return ORC_ERR_INVALID_ARG;
  for (size_t c = 0; c < channels; c++) {
    const float *row = data + c * channel_size;
    int8_t *orow = out + c * channel_size;
    float max_abs = 0.0f;
    for (size_t j = 0; j < channel_size; j++) {
      float av = fabsf(row[j]);
      if (av > max_abs) max_abs = av;
    }
    if (max_abs == 0.0f) {
      scales[c] = 1.0f;
      memset(orow, 0, channel_size);
      continue;
    }
    scales[c] = max_abs / 127.0f;
    float inv = 127.0f / max_abs;
    for (size_t j = 0; j < channel_size; j++) {
      float r = roundf(row[j] * inv); /* @round: half away from zero */
      if (r > 127.0f) r = 127.0f;
      if (r < -127.0f) r = -127.0f;
      orow[j] = (int8_t)r;
    }
  }
  return ORC_OK;
}

/* calibration.rs:11-24 (fold with f32::max from 0.0) and
 * int8_linear.rs:43-70 (inv_s = 1/s, round half away, clamp [-128,127],
 * transpose to [in, out]). */
void orc_quantize_weights_int8(const float *w, size_t n, size_t k,
                               int8_t *out_kn, float *scales) {
  for (size_t ch = 0; ch < n; ch++) {
    const float *row = w + ch * k;
    float max_abs = 0.0f;
    for (size_t j = 0; j < k; j++) max_abs = fmaxf(max_abs, fabsf(row[j]));
    scales[ch] = (max_abs == 0.0f) ? 1.0f : max_abs / 127.0f;
  }
  memset(out_kn, 0, n * k);
  for (size_t ch = 0; ch < n; ch++) {
    float s = scales[ch];
    if (s == 0.0f) continue;
    float inv_s = 1.0f / s;
    for (size_t j = 0; j < k; j++) {
      float r = roundf(w[ch * k + j] * inv_s);
      if (r < -128.0f) r = -128.0f;
      if (r > 127.0f) r = 127.0f;
      out_kn[j * n + ch] = (int8_t)r;
    }
  }
}

/* int8GemvRow (qmatmul.zig:171-256): one exact int32 accumulator per column
 * over all of K; epilogue float(acc) * scale_a * scales_b[j], left to right.
 * The 64/8/1 column blocking does not change any result (integer sums). */
static void int8_gemv_row(size_t n, size_t k, const int8_t *a, const int8_t *b,
                          size_t ldb, float *c, float scale_a,
                          const float *scales_b) {
  for (size_t j = 0; j < n; j++) {
    int32_t acc = 0;
    for (size_t p = 0; p < k; p++) acc += (int32_t)a[p] * (int32_t)b[p * ldb + j];
    c[j] = ((float)acc * scale_a) * scales_b[j];
  }
}

#define ORC_KC 512

/* int8GemmTiled (qmatmul.zig:37-99). M<=16: per-row GEMV. M>16: C zeroed,
 * then for every KC=512 chunk of K (in increasing order) C += float(acc_chunk)
 * * sa * sb (microKernel8x8 :494-525 and microKernelEdge :528-549 use the
 * same formula). NC/MC/MR/NR blocking never adds into one element twice per
 * chunk, so only the K chunking is visible in the result. */
int orc_qgemm_int8(size_t m, size_t n, size_t k, const int8_t *a, size_t lda,
                   const int8_t *b, size_t ldb, float *c, size_t ldc,
                   const float *scales_a, const float *scales_b) {
  if (!a || !b || !c || !scales_a || !scales_b) return ORC_ERR_NULL_PTR;
  if (m == 0 || n == 0 || k == 0) return ORC_OK;
  if (m <= 16) {
    for (size_t i = 0; i < m; i++)
      int8_gemv_row(n, k, a + i * lda, b, ldb, c + i * ldc, scales_a[i], scales_b);
    return ORC_OK;
  }
  for (size_t i = 0; i < m; i++) memset(c + i * ldc, 0, n * sizeof(float));
  for (size_t pc = 0; pc < k; pc += ORC_KC) {
    size_t kc = (k - pc < ORC_KC) ? k - pc : ORC_KC;
    for (size_t i = 0; i < m; i++) {
      const int8_t *arow = a + i * lda + pc;
      for (size_t j = 0; j < n; j++) {
        int32_t acc = 0;
        for (size_t p = 0; p < kc; p++)
          acc += (int32_t)arow[p] * (int32_t)b[(pc + p) * ldb + j];
        c[i * ldc + j] = c[i * ldc + j] + ((float)acc * scales_a[i]) * scales_b[j];
      }
    }
  }
  return ORC_OK;
}

/* qmatmul.zig:106-128 */
void orc_naive_int8_gemm(size_t m, size_t n, size_t k, const int8_t *a,
                         size_t lda, const int8_t *b, size_t ldb, float *c,
                         size_t ldc, const float *scales_a,
                         const float *scales_b) {
  for (size_t i = 0; i < m; i++)
    for (size_t j = 0; j < n; j++) {
      int32_t acc = 0;
      for (size_t p = 0; p < k; p++)
        acc += (int32_t)a[i * lda + p] * (int32_t)b[p * ldb + j];
      c[i * ldc + j] = ((float)acc * scales_a[i]) * scales_b[j];
    }
}

/* q4_0GemvRow (qmatmul.zig:276-343). Rows in groups of 4: per block
 * block_sum += a[2i]*lo + a[2i+1]*hi, then sums += block_sum * scale. The
 * n%4 tail rows instead do sum += (a[2i]*lo + a[2i+1]*hi) * scale per pair.
 * Element 2i is the low nibble of byte i (interleaved order). */
int orc_q4_0_gemv(size_t n, size_t k, const float *a, const uint8_t *b_q4,
                  float *c) {
  if (!a || !b_q4 || !c) return ORC_ERR_NULL_PTR;
  if (n == 0 || k == 0) return ORC_OK;
  if (k % 32 != 0) return ORC_ERR_SHAPE_MISMATCH;
  size_t bpr = k / 32, row_bytes = bpr * 18;
  size_t j = 0;
  for (; j + 4 <= n; j += 4) {
    float sums[4] = {0, 0, 0, 0};
    for (size_t blk = 0; blk < bpr; blk++) {
      const float *ab = a + blk * 32;
      for (int r = 0; r < 4; r++) {
        const uint8_t *bs = b_q4 + (j + r) * row_bytes + blk * 18;
        float scale = orc_f16_zig((uint16_t)(bs[0] | (bs[1] << 8)));
        float block_sum = 0.0f;
        for (int i = 0; i < 16; i++) {
          uint8_t byte = bs[2 + i];
          float lo = (float)((int)(byte & 0x0F) - 8);
          float hi = (float)((int)(byte >> 4) - 8);
          float t = ab[2 * i] * lo + ab[2 * i + 1] * hi;
          block_sum = block_sum + t;
        }
        sums[r] = sums[r] + block_sum * scale;
      }
    }
    for (int r = 0; r < 4; r++) c[j + r] = sums[r];
  }
  for (; j < n; j++) {
    float sum = 0.0f;
    for (size_t blk = 0; blk < bpr; blk++) {
      const float *ab = a + blk * 32;
      const uint8_t *bs = b_q4 + j * row_bytes + blk * 18;
      float scale = orc_f16_zig((uint16_t)(bs[0] | (bs[1] << 8)));
      for (int i = 0; i < 16; i++) {
        uint8_t byte = bs[2 + i];
        float lo = (float)((int)(byte & 0x0F) - 8);
        float hi = (float)((int)(byte >> 4) - 8);
        sum = sum + (ab[2 * i] * lo + ab[2 * i + 1] * hi) * scale;
      }
    }
    c[j] = sum;
  }
  return ORC_OK;
}

size_t orc_row_bytes(int fmt, size_t k) {
  switch (fmt) {
    case ORC_FMT_INT8_KN: return k;
    case ORC_FMT_Q4_0: return (k % 32) ? 0 : k / 32 * 18;
    case ORC_FMT_Q8_0: return (k % 32) ? 0 : k / 32 * 34;
    case ORC_FMT_Q4_K: return (k % 256) ? 0 : k / 256 * 144;
    case ORC_FMT_Q6_K: return (k % 256) ? 0 : k / 256 * 210;
  }
  return 0;
}

static uint16_t le16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* gguf.rs:255-288 (Q8_0: scale * q), :294-330 (Q4_0: delta * (nib - 8),
 * low nibble first), :375-431 (Q4_K: 6-bit scale/min unpack, lo*sc - m with
 * separate multiply and subtract), :440-487 (Q6_K: q * (float(sc) * d)). */
int orc_dequant(int fmt, const uint8_t *blk, size_t numel, float *out) {
  if (!blk || !out) return ORC_ERR_NULL_PTR;
  switch (fmt) {
    case ORC_FMT_Q8_0: {
      if (numel % 32) return ORC_ERR_SHAPE_MISMATCH;
      for (size_t b = 0; b < numel / 32; b++) {
        const uint8_t *p = blk + b * 34;
        float scale = orc_f16_rust(le16(p));
        for (int i = 0; i < 32; i++) out[b * 32 + i] = scale * (float)(int8_t)p[2 + i];
      }
      return ORC_OK;
    }
    case ORC_FMT_Q4_0: {
      if (numel % 32) return ORC_ERR_SHAPE_MISMATCH;
      for (size_t b = 0; b < numel / 32; b++) {
        const uint8_t *p = blk + b * 18;
        float delta = orc_f16_rust(le16(p));
        for (int i = 0; i < 16; i++) {
          uint8_t byte = p[2 + i];
          out[b * 32 + 2 * i] = delta * (float)((int)(byte & 0x0F) - 8);
          out[b * 32 + 2 * i + 1] = delta * (float)((int)((byte >> 4) & 0x0F) - 8);
        }
      }
      return ORC_OK;
    }
    case ORC_FMT_Q4_K: {
      if (numel % 256) return ORC_ERR_SHAPE_MISMATCH;
      for (size_t b = 0; b < numel / 256; b++) {
        const uint8_t *p = blk + b * 144;
        float d = orc_f16_rust(le16(p));
        float dmin = orc_f16_rust(le16(p + 2));
        const uint8_t *sb = p + 4;
        uint8_t sc[8], mn[8];
        for (int i = 0; i < 4; i++) {
          sc[i] = sb[i] & 0x3F;
          sc[i + 4] = (uint8_t)((sb[i + 4] & 0x0F) | ((sb[i] >> 6) << 4));
          mn[i] = (uint8_t)((sb[i + 4] >> 4) | ((sb[i + 8] & 0x0F) << 4));
          mn[i + 4] = (uint8_t)((sb[i + 8] >> 4) | (((sb[i] >> 4) & 0x0C) << 4));
        }
        for (int s = 0; s < 8; s++) {
          float scl = d * (float)sc[s];
          float m = dmin * (float)mn[s];
          const uint8_t *q = p + 16 + s * 16;
          for (int i = 0; i < 16; i++) {
            float lo = (float)(q[i] & 0x0F), hi = (float)((q[i] >> 4) & 0x0F);
            out[b * 256 + s * 32 + 2 * i] = lo * scl - m;
            out[b * 256 + s * 32 + 2 * i + 1] = hi * scl - m;
          }
        }
      }
      return ORC_OK;
    }
    case ORC_FMT_Q6_K: {
      if (numel % 256) return ORC_ERR_SHAPE_MISMATCH;
      for (size_t b = 0; b < numel / 256; b++) {
        const uint8_t *p = blk + b * 210;
        const uint8_t *ql = p, *qh = p + 128, *sc = p + 192;
        float d = orc_f16_rust(le16(p + 208));
        for (int sub = 0; sub < 16; sub++) {
          float scale = (float)(int8_t)sc[sub] * d;
          for (int i = 0; i < 16; i++) {
            int idx = sub * 16 + i;
            uint8_t qlb = ql[idx / 2];
            uint8_t lo = (idx % 2 == 0) ? (qlb & 0x0F) : (qlb >> 4);
            uint8_t hi = (qh[idx / 4] >> ((idx % 4) * 2)) & 0x03;
            float q = (float)((int)(lo | (hi << 4)) - 32);
            out[b * 256 + idx] = q * scale;
          }
        }
      }
      return ORC_OK;
    }
  }
  return ORC_ERR_INVALID_ARG;
}

/* f32GemvRow with trans_b (zig/src/ops/matmul.zig:223-300): columns in
 * blocks of 32 then 8 accumulate with @mulAdd sequentially over k; the
 * remaining n%8 columns use sum += a*b (two roundings). */
static void f32_gemv_row_t(size_t n, size_t k, const float *a, const float *b,
                           size_t ldb, float *c) {
  size_t j8 = n - (n % 8); /* columns below j8 take a 32- or 8-wide block */
  for (size_t j = 0; j < n; j++) {
    const float *brow = b + j * ldb;
    float acc = 0.0f;
    if (j < j8) {
      for (size_t p = 0; p < k; p++) acc = fmaf(a[p], brow[p], acc);
    } else {
      for (size_t p = 0; p < k; p++) acc = acc + a[p] * brow[p];
    }
    c[j] = acc;
  }
}

/* syn_sgemm (exports.zig:725-763) + sgemmTiled (matmul.zig:125-184). M<=16:
 * per-row f32GemvRow. M>16: C starts at zero (matmul_t allocates zeros) and
 * each element is a sequential chain over k, carried across the KC=512
 * chunks through C: @mulAdd in full 8x8 tiles (microKernel8x8 :452-492),
 * sum += a*b in edge tiles (microKernelEdge :495-515). Because NC=4096 and
 * MC=256 are multiples of 8, an element is in an edge tile exactly when its
 * row is in the last m%8 rows or its column in the last n%8 columns. */
int orc_sgemm_nt(size_t m, size_t n, size_t k, const float *a, size_t lda,
                 const float *b, size_t ldb, float *c, size_t ldc) {
  if (!a || !b || !c) return ORC_ERR_NULL_PTR;
  for (size_t i = 0; i < m; i++) memset(c + i * ldc, 0, n * sizeof(float));
  if (m == 0 || n == 0 || k == 0) return ORC_OK;
  if (m <= 16) {
    for (size_t i = 0; i < m; i++) f32_gemv_row_t(n, k, a + i * lda, b, ldb, c + i * ldc);
    return ORC_OK;
  }
  size_t m_full = m - (m % 8), n_full = n - (n % 8);
  for (size_t i = 0; i < m; i++) {
    const float *arow = a + i * lda;
    for (size_t j = 0; j < n; j++) {
      const float *brow = b + j * ldb;
      float acc = 0.0f;
      if (i < m_full && j < n_full) {
        for (size_t p = 0; p < k; p++) acc = fmaf(arow[p], brow[p], acc);
      } else {
        for (size_t p = 0; p < k; p++) acc = acc + arow[p] * brow[p];
      }
      c[i * ldc + j] = acc;
    }
  }
  return ORC_OK;
}

int orc_block_matmul(int fmt, size_t m, size_t n, size_t k, const float *x,
                     const uint8_t *w_blocks, float *w_f32, float *y) {
  int st = orc_dequant(fmt, w_blocks, n * k, w_f32);
  if (st) return st;
  return orc_sgemm_nt(m, n, k, x, k, w_f32, k, y, n);
}
