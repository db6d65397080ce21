/*
 * synapse_oracle_lm.c -- CPU restatement of the reference's language-model
 * epilogue arithmetic around the quantized matmuls: RMSNorm, RoPE, softmax,
 * cached GQA attention (decode and prefill), SwiGLU and greedy argmax.
 * TEST INFRASTRUCTURE ONLY (see synapse_oracle.h).
 *
 * Same build rules as synapse_oracle.c: -ffp-contract=off, fmaf() exactly
 * where the Zig source writes @mulAdd, one rounding per Rust/Zig operation.
 *
 * exp: the reference calls f32 exp (Rust f32::exp -> the platform expf; Zig
 * @exp). Both sides of the parity check use orc_exp = exp evaluated in double
 * and rounded once to float, i.e. the correctly rounded expf except in the
 * rare cases where the double result lies within 2^-53 relative of a float
 * rounding boundary. Whether that equals the reference binary's expf on every
 * input cannot be checked without its toolchain.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "synapse_oracle.h"

float orc_exp(float x) { return (float)exp((double)x); }

/* vecHsum (zig/src/ffi/exports.zig:503-514): four lane accumulators over
 * groups of 4 (acc += v, F32x4), @reduce(.Add) in lane order (strict float
 * mode keeps the association ((l0+l1)+l2)+l3), then the tail in order. */
static float vec_hsum(const float *src, size_t len) {
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  size_t i = 0;
  for (; i + 4 <= len; i += 4)
    for (int l = 0; l < 4; l++) acc[l] = acc[l] + src[i + l];
  float s = ((acc[0] + acc[1]) + acc[2]) + acc[3];
  for (; i < len; i++) s = s + src[i];
  return s;
}

/* rmsnorm (ops/norm.rs:8-37): sq = x*x (syn_vmul, exports.zig:968-975),
 * sum_sq = vecHsum(sq) (syn_vreduce_sum, exports.zig:987-996),
 * scale = 1 / sqrt(sum_sq / h + eps), out = (x * w) * scale. */
void orc_rmsnorm(const float *x, const float *w, size_t rows, size_t h, float eps,
                 float *out) {
  float *sq = (float *)malloc(h * sizeof(float));
  for (size_t r = 0; r < rows; r++) {
    const float *xr = x + r * h;
    float *o = out + r * h;
    for (size_t j = 0; j < h; j++) sq[j] = xr[j] * xr[j];
    float sum_sq = vec_hsum(sq, h);
    float scale = 1.0f / sqrtf(sum_sq / (float)h + eps);
    for (size_t j = 0; j < h; j++) o[j] = (xr[j] * w[j]) * scale;
  }
  free(sq);
}

/* precompute_rope_tables (models/lm/builder.rs:88-133), no scaling:
 * freq = 1 / base_f32^(2i/hd), angle = pos * freq, all in f32. */
void orc_rope_tables(double base, size_t max_pos, size_t hd, float *cos_t, float *sin_t) {
  size_t half = hd / 2;
  for (size_t pos = 0; pos < max_pos; pos++)
    for (size_t i = 0; i < half; i++) {
      float freq = 1.0f / powf((float)base, (2.0f * (float)i) / (float)hd);
      float scaled = freq / 1.0f;
      float angle = (float)pos * scaled;
      cos_t[pos * half + i] = cosf(angle);
      sin_t[pos * half + i] = sinf(angle);
    }
}

/* apply_rope_inplace, RotateHalf (ops/rope.rs:13-60). */
void orc_rope_inplace(float *qk, const float *cos_t, const float *sin_t, size_t seq,
                      size_t heads, size_t hd, size_t pos_off) {
  size_t half = hd / 2, total = heads * hd;
  for (size_t t = 0; t < seq; t++) {
    size_t row = (pos_off + t) * half;
    for (size_t h = 0; h < heads; h++) {
      float *b = qk + t * total + h * hd;
      for (size_t i = 0; i < half; i++) {
        float c = cos_t[row + i], s = sin_t[row + i];
        float x1 = b[i], x2 = b[half + i];
        b[i] = x1 * c - x2 * s;
        b[half + i] = x2 * c + x1 * s;
      }
    }
  }
}

/* softmax_slice (ops/activation.rs:117-130). */
void orc_softmax(float *x, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    x[i] = orc_exp(x[i] - mx);
    sum = sum + x[i];
  }
  if (sum > 0.0f)
    for (size_t i = 0; i < n; i++) x[i] = x[i] / sum;
}

/* f32GemvRow without trans_b (zig/src/ops/matmul.zig:302-343): columns in
 * blocks of 32 accumulate with @mulAdd sequentially over k; the remaining
 * n%32 columns use sum += a*b. */
static void f32_gemv_row_n(size_t n, size_t k, const float *a, const float *b, size_t ldb,
                           float *c) {
  size_t j32 = n - (n % 32);
  for (size_t j = 0; j < n; j++) {
    float acc = 0.0f;
    if (j < j32)
      for (size_t p = 0; p < k; p++) acc = fmaf(a[p], b[p * ldb + j], acc);
    else
      for (size_t p = 0; p < k; p++) acc = acc + a[p] * b[p * ldb + j];
    c[j] = acc;
  }
}

/* matmul_nn (ops/matmul.rs:82-101): out zeroed, syn_sgemm(trans_b=0) ->
 * sgemmTiled. Same chain structure as orc_sgemm_nt: M<=16 per-row GEMV; M>16
 * full 8x8 tiles with @mulAdd and edge tiles with sum += a*b. */
int orc_sgemm_nn(size_t m, size_t n, size_t k, const float *a, size_t lda, const float *b,
                 size_t ldb, float *c, size_t ldc) {
  if (!a || !b || !c) return ORC_ERR_NULL_PTR;
  for (size_t i = 0; i < m; i++) memset(c + i * ldc, 0, n * sizeof(float));
  if (m == 0 || n == 0 || k == 0) return ORC_OK;
  if (m <= 16) {
    for (size_t i = 0; i < m; i++) f32_gemv_row_n(n, k, a + i * lda, b, ldb, c + i * ldc);
    return ORC_OK;
  }
  size_t m_full = m - (m % 8), n_full = n - (n % 8);
  for (size_t i = 0; i < m; i++)
    for (size_t j = 0; j < n; j++) {
      float acc = 0.0f;
      if (i < m_full && j < n_full)
        for (size_t p = 0; p < k; p++) acc = fmaf(a[i * lda + p], b[p * ldb + j], acc);
      else
        for (size_t p = 0; p < k; p++) acc = acc + a[i * lda + p] * b[p * ldb + j];
      c[i * ldc + j] = acc;
    }
  return ORC_OK;
}

/* cached_attention_decode after the cache append (ops/attention.rs:70-147).
 * kc, vc: the cache [len, n_kv*hd]; q: [n_heads*hd] (normed, RoPE'd).
 * window 0 = none. Below 64 effective positions: scalar dot products and
 * weighted sums (sum += a*b); from 64 on: matmul_t (f32GemvRow with trans_b)
 * for the scores and matmul_nn (f32GemvRow) for score*V. */
void orc_attention_decode(const float *q, const float *kc, const float *vc, size_t len,
                          size_t n_heads, size_t n_kv, size_t hd, size_t window, float *out) {
  size_t kv_dim = n_kv * hd, groups = n_heads / n_kv;
  float scale = 1.0f / sqrtf((float)hd);
  size_t eff = len, off = 0;
  if (window && len > window) {
    off = len - window;
    eff = window;
  }
  const float *ek = kc + off * kv_dim, *ev = vc + off * kv_dim;
  float *scores = (float *)malloc((eff ? eff : 1) * sizeof(float));
  if (eff >= 64) {
    float *kb = (float *)malloc(eff * hd * sizeof(float));
    float *vb = (float *)malloc(eff * hd * sizeof(float));
    for (size_t h = 0; h < n_heads; h++) {
      size_t kvh = h / groups;
      for (size_t s = 0; s < eff; s++) {
        memcpy(kb + s * hd, ek + s * kv_dim + kvh * hd, hd * sizeof(float));
        memcpy(vb + s * hd, ev + s * kv_dim + kvh * hd, hd * sizeof(float));
      }
      orc_sgemm_nt(1, eff, hd, q + h * hd, hd, kb, hd, scores, eff);
      for (size_t s = 0; s < eff; s++) scores[s] = scores[s] * scale;
      orc_softmax(scores, eff);
      orc_sgemm_nn(1, hd, eff, scores, eff, vb, hd, out + h * hd, hd);
    }
    free(kb);
    free(vb);
  } else {
    for (size_t h = 0; h < n_heads; h++) {
      size_t kvh = h / groups;
      for (size_t s = 0; s < eff; s++) {
        float dot = 0.0f;
        for (size_t d = 0; d < hd; d++)
          dot = dot + q[h * hd + d] * ek[s * kv_dim + kvh * hd + d];
        scores[s] = dot * scale;
      }
      orc_softmax(scores, eff);
      for (size_t d = 0; d < hd; d++) {
        float sum = 0.0f;
        for (size_t s = 0; s < eff; s++) sum = sum + scores[s] * ev[s * kv_dim + kvh * hd + d];
        out[h * hd + d] = sum;
      }
    }
  }
  free(scores);
}

/* syn_fused_attention (zig/src/ffi/exports.zig:1364-1478): per tile of
 * TILE_Q=32 query rows (ops/attention.zig:25): S = Q K^T (sgemmTiled),
 * S *= scale, causal -inf mask, online max/sum per row, P = exp(S-mx)*(1/se),
 * O = P V (sgemmTiled). q,k,v,out: [seq, hd] of one head. */
int orc_fused_attention(size_t seq_q, size_t seq_k, size_t hd, const float *q, const float *k,
                        const float *v, float *out) {
  if (!q || !k || !v || !out) return ORC_ERR_NULL_PTR;
  if (seq_q == 0 || seq_k == 0 || hd == 0) return ORC_OK;
  const size_t TILE_Q = 32;
  float *s = (float *)malloc(TILE_Q * seq_k * sizeof(float));
  float scale = 1.0f / sqrtf((float)hd);
  for (size_t tq = 0; tq < seq_q; tq += TILE_Q) {
    size_t tqs = seq_q - tq < TILE_Q ? seq_q - tq : TILE_Q;
    orc_sgemm_nt(tqs, seq_k, hd, q + tq * hd, hd, k, hd, s, seq_k);
    for (size_t i = 0; i < tqs * seq_k; i++) s[i] = s[i] * scale;
    for (size_t i = 0; i < tqs; i++)
      for (size_t j = tq + i + 1; j < seq_k; j++) s[i * seq_k + j] = -INFINITY;
    for (size_t i = 0; i < tqs; i++) {
      float *r = s + i * seq_k;
      float mx = -INFINITY, se = 0.0f;
      for (size_t j = 0; j < seq_k; j++) {
        float x = r[j];
        if (x > mx) {
          se = se * orc_exp(mx - x) + 1.0f;
          mx = x;
        } else {
          se = se + orc_exp(x - mx);
        }
      }
      float inv = 1.0f / se;
      for (size_t j = 0; j < seq_k; j++) r[j] = orc_exp(r[j] - mx) * inv;
    }
    orc_sgemm_nn(tqs, hd, seq_k, s, seq_k, v, hd, out + tq * hd, hd);
  }
  free(s);
  return ORC_OK;
}

/* INT8 model SwiGLU (quantization/lm/int8.rs:500-503): silu(g) * u with
 * silu(x) = x / (1 + exp(-x)) (ops/activation.rs:30-32). */
void orc_silu_mul(const float *g, const float *u, size_t n, float *out) {
  for (size_t i = 0; i < n; i++) {
    float x = g[i];
    out[i] = (x / (1.0f + orc_exp(-x))) * u[i];
  }
}

/* syn_swiglu -> swigluFused (zig/src/ops/silu.zig:85-114): groups of 4
 * (F32x4, also inside the 2x-unrolled loop) compute g * (1/(1+exp(-g))) * u;
 * the scalar tail computes (g / (1+exp(-g))) * u. */
void orc_swiglu(const float *g, const float *u, size_t n, float *out) {
  size_t n4 = n - (n % 4), i = 0;
  for (; i < n4; i++) {
    float sig = 1.0f / (1.0f + orc_exp(-g[i]));
    out[i] = (g[i] * sig) * u[i];
  }
  for (; i < n; i++) out[i] = (g[i] / (1.0f + orc_exp(-g[i]))) * u[i];
}

/* argmax (generation/sampler.rs:217-224): Iterator::max_by with
 * partial_cmp, NaN comparing Equal: the running best is replaced unless it
 * compares strictly Greater, so the last maximal index wins ties and a NaN
 * restarts the scan. */
uint32_t orc_argmax(const float *x, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  for (size_t i = 1; i < n; i++) {
    float b = x[best], e = x[i];
    int greater = !isnan(b) && !isnan(e) && b > e;
    if (!greater) best = i;
  }
  return (uint32_t)best;
}
