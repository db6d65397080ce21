// gemv.cu -- decode-path fused dequant GEMV for all five weight formats.
//
// One kernel per (format, activation rows MT, weight rows per warp R):
//  1. Prologue (per CTA, into shared memory): the MT activation rows are
//     converted once. INT8 weights: per-row INT8 quantisation exactly as
//     quantize.zig:12-47 (W8A8 like QuantizedLinear::forward,
//     int8_linear.rs:87-117). Block formats: each 32-element block of x is
//     scaled to 16-bit integers (|xq| <= 32767, per-block f32 scale) and
//     split into a signed high byte and an unsigned low byte, so that every
//     product runs as exact 4-way integer dot products (dp4a); the per-block
//     integer sums are exact and the only rounding is the 2^-16 relative
//     activation quantisation plus the f32 sum over blocks.
//  2. Main loop: each warp owns R output rows; lane l streams 32-element
//     block b = l + 32 i of each row with 16-byte non-allocating loads
//     (512 contiguous bytes per warp per plane), dequantises with one or two
//     logic ops per 8 weights, and accumulates; a warp-shuffle reduction
//     finishes each row.
// The grid is persistent (bounded by occupancy) and strides over rows.
#include <mutex>
#include <unordered_map>

#include "internal.cuh"

namespace syn {
namespace {

enum : int { F_INT8 = SYN_QFMT_INT8_KN, F_Q4_0 = SYN_QFMT_Q4_0, F_Q8_0 = SYN_QFMT_Q8_0,
             F_Q4_K = SYN_QFMT_Q4_K, F_Q6_K = SYN_QFMT_Q6_K, F_Q4_0RAW = 100 };

struct GemvParams {
  const uint8_t* q;
  const uint16_t* d;
  const float* sb;
  const uint8_t* hdr;
  const uint8_t* qh;
  const int8_t* sc;
  long long n, k, kp, nblk;
  const float* x;
  long long ldx;
  const int8_t* xq;
  long long ldxq;
  const float* sx;
  long long m;
  float* y;
  long long ldy;
  int chunked;
};

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;

__host__ __device__ constexpr bool interleaved(int f) {
  return f == F_Q4_0 || f == F_Q4_K || f == F_Q6_K || f == F_Q4_0RAW;
}

// Shared-memory bytes per activation row.
__host__ __device__ inline long long act_stride(int fmt, long long kp, long long nblk) {
  if (fmt == F_INT8) return kp + 16;
  return ((76 * nblk) + 15) / 16 * 16;
}

// ---------------------------------------------------------------------------
// Prologues
// ---------------------------------------------------------------------------
template <int MT>
__device__ void prologue_int8(const GemvParams& p, long long m0, uint8_t* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float red[WARPS];
  const long long stride = act_stride(F_INT8, p.kp, p.nblk);
  for (int mm = 0; mm < MT; mm++) {
    long long m = m0 + mm;
    int8_t* xs = reinterpret_cast<int8_t*>(smem + mm * stride);
    float* sa = reinterpret_cast<float*>(smem + mm * stride + p.kp);
    if (m >= p.m) {
      for (long long i = threadIdx.x; i < p.kp; i += THREADS) xs[i] = 0;
      if (threadIdx.x == 0) *sa = 0.0f;
      continue;
    }
    if (p.xq) {  // pre-quantised activations (forward_pre_quantized)
      const int8_t* src = p.xq + m * p.ldxq;
      for (long long i = threadIdx.x; i < p.kp; i += THREADS) xs[i] = i < p.k ? src[i] : 0;
      if (threadIdx.x == 0) *sa = p.sx[m];
      continue;
    }
    const float* xr = p.x + m * p.ldx;
    float amax = 0.0f;
    for (long long i = threadIdx.x; i < p.k; i += THREADS) amax = fmaxf(amax, fabsf(xr[i]));
    amax = warp_max(amax);
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < WARPS; w++) amax = fmaxf(amax, red[w]);
    __syncthreads();
    // quantize.zig:28-45: zero row -> scale 1, q 0; else scale = max/127,
    // q = clamp(round(x * (127/max)), -127, 127), round half away from zero.
    if (amax == 0.0f) {
      for (long long i = threadIdx.x; i < p.kp; i += THREADS) xs[i] = 0;
      if (threadIdx.x == 0) *sa = 1.0f;
    } else {
      float inv = __fdiv_rn(127.0f, amax);
      for (long long i = threadIdx.x; i < p.kp; i += THREADS) {
        int8_t v = 0;
        if (i < p.k) {
          float r = roundf(__fmul_rn(xr[i], inv));
          r = fminf(127.0f, fmaxf(-127.0f, r));
          v = (int8_t)(int)r;
        }
        xs[i] = v;
      }
      if (threadIdx.x == 0) *sa = __fdiv_rn(amax, 127.0f);
    }
  }
}

template <int FMT, int MT>
__device__ void prologue_blocks(const GemvParams& p, long long m0, uint8_t* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nblk = p.nblk;
  const long long stride = act_stride(FMT, p.kp, nblk);
  for (long long t = warp; t < MT * nblk; t += WARPS) {
    int mm = (int)(t / nblk);
    long long b = t - (long long)mm * nblk;
    long long m = m0 + mm;
    uint8_t* base = smem + mm * stride;
    float x = (m < p.m) ? p.x[m * p.ldx + b * 32 + lane] : 0.0f;
    float amax = warp_max(fabsf(x));
    int xq = 0;
    float s = 0.0f;
    if (amax > 0.0f) {
      float inv = 32767.0f / amax;
      xq = __float2int_rn(x * inv);
      xq = max(-32767, min(32767, xq));
      s = amax / 32767.0f;
    }
    uint8_t hb = (uint8_t)((xq >> 8) & 0xFF);  // signed high byte
    uint8_t lb = (uint8_t)(xq & 0xFF);         // unsigned low byte
    int plane, slot;
    if (interleaved(FMT)) {
      plane = lane & 1;  // element 2i -> even plane, 2i+1 -> odd plane
      slot = lane >> 1;
    } else {
      plane = lane >> 4;  // natural order: bytes 0-15, 16-31
      slot = lane & 15;
    }
    base[(plane)*nblk * 16 + b * 16 + slot] = hb;
    base[(plane + 2) * nblk * 16 + b * 16 + slot] = lb;
    int s0 = warp_sum_i(lane < 16 ? xq : 0);
    int s1 = warp_sum_i(lane >= 16 ? xq : 0);
    if (lane == 0) {
      reinterpret_cast<int2*>(base + 64 * nblk)[b] = make_int2(s0, s1);
      reinterpret_cast<float*>(base + 72 * nblk)[b] = s;
    }
  }
}

// ---------------------------------------------------------------------------
// Per-format block dot products. Each returns this lane's contribution of
// one 32-element block of one weight row against one activation row.
// ---------------------------------------------------------------------------
struct WBlk {
  uint4 a, b;      // weight bytes (b used by INT8/Q8_0)
  uint32_t meta0;  // f16 scale bits / packed int8 scales
  uint2 meta1;     // Q6_K high bits or Q4_K 16-byte header (first half)
  uint2 meta2;     // Q4_K header second half
};

struct ABlk {
  uint4 p0, p1, p2, p3;
  int2 sums;
  float s;
};

template <int FMT>
__device__ __forceinline__ void load_w(const GemvParams& p, long long n, long long b, WBlk& w) {
  if constexpr (FMT == F_INT8) {
    const uint8_t* src = p.q + n * p.kp + b * 32;
    w.a = ld_stream16(src);
    w.b = ld_stream16(src + 16);
  } else if constexpr (FMT == F_Q8_0) {
    const uint8_t* src = p.q + n * p.k + b * 32;
    w.a = ld_stream16(src);
    w.b = ld_stream16(src + 16);
    w.meta0 = ld_nc_u16(p.d + n * p.nblk + b);
  } else if constexpr (FMT == F_Q4_0) {
    w.a = ld_stream16(p.q + n * (p.k / 2) + b * 16);
    w.meta0 = ld_nc_u16(p.d + n * p.nblk + b);
  } else if constexpr (FMT == F_Q4_K) {
    w.a = ld_stream16(p.q + n * (p.k / 2) + b * 16);
    const uint4 h = __ldg(reinterpret_cast<const uint4*>(p.hdr + (n * (p.k / 256) + (b >> 3)) * 16));
    w.meta1 = make_uint2(h.x, h.y);
    w.meta2 = make_uint2(h.z, h.w);
  } else if constexpr (FMT == F_Q6_K) {
    w.a = ld_stream16(p.q + n * (p.k / 2) + b * 16);
    w.meta1 = ld_stream8(p.qh + (n * p.nblk + b) * 8);
    uint32_t scp = ld_nc_u16(reinterpret_cast<const uint16_t*>(p.sc) + n * p.nblk + b);
    uint32_t dd = ld_nc_u16(p.d + n * (p.k / 256) + (b >> 3));
    w.meta0 = scp | (dd << 16);
  } else {  // F_Q4_0RAW: reference 18-byte blocks, 2-byte aligned
    const uint16_t* src = reinterpret_cast<const uint16_t*>(p.q + (n * p.nblk + b) * 18);
    uint32_t h[9];
#pragma unroll
    for (int i = 0; i < 9; i++) h[i] = ld_nc_u16(src + i);
    w.meta0 = h[0];
    w.a = make_uint4(h[1] | (h[2] << 16), h[3] | (h[4] << 16), h[5] | (h[6] << 16),
                     h[7] | (h[8] << 16));
  }
}

template <int FMT>
__device__ __forceinline__ void load_a(const uint8_t* base, long long nblk, long long b, ABlk& a) {
  if constexpr (FMT == F_INT8) {
    const uint4* src = reinterpret_cast<const uint4*>(base + b * 32);
    a.p0 = src[0];
    a.p1 = src[1];
  } else {
    a.p0 = reinterpret_cast<const uint4*>(base)[b];
    a.p1 = reinterpret_cast<const uint4*>(base + nblk * 16)[b];
    a.p2 = reinterpret_cast<const uint4*>(base + nblk * 32)[b];
    a.p3 = reinterpret_cast<const uint4*>(base + nblk * 48)[b];
    a.sums = reinterpret_cast<const int2*>(base + 64 * nblk)[b];
    a.s = reinterpret_cast<const float*>(base + 72 * nblk)[b];
  }
}

__device__ __forceinline__ uint32_t w4(const uint4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// INT8: exact int32 partial sum of the block.
__device__ __forceinline__ int dot_int8(const WBlk& w, const ABlk& a) {
  int acc = 0;
  acc = dp4a_ss(a.p0.x, w.a.x, acc);
  acc = dp4a_ss(a.p0.y, w.a.y, acc);
  acc = dp4a_ss(a.p0.z, w.a.z, acc);
  acc = dp4a_ss(a.p0.w, w.a.w, acc);
  acc = dp4a_ss(a.p1.x, w.b.x, acc);
  acc = dp4a_ss(a.p1.y, w.b.y, acc);
  acc = dp4a_ss(a.p1.z, w.b.z, acc);
  acc = dp4a_ss(a.p1.w, w.b.w, acc);
  return acc;
}

// sum_i q_i * xq_i for unsigned nibble codes q (interleaved planes).
__device__ __forceinline__ int dot_nib(const uint4& q, const ABlk& a) {
  int hl = 0, hh = 0, ll = 0, lh = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    uint32_t wq = w4(q, j);
    uint32_t lo = wq & 0x0F0F0F0Fu;
    uint32_t hi16 = wq & 0xF0F0F0F0u;  // 16 * high nibble, exact after >> 4
    hl = dp4a_su(w4(a.p0, j), lo, hl);
    hh = dp4a_su(w4(a.p1, j), hi16, hh);
    ll = dp4a_uu(w4(a.p2, j), lo, ll);
    lh = dp4a_uu(w4(a.p3, j), hi16, lh);
  }
  return (hl + (hh >> 4)) * 256 + ll + (lh >> 4);
}

template <int FMT>
__device__ __forceinline__ float dot_f(const WBlk& w, const ABlk& a) {
  if constexpr (FMT == F_Q4_0 || FMT == F_Q4_0RAW) {
    int iq = dot_nib(w.a, a) - 8 * (a.sums.x + a.sums.y);
    float d = (FMT == F_Q4_0) ? f16_loader((uint16_t)w.meta0) : f16_exact((uint16_t)w.meta0);
    return (float)iq * (a.s * d);
  } else if constexpr (FMT == F_Q8_0) {
    int ih = 0, il = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      ih = dp4a_ss(w4(a.p0, j), w4(w.a, j), ih);
      ih = dp4a_ss(w4(a.p1, j), w4(w.b, j), ih);
      il = dp4a_us(w4(a.p2, j), w4(w.a, j), il);
      il = dp4a_us(w4(a.p3, j), w4(w.b, j), il);
    }
    float d = f16_loader((uint16_t)w.meta0);
    return (float)(ih * 256 + il) * (a.s * d);
  } else {
    return 0.0f;
  }
}

// Q4_K (gguf.rs:400-427): 6-bit scale / min unpack for sub-block s, then
// sum_i x_i (q_i sc - m) = sc * sum(q xq) - m * sum(xq), times the block scale.
__device__ __forceinline__ float dot_q4k(const WBlk& w, const ABlk& a, int s) {
  uint32_t h0 = w.meta1.x, y = w.meta1.y, z = w.meta2.x, wv = w.meta2.y;
  float dd = f16_loader((uint16_t)(h0 & 0xFFFF));
  float dmin = f16_loader((uint16_t)(h0 >> 16));
  uint32_t scv, mnv;
  if (s < 4) {
    int sh = 8 * s;
    scv = (y >> sh) & 0x3F;
    mnv = ((z >> sh) & 0xFF) >> 4 | (((wv >> sh) & 0x0F) << 4);
  } else {
    int sh = 8 * (s - 4);
    uint32_t ys = (y >> sh) & 0xFF;
    scv = ((z >> sh) & 0x0F) | ((ys >> 6) << 4);
    mnv = (((wv >> sh) & 0xFF) >> 4) | (((ys >> 4) & 0x0C) << 4);
  }
  float scl = dd * (float)scv;
  float mval = dmin * (float)mnv;
  int iq = dot_nib(w.a, a);
  return a.s * (scl * (float)iq - mval * (float)(a.sums.x + a.sums.y));
}

__device__ __forceinline__ float dot_q6k(const WBlk& w, const ABlk& a) {
  int h0 = 0, l0 = 0, h1 = 0, l1 = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    uint32_t wq = w4(w.a, j);
    uint32_t H = (j < 2) ? w.meta1.x : w.meta1.y;
    uint32_t he = (j & 1) ? (H & 0x30303030u) : ((H << 4) & 0x30303030u);
    uint32_t ho = (j & 1) ? ((H >> 2) & 0x30303030u) : ((H << 2) & 0x30303030u);
    uint32_t qe = (wq & 0x0F0F0F0Fu) | he;
    uint32_t qo = ((wq >> 4) & 0x0F0F0F0Fu) | ho;
    if (j < 2) {
      h0 = dp4a_su(w4(a.p0, j), qe, h0);
      h0 = dp4a_su(w4(a.p1, j), qo, h0);
      l0 = dp4a_uu(w4(a.p2, j), qe, l0);
      l0 = dp4a_uu(w4(a.p3, j), qo, l0);
    } else {
      h1 = dp4a_su(w4(a.p0, j), qe, h1);
      h1 = dp4a_su(w4(a.p1, j), qo, h1);
      l1 = dp4a_uu(w4(a.p2, j), qe, l1);
      l1 = dp4a_uu(w4(a.p3, j), qo, l1);
    }
  }
  int i0 = h0 * 256 + l0 - 32 * a.sums.x;
  int i1 = h1 * 256 + l1 - 32 * a.sums.y;
  float dd = f16_loader((uint16_t)(w.meta0 >> 16));
  float sc0 = (float)(int8_t)(w.meta0 & 0xFF) * dd;
  float sc1 = (float)(int8_t)((w.meta0 >> 8) & 0xFF) * dd;
  return a.s * ((float)i0 * sc0 + (float)i1 * sc1);
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int FMT, int MT, int R>
__global__ void __launch_bounds__(THREADS) k_qgemv(GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const long long m0 = (long long)blockIdx.y * MT;
  if constexpr (FMT == F_INT8)
    prologue_int8<MT>(p, m0, smem);
  else
    prologue_blocks<FMT, MT>(p, m0, smem);
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long stride = act_stride(FMT, p.kp, p.nblk);
  const long long total_warps = (long long)gridDim.x * WARPS;
  const long long iters = (p.nblk + 31) / 32;

  for (long long row0 = ((long long)blockIdx.x * WARPS + warp) * R; row0 < p.n;
       row0 += total_warps * R) {
    float facc[R][MT];
    int iacc[R][MT];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int mm = 0; mm < MT; mm++) {
        facc[r][mm] = 0.0f;
        iacc[r][mm] = 0;
      }

    for (long long it = 0; it < iters; it++) {
      const long long b = it * 32 + lane;
      const bool valid = b < p.nblk;
      WBlk w[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        if (valid && row0 + r < p.n) {
          load_w<FMT>(p, row0 + r, b, w[r]);
        } else {
          w[r].a = make_uint4(0, 0, 0, 0);
          w[r].b = make_uint4(0, 0, 0, 0);
          w[r].meta0 = 0;
          w[r].meta1 = make_uint2(0, 0);
          w[r].meta2 = make_uint2(0, 0);
        }
      }
#pragma unroll
      for (int mm = 0; mm < MT; mm++) {
        ABlk a;
        if (valid) {
          load_a<FMT>(smem + mm * stride, p.nblk, b, a);
        } else {
          a.p0 = a.p1 = a.p2 = a.p3 = make_uint4(0, 0, 0, 0);
          a.sums = make_int2(0, 0);
          a.s = 0.0f;
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
          if constexpr (FMT == F_INT8) {
            int part = dot_int8(w[r], a);
            if (p.chunked) {
              // qmatmul.zig:68-98 (M>16): float sum over 512-wide K chunks in
              // increasing order. Lanes 0-15 hold chunk 2*it, 16-31 chunk 2*it+1.
#pragma unroll
              for (int o = 8; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
              int part_hi = __shfl_sync(0xffffffffu, part, 16);
              if (lane == 0 && row0 + r < p.n) {
                const float sa = reinterpret_cast<const float*>(smem + mm * stride + p.kp)[0];
                const float sbv = p.sb[row0 + r];
                facc[r][mm] = facc[r][mm] + ((float)part * sa) * sbv;
                if (it * 32 + 16 < p.nblk)
                  facc[r][mm] = facc[r][mm] + ((float)part_hi * sa) * sbv;
              }
            } else {
              iacc[r][mm] += part;
            }
          } else if constexpr (FMT == F_Q4_K) {
            facc[r][mm] += dot_q4k(w[r], a, (int)(b & 7));
          } else if constexpr (FMT == F_Q6_K) {
            facc[r][mm] += dot_q6k(w[r], a);
          } else {
            facc[r][mm] += dot_f<FMT>(w[r], a);
          }
        }
      }
    }

    // Finish each (row, activation row) pair.
#pragma unroll
    for (int r = 0; r < R; r++) {
#pragma unroll
      for (int mm = 0; mm < MT; mm++) {
        const long long n = row0 + r, m = m0 + mm;
        if constexpr (FMT == F_INT8) {
          if (p.chunked) {
            if (lane == 0 && n < p.n && m < p.m) p.y[m * p.ldy + n] = facc[r][mm];
          } else {
            int tot = warp_sum_i(iacc[r][mm]);
            if (lane == 0 && n < p.n && m < p.m) {
              const float sa = reinterpret_cast<const float*>(smem + mm * stride + p.kp)[0];
              // qmatmul.zig:218-223: f_acc * sa * sb, left to right.
              p.y[m * p.ldy + n] = __fmul_rn(__fmul_rn((float)tot, sa), p.sb[n]);
            }
          }
        } else {
          float v = warp_sum(facc[r][mm]);
          if (lane == 0 && n < p.n && m < p.m) p.y[m * p.ldy + n] = v;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side launch
// ---------------------------------------------------------------------------
struct OccKey {
  const void* f;
  long long smem;
  bool operator==(const OccKey& o) const { return f == o.f && smem == o.smem; }
};
struct OccHash {
  size_t operator()(const OccKey& k) const {
    return std::hash<const void*>()(k.f) ^ (std::hash<long long>()(k.smem) << 1);
  }
};

int occupancy(const void* f, long long smem) {
  static std::mutex mu;
  static std::unordered_map<OccKey, int, OccHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  OccKey key{f, smem * 64 + dev};
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int nb = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, f, THREADS, (size_t)smem);
  if (nb < 1) nb = 0;
  cache[key] = nb;
  return nb;
}

template <int FMT, int MT, int R>
syn_status_t launch_t(const GemvParams& p, cudaStream_t st) {
  const void* f = reinterpret_cast<const void*>(&k_qgemv<FMT, MT, R>);
  long long smem = MT * act_stride(FMT, p.kp, p.nblk);
  if (smem > 227 * 1024) return SYN_ERR_UNSUPPORTED;
  int occ = occupancy(f, smem);
  if (occ < 1) return SYN_ERR_UNSUPPORTED;
  long long need = (p.n + (long long)WARPS * R - 1) / ((long long)WARPS * R);
  long long cap = (long long)num_sms() * occ;
  dim3 grid((unsigned)(need < cap ? need : cap), (unsigned)((p.m + MT - 1) / MT));
  k_qgemv<FMT, MT, R><<<grid, THREADS, (size_t)smem, st>>>(p);
  SYN_LAUNCH_CHECK("k_qgemv");
  return SYN_OK;
}

template <int FMT, int MT>
syn_status_t launch_r(const GemvParams& p, cudaStream_t st) {
  const long long sms = num_sms();
  if (p.n >= WARPS * 4 * 2 * sms) return launch_t<FMT, MT, 4>(p, st);
  if (p.n >= WARPS * 2 * 2 * sms) return launch_t<FMT, MT, 2>(p, st);
  return launch_t<FMT, MT, 1>(p, st);
}

template <int FMT>
syn_status_t launch_m(const GemvParams& p, cudaStream_t st) {
  if (p.m == 1) return launch_r<FMT, 1>(p, st);
  if (p.m == 2) return launch_r<FMT, 2>(p, st);
  syn_status_t s = launch_r<FMT, 4>(p, st);
  if (s == SYN_ERR_UNSUPPORTED) s = launch_r<FMT, 1>(p, st);  // shared memory bound
  return s;
}

}  // namespace

syn_status_t launch_qgemv(const syn_cuda_weight_s* w, const float* x, size_t ldx,
                          const int8_t* xq, const float* sx, size_t m, float* y,
                          size_t ldy, int chunked, cudaStream_t st) {
  GemvParams p{};
  p.q = w->q;
  p.d = w->d;
  p.sb = w->sb;
  p.hdr = w->hdr;
  p.qh = w->qh;
  p.sc = w->sc;
  p.n = (long long)w->n;
  p.k = (long long)w->k;
  p.kp = (long long)w->kp;
  p.nblk = (long long)(w->kp / 32);
  p.x = x;
  p.ldx = (long long)ldx;
  p.xq = xq;
  p.ldxq = (long long)ldx;
  p.sx = sx;
  p.m = (long long)m;
  p.y = y;
  p.ldy = (long long)ldy;
  p.chunked = chunked;
  switch (w->fmt) {
    case SYN_QFMT_INT8_KN: return launch_m<F_INT8>(p, st);
    case SYN_QFMT_Q4_0: return launch_m<F_Q4_0>(p, st);
    case SYN_QFMT_Q8_0: return launch_m<F_Q8_0>(p, st);
    case SYN_QFMT_Q4_K: return launch_m<F_Q4_K>(p, st);
    case SYN_QFMT_Q6_K: return launch_m<F_Q6_K>(p, st);
  }
  return SYN_ERR_INVALID_ARG;
}

syn_status_t launch_q4_0_raw(size_t n, size_t k, const float* a, const uint8_t* b, float* c,
                             cudaStream_t st) {
  GemvParams p{};
  p.q = b;
  p.n = (long long)n;
  p.k = (long long)k;
  p.kp = (long long)k;
  p.nblk = (long long)(k / 32);
  p.x = a;
  p.ldx = (long long)k;
  p.m = 1;
  p.y = c;
  p.ldy = (long long)n;
  return launch_r<F_Q4_0RAW, 1>(p, st);
}

}  // namespace syn
