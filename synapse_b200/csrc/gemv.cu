// gemv.cu -- decode-path fused dequant GEMV for all five weight formats.
//
// Layout. Weights are repacked row-interleaved by 32 (repack.cu): for a
// group of 32 rows and one 32-element block, the 32 rows' bytes are stored
// back to back, and all tiles of one row group follow each other in K order.
// Lane l of a warp owns row 32g + l, so every lane accumulates its own row:
// no cross-lane reduction.
//
// Work decomposition. Grid = (row groups, K splits, activation-row slices).
// A CTA covers 32 rows x a contiguous range of kr blocks (a multiple of 16,
// i.e. of 512 K elements). The CTA's weights are therefore one contiguous run
// of bytes per array, which k_qgemv_tma streams into a ring of shared-memory
// stages (16 blocks each) with 1-D bulk TMA copies issued by a producer warp;
// the copies are issued before griddepcontrol.wait (weights never depend on
// the preceding kernel), so under programmatic dependent launch they overlap
// the tail of the kernel before. Eight consumer warps each take two blocks of
// a stage. Warp partials are summed in warp order through shared memory;
// when K is split across CTAs, the CTA partials go to scratch and the last
// CTA to arrive for a row group (atomic counter, reset by that CTA) sums them
// in K order. Results are deterministic.
//
// The plan keeps the whole grid resident in one wave: block formats at M = 1
// pair two row groups per CTA (sharing each activation block) only while two
// such CTAs fit on an SM, the ring depth (2-4 stages) is the deepest at which
// every CTA fits, and failing that K is split fewer times.
//
// The raw-layout Q4_0 GEMV (syn_q4_0_gemv, 18-byte blocks, 2-byte aligned)
// cannot be bulk-copied; k_qgemv streams it with direct loads instead.
//
// Activations (converted per CTA, only for its K range, in shared memory).
//   INT8 weights: per-row INT8 quantisation exactly as quantize.zig:12-47
//     (row max over all of K); W8A8 like QuantizedLinear::forward
//     (int8_linear.rs:87-117). Products are exact int32 per 512-element K
//     chunk, and the epilogue reproduces qmatmul.zig: float(acc) * sa * sb
//     for M <= 16 (one accumulator over K) and, for M > 16, C = 0; C +=
//     float(chunk) * sa * sb in chunk order (qmatmul.zig:68-98), every op
//     rounded.
//   Block formats: each 32-element block is scaled to 16-bit integers
//     (|xq| <= 32767, one f32 scale per block) and split into a signed high
//     byte and an unsigned low byte ("planes"), so every product runs as
//     exact 4-way integer dot products (dp4a) with exact block sums; the only
//     roundings are the 2^-16 relative activation quantisation and the f32
//     sums over blocks.
#include <algorithm>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "internal.cuh"

namespace syn {
namespace {

enum : int { F_INT8 = SYN_QFMT_INT8_KN, F_Q4_0 = SYN_QFMT_Q4_0, F_Q8_0 = SYN_QFMT_Q8_0,
             F_Q4_K = SYN_QFMT_Q4_K, F_Q6_K = SYN_QFMT_Q6_K, F_Q4_0RAW = 100 };

constexpr int WARPS = 8;              // consumer warps
constexpr int THREADS = WARPS * 32;   // consumer threads (named barrier 1)
constexpr int U = 4;                  // direct kernel: tiles in flight per warp
constexpr int SB = 16;                // blocks per stage (one 512-element chunk)

__host__ __device__ constexpr bool interleaved(int f) {
  return f == F_Q4_0 || f == F_Q4_K || f == F_Q6_K || f == F_Q4_0RAW;
}
__host__ __device__ constexpr bool eight_bit(int f) { return f == F_INT8 || f == F_Q8_0; }

// Shared-memory bytes of one activation block (one 32-element block of one
// activation row):
//   INT8  : 32 int8 codes.
//   blocks: 4 planes of 16 bytes -- interleaved formats: p0/p1 = high bytes
//           of even/odd elements, p2/p3 = low bytes (element 2i of a block
//           pairs with the low nibble of byte i); natural order (Q8_0):
//           p0/p1 = high bytes of elements 0-15 / 16-31, p2/p3 = low bytes --
//           then float2 sums (sum of xq over elements 0-15 / 16-31, exact),
//           f32 block scale, pad.
__host__ __device__ constexpr int act_block_bytes(int fmt) { return fmt == F_INT8 ? 32 : 80; }

// Stage layout (TMA kernel): per block of the stage, the 32-row tile of each
// array, in the same order as in HBM.
template <int FMT>
struct Stage {
  static constexpr int QT = eight_bit(FMT) ? 1024 : 512;                    // q tile
  static constexpr int DT = (FMT == F_Q4_0 || FMT == F_Q8_0) ? 64 : 0;      // d tile
  static constexpr int HT = (FMT == F_Q4_K) ? 512 : 0;   // header tile, per 8 blocks
  static constexpr int QHT = (FMT == F_Q6_K) ? 256 : 0;  // high-bit tile
  static constexpr int SCT = (FMT == F_Q6_K) ? 64 : 0;   // scale tile
  static constexpr int D6T = (FMT == F_Q6_K) ? 64 : 0;   // super-block scale tile, per 8
  static constexpr int OFF_D = SB * QT;
  static constexpr int OFF_H = OFF_D + SB * DT;
  static constexpr int OFF_QH = OFF_H + (SB / 8) * HT;
  static constexpr int OFF_SC = OFF_QH + SB * QHT;
  static constexpr int OFF_D6 = OFF_SC + SB * SCT;
  static constexpr int BYTES = (OFF_D6 + (SB / 8) * D6T + 127) / 128 * 128;
  static constexpr int NS = 6;                                   // deepest ring
  static constexpr int NS_WIDE = eight_bit(FMT) ? 3 : 4;         // grids of >= 1 CTA per SM
};

struct GemvParams {
  const uint8_t* q;
  const uint16_t* d;
  const float* sb;
  const uint8_t* hdr;
  const uint8_t* qh;
  const uint16_t* sc;
  const float* x;
  const int8_t* xq;
  const float* sx;
  long long ldx;
  int n, k, kp, nblk, nsb, groups;
  int kr, nks, nchunks;
  int m;
  float* y;
  long long ldy;
  int chunked;
  float* part;  // [m][nks or nchunks][groups*32]
  int* cnt;     // [m slices][groups]
  int* err;
  // optional fused prologue (M = 1): x = RMSNorm(nres (+ ndelta)) with weight
  // nw; the CTA at the grid origin stores nres + ndelta into nres_out
  const float* nres;
  const float* ndelta;
  const float* nw;
  float neps;
  float* nres_out;
  int nfast;  // 1: parallel sum of squares; 0: the reference's vecHsum order
  int xs_off; // byte offset of the normalised row in dynamic shared memory
  int ns;     // k_qgemv_tma ring depth
  // K split reduced through the thread-block cluster (1) instead of global
  // scratch (0): the nks CTAs of a row group form one cluster along y, and
  // rank 0 sums the others' partials from its shared memory (recv_off).
  int cluster;
  int recv_off;
  // SwiGLU epilogue (gate/up weights interleaved by 16 rows: group g holds
  // gate rows 16g.. in lanes 0-15 and the matching up rows in lanes 16-31):
  // lanes 0-15 write swiglu(gate, up) to sw_out[m * sw_ld + 16g + lane]
  // instead of y (ops/activation.rs:30-32 / silu.zig:85-110, variant as
  // launch_swiglu; sw_n = the FFN width).
  float* sw_out;
  long long sw_ld;
  int sw_n, sw_variant;
};

// Final store of output `row` of activation row m; called by all 32 lanes of
// a warp (valid = this lane's row exists).
__device__ __forceinline__ void store_y(const GemvParams& p, int m, int row, float out,
                                        bool valid) {
  if (!p.sw_out) {
    if (valid) p.y[(long long)m * p.ldy + row] = out;
    return;
  }
  const float up = __shfl_down_sync(0xffffffffu, out, 16);
  const int lane = threadIdx.x & 31;
  if (valid && lane < 16) {
    const int j = (row >> 5) * 16 + lane;
    p.sw_out[(long long)m * p.sw_ld + j] = swiglu_elem(out, up, j, p.sw_n & ~3, p.sw_variant);
  }
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

__device__ __forceinline__ void report(const GemvParams& p, int code) {
  if (p.err) atomicExch(p.err, code);
}

// ---------------------------------------------------------------------------
// Weight tiles
// ---------------------------------------------------------------------------
template <int FMT> struct WB;
template <> struct WB<F_INT8> { uint4 a, b; };
template <> struct WB<F_Q8_0> { uint4 a, b; uint32_t d; };
template <> struct WB<F_Q4_0> { uint4 a; uint32_t d; };
template <> struct WB<F_Q4_0RAW> { uint4 a; uint32_t d; };
template <> struct WB<F_Q4_K> { uint4 a; uint4 h; };
template <> struct WB<F_Q6_K> { uint4 a; uint2 qh; uint32_t sd; };

// Direct global load of block b of this lane's row (group g, lane l).
template <int FMT>
__device__ __forceinline__ void load_w(const GemvParams& p, int g, int b, int l, WB<FMT>& w) {
  const size_t t = ((size_t)g * p.nblk + b) * 32 + l;  // row-interleaved tile index
  if constexpr (FMT == F_INT8) {
    const uint8_t* src = p.q + (t >> 5) * 1024 + (t & 31) * 16;  // two half-planes
    w.a = ld_stream16(src);
    w.b = ld_stream16(src + 512);
  } else if constexpr (FMT == F_Q8_0) {
    const uint8_t* src = p.q + (t >> 5) * 1024 + (t & 31) * 16;
    w.a = ld_stream16(src);
    w.b = ld_stream16(src + 512);
    w.d = ld_nc_u16(p.d + t);
  } else if constexpr (FMT == F_Q4_0) {
    w.a = ld_stream16(p.q + t * 16);
    w.d = ld_nc_u16(p.d + t);
  } else if constexpr (FMT == F_Q4_K) {
    w.a = ld_stream16(p.q + t * 16);
    const size_t th = ((size_t)g * p.nsb + (b >> 3)) * 32 + l;
    w.h = __ldg(reinterpret_cast<const uint4*>(p.hdr + th * 16));
  } else if constexpr (FMT == F_Q6_K) {
    w.a = ld_stream16(p.q + t * 16);
    w.qh = ld_stream8(p.qh + t * 8);
    const size_t th = ((size_t)g * p.nsb + (b >> 3)) * 32 + l;
    w.sd = (uint32_t)ld_nc_u16(p.sc + t) | ((uint32_t)__ldg(p.d + th) << 16);
  } else {  // F_Q4_0RAW: reference 18-byte blocks of row 32g + l, 2-byte aligned
    const int row = g * 32 + l;
    if (row >= p.n) {
      w.a = make_uint4(0, 0, 0, 0);
      w.d = 0;
      return;
    }
    const uint16_t* src =
        reinterpret_cast<const uint16_t*>(p.q + ((size_t)row * p.nblk + b) * 18);
    uint32_t h[9];
#pragma unroll
    for (int i = 0; i < 9; i++) h[i] = __ldg(src + i);
    w.d = h[0];
    w.a = make_uint4(h[1] | (h[2] << 16), h[3] | (h[4] << 16), h[5] | (h[6] << 16),
                     h[7] | (h[8] << 16));
  }
}

// Block bl (0..15) of a stage in shared memory, this lane's row.
template <int FMT>
__device__ __forceinline__ void load_w_smem(const uint8_t* st, int bl, int l, WB<FMT>& w) {
  using S = Stage<FMT>;
  const int t = bl * 32 + l;
  if constexpr (eight_bit(FMT)) {
    const uint8_t* src = st + bl * 1024 + l * 16;
    w.a = *reinterpret_cast<const uint4*>(src);
    w.b = *reinterpret_cast<const uint4*>(src + 512);
    if constexpr (FMT == F_Q8_0) w.d = reinterpret_cast<const uint16_t*>(st + S::OFF_D)[t];
  } else {
    w.a = *reinterpret_cast<const uint4*>(st + t * 16);
    if constexpr (FMT == F_Q4_0) w.d = reinterpret_cast<const uint16_t*>(st + S::OFF_D)[t];
    if constexpr (FMT == F_Q4_K)
      w.h = reinterpret_cast<const uint4*>(st + S::OFF_H)[(bl >> 3) * 32 + l];
    if constexpr (FMT == F_Q6_K) {
      w.qh = reinterpret_cast<const uint2*>(st + S::OFF_QH)[t];
      w.sd = (uint32_t)reinterpret_cast<const uint16_t*>(st + S::OFF_SC)[t] |
             ((uint32_t)reinterpret_cast<const uint16_t*>(st + S::OFF_D6)[(bl >> 3) * 32 + l]
              << 16);
    }
  }
}

__device__ __forceinline__ uint32_t w4(const uint4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

struct AB {
  uint4 p0, p1, p2, p3;
  float2 sums;
  float s;
};

template <int FMT>
__device__ __forceinline__ void load_act(const uint8_t* blk, AB& a) {
  const uint4* v = reinterpret_cast<const uint4*>(blk);
  a.p0 = v[0];
  a.p1 = v[1];
  if constexpr (FMT != F_INT8) {
    a.p2 = v[2];
    a.p3 = v[3];
    const float4 t = reinterpret_cast<const float4*>(blk)[4];
    a.sums = make_float2(t.x, t.y);
    a.s = t.z;
  }
}

__device__ __forceinline__ int dot_int8(const WB<F_INT8>& w, const AB& a) {
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

// sum_i q_i * xq_i (exact, as float) for unsigned nibble codes q against
// interleaved planes: the high-plane and low-plane sums are each below 2^17.
__device__ __forceinline__ float dot_nib(const uint4& q, const AB& a) {
  int hl = 0, hh = 0, ll = 0, lh = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint32_t wq = w4(q, j);
    const uint32_t lo = wq & 0x0F0F0F0Fu;
    const uint32_t hi16 = wq & 0xF0F0F0F0u;  // 16 * high nibble; exact after >> 4
    hl = dp4a_su(w4(a.p0, j), lo, hl);
    hh = dp4a_su(w4(a.p1, j), hi16, hh);
    ll = dp4a_uu(w4(a.p2, j), lo, ll);
    lh = dp4a_uu(w4(a.p3, j), hi16, lh);
  }
  return fmaf(256.0f, i2f_small(hl + (hh >> 4)), i2f_small(ll + (lh >> 4)));
}

template <int FMT>
__device__ __forceinline__ float dot_block(const WB<FMT>& w, const AB& a, int b) {
  if constexpr (FMT == F_Q4_0 || FMT == F_Q4_0RAW) {
    // gguf.rs:318-324 / qmatmul.zig:306-311: value = (nib - 8) * d
    const float iq = dot_nib(w.a, a) - 8.0f * (a.sums.x + a.sums.y);
    const float d = (FMT == F_Q4_0) ? f16_loader((uint16_t)w.d) : f16_exact((uint16_t)w.d);
    return iq * (a.s * d);
  } else if constexpr (FMT == F_Q8_0) {
    // gguf.rs:276-285: value = d * q
    int ih = 0, il = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      ih = dp4a_ss(w4(a.p0, j), w4(w.a, j), ih);
      ih = dp4a_ss(w4(a.p1, j), w4(w.b, j), ih);
      il = dp4a_us(w4(a.p2, j), w4(w.a, j), il);
      il = dp4a_us(w4(a.p3, j), w4(w.b, j), il);
    }
    const float iq = fmaf(256.0f, i2f_small(ih), i2f_small(il));
    return iq * (a.s * f16_loader((uint16_t)w.d));
  } else if constexpr (FMT == F_Q4_K) {
    // gguf.rs:400-427: 6-bit scale/min unpack for sub-block s; value =
    // q * (d * scale_s) - dmin * min_s, so the block contributes
    // sc * sum(q xq) - m * sum(xq), times the activation block scale.
    const int s = b & 7;
    const uint32_t y = w.h.y, z = w.h.z, wv = w.h.w;
    const float dd = f16_loader((uint16_t)(w.h.x & 0xFFFF));
    const float dmin = f16_loader((uint16_t)(w.h.x >> 16));
    uint32_t scv, mnv;
    if (s < 4) {
      const int sh = 8 * s;
      scv = (y >> sh) & 0x3F;
      mnv = (((z >> sh) & 0xFF) >> 4) | (((wv >> sh) & 0x0F) << 4);
    } else {
      const int sh = 8 * (s - 4);
      const uint32_t ys = (y >> sh) & 0xFF;
      scv = ((z >> sh) & 0x0F) | ((ys >> 6) << 4);
      mnv = (((wv >> sh) & 0xFF) >> 4) | (((ys >> 4) & 0x0C) << 4);
    }
    const float iq = dot_nib(w.a, a);
    return a.s * ((dd * (float)scv) * iq - (dmin * (float)mnv) * (a.sums.x + a.sums.y));
  } else {  // F_Q6_K, gguf.rs:462-483: value = (q6 - 32) * (sc * d)
    int h0 = 0, l0 = 0, h1 = 0, l1 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t wq = w4(w.a, j);
      const uint32_t H = (j < 2) ? w.qh.x : w.qh.y;
      const uint32_t he = (j & 1) ? (H & 0x30303030u) : ((H << 4) & 0x30303030u);
      const uint32_t ho = (j & 1) ? ((H >> 2) & 0x30303030u) : ((H << 2) & 0x30303030u);
      const uint32_t qe = (wq & 0x0F0F0F0Fu) | he;
      const uint32_t qo = ((wq >> 4) & 0x0F0F0F0Fu) | ho;
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
    const float i0 = fmaf(256.0f, i2f_small(h0), i2f_small(l0)) - 32.0f * a.sums.x;
    const float i1 = fmaf(256.0f, i2f_small(h1), i2f_small(l1)) - 32.0f * a.sums.y;
    const float dd = f16_loader((uint16_t)(w.sd >> 16));
    const float sc0 = (float)(int8_t)(w.sd & 0xFF) * dd;
    const float sc1 = (float)(int8_t)((w.sd >> 8) & 0xFF) * dd;
    return a.s * (i0 * sc0 + i1 * sc1);
  }
}

// ---------------------------------------------------------------------------
// Activation conversion (per warp, over the warp's share [wb0, wb1) of the
// CTA's blocks).
// ---------------------------------------------------------------------------
// Two lanes per block: lane half h = lane & 1 quantises elements
// [16h, 16h + 16) of block b. The block max takes one shuffle; each half's
// code sum is its own (sums[h]), so no other cross-lane step is needed.
template <int FMT>
__device__ void prep_blocks(const float* xr, bool live, int wb0, int wb1, uint8_t* act, int cb0) {
  const int lane = threadIdx.x & 31;
  const int h = lane & 1;
  constexpr int PF = 2;  // 16-block iterations whose loads are issued together
  for (int base = wb0; base < wb1; base += 16 * PF) {
    float4 vv[PF][4];
#pragma unroll
    for (int u = 0; u < PF; u++) {
      const int b = base + 16 * u + (lane >> 1);
#pragma unroll
      for (int e = 0; e < 4; e++) {
        vv[u][e] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live && b < wb1)
          vv[u][e] = *reinterpret_cast<const float4*>(xr + (size_t)b * 32 + 16 * h + 4 * e);
      }
    }
#pragma unroll
    for (int u = 0; u < PF; u++) {
      if (base + 16 * u >= wb1) break;  // uniform across the warp
      const int b = base + 16 * u + (lane >> 1);
      float v[16];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        v[4 * e] = vv[u][e].x;
        v[4 * e + 1] = vv[u][e].y;
        v[4 * e + 2] = vv[u][e].z;
        v[4 * e + 3] = vv[u][e].w;
      }
      float amax = 0.0f;
#pragma unroll
      for (int e = 0; e < 16; e++) amax = fmaxf(amax, fabsf(v[e]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      int q[16];
      int ssum = 0;
      const float inv = amax > 0.0f ? 32767.0f * __frcp_rn(amax) : 0.0f;
#pragma unroll
      for (int e = 0; e < 16; e++) {
        q[e] = max(-32767, min(32767, __float2int_rn(v[e] * inv)));
        ssum += q[e];
      }
      if (b >= wb1) continue;
      uint8_t* blk = act + (size_t)(b - cb0) * act_block_bytes(FMT);
      // byte 1 (signed high byte) or byte 0 (unsigned low byte) of four codes
      auto hi4 = [](int a, int b2, int c, int d) {
        return __byte_perm(__byte_perm(a, b2, 0x0051), __byte_perm(c, d, 0x0051), 0x5410);
      };
      auto lo4 = [](int a, int b2, int c, int d) {
        return __byte_perm(__byte_perm(a, b2, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
      };
      if constexpr (interleaved(FMT)) {
        // element 16h + j sits in the even (j even) or odd plane at byte
        // 8h + j/2: this lane fills words 2h, 2h + 1 of each plane
        const uint2 he = make_uint2(hi4(q[0], q[2], q[4], q[6]), hi4(q[8], q[10], q[12], q[14]));
        const uint2 ho = make_uint2(hi4(q[1], q[3], q[5], q[7]), hi4(q[9], q[11], q[13], q[15]));
        const uint2 le = make_uint2(lo4(q[0], q[2], q[4], q[6]), lo4(q[8], q[10], q[12], q[14]));
        const uint2 lo = make_uint2(lo4(q[1], q[3], q[5], q[7]), lo4(q[9], q[11], q[13], q[15]));
        *reinterpret_cast<uint2*>(blk + 0 + 8 * h) = he;
        *reinterpret_cast<uint2*>(blk + 16 + 8 * h) = ho;
        *reinterpret_cast<uint2*>(blk + 32 + 8 * h) = le;
        *reinterpret_cast<uint2*>(blk + 48 + 8 * h) = lo;
      } else {
        // natural order: plane h (high bytes) and plane 2 + h (low bytes)
        *reinterpret_cast<uint4*>(blk + 16 * h) =
            make_uint4(hi4(q[0], q[1], q[2], q[3]), hi4(q[4], q[5], q[6], q[7]),
                       hi4(q[8], q[9], q[10], q[11]), hi4(q[12], q[13], q[14], q[15]));
        *reinterpret_cast<uint4*>(blk + 32 + 16 * h) =
            make_uint4(lo4(q[0], q[1], q[2], q[3]), lo4(q[4], q[5], q[6], q[7]),
                       lo4(q[8], q[9], q[10], q[11]), lo4(q[12], q[13], q[14], q[15]));
      }
      float* tail = reinterpret_cast<float*>(blk + 64);
      tail[h] = (float)ssum;
      if (h == 0) tail[2] = amax > 0.0f ? amax * (1.0f / 32767.0f) : 0.0f;
    }
  }
}

// INT8: codes of the warp's blocks, given the row's 127/max factor.
__device__ void prep_int8(const GemvParams& p, int m, bool live, float inv, bool zero_row, int wb0,
                          int wb1, uint8_t* act, int cb0) {
  const int lane = threadIdx.x & 31;
  for (int b0 = wb0; b0 < wb1; b0 += 4) {
    const int b = b0 + (lane >> 3), j = lane & 7;
    if (b >= wb1) continue;
    uint32_t word = 0;
    if (live && !zero_row) {
      if (p.xq) {
        const int8_t* src = p.xq + (long long)m * p.ldx + (size_t)b * 32 + 4 * j;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int kk = b * 32 + 4 * j + e;
          const uint32_t v = kk < p.k ? (uint8_t)src[e] : 0u;
          word |= v << (8 * e);
        }
      } else {
        const float* src = p.x + (long long)m * p.ldx + (size_t)b * 32 + 4 * j;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int kk = b * 32 + 4 * j + e;
          int8_t v = 0;
          if (kk < p.k) {
            float r = roundf(__fmul_rn(src[e], inv));
            r = fminf(127.0f, fmaxf(-127.0f, r));
            v = (int8_t)(int)r;
          }
          word |= (uint32_t)(uint8_t)v << (8 * e);
        }
      }
    }
    reinterpret_cast<uint32_t*>(act + (size_t)(b - cb0) * 32)[j] = word;
  }
}

template <int MT>
struct CtaShared {
  float red[WARPS][MT][32];
  float srow[MT];  // INT8: per-row activation scale sa
  float sinv[MT];  // INT8: 127 / max (0 for an all-zero row)
  int slast;
  uint64_t rbar;   // cluster K split: the peers' partials have arrived (rank 0)
};

// Converts the CTA's activation blocks [cb0, cb1) of MT rows into `act`
// (consumer threads only; ends with a consumer barrier). INT8 also zeroes
// the chunk sums `csum` ([MT][ncc][32]).
template <int FMT, int MT>
__device__ void cta_prologue(const GemvParams& p, int m0, int cb0, int cb1, uint8_t* act,
                             int* csum, int ncc, CtaShared<MT>& sh) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = (cb1 - cb0 + WARPS - 1) / WARPS;
  const int wb0 = min(cb1, cb0 + warp * per), wb1 = min(cb1, wb0 + per);
  const int act_stride = p.kr * act_block_bytes(FMT);
  if constexpr (FMT == F_INT8) {
    for (int i = threadIdx.x; i < MT * ncc * 32; i += THREADS) csum[i] = 0;
    constexpr int XR = 16;  // x values per thread held in registers
    const int k0 = cb0 * 32, k1 = min(cb1 * 32, p.kp);
    if (MT == 1 && !p.xq && m0 < p.m && k1 - k0 <= XR * THREADS) {
      // one pass over x: the row max spans all of K (quantize.zig:12-47), so
      // this CTA's elements are kept in registers while it is reduced
      const float* xr = p.x + (long long)m0 * p.ldx;
      float xv[XR];
      float amax = 0.0f;
#pragma unroll
      for (int u = 0; u < XR; u++) {
        const int kk = k0 + threadIdx.x + u * THREADS;
        xv[u] = kk < k1 && kk < p.k ? xr[kk] : 0.0f;
        amax = fmaxf(amax, fabsf(xv[u]));
      }
      const bool whole = k0 == 0 && k1 >= p.k;
      if (!whole)  // the max also spans the elements outside this CTA's range
        for (int i = threadIdx.x; i < p.k; i += THREADS)
          if (i < k0 || i >= k1) amax = fmaxf(amax, fabsf(xr[i]));
      amax = warp_max(amax);
      if (lane == 0) sh.red[warp][0][0] = amax;
      consumer_sync();
      float a = sh.red[0][0][0];
#pragma unroll
      for (int i = 1; i < WARPS; i++) a = fmaxf(a, sh.red[i][0][0]);
      if (threadIdx.x == 0) sh.srow[0] = (a == 0.0f) ? 1.0f : __fdiv_rn(a, 127.0f);
      const float inv = (a == 0.0f) ? 0.0f : __fdiv_rn(127.0f, a);
      int8_t* codes = reinterpret_cast<int8_t*>(act) - k0;
#pragma unroll
      for (int u = 0; u < XR; u++) {
        const int kk = k0 + threadIdx.x + u * THREADS;
        if (kk < k1) {
          int8_t v = 0;
          if (a != 0.0f && kk < p.k) {
            float r = roundf(__fmul_rn(xv[u], inv));
            r = fminf(127.0f, fmaxf(-127.0f, r));
            v = (int8_t)(int)r;
          }
          codes[kk] = v;
        }
      }
      consumer_sync();
      return;
    }
    for (int mm = 0; mm < MT; mm++) {
      const int m = m0 + mm;
      if (m >= p.m) continue;  // uniform across the CTA
      if (p.xq) {
        if (threadIdx.x == 0) sh.srow[mm] = p.sx[m];
        continue;
      }
      // quantize.zig:12-47: the row max spans all of K
      const float* xr = p.x + (long long)m * p.ldx;
      float amax = 0.0f;
      for (int i = threadIdx.x; i < p.k; i += THREADS) amax = fmaxf(amax, fabsf(xr[i]));
      amax = warp_max(amax);
      if (lane == 0) sh.red[warp][mm][0] = amax;
      consumer_sync();
      if (threadIdx.x == 0) {
        float a = sh.red[0][mm][0];
        for (int i = 1; i < WARPS; i++) a = fmaxf(a, sh.red[i][mm][0]);
        sh.srow[mm] = (a == 0.0f) ? 1.0f : __fdiv_rn(a, 127.0f);
        sh.sinv[mm] = (a == 0.0f) ? 0.0f : __fdiv_rn(127.0f, a);
      }
      consumer_sync();
    }
    consumer_sync();
    for (int mm = 0; mm < MT; mm++) {
      const int m = m0 + mm;
      const bool live = m < p.m;
      const float inv = (live && !p.xq) ? sh.sinv[mm] : 0.0f;
      prep_int8(p, m, live, inv, live && !p.xq && inv == 0.0f, wb0, wb1, act + mm * act_stride,
                cb0);
    }
  } else {
    for (int mm = 0; mm < MT; mm++) {
      const int m = m0 + mm;
      prep_blocks<FMT>(p.x + (long long)(m < p.m ? m : 0) * p.ldx, m < p.m, wb0, wb1,
                       act + mm * act_stride, cb0);
    }
  }
  consumer_sync();
}

// Reduces the CTA's warp partials (block formats: sh.red; INT8: csum) and
// writes y or, with K split across CTAs, the CTA partials plus the ordered
// final sum by the last CTA of the row group. Consumer threads only.
// Cluster K split (p.cluster): every CTA of the row group's cluster (rank =
// ks) stores its partials into rank 0's shared memory -- block formats
// recv[ks][mm][lane] (f32); INT8 the exact int32 sum of its chunks
// recv[ks][mm][lane], or with the chunked epilogue every chunk's sum
// recv[mm][chunk][lane] -- and arrives on rank 0's mbarrier; rank 0 waits
// (bounded) and sums them in K order, as the global-scratch path does: the
// same bits, without the scratch round trips through L2.
template <int FMT, int MT>
__device__ void cluster_finish(const GemvParams& p, int g, int ks, int m0, int cc0, int ncc,
                               const int* csum, CtaShared<MT>& sh, float sb_pre, bool have_sb) {
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* recv = dsm + p.recv_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = g * 32 + lane;
  cluster_wait();  // every peer has initialised its barrier and buffers
  if (warp < MT && m0 + warp < p.m) {
    const int mm = warp;
    if constexpr (FMT == F_INT8) {
      if (MT > 1 && p.chunked) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(recv) + ((size_t)mm * p.nchunks + cc0) * 32 + lane;
        for (int c = 0; c < ncc; c++) {
          const uint32_t v = (uint32_t)csum[(mm * ncc + c) * 32 + lane];
          if (ks == 0) dst[c * 32] = v;
          else st_cluster_u32(cluster_map(dst + c * 32, 0), v);
        }
      } else {
        int t = 0;
        for (int c = 0; c < ncc; c++) t += csum[(mm * ncc + c) * 32 + lane];
        uint32_t* dst = reinterpret_cast<uint32_t*>(recv) + ((size_t)ks * MT + mm) * 32 + lane;
        if (ks == 0) *dst = (uint32_t)t;
        else st_cluster_u32(cluster_map(dst, 0), (uint32_t)t);
      }
    } else {
      float v = 0.0f;
#pragma unroll
      for (int i = 0; i < WARPS; i++) v += sh.red[i][mm][lane];
      float* dst = reinterpret_cast<float*>(recv) + ((size_t)ks * MT + mm) * 32 + lane;
      if (ks == 0) *dst = v;
      else st_cluster_u32(cluster_map(dst, 0), __float_as_uint(v));
    }
  }
  if (ks != 0) {
    fence_acq_rel_cluster();
    consumer_sync();
    if (threadIdx.x == 0) mbar_arrive_remote(cluster_map(&sh.rbar, 0));
    return;
  }
  if (threadIdx.x == 0 && !mbar_wait_cluster_bounded(&sh.rbar, 0)) report(p, SYN_ERR_TIMEOUT);
  consumer_sync();
  if (warp < MT) {
    const int mm = warp, m = m0 + mm;
    if (m < p.m) {
      float out = 0.0f;
      if (row >= p.n) {
      } else if constexpr (FMT == F_INT8) {
        const float sa = sh.srow[mm], sbv = have_sb ? sb_pre : p.sb[row];
        if (MT > 1 && p.chunked) {
          const int* src = reinterpret_cast<const int*>(recv) + (size_t)mm * p.nchunks * 32 + lane;
          for (int c = 0; c < p.nchunks; c++)
            out = __fadd_rn(out, __fmul_rn(__fmul_rn((float)src[c * 32], sa), sbv));
        } else {
          const int* src = reinterpret_cast<const int*>(recv) + (size_t)mm * 32 + lane;
          int tot = 0;
          for (int s = 0; s < p.nks; s++) tot += src[(size_t)s * MT * 32];
          out = __fmul_rn(__fmul_rn((float)tot, sa), sbv);
        }
      } else {
        const float* src = reinterpret_cast<const float*>(recv) + (size_t)mm * 32 + lane;
        for (int s = 0; s < p.nks; s++) out += src[(size_t)s * MT * 32];
      }
      store_y(p, m, row, out, row < p.n);
    }
  }
}

// CL: the kernel may be launched as clusters (k_qgemv_tma with one row group
// per CTA; row-group pairs only run unsplit).
template <int FMT, int MT, bool CL = false>
__device__ void cta_finish(const GemvParams& p, int g, int ks, int m0, int cc0, int ncc,
                           const int* csum, CtaShared<MT>& sh, float sb_pre = 0.0f,
                           bool have_sb = false) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = g * 32 + lane;
  const bool split = p.nks > 1;
  const long long G32 = (long long)p.groups * 32;
  consumer_sync();
  // (not compiled for the one-row INT8 kernel: it would cost that kernel
  // 16 registers and a CTA per SM; its K splits reduce through scratch)
  if constexpr (CL && !(FMT == F_INT8 && MT == 1)) {
    if (split && p.cluster) {
      cluster_finish<FMT, MT>(p, g, ks, m0, cc0, ncc, csum, sh, sb_pre, have_sb);
      return;
    }
  }
  if (warp < MT) {
    const int mm = warp, m = m0 + mm;
    if (m < p.m) {
      if constexpr (FMT == F_INT8) {
        if (!split) {
          float out = 0.0f;
          if (row < p.n) {
            const float sa = sh.srow[mm], sbv = have_sb ? sb_pre : p.sb[row];
            if (p.chunked) {
              for (int c = 0; c < ncc; c++)
                out = __fadd_rn(
                    out, __fmul_rn(__fmul_rn((float)csum[(mm * ncc + c) * 32 + lane], sa), sbv));
            } else {
              int tot = 0;
              for (int c = 0; c < ncc; c++) tot += csum[(mm * ncc + c) * 32 + lane];
              out = __fmul_rn(__fmul_rn((float)tot, sa), sbv);
            }
          }
          store_y(p, m, row, out, row < p.n);
        } else {
          float* dst = p.part + (long long)m * p.nchunks * G32;
          for (int c = 0; c < ncc; c++)
            dst[(long long)(cc0 + c) * G32 + row] = __int_as_float(csum[(mm * ncc + c) * 32 + lane]);
        }
      } else {
        float v = 0.0f;
#pragma unroll
        for (int i = 0; i < WARPS; i++) v += sh.red[i][mm][lane];
        if (!split) {
          store_y(p, m, row, v, row < p.n);
        } else {
          p.part[((long long)m * p.nks + ks) * G32 + row] = v;
        }
      }
    }
  }
  if (!split) return;

  // split K: the last CTA of this row group sums the partials in K order
  __threadfence();
  consumer_sync();
  if (threadIdx.x == 0) {
    int* c = p.cnt + (long long)blockIdx.z * p.groups + g;
    const int arrived = atomicAdd(c, 1);
    sh.slast = (arrived == p.nks - 1);
    if (sh.slast) *c = 0;  // self-reset for the next launch
  }
  consumer_sync();
  if (!sh.slast) return;
  __threadfence();
  if (warp < MT) {
    const int mm = warp, m = m0 + mm;
    if (m < p.m) {
      float out = 0.0f;
      if (row >= p.n) {
      } else if constexpr (FMT == F_INT8) {
        const float* src = p.part + (long long)m * p.nchunks * G32;
        const float sa = sh.srow[mm], sbv = have_sb ? sb_pre : p.sb[row];
        if (p.chunked) {
          for (int c = 0; c < p.nchunks; c++) {
            const int cv = __float_as_int(__ldcg(src + c * G32 + row));
            out = __fadd_rn(out, __fmul_rn(__fmul_rn((float)cv, sa), sbv));
          }
        } else {
          int tot = 0;
          for (int c = 0; c < p.nchunks; c++) tot += __float_as_int(__ldcg(src + c * G32 + row));
          out = __fmul_rn(__fmul_rn((float)tot, sa), sbv);
        }
      } else {
        const float* src = p.part + (long long)m * p.nks * G32;
        for (int s = 0; s < p.nks; s++) out += __ldcg(src + s * G32 + row);
      }
      store_y(p, m, row, out, row < p.n);
    }
  }
}

// Fused RMSNorm prologue (consumer threads): xs[0, k) = (v * w) * scale with
// v = nres (+ ndelta) and scale = 1 / sqrt(sum(v*v)/k + eps), the sum in the
// reference's vecHsum order (four lanes of stride 4, lanes in order, tail)
// or, with nfast, in a parallel order. Same arithmetic as k_add_rmsnorm.
constexpr int NW_PRE = 16;  // norm weights per thread held in registers (k <= 4096)

template <int MT>
__device__ void norm_prologue(const GemvParams& p, float* xs, CtaShared<MT>& sh,
                              const float (&nwp)[NW_PRE]) {
  const int tid = threadIdx.x, k = p.k;
  const bool origin = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  for (int j0 = 0; j0 < k; j0 += THREADS * 4) {
    float v[4], dl[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int j = j0 + tid + u * THREADS;
      v[u] = j < k ? p.nres[j] : 0.0f;
      dl[u] = (j < k && p.ndelta) ? p.ndelta[j] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int j = j0 + tid + u * THREADS;
      if (j < k) {
        const float x = p.ndelta ? __fadd_rn(v[u], dl[u]) : v[u];
        xs[j] = x;
        if (origin && p.nres_out) p.nres_out[j] = x;
      }
    }
  }
  consumer_sync();
  float* lanes = &sh.red[0][0][0];
  if (p.nfast) {
    float a = 0.0f;
    for (int j = tid; j < k; j += THREADS) a = fmaf(xs[j], xs[j], a);
    a = warp_sum(a);
    if ((tid & 31) == 0) lanes[8 + (tid >> 5)] = a;
    consumer_sync();
    if (tid == 0) {
      float t = 0.0f;
      for (int w = 0; w < WARPS; w++) t += lanes[8 + w];
      lanes[16] = 1.0f / sqrtf(t / (float)k + p.neps);
    }
  } else {
    if (tid < 4) {
      const int n4 = k & ~3;
      float acc = 0.0f;
      int i = tid;
      for (; i + 60 < n4; i += 64) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; u++) v[u] = xs[i + 4 * u];
#pragma unroll
        for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(v[u], v[u]));
      }
      for (; i < n4; i += 4) acc = __fadd_rn(acc, __fmul_rn(xs[i], xs[i]));
      lanes[tid] = acc;
    }
    consumer_sync();
    if (tid == 0) {
      float t = __fadd_rn(__fadd_rn(__fadd_rn(lanes[0], lanes[1]), lanes[2]), lanes[3]);
      for (int i = k & ~3; i < k; i++) t = __fadd_rn(t, __fmul_rn(xs[i], xs[i]));
      lanes[16] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)k), p.neps)));
    }
  }
  consumer_sync();
  const float scale = lanes[16];
  if (k <= NW_PRE * THREADS) {
#pragma unroll
    for (int u = 0; u < NW_PRE; u++) {
      const int j = tid + u * THREADS;
      if (j < k) xs[j] = __fmul_rn(__fmul_rn(xs[j], nwp[u]), scale);
    }
  } else {
    for (int j = tid; j < k; j += THREADS) xs[j] = __fmul_rn(__fmul_rn(xs[j], p.nw[j]), scale);
  }
  consumer_sync();
}

// ---------------------------------------------------------------------------
// k_qgemv_tma: repacked formats; weights through a TMA-filled smem ring.
// Threads 0-255 consume, warp 8 (threads 256-287) produces.
// ---------------------------------------------------------------------------
template <int FMT, int MT, int RG>
__global__ void __launch_bounds__(THREADS + 32) k_qgemv_tma(const GemvParams p) {
  using S = Stage<FMT>;
  static_assert(RG == 1 || (FMT != F_INT8 && MT == 1), "row-group pairs: block formats, M=1");
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[S::NS], empty[S::NS];
  __shared__ CtaShared<MT> sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // RG row groups per CTA: their stages share the activation blocks
  const int g = blockIdx.x * RG, ks = blockIdx.y, m0 = blockIdx.z * MT;
  const int ng = min(RG, p.groups - g);
  const int cb0 = ks * p.kr, cb1 = min(p.nblk, cb0 + p.kr);
  const int nst = (cb1 - cb0 + SB - 1) / SB;
  constexpr int SBYTES = RG * S::BYTES;  // one stage: RG sub-stages
  uint8_t* ring = sm;
  const int ns = p.ns;  // ring depth, <= S::NS (chosen by the plan for occupancy)
  uint8_t* act = sm + ns * SBYTES;
  const int act_stride = p.kr * act_block_bytes(FMT);
  const int cc0 = cb0 >> 4, ncc = ((cb1 + 15) >> 4) - cc0;
  int* csum = reinterpret_cast<int*>(act + MT * act_stride);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], WARPS);
    }
    if (p.cluster) mbar_init(&sh.rbar, p.nks - 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (p.cluster) cluster_arrive_relaxed();  // all threads, before the producer leaves

  if (warp == WARPS) {
    // ---- producer: stream this CTA's weight bytes, stage by stage ----
    griddep_launch();
    if (lane == 0) {
      for (int s = 0, slot = 0, round = 0; s < nst; s++) {
        if (s > 0 && ++slot == ns) {
          slot = 0;
          round++;
        }
        if (round > 0 && !mbar_wait_bounded(&empty[slot], (round - 1) & 1)) {
          report(p, SYN_ERR_TIMEOUT);
          break;
        }
        const int b0 = cb0 + s * SB, nbs = min(SB, cb1 - b0);
        const uint32_t bytes = nbs * S::QT + nbs * S::DT + (nbs / 8) * S::HT + nbs * S::QHT +
                               nbs * S::SCT + (nbs / 8) * S::D6T;
        mbar_expect_tx(&full[slot], bytes * ng);
        for (int r = 0; r < ng; r++) {
        const size_t tile0 = (size_t)(g + r) * p.nblk;  // first tile of this row group
        const size_t stile0 = (size_t)(g + r) * p.nsb;  // first super-block tile
        uint8_t* st = ring + slot * SBYTES + r * S::BYTES;
        bulk_g2s(st, p.q + (tile0 + b0) * S::QT, nbs * S::QT, &full[slot]);
        if constexpr (S::DT)
          bulk_g2s(st + S::OFF_D, reinterpret_cast<const uint8_t*>(p.d) + (tile0 + b0) * 64,
                   nbs * 64, &full[slot]);
        if constexpr (S::HT)
          bulk_g2s(st + S::OFF_H, p.hdr + (stile0 + b0 / 8) * 512, (nbs / 8) * 512, &full[slot]);
        if constexpr (S::QHT) {
          bulk_g2s(st + S::OFF_QH, p.qh + (tile0 + b0) * 256, nbs * 256, &full[slot]);
          bulk_g2s(st + S::OFF_SC, reinterpret_cast<const uint8_t*>(p.sc) + (tile0 + b0) * 64,
                   nbs * 64, &full[slot]);
          bulk_g2s(st + S::OFF_D6, reinterpret_cast<const uint8_t*>(p.d) + (stile0 + b0 / 8) * 64,
                   (nbs / 8) * 64, &full[slot]);
        }
        }
      }
    }
    return;
  }

  // ---- consumers ----
  // Constants of the weight (per-row INT8 scales, the fused norm's weights)
  // are read before griddepcontrol.wait: they do not depend on the
  // preceding kernel, so their latency overlaps it.
  float sb_pre[RG];
#pragma unroll
  for (int r = 0; r < RG; r++) {
    const int row = (g + r) * 32 + lane;
    sb_pre[r] = (FMT == F_INT8 && r < ng && row < p.n) ? p.sb[row] : 0.0f;
  }
  float nwp[NW_PRE];
  if (p.nw && p.k <= NW_PRE * THREADS) {
#pragma unroll
    for (int u = 0; u < NW_PRE; u++) {
      const int j = threadIdx.x + u * THREADS;
      nwp[u] = j < p.k ? p.nw[j] : 0.0f;
    }
  }
  griddep_wait();  // x may be written by the preceding kernel
  griddep_launch();
  if (p.nw) {  // fused RMSNorm (M = 1): the normalised row becomes x
    float* xs = reinterpret_cast<float*>(sm + p.xs_off);
    norm_prologue<MT>(p, xs, sh, nwp);
    GemvParams q = p;
    q.x = xs;
    q.ldx = 0;
    cta_prologue<FMT, MT>(q, m0, cb0, cb1, act, csum, ncc, sh);
  } else {
    cta_prologue<FMT, MT>(p, m0, cb0, cb1, act, csum, ncc, sh);
  }

  float facc[MT][RG];
#pragma unroll
  for (int mm = 0; mm < MT; mm++)
#pragma unroll
    for (int r = 0; r < RG; r++) facc[mm][r] = 0.0f;
  for (int s = 0, slot = 0, round = 0; s < nst; s++) {
    if (s > 0 && ++slot == ns) {
      slot = 0;
      round++;
    }
    const bool ok = mbar_wait_bounded(&full[slot], round & 1);
    if (!ok && lane == 0) report(p, SYN_ERR_TIMEOUT);
    const int b0 = cb0 + s * SB, nbs = min(SB, cb1 - b0);
    const uint8_t* st = ring + slot * SBYTES;
    int ich[MT];
#pragma unroll
    for (int mm = 0; mm < MT; mm++) ich[mm] = 0;
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int bl = warp * 2 + u;
      if (!ok || bl >= nbs) break;
      WB<FMT> w[RG];
#pragma unroll
      for (int r = 0; r < RG; r++)
        if (r < ng) load_w_smem<FMT>(st + r * S::BYTES, bl, lane, w[r]);
#pragma unroll
      for (int mm = 0; mm < MT; mm++) {
        AB a;
        load_act<FMT>(act + mm * act_stride + (b0 + bl - cb0) * act_block_bytes(FMT), a);
        if constexpr (FMT == F_INT8) {
          ich[mm] += dot_int8(w[0], a);
        } else {
#pragma unroll
          for (int r = 0; r < RG; r++)
            if (r < ng) facc[mm][r] += dot_block<FMT>(w[r], a, b0 + bl);
        }
      }
    }
    if constexpr (FMT == F_INT8) {
      // one stage = one 512-element chunk (stages start on chunk boundaries)
#pragma unroll
      for (int mm = 0; mm < MT; mm++)
        if (warp * 2 < nbs) atomicAdd(&csum[(mm * ncc + (b0 >> 4) - cc0) * 32 + lane], ich[mm]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
#pragma unroll
  for (int r = 0; r < RG; r++) {
    if (r >= ng) break;
    consumer_sync();  // the previous group's finish has read sh.red
    if constexpr (FMT != F_INT8) {
#pragma unroll
      for (int mm = 0; mm < MT; mm++) sh.red[warp][mm][lane] = facc[mm][r];
    }
    cta_finish<FMT, MT, RG == 1>(p, g + r, ks, m0, cc0, ncc, csum, sh, sb_pre[r], FMT == F_INT8);
  }
}

// ---------------------------------------------------------------------------
// k_qgemv: direct global loads (the raw 18-byte Q4_0 layout).
// ---------------------------------------------------------------------------
template <int FMT, int MT>
__global__ void __launch_bounds__(THREADS) k_qgemv(const GemvParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ CtaShared<MT> sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x, ks = blockIdx.y, m0 = blockIdx.z * MT;
  const int cb0 = ks * p.kr, cb1 = min(p.nblk, cb0 + p.kr);
  const int per = (cb1 - cb0 + WARPS - 1) / WARPS;
  const int wb0 = min(cb1, cb0 + warp * per), wb1 = min(cb1, wb0 + per);
  const int act_stride = p.kr * act_block_bytes(FMT);
  const int cc0 = cb0 >> 4, ncc = ((cb1 + 15) >> 4) - cc0;
  int* csum = reinterpret_cast<int*>(sm + MT * act_stride);

  // First tiles: independent of the preceding kernel.
  WB<FMT> w[U];
#pragma unroll
  for (int u = 0; u < U; u++)
    if (wb0 + u < wb1) load_w<FMT>(p, g, wb0 + u, lane, w[u]);

  griddep_wait();  // x may be written by the preceding kernel
  griddep_launch();
  cta_prologue<FMT, MT>(p, m0, cb0, cb1, sm, csum, ncc, sh);

  float facc[MT];
  int ich[MT];
#pragma unroll
  for (int mm = 0; mm < MT; mm++) {
    facc[mm] = 0.0f;
    ich[mm] = 0;
  }
  int cur_chunk = wb0 >> 4;
  for (int b0 = wb0; b0 < wb1; b0 += U) {
    if (b0 != wb0) {
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b0 + u < wb1) load_w<FMT>(p, g, b0 + u, lane, w[u]);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int b = b0 + u;
      if (b >= wb1) break;
      if constexpr (FMT == F_INT8) {
        if ((b >> 4) != cur_chunk) {  // flush the finished 512-element chunk
#pragma unroll
          for (int mm = 0; mm < MT; mm++) {
            atomicAdd(&csum[(mm * ncc + cur_chunk - cc0) * 32 + lane], ich[mm]);
            ich[mm] = 0;
          }
          cur_chunk = b >> 4;
        }
      }
#pragma unroll
      for (int mm = 0; mm < MT; mm++) {
        AB a;
        load_act<FMT>(sm + mm * act_stride + (b - cb0) * act_block_bytes(FMT), a);
        if constexpr (FMT == F_INT8)
          ich[mm] += dot_int8(w[u], a);
        else
          facc[mm] += dot_block<FMT>(w[u], a, b);
      }
    }
  }
  if constexpr (FMT == F_INT8) {
    if (wb0 < wb1) {
#pragma unroll
      for (int mm = 0; mm < MT; mm++)
        atomicAdd(&csum[(mm * ncc + cur_chunk - cc0) * 32 + lane], ich[mm]);
    }
  } else {
#pragma unroll
    for (int mm = 0; mm < MT; mm++) sh.red[warp][mm][lane] = facc[mm];
  }
  cta_finish<FMT, MT>(p, g, ks, m0, cc0, ncc, csum, sh);
}

// ---------------------------------------------------------------------------
// Host-side planning and launch
// ---------------------------------------------------------------------------
struct Plan {
  int groups, nblk, kr, nks, nchunks, mt, rg;
  int ns;  // ring depth of k_qgemv_tma
  size_t xs_bytes;  // fused-norm row in shared memory (0 = none)
  size_t act_smem;  // activations + INT8 chunk sums
  int cluster;      // K split reduced through the cluster (nks CTAs along y)
  size_t recv_bytes;  // cluster rank 0's receive buffer for the peers' partials
};

int mt_for(size_t m) { return m == 1 ? 1 : (m == 2 ? 2 : 4); }

// Launch-planning defaults, overridable through the environment for tuning
// experiments (read once per process).
int tune(const char* name, int dflt) {
  static std::mutex mu;
  static std::vector<std::pair<std::string, int>> cache;
  std::lock_guard<std::mutex> g(mu);
  for (auto& kv : cache)
    if (kv.first == name) return kv.second;
  const char* v = getenv(name);
  const int r = v ? atoi(v) : dflt;
  cache.emplace_back(name, r);
  return r;
}

// Dynamic shared memory of k_qgemv_tma: the ring, the activations and, for
// the fused norm, the normalised row.
size_t stage_bytes(int fmt);
size_t tma_smem_no_recv(const Plan& pl, int fmt, int rg, int ns) {
  const size_t ring = (size_t)ns * rg * stage_bytes(fmt);
  const size_t base = ring + pl.act_smem;
  return pl.xs_bytes ? ((base + 15) & ~size_t(15)) + pl.xs_bytes : base;
}
size_t tma_smem(const Plan& pl, int fmt, int rg, int ns) {
  const size_t b = tma_smem_no_recv(pl, fmt, rg, ns);
  return pl.recv_bytes ? ((b + 15) & ~size_t(15)) + pl.recv_bytes : b;
}

int tma_occupancy(int fmt, int mt, int rg, size_t smem);
size_t stage_bytes(int fmt);
int stage_depth(int fmt);
int stage_depth_wide(int fmt);

// xs_bytes: the fused norm's row staged in shared memory (all of K).
Plan make_plan(int fmt, size_t m, size_t n, size_t kp, size_t xs_bytes = 0) {
  Plan pl{};
  pl.groups = (int)((n + 31) / 32);
  pl.nblk = (int)(kp / 32);
  pl.nchunks = (pl.nblk + 15) / 16;
  pl.mt = mt_for(m);
  const int sms = num_sms();
  // Aim at ~4 CTAs per SM: split K until the grid fills the GPU, keeping at
  // least one 16-block stage (one 512-element chunk) per CTA.
  const int target = sms * tune("SYN_GEMV_CTAS_PER_SM", 4);
  const int mslices = (int)((m + pl.mt - 1) / pl.mt);
  int nks = target / std::max(1, pl.groups * mslices);
  nks = std::max(1, std::min(nks, std::max(1, pl.nblk / SB)));
  // K splits only pay off when each CTA still streams a sizeable range
  // (measured on B200: the cross-CTA reduction costs more than it gains when
  // a split CTA would stream fewer than 64 blocks)
  const int min_split_blocks = tune("SYN_GEMV_MIN_SPLIT_BLOCKS", 64);
  while (nks > 1 && pl.nblk / nks < min_split_blocks) nks--;
  // Cluster K splits: at most 8 CTAs per cluster (the portable size).
  const bool use_cluster = fmt != F_Q4_0RAW && !(fmt == F_INT8 && pl.mt == 1) &&
                           tune("SYN_GEMV_CLUSTER", 1) != 0;
  if (use_cluster) nks = std::min(nks, 8);
  const int abb = fmt == F_INT8 ? 32 : 80;
  auto set_split = [&](int splits) {
    int kr = (pl.nblk + splits - 1) / splits;
    kr = (kr + SB - 1) / SB * SB;
    // shared memory bound (activations of MT rows)
    while ((size_t)pl.mt * kr * abb > 96 * 1024 && kr > SB) kr = ((kr + 1) / 2 + SB - 1) / SB * SB;
    pl.kr = kr;
    pl.nks = (pl.nblk + kr - 1) / kr;
    const int ncc = kr / 16 + 1;
    pl.act_smem =
        (size_t)pl.mt * kr * abb + (fmt == F_INT8 ? (size_t)pl.mt * ncc * 32 * 4 : 0);
    pl.xs_bytes = xs_bytes;
    pl.cluster = use_cluster && pl.nks > 1 && pl.nks <= 8;
    pl.recv_bytes = !pl.cluster ? 0
                    : std::max((size_t)pl.nks, fmt == F_INT8 ? (size_t)pl.nchunks : (size_t)0) *
                          pl.mt * 32 * 4;
  };
  set_split(nks);
  // Row-group pairs (block formats, M = 1, K not split): two groups share
  // each activation block, which saves about a third of the instructions per
  // weight; taken when the busiest SM's load goes down (per-SM CTA counts).
  pl.rg = 1;
  if (fmt != F_INT8 && fmt != F_Q4_0RAW && pl.mt == 1 && pl.nks == 1 &&
      tune("SYN_GEMV_ROW_PAIRS", 1)) {
    const double t1 = (double)((pl.groups + sms - 1) / sms);
    const double t2 = 2.0 * 0.7 * (double)(((pl.groups + 1) / 2 + sms - 1) / sms);
    if (t2 < t1) pl.rg = 2;
  }
  pl.ns = 0;
  if (fmt != F_Q4_0RAW) {
    // All CTAs resident at once: row pairs only while two CTAs still fit on
    // an SM, and a shallower ring where one more CTA per SM would otherwise
    // spill the grid into a second wave.
    // Grids of at least one CTA per SM: 3 stages (8-bit formats) or 4. A
    // smaller grid (the decode step's narrow matmuls) gets a ring as deep as
    // its CTAs' stage count, up to 6, so that every stage is requested before
    // griddepcontrol.wait instead of after the first ones are consumed.
    const long long grid0 =
        (long long)((pl.groups + pl.rg - 1) / pl.rg) * pl.nks * mslices;
    const int cta_stages = (pl.kr + SB - 1) / SB;
    int nsmax = stage_depth_wide(fmt);
    if (grid0 < sms && cta_stages > nsmax)
      nsmax = std::min(stage_depth(fmt), cta_stages);
    auto occ = [&](int rg, int ns) {
      return tma_occupancy(fmt, pl.mt, rg, tma_smem(pl, fmt, rg, ns));
    };
    if (pl.rg == 2 && occ(2, nsmax) < 2) pl.rg = 1;
    // deepest ring that keeps the grid in one wave; failing that, fewer K
    // splits (registers, not shared memory, may be what limits residency)
    auto pick_ns = [&]() {
      const long long ctas = (long long)((pl.groups + pl.rg - 1) / pl.rg) * pl.nks * mslices;
      for (int t = nsmax; t >= 2; t--)
        if (ctas <= (long long)sms * occ(pl.rg, t)) return t;
      return 0;
    };
    int ns = pick_ns();
    // SYN_GEMV_ONE_WAVE=0 keeps the K splits even when the grid runs in
    // several waves (the deepest ring is used then)
    while (ns == 0 && pl.nks > 1 && tune("SYN_GEMV_ONE_WAVE", 1)) {
      const int before = pl.nks;
      set_split(before - 1);
      if (pl.nks >= before) break;  // the shared-memory bound split it again
      ns = pick_ns();
    }
    if (ns == 0) ns = nsmax;
    const int forced = tune("SYN_GEMV_NS", 0);
    pl.ns = forced >= 2 && forced <= nsmax ? forced : ns;
  }
  return pl;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, int cluster_y, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = tune("SYN_GEMV_PDL", 1) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster_y > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = (unsigned)cluster_y;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Allows up to 200 KB of dynamic shared memory, once per kernel and device.
// (Keyed by the kernel's address: all GEMV instantiations share one type.)
template <typename K>
void allow_smem(K kern) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kern), dev);
  std::lock_guard<std::mutex> guard(mu);
  if (done.count(key)) return;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  done.insert(key);
}

size_t stage_bytes(int fmt) {
  switch (fmt) {
    case F_INT8: return Stage<F_INT8>::BYTES;
    case F_Q4_0: return Stage<F_Q4_0>::BYTES;
    case F_Q8_0: return Stage<F_Q8_0>::BYTES;
    case F_Q4_K: return Stage<F_Q4_K>::BYTES;
    case F_Q6_K: return Stage<F_Q6_K>::BYTES;
  }
  return 0;
}

int stage_depth_wide(int fmt) { return eight_bit(fmt) ? Stage<F_INT8>::NS_WIDE : Stage<F_Q4_0>::NS_WIDE; }

int stage_depth(int fmt) {
  switch (fmt) {
    case F_INT8: return Stage<F_INT8>::NS;
    case F_Q4_0: return Stage<F_Q4_0>::NS;
    case F_Q8_0: return Stage<F_Q8_0>::NS;
    case F_Q4_K: return Stage<F_Q4_K>::NS;
    case F_Q6_K: return Stage<F_Q6_K>::NS;
  }
  return 2;
}

template <typename K>
int occ_of(K kern, size_t smem) {
  allow_smem(kern);
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, THREADS + 32, smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  return occ;
}

template <int FMT>
int tma_occ_f(int mt, int rg, size_t smem) {
  if constexpr (FMT != F_INT8) {
    if (mt == 1) return rg == 2 ? occ_of(k_qgemv_tma<FMT, 1, 2>, smem)
                                : occ_of(k_qgemv_tma<FMT, 1, 1>, smem);
  } else {
    if (mt == 1) return occ_of(k_qgemv_tma<FMT, 1, 1>, smem);
  }
  return mt == 2 ? occ_of(k_qgemv_tma<FMT, 2, 1>, smem) : occ_of(k_qgemv_tma<FMT, 4, 1>, smem);
}

// CTAs of k_qgemv_tma resident per SM at `smem` bytes (cached per device).
int tma_occupancy(int fmt, int mt, int rg, size_t smem) {
  struct Key {
    int fmt, mt, rg, dev;
    size_t smem;
    int occ;
  };
  static std::mutex mu;
  static std::vector<Key> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> g(mu);
    for (const Key& k : cache)
      if (k.fmt == fmt && k.mt == mt && k.rg == rg && k.dev == dev && k.smem == smem) return k.occ;
  }
  int occ = 1;
  switch (fmt) {
    case F_INT8: occ = tma_occ_f<F_INT8>(mt, rg, smem); break;
    case F_Q4_0: occ = tma_occ_f<F_Q4_0>(mt, rg, smem); break;
    case F_Q8_0: occ = tma_occ_f<F_Q8_0>(mt, rg, smem); break;
    case F_Q4_K: occ = tma_occ_f<F_Q4_K>(mt, rg, smem); break;
    case F_Q6_K: occ = tma_occ_f<F_Q6_K>(mt, rg, smem); break;
  }
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.push_back(Key{fmt, mt, rg, dev, smem, occ});
  return occ;
}

template <int FMT, int MT>
syn_status_t launch_t(const GemvParams& p, const Plan& pl, cudaStream_t st) {
  dim3 grid((unsigned)pl.groups, (unsigned)pl.nks, (unsigned)((p.m + MT - 1) / MT));
  cudaError_t e;
  if constexpr (FMT == F_Q4_0RAW) {
    allow_smem(k_qgemv<FMT, MT>);
    e = launch_pdl(k_qgemv<FMT, MT>, grid, dim3(THREADS), pl.act_smem, st, 1, p);
  } else {
    GemvParams q = p;
    const int rg = (FMT != F_INT8 && MT == 1) ? pl.rg : 1;
    q.ns = pl.ns;
    q.xs_off = (int)(((size_t)pl.ns * rg * Stage<FMT>::BYTES + pl.act_smem + 15) & ~size_t(15));
    q.cluster = pl.cluster;
    q.recv_off = (int)((tma_smem_no_recv(pl, FMT, rg, pl.ns) + 15) & ~size_t(15));
    const size_t smem = tma_smem(pl, FMT, rg, pl.ns);
    const int cy = pl.cluster ? pl.nks : 1;
    if constexpr (FMT != F_INT8 && MT == 1) {
      if (rg == 2) {
        allow_smem(k_qgemv_tma<FMT, 1, 2>);
        grid.x = (unsigned)((pl.groups + 1) / 2);
        e = launch_pdl(k_qgemv_tma<FMT, 1, 2>, grid, dim3(THREADS + 32), smem, st, cy, q);
      } else {
        allow_smem(k_qgemv_tma<FMT, 1, 1>);
        e = launch_pdl(k_qgemv_tma<FMT, 1, 1>, grid, dim3(THREADS + 32), smem, st, cy, q);
      }
    } else {
      allow_smem(k_qgemv_tma<FMT, MT, 1>);
      e = launch_pdl(k_qgemv_tma<FMT, MT, 1>, grid, dim3(THREADS + 32), smem, st, cy, q);
    }
  }
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "k_qgemv");
    return SYN_ERR_CUDA;
  }
  return SYN_OK;
}

template <int FMT>
syn_status_t launch_m(const GemvParams& p, const Plan& pl, cudaStream_t st) {
  if (pl.mt == 1) return launch_t<FMT, 1>(p, pl, st);
  if (pl.mt == 2) return launch_t<FMT, 2>(p, pl, st);
  return launch_t<FMT, 4>(p, pl, st);
}

syn_status_t run_gemv(int fmt, const GemvParams& p, const Plan& pl, cudaStream_t st) {
  switch (fmt) {
    case F_INT8: return launch_m<F_INT8>(p, pl, st);
    case F_Q4_0: return launch_m<F_Q4_0>(p, pl, st);
    case F_Q8_0: return launch_m<F_Q8_0>(p, pl, st);
    case F_Q4_K: return launch_m<F_Q4_K>(p, pl, st);
    case F_Q6_K: return launch_m<F_Q6_K>(p, pl, st);
    case F_Q4_0RAW: return launch_t<F_Q4_0RAW, 1>(p, pl, st);
  }
  return SYN_ERR_INVALID_ARG;
}

// Bytes of split-K partial sums a launch of plan `pl` writes (0 unsplit).
size_t plan_part_bytes(int fk, const Plan& pl, size_t m) {
  if (pl.nks <= 1 || pl.cluster) return 0;
  const size_t per = fk == F_INT8 ? (size_t)pl.nchunks : (size_t)pl.nks;
  return m * per * (size_t)pl.groups * 32 * sizeof(float);
}

void fill_common(GemvParams& p, const Plan& pl, float* part, int* cnt, int* err) {
  p.groups = pl.groups;
  p.nblk = pl.nblk;
  p.kr = pl.kr;
  p.nks = pl.nks;
  p.nchunks = pl.nchunks;
  p.part = part;
  p.cnt = cnt;
  p.err = err;
}

}  // namespace

size_t gemv_partial_bytes(int fmt, size_t m, size_t n, size_t kp, size_t k) {
  // the weight's own plan, as the launches make it (the K split depends on
  // each format's occupancy); for one row also the fused-RMSNorm plan
  const int fk = fmt == SYN_QFMT_INT8_KN ? F_INT8 : fmt;
  size_t b = plan_part_bytes(fk, make_plan(fk, m, n, kp), m);
  if (m == 1 && k > 0 && k <= 16384)
    b = std::max(b, plan_part_bytes(fk, make_plan(fk, 1, n, kp, k * sizeof(float)), 1));
  return b;
}

size_t gemv_counter_bytes(size_t m, size_t n) {
  return ((m + 3) / 4 * 4) * ((n + 31) / 32) * sizeof(int);
}

syn_status_t launch_qgemv(const syn_cuda_weight_s* w, const float* x, size_t ldx,
                          const int8_t* xq, const float* sx, size_t m, float* y, size_t ldy,
                          int chunked, float* part, size_t part_cap, int* cnt, int* err,
                          cudaStream_t st) {
  if (w->n > 0x7FFFFFFFull || w->kp > 0x3FFFFFFFull || m > 0xFFFFull) return SYN_ERR_UNSUPPORTED;
  // the float4 activation loads of the block formats need 16-byte aligned rows
  if (w->fmt != SYN_QFMT_INT8_KN && ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & 3)))
    return SYN_ERR_NOT_CONTIGUOUS;
  const int fk = w->fmt == SYN_QFMT_INT8_KN ? F_INT8 : w->fmt;
  const Plan pl = make_plan(fk, m, w->n, w->kp);
  GemvParams p{};
  p.q = w->q;
  p.d = w->d;
  p.sb = w->sb;
  p.hdr = w->hdr;
  p.qh = w->qh;
  p.sc = reinterpret_cast<const uint16_t*>(w->sc);
  p.x = x;
  p.xq = xq;
  p.sx = sx;
  p.ldx = (long long)ldx;
  p.n = (int)w->n;
  p.k = (int)w->k;
  p.kp = (int)w->kp;
  p.nsb = (int)(w->k / 256);
  p.m = (int)m;
  p.y = y;
  p.ldy = (long long)ldy;
  p.chunked = chunked;
  fill_common(p, pl, part, cnt, err);
  if (pl.nks > 1 && !pl.cluster && (!part || !cnt || plan_part_bytes(fk, pl, m) > part_cap))
    return SYN_ERR_INTERNAL;
  return run_gemv(fk, p, pl, st);
}

syn_status_t launch_qgemv_norm(const syn_cuda_weight_s* w, const GemvNorm& nm, float* y,
                               float* part, size_t part_cap, int* cnt, int* err,
                               cudaStream_t st) {
  if (w->n > 0x7FFFFFFFull || w->kp > 0x3FFFFFFFull) return SYN_ERR_UNSUPPORTED;
  if (w->k > 16384) return SYN_ERR_UNSUPPORTED;  // the row is staged in shared memory
  const int fk = w->fmt == SYN_QFMT_INT8_KN ? F_INT8 : w->fmt;
  const Plan pl = make_plan(fk, 1, w->n, w->kp, w->k * sizeof(float));
  GemvParams p{};
  p.q = w->q;
  p.d = w->d;
  p.sb = w->sb;
  p.hdr = w->hdr;
  p.qh = w->qh;
  p.sc = reinterpret_cast<const uint16_t*>(w->sc);
  p.x = nullptr;  // replaced by the normalised row in shared memory
  p.n = (int)w->n;
  p.k = (int)w->k;
  p.kp = (int)w->kp;
  p.nsb = (int)(w->k / 256);
  p.m = 1;
  p.y = y;
  p.ldy = (long long)w->n;
  p.nres = nm.res;
  p.ndelta = nm.delta;
  p.nw = nm.w;
  p.neps = nm.eps;
  p.nres_out = nm.res_out;
  p.nfast = nm.fast;
  p.sw_out = nm.sw_out;
  p.sw_ld = nm.sw_n;
  p.sw_n = nm.sw_n;
  p.sw_variant = nm.sw_variant;
  if (nm.sw_out && (w->n != 2 * (size_t)nm.sw_n || nm.sw_n % 16)) return SYN_ERR_SHAPE_MISMATCH;
  fill_common(p, pl, part, cnt, err);
  if (pl.nks > 1 && !pl.cluster && (!part || !cnt || plan_part_bytes(fk, pl, 1) > part_cap))
    return SYN_ERR_INTERNAL;
  return run_gemv(fk, p, pl, st);
}

syn_status_t launch_q4_0_raw(size_t n, size_t k, const float* a, const uint8_t* b, float* c,
                             float* part, size_t part_cap, int* cnt, int* err,
                             cudaStream_t st) {
  if (n > 0x7FFFFFFFull || k > 0x3FFFFFFFull) return SYN_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(a) & 15) return SYN_ERR_NOT_CONTIGUOUS;
  const Plan pl = make_plan(F_Q4_0RAW, 1, n, k);
  GemvParams p{};
  p.q = b;
  p.x = a;
  p.ldx = (long long)k;
  p.n = (int)n;
  p.k = (int)k;
  p.kp = (int)k;
  p.m = 1;
  p.y = c;
  p.ldy = (long long)n;
  fill_common(p, pl, part, cnt, err);
  if (pl.nks > 1 && (!part || !cnt || plan_part_bytes(F_Q4_0RAW, pl, 1) > part_cap))
    return SYN_ERR_INTERNAL;
  return run_gemv(F_Q4_0RAW, p, pl, st);
}

}  // namespace syn
