// gemm.cu -- prefill / batched path: quantized matmul on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in tensor memory).
//
//   y[M, N] = x[M, K] * W[N, K]^T for batched rows (tokens), all five
//   formats; gemm_min_rows() decides, per weight row count, from which M the
//   GEMM runs instead of the GEMV.
//
// Operands in shared memory are K-major.
//   INT8 uses the plain layout (core matrices of 8 rows x 16 bytes; a
//   [rows][16 B] column of 128 rows is 2 KB). fp16 (block formats) uses the
//   128-byte-swizzled layout: 1024-byte atoms of 8 rows x 128 B (64 halves of
//   K), chunk j of row r stored at j ^ (r & 7), two atom columns per stage.
//   A (activations) is prepared by k_prep_a_* into global memory already in
//   the stage layout, so one stage of A is one contiguous 1-D bulk copy.
//     INT8 weights: A = int8 codes of the reference's per-row quantisation
//       (quantize.zig:12-47), bit-exact; products are exact int32
//       (kind::i8). M <= 16: one int32 accumulator over K, then
//       float(acc) * sa * sb (qmatmul.zig:52-66, 218-223). M > 16: the
//       reference's per-512-K-chunk epilogue C += float(chunk) * sa * sb in
//       chunk order (qmatmul.zig:68-98), every op rounded -- bit-exact for
//       every M.
//     Block formats: A = fp16(x * 2^-s) with a power-of-two scale per row
//       (no fp16 overflow; undone exactly in the epilogue); the weights are
//       dequantised in shared memory with the reference's formulas
//       (gguf.rs:255-487), rounded to fp16 and multiplied with kind::f16,
//       fp32 accumulation.
//   B (weights) comes from the row-interleaved repack (repack.cu). For INT8
//   a 4-D tensor map (TMA) gathers the 4 row groups' tiles of a stage into
//   [16-byte K column][128 rows][16 B]; block formats bring the raw tiles in
//   with 1-D bulk copies and the worker warps write the dequantised fp16
//   tiles. Each K step is one 128 x 128 x 16 (fp16) or x 32 (int8) MMA.
//   Up to 32 tokens (block formats) the roles swap (SW): the 128 weight rows
//   are the MMA's M and the tokens, each as an fp16 hi and lo row, its N.
//   From 129 tokens (block formats) k_qgemm_tm keeps the dequantised weights
//   in tensor memory as the MMA's A operand, with tiles of up to 256 tokens
//   as B.
//
// CTA = 18 warps: warp 0 issues the copies into a smem ring; warp 1 owns
// tensor memory and one of its threads issues the MMAs; warps 2-17
// dequantise B (block formats) and run the epilogue (tensor memory ->
// registers -> y). Tile: 128 tokens x 128 weight rows. Every wait is bounded
// and reports SYN_ERR_TIMEOUT instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>

#include "internal.cuh"

namespace syn {
namespace {

enum : int { F_INT8 = SYN_QFMT_INT8_KN, F_Q4_0 = SYN_QFMT_Q4_0, F_Q8_0 = SYN_QFMT_Q8_0,
             F_Q4_K = SYN_QFMT_Q4_K, F_Q6_K = SYN_QFMT_Q6_K };

constexpr int BM = 128;  // tokens per tile (MMA M)
constexpr int BN = 128;  // weight rows per tile (4 row groups of 32) = MMA N
constexpr int NG = BN / 32;
constexpr int WORKERS = 16;                      // dequant / epilogue warps
constexpr int WSETS = WORKERS / 4;               // warps per tensor-memory lane quarter
constexpr int CGW = 4 / WSETS;                   // 32-column groups per epilogue warp
constexpr int GEMM_THREADS = 64 + WORKERS * 32;  // producer + MMA + workers

// ---------------------------------------------------------------------------
// tcgen05 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// smem matrix descriptor: K-major, no swizzle (core matrices 8 rows x 16 B).
// lbo = bytes to the next 16 bytes of K, sbo = bytes to the next 8 rows.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;                // base offset 0, legacy LBO mode, layout SWIZZLE_NONE
}

// fp16 operands use the 128-byte-swizzled K-major layout: atoms of 8 rows x
// 128 B (64 halves of K) at 1024-byte-aligned addresses, 8-row groups 1024 B
// apart, and within a row the 16-byte chunk j stored at chunk j ^ (row & 7).
// A tile of R rows and 128 K (one stage) is two atoms columns of R * 128 B.
// Descriptor: SBO = 1024 B, LBO = 16 B, layout type 2 (SWIZZLE_128B); a K
// step inside an atom advances the start address (the hardware applies the
// XOR to the final address bits).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;          // LBO = 16 B
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO = 1024 B
  d |= (uint64_t)1 << 46;          // descriptor version for sm_100
  d |= (uint64_t)2 << 61;          // SWIZZLE_128B
  return d;
}

// Byte offset of 16-byte K column c (0..15 within a stage) of row r in a
// swizzled stage tile of `rows` rows.
__host__ __device__ __forceinline__ uint32_t sw128_off(int c, int r, int rows) {
  return (uint32_t)((c >> 3) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                    (((c & 7) ^ (r & 7)) << 4));
}

// Instruction descriptor: M = 128, N = 128, K-major A and B.
// c_format (bits 4-5): 1 = F32, 2 = S32; a/b format (7-9, 10-12): kind::f16
// -> 0 = F16, kind::i8 -> 1 = signed; n_dim (17-22) = N >> 3; m_dim (24-28)
// = M >> 4.
template <bool I8>
__host__ __device__ constexpr uint32_t idesc_tile() {
  return (I8 ? (2u << 4) : (1u << 4)) | (I8 ? (1u << 7) : 0u) | (I8 ? (1u << 10) : 0u) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

template <bool I8>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  constexpr uint32_t id = idesc_tile<I8>();
  if constexpr (I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(
            tmem_d),
        "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(0u));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(
            tmem_d),
        "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(0u));
  }
}

// kind::f16 MMA with a runtime instruction descriptor (SW: N = npad).
__device__ __forceinline__ void mma_f16_id(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(
          tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(0u));
}

// Arrives on `bar` once every MMA issued so far by this thread is complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 4-D tiled TMA load into this CTA's own shared memory only.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; thread i gets lane (base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
      "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; thread i writes lane (base + i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// kind::f16 MMA with A from tensor memory (128 lanes = rows of A, K along the
// columns, two halves per 32-bit column) and B from shared memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b,
                                           uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(id), "r"(accumulate));
}

// ---------------------------------------------------------------------------
// Per-format stage geometry
// ---------------------------------------------------------------------------
// Raw block-format bytes of one 32-row group for a stage of KBX blocks: the
// q tiles, then per-block aux arrays, then one super-block tile (Q4_K
// header, Q6_K scale; a stage never crosses a 256-element super-block).
template <int FMT, int KBX>
struct RawG {
  static constexpr int QT = (FMT == F_Q8_0) ? 1024 : 512;
  static constexpr int DT = (FMT == F_Q4_0 || FMT == F_Q8_0) ? 64 : 0;
  static constexpr int QHT = (FMT == F_Q6_K) ? 256 : 0;
  static constexpr int SCT = (FMT == F_Q6_K) ? 64 : 0;
  static constexpr int HT = (FMT == F_Q4_K) ? 512 : 0;
  static constexpr int D6T = (FMT == F_Q6_K) ? 64 : 0;
  static constexpr int G_Q = 0;
  static constexpr int G_D = G_Q + KBX * QT;
  static constexpr int G_QH = G_D + KBX * DT;
  static constexpr int G_SC = G_QH + KBX * QHT;
  static constexpr int G_H = G_SC + KBX * SCT;
  static constexpr int G_D6 = G_H + HT;
  static constexpr int G_BYTES = (G_D6 + D6T + 127) / 128 * 128;
};
// SW (few tokens, block formats): the operands swap roles -- the 128
// dequantised weight rows are the MMA's M and the tokens its N -- so a
// stage's activation tile is small and the ring can be deeper. Each token
// enters as two fp16 rows, x = hi + lo (hi = fp16(x), lo = fp16(x - hi)), so
// only the weights are rounded: N = 2 npad <= 64 (npad = tokens padded to a
// multiple of 16), and the epilogue adds the hi and lo columns.
template <int FMT, bool SW = false>
struct GS {
  static constexpr bool I8 = FMT == F_INT8;
  static constexpr int KB = I8 ? 8 : 4;                        // 32-element blocks per stage
  static constexpr int A_BYTES =
      SW ? KB * 4 * 64 * 16 : BM * KB * 32 * (I8 ? 1 : 2);     // 16 KB (SW) / 32 KB
  // INT8: B stage = [2*KB K columns][128 rows][16 B] (tensor-map gather)
  static constexpr int B8_BYTES = I8 ? BN * KB * 32 : 0;       // 32 KB
  // block formats: raw bytes per row group (q tiles + per-block aux)
  static constexpr int QT = (FMT == F_Q8_0) ? 1024 : 512;
  static constexpr int DT = (FMT == F_Q4_0 || FMT == F_Q8_0) ? 64 : 0;
  static constexpr int QHT = (FMT == F_Q6_K) ? 256 : 0;
  static constexpr int SCT = (FMT == F_Q6_K) ? 64 : 0;
  static constexpr int HT = (FMT == F_Q4_K) ? 512 : 0;  // one super-block tile per stage
  static constexpr int D6T = (FMT == F_Q6_K) ? 64 : 0;  // one super-block tile per stage
  static constexpr int G_Q = 0;
  static constexpr int G_D = G_Q + KB * QT;
  static constexpr int G_QH = G_D + KB * DT;
  static constexpr int G_SC = G_QH + KB * QHT;
  static constexpr int G_H = G_SC + KB * SCT;
  static constexpr int G_D6 = G_H + HT;
  static constexpr int G_BYTES = I8 ? 0 : (G_D6 + D6T + 127) / 128 * 128;  // per row group
  static constexpr int RAW_BYTES = I8 ? B8_BYTES : NG * G_BYTES;
  static constexpr int STAGE_BYTES = (A_BYTES + RAW_BYTES + 1023) / 1024 * 1024;  // atom aligned
  // block formats: dequantised fp16 B = [block][4 K columns][128 rows][16 B]
  static constexpr int BH_BYTES = I8 ? 0 : BN * KB * 32 * 2;   // 32 KB
  static constexpr int NBH = I8 ? 0 : 2;
  static constexpr int NS_FIT = (230400 - NBH * BH_BYTES) / STAGE_BYTES;
  static constexpr int NS = SW ? (NS_FIT < 8 ? NS_FIT : 8) : 3;  // ring depth
  static constexpr int SMEM = NS * STAGE_BYTES + NBH * BH_BYTES;
  static constexpr uint32_t TMEM_COLS = I8 ? 512 : 128;
};

struct GemmParams {
  const uint8_t* q;
  const uint16_t* d;
  const float* sb;
  const uint8_t* hdr;
  const uint8_t* qh;
  const uint16_t* sc;
  int n, k, nblk, nsb, groups;
  const uint8_t* a;  // prepared activations
  int kcols;         // 16-byte K columns per A row
  const float* sa;   // INT8: per-row activation scale
  int m;
  float* y;
  long long ldy;
  int chunked;
  int* err;
  int short_rows;  // m-tiles with at most this many valid rows copy only those
  int npad;        // SW: tokens padded to a multiple of 16 (the MMA's N is 2 npad)
  int astg;        // fp16 A: stages (16 K columns each) per m-tile in the prepared buffer
};

__device__ __forceinline__ void greport(const GemmParams& p) {
  if (p.err) atomicExch(p.err, SYN_ERR_TIMEOUT);
}

__device__ __forceinline__ bool bwait(const GemmParams& p, uint64_t* bar, uint32_t parity) {
  if (mbar_wait_bounded(bar, parity)) return true;
  greport(p);
  return false;
}

// Dequantises block bl of one row group's raw stage of KBX blocks (thread =
// row l of the group) into 32 fp16 values in K order, packed in pairs:
// o[i] = (value 2i, value 2i+1). Reference formulas: gguf.rs:255-487.
// With LO (Q4_K, Q6_K in k_qgemm_tm), lo[i] receives the fp16 remainders
// v - fp16(v) of the same pairs, so that hi + lo carries about 22 bits of
// the reference's f32 value.
template <int FMT, int KBX, bool LO = false>
__device__ __forceinline__ void dequant_regs(const uint8_t* raw, int l, int bl, int b,
                                             uint32_t (&o)[16], uint32_t* lo = nullptr) {
  using S = RawG<FMT, KBX>;
  if constexpr (FMT == F_Q4_0 || FMT == F_Q8_0) {
    // fp16 arithmetic, same values: (q - 8) and q are exact in fp16, d is an
    // fp16 value, and the product of two fp16 values rounded once to fp16
    // equals the reference's exact f32 product (gguf.rs:276-285, 318-324)
    // rounded to fp16. The loader's subnormal quirk (a halved scale) is kept
    // by halving q first, which is exact. Codes become fp16 with the
    // 0x6400 (1024.0) mantissa trick: no int-to-float conversions.
    const uint16_t dbits = reinterpret_cast<const uint16_t*>(raw + S::G_D + bl * 64)[l];
    const __half2 d2 = __half2half2(__ushort_as_half(dbits));
    const bool sub = (dbits & 0x7C00u) == 0;
    const __half2 half2_05 = __float2half2_rn(0.5f);
    if constexpr (FMT == F_Q4_0) {
      const uint4 q = reinterpret_cast<const uint4*>(raw + S::G_Q + bl * 512)[l];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      const __half2 bias = __float2half2_rn(1032.0f);  // 1024 + 8
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
        const uint32_t pr = (byte & 0x0Fu) | ((byte & 0xF0u) << 12) | 0x64006400u;
        __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&pr), bias);  // (lo-8, hi-8)
        if (sub) h = __hmul2(h, half2_05);
        h = __hmul2(h, d2);
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    } else {
      const uint4 q0 = reinterpret_cast<const uint4*>(raw + S::G_Q + bl * 1024)[l];
      const uint4 q1 = reinterpret_cast<const uint4*>(raw + S::G_Q + bl * 1024 + 512)[l];
      const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      const __half2 bias = __float2half2_rn(1152.0f);  // 1024 + 128
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const uint32_t two = (w[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;  // codes 2i, 2i+1
        const uint32_t pr = (((two & 0xFFu) ^ 0x80u) | (((two >> 8) ^ 0x80u) << 16)) | 0x64006400u;
        __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&pr), bias);
        if (sub) h = __hmul2(h, half2_05);
        h = __hmul2(h, d2);
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    return;
  } else {
    float v[32];
    if constexpr (FMT == F_Q4_K) {
      const uint4 q = reinterpret_cast<const uint4*>(raw + S::G_Q + bl * 512)[l];
      const uint4 h = reinterpret_cast<const uint4*>(raw + S::G_H)[l];
      const int s = b & 7;
      const float dd = f16_loader((uint16_t)(h.x & 0xFFFF));
      const float dmin = f16_loader((uint16_t)(h.x >> 16));
      uint32_t scv, mnv;
      if (s < 4) {
        const int sh = 8 * s;
        scv = (h.y >> sh) & 0x3F;
        mnv = (((h.z >> sh) & 0xFF) >> 4) | (((h.w >> sh) & 0x0F) << 4);
      } else {
        const int sh = 8 * (s - 4);
        const uint32_t ys = (h.y >> sh) & 0xFF;
        scv = ((h.z >> sh) & 0x0F) | ((ys >> 6) << 4);
        mnv = (((h.w >> sh) & 0xFF) >> 4) | (((ys >> 4) & 0x0C) << 4);
      }
      const float scl = __fmul_rn(dd, (float)scv), mv = __fmul_rn(dmin, (float)mnv);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFF;
        v[2 * i] = __fsub_rn(__fmul_rn(i2f_small((int)(byte & 15)), scl), mv);
        v[2 * i + 1] = __fsub_rn(__fmul_rn(i2f_small((int)(byte >> 4)), scl), mv);
      }
    } else {  // F_Q6_K
      const uint4 q = reinterpret_cast<const uint4*>(raw + S::G_Q + bl * 512)[l];
      const uint2 hq = reinterpret_cast<const uint2*>(raw + S::G_QH + bl * 256)[l];
      const uint32_t scp = reinterpret_cast<const uint16_t*>(raw + S::G_SC + bl * 64)[l];
      const float dd = f16_loader(reinterpret_cast<const uint16_t*>(raw + S::G_D6)[l]);
      const float s0 = __fmul_rn((float)(int8_t)(scp & 0xFF), dd);
      const float s1 = __fmul_rn((float)(int8_t)(scp >> 8), dd);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const uint32_t byte = (w[e >> 3] >> (8 * ((e >> 1) & 3))) & 0xFF;
        const uint32_t lo = (e & 1) ? (byte >> 4) : (byte & 15);
        // invert the high-bit re-arrangement of repack.cu (k_repack_q6_k)
        const int half = e >> 4, r = e & 15, f = 2 * (r >> 3) + (r & 1), tt = (r & 7) >> 1;
        const uint32_t H = half ? hq.y : hq.x;
        const uint32_t hi = (H >> (8 * tt + 2 * f)) & 3u;
        v[e] = __fmul_rn(i2f_small((int)(lo | (hi << 4)) - 32), half ? s1 : s0);
      }
    }
#pragma unroll
    for (int i = 0; i < 16; i++) {  // paired f32 -> f16 conversions (round to nearest)
      const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      o[i] = *reinterpret_cast<const uint32_t*>(&h);
      if constexpr (LO) {
        // v - fp16(v) is exact in f32
        const __half2 r = __floats2half2_rn(__fsub_rn(v[2 * i], __low2float(h)),
                                            __fsub_rn(v[2 * i + 1], __high2float(h)));
        lo[i] = *reinterpret_cast<const uint32_t*>(&r);
      }
    }
  }
}

// dequant_regs into the swizzled 128-row fp16 tile in shared memory: the 4
// K columns (8 halves each) of block bl, row `row`.
template <int FMT>
__device__ __forceinline__ void dequant_block(const uint8_t* raw, uint8_t* out, int l, int row,
                                              int bl, int b) {
  uint32_t o[16];
  dequant_regs<FMT, GS<FMT>::KB>(raw, l, bl, b, o);
#pragma unroll
  for (int c = 0; c < 4; c++)
    *reinterpret_cast<uint4*>(out + sw128_off(bl * 4 + c, row, BN)) =
        make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}

template <int FMT, bool SW = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_qgemm(const GemmParams p, const __grid_constant__ CUtensorMap tmb) {
  using S = GS<FMT, SW>;
  static_assert(!SW || FMT != F_INT8, "swapped operands: block formats");
  constexpr bool I8 = S::I8;
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[S::NS], empty[S::NS];
  __shared__ __align__(8) uint64_t bfull[2], bempty[2];      // fp16 B buffers
  __shared__ __align__(8) uint64_t accfull[2], accempty[2];  // accumulators
  __shared__ uint32_t tmem_base_sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x, nt = blockIdx.y;
  const int nst = (p.nblk + S::KB - 1) / S::KB;
  const bool chunked = I8 && p.chunked;  // INT8: chunk = 16 blocks = 2 stages
  const int nchunks = (p.nblk + 15) / 16;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], I8 ? 1 : 1 + WORKERS);  // MMA commit (+ dequant warps)
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&bfull[i], WORKERS);
      mbar_init(&bempty[i], 1);
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], WORKERS);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"(S::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_sh;
  // A, sa (and y's previous readers) belong to the kernels launched before
  griddep_wait();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      constexpr int cpb = I8 ? 2 : 4;  // 16-byte A columns per block
      int ngr = 0;
      for (int gi = 0; gi < NG; gi++)
        if (nt * NG + gi < p.groups) ngr++;
      for (int s = 0; s < nst; s++) {
        const int slot = s % S::NS;
        if (s >= S::NS && !bwait(p, &empty[slot], ((s / S::NS) - 1) & 1)) break;
        const int b0 = s * S::KB, nbs = min(S::KB, p.nblk - b0);
        uint8_t* st = sm + slot * S::STAGE_BYTES;
        uint8_t* raw = st + S::A_BYTES;
        // A: a short m-tile (few tokens) copies only its valid rows of every
        // 16-byte K column (the rows beyond are never stored to y)
        const int rv = (min(BM, p.m - mt * BM) + 7) & ~7;
        const bool short_a = !SW && rv <= p.short_rows;
        // fp16 A: swizzled stage tiles [atom][rows][128 B], one atom per 2 blocks
        const int arows = SW ? 2 * p.npad : BM, atoms = (nbs + 1) / 2;
        uint32_t a_bytes;
        if constexpr (I8)
          a_bytes = short_a ? (uint32_t)(nbs * cpb * rv * 16) : nbs * cpb * 2048;
        else
          a_bytes = (uint32_t)(atoms * (short_a ? rv : arows) * 128);
        uint32_t bytes = a_bytes;
        if constexpr (I8)
          bytes += S::B8_BYTES;  // the full tensor-map box (out of range reads as zero)
        else
          bytes += ngr * (nbs * (S::QT + S::DT + S::QHT + S::SCT) + S::HT + S::D6T);
        mbar_expect_tx(&full[slot], bytes);
        if constexpr (I8) {
          const uint8_t* asrc = p.a + ((size_t)mt * p.kcols + (size_t)b0 * cpb) * 2048;
          if (short_a) {
            for (int c = 0; c < nbs * cpb; c++)
              bulk_g2s(st + c * 2048, asrc + (size_t)c * 2048, rv * 16, &full[slot]);
          } else {
            bulk_g2s(st, asrc, a_bytes, &full[slot]);
          }
        } else {
          const uint8_t* asrc = p.a + ((size_t)mt * p.astg + s) * arows * 256;
          if (short_a) {  // the valid rows' 8-row groups of each atom
            for (int a = 0; a < atoms; a++)
              bulk_g2s(st + a * BM * 128, asrc + (size_t)a * BM * 128, rv * 128, &full[slot]);
          } else {
            bulk_g2s(st, asrc, a_bytes, &full[slot]);
          }
        }
        if constexpr (I8) {
          tma_load_4d(raw, &tmb, 0, 0, nt * NG, 2 * b0, &full[slot]);
        } else {
          for (int gi = 0; gi < ngr; gi++) {
            const size_t g = (size_t)nt * NG + gi;
            uint8_t* gr = raw + gi * S::G_BYTES;
            const size_t t0 = g * p.nblk + b0;
            bulk_g2s(gr + S::G_Q, p.q + t0 * S::QT, nbs * S::QT, &full[slot]);
            if constexpr (S::DT)
              bulk_g2s(gr + S::G_D, reinterpret_cast<const uint8_t*>(p.d) + t0 * 64, nbs * 64,
                       &full[slot]);
            if constexpr (S::QHT) {
              bulk_g2s(gr + S::G_QH, p.qh + t0 * 256, nbs * 256, &full[slot]);
              bulk_g2s(gr + S::G_SC, reinterpret_cast<const uint8_t*>(p.sc) + t0 * 64, nbs * 64,
                       &full[slot]);
            }
            if constexpr (S::HT)
              bulk_g2s(gr + S::G_H, p.hdr + (g * p.nsb + b0 / 8) * 512, 512, &full[slot]);
            if constexpr (S::D6T)
              bulk_g2s(gr + S::G_D6,
                       reinterpret_cast<const uint8_t*>(p.d) + (g * p.nsb + b0 / 8) * 64, 64,
                       &full[slot]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      int chunk = 0;  // INT8 chunked: accumulator buffer = chunk & 1
      for (int s = 0; s < nst; s++) {
        const int slot = s % S::NS;
        if (!bwait(p, &full[slot], (s / S::NS) & 1)) { ok = false; break; }
        const int b0 = s * S::KB, nbs = min(S::KB, p.nblk - b0);
        const uint8_t* st = sm + slot * S::STAGE_BYTES;
        const uint32_t a_addr = smem_u32(st);
        uint32_t b_addr;
        if constexpr (I8) {
          b_addr = smem_u32(st + S::A_BYTES);
          if (chunked && (b0 & 15) == 0 && chunk >= 2) {
            // accumulator buffer (chunk & 1) must have been drained
            if (!bwait(p, &accempty[chunk & 1], ((chunk >> 1) - 1) & 1)) { ok = false; break; }
          }
        } else {
          if (!bwait(p, &bfull[s & 1], (s >> 1) & 1)) { ok = false; break; }
          b_addr = smem_u32(sm + S::NS * S::STAGE_BYTES + (s & 1) * S::BH_BYTES);
        }
        tc_fence_after();
        const uint32_t dcol = tbase + (chunked ? (uint32_t)(chunk & 1) * BN : 0u);
        // Descriptors are built once per stage and stepped by adding the
        // operand offset (in 16-byte units) to their address field: the
        // issuing thread shares its scheduler with busy dequant warps, so
        // each MMA must cost it only a few instructions.
        if constexpr (I8) {
          const uint64_t da0 = sdesc(a_addr, 2048, 128), db0 = sdesc(b_addr, 2048, 128);
#pragma unroll
          for (int bl = 0; bl < S::KB; bl++) {
            if (bl >= nbs) break;
            // one block = K of 32 int8 = one 128 x 128 x 32 MMA
            const int b = b0 + bl;
            const bool first = chunked ? ((b & 15) == 0) : (b == 0);
            const uint64_t off = (uint64_t)(bl * 2 * 2048 / 16);
            mma<true>(dcol, da0 + off, db0 + off, first ? 0u : 1u);
          }
        } else {
          // weights (128 rows) x activations: 128 or 2 npad token rows (SW)
          const int rows = SW ? 2 * p.npad : BM;
          const uint32_t id = (1u << 4) | ((uint32_t)((SW ? rows : BN) >> 3) << 17) |
                              ((uint32_t)(BM >> 4) << 24);
          const uint64_t dw0 = sdesc_sw128(b_addr), dx0 = sdesc_sw128(a_addr);
          const uint32_t w_atom = BN * 128 / 16, x_atom = (uint32_t)rows * 128 / 16;
#pragma unroll
          for (int bl = 0; bl < S::KB; bl++) {
            if (bl >= nbs) break;
#pragma unroll
            for (int kh = 0; kh < 2; kh++) {
              const uint32_t ko = ((bl & 1) * 64 + kh * 32) / 16;  // K offset inside the atom
              const uint64_t dw = dw0 + (uint64_t)((bl >> 1) * w_atom + ko);
              const uint64_t dx = dx0 + (uint64_t)((bl >> 1) * x_atom + ko);
              const uint32_t acc = (b0 + bl == 0 && kh == 0) ? 0u : 1u;
              if constexpr (SW)
                mma_f16_id(dcol, dw, dx, id, acc);  // A = weights, B = tokens
              else
                mma_f16_id(dcol, dx, dw, id, acc);  // A = tokens, B = weights
            }
          }
        }
        mma_commit(&empty[slot]);
        if constexpr (!I8) mma_commit(&bempty[s & 1]);
        if constexpr (I8) {
          if (chunked && (((b0 + nbs) & 15) == 0 || b0 + nbs == p.nblk)) {
            mma_commit(&accfull[chunk & 1]);
            chunk++;
          }
        }
      }
      if (!chunked) mma_commit(&accfull[0]);
      if (!ok)  // release the epilogue of any chunk it still waits for
        for (int c = chunk; c < (chunked ? nchunks : 1); c++) mbar_arrive(&accfull[c & 1]);
    }
  } else {
    // ---------------- warps 2-17: dequantise B / epilogue ---------------
    const int ew = warp - 2;          // 0..7
    const int quarter = warp & 3;     // tensor memory lane quarter of this warp
    const int chalf = ew >> 2;        // epilogue column share: CGW groups of 32 columns
    const int tok = mt * BM + quarter * 32 + lane;
    const uint32_t tq = tbase + ((uint32_t)(quarter * 32) << 16);
    if constexpr (!I8) {
      const int gi = ew & 3, bpar = ew >> 2, row = gi * 32 + lane;
      const bool gvalid = nt * NG + gi < p.groups;
      for (int s = 0; s < nst; s++) {
        const int slot = s % S::NS;
        const bool ok1 = bwait(p, &full[slot], (s / S::NS) & 1);
        const bool ok2 = s < 2 || bwait(p, &bempty[s & 1], ((s >> 1) - 1) & 1);
        const int b0 = s * S::KB, nbs = min(S::KB, p.nblk - b0);
        const uint8_t* raw = sm + slot * S::STAGE_BYTES + S::A_BYTES + gi * S::G_BYTES;
        uint8_t* out = sm + S::NS * S::STAGE_BYTES + (s & 1) * S::BH_BYTES;
        if (ok1 && ok2 && gvalid)
          for (int bl = bpar; bl < nbs; bl += WSETS)
            dequant_block<FMT>(raw, out, lane, row, bl, b0 + bl);
        fence_async_smem();  // generic-proxy smem writes -> visible to the MMA
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bfull[s & 1]);
          mbar_arrive(&empty[slot]);
        }
      }
      // epilogue: fp32 accumulators -> y (nothing on a timed-out wait)
      const bool accok = __all_sync(0xffffffffu, bwait(p, &accfull[0], 0));
      tc_fence_after();
      if constexpr (SW) {
        // lane = weight row; column t = token t's hi part, npad + t its lo
        // part (npad is 16 or 32: columns [0, 32) and, for 32, [32, 64))
        if (chalf == 0 && accok) {
          uint32_t r0[32], r1[32];
          tmem_ld32(tq, r0);
          if (p.npad == 32) tmem_ld32(tq + 32, r1);
          const int n = nt * BN + quarter * 32 + lane;
          if (n < p.n) {
#pragma unroll
            for (int t = 0; t < 32; t++) {
              if (t >= p.npad) break;
              const float hi = __uint_as_float(r0[t]);
              const float lo = __uint_as_float(p.npad == 32 ? r1[t] : r0[16 + (t & 15)]);
              if (t < p.m) p.y[(long long)t * p.ldy + n] = __fmul_rn(__fadd_rn(hi, lo), p.sa[t]);
            }
          }
        }
      }
      for (int h = 0; h < (SW || !accok ? 0 : CGW); h++) {
        const int cg = chalf * CGW + h;
        uint32_t r[32];
        tmem_ld32(tq + cg * 32, r);
        const int n0 = nt * BN + cg * 32;
        if (tok < p.m) {
          float* yr = p.y + (long long)tok * p.ldy;
          const float rs = p.sa[tok];  // 2^s of the row's fp16 scaling
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (n0 + j < p.n) yr[n0 + j] = __fmul_rn(__uint_as_float(r[j]), rs);
        }
      }
    } else {
      const float sa = tok < p.m ? p.sa[tok] : 0.0f;
      if (!chunked) {
        // one int32 accumulator over all of K: float(acc) * sa * sb
        const bool accok = __all_sync(0xffffffffu, bwait(p, &accfull[0], 0));
        tc_fence_after();
        for (int h = 0; h < (accok ? CGW : 0); h++) {
          const int cg = chalf * CGW + h;
          uint32_t r[32];
          tmem_ld32(tq + cg * 32, r);
          const int n0 = nt * BN + cg * 32;
          if (tok < p.m) {
            float* yr = p.y + (long long)tok * p.ldy;
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (n0 + j < p.n)
                yr[n0 + j] = __fmul_rn(__fmul_rn((float)(int)r[j], sa), p.sb[n0 + j]);
          }
        }
      } else {
        // C = 0; per chunk C += float(acc) * sa * sb (running C in tensor
        // memory columns 256..383)
        bool cok = true;  // every chunk arrived (a timeout writes no output)
        for (int c = 0; c < nchunks; c++) {
          cok = __all_sync(0xffffffffu, bwait(p, &accfull[c & 1], (c >> 1) & 1)) && cok;
          tc_fence_after();
          for (int h = 0; h < CGW; h++) {
            const int cg = chalf * CGW + h;
            const int n0 = nt * BN + cg * 32;
            uint32_t r[32], cr[32];
            tmem_ld32(tq + (c & 1) * BN + cg * 32, r);
            if (c > 0) tmem_ld32(tq + 2 * BN + cg * 32, cr);
#pragma unroll
            for (int j = 0; j < 32; j++) {
              const float sbv = (n0 + j < p.n) ? p.sb[n0 + j] : 0.0f;
              const float prev = c > 0 ? __uint_as_float(cr[j]) : 0.0f;
              cr[j] = __float_as_uint(
                  __fadd_rn(prev, __fmul_rn(__fmul_rn((float)(int)r[j], sa), sbv)));
            }
            tmem_st32(tq + 2 * BN + cg * 32, cr);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[c & 1]);
        }
        tc_fence_after();
        for (int h = 0; h < (cok ? CGW : 0); h++) {
          const int cg = chalf * CGW + h;
          uint32_t cr[32];
          tmem_ld32(tq + 2 * BN + cg * 32, cr);
          const int n0 = nt * BN + cg * 32;
          if (tok < p.m) {
            float* yr = p.y + (long long)tok * p.ldy;
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (n0 + j < p.n) yr[n0 + j] = __uint_as_float(cr[j]);
          }
        }
      }
    }
  }
  griddep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                 "r"(S::TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// k_qgemm_tm: block formats, more than 32 tokens. The dequantised weights go
// to tensor memory instead of shared memory: a dequant thread owns one weight
// row, which is one tensor-memory lane, and writes its 32 fp16 values of a
// block with tcgen05.st. The MMA reads them as its A operand (M = 128 weight
// rows) and the token tile (N = up to 256 tokens, swizzled K-major) from
// shared memory as B. Shared memory then carries only the TMA traffic and the
// token-operand reads, instead of also the dequantised tile's writes and
// reads.
//   stage: KB = 2 blocks (64 K) = one 128-byte swizzle atom column of tokens
//   tensor memory: accumulator columns [0, 256) (lane = weight row, column =
//   token); NA weight buffers of AW columns from column 256.
// Split operands (Q4_K, Q6_K): both operands enter as fp16 pairs, weights
// w = wh + wl (dequant_regs<LO>) and tokens x = xh + xl (k_prep_a_f16's lo
// rows), and three MMAs per K step accumulate wh*xh + wh*xl + wl*xh into
// the same fp32 accumulator. The dropped wl*xl term is below 2^-22 of the
// products, so the result is within f32 summation error of the reference's
// f32 dequantise + sgemm (gguf.rs:375-487, matmul.zig:125-347). Without the
// split, a single fp16 rounding of each operand gives 3-6e-4 normwise per
// row, and for Q4_K's and Q6_K's sums up to about 1.1e-3 on narrow rows.
// ---------------------------------------------------------------------------
template <int FMT>
struct TM {
  static constexpr bool SPLIT = FMT == F_Q4_K || FMT == F_Q6_K;
  static constexpr int KB = 2;
  using R = RawG<FMT, KB>;
  static constexpr int X_BYTES = (SPLIT ? 2 : 1) * 256 * 128;  // up to 256 token rows x 128 B (x2)
  static constexpr int RAW_BYTES = NG * R::G_BYTES;
  static constexpr int STAGE_BYTES = (X_BYTES + RAW_BYTES + 1023) / 1024 * 1024;
  static constexpr int NS_FIT = 230400 / STAGE_BYTES;
  static constexpr int NS = NS_FIT < 6 ? NS_FIT : 6;
  static constexpr int SMEM = NS * STAGE_BYTES;
  static constexpr int NA = 4;               // weight buffers in tensor memory
  static constexpr uint32_t AW = SPLIT ? 64 : 32;  // columns per buffer (hi, then lo)
  static constexpr uint32_t A_COL0 = 256;    // first weight-buffer column
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int TN = 256;             // tokens per tile (MMA N, at most)
  static_assert(A_COL0 + NA * AW <= TMEM_COLS, "tensor memory columns");
};

template <int FMT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_qgemm_tm(const GemmParams p) {
  using S = TM<FMT>;
  using R = typename S::R;
  static_assert(FMT != F_INT8, "block formats");
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[S::NS], empty[S::NS];
  __shared__ __align__(8) uint64_t afull[S::NA], aempty[S::NA], accfull;
  __shared__ uint32_t tmem_base_sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x, nt = blockIdx.y;
  const int ntok = p.npad;  // token rows of a tile: min(256, tokens rounded up to 16)
  const int nst = (p.nblk + S::KB - 1) / S::KB;
  constexpr int DQ = 8;     // dequant warps per stage (2 per tensor-memory lane quarter)
  static_assert(WORKERS == 2 * DQ && S::NA % 2 == 0, "two alternating dequant sets");

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + DQ);  // MMA commit + dequant warps
    }
    for (int i = 0; i < S::NA; i++) {
      mbar_init(&afull[i], DQ);
      mbar_init(&aempty[i], 1);
    }
    mbar_init(&accfull, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"(S::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_sh;
  griddep_wait();  // the token tile and sa come from the kernel before

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int ngr = 0;
      for (int gi = 0; gi < NG; gi++)
        if (nt * NG + gi < p.groups) ngr++;
      for (int s = 0; s < nst; s++) {
        const int slot = s % S::NS;
        if (s >= S::NS && !bwait(p, &empty[slot], ((s / S::NS) - 1) & 1)) break;
        const int b0 = s * S::KB, nbs = min(S::KB, p.nblk - b0);
        uint8_t* st = sm + slot * S::STAGE_BYTES;
        uint8_t* raw = st + S::X_BYTES;
        const uint32_t x_bytes = (uint32_t)ntok * 128 * (S::SPLIT ? 2 : 1);
        mbar_expect_tx(&full[slot],
                       x_bytes + ngr * (nbs * (R::QT + R::DT + R::QHT + R::SCT) + R::HT + R::D6T));
        // tokens: [m-tile][stage][ntok rows (hi, then ntok lo rows)][128 B], one copy
        bulk_g2s(st, p.a + ((size_t)mt * p.astg + s) * x_bytes, x_bytes, &full[slot]);
        for (int gi = 0; gi < ngr; gi++) {
          const size_t g = (size_t)nt * NG + gi;
          uint8_t* gr = raw + gi * R::G_BYTES;
          const size_t t0 = g * p.nblk + b0;
          bulk_g2s(gr + R::G_Q, p.q + t0 * R::QT, nbs * R::QT, &full[slot]);
          if constexpr (R::DT)
            bulk_g2s(gr + R::G_D, reinterpret_cast<const uint8_t*>(p.d) + t0 * 64, nbs * 64,
                     &full[slot]);
          if constexpr (R::QHT) {
            bulk_g2s(gr + R::G_QH, p.qh + t0 * 256, nbs * 256, &full[slot]);
            bulk_g2s(gr + R::G_SC, reinterpret_cast<const uint8_t*>(p.sc) + t0 * 64, nbs * 64,
                     &full[slot]);
          }
          if constexpr (R::HT)
            bulk_g2s(gr + R::G_H, p.hdr + (g * p.nsb + b0 / 8) * 512, 512, &full[slot]);
          if constexpr (R::D6T)
            bulk_g2s(gr + R::G_D6,
                     reinterpret_cast<const uint8_t*>(p.d) + (g * p.nsb + b0 / 8) * 64, 64,
                     &full[slot]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id = (1u << 4) | ((uint32_t)(ntok >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      for (int s = 0; s < nst; s++) {
        const int slot = s % S::NS, buf = s % S::NA;
        if (!bwait(p, &full[slot], (s / S::NS) & 1)) break;
        if (!bwait(p, &afull[buf], (s / S::NA) & 1)) break;
        tc_fence_after();
        const int b0 = s * S::KB, nbs = min(S::KB, p.nblk - b0);
        const uint64_t dx0 = sdesc_sw128(smem_u32(sm + slot * S::STAGE_BYTES));
        const uint64_t dxl = dx0 + (uint64_t)(ntok * 128 / 16);  // lo token rows (split)
        const uint32_t ta = tbase + S::A_COL0 + (uint32_t)buf * S::AW;
#pragma unroll
        for (int bl = 0; bl < S::KB; bl++) {
          if (bl >= nbs) break;
#pragma unroll
          for (int kh = 0; kh < 2; kh++) {
            // K offset kh*16 + bl*32 halves: 8 columns of A, 32 bytes of the atom
            const uint32_t tak = ta + (uint32_t)(bl * 16 + kh * 8);
            const uint64_t ko = (uint64_t)((bl * 64 + kh * 32) / 16);
            mma_f16_ts(tbase, tak, dx0 + ko, id, (b0 + bl == 0 && kh == 0) ? 0u : 1u);
            if constexpr (S::SPLIT) {
              mma_f16_ts(tbase, tak, dxl + ko, id, 1u);       // wh * xl
              mma_f16_ts(tbase, tak + 32, dx0 + ko, id, 1u);  // wl * xh
            }
          }
        }
        mma_commit(&empty[slot]);
        mma_commit(&aempty[buf]);
      }
      mma_commit(&accfull);
    }
  } else {
    // ---------------- warps 2-17: dequantise into tensor memory / epilogue ----------------
    const int ew = warp - 2;         // 0..15
    const int quarter = warp & 3;    // tensor-memory lane quarter = row group of the tile
    const uint32_t tq = tbase + ((uint32_t)(quarter * 32) << 16);
    {
      // two sets of DQ warps take alternate stages, so one set's dequant
      // latency overlaps the other's
      const int bl = (ew >> 2) & 1;  // block of the stage this warp dequantises
      const bool gvalid = nt * NG + quarter < p.groups;
      for (int s = ew / DQ; s < nst; s += WORKERS / DQ) {
        const int slot = s % S::NS, buf = s % S::NA;
        const bool ok1 = bwait(p, &full[slot], (s / S::NS) & 1);
        const bool ok2 = s < S::NA || bwait(p, &aempty[buf], ((s / S::NA) - 1) & 1);
        const int b0 = s * S::KB, nbs = min(S::KB, p.nblk - b0);
        // tcgen05.st is warp-wide: the whole warp decides together
        if (__all_sync(0xffffffffu, ok1 && ok2) && gvalid && bl < nbs) {
          const uint8_t* raw = sm + slot * S::STAGE_BYTES + S::X_BYTES + quarter * R::G_BYTES;
          uint32_t o[16], ol[16];
          dequant_regs<FMT, S::KB, S::SPLIT>(raw, lane, bl, b0 + bl, o, ol);
          const uint32_t ta = tq + S::A_COL0 + (uint32_t)buf * S::AW + (uint32_t)bl * 16;
          tmem_st16(ta, o);
          if constexpr (S::SPLIT) tmem_st16(ta + 32, ol);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&afull[buf]);
          mbar_arrive(&empty[slot]);
        }
      }
    }
    // epilogue: lane = weight row, column = token; warp column share
    // [64 cs, 64 cs + 64). A timed-out wait (reported in p.err) writes no
    // output.
    const bool accok = __all_sync(0xffffffffu, bwait(p, &accfull, 0));
    tc_fence_after();
    const int cs = ew >> 2;
    const int n = nt * BN + quarter * 32 + lane;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int c0 = cs * 64 + h * 32;
      if (c0 >= ntok || !accok) break;  // uniform across the warp
      uint32_t r[32];
      tmem_ld32(tq + (uint32_t)c0, r);
      if (n < p.n) {
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int t = mt * S::TN + c0 + j;
          if (c0 + j < ntok && t < p.m)
            p.y[(long long)t * p.ldy + n] = __fmul_rn(__uint_as_float(r[j]), p.sa[t]);
        }
      }
    }
  }
  griddep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                 "r"(S::TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// A preparation: canonical K-major tiles [m-tile][16-byte column][128][16 B]
// ---------------------------------------------------------------------------
// INT8: per-row quantisation (quantize.zig:12-47) or copy of given codes.
__global__ void __launch_bounds__(256) k_prep_a_i8(const float* __restrict__ x,
                                                   const int8_t* __restrict__ xq,
                                                   const float* __restrict__ sx, long long ldx,
                                                   int m, int k, int kcols,
                                                   uint8_t* __restrict__ a,
                                                   float* __restrict__ sa) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;  // 0 .. mtiles*128
  const int mt = row >> 7, rr = row & 127;
  __shared__ float red[8];
  float inv = 0.0f;
  bool zero = true;
  if (row < m && !xq) {
    const float* xr = x + (long long)row * ldx;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < k; i += 256) amax = fmaxf(amax, fabsf(xr[i]));
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
    for (int w = 1; w < 8; w++) amax = fmaxf(amax, red[w]);
    zero = amax == 0.0f;
    if (!zero) inv = __fdiv_rn(127.0f, amax);
    if (threadIdx.x == 0) sa[row] = zero ? 1.0f : __fdiv_rn(amax, 127.0f);
  } else if (row < m) {
    zero = false;
    if (threadIdx.x == 0) sa[row] = sx[row];
  }
  for (int c = threadIdx.x; c < kcols; c += 256) {
    uint32_t wv[4] = {0, 0, 0, 0};
    if (row < m && !zero) {
#pragma unroll
      for (int e = 0; e < 16; e++) {
        const int kk = c * 16 + e;
        int8_t v = 0;
        if (kk < k) {
          if (xq) {
            v = xq[(long long)row * ldx + kk];
          } else {
            float r = roundf(__fmul_rn(x[(long long)row * ldx + kk], inv));
            r = fminf(127.0f, fmaxf(-127.0f, r));
            v = (int8_t)(int)r;
          }
        }
        wv[e >> 2] |= (uint32_t)(uint8_t)v << (8 * (e & 3));
      }
    }
    reinterpret_cast<uint4*>(a + (((size_t)mt * kcols + c) * 128 + rr) * 16)[0] =
        make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// Block formats (tile_rows tokens per tile, rows_pad rows per tile in the
// buffer: 128; 2 npad for the swapped small-M kernel, whose lo_off = npad
// rows further hold x - fp16(x); the tile's token count for k_qgemm_tm,
// twice that for its split formats, lo rows again at lo_off = the token
// count; cps = 16-byte columns per stage: 16, or 8 for k_qgemm_tm):
// fp16(x * 2^-s) per row, with the power of two s chosen so
// that the row's largest magnitude lands in [2^14, 2^15): no fp16 overflow
// and full fp16 precision whatever the activations' range. The scaling is
// exact; the epilogue multiplies the row's accumulators by 2^s (sa[row]).
__global__ void __launch_bounds__(256) k_prep_a_f16(const float* __restrict__ x, long long ldx,
                                                    int m, int k, int kcols,
                                                    uint8_t* __restrict__ a,
                                                    float* __restrict__ sa, int rows_pad, int lo_off,
                                                    int cps, int tile_rows) {
  __shared__ float red[8];
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  const int mt = row / tile_rows, rr = row - mt * tile_rows;
  float inv = 1.0f;
  if (row < m) {
    const float* xr = x + (long long)row * ldx;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < k; i += 256) amax = fmaxf(amax, fabsf(xr[i]));
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
    for (int w = 1; w < 8; w++) amax = fmaxf(amax, red[w]);
    int ex = 0;
    if (amax > 0.0f && amax <= 3.0e38f) {
      frexpf(amax, &ex);  // amax < 2^ex
      ex -= 15;
    }
    inv = ldexpf(1.0f, -ex);
    if (threadIdx.x == 0) sa[row] = ldexpf(1.0f, ex);
  }
  for (int c = threadIdx.x; c < kcols; c += 256) {
    uint32_t wv[4] = {0, 0, 0, 0}, lv[4] = {0, 0, 0, 0};
    if (row < m) {
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int kk = c * 8 + e;
        const float v = kk < k ? __fmul_rn(x[(long long)row * ldx + kk], inv) : 0.0f;
        const __half h = __float2half_rn(v);
        wv[e >> 1] |= (uint32_t)__half_as_ushort(h) << (16 * (e & 1));
        if (lo_off) {
          const __half l = __float2half_rn(__fsub_rn(v, __half2float(h)));
          lv[e >> 1] |= (uint32_t)__half_as_ushort(l) << (16 * (e & 1));
        }
      }
    }
    // swizzled stage tiles: [m-tile][stage of cps columns][atom][rows_pad][128 B]
    const int nstg = (kcols + cps - 1) / cps, sc = c / cps, cc = c - sc * cps;
    uint8_t* tile = a + ((size_t)mt * nstg + sc) * rows_pad * cps * 16;
    *reinterpret_cast<uint4*>(tile + sw128_off(cc, rr, rows_pad)) =
        make_uint4(wv[0], wv[1], wv[2], wv[3]);
    if (lo_off)
      *reinterpret_cast<uint4*>(tile + sw128_off(cc, rr + lo_off, rows_pad)) =
          make_uint4(lv[0], lv[1], lv[2], lv[3]);
  }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl2(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                        cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda directly).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// INT8 weights: view of the row-interleaved tiles as a 4-D byte tensor
// (256 B, 2 halves of a 512-B half-plane, row group, 16-byte K column) whose
// box (256, 2, 4, 2 * KB) lands in shared memory as [K column][128 rows][16 B].
bool make_int8_map(CUtensorMap* map, const syn_cuda_weight_s* w, int groups) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t nblk = w->kp / 32;
  const cuuint64_t dims[4] = {256, 2, (cuuint64_t)groups, 2 * nblk};
  const cuuint64_t strides[3] = {256, nblk * 1024, 512};
  const cuuint32_t box[4] = {256, 2, (cuuint32_t)NG, (cuuint32_t)(2 * GS<F_INT8>::KB)};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w->q, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int FMT, bool SW>
syn_status_t launch_gemm_k(const GemmParams& p, const CUtensorMap& map, int mtiles, int ntiles,
                           cudaStream_t st) {
  static std::mutex mu;
  static std::set<int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> g(mu);
    if (!done.count(dev)) {
      cudaFuncSetAttribute(k_qgemm<FMT, SW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           GS<FMT, SW>::SMEM);
      done.insert(dev);
    }
  }
  cudaError_t e = launch_pdl2(k_qgemm<FMT, SW>, dim3(mtiles, ntiles), dim3(GEMM_THREADS),
                              (size_t)GS<FMT, SW>::SMEM, st, p, map);
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "k_qgemm");
    return SYN_ERR_CUDA;
  }
  return SYN_OK;
}

template <int FMT>
syn_status_t launch_gemm_t(const GemmParams& p, const CUtensorMap& map, int mtiles, int ntiles,
                           cudaStream_t st) {
  if constexpr (FMT != F_INT8)
    if (p.npad) return launch_gemm_k<FMT, true>(p, map, 1, ntiles, st);
  return launch_gemm_k<FMT, false>(p, map, mtiles, ntiles, st);
}

template <int FMT>
syn_status_t launch_tm(const GemmParams& p, int mtiles, int ntiles, cudaStream_t st) {
  static std::mutex mu;
  static std::set<int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> g(mu);
    if (!done.count(dev)) {
      cudaFuncSetAttribute(k_qgemm_tm<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TM<FMT>::SMEM);
      done.insert(dev);
    }
  }
  cudaError_t e = launch_pdl2(k_qgemm_tm<FMT>, dim3(mtiles, ntiles), dim3(GEMM_THREADS),
                              (size_t)TM<FMT>::SMEM, st, p);
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "k_qgemm_tm");
    return SYN_ERR_CUDA;
  }
  return SYN_OK;
}

}  // namespace

// Split-operand formats of k_qgemm_tm (hi and lo fp16 parts of both
// operands); they take k_qgemm_tm from 33 rows, above the swapped kernel.
bool tm_split_fmt(int fmt) { return fmt == SYN_QFMT_Q4_K || fmt == SYN_QFMT_Q6_K; }

size_t gemm_a_bytes(int fmt, size_t m, size_t kp) {
  // fp16: whole stages of 16 columns (the swizzled tiles), rows for 256-token
  // tiles (k_qgemm_tm, twice for the split formats' lo rows) or 128-token
  // tiles, whichever is more
  const bool i8 = fmt == SYN_QFMT_INT8_KN;
  const size_t rows = i8 ? (m + BM - 1) / BM * BM
                         : (m + 255) / 256 * 256 * (tm_split_fmt(fmt) ? 2 : 1);
  const size_t kcols = i8 ? kp / 16 : (kp / 8 + 15) / 16 * 16;
  return rows * kcols * 16 + rows * sizeof(float) + 256;
}

size_t gemm_min_rows(int fmt, size_t n) {
  static const size_t forced = [] {
    const char* v = getenv("SYN_GEMM_MIN_ROWS");
    return v ? (size_t)atoll(v) : (size_t)0;
  }();
  if (forced) return forced;
  (void)fmt;
  // The GEMM runs one CTA per 128 weight rows over all of K, so with few
  // row tiles it is latency-bound and the GEMV (all SMs, weights re-read
  // from L2 per 4-row slice) is faster. Crossovers measured on B200: N =
  // 2048 -> GEMV up to 32 rows; N = 4096 -> up to about 16; N = 14336 -> the
  // GEMM from 8 rows.
  if (n >= 8192) return 8;
  if (n >= 4096) return 24;
  return 40;
}

syn_status_t launch_qgemm(const syn_cuda_weight_s* w, const float* x, size_t ldx,
                          const int8_t* xq, const float* sx, size_t m, float* y, size_t ldy,
                          int chunked, uint8_t* abuf, int* err, cudaStream_t st) {
  if (w->n > 0x7FFFFFFFull || w->kp > 0x3FFFFFFFull || m > 0x7FFFFFFFull) return SYN_ERR_UNSUPPORTED;
  const bool i8 = w->fmt == SYN_QFMT_INT8_KN;
  const int mtiles = (int)((m + BM - 1) / BM);
  const int groups = (int)((w->n + 31) / 32);
  const int ntiles = (groups + NG - 1) / NG;
  const int kcols = (int)(i8 ? w->kp / 16 : w->kp / 8);
  alignas(64) CUtensorMap map;
  memset(&map, 0, sizeof(map));
  if (i8 && !make_int8_map(&map, w, groups)) return SYN_ERR_UNSUPPORTED;
  // few tokens (block formats): the swapped-operand kernel, tokens padded to
  // a multiple of 16
  static const int swap_max = [] {
    const char* v = getenv("SYN_GEMM_SWAP_MAX");
    return v ? atoi(v) : 32;
  }();
  const int npad =
      (!i8 && (long long)m <= std::min(swap_max, 32)) ? (int)((m + 15) / 16 * 16) : 0;
  // more than 128 tokens (block formats): weights in tensor memory, tiles of
  // up to 256 tokens (k_qgemm_tm). Measured on B200 (Q4_0 14336x4096): 64
  // tokens 53 us vs 44 us on the 128-token tiles, 512 tokens 109 vs 177 us,
  // 2048 tokens 347 vs 611 us.
  // Q4_K and Q6_K (split operands, the f32-grade path) take it from 33 rows.
  static const int tm_min_env = [] {
    const char* v = getenv("SYN_GEMM_TM_MIN_ROWS");
    return v ? atoi(v) : -1;
  }();
  const bool split = tm_split_fmt(w->fmt);
  const int tm_min = tm_min_env >= 0 ? tm_min_env : split ? 33 : 129;
  const bool tm = !i8 && !npad && tm_min > 0 && (long long)m >= tm_min;
  const int tm_tiles = (int)((m + 255) / 256);
  const int tm_ntok = m >= 256 ? 256 : (int)((m + 15) / 16 * 16);
  uint8_t* a = abuf;
  const int acols = i8 ? kcols : (kcols + 15) / 16 * 16;  // fp16: whole swizzled stages
  const size_t a_rows = i8 ? (size_t)mtiles * BM : (m + 255) / 256 * 256 * (split ? 2 : 1);
  float* sa = reinterpret_cast<float*>(abuf + a_rows * acols * 16);
  cudaError_t e;
  if (i8)
    e = launch_pdl2(k_prep_a_i8, dim3(mtiles * BM), dim3(256), 0, st, x, xq, sx, (long long)ldx,
                    (int)m, (int)w->k, kcols, a, sa);
  else
    e = launch_pdl2(k_prep_a_f16, dim3(tm ? tm_tiles * tm_ntok : npad ? npad : mtiles * BM),
                    dim3(256), 0, st, x, (long long)ldx, (int)m, (int)w->k, kcols, a, sa,
                    tm ? tm_ntok * (split ? 2 : 1) : npad ? 2 * npad : BM,
                    tm ? (split ? tm_ntok : 0) : npad, tm ? 8 : 16,
                    tm ? tm_ntok : npad ? 2 * npad : BM);
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "k_prep_a");
    return SYN_ERR_CUDA;
  }
  GemmParams p{};
  p.q = w->q;
  p.d = w->d;
  p.sb = w->sb;
  p.hdr = w->hdr;
  p.qh = w->qh;
  p.sc = reinterpret_cast<const uint16_t*>(w->sc);
  p.n = (int)w->n;
  p.k = (int)w->k;
  p.nblk = (int)(w->kp / 32);
  p.nsb = (int)(w->k / 256);
  p.groups = groups;
  p.a = a;
  p.kcols = kcols;
  p.sa = sa;
  p.m = (int)m;
  p.y = y;
  p.ldy = (long long)ldy;
  p.chunked = chunked;
  p.err = err;
  static const int short_rows = [] {
    const char* v = getenv("SYN_GEMM_SHORT_ROWS");
    return v ? atoi(v) : 64;
  }();
  p.short_rows = short_rows;
  p.npad = tm ? tm_ntok : npad;
  p.astg = tm ? (kcols + 7) / 8 : (kcols + 15) / 16;
  if (tm) {
    switch (w->fmt) {
      case SYN_QFMT_Q4_0: return launch_tm<F_Q4_0>(p, tm_tiles, ntiles, st);
      case SYN_QFMT_Q8_0: return launch_tm<F_Q8_0>(p, tm_tiles, ntiles, st);
      case SYN_QFMT_Q4_K: return launch_tm<F_Q4_K>(p, tm_tiles, ntiles, st);
      case SYN_QFMT_Q6_K: return launch_tm<F_Q6_K>(p, tm_tiles, ntiles, st);
    }
    return SYN_ERR_INVALID_ARG;
  }
  switch (w->fmt) {
    case SYN_QFMT_INT8_KN: return launch_gemm_t<F_INT8>(p, map, mtiles, ntiles, st);
    case SYN_QFMT_Q4_0: return launch_gemm_t<F_Q4_0>(p, map, mtiles, ntiles, st);
    case SYN_QFMT_Q8_0: return launch_gemm_t<F_Q8_0>(p, map, mtiles, ntiles, st);
    case SYN_QFMT_Q4_K: return launch_gemm_t<F_Q4_K>(p, map, mtiles, ntiles, st);
    case SYN_QFMT_Q6_K: return launch_gemm_t<F_Q6_K>(p, map, mtiles, ntiles, st);
  }
  return SYN_ERR_INVALID_ARG;
}

}  // namespace syn
