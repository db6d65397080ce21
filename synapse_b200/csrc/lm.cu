// lm.cu -- the decoder-layer kernels around the quantized matmuls: RMSNorm
// (fused with the residual add and, for layer 0, the embedding gather),
// headwise q/k RMSNorm + RoPE + KV-cache append, cached GQA attention
// (decode, fused with the norm/RoPE/append of its own heads; prefill), SwiGLU
// and greedy argmax.
//
// Every reduction follows the reference's order, so that a greedy decode
// reproduces the reference's token ids:
//   * RMSNorm sums x*x in four lane accumulators of stride 4, adds the lanes
//     in order, then the tail (vecHsum, zig/src/ffi/exports.zig:503-514);
//   * attention dot products and weighted sums are sequential chains over the
//     head dimension / positions, with fused multiply-add exactly where the
//     reference's f32 GEMV/GEMM uses @mulAdd (zig/src/ops/matmul.zig:
//     223-343, 452-515) and a rounded multiply then add where it writes
//     `sum += a * b` (ops/attention.rs:118-144, the edge tiles);
//   * the softmax sum is sequential (ops/activation.rs:117-130); the prefill
//     online softmax keeps the reference's running (max, sum) recurrence
//     (exports.zig:1420-1436), with the exponentials evaluated in parallel
//     once the running maxima are known (a prefix-max scan);
//   * exp is evaluated in double and rounded once to float (the correctly
//     rounded expf except in rare ties), the same function as the CPU oracle.
// Long-context attention therefore runs on the CUDA cores as sequential
// chains; its cost is latency of the chain, not bandwidth.
#include <math.h>

#include <algorithm>
#include <mutex>
#include <new>
#include <set>

#include <cuda_bf16.h>

#include "internal.cuh"

namespace syn {
namespace {


// one step of a sum-of-products chain: fused (@mulAdd) or two roundings
__device__ __forceinline__ float chain(bool fused, float a, float b, float acc) {
  return fused ? __fmaf_rn(a, b, acc) : __fadd_rn(acc, __fmul_rn(a, b));
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
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

syn_status_t allow_smem(const void* fn, size_t bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  if (bytes <= 48 * 1024) return SYN_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  if (done.count({fn, dev})) return SYN_OK;
  // the most dynamic shared memory the kernel can have next to its static part
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, fn);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(227 * 1024 - fa.sharedSizeBytes));
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "cudaFuncSetAttribute");
    return SYN_ERR_CUDA;
  }
  done.insert({fn, dev});
  return SYN_OK;
}

constexpr size_t kMaxSmem = 200 * 1024;

// ---------------------------------------------------------------------------
// RMSNorm, fused with the residual add / embedding gather
// ---------------------------------------------------------------------------
constexpr int NORM_THREADS = 256;

struct NormParams {
  const float* x;      // input rows (unused when ids != nullptr)
  long long ldx;
  const float* delta;  // optional: x + delta is normalised (and stored in x_out)
  long long ldd;
  const int32_t* ids;  // optional: rows are embedding rows table[ids[r]]
  const float* table;
  unsigned vocab;
  float* x_out;        // optional: the (residual) input row actually normalised
  long long ldxo;
  const float* w;
  int h;
  float eps;
  float* out;
  long long ldo;
  int fast;            // 1: parallel sum of squares (block-format models)
};

// sum of squares in the reference's order; every thread returns the same value
__device__ float norm_scale(const float* sx, int h, float eps, float* lane) {
  if (threadIdx.x < 4) {
    const int n4 = h & ~3;
    float acc = 0.0f;
    int i = threadIdx.x;
    for (; i + 60 < n4; i += 64) {  // 16 loads in flight, then the add chain
      float v[16];
#pragma unroll
      for (int u = 0; u < 16; u++) v[u] = sx[i + 4 * u];
#pragma unroll
      for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, __fmul_rn(v[u], v[u]));
    }
    for (; i < n4; i += 4) acc = __fadd_rn(acc, __fmul_rn(sx[i], sx[i]));
    lane[threadIdx.x] = acc;
  }
  __syncthreads();
  float s = __fadd_rn(__fadd_rn(__fadd_rn(lane[0], lane[1]), lane[2]), lane[3]);
  for (int i = h & ~3; i < h; i++) s = __fadd_rn(s, __fmul_rn(sx[i], sx[i]));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)h), eps)));
}

__global__ void __launch_bounds__(NORM_THREADS) k_add_rmsnorm(const NormParams p) {
  extern __shared__ float sx[];
  __shared__ float lane[4];
  griddep_wait();
  const int row = blockIdx.x;
  const float* src = p.x + row * p.ldx;
  bool zero = false;
  if (p.ids) {
    const unsigned id = (unsigned)p.ids[row];
    zero = id >= p.vocab;  // ids outside the vocabulary embed as zeros
    src = p.table + (size_t)(zero ? 0 : id) * p.h;
  }
  // all loads of a batch are issued before any store (x_out may alias x)
  constexpr int NV = 8;
  const int tid = threadIdx.x;
  for (int j0 = 0; j0 < p.h; j0 += NORM_THREADS * NV) {
    float v[NV], dl[NV];
#pragma unroll
    for (int u = 0; u < NV; u++) {
      const int j = j0 + tid + u * NORM_THREADS;
      v[u] = (j < p.h && !zero) ? src[j] : 0.0f;
      dl[u] = (j < p.h && p.delta) ? p.delta[row * p.ldd + j] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < NV; u++) {
      const int j = j0 + tid + u * NORM_THREADS;
      if (j < p.h) {
        const float x = p.delta ? __fadd_rn(v[u], dl[u]) : v[u];
        sx[j] = x;
        if (p.x_out) p.x_out[row * p.ldxo + j] = x;
      }
    }
  }
  __syncthreads();
  float scale;
  if (p.fast) {  // tree sum: a parallel order, for models with a tolerance
    __shared__ float red[NORM_THREADS / 32];
    float a = 0.0f;
    for (int j = tid; j < p.h; j += NORM_THREADS) a = fmaf(sx[j], sx[j], a);
    for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if ((tid & 31) == 0) red[tid >> 5] = a;
    __syncthreads();
    float ss = 0.0f;
    for (int w = 0; w < NORM_THREADS / 32; w++) ss += red[w];
    scale = 1.0f / sqrtf(ss / (float)p.h + p.eps);
  } else {
    scale = norm_scale(sx, p.h, p.eps, lane);
  }
  griddep_launch();
  for (int j0 = 0; j0 < p.h; j0 += NORM_THREADS * NV) {
    float wv[NV];
#pragma unroll
    for (int u = 0; u < NV; u++) {
      const int j = j0 + tid + u * NORM_THREADS;
      wv[u] = j < p.h ? p.w[j] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < NV; u++) {
      const int j = j0 + tid + u * NORM_THREADS;
      if (j < p.h) p.out[row * p.ldo + j] = __fmul_rn(__fmul_rn(sx[j], wv[u]), scale);
    }
  }
}

// ---------------------------------------------------------------------------
// Shared by the attention kernels: where q/k/v rows live, the cache, RoPE
// ---------------------------------------------------------------------------
struct AttnParams {
  float* q;            // q rows (row stride ld); prefill rewrites them in place
  const float* k;      // k rows (row stride ld)
  const float* v;      // v rows (row stride ld)
  long long ld;
  int n_heads, n_kv, hd;
  const float* qn;     // optional headwise norm weights [hd]
  const float* kn;
  float eps;
  const float* cos_t;  // [max_pos, hd/2]
  const float* sin_t;
  int window;          // 0 = none
  float* kc;           // cache of this layer: [batch][max_seq][n_kv*hd]
  float* vc;
  int max_seq;
  const int* len;      // [batch] positions already committed
  int seq0;            // prefill: the sequence; decode: row b is sequence b
  int n_tokens;        // prefill tokens
  // Decode kernels, span mode: row b is position len[seq0] + b of sequence
  // seq0 (a multi-token verification step); q is already normalised and
  // rotated and K/V already appended (k_norm_rope_append with rope_at_slot).
  int span;
  // Paged cache: position `pos` of sequence `sq` lives in slot
  // ptab[sq * maxp + pos / page] * page + pos % page of the layer's pool;
  // ptab == nullptr: contiguous, slot sq * max_seq + pos.
  const int* ptab;
  int page, maxp;
  // Decode kernels: row b's sequence is slots[b] (nullptr: b).
  const int* slots;
  // k_norm_rope_append: RoPE at the cache slot (len + t) instead of the
  // reference prefill's offset t (attention.rs:171-190)
  int rope_at_slot;
  // k_attn_decode: K / V rows staged in shared memory (set by the launch)
  int krows, vrows;
  float* out;          // [rows][n_heads*hd]
  long long ldo;
  float scale;
  int* err;
};

// Cache slot (row index of the layer's K/V pool) of position pos of sequence sq.
__device__ __forceinline__ size_t kv_slot(const AttnParams& p, int sq, int pos) {
  if (!p.ptab) return (size_t)sq * p.max_seq + pos;
  return (size_t)p.ptab[(size_t)sq * p.maxp + pos / p.page] * p.page + pos % p.page;
}

// Headwise RMSNorm of `nv` vectors of length hd in smem (x, in place), with
// weight w (nullptr = identity), then RotateHalf RoPE at position pos
// (ops/norm.rs:78-92, ops/rope.rs:13-60). `lanes`: 4*nv floats, `scl`: nv.
__device__ void norm_rope(float* x, int nv, int hd, const float* wq, const float* wk, int nq,
                          float eps, const float* cos_t, const float* sin_t, int pos,
                          float* lanes, float* scl, int nthreads) {
  const int tid = threadIdx.x;
  for (int t = tid; t < 4 * nv; t += nthreads) {
    const int vi = t >> 2, l = t & 3;
    const float* xv = x + vi * hd;
    float acc = 0.0f;
    for (int i = l; i < (hd & ~3); i += 4) acc = __fadd_rn(acc, __fmul_rn(xv[i], xv[i]));
    lanes[t] = acc;
  }
  __syncthreads();
  for (int vi = tid; vi < nv; vi += nthreads) {
    const float* xv = x + vi * hd;
    const float* ln = lanes + 4 * vi;
    float s = __fadd_rn(__fadd_rn(__fadd_rn(ln[0], ln[1]), ln[2]), ln[3]);
    for (int i = hd & ~3; i < hd; i++) s = __fadd_rn(s, __fmul_rn(xv[i], xv[i]));
    scl[vi] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)hd), eps)));
  }
  __syncthreads();
  const int half = hd >> 1;
  for (int t = tid; t < nv * half; t += nthreads) {
    const int vi = t / half, i = t - vi * half;
    float* xv = x + vi * hd;
    const float* w = vi < nq ? wq : wk;
    float x1 = xv[i], x2 = xv[half + i];
    if (w) {
      x1 = __fmul_rn(__fmul_rn(x1, w[i]), scl[vi]);
      x2 = __fmul_rn(__fmul_rn(x2, w[half + i]), scl[vi]);
    }
    const float c = cos_t[(size_t)pos * half + i], s = sin_t[(size_t)pos * half + i];
    xv[i] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    xv[half + i] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
  __syncthreads();
}

// Sequential left-to-right sum (the reference's `sum += x`), with the smem
// loads issued in batches so that only the add chain is serial.
__device__ __forceinline__ float serial_sum(const float* r, int n) {
  float sum = 0.0f;
  int s = 0;
  for (; s + 16 <= n; s += 16) {
    float v[16];
#pragma unroll
    for (int u = 0; u < 16; u++) v[u] = r[s + u];
#pragma unroll
    for (int u = 0; u < 16; u++) sum = __fadd_rn(sum, v[u]);
  }
  for (; s < n; s++) sum = __fadd_rn(sum, r[s]);
  return sum;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < nw; i++) m = fmaxf(m, red[i]);
  return m;
}

constexpr int DEC_THREADS = 128;
constexpr int DEC_KR = DEC_THREADS;  // K rows staged (one per thread)
constexpr int DEC_VMAX = 256;        // V rows staged per pass

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Copies cached rows [ra, rb) (positions off + r) of one KV head into
// staged rows r * VS, 16 bytes per copy, all threads.
template <int HD>
__device__ __forceinline__ void stage_rows_async(float* dst, const float* cb, const AttnParams& p,
                                                 int sq, int off, int ra, int rb, int kvd) {
  constexpr int Q4 = HD / 4, VS = HD + 4;
  for (int t = threadIdx.x + ra * Q4; t < rb * Q4; t += DEC_THREADS) {
    const int r = t / Q4, c4 = t - r * Q4;
    cp_async16(dst + r * VS + 4 * c4, cb + kv_slot(p, sq, off + r) * kvd + 4 * c4);
  }
}

// acc = q . k in element order, each product rounded then added, or fused
// (the reference's @mulAdd), as chain() does
template <int HD>
__device__ __forceinline__ float dot_in_order(const float* q, const float* k, bool fused) {
  const float4* q4 = reinterpret_cast<const float4*>(q);
  const float4* k4 = reinterpret_cast<const float4*>(k);
  float acc = 0.0f;
  if (fused) {
#pragma unroll 4
    for (int c = 0; c < HD / 4; c++) {
      const float4 a = q4[c], b = k4[c];
      acc = __fmaf_rn(a.x, b.x, acc);
      acc = __fmaf_rn(a.y, b.y, acc);
      acc = __fmaf_rn(a.z, b.z, acc);
      acc = __fmaf_rn(a.w, b.w, acc);
    }
  } else {
#pragma unroll 4
    for (int c = 0; c < HD / 4; c++) {
      const float4 a = q4[c], b = k4[c];
      acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
      acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
      acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
      acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
    }
  }
  return acc;
}

// Decode: one CTA of DEC_THREADS per (row, query head):
// cached_attention_decode (ops/attention.rs:24-147), in its order. Every CTA
// of a KV group normalises and rotates the new K itself (same bits), the
// group's first CTA appends K and V to the cache, and the new position is
// read from shared memory, so no CTA waits for another. The first DEC_KR K
// rows and the first p.vrows V rows of the context are copied into shared
// memory with cp.async before griddepcontrol.wait (they were written by
// earlier steps), so their latency overlaps the preceding QKV matmul and no
// row lives in registers.
template <int HD>
__global__ void __launch_bounds__(DEC_THREADS) k_attn_decode(const AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  constexpr int VS = HD + 4;             // staged row stride (conflict-free float4 rows)
  const int KR = p.krows, VR = p.vrows;  // staged K / V rows (<= the longest context)
  float* xs = sm;                        // q (HD) then k (HD), then v (HD)
  float* cs = xs + 3 * HD;               // RoPE cos (HD/2) then sin (HD/2) at pos
  float* kst = cs + HD;                  // KR staged K rows
  float* vst = kst + KR * VS;            // VR staged V rows
  float* lanes = vst + VR * VS;          // 8
  float* scl = lanes + 8;                // 2 (+2 pad)
  float* red = scl + 4;                  // DEC_THREADS / 32
  float* sc = red + DEC_THREADS / 32;    // scores, eff
  const int b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int G = p.n_heads / p.n_kv, kvh = h / G, kvd = p.n_kv * HD;
  // Before griddepcontrol.wait only data written two or more kernels back is
  // read: the committed length (argmax of the previous step), the cached
  // rows below it (previous steps' attention) and the RoPE tables. Span
  // mode: rows from len0 on were appended by the kernel before, so only rows
  // below len0 are read early.
  const int sq = p.span ? p.seq0 : p.slots ? p.slots[b] : b;  // this row's sequence
  const int len0 = p.len[sq];
  const int pos = p.span ? len0 + b : len0;
  const int early = p.span ? len0 : pos;  // rows [0, early) may be read before the wait
  if (pos >= p.max_seq) {  // cache full: nothing is written (the host reports it)
    griddep_wait();
    if (tid == 0 && p.err) atomicExch(p.err, SYN_ERR_INVALID_ARG);
    return;
  }
  float* kcb = p.kc + kvh * HD;  // row r of the sequence: + kv_slot(p, sq, r) * kvd
  float* vcb = p.vc + kvh * HD;
  const int L = pos + 1;
  const int off = (p.window > 0 && L > p.window) ? L - p.window : 0;
  const int eff = L - off;
  const bool fresh = !p.span;  // the new row's K/V come from q/k/v, not the cache
  for (int i = tid; i < HD / 2; i += DEC_THREADS) {
    cs[i] = p.cos_t[(size_t)pos * (HD / 2) + i];
    cs[HD / 2 + i] = p.sin_t[(size_t)pos * (HD / 2) + i];
  }
  const int kn = min(KR, eff), vn = min(VR, eff);
  const int pre = max(0, min(early - off, eff));  // staged rows available before the wait
  stage_rows_async<HD>(kst, kcb, p, sq, off, 0, min(kn, pre), kvd);
  stage_rows_async<HD>(vst, vcb, p, sq, off, 0, min(vn, pre), kvd);
  griddep_wait();
  const float* qrow = p.q + (long long)b * p.ld + (long long)h * HD;
  const float* krow = p.k + (long long)b * p.ld + (long long)kvh * HD;
  const float* vrow = p.v + (long long)b * p.ld + (long long)kvh * HD;
  if (!fresh) {  // q is ready; this step's K/V rows are in the cache
    for (int i = tid; i < HD; i += DEC_THREADS) xs[i] = qrow[i];
    stage_rows_async<HD>(kst, kcb, p, sq, off, min(kn, pre), kn, kvd);
    stage_rows_async<HD>(vst, vcb, p, sq, off, min(vn, pre), vn, kvd);
    __syncthreads();
  } else {
    for (int i = tid; i < HD; i += DEC_THREADS) {
      xs[i] = qrow[i];
      xs[HD + i] = krow[i];
      xs[2 * HD + i] = vrow[i];
    }
    __syncthreads();
    norm_rope(xs, 2, HD, p.qn, p.kn, 1, p.eps, cs, cs + HD / 2, 0, lanes, scl, DEC_THREADS);
    if (h % G == 0)
      for (int i = tid; i < HD; i += DEC_THREADS) {
        kcb[kv_slot(p, sq, pos) * kvd + i] = xs[HD + i];
        vcb[kv_slot(p, sq, pos) * kvd + i] = xs[2 * HD + i];
      }
    // the new row into the staged rows (it is the last of the context)
    const int r = pos - off;
    for (int i = tid; i < HD; i += DEC_THREADS) {
      if (r < kn) kst[r * VS + i] = xs[HD + i];
      if (r < vn) vst[r * VS + i] = xs[2 * HD + i];
    }
  }
  cp_async_wait_all();
  __syncthreads();

  // scores: below 64 positions the reference's scalar loop (sum += a*b);
  // from 64 on matmul_t (@mulAdd except the last eff%8 columns)
  const int s_full = eff < 64 ? 0 : eff - (eff & 7);
  for (int s = tid; s < eff; s += DEC_THREADS) {
    const int row = off + s;
    const float* kr = s < kn                   ? kst + s * VS
                      : (row == pos && fresh) ? xs + HD
                                              : kcb + kv_slot(p, sq, row) * kvd;
    sc[s] = __fmul_rn(dot_in_order<HD>(xs, kr, s < s_full), p.scale);
  }
  __syncthreads();
  // softmax_slice (ops/activation.rs:117-130)
  float mx = -INFINITY;
  for (int s = tid; s < eff; s += DEC_THREADS) mx = fmaxf(mx, sc[s]);
  mx = block_max(mx, red);
  for (int s = tid; s < eff; s += DEC_THREADS) sc[s] = exp_f32(__fsub_rn(sc[s], mx));
  __syncthreads();
  if (tid == 0) red[0] = serial_sum(sc, eff);
  __syncthreads();
  const float sum = red[0];
  if (sum > 0.0f)
    for (int s = tid; s < eff; s += DEC_THREADS) sc[s] = __fdiv_rn(sc[s], sum);
  griddep_launch();
  // score * V: below 64 positions sum += p*v; from 64 on matmul_nn
  // (@mulAdd except the last hd%32 columns). Rows past the staged ones pass
  // through the same buffer VR at a time.
  const bool vfused = eff >= 64 && tid < HD - (HD & 31);
  float acc = 0.0f;
  for (int c0 = 0; c0 < eff; c0 += VR) {
    const int cn = min(VR, eff - c0);
    if (c0 > 0) {
      __syncthreads();  // the previous rows are consumed (and sc is final)
      stage_rows_async<HD>(vst, vcb, p, sq, off + c0, 0, cn, kvd);
      cp_async_wait_all();
      __syncthreads();
      if (fresh && pos - off - c0 < cn) {  // the new row was not in the cache when staged
        for (int i = tid; i < HD; i += DEC_THREADS) vst[(pos - off - c0) * VS + i] = xs[2 * HD + i];
        __syncthreads();
      }
    }
    if (tid < HD) {
      const float* pr = sc + c0;
      int s = 0;
      for (; s + 8 <= cn; s += 8) {
        float pv[8], vv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
          pv[u] = pr[s + u];
          vv[u] = vst[(s + u) * VS + tid];
        }
#pragma unroll
        for (int u = 0; u < 8; u++) acc = chain(vfused, pv[u], vv[u], acc);
      }
      for (; s < cn; s++) acc = chain(vfused, pr[s], vst[s * VS + tid], acc);
    }
  }
  if (tid < HD) p.out[(long long)b * p.ldo + (long long)h * HD + tid] = acc;
}

// Staged rows of k_attn_decode for contexts up to `eff` positions.
void decode_stage_rows(int hd, int eff, int* kr, int* vr) {
  *kr = std::min(eff, DEC_KR);
  int v = std::min(eff, DEC_VMAX);
  auto bytes = [&](int vv) {
    return ((size_t)4 * hd + (size_t)(*kr + vv) * (hd + 4) + 8 + 4 + DEC_THREADS / 32 + eff) *
           sizeof(float);
  };
  while (v > 8 && bytes(v) > kMaxSmem) v /= 2;
  *vr = v;
}

size_t decode_smem_floats(int hd, int eff) {
  int kr, vr;
  decode_stage_rows(hd, eff, &kr, &vr);
  return (size_t)4 * hd + (size_t)(kr + vr) * (hd + 4) + 8 + 4 + DEC_THREADS / 32 + eff;
}

// ---------------------------------------------------------------------------
// Prefill step 1: headwise norm + RoPE of every q/k head in place, K and raw
// V appended to the cache at positions len[seq] + t.
// grid (tokens, n_heads + n_kv), block hd/2 (>= 32)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) k_norm_rope_append(const AttnParams p) {
  extern __shared__ float sm[];
  const int t = blockIdx.x, hh = blockIdx.y, hd = p.hd, kvd = p.n_kv * hd;
  const bool is_q = hh < p.n_heads;
  float* xs = sm;
  float* lanes = xs + hd;
  float* scl = lanes + 4;
  griddep_wait();
  const int slot = p.len[p.seq0] + t;  // cache slot; RoPE uses offset 0 (attention.rs:171-190)
  if (slot >= p.max_seq) {
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, SYN_ERR_INVALID_ARG);
    return;
  }
  float* src = is_q ? p.q + (long long)t * p.ld + (long long)hh * hd
                    : const_cast<float*>(p.k) + (long long)t * p.ld + (long long)(hh - p.n_heads) * hd;
  for (int i = threadIdx.x; i < hd; i += blockDim.x) xs[i] = src[i];
  __syncthreads();
  norm_rope(xs, 1, hd, is_q ? p.qn : p.kn, nullptr, 1, p.eps, p.cos_t, p.sin_t,
            p.rope_at_slot ? slot : t, lanes, scl, blockDim.x);
  griddep_launch();
  if (is_q) {
    for (int i = threadIdx.x; i < hd; i += blockDim.x) src[i] = xs[i];
  } else {
    const int kh = hh - p.n_heads;
    float* kd = p.kc + kv_slot(p, p.seq0, slot) * kvd + kh * hd;
    float* vd = p.vc + kv_slot(p, p.seq0, slot) * kvd + kh * hd;
    const float* vs = p.v + (long long)t * p.ld + (long long)kh * hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
      kd[i] = xs[i];
      vd[i] = vs[i];
    }
  }
}

// ---------------------------------------------------------------------------
// Prefill step 2: syn_fused_attention (zig/src/ffi/exports.zig:1364-1478) per
// head over the prompt: CTA = (head, PR query rows), 256 threads.
// Chain kinds follow sgemmTiled per 32-row query tile (TILE_Q,
// zig/src/ops/attention.zig:25): tiles of <= 16 rows use the per-row GEMV
// (@mulAdd except trailing columns), larger tiles the 8x8 micro-kernels
// (@mulAdd in full tiles, sum += a*b in edge tiles).
// ---------------------------------------------------------------------------
constexpr int PF_THREADS = 256;
constexpr int PF_CH = 32;  // keys staged per chunk

// Copies cache rows row0 .. row0+cn-1 of sequence sq (hd floats each from
// `cache`, which points at the head's columns) into smem rows of stride ss,
// all loads of a thread issued before its stores.
__device__ __forceinline__ void stage_rows_pf(float* dst, int ss, const float* cache,
                                              const AttnParams& p, int sq, int row0, int kvd,
                                              int cn, int hd, int tid) {
  const int q = hd >> 2, tot = cn * q;
  constexpr int U = 8;
  for (int t0 = 0; t0 < tot; t0 += U * PF_THREADS) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int t = t0 + tid + u * PF_THREADS;
      if (t < tot) {
        const int r = t / q, c4 = t - r * q;
        v[u] = *reinterpret_cast<const float4*>(cache + kv_slot(p, sq, row0 + r) * kvd + 4 * c4);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int t = t0 + tid + u * PF_THREADS;
      if (t < tot) {
        const int r = t / q, c4 = t - r * q;
        *reinterpret_cast<float4*>(dst + r * ss + 4 * c4) = v[u];
      }
    }
  }
}

__device__ __forceinline__ void tile_of(int q, int S, int& tqs, int& i) {
  const int tq = q & ~31;
  tqs = min(32, S - tq);
  i = q - tq;
}
__device__ __forceinline__ bool s_fused(int q, int j, int S) {
  int tqs, i;
  tile_of(q, S, tqs, i);
  const bool jfull = j < S - (S & 7);
  if (tqs <= 16) return jfull;
  return i < tqs - (tqs & 7) && jfull;
}
__device__ __forceinline__ bool o_fused(int q, int d, int S, int hd) {
  int tqs, i;
  tile_of(q, S, tqs, i);
  if (tqs <= 16) return d < hd - (hd & 31);
  return i < tqs - (tqs & 7) && d < hd - (hd & 7);
}

__global__ void __launch_bounds__(PF_THREADS) k_attn_prefill(const AttnParams p, int PR) {
  extern __shared__ float sm[];
  const int hh = blockIdx.x, r0 = blockIdx.y * PR;
  const int G = p.n_heads / p.n_kv, kvh = hh / G, hd = p.hd, kvd = p.n_kv * hd;
  const int S = p.n_tokens, rows = min(PR, S - r0), jn = r0 + rows;  // keys [0, jn)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ks = hd + 4;
  float* qs = sm;                      // [rows][hd]
  float* kb = qs + PR * hd;            // PF_CH staged K or V rows (16-byte aligned)
  float* sc = kb + PF_CH * ks;         // [rows][jn]
  float* chv = sc + (size_t)PR * jn;   // per warp: 32 values + 32 flags
  griddep_wait();
  // the prompt's own K/V: cache slots from the sequence's first free one on
  const int base = p.len[p.seq0];
  const float* kcb = p.kc + kvh * hd;  // rows base + j of sequence seq0
  const float* vcb = p.vc + kvh * hd;
  for (int t = tid; t < rows * hd; t += PF_THREADS) {
    const int i = t / hd, d = t - i * hd;
    qs[t] = p.q[(long long)(r0 + i) * p.ld + (long long)hh * hd + d];
  }
  // S = Q K^T * scale, K rows staged through smem PF_CH keys at a time
  // (masked entries are not needed: set to 0, a no-op in P V)
  for (int j0 = 0; j0 < jn; j0 += PF_CH) {
    const int cn = min(PF_CH, jn - j0);
    __syncthreads();
    stage_rows_pf(kb, ks, kcb, p, p.seq0, base + j0, kvd, cn, hd, tid);
    __syncthreads();
    for (int t = tid; t < rows * cn; t += PF_THREADS) {
      const int i = t / cn, jj = t - i * cn, j = j0 + jj, q = r0 + i;
      float* dst = sc + (size_t)i * jn + j;
      if (j > q) {
        *dst = 0.0f;
        continue;
      }
      const bool fused = s_fused(q, j, S);
      const float* kr = kb + jj * ks;
      const float* qr = qs + i * hd;
      float acc = 0.0f;
      for (int d = 0; d < hd; d += 4) {
        const float4 kv = *reinterpret_cast<const float4*>(kr + d);
        const float4 qv = *reinterpret_cast<const float4*>(qr + d);
        acc = chain(fused, qv.x, kv.x, acc);
        acc = chain(fused, qv.y, kv.y, acc);
        acc = chain(fused, qv.z, kv.z, acc);
        acc = chain(fused, qv.w, kv.w, acc);
      }
      *dst = __fmul_rn(acc, p.scale);
    }
  }
  __syncthreads();
  // online softmax per row (warp per row): running max known from a prefix
  // scan, exponentials in parallel, the (se) recurrence sequential
  float* wv = chv + warp * 64;
  for (int i = warp; i < rows; i += PF_THREADS / 32) {
    const int q = r0 + i;
    float* r = sc + (size_t)i * jn;
    float M = -INFINITY, se = 0.0f;
    for (int c0 = 0; c0 <= q; c0 += 32) {
      const int j = c0 + lane;
      const float x = j <= q ? r[j] : -INFINITY;
      float incl = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = fmaxf(incl, y);
      }
      float excl = __shfl_up_sync(0xffffffffu, incl, 1);
      const float mprev = lane == 0 ? M : fmaxf(M, excl);
      const bool up = x > mprev;
      wv[lane] = up ? exp_f32(__fsub_rn(mprev, x)) : exp_f32(__fsub_rn(x, mprev));
      wv[32 + lane] = up ? 1.0f : 0.0f;
      __syncwarp();
      if (lane == 0) {
        const int cn = min(32, q + 1 - c0);
        for (int l = 0; l < cn; l++)
          se = wv[32 + l] != 0.0f ? __fadd_rn(__fmul_rn(se, wv[l]), 1.0f) : __fadd_rn(se, wv[l]);
      }
      __syncwarp();
      M = fmaxf(M, __shfl_sync(0xffffffffu, incl, 31));
    }
    se = __shfl_sync(0xffffffffu, se, 0);
    const float inv = __fdiv_rn(1.0f, se);
    for (int j = lane; j <= q; j += 32) r[j] = __fmul_rn(exp_f32(__fsub_rn(r[j], M)), inv);
  }
  __syncthreads();
  griddep_launch();
  // O = P V: each thread owns up to 16 outputs, chains advanced together
  constexpr int NPER = 16;
  float acc[NPER];
  int oi[NPER];
  bool fz[NPER];
  int nown = 0;
#pragma unroll
  for (int u = 0; u < NPER; u++) {
    const int t = tid + u * PF_THREADS;
    acc[u] = 0.0f;
    oi[u] = t < rows * hd ? t : -1;
    fz[u] = false;
    if (oi[u] >= 0) {
      const int i = t / hd, d = t - i * hd;
      fz[u] = o_fused(r0 + i, d, S, hd);
      nown = u + 1;
    }
  }
  int srow[NPER], vcol[NPER];
#pragma unroll
  for (int u = 0; u < NPER; u++) {
    const int i = oi[u] >= 0 ? oi[u] / hd : 0;
    srow[u] = i * jn;
    vcol[u] = oi[u] >= 0 ? oi[u] - i * hd : 0;
  }
  for (int j0 = 0; j0 < jn; j0 += PF_CH) {
    const int cn = min(PF_CH, jn - j0);
    __syncthreads();
    stage_rows_pf(kb, ks, vcb, p, p.seq0, base + j0, kvd, cn, hd, tid);
    __syncthreads();
    for (int jj = 0; jj < cn; jj++) {
      const float* vr = kb + jj * ks;
#pragma unroll
      for (int u = 0; u < NPER; u++)
        if (u < nown && oi[u] >= 0)
          acc[u] = chain(fz[u], sc[srow[u] + j0 + jj], vr[vcol[u]], acc[u]);
    }
  }
#pragma unroll
  for (int u = 0; u < NPER; u++) {
    if (u < nown && oi[u] >= 0) {
      const int i = oi[u] / hd, d = oi[u] - i * hd;
      p.out[(long long)(r0 + i) * p.ldo + (long long)hh * hd + d] = acc[u];
    }
  }
}

// ---------------------------------------------------------------------------
// Parallel ("flash") attention for the block-format models, whose matmuls
// already carry the 1e-3 tolerance: same inputs, outputs and cache effects
// as the exact kernels above, but reductions in a parallel order (split over
// positions with a max/sum rescaling combine), so long contexts are not
// latency-bound. The exact kernels stay the reference-order path (INT8).
// ---------------------------------------------------------------------------
constexpr int FD_THREADS = 128, FD_CH = 64;  // decode: positions per split CTA

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float s = 0.0f;
  for (int i = 0; i < nw; i++) s += red[i];
  return s;
}

// grid (batch, heads, splits): partial (max, sum, o[HD]) of one position
// range; the last CTA of a head to finish (arrival counter, left at zero)
// combines the partials with the max/sum rescaling.
template <int HD>
__global__ void __launch_bounds__(FD_THREADS) k_attn_decode_split(const AttnParams p, float* part,
                                                                  int* cnt, int nsplit) {
  extern __shared__ __align__(16) float sm[];
  constexpr int Q4 = HD / 4, VS = HD + 4, VCH = 32;
  float* xs = sm;                   // q, k, v (3*HD)
  float* vb = sm + 3 * HD;          // VCH staged V rows
  float* lanes = vb + VCH * VS;     // 8
  float* scl = lanes + 8;           // 4
  float* red = scl + 4;             // 4
  float* sc = red + 4;              // FD_CH
  __shared__ int last;
  const int b = blockIdx.x, h = blockIdx.y, sp = blockIdx.z, tid = threadIdx.x;
  const int G = p.n_heads / p.n_kv, kvh = h / G, kvd = p.n_kv * HD;
  float* base = part + ((size_t)b * p.n_heads + h) * nsplit * (HD + 2);
  float* dst = base + (size_t)sp * (HD + 2);
  griddep_wait();
  // this row's sequence (span: row b = position len + b)
  const int sq = p.span ? p.seq0 : p.slots ? p.slots[b] : b;
  const int pos = p.span ? p.len[sq] + b : p.len[sq];
  if (pos >= p.max_seq) {
    if (tid == 0 && p.err) atomicExch(p.err, SYN_ERR_INVALID_ARG);
    return;
  }
  const int L = pos + 1;
  const int off = (p.window > 0 && L > p.window) ? L - p.window : 0;
  const int eff = L - off, c0 = sp * FD_CH;
  const bool owner = sp == 0 && h % G == 0 && !p.span;
  const int cn = min(FD_CH, eff - c0);
  float mx = -INFINITY, ls = 0.0f, acc = 0.0f;
  if (cn > 0 || owner) {
    const float* qrow = p.q + (long long)b * p.ld + (long long)h * HD;
    const float* krow = p.k + (long long)b * p.ld + (long long)kvh * HD;
    const float* vrow = p.v + (long long)b * p.ld + (long long)kvh * HD;
    float* kcb = p.kc + kvh * HD;  // row r: + kv_slot(p, sq, r) * kvd
    float* vcb = p.vc + kvh * HD;
    for (int i = tid; i < HD; i += FD_THREADS) {
      xs[i] = qrow[i];
      xs[HD + i] = krow[i];
      xs[2 * HD + i] = vrow[i];
    }
    __syncthreads();
    if (!p.span)  // span mode: q ready, K/V already in the cache
      norm_rope(xs, 2, HD, p.qn, p.kn, 1, p.eps, p.cos_t, p.sin_t, pos, lanes, scl, FD_THREADS);
    if (owner)
      for (int i = tid; i < HD; i += FD_THREADS) {
        kcb[kv_slot(p, sq, pos) * kvd + i] = xs[HD + i];
        vcb[kv_slot(p, sq, pos) * kvd + i] = xs[2 * HD + i];
      }
    if (cn > 0) {
      for (int t = tid; t < cn; t += FD_THREADS) {
        const int row = off + c0 + t;
        const float* kr = row == pos && !p.span ? xs + HD : kcb + kv_slot(p, sq, row) * kvd;
        float4 kv[Q4];
#pragma unroll
        for (int c = 0; c < Q4; c++) kv[c] = reinterpret_cast<const float4*>(kr)[c];
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int c = 0; c < Q4; c++) {
          const float4 q = reinterpret_cast<const float4*>(xs)[c];
          a0 = fmaf(q.x, kv[c].x, a0);
          a1 = fmaf(q.y, kv[c].y, a1);
          a2 = fmaf(q.z, kv[c].z, a2);
          a3 = fmaf(q.w, kv[c].w, a3);
        }
        sc[t] = ((a0 + a1) + (a2 + a3)) * p.scale;
      }
      __syncthreads();
      for (int t = tid; t < cn; t += FD_THREADS) mx = fmaxf(mx, sc[t]);
      mx = block_max(mx, red);
      for (int t = tid; t < cn; t += FD_THREADS) {
        const float e = expf(sc[t] - mx);
        sc[t] = e;
        ls += e;
      }
      ls = block_sum(ls, red);
      constexpr int PER = (VCH * Q4 + FD_THREADS - 1) / FD_THREADS;
      for (int v0 = 0; v0 < cn; v0 += VCH) {
        const int vn = min(VCH, cn - v0);
        __syncthreads();
        float4 tmp[PER];
#pragma unroll
        for (int u = 0; u < PER; u++) {
          const int t = tid + u * FD_THREADS, r = t / Q4, c4 = t - r * Q4;
          if (r < vn) {
            const int row = off + c0 + v0 + r;
            tmp[u] = row == pos && !p.span
                         ? reinterpret_cast<const float4*>(xs + 2 * HD)[c4]
                         : reinterpret_cast<const float4*>(vcb + kv_slot(p, sq, row) * kvd)[c4];
          }
        }
#pragma unroll
        for (int u = 0; u < PER; u++) {
          const int t = tid + u * FD_THREADS, r = t / Q4, c4 = t - r * Q4;
          if (r < vn) reinterpret_cast<float4*>(vb + r * VS)[c4] = tmp[u];
        }
        __syncthreads();
        if (tid < HD)
          for (int s2 = 0; s2 < vn; s2++) acc = fmaf(sc[v0 + s2], vb[s2 * VS + tid], acc);
      }
    }
  }
  if (tid < HD) dst[2 + tid] = acc;
  if (tid == 0) {
    dst[0] = mx;
    dst[1] = ls;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&cnt[b * p.n_heads + h], 1) == nsplit - 1;
  __syncthreads();
  griddep_launch();
  if (!last) return;
  __threadfence();
  // combine: split maxima and rescaled sums in parallel over the splits (the
  // factors go to smem, reusing the V staging rows), then each output column
  // sums its splits with the loads issued in batches
  float* fac = vb;  // nsplit floats
  float M = -INFINITY;
  for (int c = tid; c < nsplit; c += FD_THREADS) M = fmaxf(M, __ldcg(base + c * (HD + 2)));
  M = block_max(M, red);
  float lsum = 0.0f;
  for (int c = tid; c < nsplit; c += FD_THREADS) {
    const float m = __ldcg(base + c * (HD + 2));
    const float f = m == -INFINITY ? 0.0f : expf(m - M);
    fac[c] = f;
    lsum += f * __ldcg(base + c * (HD + 2) + 1);
  }
  lsum = block_sum(lsum, red);  // (its barriers also publish fac)
  if (tid < HD) {
    float o = 0.0f;
    int c = 0;
    for (; c + 8 <= nsplit; c += 8) {
      float ov[8];
#pragma unroll
      for (int u = 0; u < 8; u++) ov[u] = __ldcg(base + (c + u) * (HD + 2) + 2 + tid);
#pragma unroll
      for (int u = 0; u < 8; u++) o = fmaf(ov[u], fac[c + u], o);
    }
    for (; c < nsplit; c++) o = fmaf(__ldcg(base + c * (HD + 2) + 2 + tid), fac[c], o);
    p.out[(long long)b * p.ldo + (long long)h * HD + tid] = o / lsum;
  }
  if (tid == 0) cnt[b * p.n_heads + h] = 0;  // ready for the next launch
}

// ---------------------------------------------------------------------------
// Decode attention for the block-format models, grouped by KV head: one CTA
// per (row, KV head, split) serves the G query heads that share the KV head,
// so each cached K/V row crosses HBM once per step (the per-query-head
// kernel above reads it G times). The split length follows the row's actual
// context, ceil(eff / nsplit) rounded up to the warp step, so a graph
// captured for max_seq keeps every split busy at whatever length it replays.
// A warp takes GQ_RB consecutive rows per step, with the next step's rows in
// flight: lane l holds elements [E*l, E*l + E) of a row (512 coalesced bytes
// for HD 128), the q.k partials are summed across the warp by butterfly
// shuffles, and each head keeps a running max, sum and output slice in
// registers (online softmax). The four warps merge in shared memory into one
// partial (max, sum, o[HD]) per head and split; the last CTA of the (row, KV
// head) merges the splits. q and the new row's k are normalised and rotated
// by norm_rope, the same bits as the other kernels, and the CTA whose range
// holds the new position appends its K and V.
// ---------------------------------------------------------------------------
constexpr int GQ_THREADS = 128, GQ_WARPS = 4, GQ_RB = 4;

template <int HD> struct GqVec;
template <> struct GqVec<64> {
  using T = float2;
  __device__ static float at(const float2& v, int e) { return e == 0 ? v.x : v.y; }
};
template <> struct GqVec<128> {
  using T = float4;
  __device__ static float at(const float4& v, int e) {
    return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
  }
};

template <int HD, int G>
__global__ void __launch_bounds__(GQ_THREADS) k_attn_decode_gqa(const AttnParams p, float* part,
                                                                int* cnt, int nsplit) {
  constexpr int E = HD / 32;
  using VT = GqVec<HD>;
  using V = typename VT::T;
  __shared__ __align__(16) float xs[(G + 2) * HD];  // q heads, then k and v of the new row
  __shared__ float lanes[4 * (G + 1)], scl[G + 1];
  __shared__ float wst[GQ_WARPS][G][2];              // per-warp (max, sum)
  __shared__ __align__(16) float wo[GQ_WARPS][G][HD];  // per-warp output slices
  __shared__ int last;
  const int b = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int kvd = p.n_kv * HD;
  // Before griddepcontrol.wait only data written two or more kernels back is
  // read: the committed length and the cached rows below it.
  const int sq = p.span ? p.seq0 : p.slots ? p.slots[b] : b;
  const int len0 = p.len[sq];
  const int pos = p.span ? len0 + b : len0;
  const int early = p.span ? len0 : pos;  // rows [0, early) may be read before the wait
  if (pos >= p.max_seq) {  // cache full: nothing is written (the host reports it)
    griddep_wait();
    if (tid == 0 && p.err) atomicExch(p.err, SYN_ERR_INVALID_ARG);
    return;
  }
  const int L = pos + 1;
  const int off = (p.window > 0 && L > p.window) ? L - p.window : 0;
  const int eff = L - off;
  int sl = (eff + nsplit - 1) / nsplit;
  sl = (sl + GQ_RB - 1) / GQ_RB * GQ_RB;
  const int r0 = off + min(eff, sp * sl), r1 = off + min(eff, (sp + 1) * sl);
  const float* kcb = p.kc + kvh * HD;
  const float* vcb = p.vc + kvh * HD;
  const bool fresh = !p.span;  // the new row's K/V come from q/k/v, not the cache
  const V zero = {};

  V kr[GQ_RB], vr[GQ_RB];
  const int rb0 = r0 + warp * GQ_RB;
#pragma unroll
  for (int j = 0; j < GQ_RB; j++) {
    kr[j] = zero;
    vr[j] = zero;
    const int row = rb0 + j;
    if (row < r1 && row < early) {
      const size_t s = kv_slot(p, sq, row) * kvd;
      kr[j] = reinterpret_cast<const V*>(kcb + s)[lane];
      vr[j] = reinterpret_cast<const V*>(vcb + s)[lane];
    }
  }
  griddep_wait();
  const bool has_new = fresh && pos >= r0 && pos < r1;
  {
    const float* qrow = p.q + (long long)b * p.ld + (long long)kvh * G * HD;
    for (int i = tid; i < G * HD; i += GQ_THREADS) xs[i] = qrow[i];
    if (has_new) {
      const float* krow = p.k + (long long)b * p.ld + (long long)kvh * HD;
      const float* vrow = p.v + (long long)b * p.ld + (long long)kvh * HD;
      for (int i = tid; i < HD; i += GQ_THREADS) {
        xs[G * HD + i] = krow[i];
        xs[(G + 1) * HD + i] = vrow[i];
      }
    }
    __syncthreads();
    if (fresh)
      norm_rope(xs, has_new ? G + 1 : G, HD, p.qn, p.kn, G, p.eps, p.cos_t, p.sin_t, pos, lanes,
                scl, GQ_THREADS);
    if (has_new) {
      const size_t s = kv_slot(p, sq, pos) * kvd;
      for (int i = tid; i < HD; i += GQ_THREADS) {
        p.kc[s + kvh * HD + i] = xs[G * HD + i];
        p.vc[s + kvh * HD + i] = xs[(G + 1) * HD + i];
      }
    }
  }
  float q[G][E];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int e = 0; e < E; e++) q[g][e] = xs[g * HD + lane * E + e];
  if (!fresh) {  // span: rows from len0 on were appended by the preceding kernel
#pragma unroll
    for (int j = 0; j < GQ_RB; j++) {
      const int row = rb0 + j;
      if (row < r1 && row >= early) {
        const size_t s = kv_slot(p, sq, row) * kvd;
        kr[j] = reinterpret_cast<const V*>(kcb + s)[lane];
        vr[j] = reinterpret_cast<const V*>(vcb + s)[lane];
      }
    }
  }

  float m[G], l[G], o[G][E];
#pragma unroll
  for (int g = 0; g < G; g++) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < E; e++) o[g][e] = 0.0f;
  }
  constexpr int STEP = GQ_WARPS * GQ_RB;
  for (int rb = rb0; rb < r1; rb += STEP) {
    if (has_new) {
#pragma unroll
      for (int j = 0; j < GQ_RB; j++)
        if (rb + j == pos) {
          kr[j] = reinterpret_cast<const V*>(xs + G * HD)[lane];
          vr[j] = reinterpret_cast<const V*>(xs + (G + 1) * HD)[lane];
        }
    }
    V kn[GQ_RB], vn[GQ_RB];  // the next step's rows, in flight meanwhile
#pragma unroll
    for (int j = 0; j < GQ_RB; j++) {
      kn[j] = zero;
      vn[j] = zero;
      const int row = rb + STEP + j;
      if (row < r1 && !(fresh && row == pos)) {
        const size_t s = kv_slot(p, sq, row) * kvd;
        kn[j] = reinterpret_cast<const V*>(kcb + s)[lane];
        vn[j] = reinterpret_cast<const V*>(vcb + s)[lane];
      }
    }
    float s[G][GQ_RB];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
      for (int j = 0; j < GQ_RB; j++) {
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++) a = fmaf(q[g][e], VT::at(kr[j], e), a);
        s[g][j] = a;
      }
#pragma unroll
    for (int x = 16; x; x >>= 1)
#pragma unroll
      for (int g = 0; g < G; g++)
#pragma unroll
        for (int j = 0; j < GQ_RB; j++) s[g][j] += __shfl_xor_sync(0xffffffffu, s[g][j], x);
#pragma unroll
    for (int g = 0; g < G; g++) {
      float mx = m[g];
#pragma unroll
      for (int j = 0; j < GQ_RB; j++) {
        s[g][j] = rb + j < r1 ? s[g][j] * p.scale : -INFINITY;
        mx = fmaxf(mx, s[g][j]);
      }
      const float corr = m[g] == -INFINITY ? 0.0f : expf(m[g] - mx);
      l[g] *= corr;
#pragma unroll
      for (int e = 0; e < E; e++) o[g][e] *= corr;
#pragma unroll
      for (int j = 0; j < GQ_RB; j++) {
        const float pj = s[g][j] == -INFINITY ? 0.0f : expf(s[g][j] - mx);
        l[g] += pj;
#pragma unroll
        for (int e = 0; e < E; e++) o[g][e] = fmaf(pj, VT::at(vr[j], e), o[g][e]);
      }
      m[g] = mx;
    }
#pragma unroll
    for (int j = 0; j < GQ_RB; j++) {
      kr[j] = kn[j];
      vr[j] = vn[j];
    }
  }

  // merge the warps: one partial per head of this split
#pragma unroll
  for (int g = 0; g < G; g++) {
    if (lane == 0) {
      wst[warp][g][0] = m[g];
      wst[warp][g][1] = l[g];
    }
#pragma unroll
    for (int e = 0; e < E; e++) wo[warp][g][lane * E + e] = o[g][e];
  }
  __syncthreads();
  const size_t hstride = (size_t)nsplit * (HD + 2);  // one head's partials
  float* hbase = part + ((size_t)b * p.n_heads + (size_t)kvh * G) * hstride;
  for (int i = tid; i < G * HD; i += GQ_THREADS) {
    const int g = i / HD, d = i - g * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < GQ_WARPS; w++) M = fmaxf(M, wst[w][g][0]);
    float O = 0.0f, Ls = 0.0f;
#pragma unroll
    for (int w = 0; w < GQ_WARPS; w++) {
      const float f = wst[w][g][0] == -INFINITY ? 0.0f : expf(wst[w][g][0] - M);
      O = fmaf(f, wo[w][g][d], O);
      Ls = fmaf(f, wst[w][g][1], Ls);
    }
    float* dst = hbase + g * hstride + (size_t)sp * (HD + 2);
    dst[2 + d] = O;
    if (d == 0) {
      dst[0] = M;
      dst[1] = Ls;
    }
  }
  __threadfence();
  __syncthreads();
  int* cn = &cnt[b * p.n_heads + kvh * G];
  if (tid == 0) last = atomicAdd(cn, 1) == nsplit - 1;
  __syncthreads();
  griddep_launch();
  if (!last) return;
  __threadfence();
  // merge the splits: warp w takes heads w, w + 4, ...; lanes stride over
  // the splits for the maximum and the rescaled sums, then each lane sums
  // its E output columns over the splits (factors in shared memory)
  for (int g = warp; g < G; g += GQ_WARPS) {
    const float* base = hbase + g * hstride;
    float* fac = &wo[warp][0][0];  // nsplit <= G * HD factors of this warp
    float M = -INFINITY;
    for (int c = lane; c < nsplit; c += 32) M = fmaxf(M, __ldcg(base + c * (HD + 2)));
    M = warp_max(M);
    float lsum = 0.0f;
    for (int c = lane; c < nsplit; c += 32) {
      const float mc = __ldcg(base + c * (HD + 2));
      const float f = mc == -INFINITY ? 0.0f : expf(mc - M);
      fac[c] = f;
      lsum += f * __ldcg(base + c * (HD + 2) + 1);
    }
    lsum = warp_sum(lsum);
    __syncwarp();
    float ov[E];
#pragma unroll
    for (int e = 0; e < E; e++) ov[e] = 0.0f;
    // (o sits 2 floats into a record: scalar loads), 8 splits' loads in
    // flight at a time: each is an L2 round trip
    int c = 0;
    for (; c + 8 <= nsplit; c += 8) {
      float t[8][E];
#pragma unroll
      for (int u = 0; u < 8; u++)
#pragma unroll
        for (int e = 0; e < E; e++) t[u][e] = __ldcg(base + (c + u) * (HD + 2) + 2 + lane * E + e);
#pragma unroll
      for (int u = 0; u < 8; u++)
#pragma unroll
        for (int e = 0; e < E; e++) ov[e] = fmaf(t[u][e], fac[c + u], ov[e]);
    }
    for (; c < nsplit; c++) {
      const float f = fac[c];
      const float* t = base + c * (HD + 2) + 2 + lane * E;
#pragma unroll
      for (int e = 0; e < E; e++) ov[e] = fmaf(__ldcg(t + e), f, ov[e]);
    }
    float* orow = p.out + (long long)b * p.ldo + (long long)(kvh * G + g) * HD + lane * E;
#pragma unroll
    for (int e = 0; e < E; e++) orow[e] = ov[e] / lsum;
    __syncwarp();  // fac is rewritten for the warp's next head
  }
  if (tid == 0) *cn = 0;  // ready for the next launch
}

size_t flash_decode_smem(int hd) {
  return ((size_t)3 * hd + 32 * (hd + 4) + 8 + 4 + 4 + FD_CH) * sizeof(float);
}

// Prefill: CTA = (head, 64 queries), 256 threads; key tiles of 64 staged in
// smem; 4x4 score tile and 4 rows x HD/16 output columns per thread; online
// softmax with rescaling.
constexpr int FP_B = 64, FP_THREADS = 256;

template <int HD>
__global__ void __launch_bounds__(FP_THREADS) k_attn_prefill_flash(const AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  constexpr int S4 = HD + 4, PS = FP_B + 4, OC = HD / 16;
  float* qs = sm;                 // [64][S4]
  float* ks = qs + FP_B * S4;     // [64][S4]
  float* vs = ks + FP_B * S4;     // [64][S4]
  float* ps = vs + FP_B * S4;     // [64][PS]
  const int hh = blockIdx.x, q0 = blockIdx.y * FP_B, tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;  // rows 4ty..4ty+3; score cols 4tx..; out cols tx*OC..
  const int G = p.n_heads / p.n_kv, kvh = hh / G, kvd = p.n_kv * HD, S = p.n_tokens;
  griddep_wait();
  const int base = p.len[p.seq0];
  const float* kcb = p.kc + kvh * HD;  // rows base + j of sequence seq0
  const float* vcb = p.vc + kvh * HD;
  for (int t = tid; t < FP_B * (HD / 4); t += FP_THREADS) {
    const int r = t / (HD / 4), c4 = t - r * (HD / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < S)
      v = reinterpret_cast<const float4*>(p.q + (long long)(q0 + r) * p.ld + (long long)hh * HD)[c4];
    reinterpret_cast<float4*>(qs + r * S4)[c4] = v;
  }
  float m[4], l[4], o[4][OC];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int c = 0; c < OC; c++) o[r][c] = 0.0f;
  }
  const int kend = min(S, q0 + FP_B);  // causal: keys < kend
  for (int k0 = 0; k0 < kend; k0 += FP_B) {
    __syncthreads();
    for (int t = tid; t < FP_B * (HD / 4); t += FP_THREADS) {
      const int r = t / (HD / 4), c4 = t - r * (HD / 4);
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (k0 + r < S) {
        const size_t sl = kv_slot(p, p.seq0, base + k0 + r) * kvd;
        kv = reinterpret_cast<const float4*>(kcb + sl)[c4];
        vv = reinterpret_cast<const float4*>(vcb + sl)[c4];
      }
      reinterpret_cast<float4*>(ks + r * S4)[c4] = kv;
      reinterpret_cast<float4*>(vs + r * S4)[c4] = vv;
    }
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) sc[i][j] = 0.0f;
    for (int d = 0; d < HD; d += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const float4*>(qs + (4 * ty + i) * S4 + d);
#pragma unroll
      for (int j = 0; j < 4; j++) kv[j] = *reinterpret_cast<const float4*>(ks + (4 * tx + j) * S4 + d);
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
          sc[i][j] = fmaf(qv[i].x, kv[j].x, sc[i][j]);
          sc[i][j] = fmaf(qv[i].y, kv[j].y, sc[i][j]);
          sc[i][j] = fmaf(qv[i].z, kv[j].z, sc[i][j]);
          sc[i][j] = fmaf(qv[i].w, kv[j].w, sc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int q = q0 + 4 * ty + i;
      float rm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int k = k0 + 4 * tx + j;
        sc[i][j] = (k <= q && k < S) ? sc[i][j] * p.scale : -INFINITY;
        rm = fmaxf(rm, sc[i][j]);
      }
      for (int off = 1; off < 16; off <<= 1) rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, off));
      const float mn = fmaxf(m[i], rm);
      const float corr = mn == -INFINITY ? 1.0f : expf(m[i] - mn);
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float e = mn == -INFINITY ? 0.0f : expf(sc[i][j] - mn);
        rs += e;
        ps[(4 * ty + i) * PS + 4 * tx + j] = e;
      }
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * corr + rs;
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < OC; c++) o[i][c] *= corr;
    }
    __syncthreads();
    for (int j = 0; j < FP_B; j++) {
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) pv[i] = ps[(4 * ty + i) * PS + j];
      const float* vr = vs + j * S4 + tx * OC;
#pragma unroll
      for (int c = 0; c < OC; c++) {
        const float v = vr[c];
#pragma unroll
        for (int i = 0; i < 4; i++) o[i][c] = fmaf(pv[i], v, o[i][c]);
      }
    }
  }
  griddep_launch();
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int q = q0 + 4 * ty + i;
    if (q < S) {
      float* orow = p.out + (long long)q * p.ldo + (long long)hh * HD + tx * OC;
#pragma unroll
      for (int c = 0; c < OC; c++) orow[c] = o[i][c] / l[i];
    }
  }
}

size_t flash_prefill_smem(int hd) {
  return ((size_t)3 * FP_B * (hd + 4) + (size_t)FP_B * (FP_B + 4)) * sizeof(float);
}

// ---------------------------------------------------------------------------
// Prefill attention on the tensor cores (block-format models): CTA = (head,
// 128 queries), 128 threads, thread t owns query row t (tensor-memory lane
// t). Per key tile of 64:
//   S = Q K^T with tcgen05.mma kind::f16 (bf16 operands, fp32 accumulation
//   in tensor memory), each f32 operand entering as bf16 hi + lo parts
//   (x = hi + lo, lo = bf16(x - hi)) and the four products hi*hi + hi*lo +
//   lo*hi + lo*lo summed, so a score carries about 2^-24 relative error:
//   the f32 products of the CUDA-core kernel, in another summation order;
//   online softmax (row max, rescale, exp) in registers, one row per thread;
//   O_tile = P V the same way (P and V split likewise), added to the
//   thread's f32 output row with the rescaling.
// Operands live in shared memory in the 128-byte-swizzled K-major layout
// (atoms of 8 rows x 128 B): Q [128][HD], K [64][HD], V^T [HD][64] (staged
// transposed, so both MMAs read K-major operands), P [128][64]. Waits are
// bounded (SYN_ERR_TIMEOUT). Reference: syn_fused_attention
// (zig/src/ffi/exports.zig:1364-1478), causal, no window.
// ---------------------------------------------------------------------------
constexpr int TCA_Q = 128, TCA_K = 64, TCA_THREADS = 128;

__device__ __forceinline__ uint32_t tca_sw(int c, int r, int rows) {  // 16-byte column c of row r
  return (uint32_t)((c >> 3) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                    (((c & 7) ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint64_t tca_desc(uint32_t addr) {  // K-major, 128B swizzle
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;             // LBO 16 B
  d |= (uint64_t)(1024 >> 4) << 32;   // SBO 1024 B
  d |= (uint64_t)1 << 46;             // sm_100 descriptor version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}
__device__ __forceinline__ void tca_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id,
                                        uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc), "r"(0u));
}
__device__ __forceinline__ void tca_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tca_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t u[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
        "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]),
        "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]),
        "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) r[i] = __uint_as_float(u[i]);
}
// 8 f32 -> bf16 hi (16 B) and lo (16 B)
__device__ __forceinline__ void tca_split8(const float (&v)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    const float2 bf = __bfloat1622float2(b);
    const __nv_bfloat162 r = __floats2bfloat162_rn(v[2 * i] - bf.x, v[2 * i + 1] - bf.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&b);
    l[i] = *reinterpret_cast<const uint32_t*>(&r);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int HD>
struct TcaSmem {
  static constexpr int Q = TCA_Q * HD * 2;    // one bf16 part of Q
  static constexpr int K = TCA_K * HD * 2;    // of K
  static constexpr int V = HD * TCA_K * 2;    // of V^T
  static constexpr int P = TCA_Q * TCA_K * 2; // of P
  static constexpr int OQ = 0, OK = 2 * Q, OV = OK + 2 * K, OP = OV + 2 * V;
  static constexpr int BYTES = OP + 2 * P + 1024;  // + alignment slack
};

template <int HD>
__global__ void __launch_bounds__(TCA_THREADS, 1) k_attn_prefill_tc(const AttnParams p) {
  using L = TcaSmem<HD>;
  extern __shared__ uint8_t tca_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tca_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar_s, bar_o;
  __shared__ uint32_t tbase_sh;
  __shared__ int fail;
  const int hh = blockIdx.x, q0 = blockIdx.y * TCA_Q, t = threadIdx.x, warp = t >> 5;
  const int G = p.n_heads / p.n_kv, kvh = hh / G, kvd = p.n_kv * HD, S = p.n_tokens;
  constexpr uint32_t TMEM_COLS = 256, S_COL = 0, O_COL = 64;
  if (t == 0) {
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    fail = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tbase_sh)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tb = tbase_sh;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  griddep_wait();
  const int base = p.len[p.seq0];  // the prompt's first cache position
  // Q: row t (zero beyond the prompt)
  {
    const float* qr = p.q + (long long)(q0 + t) * p.ld + (long long)hh * HD;
    for (int c = 0; c < HD / 8; c++) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = q0 + t < S ? qr[c * 8 + e] : 0.0f;
      uint4 hi, lo;
      tca_split8(v, hi, lo);
      *reinterpret_cast<uint4*>(sm + L::OQ + tca_sw(c, t, TCA_Q)) = hi;
      *reinterpret_cast<uint4*>(sm + L::OQ + L::Q + tca_sw(c, t, TCA_Q)) = lo;
    }
  }
  float o[HD];
#pragma unroll
  for (int d = 0; d < HD; d++) o[d] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  const int qi = q0 + t;
  const int kend = min(S, q0 + TCA_Q);  // causal: keys < kend
  const uint32_t id_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TCA_K >> 3) << 17) |
                        ((uint32_t)(TCA_Q >> 4) << 24);
  const uint32_t id_o = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(HD >> 3) << 17) |
                        ((uint32_t)(TCA_Q >> 4) << 24);
  const uint32_t sq = smem_u32(sm + L::OQ), sk = smem_u32(sm + L::OK), sv = smem_u32(sm + L::OV),
                 sp = smem_u32(sm + L::OP);
  int tile = 0;
  for (int k0 = 0; k0 < kend; k0 += TCA_K, tile++) {
    // stage K [64 keys][HD] and V^T [HD][64 keys] as bf16 hi / lo
    for (int w = t; w < TCA_K * (HD / 8); w += TCA_THREADS) {
      const int r = w / (HD / 8), c = w - r * (HD / 8);
      float v[8];
      if (k0 + r < S) {
        const float* kr = p.kc + kvh * HD + kv_slot(p, p.seq0, base + k0 + r) * kvd + c * 8;
        const float4 a = reinterpret_cast<const float4*>(kr)[0], b = reinterpret_cast<const float4*>(kr)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = 0.0f;
      }
      uint4 hi, lo;
      tca_split8(v, hi, lo);
      *reinterpret_cast<uint4*>(sm + L::OK + tca_sw(c, r, TCA_K)) = hi;
      *reinterpret_cast<uint4*>(sm + L::OK + L::K + tca_sw(c, r, TCA_K)) = lo;
    }
    for (int w = t; w < HD * (TCA_K / 8); w += TCA_THREADS) {
      const int d = w % HD, c = w / HD;  // V^T row d, keys 8c .. 8c+7
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int kk = k0 + c * 8 + e;
        v[e] = kk < S ? p.vc[kvh * HD + kv_slot(p, p.seq0, base + kk) * kvd + d] : 0.0f;
      }
      uint4 hi, lo;
      tca_split8(v, hi, lo);
      *reinterpret_cast<uint4*>(sm + L::OV + tca_sw(c, d, HD)) = hi;
      *reinterpret_cast<uint4*>(sm + L::OV + L::V + tca_sw(c, d, HD)) = lo;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    // S = Q K^T: 4 products per 16-wide K step
    if (t == 0 && !fail) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int ks = 0; ks < HD / 16; ks++) {
        const uint32_t qa = (uint32_t)((ks >> 2) * TCA_Q * 128 + (ks & 3) * 32);
        const uint32_t ka = (uint32_t)((ks >> 2) * TCA_K * 128 + (ks & 3) * 32);
#pragma unroll
        for (int term = 0; term < 4; term++) {
          const uint64_t da = tca_desc(sq + qa + ((term >> 1) ? L::Q : 0));
          const uint64_t db = tca_desc(sk + ka + ((term & 1) ? L::K : 0));
          tca_mma(tb + S_COL, da, db, id_s, (ks | term) ? 1u : 0u);
        }
      }
      tca_commit(&bar_s);
    }
    if (!mbar_wait_bounded(&bar_s, tile & 1)) fail = 1;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // softmax on row t
    float sc[TCA_K];
    {
      float a[32];
      tca_ld32(tb + lane_off + S_COL, a);
#pragma unroll
      for (int j = 0; j < 32; j++) sc[j] = a[j];
      tca_ld32(tb + lane_off + S_COL + 32, a);
#pragma unroll
      for (int j = 0; j < 32; j++) sc[32 + j] = a[j];
    }
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < TCA_K; j++) {
      const int kk = k0 + j;
      sc[j] = (kk <= qi && kk < S) ? sc[j] * p.scale : -INFINITY;
      mt = fmaxf(mt, sc[j]);
    }
    const float mn = fmaxf(m, mt);
    const float corr = mn == -INFINITY ? 1.0f : expf(m - mn);
    float rs = 0.0f;
#pragma unroll
    for (int c = 0; c < TCA_K / 8; c++) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const float x = sc[c * 8 + e];
        v[e] = mn == -INFINITY ? 0.0f : expf(x - mn);
        rs += v[e];
      }
      uint4 hi, lo;
      tca_split8(v, hi, lo);
      *reinterpret_cast<uint4*>(sm + L::OP + tca_sw(c, t, TCA_Q)) = hi;
      *reinterpret_cast<uint4*>(sm + L::OP + L::P + tca_sw(c, t, TCA_Q)) = lo;
    }
    l = l * corr + rs;
    m = mn;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    // O_tile = P V
    if (t == 0 && !fail) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int ks = 0; ks < TCA_K / 16; ks++) {
        const uint32_t off = (uint32_t)(ks * 32);
#pragma unroll
        for (int term = 0; term < 4; term++) {
          const uint64_t da = tca_desc(sp + off + ((term >> 1) ? L::P : 0));
          const uint64_t db = tca_desc(sv + off + ((term & 1) ? L::V : 0));
          tca_mma(tb + O_COL, da, db, id_o, (ks | term) ? 1u : 0u);
        }
      }
      tca_commit(&bar_o);
    }
    if (!mbar_wait_bounded(&bar_o, tile & 1)) fail = 1;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
    for (int d0 = 0; d0 < HD; d0 += 32) {
      float a[32];
      tca_ld32(tb + lane_off + O_COL + d0, a);
#pragma unroll
      for (int j = 0; j < 32; j++) o[d0 + j] = fmaf(o[d0 + j], corr, a[j]);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
  }
  griddep_launch();
  if (fail) {
    if (t == 0 && p.err) atomicExch(p.err, SYN_ERR_TIMEOUT);
  } else if (qi < S) {
    float* orow = p.out + (long long)qi * p.ldo + (long long)hh * HD;
#pragma unroll
    for (int d = 0; d < HD; d += 4)
      *reinterpret_cast<float4*>(orow + d) =
          make_float4(o[d] / l, o[d + 1] / l, o[d + 2] / l, o[d + 3] / l);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tb), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// SwiGLU: variant 0 = the INT8 model's silu(g) * u with silu = g/(1+exp(-g))
// (quantization/lm/int8.rs:500-503, ops/activation.rs:30-32); variant 1 =
// swigluFused (zig/src/ops/silu.zig:85-114): g * (1/(1+exp(-g))) * u for the
// first n - n%4 elements, (g/(1+exp(-g))) * u for the tail.
// ---------------------------------------------------------------------------
__global__ void k_swiglu(const float* __restrict__ gate, const float* __restrict__ up,
                         long long ld_in, int rows, int n, int variant, float* __restrict__ out,
                         long long ldo, int il16) {
  griddep_wait();
  griddep_launch();
  const long long total = (long long)rows * n;
  const int n4 = n & ~3;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(t / n), i = (int)(t - (long long)r * n);
    const int c = il16 ? ((i >> 4) << 5) + (i & 15) : i;
    out[r * ldo + i] = swiglu_elem(gate[r * ld_in + c], up[r * ld_in + c], i, n4, variant);
  }
}

// ---------------------------------------------------------------------------
// argmax (generation/sampler.rs:217-224): Iterator::max_by with partial_cmp,
// NaN comparing Equal. The running best is replaced unless it is strictly
// greater, so the answer is the last index of the maximum over the elements
// after the last NaN (or that NaN itself when nothing follows it).
// That rule is a fold over contiguous segments with an associative combine,
// so the row is split over CTAs of AM_THREADS * AM_PER elements, reduced in
// index order inside each CTA, and the last CTA of a row (arrival counter)
// combines the CTA states in order. It can also advance the KV-cache lengths.
// ---------------------------------------------------------------------------
constexpr int AM_THREADS = 256, AM_PER = 8, AM_SEG = AM_THREADS * AM_PER;

struct AmState {
  int nan;  // last NaN index in the segment, -1 if none
  int i;    // best index after `nan`, -1 if none
  float v;
};

__device__ __forceinline__ AmState am_combine(AmState l, const AmState& r) {
  if (r.nan >= 0) return r;  // nothing before r's NaN survives
  if (r.i >= 0 && (l.i < 0 || r.v >= l.v)) {  // the later segment wins ties
    l.i = r.i;
    l.v = r.v;
  }
  return l;
}

__device__ __forceinline__ AmState am_shfl_down(const AmState& s, int o) {
  AmState r;
  r.nan = __shfl_down_sync(0xffffffffu, s.nan, o);
  r.i = __shfl_down_sync(0xffffffffu, s.i, o);
  r.v = __shfl_down_sync(0xffffffffu, s.v, o);
  return r;
}

__global__ void __launch_bounds__(AM_THREADS) k_argmax(const float* __restrict__ x, long long ldx,
                                                       int n, int32_t* __restrict__ out,
                                                       int* len_adv, int adv, int max_len,
                                                       int32_t* hist, int hist_ld,
                                                       AmState* __restrict__ part,
                                                       int* __restrict__ cnt,
                                                       int4* __restrict__ pair_out, int idx_off) {
  __shared__ AmState ws[AM_THREADS / 32];
  __shared__ int last;
  griddep_wait();
  const int row = blockIdx.y, c = blockIdx.x, nct = gridDim.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* xr = x + row * ldx;
  const int base = c * AM_SEG + tid * AM_PER;
  float v[AM_PER];
#pragma unroll
  for (int u = 0; u < AM_PER; u++) v[u] = base + u < n ? xr[base + u] : 0.0f;
  AmState st{-1, -1, 0.0f};
#pragma unroll
  for (int u = 0; u < AM_PER; u++) {
    if (base + u < n) {
      if (isnan(v[u])) {
        st.nan = base + u;
        st.i = -1;
      } else if (st.i < 0 || v[u] >= st.v) {
        st.i = base + u;
        st.v = v[u];
      }
    }
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const AmState r = am_shfl_down(st, o);
    if ((lane & (2 * o - 1)) == 0) st = am_combine(st, r);
  }
  if (lane == 0) ws[warp] = st;
  __syncthreads();
  if (tid == 0) {
    AmState t = ws[0];
    for (int w = 1; w < AM_THREADS / 32; w++) t = am_combine(t, ws[w]);
    part[row * nct + c] = t;
    __threadfence();
    last = atomicAdd(&cnt[row], 1) == nct - 1;
  }
  __syncthreads();
  griddep_launch();
  if (last && tid == 0) {
    __threadfence();
    AmState t = part[row * nct];
    for (int k = 1; k < nct; k++) t = am_combine(t, part[row * nct + k]);
    if (pair_out) {  // a vocabulary slice: its state, with global indices
      cnt[row] = 0;
      pair_out[row] = make_int4(t.nan >= 0 ? t.nan + idx_off : -1, t.i >= 0 ? t.i + idx_off : -1,
                                __float_as_int(t.v), 0);
      return;
    }
    const int r = t.i >= 0 ? t.i : (t.nan >= 0 ? t.nan : 0);
    out[row] = r;
    cnt[row] = 0;  // ready for the next launch
    if (len_adv) {
      int nl = len_adv[row] + adv;
      nl = nl <= max_len ? nl : max_len;
      len_adv[row] = nl;
      // token history: the generated token will occupy position nl
      if (hist) hist[(size_t)row * hist_ld + nl] = r;
    }
  }
}

__global__ void k_kv_set(int* len, int seq, int value, int add) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) len[seq] = add ? len[seq] + value : value;
}

syn_status_t cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return SYN_OK;
  set_last_cuda_error(e, where);
  return SYN_ERR_CUDA;
}

}  // namespace

// ---- internal launchers (also used by the runner) --------------------------
syn_status_t launch_add_rmsnorm(const float* x, size_t ldx, const float* delta, size_t ldd,
                                const int32_t* ids, const float* table, size_t vocab,
                                float* x_out, size_t ldxo, const float* w, size_t rows, size_t h,
                                float eps, float* out, size_t ldo, cudaStream_t st, int fast) {
  if (h == 0 || rows == 0) return SYN_OK;
  if (h > 40000 || rows > 0x7FFFFFFF) return SYN_ERR_UNSUPPORTED;
  NormParams p{x, (long long)ldx, delta, (long long)ldd, ids, table, (unsigned)vocab,
               x_out, (long long)ldxo, w, (int)h, eps, out, (long long)ldo, fast};
  const size_t smem = h * sizeof(float);
  syn_status_t s = allow_smem((const void*)k_add_rmsnorm, smem);
  if (s) return s;
  return cuda_status(launch_pdl(k_add_rmsnorm, dim3((unsigned)rows), dim3(NORM_THREADS), smem, st, p),
                     "k_add_rmsnorm");
}

syn_status_t launch_swiglu(const float* gate, const float* up, size_t ld_in, size_t rows, size_t n,
                           int variant, float* out, size_t ldo, cudaStream_t st, int il16) {
  if (!rows || !n) return SYN_OK;
  const long long total = (long long)rows * n;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  return cuda_status(launch_pdl(k_swiglu, dim3(blocks), dim3(256), 0, st, gate, up,
                                (long long)ld_in, (int)rows, (int)n, variant, out, (long long)ldo,
                                il16),
                     "k_swiglu");
}

// Scratch: AM_MAX_ROWS arrival counters at a fixed place (they must stay
// zero between launches whatever the rows of a call), then the states.
constexpr size_t AM_MAX_ROWS = 4096;
size_t argmax_scratch_bytes(size_t rows, size_t n) {
  const size_t nct = (n + AM_SEG - 1) / AM_SEG;
  return rows * nct * sizeof(AmState) + AM_MAX_ROWS * sizeof(int) + 64;
}

syn_status_t launch_argmax(const float* x, size_t ldx, size_t rows, size_t n, int32_t* out,
                           int* len_adv, int adv, int max_len, int32_t* hist, int hist_ld,
                           void* scratch, cudaStream_t st) {
  if (!rows || !n) return SYN_OK;
  const size_t nct = (n + AM_SEG - 1) / AM_SEG;
  if (nct > 65535 || rows > AM_MAX_ROWS) return SYN_ERR_UNSUPPORTED;
  int* cnt = static_cast<int*>(scratch);  // zero before the first launch; left zero
  AmState* part = reinterpret_cast<AmState*>(static_cast<uint8_t*>(scratch) +
                                             AM_MAX_ROWS * sizeof(int));
  return cuda_status(launch_pdl(k_argmax, dim3((unsigned)nct, (unsigned)rows), dim3(AM_THREADS), 0,
                                st, x, (long long)ldx, (int)n, out, len_adv, adv, max_len, hist,
                                hist_ld, part,
                                cnt, static_cast<int4*>(nullptr), 0),
                     "k_argmax");
}

// Tensor-parallel greedy token: each rank's argmax state over its vocabulary
// slice (global indices) into pairs[row] ...
syn_status_t launch_argmax_slice(const float* x, size_t ldx, size_t rows, size_t n, int idx_off,
                                 void* pairs, void* scratch, cudaStream_t st) {
  if (!rows || !n) return SYN_OK;
  const size_t nct = (n + AM_SEG - 1) / AM_SEG;
  if (nct > 65535 || rows > AM_MAX_ROWS) return SYN_ERR_UNSUPPORTED;
  int* cnt = static_cast<int*>(scratch);
  AmState* part = reinterpret_cast<AmState*>(static_cast<uint8_t*>(scratch) +
                                             AM_MAX_ROWS * sizeof(int));
  return cuda_status(launch_pdl(k_argmax, dim3((unsigned)nct, (unsigned)rows), dim3(AM_THREADS), 0,
                                st, x, (long long)ldx, (int)n, static_cast<int32_t*>(nullptr),
                                static_cast<int*>(nullptr), 0, 0, static_cast<int32_t*>(nullptr),
                                0, part, cnt, static_cast<int4*>(pairs), idx_off),
                     "k_argmax");
}

// ... and, after the all-gather of the pairs ([world][rows], rank = vocabulary
// order), the combine in rank order: the same token as one argmax over the
// whole row (the later slice wins ties; the last NaN wins), then the length
// advance and token history of k_argmax.
__global__ void k_argmax_pairs(const int4* __restrict__ pairs, int world, int rows,
                               int32_t* __restrict__ out, int* len_adv, int adv, int max_len,
                               int32_t* hist, int hist_ld) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  AmState t{-1, -1, 0.0f};
  for (int r = 0; r < world; r++) {
    const int4 q = pairs[(size_t)r * rows + row];
    t = am_combine(t, AmState{q.x, q.y, __int_as_float(q.z)});
  }
  const int tok = t.i >= 0 ? t.i : (t.nan >= 0 ? t.nan : 0);
  out[row] = tok;
  if (len_adv) {
    int nl = len_adv[row] + adv;
    nl = nl <= max_len ? nl : max_len;
    len_adv[row] = nl;
    if (hist) hist[(size_t)row * hist_ld + nl] = tok;
  }
}

syn_status_t launch_argmax_pairs(const void* pairs, int world, size_t rows, int32_t* out,
                                 int* len_adv, int adv, int max_len, int32_t* hist, int hist_ld,
                                 cudaStream_t st) {
  if (!rows) return SYN_OK;
  const unsigned blocks = (unsigned)((rows + 127) / 128);
  return cuda_status(launch_pdl(k_argmax_pairs, dim3(blocks), dim3(128), 0, st,
                                static_cast<const int4*>(pairs), world, (int)rows, out, len_adv,
                                adv, max_len, hist, hist_ld),
                     "k_argmax_pairs");
}

}  // namespace syn

// ---------------------------------------------------------------------------
// decode / prefill launchers (need AttnParams, defined in the unnamed space)
// ---------------------------------------------------------------------------
namespace syn {
namespace {


size_t prefill_smem(int pr, int S, int hd) {
  return ((size_t)pr * hd + (size_t)PF_CH * (hd + 4) + (size_t)pr * S + 8 * 64) * sizeof(float);
}

int prefill_rows(int S, int hd) {
  for (int pr = 16; pr >= 1; pr >>= 1) {
    const size_t smem = prefill_smem(pr, S, hd);
    if (smem <= kMaxSmem && pr * hd <= 16 * PF_THREADS) return pr;
  }
  return 0;
}


syn_status_t make_params(const AttnArgs& a, AttnParams& p, int seq0, int ntok) {
  const syn_cuda_kvcache_t* c = a.cache;
  if (a.n_heads == 0 || a.n_heads % c->n_kv) return SYN_ERR_SHAPE_MISMATCH;
  if (a.layer >= c->layers) return SYN_ERR_INVALID_ARG;
  if (c->hd % 4 || c->hd < 8 || c->hd > 1024) return SYN_ERR_UNSUPPORTED;
  p.q = a.q;
  p.k = a.k;
  p.v = a.v;
  p.ld = (long long)a.ld;
  p.n_heads = (int)a.n_heads;
  p.n_kv = (int)c->n_kv;
  p.hd = (int)c->hd;
  p.qn = a.qn;
  p.kn = a.kn;
  p.eps = a.eps;
  p.cos_t = a.cos_t;
  p.sin_t = a.sin_t;
  p.window = (int)a.window;
  const size_t kvd = c->n_kv * c->hd;
  const size_t rows_per_layer = c->page ? c->n_pages * c->page : c->batch * c->max_seq;
  p.kc = c->k + a.layer * rows_per_layer * kvd;
  p.vc = c->v + a.layer * rows_per_layer * kvd;
  p.ptab = c->page ? c->d_ptab : nullptr;
  p.page = (int)c->page;
  p.maxp = (int)c->maxp;
  p.slots = a.slots;
  p.max_seq = (int)c->max_seq;
  p.len = c->d_len;
  p.seq0 = seq0;
  p.n_tokens = ntok;
  p.out = a.out;
  p.ldo = (long long)a.ldo;
  p.scale = 1.0f / sqrtf((float)c->hd);  // host: 1 / sqrt(hd) in f32
  p.err = nullptr;
  p.span = 0;
  p.rope_at_slot = 0;
  return SYN_OK;
}

}  // namespace

template <int HD>
void* gqa_kernel(int g) {
  switch (g) {
    case 1: return (void*)k_attn_decode_gqa<HD, 1>;
    case 2: return (void*)k_attn_decode_gqa<HD, 2>;
    case 4: return (void*)k_attn_decode_gqa<HD, 4>;
    case 8: return (void*)k_attn_decode_gqa<HD, 8>;
  }
  return nullptr;
}

syn_status_t launch_decode_flash(const AttnArgs& a, const AttnParams& p, size_t batch, size_t eff,
                                 cudaStream_t st) {
  syn_cuda_kvcache_t* c = a.cache;
  // KV-head-grouped kernel for head dims 64/128 and 1, 2, 4 or 8 query heads
  // per KV head (SYN_ATTN_GQA=0: the per-query-head kernel). Splits: about
  // four CTAs per SM over all (row, KV head) pairs, at most one per 64
  // positions of the longest context the launch may see.
  const int G = p.n_heads / p.n_kv;
  void* gqa = nullptr;
  static const bool gqa_on = [] {
    const char* e = getenv("SYN_ATTN_GQA");
    return !(e && e[0] == '0');
  }();
  if (gqa_on) gqa = p.hd == 128 ? gqa_kernel<128>(G) : p.hd == 64 ? gqa_kernel<64>(G) : nullptr;
  int nsplit;
  if (gqa) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long pairs = (long long)batch * p.n_kv;
    const long long want = (4LL * sms + pairs - 1) / pairs;
    // (the merge keeps a warp's split factors in its G * hd output slice)
    const long long cap = std::min<long long>(std::min(256, G * p.hd), ((long long)eff + 63) / 64);
    nsplit = (int)std::max<long long>(1, std::min(want, cap));
  } else {
    nsplit = (int)((eff + FD_CH - 1) / FD_CH);
  }
  if (nsplit > 32 * (p.hd + 4)) return SYN_ERR_UNSUPPORTED;  // combine factors fit in smem
  // arrival counters first, sized for every sequence slot, so that their
  // place does not move with the batch of a call (they must stay zero
  // between launches); the partials after them
  const size_t cbytes = (c->batch * p.n_heads * sizeof(int) + 255) & ~size_t(255);
  const size_t pbytes = batch * p.n_heads * (size_t)nsplit * (p.hd + 2) * sizeof(float);
  const size_t need = cbytes + pbytes;
  if (need > c->part_bytes || c->part_heads != p.n_heads) {
    // grows outside graph capture only; counters start at zero
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs != cudaStreamCaptureStatusNone) return SYN_ERR_UNSUPPORTED;
    cudaStreamSynchronize(st);
    cudaFree(c->part);
    c->part = nullptr;
    c->part_bytes = 0;
    if (cudaMalloc(&c->part, need) != cudaSuccess) return SYN_ERR_OUT_OF_MEMORY;
    if (cudaMemset(c->part, 0, need) != cudaSuccess) return SYN_ERR_CUDA;
    c->part_bytes = need;
    c->part_heads = p.n_heads;
  }
  int* cnt = reinterpret_cast<int*>(c->part);
  float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(c->part) + cbytes);
  if (gqa) {
    using K = void (*)(const AttnParams, float*, int*, int);
    return cuda_status(launch_pdl(reinterpret_cast<K>(gqa),
                                  dim3((unsigned)batch, (unsigned)p.n_kv, (unsigned)nsplit),
                                  dim3(GQ_THREADS), 0, st, p, part, cnt, nsplit),
                       "k_attn_decode_gqa");
  }
  void (*split)(const AttnParams, float*, int*, int) = nullptr;
  switch (p.hd) {
    case 32: split = k_attn_decode_split<32>; break;
    case 64: split = k_attn_decode_split<64>; break;
    case 128: split = k_attn_decode_split<128>; break;
    default: return SYN_ERR_UNSUPPORTED;
  }
  const size_t smem = flash_decode_smem(p.hd);
  syn_status_t s = allow_smem((const void*)split, smem);
  if (s) return s;
  return cuda_status(launch_pdl(split, dim3((unsigned)batch, (unsigned)p.n_heads, (unsigned)nsplit),
                                dim3(FD_THREADS), smem, st, p, part, cnt, nsplit),
                     "k_attn_decode_split");
}

syn_status_t launch_decode_p(const AttnArgs& a, AttnParams& p, size_t batch, cudaStream_t st);

syn_status_t launch_attn_decode_args(const AttnArgs& a, size_t batch, int* err, cudaStream_t st) {
  AttnParams p;
  syn_status_t s = make_params(a, p, 0, 1);
  if (s) return s;
  p.err = err;
  if (batch > a.cache->batch) return SYN_ERR_INVALID_ARG;
  if (!a.slots)  // (with a slot map the caller checks and maps the sequences)
    for (size_t b = 0; b < batch; b++) {
      if (a.cache->len[b] >= a.cache->max_seq) return SYN_ERR_INVALID_ARG;  // CacheFull
      if ((s = kv_reserve(a.cache, b, a.cache->len[b] + 1, st))) return s;
    }
  return launch_decode_p(a, p, batch, st);
}

// ntok new positions of sequence `seq` from its current length (a
// speculative-decoding verification): norm / RoPE at the cache slots and
// append, then each row attends to the cache up to its own position with
// the decode kernels (the same reductions as a one-token decode step).
syn_status_t launch_attn_span_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                   cudaStream_t st) {
  AttnParams p;
  syn_status_t s = make_params(a, p, (int)seq, (int)ntok);
  if (s) return s;
  p.err = err;
  if (seq >= a.cache->batch || ntok == 0) return SYN_ERR_INVALID_ARG;
  if (a.cache->len[seq] + ntok > a.cache->max_seq) return SYN_ERR_INVALID_ARG;  // CacheFull
  if ((s = kv_reserve(a.cache, seq, a.cache->len[seq] + ntok, st))) return s;
  p.rope_at_slot = 1;
  const int thr = std::max(32, p.hd / 2);
  s = cuda_status(launch_pdl(k_norm_rope_append, dim3((unsigned)ntok, (unsigned)(p.n_heads + p.n_kv)),
                             dim3(thr), (p.hd + 8) * sizeof(float), st, p),
                  "k_norm_rope_append");
  if (s) return s;
  p.rope_at_slot = 0;
  p.span = 1;
  return launch_decode_p(a, p, ntok, st);
}

syn_status_t launch_decode_p(const AttnArgs& a, AttnParams& p, size_t batch, cudaStream_t st) {
  syn_status_t s;
  // A captured graph replays at growing positions: size for the window.
  size_t eff = a.cache->max_seq;
  if (a.window && a.window < eff) eff = a.window;
  if (a.flash) return launch_decode_flash(a, p, batch, eff, st);
  const size_t smem = decode_smem_floats(p.hd, (int)eff) * sizeof(float);
  if (smem > kMaxSmem) return SYN_ERR_UNSUPPORTED;
  decode_stage_rows(p.hd, (int)eff, &p.krows, &p.vrows);
  void (*kern)(const AttnParams) = nullptr;
  switch (p.hd) {
    case 32: kern = k_attn_decode<32>; break;
    case 64: kern = k_attn_decode<64>; break;
    case 128: kern = k_attn_decode<128>; break;
    default: return SYN_ERR_UNSUPPORTED;
  }
  s = allow_smem((const void*)kern, smem);
  if (s) return s;
  return cuda_status(launch_pdl(kern, dim3((unsigned)batch, (unsigned)p.n_heads), dim3(DEC_THREADS),
                                smem, st, p),
                     "k_attn_decode");
}

syn_status_t launch_norm_rope_append_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                          cudaStream_t st) {
  AttnParams p;
  syn_status_t s = make_params(a, p, (int)seq, (int)ntok);
  if (s) return s;
  p.err = err;
  if (seq >= a.cache->batch) return SYN_ERR_INVALID_ARG;
  if (a.cache->len[seq] + ntok > a.cache->max_seq) return SYN_ERR_INVALID_ARG;  // CacheFull
  if (ntok == 0) return SYN_OK;
  if ((s = kv_reserve(a.cache, seq, a.cache->len[seq] + ntok, st))) return s;
  const int thr = std::max(32, p.hd / 2);
  const size_t smem = (p.hd + 8) * sizeof(float);
  return cuda_status(
      launch_pdl(k_norm_rope_append, dim3((unsigned)ntok, (unsigned)(p.n_heads + p.n_kv)),
                 dim3(thr), smem, st, p),
      "k_norm_rope_append");
}

syn_status_t launch_prefill_attention_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                           cudaStream_t st) {
  AttnParams p;
  syn_status_t s = make_params(a, p, (int)seq, (int)ntok);
  if (s) return s;
  p.err = err;
  if (seq >= a.cache->batch) return SYN_ERR_INVALID_ARG;
  if (a.cache->len[seq] + ntok > a.cache->max_seq) return SYN_ERR_INVALID_ARG;
  if (ntok == 0) return SYN_OK;
  static const int use_tc = [] {
    const char* v = getenv("SYN_ATTN_TC");
    return v ? atoi(v) : 1;
  }();
  if (a.flash && use_tc && (p.hd == 64 || p.hd == 128)) {
    void (*kern)(const AttnParams) = p.hd == 64 ? k_attn_prefill_tc<64> : k_attn_prefill_tc<128>;
    const size_t fs = p.hd == 64 ? TcaSmem<64>::BYTES : TcaSmem<128>::BYTES;
    if ((s = allow_smem((const void*)kern, fs))) return s;
    return cuda_status(launch_pdl(kern, dim3((unsigned)p.n_heads, (unsigned)((ntok + TCA_Q - 1) / TCA_Q)),
                                  dim3(TCA_THREADS), fs, st, p),
                       "k_attn_prefill_tc");
  }
  if (a.flash && (p.hd == 64 || p.hd == 128)) {
    void (*kern)(const AttnParams) = p.hd == 64 ? k_attn_prefill_flash<64> : k_attn_prefill_flash<128>;
    const size_t fs = flash_prefill_smem(p.hd);
    if ((s = allow_smem((const void*)kern, fs))) return s;
    return cuda_status(launch_pdl(kern, dim3((unsigned)p.n_heads, (unsigned)((ntok + FP_B - 1) / FP_B)),
                                  dim3(FP_THREADS), fs, st, p),
                       "k_attn_prefill_flash");
  }
  const int pr = prefill_rows((int)ntok, p.hd);
  if (!pr) return SYN_ERR_UNSUPPORTED;
  const size_t smem = prefill_smem(pr, (int)ntok, p.hd);
  s = allow_smem((const void*)k_attn_prefill, smem);
  if (s) return s;
  return cuda_status(launch_pdl(k_attn_prefill,
                                dim3((unsigned)p.n_heads, (unsigned)((ntok + pr - 1) / pr)),
                                dim3(PF_THREADS), smem, st, p, pr),
                     "k_attn_prefill");
}

syn_status_t launch_attn_prefill_args(const AttnArgs& a, size_t seq, size_t ntok, int* err,
                                      cudaStream_t st) {
  syn_status_t s = launch_norm_rope_append_args(a, seq, ntok, err, st);
  if (s) return s;
  return launch_prefill_attention_args(a, seq, ntok, err, st);
}

syn_status_t kv_reserve(syn_cuda_kvcache_t* c, size_t seq, size_t new_len, cudaStream_t st) {
  if (!c->page) return SYN_OK;
  if (seq >= c->batch || new_len > c->max_seq) return SYN_ERR_INVALID_ARG;
  int* row = c->ptab_h + seq * c->maxp;
  const size_t need = (new_len + c->page - 1) / c->page;
  size_t first = need;
  for (size_t i = 0; i < need; i++) {
    if (row[i] >= 0) continue;
    if (!c->n_free) {
      set_last_cuda_error(cudaErrorMemoryAllocation, "paged KV cache: no free page");
      return SYN_ERR_OUT_OF_MEMORY;
    }
    row[i] = c->free_pages[--c->n_free];
    first = std::min(first, i);
  }
  if (first < need)
    SYN_CUDA_TRY(cudaMemcpyAsync(c->d_ptab + seq * c->maxp + first, row + first,
                                 (need - first) * sizeof(int), cudaMemcpyHostToDevice, st));
  return SYN_OK;
}

// Returns the pages of sequence seq beyond position keep_len to the free
// list. The stream is drained first: queued work may still read the table.
syn_status_t kv_release(syn_cuda_kvcache_t* c, size_t seq, size_t keep_len, cudaStream_t st) {
  if (!c->page) return SYN_OK;
  SYN_CUDA_TRY(cudaStreamSynchronize(st));
  int* row = c->ptab_h + seq * c->maxp;
  const size_t keep = (keep_len + c->page - 1) / c->page;
  bool changed = false;
  for (size_t i = keep; i < c->maxp; i++)
    if (row[i] >= 0) {
      c->free_pages[c->n_free++] = row[i];
      row[i] = -1;
      changed = true;
    }
  if (changed)
    SYN_CUDA_TRY(cudaMemcpy(c->d_ptab + seq * c->maxp, row, c->maxp * sizeof(int),
                            cudaMemcpyHostToDevice));
  return SYN_OK;
}

__global__ void k_kv_advance_slots(int* len, const int* slots, int n) {
  griddep_wait();
  griddep_launch();
  for (int i = threadIdx.x; i < n; i += blockDim.x) len[slots[i]] += 1;
}

syn_status_t launch_kv_advance_slots(syn_cuda_kvcache_t* c, const int* slots, size_t n,
                                     cudaStream_t st) {
  return cuda_status(launch_pdl(k_kv_advance_slots, dim3(1), dim3(128), 0, st, c->d_len, slots,
                                (int)n),
                     "k_kv_advance_slots");
}

syn_status_t launch_kv_set(syn_cuda_kvcache_t* c, size_t seq, int value, int add, cudaStream_t st) {
  return cuda_status(launch_pdl(k_kv_set, dim3(1), dim3(32), 0, st, c->d_len, (int)seq, value, add),
                     "k_kv_set");
}

}  // namespace syn

// ===========================================================================
// C ABI
// ===========================================================================
using namespace syn;

extern "C" {

syn_status_t syn_cuda_rope_tables(double base, size_t max_pos, size_t head_dim, float* cos_out,
                                  float* sin_out) {
  if (!cos_out || !sin_out) return SYN_ERR_NULL_PTR;
  if (head_dim == 0 || head_dim % 2) return SYN_ERR_INVALID_ARG;
  const size_t half = head_dim / 2;
  for (size_t pos = 0; pos < max_pos; pos++)
    for (size_t i = 0; i < half; i++) {
      const float freq = 1.0f / powf((float)base, (2.0f * (float)i) / (float)head_dim);
      const float scaled = freq / 1.0f;
      const float angle = (float)pos * scaled;
      cos_out[pos * half + i] = cosf(angle);
      sin_out[pos * half + i] = sinf(angle);
    }
  return SYN_OK;
}

syn_status_t syn_cuda_rmsnorm(const float* x, const float* weight, size_t rows, size_t hidden,
                              float eps, float* out, void* stream) {
  if (!x || !weight || !out) return SYN_ERR_NULL_PTR;
  return launch_add_rmsnorm(x, hidden, nullptr, 0, nullptr, nullptr, 0, nullptr, 0, weight, rows,
                            hidden, eps, out, hidden, (cudaStream_t)stream);
}

syn_status_t syn_cuda_add_rmsnorm(float* residual, const float* delta, const float* weight,
                                  size_t rows, size_t hidden, float eps, float* out,
                                  void* stream) {
  if (!residual || !delta || !weight || !out) return SYN_ERR_NULL_PTR;
  return launch_add_rmsnorm(residual, hidden, delta, hidden, nullptr, nullptr, 0, residual, hidden,
                            weight, rows, hidden, eps, out, hidden, (cudaStream_t)stream);
}

syn_status_t syn_cuda_embed_rmsnorm(const float* table, size_t vocab, const int32_t* ids,
                                    size_t rows, size_t hidden, const float* weight, float eps,
                                    float* x_out, float* out, void* stream) {
  if (!table || !ids || !weight || !out) return SYN_ERR_NULL_PTR;
  return launch_add_rmsnorm(nullptr, 0, nullptr, 0, ids, table, vocab, x_out, hidden, weight, rows,
                            hidden, eps, out, hidden, (cudaStream_t)stream);
}

syn_status_t syn_cuda_kvcache_create_paged(syn_cuda_ctx_t* ctx, size_t max_seq,
                                           size_t n_kv_heads, size_t head_dim, size_t num_layers,
                                           size_t batch, size_t page, size_t n_pages,
                                           syn_cuda_kvcache_t** out) {
  if (!ctx || !out) return SYN_ERR_NULL_PTR;
  *out = nullptr;
  if (!max_seq || !n_kv_heads || !head_dim || !num_layers || !batch)
    return SYN_ERR_INVALID_DIMENSIONS;  // kvcache.zig:31-34
  if (max_seq > 0x7FFFFFF || head_dim % 4) return SYN_ERR_UNSUPPORTED;
  if (page && (!n_pages || n_pages > 0x7FFFFFF || page > max_seq)) return SYN_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  if (!g.ok) return SYN_ERR_CUDA;
  auto* c = new (std::nothrow) syn_cuda_kvcache_s();
  if (!c) return SYN_ERR_OUT_OF_MEMORY;
  c->device = ctx->device;
  c->max_seq = max_seq;
  c->n_kv = n_kv_heads;
  c->hd = head_dim;
  c->layers = num_layers;
  c->batch = batch;
  c->page = page;
  c->n_pages = page ? n_pages : 0;
  c->maxp = page ? (max_seq + page - 1) / page : 0;
  const size_t rows = page ? n_pages * page : batch * max_seq;
  const size_t elems = num_layers * rows * n_kv_heads * head_dim;
  c->len = new (std::nothrow) size_t[batch]();
  cudaError_t e = c->len ? cudaMalloc(&c->k, elems * sizeof(float)) : cudaErrorMemoryAllocation;
  if (e == cudaSuccess) e = cudaMalloc(&c->v, elems * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&c->d_len, batch * sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->k, 0, elems * sizeof(float));
  if (e == cudaSuccess) e = cudaMemset(c->v, 0, elems * sizeof(float));
  if (e == cudaSuccess) e = cudaMemset(c->d_len, 0, batch * sizeof(int));
  if (e == cudaSuccess && page) {
    e = cudaMallocHost(&c->ptab_h, batch * c->maxp * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&c->d_ptab, batch * c->maxp * sizeof(int));
    c->free_pages = e == cudaSuccess ? new (std::nothrow) int[n_pages] : nullptr;
    if (e == cudaSuccess && !c->free_pages) e = cudaErrorMemoryAllocation;
    if (e == cudaSuccess) {
      for (size_t i = 0; i < batch * c->maxp; i++) c->ptab_h[i] = -1;
      for (size_t i = 0; i < n_pages; i++) c->free_pages[i] = (int)(n_pages - 1 - i);
      c->n_free = n_pages;
      e = cudaMemcpy(c->d_ptab, c->ptab_h, batch * c->maxp * sizeof(int), cudaMemcpyHostToDevice);
    }
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "syn_cuda_kvcache_create");
    cudaFree(c->k);
    cudaFree(c->v);
    cudaFree(c->d_len);
    cudaFree(c->d_ptab);
    if (c->ptab_h) cudaFreeHost(c->ptab_h);
    delete[] c->free_pages;
    delete[] c->len;
    delete c;
    return SYN_ERR_OUT_OF_MEMORY;
  }
  *out = c;
  return SYN_OK;
}

syn_status_t syn_cuda_kvcache_create(syn_cuda_ctx_t* ctx, size_t max_seq, size_t n_kv_heads,
                                     size_t head_dim, size_t num_layers, size_t batch,
                                     syn_cuda_kvcache_t** out) {
  return syn_cuda_kvcache_create_paged(ctx, max_seq, n_kv_heads, head_dim, num_layers, batch, 0,
                                       0, out);
}

syn_status_t syn_cuda_kvcache_pages_free(const syn_cuda_kvcache_t* c, size_t* n) {
  if (!c || !n) return SYN_ERR_NULL_PTR;
  *n = c->page ? c->n_free : 0;
  return SYN_OK;
}

syn_status_t syn_cuda_kvcache_destroy(syn_cuda_kvcache_t* c) {
  if (!c) return SYN_ERR_NULL_PTR;
  DeviceGuard g(c->device);
  cudaDeviceSynchronize();
  cudaFree(c->k);
  cudaFree(c->v);
  cudaFree(c->d_len);
  cudaFree(c->part);
  cudaFree(c->d_ptab);
  if (c->ptab_h) cudaFreeHost(c->ptab_h);
  delete[] c->free_pages;
  delete[] c->len;
  delete c;
  return SYN_OK;
}

syn_status_t syn_cuda_kvcache_len(const syn_cuda_kvcache_t* c, size_t seq, size_t* len) {
  if (!c || !len) return SYN_ERR_NULL_PTR;
  if (seq >= c->batch) return SYN_ERR_INVALID_ARG;
  *len = c->len[seq];
  return SYN_OK;
}

syn_status_t syn_cuda_kvcache_view(const syn_cuda_kvcache_t* c, size_t layer, size_t seq,
                                   float** k, float** v) {
  if (!c) return SYN_ERR_NULL_PTR;
  if (layer >= c->layers || seq >= c->batch) return SYN_ERR_INVALID_ARG;
  if (c->page) return SYN_ERR_UNSUPPORTED;  // a paged sequence is not one contiguous range
  const size_t off = (layer * c->batch + seq) * c->max_seq * c->n_kv * c->hd;
  if (k) *k = c->k + off;
  if (v) *v = c->v + off;
  return SYN_OK;
}

syn_status_t syn_cuda_kvcache_append(syn_cuda_kvcache_t* c, size_t layer, size_t seq,
                                     const float* k, const float* v, size_t n_tokens,
                                     void* stream) {
  if (!c || !k || !v) return SYN_ERR_NULL_PTR;
  if (layer >= c->layers || seq >= c->batch) return SYN_ERR_INVALID_ARG;
  if (c->len[seq] + n_tokens > c->max_seq) return SYN_ERR_INVALID_ARG;  // CacheFull
  if (!n_tokens) return SYN_OK;
  DeviceGuard g(c->device);
  const size_t row = c->n_kv * c->hd;
  cudaStream_t st = (cudaStream_t)stream;
  if (c->page) {  // page by page
    syn_status_t s = kv_reserve(c, seq, c->len[seq] + n_tokens, st);
    if (s) return s;
    const size_t base = layer * c->n_pages * c->page;
    for (size_t t = 0; t < n_tokens;) {
      const size_t pos = c->len[seq] + t, in = pos % c->page;
      const size_t run = std::min(n_tokens - t, c->page - in);
      const size_t slot = base + (size_t)c->ptab_h[seq * c->maxp + pos / c->page] * c->page + in;
      SYN_CUDA_TRY(cudaMemcpyAsync(c->k + slot * row, k + t * row, run * row * 4,
                                   cudaMemcpyDeviceToDevice, st));
      SYN_CUDA_TRY(cudaMemcpyAsync(c->v + slot * row, v + t * row, run * row * 4,
                                   cudaMemcpyDeviceToDevice, st));
      t += run;
    }
    return SYN_OK;
  }
  float *kd, *vd;
  syn_cuda_kvcache_view(c, layer, seq, &kd, &vd);
  const size_t off = c->len[seq] * row, bytes = n_tokens * row * 4;
  SYN_CUDA_TRY(cudaMemcpyAsync(kd + off, k, bytes, cudaMemcpyDeviceToDevice, st));
  SYN_CUDA_TRY(cudaMemcpyAsync(vd + off, v, bytes, cudaMemcpyDeviceToDevice, st));
  return SYN_OK;
}

syn_status_t syn_cuda_kvcache_advance(syn_cuda_kvcache_t* c, size_t seq, size_t n, void* stream) {
  if (!c) return SYN_ERR_NULL_PTR;
  if (seq >= c->batch) return SYN_ERR_INVALID_ARG;
  if (c->len[seq] + n > c->max_seq) return SYN_ERR_INVALID_ARG;  // CacheFull
  DeviceGuard g(c->device);
  syn_status_t s = kv_reserve(c, seq, c->len[seq] + n, (cudaStream_t)stream);
  if (s) return s;
  s = launch_kv_set(c, seq, (int)n, 1, (cudaStream_t)stream);
  if (s == SYN_OK) c->len[seq] += n;
  return s;
}

syn_status_t syn_cuda_kvcache_truncate(syn_cuda_kvcache_t* c, size_t seq, size_t new_len,
                                       void* stream) {
  if (!c) return SYN_ERR_NULL_PTR;
  if (seq >= c->batch) return SYN_ERR_INVALID_ARG;
  if (new_len >= c->len[seq]) return SYN_OK;  // kvcache.zig:109-113
  DeviceGuard g(c->device);
  syn_status_t s = launch_kv_set(c, seq, (int)new_len, 0, (cudaStream_t)stream);
  if (s == SYN_OK) c->len[seq] = new_len;
  if (s == SYN_OK) s = kv_release(c, seq, new_len, (cudaStream_t)stream);
  return s;
}

syn_status_t syn_cuda_kvcache_reset(syn_cuda_kvcache_t* c, size_t seq, void* stream) {
  if (!c) return SYN_ERR_NULL_PTR;
  if (seq >= c->batch) return SYN_ERR_INVALID_ARG;
  DeviceGuard g(c->device);
  syn_status_t s = launch_kv_set(c, seq, 0, 0, (cudaStream_t)stream);
  if (s == SYN_OK) c->len[seq] = 0;
  if (s == SYN_OK) s = kv_release(c, seq, 0, (cudaStream_t)stream);
  return s;
}

syn_status_t syn_cuda_attention_decode(syn_cuda_kvcache_t* cache, size_t layer, size_t batch,
                                       float* q, const float* k, const float* v, size_t ld,
                                       size_t n_heads, const float* q_norm, const float* k_norm,
                                       float eps, const float* rope_cos, const float* rope_sin,
                                       size_t window, float* out, size_t ldo, void* stream) {
  if (!cache || !q || !k || !v || !rope_cos || !rope_sin || !out) return SYN_ERR_NULL_PTR;
  if (!batch) return SYN_OK;
  DeviceGuard g(cache->device);
  AttnArgs a{q, k, v, ld, n_heads, q_norm, k_norm, eps, rope_cos, rope_sin, window, cache, layer,
             out, ldo};
  return launch_attn_decode_args(a, batch, nullptr, (cudaStream_t)stream);
}

syn_status_t syn_cuda_qk_norm_rope_kv_append(syn_cuda_kvcache_t* cache, size_t layer, size_t seq,
                                             size_t n_tokens, float* q, const float* k,
                                             const float* v, size_t ld, size_t n_heads,
                                             const float* q_norm, const float* k_norm, float eps,
                                             const float* rope_cos, const float* rope_sin,
                                             void* stream) {
  if (!cache || !q || !k || !v || !rope_cos || !rope_sin) return SYN_ERR_NULL_PTR;
  DeviceGuard g(cache->device);
  AttnArgs a{q, k, v, ld, n_heads, q_norm, k_norm, eps, rope_cos, rope_sin, 0, cache, layer,
             nullptr, 0};
  return launch_norm_rope_append_args(a, seq, n_tokens, nullptr, (cudaStream_t)stream);
}

syn_status_t syn_cuda_attention_prefill(syn_cuda_kvcache_t* cache, size_t layer, size_t seq,
                                        size_t n_tokens, float* q, const float* k, const float* v,
                                        size_t ld, size_t n_heads, const float* q_norm,
                                        const float* k_norm, float eps, const float* rope_cos,
                                        const float* rope_sin, float* out, size_t ldo,
                                        void* stream) {
  if (!cache || !q || !k || !v || !rope_cos || !rope_sin || !out) return SYN_ERR_NULL_PTR;
  DeviceGuard g(cache->device);
  AttnArgs a{q, k, v, ld, n_heads, q_norm, k_norm, eps, rope_cos, rope_sin, 0, cache, layer,
             out, ldo};
  return launch_attn_prefill_args(a, seq, n_tokens, nullptr, (cudaStream_t)stream);
}

syn_status_t syn_cuda_attention_decode_flash(
    syn_cuda_kvcache_t* cache, size_t layer, size_t batch, float* q, const float* k,
    const float* v, size_t ld, size_t n_heads, const float* q_norm, const float* k_norm, float eps,
    const float* rope_cos, const float* rope_sin, size_t window, float* out, size_t ldo,
    void* stream) {
  if (!cache || !q || !k || !v || !rope_cos || !rope_sin || !out) return SYN_ERR_NULL_PTR;
  if (!batch) return SYN_OK;
  DeviceGuard g(cache->device);
  AttnArgs a{q, k, v, ld, n_heads, q_norm, k_norm, eps, rope_cos, rope_sin, window, cache, layer,
             out, ldo, 1};
  return launch_attn_decode_args(a, batch, nullptr, (cudaStream_t)stream);
}

syn_status_t syn_cuda_attention_prefill_flash(
    syn_cuda_kvcache_t* cache, size_t layer, size_t seq, size_t n_tokens, float* q, const float* k,
    const float* v, size_t ld, size_t n_heads, const float* q_norm, const float* k_norm, float eps,
    const float* rope_cos, const float* rope_sin, float* out, size_t ldo, void* stream) {
  if (!cache || !q || !k || !v || !rope_cos || !rope_sin || !out) return SYN_ERR_NULL_PTR;
  DeviceGuard g(cache->device);
  AttnArgs a{q, k, v, ld, n_heads, q_norm, k_norm, eps, rope_cos, rope_sin, 0, cache, layer,
             out, ldo, 1};
  return launch_attn_prefill_args(a, seq, n_tokens, nullptr, (cudaStream_t)stream);
}

syn_status_t syn_cuda_swiglu(const float* gate, const float* up, size_t ld_in, size_t rows,
                             size_t n, int variant, float* out, size_t ldo, void* stream) {
  if (!gate || !up || !out) return SYN_ERR_NULL_PTR;
  if (variant != 0 && variant != 1) return SYN_ERR_INVALID_ARG;
  return launch_swiglu(gate, up, ld_in, rows, n, variant, out, ldo, (cudaStream_t)stream);
}

syn_status_t syn_cuda_argmax(const float* logits, size_t rows, size_t n, int32_t* out_idx,
                             void* stream) {
  if (!logits || !out_idx) return SYN_ERR_NULL_PTR;
  if (n > 0x7FFFFFFF) return SYN_ERR_UNSUPPORTED;
  if (!rows || !n) return SYN_OK;
  cudaStream_t st = (cudaStream_t)stream;
  // stream-ordered scratch: zeroed arrival counters + per-CTA states
  void* scratch = nullptr;
  const size_t bytes = argmax_scratch_bytes(rows, n);
  SYN_CUDA_TRY(cudaMallocAsync(&scratch, bytes, st));
  cudaError_t e = cudaMemsetAsync(scratch, 0, bytes, st);
  syn_status_t s = e == cudaSuccess
                       ? launch_argmax(logits, n, rows, n, out_idx, nullptr, 0, 0, nullptr, 0, scratch, st)
                       : cuda_status(e, "cudaMemsetAsync");
  e = cudaFreeAsync(scratch, st);
  if (s == SYN_OK && e != cudaSuccess) s = cuda_status(e, "cudaFreeAsync");
  return s;
}

}  // extern "C"
