// capi.cu -- the extern "C" boundary declared in include/synapse_cuda.h.
//
// Argument checking follows zig/src/ffi/exports.zig: null pointers first
// (SYN_ERR_NULL_PTR), then the zero-size early-out (SYN_OK), then shape
// checks. Nothing throws across the boundary.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "internal.cuh"

namespace syn {

static thread_local char g_last_error[256] = "";

void set_last_cuda_error(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorName(e),
           cudaGetErrorString(e));
}

int num_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> g(mu);
  if (!cache[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 148;
  }
  return cache[dev];
}

namespace {

size_t block_elems(int fmt) {
  switch (fmt) {
    case SYN_QFMT_Q4_0:
    case SYN_QFMT_Q8_0: return 32;
    case SYN_QFMT_Q4_K:
    case SYN_QFMT_Q6_K: return 256;
  }
  return 1;
}

size_t src_row_bytes(int fmt, size_t k) {
  switch (fmt) {
    case SYN_QFMT_Q4_0: return k / 32 * 18;
    case SYN_QFMT_Q8_0: return k / 32 * 34;
    case SYN_QFMT_Q4_K: return k / 256 * 144;
    case SYN_QFMT_Q6_K: return k / 256 * 210;
  }
  return k;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Lays out the repacked arrays of `w` inside one allocation; returns bytes.
// Rows are stored in groups of 32 (row-interleaved tiles), zero padded.
size_t layout(syn_cuda_weight_s* w, uint8_t* base) {
  size_t off = 0;
  const size_t n = (w->n + 31) / 32 * 32, k = w->k;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off = align256(off + bytes);
    return p;
  };
  switch (w->fmt) {
    case SYN_QFMT_INT8_KN:
      w->q = take(n * w->kp);
      w->sb = reinterpret_cast<float*>(take(n * 4));
      break;
    case SYN_QFMT_Q4_0:
      w->q = take(n * k / 2);
      w->d = reinterpret_cast<uint16_t*>(take(n * (k / 32) * 2));
      break;
    case SYN_QFMT_Q8_0:
      w->q = take(n * k);
      w->d = reinterpret_cast<uint16_t*>(take(n * (k / 32) * 2));
      break;
    case SYN_QFMT_Q4_K:
      w->q = take(n * k / 2);
      w->hdr = take(n * (k / 256) * 16);
      break;
    case SYN_QFMT_Q6_K:
      w->q = take(n * k / 2);
      w->qh = take(n * (k / 32) * 8);
      w->sc = reinterpret_cast<int8_t*>(take(n * (k / 32) * 2));
      w->d = reinterpret_cast<uint16_t*>(take(n * (k / 256) * 2));
      break;
  }
  return off;
}

// Grows one of the context's scratch buffers (zero-filled). Growth frees the
// old buffer, so it waits for the device first; it is refused while `st` is
// being captured into a graph.
syn_status_t grow(void** buf, size_t* cap, size_t bytes, cudaStream_t st) {
  if (bytes <= *cap) return SYN_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  SYN_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
  if (cs != cudaStreamCaptureStatusNone) return SYN_ERR_UNSUPPORTED;
  SYN_CUDA_TRY(cudaDeviceSynchronize());
  cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  const size_t want = align256(bytes) * 2;
  cudaError_t e = cudaMalloc(buf, want);
  if (e == cudaSuccess) e = cudaMemset(*buf, 0, want);
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "cudaMalloc(scratch)");
    return SYN_ERR_OUT_OF_MEMORY;
  }
  *cap = want;
  return SYN_OK;
}

}  // namespace

syn_status_t ensure_scratch(syn_cuda_ctx_s* ctx, const syn_cuda_weight_s* w, size_t m,
                            cudaStream_t st) {
  syn_status_t s = grow(reinterpret_cast<void**>(&ctx->part), &ctx->part_bytes,
                        gemv_partial_bytes(w->fmt, m, w->n, w->kp, w->k), st);
  if (s != SYN_OK) return s;
  return grow(reinterpret_cast<void**>(&ctx->cnt), &ctx->cnt_bytes, gemv_counter_bytes(m, w->n),
              st);
}

namespace {

// Stream-ordered scratch for the context-free entry points: `extra` leading
// bytes for the caller, then partials and zeroed counters; freed after the
// launch (stream-ordered).
struct CallScratch {
  void* mem = nullptr;
  float* part = nullptr;
  size_t part_cap = 0;
  int* cnt = nullptr;
  syn_status_t init(int fmt, size_t m, size_t n, size_t kp, size_t extra, cudaStream_t st) {
    const size_t pb = align256(gemv_partial_bytes(fmt, m, n, kp));
    part_cap = pb;
    const size_t cb = align256(gemv_counter_bytes(m, n));
    SYN_CUDA_TRY(cudaMallocAsync(&mem, extra + pb + cb + 256, st));
    part = reinterpret_cast<float*>(static_cast<uint8_t*>(mem) + extra);
    cnt = reinterpret_cast<int*>(static_cast<uint8_t*>(mem) + extra + pb);
    SYN_CUDA_TRY(cudaMemsetAsync(cnt, 0, cb, st));
    return SYN_OK;
  }
  syn_status_t release(syn_status_t s, cudaStream_t st) {
    if (!mem) return s;
    cudaError_t e = cudaFreeAsync(mem, st);
    if (s == SYN_OK && e != cudaSuccess) {
      set_last_cuda_error(e, "cudaFreeAsync");
      return SYN_ERR_CUDA;
    }
    return s;
  }
};

}  // namespace

size_t weight_layout(syn_cuda_weight_s* w, uint8_t* base) { return layout(w, base); }
size_t weight_src_row_bytes(int fmt, size_t k) { return src_row_bytes(fmt, k); }

}  // namespace syn

using namespace syn;

extern "C" {

const char* syn_cuda_status_string(syn_status_t s) {
  switch (s) {
    case SYN_OK: return "ok";
    case SYN_ERR_NULL_PTR: return "null pointer";
    case SYN_ERR_INVALID_ARG: return "invalid argument";
    case SYN_ERR_OUT_OF_MEMORY: return "out of memory";
    case SYN_ERR_SHAPE_MISMATCH: return "shape mismatch";
    case SYN_ERR_NOT_CONTIGUOUS: return "not contiguous";
    case SYN_ERR_INVALID_AXIS: return "invalid axis";
    case SYN_ERR_INVALID_DIMENSIONS: return "invalid dimensions";
    case SYN_ERR_INTERNAL: return "internal error";
    case SYN_ERR_CUDA: return "CUDA error";
    case SYN_ERR_NCCL: return "NCCL error";
    case SYN_ERR_TIMEOUT: return "timeout";
    case SYN_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

const char* syn_cuda_last_error(void) { return g_last_error; }

syn_status_t syn_cuda_capability_summary(syn_capability_summary_t* out) {
  if (!out) return SYN_ERR_NULL_PTR;
  out->abi_version = 1;
  out->target_arch = 2; /* SYN_ARCH_X86_64 host */
  out->target_os = 2;   /* SYN_OS_LINUX */
  out->simd_backend = SYN_BACKEND_CUDA_SM100;
  out->runtime_profile = 1; /* SYN_RUNTIME_NATIVE_PERF */
  out->support_level = 3;   /* SYN_SUPPORT_EXPERIMENTAL */
  out->feature_bits = SYN_CUDA_FEATURE_INT8_QUANT | SYN_CUDA_FEATURE_Q4_0_GEMV |
                      SYN_CUDA_FEATURE_QMATMUL;
  return SYN_OK;
}

syn_status_t syn_cuda_context_create(int device, syn_cuda_ctx_t** out) {
  if (!out) return SYN_ERR_NULL_PTR;
  *out = nullptr;
  int count = 0;
  SYN_CUDA_TRY(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count) return SYN_ERR_INVALID_ARG;
  DeviceGuard g(device);
  if (!g.ok) return SYN_ERR_CUDA;
  auto* c = new (std::nothrow) syn_cuda_ctx_s();
  if (!c) return SYN_ERR_OUT_OF_MEMORY;
  c->device = device;
  c->sms = num_sms();
  cudaError_t e = cudaStreamCreateWithFlags(&c->upload_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof(int));
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "syn_cuda_context_create");
    if (c->err) cudaFree(c->err);
    if (c->upload_stream) cudaStreamDestroy(c->upload_stream);
    delete c;
    return e == cudaErrorMemoryAllocation ? SYN_ERR_OUT_OF_MEMORY : SYN_ERR_CUDA;
  }
  *out = c;
  return SYN_OK;
}

syn_status_t syn_cuda_context_get_error(syn_cuda_ctx_t* ctx, int32_t* status) {
  if (!ctx || !status) return SYN_ERR_NULL_PTR;
  DeviceGuard g(ctx->device);
  int v = 0;
  SYN_CUDA_TRY(cudaMemcpy(&v, ctx->err, sizeof(int), cudaMemcpyDeviceToHost));
  SYN_CUDA_TRY(cudaMemset(ctx->err, 0, sizeof(int)));
  *status = v;
  return SYN_OK;
}

syn_status_t syn_cuda_context_destroy(syn_cuda_ctx_t* ctx) {
  if (!ctx) return SYN_ERR_NULL_PTR;
  {
    DeviceGuard g(ctx->device);
    cudaDeviceSynchronize();
    cudaStreamDestroy(ctx->upload_stream);
    cudaFree(ctx->part);
    cudaFree(ctx->cnt);
    cudaFree(ctx->abuf);
    cudaFree(ctx->err);
    tp_release(ctx);
  }
  delete ctx;
  return SYN_OK;
}

syn_status_t syn_cuda_quantize_per_channel_int8(const float* data, size_t channels,
                                                size_t channel_size, int8_t* out, float* scales,
                                                void* stream) {
  if (!data || !out || !scales) return SYN_ERR_NULL_PTR;
  if (channels == 0 || channel_size == 0) return SYN_ERR_INVALID_ARG;
  return launch_quantize_rows(data, channels, channel_size, out, scales, (cudaStream_t)stream);
}

syn_status_t syn_cuda_quantize_weights_int8(const float* w, size_t n, size_t k, int8_t* out_kn,
                                            float* scales, void* stream) {
  if (!w || !out_kn || !scales) return SYN_ERR_NULL_PTR;
  if (n == 0 || k == 0) return SYN_OK;
  return launch_quantize_weights(w, n, k, out_kn, scales, (cudaStream_t)stream);
}

syn_status_t syn_cuda_qgemm_int8(size_t m, size_t n, size_t k, const int8_t* a, size_t lda,
                                 const int8_t* b, size_t ldb, float* c, size_t ldc,
                                 const float* scales_a, const float* scales_b, void* stream) {
  if (!a || !b || !c || !scales_a || !scales_b) return SYN_ERR_NULL_PTR;
  if (m == 0 || n == 0 || k == 0) return SYN_OK;
  if (lda < k || ldb < n || ldc < n) return SYN_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  // The reference's [K,N] operand is transposed into the coalesced
  // row-interleaved layout in stream-ordered scratch, then the GEMV runs.
  syn_cuda_weight_s w{};
  w.fmt = SYN_QFMT_INT8_KN;
  w.n = n;
  w.k = k;
  w.kp = (k + 31) / 32 * 32;
  const size_t wbytes = align256((n + 31) / 32 * 32 * w.kp);
  const bool gemm = m >= gemm_min_rows(w.fmt, n);
  const size_t abytes = gemm ? align256(gemm_a_bytes(w.fmt, m, w.kp)) : 0;
  CallScratch cs;
  syn_status_t s = cs.init(w.fmt, m, n, w.kp, wbytes + abytes, st);
  if (s != SYN_OK) return cs.release(s, st);
  w.buf = cs.mem;
  w.bytes = wbytes;
  w.q = static_cast<uint8_t*>(cs.mem);
  w.sb = const_cast<float*>(scales_b);  // read only for rows < n
  s = repack_weight(&w, reinterpret_cast<const uint8_t*>(b), ldb, nullptr, st);
  if (s == SYN_OK && gemm)
    s = launch_qgemm(&w, nullptr, lda, a, scales_a, m, c, ldc, m > 16 ? 1 : 0,
                     static_cast<uint8_t*>(cs.mem) + wbytes, nullptr, st);
  else if (s == SYN_OK)
    s = launch_qgemv(&w, nullptr, lda, a, scales_a, m, c, ldc, m > 16 ? 1 : 0, cs.part, cs.part_cap,
                     cs.cnt, nullptr, st);
  return cs.release(s, st);
}

syn_status_t syn_cuda_q4_0_gemv(size_t n, size_t k, const float* a, const uint8_t* b_q4, float* c,
                                void* stream) {
  if (!a || !b_q4 || !c) return SYN_ERR_NULL_PTR;
  if (n == 0 || k == 0) return SYN_OK;
  if (k % 32 != 0) return SYN_ERR_SHAPE_MISMATCH;
  cudaStream_t st = (cudaStream_t)stream;
  CallScratch cs;
  syn_status_t s = cs.init(GEMV_FMT_Q4_0_RAW, 1, n, k, 0, st);
  if (s == SYN_OK) s = launch_q4_0_raw(n, k, a, b_q4, c, cs.part, cs.part_cap, cs.cnt, nullptr, st);
  return cs.release(s, st);
}

syn_status_t syn_cuda_weight_upload(syn_cuda_ctx_t* ctx, syn_qformat_t fmt, const void* host,
                                    size_t n, size_t k, const float* scales_or_null,
                                    syn_cuda_weight_t** out) {
  if (!ctx || !host || !out) return SYN_ERR_NULL_PTR;
  *out = nullptr;
  if (fmt < SYN_QFMT_INT8_KN || fmt > SYN_QFMT_Q6_K) return SYN_ERR_INVALID_ARG;
  if (fmt == SYN_QFMT_INT8_KN && !scales_or_null) return SYN_ERR_NULL_PTR;
  if (n == 0 || k == 0) return SYN_ERR_INVALID_ARG;
  if (k % block_elems(fmt) != 0) return SYN_ERR_SHAPE_MISMATCH;
  DeviceGuard g(ctx->device);
  if (!g.ok) return SYN_ERR_CUDA;

  auto* w = new (std::nothrow) syn_cuda_weight_s();
  if (!w) return SYN_ERR_OUT_OF_MEMORY;
  w->fmt = fmt;
  w->device = ctx->device;
  w->n = n;
  w->k = k;
  w->kp = (fmt == SYN_QFMT_INT8_KN) ? (k + 31) / 32 * 32 : k;
  const size_t src_bytes = n * src_row_bytes(fmt, k);
  w->algo_bytes = src_bytes + (fmt == SYN_QFMT_INT8_KN ? n * 4 : 0);
  w->bytes = layout(w, nullptr);
  cudaError_t e = cudaMalloc(&w->buf, w->bytes);
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "cudaMalloc(weight)");
    delete w;
    return e == cudaErrorMemoryAllocation ? SYN_ERR_OUT_OF_MEMORY : SYN_ERR_CUDA;
  }
  layout(w, static_cast<uint8_t*>(w->buf));

  // raw bytes (and INT8 scales) staged in a temporary device buffer
  void* tmp = nullptr;
  syn_status_t s = SYN_OK;
  cudaStream_t st = ctx->upload_stream;
  const size_t sc_off = align256(src_bytes);
  do {
    e = cudaMalloc(&tmp, sc_off + n * sizeof(float) + 16);
    if (e != cudaSuccess) { s = SYN_ERR_OUT_OF_MEMORY; break; }
    e = cudaMemcpyAsync(tmp, host, src_bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) { s = SYN_ERR_CUDA; break; }
    float* d_sc = nullptr;
    if (fmt == SYN_QFMT_INT8_KN) {
      d_sc = reinterpret_cast<float*>(static_cast<uint8_t*>(tmp) + sc_off);
      e = cudaMemcpyAsync(d_sc, scales_or_null, n * sizeof(float), cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) { s = SYN_ERR_CUDA; break; }
    }
    s = repack_weight(w, static_cast<const uint8_t*>(tmp), 0, d_sc, st);
    if (s != SYN_OK) break;
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { s = SYN_ERR_CUDA; break; }
  } while (0);
  if (e != cudaSuccess) set_last_cuda_error(e, "syn_cuda_weight_upload");
  if (tmp) cudaFree(tmp);
  if (s != SYN_OK) {
    cudaFree(w->buf);
    delete w;
    return s;
  }
  *out = w;
  return SYN_OK;
}

syn_status_t syn_cuda_weight_destroy(syn_cuda_weight_t* w) {
  if (!w) return SYN_ERR_NULL_PTR;
  {
    DeviceGuard g(w->device);
    cudaFree(w->buf);
  }
  delete w;
  return SYN_OK;
}

syn_status_t syn_cuda_weight_bytes(const syn_cuda_weight_t* w, size_t* bytes) {
  if (!w || !bytes) return SYN_ERR_NULL_PTR;
  *bytes = w->bytes;
  return SYN_OK;
}

syn_status_t syn_cuda_weight_dequant(const syn_cuda_weight_t* w, float* host_out) {
  if (!w || !host_out) return SYN_ERR_NULL_PTR;
  DeviceGuard g(w->device);
  if (!g.ok) return SYN_ERR_CUDA;
  float* d = nullptr;
  SYN_CUDA_TRY(cudaMalloc(&d, w->n * w->k * sizeof(float)));
  syn_status_t s = dequant_weight(w, d, nullptr);
  if (s == SYN_OK) {
    cudaError_t e = cudaMemcpy(host_out, d, w->n * w->k * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
      set_last_cuda_error(e, "cudaMemcpy(dequant)");
      s = SYN_ERR_CUDA;
    }
  }
  cudaFree(d);
  return s;
}

syn_status_t syn_cuda_qmatmul(syn_cuda_ctx_t* ctx, const syn_cuda_weight_t* w, const float* x,
                              size_t m, float* y, void* stream) {
  if (!ctx || !w || !x || !y) return SYN_ERR_NULL_PTR;
  if (m == 0) return SYN_OK;
  DeviceGuard g(w->device);
  if (!g.ok) return SYN_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  const int chunked = (w->fmt == SYN_QFMT_INT8_KN && m > 16) ? 1 : 0;
  if (m >= gemm_min_rows(w->fmt, w->n)) {
    syn_status_t s = grow(reinterpret_cast<void**>(&ctx->abuf), &ctx->abuf_bytes,
                          gemm_a_bytes(w->fmt, m, w->kp), st);
    if (s != SYN_OK) return s;
    return launch_qgemm(w, x, w->k, nullptr, nullptr, m, y, w->n, chunked, ctx->abuf, ctx->err,
                        st);
  }
  syn_status_t s = ensure_scratch(ctx, w, m, st);
  if (s != SYN_OK) return s;
  return launch_qgemv(w, x, w->k, nullptr, nullptr, m, y, w->n, chunked, ctx->part,
                      ctx->part_bytes, ctx->cnt, ctx->err, st);
}

syn_status_t syn_cuda_qmatmul_int8_prequant(syn_cuda_ctx_t* ctx, const syn_cuda_weight_t* w,
                                            const int8_t* x_i8, const float* scales_x, size_t m,
                                            float* y, void* stream) {
  if (!ctx || !w || !x_i8 || !scales_x || !y) return SYN_ERR_NULL_PTR;
  if (w->fmt != SYN_QFMT_INT8_KN) return SYN_ERR_INVALID_ARG;
  if (m == 0) return SYN_OK;
  DeviceGuard g(w->device);
  if (!g.ok) return SYN_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  if (m >= gemm_min_rows(w->fmt, w->n)) {
    syn_status_t s = grow(reinterpret_cast<void**>(&ctx->abuf), &ctx->abuf_bytes,
                          gemm_a_bytes(w->fmt, m, w->kp), st);
    if (s != SYN_OK) return s;
    return launch_qgemm(w, nullptr, w->k, x_i8, scales_x, m, y, w->n, m > 16 ? 1 : 0, ctx->abuf,
                        ctx->err, st);
  }
  syn_status_t s = ensure_scratch(ctx, w, m, st);
  if (s != SYN_OK) return s;
  return launch_qgemv(w, nullptr, w->k, x_i8, scales_x, m, y, w->n, m > 16 ? 1 : 0, ctx->part,
                      ctx->part_bytes, ctx->cnt, ctx->err, st);
}

syn_status_t syn_cuda_qmatmul_rmsnorm(syn_cuda_ctx_t* ctx, const syn_cuda_weight_t* w,
                                      const float* residual, const float* delta,
                                      const float* norm_weight, float eps, float* residual_out,
                                      int parallel_sum, float* y, void* stream) {
  if (!ctx || !w || !residual || !norm_weight || !y) return SYN_ERR_NULL_PTR;
  if (residual_out && residual_out == residual) return SYN_ERR_INVALID_ARG;
  DeviceGuard g(w->device);
  if (!g.ok) return SYN_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  syn_status_t s = ensure_scratch(ctx, w, 1, st);
  if (s != SYN_OK) return s;
  GemvNorm nm{residual, delta, norm_weight, eps, residual_out, parallel_sum ? 1 : 0};
  return launch_qgemv_norm(w, nm, y, ctx->part, ctx->part_bytes, ctx->cnt, ctx->err, st);
}

}  // extern "C"
