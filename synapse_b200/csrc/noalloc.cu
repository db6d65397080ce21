// noalloc.cu -- syn_cuda_qmatmul_noalloc: the format-generic GEMV with its
// scratch memory (split-K partial sums and per-row-group arrival counters)
// taken from a fixed, statically allocated device array instead of a
// context buffer or cudaMallocAsync.
//
// It exists for callers that must not allocate device memory on the calling
// path: code running where an allocation could stall or fail unpredictably
// (latency-critical decode loops, processes whose device memory is owned by
// an external pool or budget, plug-in hosts that forbid the CUDA allocator).
// They still pass their own inputs and outputs; only the scratch is fixed.
#include <mutex>

#include "internal.cuh"

namespace syn {
namespace {

// Every GPU that loads the library holds this array until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[SYN_CUDA_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch, looked up once per device (the name of
// the array is only a host-side stand-in in host code).
void* scratch_address(int dev, cudaError_t* err) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  *err = cudaSuccess;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *err = e;
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace
}  // namespace syn

using namespace syn;

extern "C" syn_status_t syn_cuda_qmatmul_noalloc(const syn_cuda_weight_t* w, const float* x,
                                                 size_t m, float* y, void* stream) {
  if (!w || !x || !y) return SYN_ERR_NULL_PTR;
  if (m == 0) return SYN_OK;
  int dev = -1;
  SYN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != w->device) return SYN_ERR_INVALID_ARG;  // the weight's device must be current
  const size_t part_bytes = (gemv_partial_bytes(w->fmt, m, w->n, w->kp) + 255) & ~(size_t)255;
  const size_t cnt_bytes = gemv_counter_bytes(m, w->n);
  if (part_bytes + cnt_bytes > SYN_CUDA_NOALLOC_SCRATCH_BYTES) {
    set_last_cuda_error(cudaErrorMemoryAllocation,
                        "syn_cuda_qmatmul_noalloc: scratch need exceeds "
                        "SYN_CUDA_NOALLOC_SCRATCH_BYTES");
    return SYN_ERR_OUT_OF_MEMORY;
  }
  cudaError_t e;
  uint8_t* base = static_cast<uint8_t*>(scratch_address(dev, &e));
  if (!base) {
    set_last_cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    return SYN_ERR_CUDA;
  }
  cudaStream_t st = (cudaStream_t)stream;
  float* part = reinterpret_cast<float*>(base);
  int* cnt = reinterpret_cast<int*>(base + part_bytes);
  // The array keeps whatever the previous call left; the counters must start
  // at zero.
  SYN_CUDA_TRY(cudaMemsetAsync(cnt, 0, cnt_bytes, st));
  const int chunked = (w->fmt == SYN_QFMT_INT8_KN && m > 16) ? 1 : 0;
  return launch_qgemv(w, x, w->k, nullptr, nullptr, m, y, w->n, chunked, part, part_bytes, cnt, nullptr,
                      st);
}
