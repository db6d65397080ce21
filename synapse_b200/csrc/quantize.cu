// quantize.cu -- per-row INT8 quantisation kernels.
//
// k_quantize_rows: bit-exact restatement of quantizePerChannelInt8
// (zig/src/ops/quantize.zig:12-47): max_abs over the row; a zero row gets
// scale 1.0 and all-zero codes; else scale = max_abs / 127,
// q = clamp(round(x * (127 / max_abs)), -127, 127), round half away from zero.
// Division and multiply are IEEE round-to-nearest (__fdiv_rn / __fmul_rn),
// as in the Zig f32 code.
//
// k_quantize_weights: load-time weight quantisation (reference:
// MinMaxCalibration::compute_scales, quantization/primitives/calibration.rs:11-24,
// and QuantizedLinear::from_f32_with_scales + transpose_i8,
// quantization/primitives/int8_linear.rs:21-70): per output row
// s = max|w| / 127 (1.0 for a zero row), q = clamp(round(w * (1/s)), -128, 127),
// written in the reference's GEMM layout [K, N].
// k_quantize_weights_half: the same from f16 / bf16 weights (safetensors
// --quantize loads), converted as the reference's loader converts them.
#include "internal.cuh"

namespace syn {
namespace {

constexpr int QT = 256;

__device__ __forceinline__ float block_max_abs(const float* row, long long cols) {
  __shared__ float red[QT / 32];
  float amax = 0.0f;
  for (long long i = threadIdx.x; i < cols; i += QT) amax = fmaxf(amax, fabsf(row[i]));
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < QT / 32; w++) amax = fmaxf(amax, red[w]);
  return amax;
}

__global__ void __launch_bounds__(QT) k_quantize_rows(const float* __restrict__ x, long long cols,
                                                      int8_t* __restrict__ out,
                                                      float* __restrict__ scales) {
  const long long row = blockIdx.x;
  const float* xr = x + row * cols;
  int8_t* orow = out + row * cols;
  const float amax = block_max_abs(xr, cols);
  if (amax == 0.0f) {
    for (long long i = threadIdx.x; i < cols; i += QT) orow[i] = 0;
    if (threadIdx.x == 0) scales[row] = 1.0f;
    return;
  }
  const float inv = __fdiv_rn(127.0f, amax);
  for (long long i = threadIdx.x; i < cols; i += QT) {
    float r = roundf(__fmul_rn(xr[i], inv));
    r = fminf(127.0f, fmaxf(-127.0f, r));
    orow[i] = (int8_t)(int)r;
  }
  if (threadIdx.x == 0) scales[row] = __fdiv_rn(amax, 127.0f);
}

__global__ void __launch_bounds__(QT) k_quantize_weights(const float* __restrict__ w, long long n,
                                                         long long k, int8_t* __restrict__ out_kn,
                                                         float* __restrict__ scales) {
  const long long ch = blockIdx.x;
  const float* row = w + ch * k;
  const float amax = block_max_abs(row, k);
  const float s = (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
  const float inv_s = __fdiv_rn(1.0f, s);
  for (long long j = threadIdx.x; j < k; j += QT) {
    float r = roundf(__fmul_rn(row[j], inv_s));
    r = fminf(127.0f, fmaxf(-128.0f, r));
    out_kn[j * n + ch] = (int8_t)(int)r;
  }
  if (threadIdx.x == 0) scales[ch] = s;
}

// f16 / bf16 bits -> f32 as the safetensors loader converts them
// (weight_loading/converter.rs:12-48; f16 subnormals come out at half their
// value there, which f16_loader reproduces).
template <int DT>
__device__ __forceinline__ float half_bits_to_f32(uint16_t b) {
  if constexpr (DT == SYN_DTYPE_BF16) return __uint_as_float((uint32_t)b << 16);
  return f16_loader(b);
}

// k_quantize_weights on f16 / bf16 input: the row is converted to f32 by the
// loader's rule first, so the result equals quantize_model on the f32
// tensors the reference would have loaded (int8.rs:78-152).
template <int DT>
__global__ void __launch_bounds__(QT) k_quantize_weights_half(const uint16_t* __restrict__ w,
                                                              long long n, long long k,
                                                              int8_t* __restrict__ out_kn,
                                                              float* __restrict__ scales) {
  __shared__ float red[QT / 32];
  const long long ch = blockIdx.x;
  const uint16_t* row = w + ch * k;
  float amax = 0.0f;
  for (long long i = threadIdx.x; i < k; i += QT)
    amax = fmaxf(amax, fabsf(half_bits_to_f32<DT>(row[i])));
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < QT / 32; i++) amax = fmaxf(amax, red[i]);
  const float s = (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
  const float inv_s = __fdiv_rn(1.0f, s);
  for (long long j = threadIdx.x; j < k; j += QT) {
    float r = roundf(__fmul_rn(half_bits_to_f32<DT>(row[j]), inv_s));
    r = fminf(127.0f, fmaxf(-128.0f, r));
    out_kn[j * n + ch] = (int8_t)(int)r;
  }
  if (threadIdx.x == 0) scales[ch] = s;
}

}  // namespace

syn_status_t launch_quantize_weights_half(const uint16_t* w, int dtype, size_t n, size_t k,
                                          int8_t* out_kn, float* scales, cudaStream_t st) {
  if (n > 0x7FFFFFFFull) return SYN_ERR_INVALID_ARG;
  if (dtype == SYN_DTYPE_F16)
    k_quantize_weights_half<SYN_DTYPE_F16><<<(unsigned)n, QT, 0, st>>>(w, (long long)n,
                                                                       (long long)k, out_kn, scales);
  else if (dtype == SYN_DTYPE_BF16)
    k_quantize_weights_half<SYN_DTYPE_BF16><<<(unsigned)n, QT, 0, st>>>(w, (long long)n,
                                                                        (long long)k, out_kn, scales);
  else
    return SYN_ERR_INVALID_ARG;
  SYN_LAUNCH_CHECK("k_quantize_weights_half");
  return SYN_OK;
}

syn_status_t launch_quantize_rows(const float* x, size_t rows, size_t cols, int8_t* out,
                                  float* scales, cudaStream_t st) {
  if (rows > 0x7FFFFFFFull) return SYN_ERR_INVALID_ARG;
  k_quantize_rows<<<(unsigned)rows, QT, 0, st>>>(x, (long long)cols, out, scales);
  SYN_LAUNCH_CHECK("k_quantize_rows");
  return SYN_OK;
}

syn_status_t launch_quantize_weights(const float* w, size_t n, size_t k, int8_t* out_kn,
                                     float* scales, cudaStream_t st) {
  if (n > 0x7FFFFFFFull) return SYN_ERR_INVALID_ARG;
  k_quantize_weights<<<(unsigned)n, QT, 0, st>>>(w, (long long)n, (long long)k, out_kn, scales);
  SYN_LAUNCH_CHECK("k_quantize_weights");
  return SYN_OK;
}

}  // namespace syn
