// common.cuh -- shared helpers for the sm_100a quantized-matmul backend.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/synapse_cuda.h"

namespace syn {

// ----------------------------------------------------------------------------
// Error plumbing: every entry point returns a syn_status_t; CUDA errors map to
// SYN_ERR_CUDA and the last CUDA error string is kept per thread.
// ----------------------------------------------------------------------------
void set_last_cuda_error(cudaError_t e, const char* where);

#define SYN_CUDA_TRY(expr)                   \
  do {                                       \
    cudaError_t _e = (expr);                 \
    if (_e != cudaSuccess) {                 \
      ::syn::set_last_cuda_error(_e, #expr); \
      return SYN_ERR_CUDA;                   \
    }                                        \
  } while (0)

#define SYN_LAUNCH_CHECK(where)              \
  do {                                       \
    cudaError_t _e = cudaGetLastError();     \
    if (_e != cudaSuccess) {                 \
      ::syn::set_last_cuda_error(_e, where); \
      return SYN_ERR_CUDA;                   \
    }                                        \
  } while (0)

int num_sms();

// ----------------------------------------------------------------------------
// f16 -> f32. Two conversions exist in the reference and they disagree on
// subnormals:
//  * zig/src/ops/qmatmul.zig:346-371 (used by syn_q4_0_gemv) is exact IEEE;
//  * weight_loading/converter.rs:12-40 (used by every GGUF dequantiser) starts
//    its normalisation counter at 1, which halves each subnormal.
// Both are reproduced bit-exactly.
// ----------------------------------------------------------------------------
__device__ __forceinline__ float f16_exact(uint16_t h) {
  // hardware half -> single conversion: exact for every finite input
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ float f16_loader(uint16_t h) {
  // converter.rs subnormal quirk: exponent field 0 -> half the IEEE value
  // (zero stays zero); halving is exact in f32.
  return f16_exact(h) * ((h & 0x7C00u) ? 1.0f : 0.5f);
}

// Exact int -> float for |v| < 2^22 with two ALU/FMA ops (no conversion
// unit): the integer is placed in the mantissa of 1.5 * 2^23, bias removed.
__device__ __forceinline__ float i2f_small(int v) {
  return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

// ----------------------------------------------------------------------------
// 4-way byte dot products (dp4a) with explicit operand signedness.
// ----------------------------------------------------------------------------
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a_signed, uint32_t b_unsigned, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_signed), "r"(b_unsigned), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a_unsigned, uint32_t b_signed, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_unsigned), "r"(b_signed), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// exp as the reference evaluates it for f32 (one double-precision exp,
// rounded once); both the CPU oracle and these kernels use this definition.
__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }

// One SwiGLU element i of a row whose first n4 = n - n % 4 elements are the
// vector part: variant 0 = silu(g) * u with silu = g / (1 + exp(-g))
// (quantization/lm/int8.rs:500-503, ops/activation.rs:30-32); variant 1 =
// swigluFused (zig/src/ops/silu.zig:85-114): g * (1 / (1 + exp(-g))) * u on
// the vector part, (g / (1 + exp(-g))) * u on the tail.
__device__ __forceinline__ float swiglu_elem(float g, float u, int i, int n4, int variant) {
  const float e = __fadd_rn(1.0f, exp_f32(-g));
  if (variant == 1 && i < n4) return __fmul_rn(__fmul_rn(g, __fdiv_rn(1.0f, e)), u);
  return __fmul_rn(__fdiv_rn(g, e), u);
}

// Streaming loads that bypass L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint16_t ld_nc_u16(const void* p) {
  uint16_t r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ----------------------------------------------------------------------------
// Programmatic dependent launch (griddepcontrol). A kernel launched with
// programmatic stream serialisation may start before its predecessor ends;
// griddep_wait() blocks until the predecessor has completed and its memory
// is visible. Launched without the attribute both are no-ops.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----------------------------------------------------------------------------
// mbarrier and 1-D bulk (TMA) copies global -> this CTA's shared memory.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Each try_wait suspends
// the thread for a hardware-defined interval while the phase is pending; after
// 2^22 unsuccessful tries (tens of milliseconds at the least, far beyond any
// copy's latency) it gives up and returns false,
// so that a lost completion is reported (SYN_ERR_TIMEOUT) instead of hanging.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ----------------------------------------------------------------------------
// Thread-block clusters: distributed shared memory and remote mbarrier
// arrivals (plain TMA copies only).
// ----------------------------------------------------------------------------
// Split cluster barrier: every thread arrives once right after set-up, and
// waits (for all non-exited threads of the cluster) only before its first
// access to a peer's shared memory.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
// Address of the same shared variable in cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
}
// Arrival (release at cluster scope) on an mbarrier in another cluster CTA.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Bounded wait (acquire at cluster scope) for a phase that peers complete.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); i++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory by the TMA engine,
// completing on `bar` (transaction bytes). dst/src 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace syn
