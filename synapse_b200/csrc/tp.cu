// tp.cu -- Megatron-style tensor parallelism for 7B-class layers: one
// process per GPU, one NCCL communicator per context, column-parallel
// Q/K/V (by heads) and gate/up (by FFN rows), row-parallel O and down (by K,
// block-aligned) with one sum all-reduce after each, vocab-parallel LM head
// with an all-gather of the logits. The reference has no multi-GPU code; its
// single-GPU arithmetic is what each shard reproduces.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2): a process that
// already loaded NCCL (e.g. through torch.distributed) shares that copy, and
// the library itself keeps no link-time dependency on it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.cuh"

namespace syn {
namespace {

struct Nccl {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const Nccl& nccl() {
  static std::once_flag once;
  static Nccl n;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce &&
           n.all_gather && n.error_string;
  });
  return n;
}

syn_status_t nccl_status(ncclResult_t r, const char* where) {
  if (r == ncclSuccess) return SYN_OK;
  char buf[200];
  snprintf(buf, sizeof(buf), "%s: %s", where, nccl().error_string ? nccl().error_string(r) : "?");
  set_last_cuda_error(cudaErrorUnknown, buf);
  return SYN_ERR_NCCL;
}

size_t blk_elems(int fmt) {
  switch (fmt) {
    case SYN_QFMT_Q4_0:
    case SYN_QFMT_Q8_0: return 32;
    case SYN_QFMT_Q4_K:
    case SYN_QFMT_Q6_K: return 256;
  }
  return 1;
}
size_t blk_bytes(int fmt) {
  switch (fmt) {
    case SYN_QFMT_Q4_0: return 18;
    case SYN_QFMT_Q8_0: return 34;
    case SYN_QFMT_Q4_K: return 144;
    case SYN_QFMT_Q6_K: return 210;
  }
  return 1;
}

}  // namespace

void tp_release(syn_cuda_ctx_s* ctx) {
  if (ctx->nccl && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(ctx->nccl));
  ctx->nccl = nullptr;
  ctx->tp_rank = 0;
  ctx->tp_world = 0;
}

syn_status_t tp_allreduce_sum(syn_cuda_ctx_s* ctx, float* buf, size_t count, cudaStream_t st) {
  if (!ctx->nccl) return SYN_ERR_INVALID_ARG;
  return nccl_status(nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum,
                                       static_cast<ncclComm_t>(ctx->nccl), st),
                     "ncclAllReduce");
}

syn_status_t tp_allgather(syn_cuda_ctx_s* ctx, const float* send, float* recv, size_t count,
                          cudaStream_t st) {
  if (!ctx->nccl) return SYN_ERR_INVALID_ARG;
  return nccl_status(nccl().all_gather(send, recv, count, ncclFloat32,
                                       static_cast<ncclComm_t>(ctx->nccl), st),
                     "ncclAllGather");
}

}  // namespace syn

using namespace syn;

extern "C" {

syn_status_t syn_cuda_tp_unique_id(uint8_t* id_out) {
  if (!id_out) return SYN_ERR_NULL_PTR;
  if (!nccl().ok) return SYN_ERR_UNSUPPORTED;
  ncclUniqueId id;
  syn_status_t s = nccl_status(nccl().get_unique_id(&id), "ncclGetUniqueId");
  if (s == SYN_OK) memcpy(id_out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return s;
}

syn_status_t syn_cuda_tp_init(syn_cuda_ctx_t* ctx, int rank, int world, const uint8_t* id) {
  if (!ctx || !id) return SYN_ERR_NULL_PTR;
  if (world < 1 || rank < 0 || rank >= world) return SYN_ERR_INVALID_ARG;
  if (ctx->nccl) return SYN_ERR_INVALID_ARG;  // already initialised
  if (world == 1) {
    ctx->tp_rank = 0;
    ctx->tp_world = 1;
    return SYN_OK;
  }
  if (!nccl().ok) return SYN_ERR_UNSUPPORTED;
  DeviceGuard g(ctx->device);
  if (!g.ok) return SYN_ERR_CUDA;
  ncclUniqueId uid;
  memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t comm = nullptr;
  syn_status_t s = nccl_status(nccl().comm_init_rank(&comm, world, uid, rank), "ncclCommInitRank");
  if (s) return s;
  ctx->nccl = comm;
  ctx->tp_rank = rank;
  ctx->tp_world = world;
  return SYN_OK;
}

syn_status_t syn_cuda_tp_allreduce_sum(syn_cuda_ctx_t* ctx, float* buf, size_t count,
                                       void* stream) {
  if (!ctx || !buf) return SYN_ERR_NULL_PTR;
  if (!count) return SYN_OK;
  DeviceGuard g(ctx->device);
  return tp_allreduce_sum(ctx, buf, count, (cudaStream_t)stream);
}

syn_status_t syn_cuda_tp_shard_linear(syn_qformat_t fmt, const void* host, size_t n, size_t k,
                                      const float* scales, int axis, int rank, int world,
                                      void* out, float* out_scales, size_t* n_out,
                                      size_t* k_out) {
  if (!host || !out || !n_out || !k_out) return SYN_ERR_NULL_PTR;
  if (world < 1 || rank < 0 || rank >= world || (axis != 0 && axis != 1))
    return SYN_ERR_INVALID_ARG;
  const bool i8 = fmt == SYN_QFMT_INT8_KN;
  if (i8 && !scales) return SYN_ERR_NULL_PTR;
  const size_t be = blk_elems(fmt), bb = blk_bytes(fmt);
  if (!i8 && k % be) return SYN_ERR_SHAPE_MISMATCH;
  const uint8_t* src = static_cast<const uint8_t*>(host);
  uint8_t* dst = static_cast<uint8_t*>(out);
  if (axis == 0) {  // output rows (column-parallel)
    if (n % world) return SYN_ERR_SHAPE_MISMATCH;
    const size_t nl = n / world, r0 = rank * nl;
    if (i8) {  // [K, N]: a column block of every K row
      for (size_t kk = 0; kk < k; kk++) memcpy(dst + kk * nl, src + kk * n + r0, nl);
      if (out_scales) memcpy(out_scales, scales + r0, nl * sizeof(float));
    } else {
      const size_t rb = k / be * bb;
      memcpy(dst, src + r0 * rb, nl * rb);
    }
    *n_out = nl;
    *k_out = k;
  } else {  // input columns (row-parallel), whole blocks
    if (k % world) return SYN_ERR_SHAPE_MISMATCH;
    const size_t kl = k / world, k0 = rank * kl;
    if (!i8 && kl % be) return SYN_ERR_SHAPE_MISMATCH;
    if (i8) {  // [K, N]: a block of K rows
      memcpy(dst, src + k0 * n, kl * n);
      if (out_scales) memcpy(out_scales, scales, n * sizeof(float));
    } else {
      const size_t rb = k / be * bb, rbl = kl / be * bb, off = k0 / be * bb;
      for (size_t r = 0; r < n; r++) memcpy(dst + r * rbl, src + r * rb + off, rbl);
    }
    *n_out = n;
    *k_out = kl;
  }
  return SYN_OK;
}

}  // extern "C"
