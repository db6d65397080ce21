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

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

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

// ---------------------------------------------------------------------------
// One-shot all-reduce over peer memory (plain NVLink P2P stores and loads).
// Every rank holds one buffer, mapped into every other rank with
// CUDA IPC: two data slots of [world][PEER_CAP] floats (double-buffered by
// call parity) and [world][PEER_CTAS] arrival flags. A call with epoch e:
//   1. each CTA stores its chunk of the local partial into slot e&1, row
//      `rank`, of every rank's buffer (its own included), fences at system
//      scope, and raises flag [rank][cta] = e+1 on every rank;
//   2. waits (bounded) until its flags from all ranks reach e+1;
//   3. sums the world rows of its chunk in rank order -- the same order, so
//      the same bits, on every rank -- into the caller's buffer.
// The last CTA advances the device epoch, so CUDA-graph replays stay in
// step. A rank can only reuse slot e&1 at epoch e+2, after every rank has
// raised its e+1 flags, i.e. finished reading epoch e.
// ---------------------------------------------------------------------------
constexpr size_t PEER_CAP = 1u << 18;  // floats per rank row (1 MiB); larger -> NCCL
constexpr int PEER_CTAS = 32;
constexpr int PEER_THREADS = 256;
constexpr int PEER_MAX_WORLD = 8;

struct PeerState {
  int world = 0, rank = 0;
  uint8_t* local = nullptr;                  // this rank's buffer (cudaMalloc)
  void* mapped[PEER_MAX_WORLD] = {nullptr};  // opened peer buffers (nullptr for self)
  float** d_bufs = nullptr;                  // device array: every rank's buffer base
  int* d_sync = nullptr;                     // device: epoch, done counter
};

size_t peer_buf_bytes(int world) {
  return 2 * (size_t)world * PEER_CAP * sizeof(float) + (size_t)world * PEER_CTAS * sizeof(int);
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// gather != nullptr: all-gather instead -- step 3 copies the world rows
// into gather[r * n4 * 4 ..] in rank order, and x is only read.
__global__ void __launch_bounds__(PEER_THREADS) k_peer_allreduce(float* x, int n4, int world,
                                                                 int rank, float* const* bufs,
                                                                 int* sync, int* err,
                                                                 float* gather) {
  griddep_wait();  // x comes from the kernel before; the epoch from the call before
  const int cta = blockIdx.x, nct = gridDim.x, tid = threadIdx.x;
  const int e = *reinterpret_cast<volatile int*>(sync);
  const int slot = e & 1;
  const int per = (n4 + nct - 1) / nct, c0 = cta * per, c1 = min(n4, c0 + per);
  const size_t row4 = PEER_CAP / 4;
  const size_t flag_off = 2 * (size_t)world * PEER_CAP * sizeof(float);
  float4* xv = reinterpret_cast<float4*>(x);
  // 1. push this rank's chunk to every rank
  for (int i = c0 + tid; i < c1; i += PEER_THREADS) {
    const float4 v = xv[i];
    for (int r = 0; r < world; r++)
      reinterpret_cast<float4*>(bufs[r])[((size_t)slot * world + rank) * row4 + i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (tid < world) {
    int* f = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bufs[tid]) + flag_off);
    st_release_sys(f + rank * PEER_CTAS + cta, e + 1);
  }
  // 2. wait (bounded) for every rank's chunk
  __shared__ int ok;
  if (tid == 0) ok = 1;
  __syncthreads();
  if (tid < world) {
    const int* f = reinterpret_cast<const int*>(reinterpret_cast<uint8_t*>(bufs[rank]) + flag_off);
    bool got = false;
    for (int it = 0; it < (1 << 24) && !got; it++) {
      got = ld_acquire_sys(f + tid * PEER_CTAS + cta) >= e + 1;
      if (!got && it > 64) __nanosleep(64);
    }
    if (!got) {
      ok = 0;
      if (err) atomicExch(err, SYN_ERR_TIMEOUT);
    }
  }
  __syncthreads();
  // 3. sum in rank order (or gather)
  if (ok && gather) {
    const float4* mine = reinterpret_cast<const float4*>(bufs[rank]) + (size_t)slot * world * row4;
    float4* g = reinterpret_cast<float4*>(gather);
    for (int r = 0; r < world; r++)
      for (int i = c0 + tid; i < c1; i += PEER_THREADS)
        g[(size_t)r * n4 + i] = __ldcv(mine + (size_t)r * row4 + i);
  } else if (ok) {
    const float4* mine = reinterpret_cast<const float4*>(bufs[rank]) + (size_t)slot * world * row4;
    for (int i = c0 + tid; i < c1; i += PEER_THREADS) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < world; r++) {
        const float4 v = __ldcv(mine + (size_t)r * row4 + i);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      xv[i] = s;
    }
  }
  griddep_launch();
  // the last CTA advances the epoch for the next call
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(sync + 1, 1) == nct - 1) {
      sync[1] = 0;
      __threadfence();
      atomicAdd(sync, 1);
    }
  }
}

void peer_release(syn_cuda_ctx_s* ctx) {
  auto* ps = static_cast<PeerState*>(ctx->tp_peer);
  if (!ps) return;
  for (int r = 0; r < ps->world; r++)
    if (ps->mapped[r]) cudaIpcCloseMemHandle(ps->mapped[r]);
  if (ps->local) cudaFree(ps->local);
  if (ps->d_bufs) cudaFree(ps->d_bufs);
  if (ps->d_sync) cudaFree(ps->d_sync);
  delete ps;
  ctx->tp_peer = nullptr;
}

// Sets up the peer buffers (collective over the communicator). Failure
// leaves ctx->tp_peer null and the NCCL path in use.
syn_status_t peer_init(syn_cuda_ctx_s* ctx) {
  if (ctx->tp_world < 2 || ctx->tp_world > PEER_MAX_WORLD) return SYN_OK;
  // Opt-in (SYN_TP_PEER_ALLREDUCE=1): on two B200s the Mistral-7B-shape
  // decode ran at 395 tok/s with it against 421 tok/s with NCCL's.
  const char* env = getenv("SYN_TP_PEER_ALLREDUCE");
  if (!(env && env[0] == '1')) return SYN_OK;
  auto* ps = new (std::nothrow) PeerState();
  if (!ps) return SYN_ERR_OUT_OF_MEMORY;
  ps->world = ctx->tp_world;
  ps->rank = ctx->tp_rank;
  ctx->tp_peer = ps;
  const int W = ps->world;
  cudaStream_t st = ctx->upload_stream;
  cudaIpcMemHandle_t* all = nullptr;
  void* d_h = nullptr;
  syn_status_t s = SYN_OK;
  auto fail = [&](cudaError_t e, const char* where) {
    set_last_cuda_error(e, where);
    s = SYN_ERR_CUDA;
  };
  do {
    cudaError_t e = cudaMalloc(&ps->local, peer_buf_bytes(W));
    if (e != cudaSuccess) { fail(e, "peer buffer"); break; }
    if ((e = cudaMemset(ps->local, 0, peer_buf_bytes(W))) != cudaSuccess) { fail(e, "peer buffer"); break; }
    if ((e = cudaMalloc(&ps->d_sync, 2 * sizeof(int))) != cudaSuccess) { fail(e, "peer sync"); break; }
    if ((e = cudaMemset(ps->d_sync, 0, 2 * sizeof(int))) != cudaSuccess) { fail(e, "peer sync"); break; }
    cudaIpcMemHandle_t mine;
    if ((e = cudaIpcGetMemHandle(&mine, ps->local)) != cudaSuccess) { fail(e, "cudaIpcGetMemHandle"); break; }
    if ((e = cudaMalloc(&d_h, (size_t)W * sizeof(mine))) != cudaSuccess) { fail(e, "ipc exchange"); break; }
    uint8_t* dh = static_cast<uint8_t*>(d_h);
    if ((e = cudaMemcpy(dh + (size_t)ps->rank * sizeof(mine), &mine, sizeof(mine),
                        cudaMemcpyHostToDevice)) != cudaSuccess) { fail(e, "ipc exchange"); break; }
    s = nccl_status(nccl().all_gather(dh + (size_t)ps->rank * sizeof(mine), dh, sizeof(mine),
                                      ncclUint8, static_cast<ncclComm_t>(ctx->nccl), st),
                    "ncclAllGather(ipc handles)");
    if (s) break;
    all = new cudaIpcMemHandle_t[W];
    if ((e = cudaMemcpyAsync(all, dh, (size_t)W * sizeof(mine), cudaMemcpyDeviceToHost, st)) !=
            cudaSuccess ||
        (e = cudaStreamSynchronize(st)) != cudaSuccess) { fail(e, "ipc exchange"); break; }
    float* bases[PEER_MAX_WORLD];
    for (int r = 0; r < W && s == SYN_OK; r++) {
      if (r == ps->rank) {
        bases[r] = reinterpret_cast<float*>(ps->local);
        continue;
      }
      void* p = nullptr;
      if ((e = cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) {
        fail(e, "cudaIpcOpenMemHandle");
        break;
      }
      ps->mapped[r] = p;
      bases[r] = static_cast<float*>(p);
    }
    if (s) break;
    if ((e = cudaMalloc(&ps->d_bufs, W * sizeof(float*))) != cudaSuccess ||
        (e = cudaMemcpy(ps->d_bufs, bases, W * sizeof(float*), cudaMemcpyHostToDevice)) !=
            cudaSuccess) { fail(e, "peer table"); break; }
  } while (0);
  delete[] all;
  if (d_h) cudaFree(d_h);
  if (s != SYN_OK) peer_release(ctx);  // fall back to NCCL
  cudaGetLastError();
  return SYN_OK;
}

}  // namespace

void tp_release(syn_cuda_ctx_s* ctx) {
  peer_release(ctx);
  if (ctx->nccl && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(ctx->nccl));
  ctx->nccl = nullptr;
  ctx->tp_rank = 0;
  ctx->tp_world = 0;
}

syn_status_t tp_allreduce_sum(syn_cuda_ctx_s* ctx, float* buf, size_t count, cudaStream_t st) {
  if (!ctx->nccl) return SYN_ERR_INVALID_ARG;
  auto* ps = static_cast<PeerState*>(ctx->tp_peer);
  if (ps && count <= PEER_CAP && count % 4 == 0 && (reinterpret_cast<uintptr_t>(buf) & 15) == 0) {
    const int n4 = (int)(count / 4);
    const int ctas = std::max(1, std::min(PEER_CTAS, (n4 + PEER_THREADS - 1) / PEER_THREADS));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(PEER_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_peer_allreduce, buf, n4, ps->world, ps->rank,
                                       (float* const*)ps->d_bufs, ps->d_sync, ctx->err,
                                       (float*)nullptr);
    if (e != cudaSuccess) {
      set_last_cuda_error(e, "k_peer_allreduce");
      return SYN_ERR_CUDA;
    }
    return SYN_OK;
  }
  return nccl_status(nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum,
                                       static_cast<ncclComm_t>(ctx->nccl), st),
                     "ncclAllReduce");
}

syn_status_t tp_allgather(syn_cuda_ctx_s* ctx, const float* send, float* recv, size_t count,
                          cudaStream_t st) {
  if (!ctx->nccl) return SYN_ERR_INVALID_ARG;
  auto* ps = static_cast<PeerState*>(ctx->tp_peer);
  if (ps && count <= PEER_CAP && count % 4 == 0 && (reinterpret_cast<uintptr_t>(send) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(recv) & 15) == 0) {
    const int n4 = (int)(count / 4);
    const int ctas = std::max(1, std::min(PEER_CTAS, (n4 + PEER_THREADS - 1) / PEER_THREADS));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(PEER_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_peer_allreduce, const_cast<float*>(send), n4,
                                       ps->world, ps->rank, (float* const*)ps->d_bufs,
                                       ps->d_sync, ctx->err, recv);
    if (e != cudaSuccess) {
      set_last_cuda_error(e, "k_peer_allreduce(gather)");
      return SYN_ERR_CUDA;
    }
    return SYN_OK;
  }
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
  return peer_init(ctx);
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
