// runner.cu -- the decoder-only LM runner on the GPU: QuantizedCausalLM
// (quantization/lm/int8.rs:171-709) for INT8 weights and CausalLM
// (models/lm/causal_lm.rs:195-280, models/lm/decoder_layer.rs:590-730) for
// the block formats, with the weights repacked in HBM, the KV cache in HBM
// and each decode step replayed as one CUDA graph.
//
// Per layer (rows = tokens of a prefill, or one per sequence in a decode):
//   add_rmsnorm(resid += down_prev; x = norm(resid))      [layer 0: embedding]
//   qkv  = x * [Wq;Wk;Wv]^T                               (one fused matmul)
//   att  = attention(qkv)            (headwise norm, RoPE, KV append, GQA)
//   o    = att * Wo^T
//   add_rmsnorm(resid += o; x = ffn_norm(resid))
//   gu   = x * [Wgate;Wup]^T                              (one fused matmul)
//   hid  = swiglu(gu)
//   down = hid * Wdown^T
// then add_rmsnorm with the final norm, the LM head and argmax. Fusing the
// weights along N is exact: every output column is computed independently.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

#include "internal.cuh"

namespace {

// ---------------------------------------------------------------------------
// Minimal JSON reader for the model config: flattens objects into
// "section.key" -> scalar text.
// ---------------------------------------------------------------------------
struct Json {
  const char* s;
  size_t i = 0;
  bool ok = true;
  std::map<std::string, std::string> flat;
  explicit Json(const char* t) : s(t) {}
  void ws() {
    while (s[i] == ' ' || s[i] == '\n' || s[i] == '\t' || s[i] == '\r') i++;
  }
  std::string str() {
    std::string out;
    if (s[i] != '"') {
      ok = false;
      return out;
    }
    i++;
    while (s[i] && s[i] != '"') {
      if (s[i] == '\\' && s[i + 1]) i++;
      out += s[i++];
    }
    if (s[i] != '"') ok = false;
    else i++;
    return out;
  }
  void value(const std::string& path) {
    ws();
    if (s[i] == '{') {
      i++;
      ws();
      if (s[i] == '}') {
        i++;
        return;
      }
      while (ok) {
        ws();
        std::string k = str();
        ws();
        if (s[i] != ':') {
          ok = false;
          return;
        }
        i++;
        value(path.empty() ? k : path + "." + k);
        ws();
        if (s[i] == ',') {
          i++;
          continue;
        }
        if (s[i] == '}') {
          i++;
          return;
        }
        ok = false;
      }
    } else if (s[i] == '[') {
      int depth = 0;  // arrays are not needed by the config: skip them
      do {
        if (s[i] == '[') depth++;
        else if (s[i] == ']') depth--;
        else if (!s[i]) {
          ok = false;
          return;
        }
        i++;
      } while (depth > 0);
    } else if (s[i] == '"') {
      flat[path] = str();
    } else {
      size_t j = i;
      while (s[i] && s[i] != ',' && s[i] != '}' && s[i] != ']' && s[i] != ' ' && s[i] != '\n' &&
             s[i] != '\r' && s[i] != '\t')
        i++;
      if (i == j) ok = false;
      flat[path] = std::string(s + j, i - j);
    }
  }
  bool parse() {
    value("");
    return ok;
  }
  bool num(const char* key, double* out) const {
    auto it = flat.find(key);
    if (it == flat.end()) return false;
    char* end = nullptr;
    *out = strtod(it->second.c_str(), &end);
    return end && *end == 0;
  }
  std::string text(const char* key) const {
    auto it = flat.find(key);
    return it == flat.end() ? std::string() : it->second;
  }
};

struct HostLinear {
  int fmt = -1;
  size_t n = 0, k = 0;
  std::vector<uint8_t> data;
  std::vector<float> scales;
};

size_t row_bytes(int fmt, size_t k) {
  switch (fmt) {
    case SYN_QFMT_Q4_0: return k / 32 * 18;
    case SYN_QFMT_Q8_0: return k / 32 * 34;
    case SYN_QFMT_Q4_K: return k / 256 * 144;
    case SYN_QFMT_Q6_K: return k / 256 * 210;
  }
  return 0;
}

size_t weight_bytes(int fmt, size_t n, size_t k) {
  return fmt == SYN_QFMT_INT8_KN ? n * k : n * row_bytes(fmt, k);
}

// Concatenates linears along N (output rows): INT8 [K,N] column blocks, block
// formats row blocks.
bool concat(const std::vector<const HostLinear*>& parts, HostLinear& out) {
  out = HostLinear();
  out.fmt = parts[0]->fmt;
  out.k = parts[0]->k;
  for (auto* p : parts) {
    if (p->fmt != out.fmt || p->k != out.k) return false;
    out.n += p->n;
  }
  out.data.resize(weight_bytes(out.fmt, out.n, out.k));
  if (out.fmt == SYN_QFMT_INT8_KN) {
    size_t c0 = 0;
    for (auto* p : parts) {
      for (size_t kk = 0; kk < out.k; kk++)
        memcpy(out.data.data() + kk * out.n + c0, p->data.data() + kk * p->n, p->n);
      out.scales.insert(out.scales.end(), p->scales.begin(), p->scales.end());
      c0 += p->n;
    }
  } else {
    size_t off = 0;
    for (auto* p : parts) {
      memcpy(out.data.data() + off, p->data.data(), p->data.size());
      off += p->data.size();
    }
  }
  return true;
}

// Gate and up (same format, k and n) interleaved by blocks of 16 output rows:
// rows 32j..32j+15 = gate rows 16j.., rows 32j+16.. = up rows 16j.., so a
// 32-row group of the GEMV holds 16 matching (gate, up) pairs and its
// epilogue can apply SwiGLU.
bool concat_il16(const HostLinear& g, const HostLinear& u, HostLinear& out) {
  if (g.fmt != u.fmt || g.k != u.k || g.n != u.n || g.n % 16) return false;
  out = HostLinear();
  out.fmt = g.fmt;
  out.k = g.k;
  out.n = 2 * g.n;
  out.data.resize(weight_bytes(out.fmt, out.n, out.k));
  if (out.fmt == SYN_QFMT_INT8_KN) {  // [K, N] columns, and per-column scales
    for (size_t kk = 0; kk < out.k; kk++)
      for (size_t j = 0; j < g.n; j += 16) {
        memcpy(out.data.data() + kk * out.n + 2 * j, g.data.data() + kk * g.n + j, 16);
        memcpy(out.data.data() + kk * out.n + 2 * j + 16, u.data.data() + kk * u.n + j, 16);
      }
    for (size_t j = 0; j < g.n; j += 16) {
      out.scales.insert(out.scales.end(), g.scales.begin() + j, g.scales.begin() + j + 16);
      out.scales.insert(out.scales.end(), u.scales.begin() + j, u.scales.begin() + j + 16);
    }
  } else {  // whole rows
    const size_t rb = row_bytes(out.fmt, out.k);
    for (size_t j = 0; j < g.n; j += 16) {
      memcpy(out.data.data() + 2 * j * rb, g.data.data() + j * rb, 16 * rb);
      memcpy(out.data.data() + (2 * j + 16) * rb, u.data.data() + j * rb, 16 * rb);
    }
  }
  return true;
}

struct LayerDev {
  float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  syn_cuda_weight_t *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
};

}  // namespace

struct syn_cuda_model_s {
  syn_cuda_ctx_t* ctx = nullptr;
  int device = 0;
  // config
  size_t h = 0, L = 0, V = 0, Hq = 0, Hkv = 0, hd = 0, ff = 0, window = 0;
  size_t qd = 0, kvd = 0, qkv_n = 0;
  // this rank's shard (tensor parallelism; equal to the full sizes at tp = 1)
  int tp = 1, tp_rank = 0;
  size_t hq_l = 0, hkv_l = 0, ff_l = 0, v_l = 0, qd_l = 0, kvd_l = 0;
  float eps = 1e-6f;
  double rope_base = 10000.0;
  size_t max_seq = 0, max_batch = 0, max_rows = 0;
  bool int8 = false;
  bool finalized = false;
  std::string cache_dir;  // repacked-weight cache (empty: none)
  int cache_hits = 0;     // weights read from the cache by finalize
  // speculative decoding: logits and tokens of up to 16 span rows
  float* span_logits = nullptr;
  int32_t* span_tok = nullptr;
  int32_t* span_tok_h = nullptr;
  // continuous batching: paged KV (kv_page = 0: contiguous) and the row ->
  // sequence map of slot-indexed decode steps
  size_t kv_page = 0, kv_pages = 0;
  int* slots_d = nullptr;
  int* slots_h = nullptr;
  // staged host weights
  std::map<std::string, HostLinear> lin;
  std::map<std::string, std::vector<float>> ten;
  // device
  cudaStream_t st = nullptr;
  std::vector<LayerDev> layers;
  syn_cuda_weight_t* lm_head = nullptr;
  float *embed = nullptr, *final_norm = nullptr, *cos_t = nullptr, *sin_t = nullptr;
  syn_cuda_kvcache_t* cache = nullptr;
  std::vector<void*> allocs;
  int32_t* ids = nullptr;
  int32_t* tok = nullptr;
  int32_t* hist = nullptr;  // [max_batch][max_seq + 1] generated token per position
  void* am_scratch = nullptr;
  float* logits_l = nullptr;  // this rank's vocabulary slice of the logits (tp > 1)
  // tp > 1, greedy steps without host logits: each row's argmax state over
  // this rank's slice (16 B) and all ranks' states ([tp][max_batch])
  int32_t* am_pair_l = nullptr;
  int32_t* am_pair_g = nullptr;
  float* resid2 = nullptr;     // second residual buffer (fused single-row steps)
  bool no_fuse = false;        // SYN_RUNNER_FUSE=0 keeps the norms as separate kernels
  float *resid = nullptr, *x = nullptr, *qkv = nullptr, *att = nullptr, *o = nullptr,
        *gu = nullptr, *hid = nullptr, *dn = nullptr, *logits = nullptr;
  // pinned host staging
  int32_t* ids_h = nullptr;
  int32_t* tok_h = nullptr;
  float* logits_h = nullptr;
  int32_t* err_h = nullptr;
  // decode graphs per (batch, with logits)
  std::map<std::pair<size_t, int>, cudaGraphExec_t> graphs;
  std::map<std::pair<size_t, int>, int> eager_runs;
  std::map<size_t, cudaGraphExec_t> chain_graphs;  // chained decode step per batch
};

namespace {

using namespace syn;

syn_status_t dev_alloc(syn_cuda_model_s* m, void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "cudaMalloc(model)");
    return SYN_ERR_OUT_OF_MEMORY;
  }
  m->allocs.push_back(*p);
  return SYN_OK;
}

}  // namespace

namespace syn {
syn_cuda_ctx_s* model_context(const syn_cuda_model_s* m) { return m->ctx; }
}  // namespace syn

namespace {

template <typename T>
syn_status_t dev_alloc_t(syn_cuda_model_s* m, T** p, size_t count) {
  return dev_alloc(m, reinterpret_cast<void**>(p), count * sizeof(T));
}

syn_status_t upload_tensor(syn_cuda_model_s* m, const std::string& name, size_t numel, float** out,
                           bool optional) {
  auto it = m->ten.find(name);
  if (it == m->ten.end()) {
    if (optional) {
      *out = nullptr;
      return SYN_OK;
    }
    set_last_cuda_error(cudaErrorInvalidValue, ("missing tensor " + name).c_str());
    return SYN_ERR_INVALID_ARG;
  }
  if (it->second.size() != numel) return SYN_ERR_SHAPE_MISMATCH;
  syn_status_t s = dev_alloc_t(m, out, numel);
  if (s) return s;
  SYN_CUDA_TRY(cudaMemcpy(*out, it->second.data(), numel * 4, cudaMemcpyHostToDevice));
  return SYN_OK;
}

syn_status_t upload_linear(syn_cuda_model_s* m, const HostLinear& hl, syn_cuda_weight_t** out) {
  const float* sc = hl.fmt == SYN_QFMT_INT8_KN ? hl.scales.data() : nullptr;
  if (!m->cache_dir.empty()) {
    int hit = 0;
    syn_status_t s = syn_cuda_weight_upload_cached(m->ctx, (syn_qformat_t)hl.fmt, hl.data.data(),
                                                   hl.n, hl.k, sc, m->cache_dir.c_str(), out, &hit);
    m->cache_hits += hit;
    return s;
  }
  return syn_cuda_weight_upload(m->ctx, (syn_qformat_t)hl.fmt, hl.data.data(), hl.n, hl.k, sc,
                                out);
}

const HostLinear* find_lin(syn_cuda_model_s* m, const std::string& name, size_t n, size_t k) {
  auto it = m->lin.find(name);
  if (it == m->lin.end() || it->second.n != n || it->second.k != k) return nullptr;
  return &it->second;
}

std::string lname(size_t i, const char* rest) {
  return "model.layers." + std::to_string(i) + "." + rest;
}

// y[rows, w.n] = x[rows, w.k] * W^T through the public matmul entry point
syn_status_t mm(syn_cuda_model_s* m, const syn_cuda_weight_t* w, const float* x, size_t rows,
                float* y) {
  return syn_cuda_qmatmul(m->ctx, w, x, rows, y, m->st);
}

// One forward over `rows` rows. Prefill: rows tokens of sequence `seq`.
// Decode: rows sequences [0, rows), one token each.
// chained: the step's input tokens are the previous step's outputs (m->tok),
// and nothing is copied to the host.
// span: rows are consecutive new positions of sequence `seq` (speculative
// drafting and verification): attention through launch_attn_span_args,
// logits and greedy tokens for every row into the span buffers, no cache
// length advanced. nlayers < L runs only the first nlayers layers (the
// reference's layer-skipping draft, pipeline.rs:281-330).
syn_status_t forward(syn_cuda_model_s* m, size_t rows, bool prefill, size_t seq, bool want_logits,
                     bool chained = false, size_t nlayers = 0, bool span = false,
                     const int* slots = nullptr) {
  cudaStream_t st = m->st;
  syn_status_t s;
  const size_t h = m->h;
  const int variant = m->int8 ? 0 : 1;
  AttnArgs a{};
  a.ld = m->qkv_n;
  a.n_heads = m->hq_l;
  a.eps = m->eps;
  a.cos_t = m->cos_t;
  a.sin_t = m->sin_t;
  a.window = m->window;
  a.cache = m->cache;
  a.ldo = m->qd_l;
  // block-format models carry a 1e-3 tolerance: parallel-order attention;
  // INT8 models keep the reference's reduction order (bit-exact tokens)
  a.flash = m->int8 ? 0 : 1;
  a.slots = slots;  // decode rows -> sequences (continuous batching)
  const bool tp = m->tp > 1;
  // One row (decode at batch 1): each RMSNorm runs in the prologue of the
  // matmul it feeds, with the residual stream ping-ponging between two
  // buffers (a kernel never rewrites the residual it reads).
  const bool fuse = rows == 1 && !m->no_fuse;
  float* cur = m->resid;
  auto other = [&](float* r) { return r == m->resid ? m->resid2 : m->resid; };
  const size_t L = nlayers ? std::min(nlayers, m->L) : m->L;
  for (size_t li = 0; li < L; li++) {
    LayerDev& ly = m->layers[li];
    if (fuse && li > 0) {
      float* nxt = other(cur);
      GemvNorm nm{cur, m->dn, ly.attn_norm, m->eps, nxt, a.flash};
      if ((s = ensure_scratch(m->ctx, ly.qkv, 1, st))) return s;
      s = launch_qgemv_norm(ly.qkv, nm, m->qkv, m->ctx->part, m->ctx->part_bytes,
                            m->ctx->cnt, m->ctx->err, st);
      if (s) return s;
      cur = nxt;
    } else {
      if (li == 0)
        s = launch_add_rmsnorm(nullptr, 0, nullptr, 0, chained ? m->tok : m->ids, m->embed, m->V,
                               cur, h, ly.attn_norm, rows, h, m->eps, m->x, h, st, a.flash);
      else
        s = launch_add_rmsnorm(cur, h, m->dn, h, nullptr, nullptr, 0, cur, h, ly.attn_norm, rows,
                               h, m->eps, m->x, h, st, a.flash);
      if (s) return s;
      if ((s = mm(m, ly.qkv, m->x, rows, m->qkv))) return s;
    }
    a.q = m->qkv;
    a.k = m->qkv + m->qd_l;
    a.v = m->qkv + m->qd_l + m->kvd_l;
    a.qn = ly.q_norm;
    a.kn = ly.k_norm;
    a.layer = li;
    a.out = m->att;
    s = span      ? launch_attn_span_args(a, seq, rows, m->ctx->err, st)
        : prefill ? launch_attn_prefill_args(a, seq, rows, m->ctx->err, st)
                  : launch_attn_decode_args(a, rows, m->ctx->err, st);
    if (s) return s;
    if ((s = mm(m, ly.o, m->att, rows, m->o))) return s;
    if (tp && (s = tp_allreduce_sum(m->ctx, m->o, rows * h, st))) return s;  // row-parallel O
    if (fuse) {
      float* nxt = other(cur);
      // SwiGLU in the GEMV's epilogue: hid comes out directly
      GemvNorm nm{cur, m->o, ly.ffn_norm, m->eps, nxt, a.flash, m->hid, (int)m->ff_l, variant};
      if ((s = ensure_scratch(m->ctx, ly.gu, 1, st))) return s;
      s = launch_qgemv_norm(ly.gu, nm, m->gu, m->ctx->part, m->ctx->part_bytes,
                            m->ctx->cnt, m->ctx->err, st);
      if (s) return s;
      cur = nxt;
    } else {
      s = launch_add_rmsnorm(cur, h, m->o, h, nullptr, nullptr, 0, cur, h, ly.ffn_norm, rows, h,
                             m->eps, m->x, h, st, a.flash);
      if (s) return s;
      if ((s = mm(m, ly.gu, m->x, rows, m->gu))) return s;
      // gate/up rows are interleaved by 16 (see concat_il16)
      s = launch_swiglu(m->gu, m->gu + 16, 2 * m->ff_l, rows, m->ff_l, variant, m->hid, m->ff_l,
                        st, 1);
      if (s) return s;
    }
    if ((s = mm(m, ly.down, m->hid, rows, m->dn))) return s;
    if (tp && (s = tp_allreduce_sum(m->ctx, m->dn, rows * h, st))) return s;  // row-parallel down
  }
  // final norm and LM head: prefill keeps only the last token (int8.rs:619-627)
  const size_t r0 = prefill ? rows - 1 : 0, nr = prefill ? 1 : rows;
  float* logits_dst = span ? m->span_logits : tp ? m->logits_l : m->logits;
  if (fuse) {
    GemvNorm nm{cur, m->dn, m->final_norm, m->eps, nullptr, a.flash};
    if ((s = ensure_scratch(m->ctx, m->lm_head, 1, st))) return s;
    s = launch_qgemv_norm(m->lm_head, nm, logits_dst, m->ctx->part, m->ctx->part_bytes,
                            m->ctx->cnt, m->ctx->err, st);
    if (s) return s;
  } else {
    s = launch_add_rmsnorm(cur + r0 * h, h, m->dn + r0 * h, h, nullptr, nullptr, 0,
                           cur + r0 * h, h, m->final_norm, nr, h, m->eps, m->x, h, st, a.flash);
    if (s) return s;
    if ((s = mm(m, m->lm_head, m->x, nr, logits_dst))) return s;
  }
  if (span) {  // every row's greedy token; lengths untouched
    s = launch_argmax(m->span_logits, m->V, nr, m->V, m->span_tok, nullptr, 0, (int)m->max_seq,
                      nullptr, 0, m->am_scratch, st);
    if (s) return s;
    SYN_CUDA_TRY(cudaMemcpyAsync(m->span_tok_h, m->span_tok, nr * sizeof(int32_t),
                                 cudaMemcpyDeviceToHost, st));
    SYN_CUDA_TRY(cudaMemcpyAsync(m->err_h, m->ctx->err, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    if (want_logits)
      SYN_CUDA_TRY(cudaMemcpyAsync(m->logits_h, m->span_logits, nr * m->V * sizeof(float),
                                   cudaMemcpyDeviceToHost, st));
    return SYN_OK;
  }
  // vocab-parallel LM head. A greedy step without host logits gathers each
  // rank's argmax state over its slice (16 bytes per row), not the logits;
  // SYN_TP_ARGMAX_PAIRS=0 gathers the logits always.
  static const bool pairs_on = [] {
    const char* e = getenv("SYN_TP_ARGMAX_PAIRS");
    return !(e && e[0] == '0');
  }();
  const bool tp_pairs = tp && pairs_on && !want_logits && !slots;
  if (tp && !tp_pairs) {  // gather each row's logits in rank (= vocab) order
    for (size_t b = 0; b < nr; b++)
      if ((s = tp_allgather(m->ctx, m->logits_l + b * m->v_l, m->logits + b * m->V, m->v_l, st)))
        return s;
  }
  if (tp_pairs) {
    s = launch_argmax_slice(m->logits_l, m->v_l, nr, m->v_l, (int)(m->tp_rank * m->v_l),
                            m->am_pair_l, m->am_scratch, st);
    if (s) return s;
    s = tp_allgather(m->ctx, reinterpret_cast<const float*>(m->am_pair_l),
                     reinterpret_cast<float*>(m->am_pair_g), 4 * nr, st);
    if (s) return s;
    s = launch_argmax_pairs(m->am_pair_g, m->tp, nr, m->tok + (prefill ? seq : 0),
                            m->cache->d_len + (prefill ? seq : 0), prefill ? (int)rows : 1,
                            (int)m->max_seq, m->hist + (prefill ? seq : 0) * (m->max_seq + 1),
                            (int)(m->max_seq + 1), st);
    if (s) return s;
    if (chained) return SYN_OK;
    SYN_CUDA_TRY(cudaMemcpyAsync(m->tok_h, m->tok + (prefill ? seq : 0), nr * sizeof(int32_t),
                                 cudaMemcpyDeviceToHost, st));
    SYN_CUDA_TRY(cudaMemcpyAsync(m->err_h, m->ctx->err, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    return SYN_OK;
  }
  if (slots) {  // row b's token into tok[b]; each mapped sequence advances by one
    s = launch_argmax(m->logits, m->V, nr, m->V, m->tok, nullptr, 0, (int)m->max_seq, nullptr, 0,
                      m->am_scratch, st);
    if (s) return s;
    if ((s = launch_kv_advance_slots(m->cache, slots, nr, st))) return s;
    SYN_CUDA_TRY(cudaMemcpyAsync(m->tok_h, m->tok, nr * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    SYN_CUDA_TRY(cudaMemcpyAsync(m->err_h, m->ctx->err, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    if (want_logits)
      SYN_CUDA_TRY(cudaMemcpyAsync(m->logits_h, m->logits, nr * m->V * sizeof(float),
                                   cudaMemcpyDeviceToHost, st));
    return SYN_OK;
  }
  // the generated token of sequence b lands in tok[b] (prefill: tok[seq])
  s = launch_argmax(m->logits, m->V, nr, m->V, m->tok + (prefill ? seq : 0),
                    m->cache->d_len + (prefill ? seq : 0), prefill ? (int)rows : 1,
                    (int)m->max_seq, m->hist + (prefill ? seq : 0) * (m->max_seq + 1),
                    (int)(m->max_seq + 1), m->am_scratch, st);
  if (s) return s;
  if (chained) return SYN_OK;
  SYN_CUDA_TRY(cudaMemcpyAsync(m->tok_h, m->tok + (prefill ? seq : 0), nr * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, st));
  SYN_CUDA_TRY(cudaMemcpyAsync(m->err_h, m->ctx->err, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  if (want_logits)
    SYN_CUDA_TRY(cudaMemcpyAsync(m->logits_h, m->logits, nr * m->V * sizeof(float),
                                 cudaMemcpyDeviceToHost, st));
  return SYN_OK;
}

syn_status_t finish(syn_cuda_model_s* m, size_t nr, int32_t* out_tokens, float* logits_host) {
  SYN_CUDA_TRY(cudaStreamSynchronize(m->st));
  if (*m->err_h != SYN_OK) {
    const syn_status_t e = *m->err_h;
    int32_t zero = 0;
    cudaMemcpy(m->ctx->err, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    *m->err_h = 0;
    return e;
  }
  if (out_tokens) memcpy(out_tokens, m->tok_h, nr * sizeof(int32_t));
  if (logits_host) memcpy(logits_host, m->logits_h, nr * m->V * sizeof(float));
  return SYN_OK;
}

syn_status_t cuda_status_r(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return SYN_OK;
  set_last_cuda_error(e, where);
  return SYN_ERR_CUDA;
}

bool use_graphs() {
  const char* e = getenv("SYN_RUNNER_GRAPH");
  return !(e && e[0] == '0');
}

}  // namespace

extern "C" {

syn_status_t syn_cuda_model_create(syn_cuda_ctx_t* ctx, const char* config_json, size_t max_seq,
                                   size_t max_batch, syn_cuda_model_t** out) {
  if (!ctx || !config_json || !out) return SYN_ERR_NULL_PTR;
  *out = nullptr;
  if (!max_seq || !max_batch) return SYN_ERR_INVALID_ARG;
  Json j(config_json);
  if (!j.parse()) return SYN_ERR_INVALID_ARG;
  double v;
  auto* m = new (std::nothrow) syn_cuda_model_s();
  if (!m) return SYN_ERR_OUT_OF_MEMORY;
  m->ctx = ctx;
  m->device = ctx->device;
  bool ok = true;
  ok &= j.num("architecture.hidden_size", &v), m->h = (size_t)v;
  ok &= j.num("architecture.num_layers", &v), m->L = (size_t)v;
  ok &= j.num("architecture.vocab_size", &v), m->V = (size_t)v;
  ok &= j.num("attention.num_heads", &v), m->Hq = (size_t)v;
  m->Hkv = j.num("attention.num_kv_heads", &v) ? (size_t)v : m->Hq;
  m->hd = j.num("attention.head_dim", &v) ? (size_t)v : (m->Hq ? m->h / m->Hq : 0);
  ok &= j.num("ffn.intermediate_size", &v), m->ff = (size_t)v;
  m->eps = j.num("norm.eps", &v) ? (float)v : 1e-6f;  // NormVariant::eps() as f32
  m->rope_base = j.num("position.base", &v) ? v : 10000.0;
  if (j.text("attention.type") == "SlidingWindow" && j.num("attention.window_size", &v))
    m->window = (size_t)v;
  if (!ok || !m->h || !m->L || !m->V || !m->Hq || !m->Hkv || !m->hd || !m->ff ||
      m->Hq % m->Hkv || j.text("ffn.type") != "SwiGLU" ||
      (!j.text("norm.type").empty() && j.text("norm.type") != "RMSNorm")) {
    delete m;
    return SYN_ERR_INVALID_ARG;
  }
  m->qd = m->Hq * m->hd;
  m->kvd = m->Hkv * m->hd;
  m->qkv_n = m->qd + 2 * m->kvd;
  m->max_seq = max_seq;
  m->max_batch = max_batch;
  m->max_rows = std::max(max_seq, max_batch);
  *out = m;
  return SYN_OK;
}

syn_status_t syn_cuda_model_set_cache_dir(syn_cuda_model_t* m, const char* dir) {
  if (!m) return SYN_ERR_NULL_PTR;
  if (m->finalized) return SYN_ERR_INVALID_ARG;
  m->cache_dir = dir ? dir : "";
  return SYN_OK;
}

syn_status_t syn_cuda_model_cache_hits(const syn_cuda_model_t* m, int* hits) {
  if (!m || !hits) return SYN_ERR_NULL_PTR;
  *hits = m->cache_hits;
  return SYN_OK;
}

syn_status_t syn_cuda_model_set_tensor(syn_cuda_model_t* m, const char* name, const float* host,
                                       size_t numel) {
  if (!m || !name || (!host && numel)) return SYN_ERR_NULL_PTR;
  if (m->finalized) return SYN_ERR_INVALID_ARG;
  m->ten[name].assign(host, host + numel);
  return SYN_OK;
}

syn_status_t syn_cuda_model_set_linear(syn_cuda_model_t* m, const char* name, syn_qformat_t fmt,
                                       const void* host, size_t n, size_t k,
                                       const float* scales_or_null) {
  if (!m || !name || !host) return SYN_ERR_NULL_PTR;
  if (m->finalized) return SYN_ERR_INVALID_ARG;
  if ((int)fmt < 0 || (int)fmt > SYN_QFMT_Q6_K) return SYN_ERR_INVALID_ARG;
  if (fmt == SYN_QFMT_INT8_KN && !scales_or_null) return SYN_ERR_NULL_PTR;
  if (fmt != SYN_QFMT_INT8_KN && k % ((fmt == SYN_QFMT_Q4_K || fmt == SYN_QFMT_Q6_K) ? 256 : 32))
    return SYN_ERR_SHAPE_MISMATCH;
  HostLinear& hl = m->lin[name];
  hl.fmt = fmt;
  hl.n = n;
  hl.k = k;
  const uint8_t* p = static_cast<const uint8_t*>(host);
  hl.data.assign(p, p + weight_bytes(fmt, n, k));
  if (fmt == SYN_QFMT_INT8_KN) hl.scales.assign(scales_or_null, scales_or_null + n);
  return SYN_OK;
}

syn_status_t syn_cuda_model_finalize(syn_cuda_model_t* m) {
  if (!m) return SYN_ERR_NULL_PTR;
  if (m->finalized) return SYN_OK;
  DeviceGuard g(m->device);
  if (!g.ok) return SYN_ERR_CUDA;
  syn_status_t s;
  const size_t h = m->h;
  SYN_CUDA_TRY(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking));
  if ((s = upload_tensor(m, "model.embed_tokens.weight", m->V * h, &m->embed, false))) return s;
  if ((s = upload_tensor(m, "model.norm.weight", h, &m->final_norm, false))) return s;
  // tensor parallelism: this rank's shard of every linear
  m->tp = m->ctx->tp_world > 1 ? m->ctx->tp_world : 1;
  m->tp_rank = m->tp > 1 ? m->ctx->tp_rank : 0;
  const size_t W = (size_t)m->tp;
  if (m->Hq % W || m->Hkv % W || m->ff % W || m->V % W) return SYN_ERR_SHAPE_MISMATCH;
  m->hq_l = m->Hq / W;
  m->hkv_l = m->Hkv / W;
  m->ff_l = m->ff / W;
  m->v_l = m->V / W;
  m->qd_l = m->hq_l * m->hd;
  m->kvd_l = m->hkv_l * m->hd;
  m->qkv_n = m->qd_l + 2 * m->kvd_l;
  auto shard = [&](const HostLinear& full, int axis, HostLinear& out) -> syn_status_t {
    if (W == 1) {
      out = full;
      return SYN_OK;
    }
    if (full.fmt == SYN_QFMT_INT8_KN) return SYN_ERR_UNSUPPORTED;  // W8A8 row-parallel
    out = HostLinear();
    out.fmt = full.fmt;
    out.data.resize(full.data.size() / W);
    return syn_cuda_tp_shard_linear((syn_qformat_t)full.fmt, full.data.data(), full.n, full.k,
                                    nullptr, axis, m->tp_rank, (int)W, out.data.data(), nullptr,
                                    &out.n, &out.k);
  };
  m->layers.resize(m->L);
  for (size_t i = 0; i < m->L; i++) {
    LayerDev& ly = m->layers[i];
    if ((s = upload_tensor(m, lname(i, "input_layernorm.weight"), h, &ly.attn_norm, false))) return s;
    if ((s = upload_tensor(m, lname(i, "post_attention_layernorm.weight"), h, &ly.ffn_norm, false)))
      return s;
    if ((s = upload_tensor(m, lname(i, "self_attn.q_norm.weight"), m->hd, &ly.q_norm, true))) return s;
    if ((s = upload_tensor(m, lname(i, "self_attn.k_norm.weight"), m->hd, &ly.k_norm, true))) return s;
    const HostLinear* q = find_lin(m, lname(i, "self_attn.q_proj.weight"), m->qd, h);
    const HostLinear* k = find_lin(m, lname(i, "self_attn.k_proj.weight"), m->kvd, h);
    const HostLinear* v = find_lin(m, lname(i, "self_attn.v_proj.weight"), m->kvd, h);
    const HostLinear* o = find_lin(m, lname(i, "self_attn.o_proj.weight"), h, m->qd);
    const HostLinear* ga = find_lin(m, lname(i, "mlp.gate_proj.weight"), m->ff, h);
    const HostLinear* up = find_lin(m, lname(i, "mlp.up_proj.weight"), m->ff, h);
    const HostLinear* dn = find_lin(m, lname(i, "mlp.down_proj.weight"), h, m->ff);
    if (!q || !k || !v || !o || !ga || !up || !dn) return SYN_ERR_SHAPE_MISMATCH;
    if (i == 0) m->int8 = q->fmt == SYN_QFMT_INT8_KN;
    HostLinear qs, ks, vs, os, gs, us, ds, cat;
    if ((s = shard(*q, 0, qs)) || (s = shard(*k, 0, ks)) || (s = shard(*v, 0, vs)) ||
        (s = shard(*o, 1, os)) || (s = shard(*ga, 0, gs)) || (s = shard(*up, 0, us)) ||
        (s = shard(*dn, 1, ds)))
      return s;
    if (!concat({&qs, &ks, &vs}, cat)) return SYN_ERR_INVALID_ARG;
    if ((s = upload_linear(m, cat, &ly.qkv))) return s;
    if (!concat_il16(gs, us, cat)) return SYN_ERR_INVALID_ARG;
    if ((s = upload_linear(m, cat, &ly.gu))) return s;
    if ((s = upload_linear(m, os, &ly.o))) return s;
    if ((s = upload_linear(m, ds, &ly.down))) return s;
  }
  const HostLinear* lm = find_lin(m, "lm_head.weight", m->V, h);
  if (!lm) return SYN_ERR_SHAPE_MISMATCH;
  {
    HostLinear ls;
    if ((s = shard(*lm, 0, ls))) return s;
    if ((s = upload_linear(m, ls, &m->lm_head))) return s;
  }
  m->lin.clear();
  m->ten.clear();
  // RoPE tables for the cache's positions
  std::vector<float> c(m->max_seq * (m->hd / 2)), sn(c.size());
  if ((s = syn_cuda_rope_tables(m->rope_base, m->max_seq, m->hd, c.data(), sn.data()))) return s;
  if ((s = dev_alloc_t(m, &m->cos_t, c.size()))) return s;
  if ((s = dev_alloc_t(m, &m->sin_t, c.size()))) return s;
  SYN_CUDA_TRY(cudaMemcpy(m->cos_t, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
  SYN_CUDA_TRY(cudaMemcpy(m->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  if ((s = syn_cuda_kvcache_create_paged(m->ctx, m->max_seq, m->hkv_l, m->hd, m->L, m->max_batch,
                                         m->kv_page, m->kv_pages, &m->cache)))
    return s;
  if ((s = dev_alloc_t(m, &m->slots_d, m->max_batch))) return s;
  SYN_CUDA_TRY(cudaMallocHost(&m->slots_h, m->max_batch * sizeof(int)));
  const size_t R = m->max_rows;
  if ((s = dev_alloc_t(m, &m->ids, R))) return s;
  if ((s = dev_alloc_t(m, &m->tok, m->max_batch))) return s;
  if ((s = dev_alloc_t(m, &m->hist, m->max_batch * (m->max_seq + 1)))) return s;
  if ((s = dev_alloc_t(m, &m->resid, R * h))) return s;
  if ((s = dev_alloc_t(m, &m->resid2, R * h))) return s;
  if ((s = dev_alloc_t(m, &m->x, R * h))) return s;
  {
    const char* e = getenv("SYN_RUNNER_FUSE");
    m->no_fuse = e && e[0] == '0';
  }
  if ((s = dev_alloc_t(m, &m->qkv, R * m->qkv_n))) return s;
  if ((s = dev_alloc_t(m, &m->att, R * m->qd_l))) return s;
  if ((s = dev_alloc_t(m, &m->o, R * h))) return s;
  if ((s = dev_alloc_t(m, &m->gu, R * 2 * m->ff_l))) return s;
  if ((s = dev_alloc_t(m, &m->hid, R * m->ff_l))) return s;
  if (m->tp > 1 && (s = dev_alloc_t(m, &m->logits_l, m->max_batch * m->v_l))) return s;
  if (m->tp > 1 && (s = dev_alloc_t(m, &m->am_pair_l, m->max_batch * 4))) return s;
  if (m->tp > 1 &&
      (s = dev_alloc_t(m, &m->am_pair_g, (size_t)m->tp * m->max_batch * 4)))
    return s;
  if ((s = dev_alloc_t(m, &m->dn, R * h))) return s;
  if ((s = dev_alloc_t(m, &m->logits, m->max_batch * m->V))) return s;
  if ((s = dev_alloc_t(m, &m->span_logits, 16 * m->V))) return s;
  if ((s = dev_alloc_t(m, &m->span_tok, 16))) return s;
  {
    const size_t ab = argmax_scratch_bytes(std::max<size_t>(m->max_batch, 16), m->V);
    if ((s = dev_alloc(m, &m->am_scratch, ab))) return s;
    SYN_CUDA_TRY(cudaMemset(m->am_scratch, 0, ab));
  }
  SYN_CUDA_TRY(cudaMallocHost(&m->ids_h, R * sizeof(int32_t)));
  SYN_CUDA_TRY(cudaMallocHost(&m->tok_h, m->max_batch * sizeof(int32_t)));
  SYN_CUDA_TRY(cudaMallocHost(&m->logits_h, std::max<size_t>(m->max_batch, 16) * m->V * sizeof(float)));
  SYN_CUDA_TRY(cudaMallocHost(&m->span_tok_h, 16 * sizeof(int32_t)));
  SYN_CUDA_TRY(cudaMallocHost(&m->err_h, sizeof(int32_t)));
  *m->err_h = 0;
  SYN_CUDA_TRY(cudaDeviceSynchronize());
  m->finalized = true;
  return SYN_OK;
}

syn_status_t syn_cuda_prefill(syn_cuda_model_t* m, size_t seq, const int32_t* tokens, size_t n,
                              float* logits_host, int32_t* next_token) {
  if (!m || !tokens || !next_token) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  if (seq >= m->max_batch || n == 0) return SYN_ERR_INVALID_ARG;
  if (m->cache->len[seq] != 0) return SYN_ERR_INVALID_ARG;  // prefill starts a sequence
  if (n > m->max_seq) return SYN_ERR_INVALID_ARG;           // CacheFull
  DeviceGuard g(m->device);
  memcpy(m->ids_h, tokens, n * sizeof(int32_t));
  SYN_CUDA_TRY(cudaMemcpyAsync(m->ids, m->ids_h, n * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
  syn_status_t s = forward(m, n, true, seq, logits_host != nullptr);
  if (s) return s;
  s = finish(m, 1, next_token, logits_host);
  if (s == SYN_OK) m->cache->len[seq] += n;
  return s;
}

syn_status_t syn_cuda_decode_step(syn_cuda_model_t* m, size_t batch, const int32_t* last_tokens,
                                  int32_t* out_tokens, float* logits_host) {
  if (!m || !last_tokens || !out_tokens) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  if (batch == 0 || batch > m->max_batch) return SYN_ERR_INVALID_ARG;
  for (size_t b = 0; b < batch; b++)
    if (m->cache->len[b] + 1 > m->max_seq) return SYN_ERR_INVALID_ARG;  // CacheFull
  DeviceGuard g(m->device);
  syn_status_t rs;
  for (size_t b = 0; b < batch; b++)  // pages for the new positions, outside any graph
    if ((rs = kv_reserve(m->cache, b, m->cache->len[b] + 1, m->st))) return rs;
  memcpy(m->ids_h, last_tokens, batch * sizeof(int32_t));
  const auto key = std::make_pair(batch, logits_host ? 1 : 0);
  syn_status_t s = SYN_OK;
  auto it = m->graphs.find(key);
  if (it != m->graphs.end()) {
    SYN_CUDA_TRY(cudaGraphLaunch(it->second, m->st));
  } else if (!use_graphs() || m->eager_runs[key] == 0) {
    // first step of this shape runs eagerly (it sizes the scratch buffers)
    SYN_CUDA_TRY(cudaMemcpyAsync(m->ids, m->ids_h, batch * sizeof(int32_t),
                                 cudaMemcpyHostToDevice, m->st));
    s = forward(m, batch, false, 0, logits_host != nullptr);
    if (s) return s;
    m->eager_runs[key]++;
  } else {
    cudaGraph_t graph = nullptr;
    SYN_CUDA_TRY(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    cudaError_t ce = cudaMemcpyAsync(m->ids, m->ids_h, batch * sizeof(int32_t),
                                     cudaMemcpyHostToDevice, m->st);
    s = ce == cudaSuccess ? forward(m, batch, false, 0, logits_host != nullptr) : SYN_ERR_CUDA;
    cudaError_t e = cudaStreamEndCapture(m->st, &graph);
    if (s == SYN_OK && e != cudaSuccess) {
      set_last_cuda_error(e, "cudaStreamEndCapture");
      s = SYN_ERR_CUDA;
    }
    if (s) {
      if (graph) cudaGraphDestroy(graph);
      return s;
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
      set_last_cuda_error(e, "cudaGraphInstantiate");
      return SYN_ERR_CUDA;
    }
    m->graphs[key] = exec;
    SYN_CUDA_TRY(cudaGraphLaunch(exec, m->st));
  }
  s = finish(m, batch, out_tokens, logits_host);
  if (s == SYN_OK)
    for (size_t b = 0; b < batch; b++) m->cache->len[b] += 1;
  return s;
}

syn_status_t syn_cuda_generate(syn_cuda_model_t* m, size_t batch, size_t n_steps,
                               int32_t* out_tokens) {
  if (!m || !out_tokens) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  if (batch == 0 || batch > m->max_batch) return SYN_ERR_INVALID_ARG;
  if (n_steps == 0) return SYN_OK;
  for (size_t b = 0; b < batch; b++)
    if (m->cache->len[b] == 0 || m->cache->len[b] + n_steps > m->max_seq)
      return SYN_ERR_INVALID_ARG;  // not started, or CacheFull
  DeviceGuard g(m->device);
  for (size_t b = 0; b < batch; b++) {  // pages for every position the steps will write
    syn_status_t rs = kv_reserve(m->cache, b, m->cache->len[b] + n_steps, m->st);
    if (rs) return rs;
  }
  std::vector<size_t> len0(m->cache->len, m->cache->len + batch);
  syn_status_t s = SYN_OK;
  size_t done = 0;
  auto it = m->chain_graphs.find(batch);
  if (it == m->chain_graphs.end()) {
    // one eager step sizes the scratch buffers, then the step is captured
    if ((s = forward(m, batch, false, 0, false, true))) return s;
    done = 1;
    if (use_graphs()) {
      cudaGraph_t graph = nullptr;
      SYN_CUDA_TRY(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
      s = forward(m, batch, false, 0, false, true);
      cudaError_t e = cudaStreamEndCapture(m->st, &graph);
      if (s == SYN_OK && e != cudaSuccess) s = cuda_status_r(e, "cudaStreamEndCapture");
      if (s) {
        if (graph) cudaGraphDestroy(graph);
        return s;
      }
      cudaGraphExec_t exec = nullptr;
      e = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) return cuda_status_r(e, "cudaGraphInstantiate");
      it = m->chain_graphs.emplace(batch, exec).first;
    }
  }
  for (; done < n_steps; done++) {
    if (it != m->chain_graphs.end()) {
      SYN_CUDA_TRY(cudaGraphLaunch(it->second, m->st));
    } else if ((s = forward(m, batch, false, 0, false, true))) {
      return s;
    }
  }
  SYN_CUDA_TRY(cudaMemcpyAsync(m->err_h, m->ctx->err, sizeof(int32_t), cudaMemcpyDeviceToHost,
                               m->st));
  SYN_CUDA_TRY(cudaStreamSynchronize(m->st));
  if (*m->err_h != SYN_OK) {
    const syn_status_t e = *m->err_h;
    int32_t zero = 0;
    cudaMemcpy(m->ctx->err, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    *m->err_h = 0;
    return e;
  }
  for (size_t b = 0; b < batch; b++) {
    // tokens generated by these steps occupy positions len0+1 .. len0+n_steps
    SYN_CUDA_TRY(cudaMemcpy(out_tokens + b * n_steps, m->hist + b * (m->max_seq + 1) + len0[b] + 1,
                            n_steps * sizeof(int32_t), cudaMemcpyDeviceToHost));
    m->cache->len[b] += n_steps;
  }
  return SYN_OK;
}

syn_status_t syn_cuda_model_set_kv_paging(syn_cuda_model_t* m, size_t page, size_t n_pages) {
  if (!m) return SYN_ERR_NULL_PTR;
  if (m->finalized || (page && !n_pages)) return SYN_ERR_INVALID_ARG;
  m->kv_page = page;
  m->kv_pages = page ? n_pages : 0;
  return SYN_OK;
}

syn_status_t syn_cuda_model_kv_pages_free(const syn_cuda_model_t* m, size_t* n) {
  if (!m || !n) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  return syn_cuda_kvcache_pages_free(m->cache, n);
}

syn_status_t syn_cuda_decode_step_slots(syn_cuda_model_t* m, size_t n, const int32_t* slots,
                                        const int32_t* last_tokens, int32_t* out_tokens,
                                        float* logits_host) {
  if (!m || !slots || !last_tokens || !out_tokens) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  if (n == 0 || n > m->max_batch) return SYN_ERR_INVALID_ARG;
  for (size_t i = 0; i < n; i++) {
    if (slots[i] < 0 || (size_t)slots[i] >= m->max_batch) return SYN_ERR_INVALID_ARG;
    for (size_t j = 0; j < i; j++)
      if (slots[j] == slots[i]) return SYN_ERR_INVALID_ARG;  // one row per sequence
    const size_t len = m->cache->len[slots[i]];
    if (len == 0 || len + 1 > m->max_seq) return SYN_ERR_INVALID_ARG;  // not started / full
  }
  DeviceGuard g(m->device);
  syn_status_t s;
  for (size_t i = 0; i < n; i++)
    if ((s = kv_reserve(m->cache, slots[i], m->cache->len[slots[i]] + 1, m->st))) return s;
  memcpy(m->ids_h, last_tokens, n * sizeof(int32_t));
  memcpy(m->slots_h, slots, n * sizeof(int32_t));
  SYN_CUDA_TRY(cudaMemcpyAsync(m->ids, m->ids_h, n * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
  SYN_CUDA_TRY(cudaMemcpyAsync(m->slots_d, m->slots_h, n * sizeof(int32_t), cudaMemcpyHostToDevice,
                               m->st));
  s = forward(m, n, false, 0, logits_host != nullptr, false, 0, false, m->slots_d);
  if (s) return s;
  s = finish(m, n, out_tokens, logits_host);
  if (s == SYN_OK)
    for (size_t i = 0; i < n; i++) m->cache->len[slots[i]] += 1;
  return s;
}

syn_status_t syn_cuda_decode_span(syn_cuda_model_t* m, size_t seq, const int32_t* tokens,
                                  size_t n, size_t n_layers, int32_t* out_tokens,
                                  float* logits_host) {
  if (!m || !tokens || !out_tokens) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  if (seq >= m->max_batch || n == 0 || n > 16 || n > m->max_rows) return SYN_ERR_INVALID_ARG;
  if (m->tp > 1) return SYN_ERR_UNSUPPORTED;
  if (m->cache->len[seq] == 0 || m->cache->len[seq] + n > m->max_seq)
    return SYN_ERR_INVALID_ARG;  // not started, or CacheFull
  DeviceGuard g(m->device);
  memcpy(m->ids_h, tokens, n * sizeof(int32_t));
  SYN_CUDA_TRY(cudaMemcpyAsync(m->ids, m->ids_h, n * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
  syn_status_t s = forward(m, n, false, seq, logits_host != nullptr, false, n_layers, true);
  if (s) return s;
  SYN_CUDA_TRY(cudaStreamSynchronize(m->st));
  if (*m->err_h != SYN_OK) {
    const syn_status_t e = *m->err_h;
    int32_t zero = 0;
    cudaMemcpy(m->ctx->err, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    *m->err_h = 0;
    return e;
  }
  memcpy(out_tokens, m->span_tok_h, n * sizeof(int32_t));
  if (logits_host) memcpy(logits_host, m->logits_h, n * m->V * sizeof(float));
  return SYN_OK;
}

// Self-speculative greedy decoding with KV rollback on the device
// (generation/pipeline.rs:281-396): k draft tokens from the first
// draft_layers layers (each one span step, its K/V kept for those layers
// only), the cache rolled back, then one span step of the full model over
// [last, d_0 .. d_{k-1}]. Unlike the reference, which accepts every draft
// token, each d_i is checked against the full model's greedy token g_i at
// its position: the accepted prefix, then g at the first mismatch (or the
// bonus g_k) are emitted, and the cache is truncated to the accepted
// positions. The output is therefore the plain greedy sequence.
syn_status_t syn_cuda_generate_speculative(syn_cuda_model_t* m, size_t seq, int32_t last_token,
                                           size_t n_steps, size_t k, size_t draft_layers,
                                           int32_t* out_tokens, size_t* drafted,
                                           size_t* accepted) {
  if (!m || !out_tokens) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  if (k == 0 || k > 15 || draft_layers == 0 || draft_layers > m->L || seq >= m->max_batch)
    return SYN_ERR_INVALID_ARG;
  DeviceGuard g(m->device);
  size_t done = 0, nd = 0, na = 0;
  int32_t last = last_token;
  syn_status_t s = SYN_OK;
  auto set_len = [&](size_t len) -> syn_status_t {
    m->cache->len[seq] = len;
    return launch_kv_set(m->cache, seq, (int)len, 0, m->st);
  };
  while (done < n_steps) {
    const size_t L0 = m->cache->len[seq];
    const size_t kk = std::min(k, m->max_seq - std::min(m->max_seq, L0 + 1));
    if (kk == 0) return SYN_ERR_INVALID_ARG;  // CacheFull
    int32_t draft[16], verify[16], greedy[16];
    int32_t t = last;
    for (size_t j = 0; j < kk; j++) {
      if ((s = syn_cuda_decode_span(m, seq, &t, 1, draft_layers, &draft[j], nullptr))) return s;
      if ((s = set_len(L0 + j + 1))) return s;
      t = draft[j];
    }
    if ((s = set_len(L0))) return s;
    verify[0] = last;
    for (size_t j = 0; j < kk; j++) verify[j + 1] = draft[j];
    if ((s = syn_cuda_decode_span(m, seq, verify, kk + 1, 0, greedy, nullptr))) return s;
    size_t a = 0;
    while (a < kk && draft[a] == greedy[a]) a++;
    nd += kk;
    na += a;
    // emitted this round: d_0 .. d_{a-1}, then greedy[a] (within n_steps);
    // the cache keeps `last` and every emitted token but the final one
    size_t e = 0;
    for (; e < a && done < n_steps; e++) out_tokens[done++] = last = draft[e];
    if (done < n_steps) {
      out_tokens[done++] = last = greedy[a];
      e++;
    }
    if ((s = set_len(L0 + e))) return s;
  }
  SYN_CUDA_TRY(cudaStreamSynchronize(m->st));
  if (drafted) *drafted = nd;
  if (accepted) *accepted = na;
  return SYN_OK;
}

syn_status_t syn_cuda_model_seq_len(const syn_cuda_model_t* m, size_t seq, size_t* len) {
  if (!m || !len) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  return syn_cuda_kvcache_len(m->cache, seq, len);
}

syn_status_t syn_cuda_model_reset(syn_cuda_model_t* m, size_t seq) {
  if (!m) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  DeviceGuard g(m->device);
  syn_status_t s = syn_cuda_kvcache_reset(m->cache, seq, m->st);
  if (s) return s;
  SYN_CUDA_TRY(cudaStreamSynchronize(m->st));
  return SYN_OK;
}

syn_status_t syn_cuda_model_truncate(syn_cuda_model_t* m, size_t seq, size_t new_len) {
  if (!m) return SYN_ERR_NULL_PTR;
  if (!m->finalized) return SYN_ERR_INVALID_ARG;
  DeviceGuard g(m->device);
  syn_status_t s = syn_cuda_kvcache_truncate(m->cache, seq, new_len, m->st);
  if (s) return s;
  SYN_CUDA_TRY(cudaStreamSynchronize(m->st));
  return SYN_OK;
}

syn_status_t syn_cuda_model_destroy(syn_cuda_model_t* m) {
  if (!m) return SYN_ERR_NULL_PTR;
  DeviceGuard g(m->device);
  if (m->st) cudaStreamSynchronize(m->st);
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : m->chain_graphs) cudaGraphExecDestroy(kv.second);
  for (auto& ly : m->layers) {
    if (ly.qkv) syn_cuda_weight_destroy(ly.qkv);
    if (ly.o) syn_cuda_weight_destroy(ly.o);
    if (ly.gu) syn_cuda_weight_destroy(ly.gu);
    if (ly.down) syn_cuda_weight_destroy(ly.down);
  }
  if (m->lm_head) syn_cuda_weight_destroy(m->lm_head);
  if (m->cache) syn_cuda_kvcache_destroy(m->cache);
  for (void* p : m->allocs) cudaFree(p);
  if (m->ids_h) cudaFreeHost(m->ids_h);
  if (m->tok_h) cudaFreeHost(m->tok_h);
  if (m->span_tok_h) cudaFreeHost(m->span_tok_h);
  if (m->slots_h) cudaFreeHost(m->slots_h);
  if (m->logits_h) cudaFreeHost(m->logits_h);
  if (m->err_h) cudaFreeHost(m->err_h);
  if (m->st) cudaStreamDestroy(m->st);
  delete m;
  return SYN_OK;
}

}  // extern "C"
