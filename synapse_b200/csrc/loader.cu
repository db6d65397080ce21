// loader.cu -- weight files into the runner: GGUF (raw quant blocks handed
// to the repacker, no f32 copy), safetensors (f32 / f16 / bf16, quantised to
// INT8 on the device), and an on-disk cache of repacked weights.
//
// GGUF: the reference parses v2/v3 headers, skips the metadata and reads the
// tensor infos (weight_loading/gguf.rs:71-152, :156-248), then dequantises
// every tensor to f32 (gguf.rs:255-487). Here the same header walk keeps the
// metadata scalars (to build the model config) and the tensor data stays in
// the memory-mapped file: Q4_0 / Q8_0 / Q4_K / Q6_K blocks go to
// syn_cuda_weight_upload as they are. GGUF's llama.cpp tensor names
// (blk.N.attn_q.weight, ...) are mapped onto the runner's Hugging Face names;
// the reference's weight map has no such table (weight_map.rs:37-135).
//
// safetensors: header and dtype handling as parse_safetensors
// (weight_loading/safetensors.rs:176-290); f16 / bf16 element conversion as
// converter.rs:12-48. Linear weights are quantised per output row on the
// device (int8.rs:78-152 with calibration.rs:11-24 and int8_linear.rs:21-70).
//
// Repack cache: a repacked weight is stored as its device bytes plus a
// header, in a file named by a 64-bit hash of the source bytes; a later load
// of the same source reads the file instead of repacking.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

#include "internal.cuh"

// ---------------------------------------------------------------------------
// Memory-mapped file
// ---------------------------------------------------------------------------
namespace {

struct MappedFile {
  int fd = -1;
  const uint8_t* data = nullptr;
  size_t size = 0;
  bool open(const char* path) {
    fd = ::open(path, O_RDONLY);
    if (fd < 0) return false;
    struct stat st;
    if (fstat(fd, &st) != 0) return false;
    size = (size_t)st.st_size;
    if (size == 0) return true;
    void* p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) return false;
    data = static_cast<const uint8_t*>(p);
    return true;
  }
  ~MappedFile() {
    if (data) munmap(const_cast<uint8_t*>(data), size);
    if (fd >= 0) ::close(fd);
  }
};

// Bounds-checked little-endian reader (an error sticks).
struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  Reader(const uint8_t* d, size_t len) : p(d), n(len) {}
  const uint8_t* take(size_t k) {
    if (!ok || k > n - pos) {
      ok = false;
      return nullptr;
    }
    const uint8_t* r = p + pos;
    pos += k;
    return r;
  }
  template <typename T>
  T get() {
    T v{};
    const uint8_t* b = take(sizeof(T));
    if (b) memcpy(&v, b, sizeof(T));
    return v;
  }
  std::string str() {
    const uint64_t len = get<uint64_t>();
    const uint8_t* b = ok && len <= n - pos ? take((size_t)len) : nullptr;
    if (!b) {
      ok = false;
      return std::string();
    }
    return std::string(reinterpret_cast<const char*>(b), (size_t)len);
  }
};

// f16 bits -> f32 with the loader's rule (converter.rs:12-40: subnormals at
// half their value; signed zero, inf and NaN kept).
float f16_loader_host(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      uint32_t ee = 1, mm = m;
      while ((mm & 0x400) == 0) {
        mm <<= 1;
        ee++;
      }
      bits = sign | ((127 - 15 + 1 - ee) << 23) | ((mm & 0x3FF) << 13);
    }
  } else if (e == 31) {
    bits = sign | (0xFFu << 23) | (m << 13);
  } else {
    bits = sign | ((e + 127 - 15) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// 64-bit hash of a byte range (word-wise multiply-rotate; not cryptographic).
uint64_t hash_bytes(const void* data, size_t len, uint64_t h) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  const uint64_t c1 = 0x9E3779B97F4A7C15ull, c2 = 0xC2B2AE3D27D4EB4Full;
  size_t i = 0;
  for (; i + 8 <= len; i += 8) {
    uint64_t v;
    memcpy(&v, p + i, 8);
    h ^= v * c1;
    h = ((h << 31) | (h >> 33)) * c2;
  }
  uint64_t t = 0;
  for (size_t j = 0; i + j < len; j++) t |= (uint64_t)p[i + j] << (8 * j);
  h ^= (t ^ len) * c1;
  h ^= h >> 29;
  h *= c2;
  h ^= h >> 32;
  return h;
}

}  // namespace

// ---------------------------------------------------------------------------
// GGUF
// ---------------------------------------------------------------------------
struct syn_gguf_s {
  MappedFile file;
  uint32_t version = 0;
  size_t alignment = 32;
  size_t data_start = 0;
  std::map<std::string, double> num;       // numeric / bool metadata
  std::map<std::string, std::string> text;  // string metadata
  struct Tensor {
    std::string name;
    uint32_t type;
    std::vector<uint64_t> dims;  // ne0 (contiguous) first
    uint64_t offset;
    size_t nbytes;
  };
  std::vector<Tensor> tensors;
  std::map<std::string, size_t> index;
};

namespace {

enum : uint32_t { GG_F32 = 0, GG_F16 = 1, GG_Q4_0 = 2, GG_Q4_1 = 3, GG_Q8_0 = 8, GG_Q4_K = 12,
                  GG_Q6_K = 14 };

// Bytes of `numel` elements of a GGML type (0 when the type is unknown).
size_t ggml_bytes(uint32_t type, uint64_t numel) {
  switch (type) {
    case GG_F32: return numel * 4;
    case GG_F16: return numel * 2;
    case GG_Q4_0: return numel % 32 ? 0 : numel / 32 * 18;
    case GG_Q4_1: return numel % 32 ? 0 : numel / 32 * 20;
    case GG_Q8_0: return numel % 32 ? 0 : numel / 32 * 34;
    case GG_Q4_K: return numel % 256 ? 0 : numel / 256 * 144;
    case GG_Q6_K: return numel % 256 ? 0 : numel / 256 * 210;
  }
  return 0;
}

int ggml_to_qfmt(uint32_t type) {
  switch (type) {
    case GG_Q4_0: return SYN_QFMT_Q4_0;
    case GG_Q8_0: return SYN_QFMT_Q8_0;
    case GG_Q4_K: return SYN_QFMT_Q4_K;
    case GG_Q6_K: return SYN_QFMT_Q6_K;
  }
  return -1;
}

// One metadata value (gguf.rs skip_metadata_value): scalars are kept.
bool gguf_value(Reader& r, uint32_t type, const std::string& key, syn_gguf_s* g, int depth) {
  switch (type) {
    case 0: g->num[key] = r.get<uint8_t>(); break;
    case 1: g->num[key] = r.get<int8_t>(); break;
    case 2: g->num[key] = r.get<uint16_t>(); break;
    case 3: g->num[key] = r.get<int16_t>(); break;
    case 4: g->num[key] = r.get<uint32_t>(); break;
    case 5: g->num[key] = r.get<int32_t>(); break;
    case 6: g->num[key] = r.get<float>(); break;
    case 7: g->num[key] = r.get<uint8_t>() ? 1.0 : 0.0; break;
    case 8: g->text[key] = r.str(); break;
    case 9: {  // array: element type, count, elements (not kept)
      const uint32_t et = r.get<uint32_t>();
      const uint64_t cnt = r.get<uint64_t>();
      if (depth > 4) return false;
      static const size_t fixed[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
      if (et <= 12 && et != 8 && et != 9) {
        if (cnt > r.n / fixed[et] + 1) return false;
        r.take((size_t)cnt * fixed[et]);
      } else {
        for (uint64_t i = 0; i < cnt && r.ok; i++)
          if (!gguf_value(r, et, std::string(), g, depth + 1)) return false;
      }
      break;
    }
    case 10: g->num[key] = (double)r.get<uint64_t>(); break;
    case 11: g->num[key] = (double)r.get<int64_t>(); break;
    case 12: g->num[key] = r.get<double>(); break;
    default: return false;
  }
  if (key.empty()) {  // array elements are not kept
    g->num.erase(key);
    g->text.erase(key);
  }
  return r.ok;
}

}  // namespace

using namespace syn;

extern "C" {

syn_status_t syn_gguf_open(const char* path, syn_gguf_t** out) {
  if (!path || !out) return SYN_ERR_NULL_PTR;
  *out = nullptr;
  auto* g = new (std::nothrow) syn_gguf_s();
  if (!g) return SYN_ERR_OUT_OF_MEMORY;
  if (!g->file.open(path)) {
    delete g;
    set_last_cuda_error(cudaErrorFileNotFound, "syn_gguf_open: cannot map the file");
    return SYN_ERR_INVALID_ARG;
  }
  Reader r(g->file.data, g->file.size);
  const uint32_t magic = r.get<uint32_t>();
  g->version = r.get<uint32_t>();
  const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
  bool ok = r.ok && magic == 0x46554747u && g->version >= 2 && g->version <= 3 &&
            nt < (1ull << 24) && nkv < (1ull << 24);
  for (uint64_t i = 0; ok && i < nkv; i++) {
    const std::string key = r.str();
    const uint32_t type = r.get<uint32_t>();
    ok = r.ok && !key.empty() && gguf_value(r, type, key, g, 0);
  }
  for (uint64_t i = 0; ok && i < nt; i++) {
    syn_gguf_s::Tensor t;
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    ok = r.ok && nd >= 1 && nd <= 4;
    uint64_t numel = 1;
    for (uint32_t d = 0; ok && d < nd; d++) {
      t.dims.push_back(r.get<uint64_t>());
      numel *= t.dims.back();
    }
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    t.nbytes = ggml_bytes(t.type, numel);
    ok = ok && r.ok;
    if (ok) {
      g->index[t.name] = g->tensors.size();
      g->tensors.push_back(std::move(t));
    }
  }
  // data section: the reference aligns to GGUF's default of 32 bytes; a
  // general.alignment key (written by llama.cpp when it differs) is honoured
  auto al = g->num.find("general.alignment");
  if (al != g->num.end() && al->second >= 1 && al->second <= 4096) g->alignment = (size_t)al->second;
  g->data_start = (r.pos + g->alignment - 1) / g->alignment * g->alignment;
  for (const auto& t : g->tensors)
    if (t.nbytes && (t.offset > g->file.size || g->data_start + t.offset + t.nbytes > g->file.size))
      ok = false;
  if (!ok) {
    delete g;
    set_last_cuda_error(cudaErrorInvalidValue, "syn_gguf_open: not a valid GGUF v2/v3 file");
    return SYN_ERR_INVALID_ARG;
  }
  *out = g;
  return SYN_OK;
}

syn_status_t syn_gguf_close(syn_gguf_t* g) {
  if (!g) return SYN_ERR_NULL_PTR;
  delete g;
  return SYN_OK;
}

syn_status_t syn_gguf_tensor_count(const syn_gguf_t* g, size_t* count) {
  if (!g || !count) return SYN_ERR_NULL_PTR;
  *count = g->tensors.size();
  return SYN_OK;
}

syn_status_t syn_gguf_tensor_info(const syn_gguf_t* g, size_t i, const char** name,
                                  uint32_t* ggml_type, size_t* n_dims, uint64_t* dims4,
                                  const void** data, size_t* nbytes) {
  if (!g || !name || !ggml_type || !n_dims || !dims4 || !data || !nbytes) return SYN_ERR_NULL_PTR;
  if (i >= g->tensors.size()) return SYN_ERR_INVALID_ARG;
  const auto& t = g->tensors[i];
  *name = t.name.c_str();
  *ggml_type = t.type;
  *n_dims = t.dims.size();
  for (size_t d = 0; d < 4; d++) dims4[d] = d < t.dims.size() ? t.dims[d] : 1;
  *data = t.nbytes ? g->file.data + g->data_start + t.offset : nullptr;
  *nbytes = t.nbytes;
  return SYN_OK;
}

syn_status_t syn_gguf_meta_num(const syn_gguf_t* g, const char* key, double* value) {
  if (!g || !key || !value) return SYN_ERR_NULL_PTR;
  auto it = g->num.find(key);
  if (it == g->num.end()) return SYN_ERR_INVALID_ARG;
  *value = it->second;
  return SYN_OK;
}

syn_status_t syn_gguf_meta_str(const syn_gguf_t* g, const char* key, const char** value) {
  if (!g || !key || !value) return SYN_ERR_NULL_PTR;
  auto it = g->text.find(key);
  if (it == g->text.end()) return SYN_ERR_INVALID_ARG;
  *value = it->second.c_str();
  return SYN_OK;
}

// llama.cpp tensor names -> the runner's (Hugging Face) names.
syn_status_t syn_gguf_runner_name(const char* gguf_name, char* out, size_t cap) {
  if (!gguf_name || !out) return SYN_ERR_NULL_PTR;
  static const std::map<std::string, std::string> top = {
      {"token_embd.weight", "model.embed_tokens.weight"},
      {"output_norm.weight", "model.norm.weight"},
      {"output.weight", "lm_head.weight"}};
  static const std::map<std::string, std::string> blk = {
      {"attn_norm.weight", "input_layernorm.weight"},
      {"ffn_norm.weight", "post_attention_layernorm.weight"},
      {"attn_q.weight", "self_attn.q_proj.weight"},
      {"attn_k.weight", "self_attn.k_proj.weight"},
      {"attn_v.weight", "self_attn.v_proj.weight"},
      {"attn_output.weight", "self_attn.o_proj.weight"},
      {"attn_q_norm.weight", "self_attn.q_norm.weight"},
      {"attn_k_norm.weight", "self_attn.k_norm.weight"},
      {"ffn_gate.weight", "mlp.gate_proj.weight"},
      {"ffn_up.weight", "mlp.up_proj.weight"},
      {"ffn_down.weight", "mlp.down_proj.weight"}};
  const std::string s(gguf_name);
  std::string res;
  auto t = top.find(s);
  if (t != top.end()) {
    res = t->second;
  } else if (s.compare(0, 4, "blk.") == 0) {
    const size_t dot = s.find('.', 4);
    if (dot == std::string::npos || dot == 4) return SYN_ERR_INVALID_ARG;
    for (size_t i = 4; i < dot; i++)
      if (s[i] < '0' || s[i] > '9') return SYN_ERR_INVALID_ARG;
    auto b = blk.find(s.substr(dot + 1));
    if (b == blk.end()) return SYN_ERR_INVALID_ARG;
    res = "model.layers." + s.substr(4, dot - 4) + "." + b->second;
  } else {
    return SYN_ERR_INVALID_ARG;
  }
  if (res.size() + 1 > cap) return SYN_ERR_INVALID_ARG;
  memcpy(out, res.c_str(), res.size() + 1);
  return SYN_OK;
}

// Model config (the reference's config-JSON schema) from GGUF metadata
// (<arch>.block_count, .embedding_length, .feed_forward_length,
// .attention.head_count[_kv], .attention.key_length,
// .attention.layer_norm_rms_epsilon, .rope.freq_base,
// .attention.sliding_window) and the vocabulary from token_embd.
syn_status_t syn_gguf_config_json(const syn_gguf_t* g, char* out, size_t cap, size_t* needed) {
  if (!g || !needed) return SYN_ERR_NULL_PTR;
  auto ta = g->text.find("general.architecture");
  if (ta == g->text.end()) return SYN_ERR_INVALID_ARG;
  const std::string a = ta->second;
  auto num = [&](const std::string& k, double dflt) {
    auto it = g->num.find(a + "." + k);
    return it == g->num.end() ? dflt : it->second;
  };
  const double L = num("block_count", 0), h = num("embedding_length", 0),
               ff = num("feed_forward_length", 0), hq = num("attention.head_count", 0);
  const double hkv = num("attention.head_count_kv", hq);
  const double hd = num("attention.key_length", hq > 0 ? h / hq : 0);
  const double eps = num("attention.layer_norm_rms_epsilon", 1e-6);
  const double base = num("rope.freq_base", 10000.0);
  const double win = num("attention.sliding_window", 0);
  auto te = g->index.find("token_embd.weight");
  if (te == g->index.end() || g->tensors[te->second].dims.size() != 2 || L <= 0 || h <= 0 ||
      ff <= 0 || hq <= 0)
    return SYN_ERR_INVALID_ARG;
  const double V = (double)g->tensors[te->second].dims[1];
  const bool tied = g->index.find("output.weight") == g->index.end();
  auto n0 = [](double v) {
    char b[64];
    snprintf(b, sizeof(b), "%.0f", v);
    return std::string(b);
  };
  auto g9 = [](double v) {
    char b[64];
    snprintf(b, sizeof(b), "%.9g", v);
    return std::string(b);
  };
  std::string js = "{\"name\": \"" + a + "\", \"architecture\": {\"hidden_size\": " + n0(h) +
                   ", \"num_layers\": " + n0(L) + ", \"vocab_size\": " + n0(V) +
                   ", \"max_sequence_length\": " + n0(num("context_length", 4096)) +
                   ", \"tie_word_embeddings\": " + (tied ? "true" : "false") +
                   "}, \"attention\": {\"type\": \"" + (win > 0 ? "SlidingWindow" : "GQA") +
                   "\", \"num_heads\": " + n0(hq) + ", \"num_kv_heads\": " + n0(hkv) +
                   ", \"head_dim\": " + n0(hd) +
                   (win > 0 ? ", \"window_size\": " + n0(win) : std::string()) +
                   "}, \"norm\": {\"type\": \"RMSNorm\", \"eps\": " + g9(eps) +
                   "}, \"ffn\": {\"type\": \"SwiGLU\", \"intermediate_size\": " + n0(ff) +
                   "}, \"position\": {\"type\": \"RoPE\", \"base\": " + g9(base) +
                   "}, \"quantization\": {\"type\": \"F32\"}}";
  *needed = js.size() + 1;
  if (!out || cap < js.size() + 1) return out ? SYN_ERR_INVALID_ARG : SYN_OK;
  memcpy(out, js.c_str(), js.size() + 1);
  return SYN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// safetensors
// ---------------------------------------------------------------------------
struct syn_safetensors_s {
  MappedFile file;
  struct Tensor {
    std::string name;
    int dtype;
    std::vector<uint64_t> shape;
    const uint8_t* data;
    size_t nbytes;
  };
  std::vector<Tensor> tensors;
  std::map<std::string, size_t> index;
};

namespace {

// The safetensors header: {"name": {"dtype": "..", "shape": [..],
// "data_offsets": [a, b]}, ..., "__metadata__": {...}}.
struct StHeader {
  const char* s;
  size_t n, i = 0;
  bool ok = true;
  void ws() {
    while (i < n && (s[i] == ' ' || s[i] == '\n' || s[i] == '\t' || s[i] == '\r')) i++;
  }
  bool eat(char c) {
    ws();
    if (i < n && s[i] == c) {
      i++;
      return true;
    }
    return false;
  }
  std::string str() {
    ws();
    std::string out;
    if (i >= n || s[i] != '"') {
      ok = false;
      return out;
    }
    i++;
    while (i < n && s[i] != '"') {
      if (s[i] == '\\' && i + 1 < n) i++;
      out += s[i++];
    }
    if (i >= n) ok = false;
    else i++;
    return out;
  }
  bool number(uint64_t* v) {
    ws();
    uint64_t x = 0;
    size_t j = i;
    while (i < n && s[i] >= '0' && s[i] <= '9') x = x * 10 + (uint64_t)(s[i++] - '0');
    *v = x;
    return i > j;
  }
  std::vector<uint64_t> numbers() {
    std::vector<uint64_t> out;
    if (!eat('[')) {
      ok = false;
      return out;
    }
    if (eat(']')) return out;
    do {
      uint64_t v;
      if (!number(&v)) {
        ok = false;
        return out;
      }
      out.push_back(v);
    } while (eat(','));
    if (!eat(']')) ok = false;
    return out;
  }
  void skip_value(int depth = 0) {  // any JSON value (the metadata object)
    ws();
    if (depth > 16 || i >= n) {
      ok = false;
      return;
    }
    if (s[i] == '"') {
      str();
    } else if (s[i] == '{' || s[i] == '[') {
      const char close = s[i] == '{' ? '}' : ']';
      i++;
      if (eat(close)) return;
      do {
        if (close == '}') {
          str();
          if (!eat(':')) {
            ok = false;
            return;
          }
        }
        skip_value(depth + 1);
      } while (ok && eat(','));
      if (!eat(close)) ok = false;
    } else {
      while (i < n && s[i] != ',' && s[i] != '}' && s[i] != ']') i++;
    }
  }
};

int st_dtype(const std::string& d, size_t* elem) {
  if (d == "F32") return *elem = 4, SYN_DTYPE_F32;
  if (d == "F16") return *elem = 2, SYN_DTYPE_F16;
  if (d == "BF16") return *elem = 2, SYN_DTYPE_BF16;
  if (d == "I64") return *elem = 8, SYN_DTYPE_I64;
  if (d == "I32") return *elem = 4, SYN_DTYPE_I32;
  if (d == "U8") return *elem = 1, SYN_DTYPE_U8;
  return -1;
}

}  // namespace

extern "C" {

syn_status_t syn_safetensors_open(const char* path, syn_safetensors_t** out) {
  if (!path || !out) return SYN_ERR_NULL_PTR;
  *out = nullptr;
  auto* f = new (std::nothrow) syn_safetensors_s();
  if (!f) return SYN_ERR_OUT_OF_MEMORY;
  syn_status_t bad = SYN_ERR_INVALID_ARG;
  const char* why = "syn_safetensors_open: invalid header";
  bool ok = f->file.open(path) && f->file.size >= 8;
  uint64_t hsize = 0;
  if (ok) {
    memcpy(&hsize, f->file.data, 8);
    ok = hsize <= f->file.size - 8;
  }
  if (ok) {
    StHeader h{reinterpret_cast<const char*>(f->file.data + 8), (size_t)hsize};
    const size_t data_start = 8 + (size_t)hsize;
    ok = h.eat('{');
    if (ok && !h.eat('}')) {
      do {
        const std::string name = h.str();
        if (!h.ok || !h.eat(':')) {
          ok = false;
          break;
        }
        if (name == "__metadata__") {
          h.skip_value();
          continue;
        }
        syn_safetensors_s::Tensor t;
        t.name = name;
        t.dtype = -1;
        std::string dt;
        std::vector<uint64_t> offs;
        bool have_shape = false;
        if (!h.eat('{')) {
          ok = false;
          break;
        }
        do {
          const std::string key = h.str();
          if (!h.ok || !h.eat(':')) {
            ok = false;
            break;
          }
          if (key == "dtype") dt = h.str();
          else if (key == "shape") t.shape = h.numbers(), have_shape = true;
          else if (key == "data_offsets") offs = h.numbers();
          else h.skip_value();
        } while (h.ok && h.eat(','));
        if (!ok || !h.ok || !h.eat('}') || dt.empty() || !have_shape || offs.size() != 2) {
          ok = false;
          break;
        }
        size_t elem = 0;
        t.dtype = st_dtype(dt, &elem);
        if (t.dtype < 0) {
          ok = false;
          bad = SYN_ERR_UNSUPPORTED;
          why = "syn_safetensors_open: unsupported dtype";
          break;
        }
        if (offs[1] < offs[0] || offs[1] > f->file.size - data_start) {
          ok = false;
          why = "syn_safetensors_open: tensor data exceeds file bounds";
          break;
        }
        t.data = f->file.data + data_start + offs[0];
        t.nbytes = (size_t)(offs[1] - offs[0]);
        uint64_t numel = 1;
        for (uint64_t d : t.shape) numel *= d;
        if (numel * elem != t.nbytes) {
          ok = false;
          why = "syn_safetensors_open: shape and data size disagree";
          break;
        }
        f->index[t.name] = f->tensors.size();
        f->tensors.push_back(std::move(t));
      } while (h.ok && h.eat(','));
      ok = ok && h.ok && h.eat('}');
    }
  }
  if (!ok) {
    delete f;
    set_last_cuda_error(cudaErrorInvalidValue, why);
    return bad;
  }
  *out = f;
  return SYN_OK;
}

syn_status_t syn_safetensors_close(syn_safetensors_t* f) {
  if (!f) return SYN_ERR_NULL_PTR;
  delete f;
  return SYN_OK;
}

syn_status_t syn_safetensors_tensor_count(const syn_safetensors_t* f, size_t* count) {
  if (!f || !count) return SYN_ERR_NULL_PTR;
  *count = f->tensors.size();
  return SYN_OK;
}

syn_status_t syn_safetensors_tensor_info(const syn_safetensors_t* f, size_t i, const char** name,
                                         syn_dtype_t* dtype, size_t* n_dims, uint64_t* dims4,
                                         const void** data, size_t* nbytes) {
  if (!f || !name || !dtype || !n_dims || !dims4 || !data || !nbytes) return SYN_ERR_NULL_PTR;
  if (i >= f->tensors.size()) return SYN_ERR_INVALID_ARG;
  const auto& t = f->tensors[i];
  if (t.shape.size() > 4) return SYN_ERR_UNSUPPORTED;
  *name = t.name.c_str();
  *dtype = (syn_dtype_t)t.dtype;
  *n_dims = t.shape.size();
  for (size_t d = 0; d < 4; d++) dims4[d] = d < t.shape.size() ? t.shape[d] : 1;
  *data = t.data;
  *nbytes = t.nbytes;
  return SYN_OK;
}

// Element conversion of the safetensors loader (safetensors.rs:233-290,
// converter.rs:12-48): f16 with the loader's subnormal rule, bf16 as the
// upper half of an f32, integers cast.
syn_status_t syn_convert_to_f32(syn_dtype_t dtype, const void* src, size_t count, float* dst) {
  if ((!src || !dst) && count) return SYN_ERR_NULL_PTR;
  const uint8_t* p = static_cast<const uint8_t*>(src);
  for (size_t i = 0; i < count; i++) {
    switch (dtype) {
      case SYN_DTYPE_F32: memcpy(dst + i, p + 4 * i, 4); break;
      case SYN_DTYPE_F16: {
        uint16_t b;
        memcpy(&b, p + 2 * i, 2);
        dst[i] = f16_loader_host(b);
        break;
      }
      case SYN_DTYPE_BF16: {
        uint16_t b;
        memcpy(&b, p + 2 * i, 2);
        const uint32_t bits = (uint32_t)b << 16;
        memcpy(dst + i, &bits, 4);
        break;
      }
      case SYN_DTYPE_I64: {
        int64_t v;
        memcpy(&v, p + 8 * i, 8);
        dst[i] = (float)v;
        break;
      }
      case SYN_DTYPE_I32: {
        int32_t v;
        memcpy(&v, p + 4 * i, 4);
        dst[i] = (float)v;
        break;
      }
      case SYN_DTYPE_U8: dst[i] = (float)p[i]; break;
      default: return SYN_ERR_INVALID_ARG;
    }
  }
  return SYN_OK;
}

// ---------------------------------------------------------------------------
// f16 / bf16 weights -> INT8 on the device
// ---------------------------------------------------------------------------
syn_status_t syn_cuda_quantize_weights_int8_half(const uint16_t* w, syn_dtype_t dtype, size_t n,
                                                 size_t k, int8_t* out_kn, float* scales,
                                                 void* stream) {
  if (!w || !out_kn || !scales) return SYN_ERR_NULL_PTR;
  if (dtype != SYN_DTYPE_F16 && dtype != SYN_DTYPE_BF16) return SYN_ERR_INVALID_ARG;
  if (n == 0 || k == 0) return SYN_OK;
  return launch_quantize_weights_half(w, dtype, n, k, out_kn, scales, (cudaStream_t)stream);
}

// Host [n, k] weights of dtype f32 / f16 / bf16 -> INT8 [k, n] + scales
// [n] on the host, quantised on the context's device. Synchronous.
syn_status_t syn_cuda_quantize_weights_int8_host(syn_cuda_ctx_t* ctx, syn_dtype_t dtype,
                                                 const void* w, size_t n, size_t k,
                                                 int8_t* out_kn, float* scales) {
  if (!ctx || !w || !out_kn || !scales) return SYN_ERR_NULL_PTR;
  if (dtype != SYN_DTYPE_F32 && dtype != SYN_DTYPE_F16 && dtype != SYN_DTYPE_BF16)
    return SYN_ERR_INVALID_ARG;
  if (n == 0 || k == 0) return SYN_OK;
  DeviceGuard g(ctx->device);
  if (!g.ok) return SYN_ERR_CUDA;
  const size_t es = dtype == SYN_DTYPE_F32 ? 4 : 2;
  const size_t in_bytes = (n * k * es + 255) & ~(size_t)255;
  void* buf = nullptr;
  SYN_CUDA_TRY(cudaMalloc(&buf, in_bytes + n * k + n * 4 + 256));
  uint8_t* b = static_cast<uint8_t*>(buf);
  int8_t* d_q = reinterpret_cast<int8_t*>(b + in_bytes);
  float* d_s = reinterpret_cast<float*>(b + in_bytes + ((n * k + 255) & ~(size_t)255));
  cudaStream_t st = ctx->upload_stream;
  syn_status_t s = SYN_OK;
  cudaError_t e = cudaMemcpyAsync(b, w, n * k * es, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    s = dtype == SYN_DTYPE_F32
            ? launch_quantize_weights(reinterpret_cast<const float*>(b), n, k, d_q, d_s, st)
            : launch_quantize_weights_half(reinterpret_cast<const uint16_t*>(b), dtype, n, k,
                                           d_q, d_s, st);
    if (s == SYN_OK) e = cudaMemcpyAsync(out_kn, d_q, n * k, cudaMemcpyDeviceToHost, st);
    if (s == SYN_OK && e == cudaSuccess)
      e = cudaMemcpyAsync(scales, d_s, n * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  cudaFree(buf);
  if (e != cudaSuccess) {
    set_last_cuda_error(e, "syn_cuda_quantize_weights_int8_host");
    return SYN_ERR_CUDA;
  }
  return s;
}

// ---------------------------------------------------------------------------
// Repack cache
// ---------------------------------------------------------------------------
namespace {
struct CacheHeader {
  char magic[8];  // "SYNWGT1\0"
  uint64_t key;
  int32_t fmt, pad;
  uint64_t n, k, kp, bytes, algo_bytes;
};
}  // namespace

syn_status_t syn_cuda_weight_upload_cached(syn_cuda_ctx_t* ctx, syn_qformat_t fmt,
                                           const void* host, size_t n, size_t k,
                                           const float* scales_or_null, const char* cache_dir,
                                           syn_cuda_weight_t** out, int* hit) {
  if (!ctx || !host || !out || !cache_dir) return SYN_ERR_NULL_PTR;
  if (hit) *hit = 0;
  if (fmt < SYN_QFMT_INT8_KN || fmt > SYN_QFMT_Q6_K) return SYN_ERR_INVALID_ARG;
  if (fmt == SYN_QFMT_INT8_KN && !scales_or_null) return SYN_ERR_NULL_PTR;
  const size_t src = n * weight_src_row_bytes(fmt, k);
  uint64_t key = hash_bytes(host, src, 0x5EED0000ull ^ ((uint64_t)fmt << 48) ^ (n << 20) ^ k);
  if (fmt == SYN_QFMT_INT8_KN) key = hash_bytes(scales_or_null, n * 4, key);
  char path[4096];
  snprintf(path, sizeof(path), "%s/%016llx.synw", cache_dir, (unsigned long long)key);
  // a hit: the header must describe this exact weight
  if (FILE* f = fopen(path, "rb")) {
    CacheHeader h;
    syn_cuda_weight_s probe{};
    probe.fmt = fmt;
    probe.n = n;
    probe.k = k;
    probe.kp = fmt == SYN_QFMT_INT8_KN ? (k + 31) / 32 * 32 : k;
    const size_t bytes = weight_layout(&probe, nullptr);
    bool good = fread(&h, sizeof(h), 1, f) == 1 && memcmp(h.magic, "SYNWGT1", 8) == 0 &&
                h.key == key && h.fmt == (int)fmt && h.n == n && h.k == k && h.kp == probe.kp &&
                h.bytes == bytes;
    std::vector<uint8_t> blob;
    if (good) {
      blob.resize(bytes);
      good = fread(blob.data(), 1, bytes, f) == bytes;
    }
    fclose(f);
    if (good) {
      DeviceGuard g(ctx->device);
      if (!g.ok) return SYN_ERR_CUDA;
      auto* w = new (std::nothrow) syn_cuda_weight_s(probe);
      if (!w) return SYN_ERR_OUT_OF_MEMORY;
      w->device = ctx->device;
      w->bytes = bytes;
      w->algo_bytes = h.algo_bytes;
      cudaError_t e = cudaMalloc(&w->buf, bytes);
      if (e == cudaSuccess) e = cudaMemcpy(w->buf, blob.data(), bytes, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) {
        if (w->buf) cudaFree(w->buf);
        delete w;
        set_last_cuda_error(e, "syn_cuda_weight_upload_cached");
        return SYN_ERR_CUDA;
      }
      weight_layout(w, static_cast<uint8_t*>(w->buf));
      *out = w;
      if (hit) *hit = 1;
      return SYN_OK;
    }
  }
  syn_status_t s = syn_cuda_weight_upload(ctx, fmt, host, n, k, scales_or_null, out);
  if (s != SYN_OK) return s;
  // store: write to a temporary name, then rename (readers never see a
  // partial file); a failure to write leaves the upload valid
  std::vector<uint8_t> blob((*out)->bytes);
  if (cudaMemcpy(blob.data(), (*out)->buf, blob.size(), cudaMemcpyDeviceToHost) != cudaSuccess)
    return SYN_OK;
  CacheHeader h{};
  memcpy(h.magic, "SYNWGT1", 8);
  h.key = key;
  h.fmt = fmt;
  h.n = n;
  h.k = k;
  h.kp = (*out)->kp;
  h.bytes = (*out)->bytes;
  h.algo_bytes = (*out)->algo_bytes;
  char tmp[4200];
  snprintf(tmp, sizeof(tmp), "%s.%d.tmp", path, (int)getpid());
  if (FILE* f = fopen(tmp, "wb")) {
    const bool good = fwrite(&h, sizeof(h), 1, f) == 1 &&
                      fwrite(blob.data(), 1, blob.size(), f) == blob.size();
    if (fclose(f) == 0 && good) rename(tmp, path);
    else remove(tmp);
  }
  return SYN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Whole models from a file
// ---------------------------------------------------------------------------
namespace {

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// f32 copy of a GGUF F32 / F16 tensor (F16 by the loader's rule).
bool gguf_f32(const syn_gguf_s::Tensor& t, const uint8_t* data, uint64_t numel,
              std::vector<float>& out) {
  out.resize(numel);
  if (t.type == GG_F32) {
    memcpy(out.data(), data, numel * 4);
    return true;
  }
  if (t.type == GG_F16) {
    for (uint64_t i = 0; i < numel; i++) {
      uint16_t b;
      memcpy(&b, data + 2 * i, 2);
      out[i] = f16_loader_host(b);
    }
    return true;
  }
  return false;
}

}  // namespace

extern "C" {

// Stages every runner tensor of a GGUF file into an unfinalised model.
// Quantised linears keep their raw blocks (Q4_0, Q8_0, Q4_K, Q6_K); norms and
// F32 / F16 embeddings are converted to f32; a quantised token_embd is
// dequantised on the device with the reference's formulas. Without
// output.weight the LM head is token_embd (tied). For
// general.architecture "llama", whose GGUF converter interleaves the rows
// of attn_q / attn_k for pairwise RoPE, the rows are put back in the
// rotate-half order the runner (and the Hugging Face checkpoint) uses: GGUF
// row h*hd + 2i + a holds checkpoint row h*hd + a*hd/2 + i.
syn_status_t syn_cuda_model_load_gguf(syn_cuda_model_t* m, const syn_gguf_t* g) {
  if (!m || !g) return SYN_ERR_NULL_PTR;
  auto arch = g->text.find("general.architecture");
  const bool unpermute = arch != g->text.end() && arch->second == "llama";
  double hq = 0, hkv = 0;
  if (arch != g->text.end()) {
    auto a = g->num.find(arch->second + ".attention.head_count");
    auto b = g->num.find(arch->second + ".attention.head_count_kv");
    hq = a == g->num.end() ? 0 : a->second;
    hkv = b == g->num.end() ? hq : b->second;
  }
  const bool tied = g->index.find("output.weight") == g->index.end();
  syn_status_t s = SYN_OK;
  for (const auto& t : g->tensors) {
    char name[512];
    if (syn_gguf_runner_name(t.name.c_str(), name, sizeof(name)) != SYN_OK) continue;
    const std::string nm(name);
    const uint8_t* data = g->file.data + g->data_start + t.offset;
    uint64_t numel = 1;
    for (uint64_t d : t.dims) numel *= d;
    if (!t.nbytes) return SYN_ERR_UNSUPPORTED;  // a GGML type this loader cannot size
    if (t.dims.size() == 1) {
      std::vector<float> v;
      if (!gguf_f32(t, data, numel, v)) return SYN_ERR_UNSUPPORTED;
      if ((s = syn_cuda_model_set_tensor(m, name, v.data(), v.size()))) return s;
      continue;
    }
    if (t.dims.size() != 2) return SYN_ERR_SHAPE_MISMATCH;
    const size_t K = (size_t)t.dims[0], N = (size_t)t.dims[1];
    const int fmt = ggml_to_qfmt(t.type);
    if (nm == "model.embed_tokens.weight") {
      std::vector<float> v;
      if (fmt < 0) {
        if (!gguf_f32(t, data, numel, v)) return SYN_ERR_UNSUPPORTED;
      } else {
        syn_cuda_weight_t* w = nullptr;
        if ((s = syn_cuda_weight_upload(model_context(m), (syn_qformat_t)fmt, data, N, K, nullptr,
                                        &w)))
          return s;
        v.resize(numel);
        s = syn_cuda_weight_dequant(w, v.data());
        syn_cuda_weight_destroy(w);
        if (s) return s;
      }
      if ((s = syn_cuda_model_set_tensor(m, name, v.data(), v.size()))) return s;
      if (tied) {
        if (fmt < 0) return SYN_ERR_UNSUPPORTED;  // the runner's LM head is a quantised matmul
        if ((s = syn_cuda_model_set_linear(m, "lm_head.weight", (syn_qformat_t)fmt, data, N, K,
                                           nullptr)))
          return s;
      }
      continue;
    }
    if (fmt < 0) return SYN_ERR_UNSUPPORTED;  // F32 / F16 / Q4_1 linears: no runner path
    const bool q = ends_with(nm, "self_attn.q_proj.weight"), k = ends_with(nm, "self_attn.k_proj.weight");
    if (unpermute && (q || k)) {
      const size_t heads = (size_t)(q ? hq : hkv);
      if (!heads || N % heads || (N / heads) % 2) return SYN_ERR_SHAPE_MISMATCH;
      const size_t hd = N / heads, rb = weight_src_row_bytes(fmt, K);
      std::vector<uint8_t> rows(N * rb);
      for (size_t h = 0; h < heads; h++)
        for (size_t i = 0; i < hd / 2; i++)
          for (size_t a = 0; a < 2; a++)
            memcpy(rows.data() + (h * hd + a * (hd / 2) + i) * rb,
                   data + (h * hd + 2 * i + a) * rb, rb);
      if ((s = syn_cuda_model_set_linear(m, name, (syn_qformat_t)fmt, rows.data(), N, K, nullptr)))
        return s;
    } else if ((s = syn_cuda_model_set_linear(m, name, (syn_qformat_t)fmt, data, N, K, nullptr))) {
      return s;
    }
  }
  return SYN_OK;
}

// Stages a safetensors checkpoint (Hugging Face names) for the INT8 runner,
// as the reference's --quantize load does (quantize_model, int8.rs:78-152):
// every 2-D *_proj.weight and lm_head.weight of dtype F32 / F16 / BF16 is
// quantised per output row on the device; other float tensors (norms, the
// embedding) are converted to f32. Without lm_head.weight the LM head is
// quantised from model.embed_tokens.weight (tied, int8.rs:127-139).
syn_status_t syn_cuda_model_load_safetensors(syn_cuda_model_t* m, const syn_safetensors_t* f) {
  if (!m || !f) return SYN_ERR_NULL_PTR;
  syn_status_t s;
  auto quant = [&](const syn_safetensors_s::Tensor& t, const char* as) -> syn_status_t {
    if (t.shape.size() != 2) return SYN_ERR_SHAPE_MISMATCH;
    const size_t n = (size_t)t.shape[0], k = (size_t)t.shape[1];
    std::vector<int8_t> q(n * k);
    std::vector<float> sc(n);
    syn_status_t st = syn_cuda_quantize_weights_int8_host(model_context(m), (syn_dtype_t)t.dtype,
                                                          t.data, n, k, q.data(), sc.data());
    if (st) return st;
    return syn_cuda_model_set_linear(m, as, SYN_QFMT_INT8_KN, q.data(), n, k, sc.data());
  };
  bool have_head = false;
  for (const auto& t : f->tensors) {
    const bool flt = t.dtype == SYN_DTYPE_F32 || t.dtype == SYN_DTYPE_F16 ||
                     t.dtype == SYN_DTYPE_BF16;
    if (!flt) continue;  // index tensors (position ids, ...) are not runner weights
    if (t.shape.size() == 2 && (ends_with(t.name, "_proj.weight") || t.name == "lm_head.weight")) {
      if ((s = quant(t, t.name.c_str()))) return s;
      have_head |= t.name == "lm_head.weight";
      continue;
    }
    uint64_t numel = 1;
    for (uint64_t d : t.shape) numel *= d;
    std::vector<float> v(numel);
    if ((s = syn_convert_to_f32((syn_dtype_t)t.dtype, t.data, numel, v.data()))) return s;
    if ((s = syn_cuda_model_set_tensor(m, t.name.c_str(), v.data(), v.size()))) return s;
  }
  if (!have_head) {
    auto e = f->index.find("model.embed_tokens.weight");
    if (e == f->index.end()) return SYN_ERR_SHAPE_MISMATCH;
    if ((s = quant(f->tensors[e->second], "lm_head.weight"))) return s;
  }
  return SYN_OK;
}

}  // extern "C"
