"""Python mirror of the reference's interface for the quantized-matmul path.

Function names, argument meaning and error behaviour follow the reference's
safe wrappers (crates/synapse-core/src/lib.rs:602-775) and the INT8 layer
(crates/synapse-inference/src/quantization/primitives/int8_linear.rs), but
operate on CUDA tensors through the C ABI in include/synapse_cuda.h. torch
is used only for device memory and the current stream.
"""
import ctypes

import torch

from . import _lib
from . import formats as _formats
from .formats import QFormat


class SynapseError(RuntimeError):
    """Mirrors synapse_core::SynapseError (status code -> variant)."""

    NAMES = {1: "NullPointer", 2: "InvalidArg", 3: "OutOfMemory", 4: "ShapeMismatch",
             5: "NotContiguous", 6: "InvalidAxis", 7: "InvalidDimensions", 8: "Internal",
             9: "Cuda", 10: "Nccl", 11: "Timeout", 12: "Unsupported"}

    def __init__(self, status, where=""):
        self.status = int(status)
        self.variant = self.NAMES.get(self.status, "Unknown")
        detail = ""
        if self.status == 9:
            detail = " " + lib().syn_cuda_last_error().decode(errors="replace")
        super().__init__(f"{where}: {self.variant} ({self.status}){detail}")


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        from . import lib as loaded
        _LIB = loaded
    return _LIB


def _check(status, where):
    if status != 0:
        raise SynapseError(status, where)


def row_bytes(fmt, k):
    """Bytes of one K-element row in the reference's storage format."""
    try:
        return _formats.row_bytes(fmt, k)
    except ValueError:
        raise SynapseError(4, "row_bytes") from None


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise SynapseError(2, "expected CUDA tensors")
        if not t.is_contiguous():
            raise SynapseError(5, "expected contiguous tensors")


def capability_summary():
    s = _lib.CapabilitySummary()
    _check(lib().syn_cuda_capability_summary(ctypes.byref(s)), "capability_summary")
    return {f: getattr(s, f) for f, _ in s._fields_}


def quantize_per_channel_int8(data, channels, channel_size):
    """synapse_core::quantize_per_channel_int8 (synapse-core/src/lib.rs:602-625):
    returns (int8 [channels*channel_size], f32 [channels])."""
    if channels == 0 or channel_size == 0:
        raise SynapseError(2, "quantize_per_channel_int8")
    if data.numel() != channels * channel_size:
        raise SynapseError(4, "quantize_per_channel_int8")
    _need_cuda(data)
    out = torch.empty(channels * channel_size, dtype=torch.int8, device=data.device)
    scales = torch.empty(channels, dtype=torch.float32, device=data.device)
    _check(lib().syn_cuda_quantize_per_channel_int8(_ptr(data), channels, channel_size,
                                                    _ptr(out), _ptr(scales), _stream(data)),
           "quantize_per_channel_int8")
    return out, scales


def quantize_weights_int8(w, out_features, in_features):
    """MinMaxCalibration + QuantizedLinear::from_f32_with_scales + transpose_i8
    (int8_linear.rs:35-70): returns (int8 [in, out] GEMM layout, f32 [out])."""
    _need_cuda(w)
    if w.numel() != out_features * in_features:
        raise SynapseError(4, "quantize_weights_int8")
    q = torch.empty(in_features * out_features, dtype=torch.int8, device=w.device)
    s = torch.empty(out_features, dtype=torch.float32, device=w.device)
    _check(lib().syn_cuda_quantize_weights_int8(_ptr(w), out_features, in_features, _ptr(q),
                                                _ptr(s), _stream(w)), "quantize_weights_int8")
    return q, s


def qgemm_int8(m, n, k, a, b, scales_a, scales_b):
    """synapse_core::qgemm_int8 (synapse-core/src/lib.rs:654-689): lda=k,
    ldb=n, ldc=n; returns f32 [m*n]."""
    if m == 0 or n == 0 or k == 0:
        return torch.zeros(m * n, dtype=torch.float32,
                           device=a.device if isinstance(a, torch.Tensor) else "cuda")
    if a.numel() < m * k or b.numel() < k * n:
        raise SynapseError(4, "qgemm_int8")
    if scales_a.numel() < m or scales_b.numel() < n:
        raise SynapseError(4, "qgemm_int8")
    _need_cuda(a, b, scales_a, scales_b)
    c = torch.empty(m * n, dtype=torch.float32, device=a.device)
    _check(lib().syn_cuda_qgemm_int8(m, n, k, _ptr(a), k, _ptr(b), n, _ptr(c), n,
                                     _ptr(scales_a), _ptr(scales_b), _stream(a)), "qgemm_int8")
    return c


def q4_0_gemv(n, k, a, b_q4):
    """synapse_core::q4_0_gemv (synapse-core/src/lib.rs:754-775): returns f32 [n]."""
    if n == 0 or k == 0:
        return torch.zeros(n, dtype=torch.float32, device="cuda")
    if k % 32 != 0:
        raise SynapseError(4, "q4_0_gemv")
    if a.numel() < k:
        raise SynapseError(4, "q4_0_gemv")
    _need_cuda(a, b_q4)
    if b_q4.numel() < n * (k // 32) * 18:
        raise SynapseError(4, "q4_0_gemv")
    c = torch.empty(n, dtype=torch.float32, device=a.device)
    _check(lib().syn_cuda_q4_0_gemv(n, k, _ptr(a), _ptr(b_q4), _ptr(c), _stream(a)),
           "q4_0_gemv")
    return c


class Context:
    """One library context per device (syn_cuda_context_create)."""

    def __init__(self, device=0):
        self.device = int(device)
        h = ctypes.c_void_p()
        _check(lib().syn_cuda_context_create(self.device, ctypes.byref(h)), "context_create")
        self.handle = h

    def tp_init(self, rank, world, unique_id):
        """Joins a tensor-parallel group (syn_cuda_tp_init); unique_id: the
        bytes of tp_unique_id() from rank 0."""
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(unique_id))
        _check(lib().syn_cuda_tp_init(self.handle, int(rank), int(world), buf), "tp_init")
        self.tp_rank, self.tp_world = int(rank), int(world)

    def tp_allreduce_sum(self, t):
        _need_cuda(t)
        _check(lib().syn_cuda_tp_allreduce_sum(self.handle, _ptr(t), t.numel(), _stream(t)),
               "tp_allreduce_sum")
        return t

    def close(self):
        if self.handle:
            lib().syn_cuda_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_unique_id():
    """A new tensor-parallel group id (rank 0; ncclGetUniqueId), as bytes."""
    buf = (ctypes.c_uint8 * 128)()
    _check(lib().syn_cuda_tp_unique_id(buf), "tp_unique_id")
    return bytes(buf)


def tp_shard_linear(fmt, data, n, k, rank, world, axis, scales=None):
    """This rank's shard of a linear weight in its storage format
    (syn_cuda_tp_shard_linear; host only). Returns (data, n, k, scales)."""
    import numpy as np
    fmt = QFormat[fmt] if isinstance(fmt, str) else QFormat(fmt)
    buf = np.ascontiguousarray(np.asarray(data).view(np.uint8).reshape(-1))
    out = np.empty(buf.size // world, dtype=np.uint8)
    sc = None
    osc = None
    if fmt == QFormat.INT8_KN:
        sc = np.ascontiguousarray(np.asarray(scales, dtype=np.float32))
        osc = np.empty(n // world if axis == 0 else n, dtype=np.float32)
    no, ko = ctypes.c_size_t(), ctypes.c_size_t()
    _check(lib().syn_cuda_tp_shard_linear(
        int(fmt), buf.ctypes.data_as(ctypes.c_void_p), n, k,
        sc.ctypes.data_as(ctypes.c_void_p) if sc is not None else None, axis, rank, world,
        out.ctypes.data_as(ctypes.c_void_p),
        osc.ctypes.data_as(ctypes.c_void_p) if osc is not None else None, ctypes.byref(no),
        ctypes.byref(ko)), "tp_shard_linear")
    return out, no.value, ko.value, osc


class QuantizedWeight:
    """A repacked weight matrix [n, k] held in HBM (syn_cuda_weight_upload).

    `data` is host bytes in the reference's storage format: for INT8_KN the
    int8 [k, n] GEMM layout with `scales` f32 [n]; for block formats the raw
    GGUF blocks of the row-major [n, k] matrix.
    """

    def __init__(self, ctx, fmt, data, n, k, scales=None):
        import numpy as np
        self.ctx, self.fmt, self.n, self.k = ctx, QFormat(fmt), int(n), int(k)
        buf = np.ascontiguousarray(np.asarray(data).view(np.uint8).reshape(-1))
        if buf.size < self.n * row_bytes(self.fmt, self.k):
            raise SynapseError(4, "QuantizedWeight")
        sc = None
        if scales is not None:
            sc = np.ascontiguousarray(np.asarray(scales, dtype=np.float32))
        h = ctypes.c_void_p()
        _check(lib().syn_cuda_weight_upload(
            ctx.handle, int(self.fmt), buf.ctypes.data_as(ctypes.c_void_p), self.n, self.k,
            sc.ctypes.data_as(ctypes.c_void_p) if sc is not None else None, ctypes.byref(h)),
            "weight_upload")
        self.handle = h

    @property
    def device_bytes(self):
        v = ctypes.c_size_t()
        _check(lib().syn_cuda_weight_bytes(self.handle, ctypes.byref(v)), "weight_bytes")
        return v.value

    @property
    def format_bytes(self):
        """Bytes of the weight in the reference's own format (roofline basis)."""
        extra = 4 * self.n if self.fmt == QFormat.INT8_KN else 0
        return self.n * row_bytes(self.fmt, self.k) + extra

    def dequant(self):
        import numpy as np
        out = np.empty((self.n, self.k), dtype=np.float32)
        _check(lib().syn_cuda_weight_dequant(self.handle, out.ctypes.data_as(ctypes.c_void_p)),
               "weight_dequant")
        return out

    def matmul(self, x, out=None):
        """y [m, n] = x [m, k] @ W^T (syn_cuda_qmatmul)."""
        _need_cuda(x)
        if x.dtype != torch.float32 or x.shape[-1] != self.k:
            raise SynapseError(4, "matmul")
        m = x.numel() // self.k
        if out is None:
            out = torch.empty(m, self.n, dtype=torch.float32, device=x.device)
        _check(lib().syn_cuda_qmatmul(self.ctx.handle, self.handle, _ptr(x), m, _ptr(out),
                                      _stream(x)), "qmatmul")
        return out

    def matmul_rmsnorm(self, residual, norm_weight, eps, delta=None, residual_out=None,
                       parallel_sum=False, out=None):
        """y [1, n] = rmsnorm(residual (+ delta)) @ W^T in one launch
        (syn_cuda_qmatmul_rmsnorm); residual_out receives residual + delta."""
        _need_cuda(residual, norm_weight)
        if out is None:
            out = torch.empty(1, self.n, dtype=torch.float32, device=residual.device)
        _check(lib().syn_cuda_qmatmul_rmsnorm(
            self.ctx.handle, self.handle, _ptr(residual), _ptr(delta), _ptr(norm_weight),
            float(eps), _ptr(residual_out), 1 if parallel_sum else 0, _ptr(out),
            _stream(residual)), "qmatmul_rmsnorm")
        return out

    def matmul_pre_quantized(self, x_int8, scales_x, m, out=None):
        _need_cuda(x_int8, scales_x)
        if out is None:
            out = torch.empty(m, self.n, dtype=torch.float32, device=x_int8.device)
        _check(lib().syn_cuda_qmatmul_int8_prequant(self.ctx.handle, self.handle, _ptr(x_int8),
                                                    _ptr(scales_x), m, _ptr(out),
                                                    _stream(x_int8)), "qmatmul_int8_prequant")
        return out

    def close(self):
        if self.handle:
            lib().syn_cuda_weight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QuantizedLinear:
    """Mirror of QuantizedLinear (int8_linear.rs:10-171) on the GPU.

    from_f32 quantises on the device with the reference's calibration and
    rounding, keeps the reference's [in, out] int8 layout plus [out] scales
    (for inspection / memory_bytes) and holds a repacked weight handle.
    """

    def __init__(self, ctx, weights_int8, scales, out_features, in_features):
        self.weights_int8 = weights_int8  # host numpy int8 [in*out]
        self.scales = scales              # host numpy f32 [out]
        self.out_features, self.in_features = out_features, in_features
        self.weight = QuantizedWeight(ctx, QFormat.INT8_KN, weights_int8, out_features,
                                      in_features, scales)

    @classmethod
    def from_f32(cls, ctx, weights, out_features, in_features):
        w = torch.as_tensor(weights, dtype=torch.float32).reshape(-1).to(f"cuda:{ctx.device}")
        q, s = quantize_weights_int8(w.contiguous(), out_features, in_features)
        return cls(ctx, q.cpu().numpy(), s.cpu().numpy(), out_features, in_features)

    def forward(self, x, m):
        if m == 0 or self.in_features == 0 or self.out_features == 0:
            return torch.zeros(m * self.out_features, dtype=torch.float32, device="cuda")
        return self.weight.matmul(x.reshape(m, self.in_features)).reshape(-1)

    def forward_pre_quantized(self, x_int8, scales_x, m):
        if m == 0:
            return torch.zeros(0, dtype=torch.float32, device="cuda")
        return self.weight.matmul_pre_quantized(x_int8, scales_x, m).reshape(-1)

    def memory_bytes(self):
        return self.weights_int8.size + 4 * self.scales.size


# ---------------------------------------------------------------------------
# Decoder-layer kernels (lm.cu) on torch CUDA tensors
# ---------------------------------------------------------------------------

def rope_tables(base, max_pos, head_dim):
    """precompute_rope_tables (models/lm/builder.rs:88-133): (cos, sin) numpy
    [max_pos, head_dim/2] computed on the host."""
    import numpy as np
    c = np.empty((max_pos, head_dim // 2), dtype=np.float32)
    s = np.empty_like(c)
    _check(lib().syn_cuda_rope_tables(float(base), max_pos, head_dim,
                                      c.ctypes.data_as(ctypes.c_void_p),
                                      s.ctypes.data_as(ctypes.c_void_p)), "rope_tables")
    return c, s


def rmsnorm(x, weight, eps, out=None):
    """rmsnorm (ops/norm.rs:8-37) over the last dimension."""
    _need_cuda(x, weight)
    h = weight.numel()
    out = torch.empty_like(x) if out is None else out
    _check(lib().syn_cuda_rmsnorm(_ptr(x), _ptr(weight), x.numel() // h, h, float(eps), _ptr(out),
                                  _stream(x)), "rmsnorm")
    return out


def add_rmsnorm(residual, delta, weight, eps, out=None):
    """residual += delta; returns rmsnorm(residual)."""
    _need_cuda(residual, delta, weight)
    h = weight.numel()
    out = torch.empty_like(residual) if out is None else out
    _check(lib().syn_cuda_add_rmsnorm(_ptr(residual), _ptr(delta), _ptr(weight),
                                      residual.numel() // h, h, float(eps), _ptr(out),
                                      _stream(residual)), "add_rmsnorm")
    return out


def swiglu(gate, up, variant=0):
    """variant 0: silu(g)*u (INT8 model); 1: syn_swiglu (f32 model)."""
    _need_cuda(gate, up)
    n = gate.shape[-1]
    rows = gate.numel() // n
    out = torch.empty_like(gate)
    _check(lib().syn_cuda_swiglu(_ptr(gate), _ptr(up), n, rows, n, int(variant), _ptr(out), n,
                                 _stream(gate)), "swiglu")
    return out


def argmax(logits):
    """Greedy argmax per row (generation/sampler.rs:217-224)."""
    _need_cuda(logits)
    n = logits.shape[-1]
    rows = logits.numel() // n
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    _check(lib().syn_cuda_argmax(_ptr(logits), rows, n, _ptr(out), _stream(logits)), "argmax")
    return out


class KVCache:
    """KV cache in HBM (syn_cuda_kvcache_*; kvcache.zig:13-170)."""

    def __init__(self, ctx, max_seq, n_kv_heads, head_dim, num_layers, batch=1, page=0,
                 n_pages=0):
        self.max_seq, self.n_kv, self.hd = max_seq, n_kv_heads, head_dim
        self.layers, self.batch = num_layers, batch
        h = ctypes.c_void_p()
        _check(lib().syn_cuda_kvcache_create_paged(ctx.handle, max_seq, n_kv_heads, head_dim,
                                                   num_layers, batch, page, n_pages,
                                                   ctypes.byref(h)),
               "kvcache_create")
        self.handle = h

    def pages_free(self):
        v = ctypes.c_size_t()
        _check(lib().syn_cuda_kvcache_pages_free(self.handle, ctypes.byref(v)), "pages_free")
        return v.value

    def length(self, seq=0):
        v = ctypes.c_size_t()
        _check(lib().syn_cuda_kvcache_len(self.handle, seq, ctypes.byref(v)), "kvcache_len")
        return v.value

    def view(self, layer, seq=0):
        """(K, V) torch views [max_seq, n_kv*hd] of one layer and sequence."""
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().syn_cuda_kvcache_view(self.handle, layer, seq, ctypes.byref(k),
                                           ctypes.byref(v)), "kvcache_view")
        n = self.max_seq * self.n_kv * self.hd
        return _wrap_device(k.value, n, (self.max_seq, self.n_kv * self.hd)), \
            _wrap_device(v.value, n, (self.max_seq, self.n_kv * self.hd))

    def append(self, layer, k, v, seq=0):
        _need_cuda(k, v)
        n = k.numel() // (self.n_kv * self.hd)
        _check(lib().syn_cuda_kvcache_append(self.handle, layer, seq, _ptr(k), _ptr(v), n,
                                             _stream(k)), "kvcache_append")

    def advance(self, n, seq=0):
        _check(lib().syn_cuda_kvcache_advance(self.handle, seq, n,
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "kvcache_advance")

    def truncate(self, new_len, seq=0):
        _check(lib().syn_cuda_kvcache_truncate(self.handle, seq, new_len,
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "kvcache_truncate")

    def reset(self, seq=0):
        _check(lib().syn_cuda_kvcache_reset(self.handle, seq,
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "kvcache_reset")

    def close(self):
        if self.handle:
            lib().syn_cuda_kvcache_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _wrap_device(addr, numel, shape):
    """A torch view of library-owned device memory (no copy, no ownership)."""
    class _Iface:
        pass
    it = _Iface()
    it.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<f4", "data": (addr, False),
                                   "version": 3, "strides": None}
    return torch.as_tensor(it, device="cuda").view(*shape)


def attention_decode(cache, layer, qkv, n_heads, q_norm, k_norm, eps, cos_t, sin_t, window=0,
                     batch=1, flash=False):
    """cached_attention_decode (ops/attention.rs:24-147) for sequences
    [0, batch); qkv rows [q | k | v] (row stride = its last dim). Returns
    [batch, n_heads*hd]; the cache length is not advanced."""
    _need_cuda(qkv, cos_t, sin_t)
    ld = qkv.shape[-1]
    qd, kvd = n_heads * cache.hd, cache.n_kv * cache.hd
    out = torch.empty(batch, qd, dtype=torch.float32, device=qkv.device)
    base = qkv.data_ptr()
    fn = lib().syn_cuda_attention_decode_flash if flash else lib().syn_cuda_attention_decode
    _check(fn(
        cache.handle, layer, batch, ctypes.c_void_p(base), ctypes.c_void_p(base + 4 * qd),
        ctypes.c_void_p(base + 4 * (qd + kvd)), ld, n_heads, _ptr(q_norm), _ptr(k_norm),
        float(eps), _ptr(cos_t), _ptr(sin_t), window, _ptr(out), qd, _stream(qkv)),
        "attention_decode")
    return out


def attention_prefill(cache, layer, qkv, n_heads, q_norm, k_norm, eps, cos_t, sin_t, seq=0,
                      flash=False):
    """cached_attention_prefill (ops/attention.rs:153-247) for sequence
    `seq`; qkv [n_tokens, q | k | v] (q rewritten in place). Returns
    [n_tokens, n_heads*hd]; the cache length is not advanced."""
    _need_cuda(qkv, cos_t, sin_t)
    ld = qkv.shape[-1]
    n = qkv.numel() // ld
    qd, kvd = n_heads * cache.hd, cache.n_kv * cache.hd
    out = torch.empty(n, qd, dtype=torch.float32, device=qkv.device)
    base = qkv.data_ptr()
    fn = lib().syn_cuda_attention_prefill_flash if flash else lib().syn_cuda_attention_prefill
    _check(fn(
        cache.handle, layer, seq, n, ctypes.c_void_p(base), ctypes.c_void_p(base + 4 * qd),
        ctypes.c_void_p(base + 4 * (qd + kvd)), ld, n_heads, _ptr(q_norm), _ptr(k_norm),
        float(eps), _ptr(cos_t), _ptr(sin_t), _ptr(out), qd, _stream(qkv)), "attention_prefill")
    return out


# ---------------------------------------------------------------------------
# Model runner (runner.cu): QuantizedCausalLM / CausalLM on the GPU
# ---------------------------------------------------------------------------

class Model:
    """Decoder-only LM on the GPU (syn_cuda_model_*), mirroring
    QuantizedCausalLM (quantization/lm/int8.rs:171-709) for INT8 weights and
    CausalLM (models/lm/causal_lm.rs:195-280) for the block formats.

    config: the reference's model config (dict or JSON text). weights: name ->
    numpy f32 array (norms, embedding) or a linear spec
    ("INT8_KN", q_kn int8 [K*N], scales [N]) / (fmt_name, block bytes).
    """

    def __init__(self, ctx, config, weights, max_seq, max_batch=1, cache_dir=None, _stage=None,
                 kv_page=0, kv_pages=0):
        import json
        import numpy as np
        cfg = json.loads(config) if isinstance(config, str) else config
        self.ctx = ctx
        self.cfg = cfg
        a, at = cfg["architecture"], cfg["attention"]
        self.vocab = a["vocab_size"]
        self.max_seq, self.max_batch = max_seq, max_batch
        h = ctypes.c_void_p()
        _check(lib().syn_cuda_model_create(ctx.handle, json.dumps(cfg).encode(), max_seq,
                                           max_batch, ctypes.byref(h)), "model_create")
        self.handle = h
        if kv_page:
            _check(lib().syn_cuda_model_set_kv_paging(h, kv_page, kv_pages), "set_kv_paging")
        if cache_dir:
            _check(lib().syn_cuda_model_set_cache_dir(h, str(cache_dir).encode()),
                   "model_set_cache_dir")
        if _stage is not None:
            _stage(h)
            weights = {}
        hd = at["head_dim"]
        qd, kvd = at["num_heads"] * hd, at["num_kv_heads"] * hd
        hid, ff = a["hidden_size"], cfg["ffn"]["intermediate_size"]
        shapes = {"q_proj": (qd, hid), "k_proj": (kvd, hid), "v_proj": (kvd, hid),
                  "o_proj": (hid, qd), "gate_proj": (ff, hid), "up_proj": (ff, hid),
                  "down_proj": (hid, ff)}
        for name, val in weights.items():
            if isinstance(val, tuple):
                if name == "lm_head.weight":
                    n, k = self.vocab, hid
                else:
                    n, k = shapes[name.split(".")[-2]]
                fmt = QFormat[val[0]] if isinstance(val[0], str) else QFormat(val[0])
                buf = np.ascontiguousarray(np.asarray(val[1]).view(np.uint8).reshape(-1))
                sc = None
                if fmt == QFormat.INT8_KN:
                    sc = np.ascontiguousarray(np.asarray(val[2], dtype=np.float32))
                _check(lib().syn_cuda_model_set_linear(
                    self.handle, name.encode(), int(fmt), buf.ctypes.data_as(ctypes.c_void_p), n,
                    k, sc.ctypes.data_as(ctypes.c_void_p) if sc is not None else None),
                    "model_set_linear " + name)
            else:
                arr = np.ascontiguousarray(np.asarray(val, dtype=np.float32).reshape(-1))
                _check(lib().syn_cuda_model_set_tensor(self.handle, name.encode(),
                                                       arr.ctypes.data_as(ctypes.c_void_p),
                                                       arr.size), "model_set_tensor " + name)
        _check(lib().syn_cuda_model_finalize(self.handle), "model_finalize")

    @classmethod
    def from_gguf(cls, ctx, path, max_seq, max_batch=1, cache_dir=None, config=None):
        """A model from a GGUF file (syn_cuda_model_load_gguf): config from
        its metadata unless given; quantised blocks go to the repacker as
        they are; cache_dir keeps the repacked weights between loads."""
        g = GGUFFile(path)
        try:
            cfg = config if config is not None else g.config()
            return cls(ctx, cfg, None, max_seq, max_batch, cache_dir=cache_dir,
                       _stage=lambda h: _check(lib().syn_cuda_model_load_gguf(h, g.handle),
                                               "model_load_gguf"))
        finally:
            g.close()

    @classmethod
    def from_safetensors(cls, ctx, path, config, max_seq, max_batch=1, cache_dir=None):
        """The reference's --quantize load of a safetensors checkpoint
        (syn_cuda_model_load_safetensors): linears quantised to INT8 on the
        device from f32 / f16 / bf16."""
        f = SafetensorsFile(path)
        try:
            return cls(ctx, config, None, max_seq, max_batch, cache_dir=cache_dir,
                       _stage=lambda h: _check(lib().syn_cuda_model_load_safetensors(h, f.handle),
                                               "model_load_safetensors"))
        finally:
            f.close()

    def cache_hits(self):
        v = ctypes.c_int()
        _check(lib().syn_cuda_model_cache_hits(self.handle, ctypes.byref(v)), "model_cache_hits")
        return v.value

    def forward_prefill(self, token_ids, seq=0, want_logits=True):
        """Prefill of an empty sequence; returns (greedy next token, logits or None)."""
        import numpy as np
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int32))
        nxt = ctypes.c_int32()
        logits = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        _check(lib().syn_cuda_prefill(self.handle, seq, ids.ctypes.data_as(ctypes.c_void_p),
                                      ids.size,
                                      logits.ctypes.data_as(ctypes.c_void_p) if want_logits else None,
                                      ctypes.byref(nxt)), "prefill")
        return nxt.value, logits

    def forward_one(self, tokens, want_logits=True):
        """One decode step of sequences [0, len(tokens)); returns (greedy
        tokens, logits [batch, vocab] or None)."""
        import numpy as np
        ids = np.ascontiguousarray(np.atleast_1d(np.asarray(tokens, dtype=np.int32)))
        b = ids.size
        out = np.empty(b, dtype=np.int32)
        logits = np.empty((b, self.vocab), dtype=np.float32) if want_logits else None
        _check(lib().syn_cuda_decode_step(self.handle, b, ids.ctypes.data_as(ctypes.c_void_p),
                                          out.ctypes.data_as(ctypes.c_void_p),
                                          logits.ctypes.data_as(ctypes.c_void_p) if want_logits
                                          else None), "decode_step")
        return out, logits

    def generate_greedy(self, prompt, steps, seq=0):
        """generation/pipeline.rs:197-280 with GreedySampler (single sequence)."""
        tok, _ = self.forward_prefill(prompt, seq, want_logits=False)
        toks = [tok]
        while len(toks) < steps:
            nxt, _ = self.forward_one([toks[-1]], want_logits=False)
            toks.append(int(nxt[0]))
        return toks

    def generate(self, n_steps, batch=1):
        """n_steps greedy tokens for sequences [0, batch), chained on the
        device (syn_cuda_generate); returns int32 [batch, n_steps]."""
        import numpy as np
        out = np.empty((batch, n_steps), dtype=np.int32)
        _check(lib().syn_cuda_generate(self.handle, batch, n_steps,
                                       out.ctypes.data_as(ctypes.c_void_p)), "generate")
        return out

    def decode_slots(self, slots, tokens, want_logits=False):
        """One decode step of the started sequences `slots` (any subset, in
        any order; syn_cuda_decode_step_slots): (greedy tokens, logits
        [n, vocab] or None)."""
        import numpy as np
        sl = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.empty(sl.size, dtype=np.int32)
        logits = np.empty((sl.size, self.vocab), dtype=np.float32) if want_logits else None
        _check(lib().syn_cuda_decode_step_slots(
            self.handle, sl.size, sl.ctypes.data_as(ctypes.c_void_p),
            ids.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
            logits.ctypes.data_as(ctypes.c_void_p) if want_logits else None), "decode_step_slots")
        return out, logits

    def kv_pages_free(self):
        v = ctypes.c_size_t()
        _check(lib().syn_cuda_model_kv_pages_free(self.handle, ctypes.byref(v)), "kv_pages_free")
        return v.value

    def decode_span(self, tokens, seq=0, n_layers=0, want_logits=False):
        """Tokens at the next positions of `seq` (syn_cuda_decode_span):
        (greedy token per row, logits [n, vocab] or None); the cache length
        is not advanced."""
        import numpy as np
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.empty(ids.size, dtype=np.int32)
        logits = np.empty((ids.size, self.vocab), dtype=np.float32) if want_logits else None
        _check(lib().syn_cuda_decode_span(self.handle, seq, ids.ctypes.data_as(ctypes.c_void_p),
                                          ids.size, n_layers, out.ctypes.data_as(ctypes.c_void_p),
                                          logits.ctypes.data_as(ctypes.c_void_p)
                                          if want_logits else None), "decode_span")
        return out, logits

    def generate_speculative(self, prompt, steps, k=4, draft_layers=None, seq=0):
        """Greedy generation with self-speculative decoding
        (syn_cuda_generate_speculative): returns (tokens, drafted, accepted);
        tokens[0] comes from the prefill, as in generate_greedy."""
        import numpy as np
        if draft_layers is None:
            draft_layers = max(1, self.cfg["architecture"]["num_layers"] // 4)
        tok, _ = self.forward_prefill(prompt, seq, want_logits=False)
        out = np.empty(max(0, steps - 1), dtype=np.int32)
        nd, na = ctypes.c_size_t(), ctypes.c_size_t()
        if steps > 1:
            _check(lib().syn_cuda_generate_speculative(
                self.handle, seq, tok, steps - 1, k, draft_layers,
                out.ctypes.data_as(ctypes.c_void_p), ctypes.byref(nd), ctypes.byref(na)),
                "generate_speculative")
        return [tok] + out.tolist(), nd.value, na.value

    def seq_len(self, seq=0):
        v = ctypes.c_size_t()
        _check(lib().syn_cuda_model_seq_len(self.handle, seq, ctypes.byref(v)), "model_seq_len")
        return v.value

    def reset(self, seq=0):
        _check(lib().syn_cuda_model_reset(self.handle, seq), "model_reset")

    def truncate(self, new_len, seq=0):
        _check(lib().syn_cuda_model_truncate(self.handle, seq, new_len), "model_truncate")

    def close(self):
        if self.handle:
            lib().syn_cuda_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GGUFFile:
    """A memory-mapped GGUF v2/v3 file (syn_gguf_*): tensor infos with the
    raw bytes, scalar metadata, and the model config built from them."""

    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(lib().syn_gguf_open(str(path).encode(), ctypes.byref(h)), "gguf_open")
        self.handle = h

    def tensors(self):
        """[(name, ggml_type, dims (ne0 first), bytes)] -- bytes copied out."""
        n = ctypes.c_size_t()
        _check(lib().syn_gguf_tensor_count(self.handle, ctypes.byref(n)), "gguf_tensor_count")
        out = []
        for i in range(n.value):
            name, typ, nd = ctypes.c_char_p(), ctypes.c_uint32(), ctypes.c_size_t()
            dims = (ctypes.c_uint64 * 4)()
            data, nb = ctypes.c_void_p(), ctypes.c_size_t()
            _check(lib().syn_gguf_tensor_info(self.handle, i, ctypes.byref(name), ctypes.byref(typ),
                                              ctypes.byref(nd), dims, ctypes.byref(data),
                                              ctypes.byref(nb)), "gguf_tensor_info")
            raw = ctypes.string_at(data.value, nb.value) if nb.value else b""
            out.append((name.value.decode(), typ.value, list(dims[:nd.value]), raw))
        return out

    def meta_num(self, key):
        v = ctypes.c_double()
        _check(lib().syn_gguf_meta_num(self.handle, key.encode(), ctypes.byref(v)), "gguf_meta_num")
        return v.value

    def meta_str(self, key):
        v = ctypes.c_char_p()
        _check(lib().syn_gguf_meta_str(self.handle, key.encode(), ctypes.byref(v)), "gguf_meta_str")
        return v.value.decode()

    def config(self):
        import json
        need = ctypes.c_size_t()
        _check(lib().syn_gguf_config_json(self.handle, None, 0, ctypes.byref(need)), "gguf_config")
        buf = ctypes.create_string_buffer(need.value)
        _check(lib().syn_gguf_config_json(self.handle, buf, need.value, ctypes.byref(need)),
               "gguf_config")
        return json.loads(buf.value.decode())

    def close(self):
        if getattr(self, "handle", None):
            lib().syn_gguf_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gguf_runner_name(name):
    """llama.cpp tensor name -> the runner's name (None if unmapped)."""
    buf = ctypes.create_string_buffer(512)
    st = lib().syn_gguf_runner_name(name.encode(), buf, 512)
    return buf.value.decode() if st == 0 else None


class SafetensorsFile:
    """A memory-mapped safetensors file (syn_safetensors_*)."""

    DTYPES = {0: "F32", 1: "F16", 2: "BF16", 3: "I64", 4: "I32", 5: "U8"}

    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(lib().syn_safetensors_open(str(path).encode(), ctypes.byref(h)), "safetensors_open")
        self.handle = h

    def tensors(self):
        """{name: (dtype name, shape, f32 numpy array as the loader converts it)}"""
        import numpy as np
        n = ctypes.c_size_t()
        _check(lib().syn_safetensors_tensor_count(self.handle, ctypes.byref(n)), "st_count")
        out = {}
        for i in range(n.value):
            name, dt, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_size_t()
            dims = (ctypes.c_uint64 * 4)()
            data, nb = ctypes.c_void_p(), ctypes.c_size_t()
            _check(lib().syn_safetensors_tensor_info(self.handle, i, ctypes.byref(name),
                                                     ctypes.byref(dt), ctypes.byref(nd), dims,
                                                     ctypes.byref(data), ctypes.byref(nb)),
                   "st_info")
            shape = list(dims[:nd.value])
            cnt = int(np.prod(shape)) if shape else 1
            arr = np.empty(cnt, np.float32)
            _check(lib().syn_convert_to_f32(dt.value, data, cnt, arr.ctypes.data_as(ctypes.c_void_p)),
                   "convert_to_f32")
            out[name.value.decode()] = (self.DTYPES[dt.value], shape, arr.reshape(shape))
        return out

    def close(self):
        if getattr(self, "handle", None):
            lib().syn_safetensors_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def quantize_weights_int8_half(bits, dtype, out_features, in_features):
    """f16 / bf16 weight bits (device uint16/int16 tensor [N, K]) -> (int8
    [K, N], f32 scales [N]) on the device (syn_cuda_quantize_weights_int8_half),
    bit-exact with the reference's load-and-quantize route."""
    _need_cuda(bits)
    dt = {"F16": 1, "BF16": 2}[dtype]
    q = torch.empty(in_features * out_features, dtype=torch.int8, device=bits.device)
    s = torch.empty(out_features, dtype=torch.float32, device=bits.device)
    _check(lib().syn_cuda_quantize_weights_int8_half(_ptr(bits), dt, out_features, in_features,
                                                     _ptr(q), _ptr(s), _stream(bits)),
           "quantize_weights_int8_half")
    return q, s
