"""ctypes wrapper of the CPU oracle (liboracle.so, built from synapse_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py as the checker. The shipped CUDA path never
imports it. Parity status: partially pinned (see synapse_oracle.h).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
FMT = {"INT8_KN": 0, "Q4_0": 1, "Q8_0": 2, "Q4_K": 3, "Q6_K": 4}
_LIBS = {}


def build():
    subprocess.check_call(["make", "-s", "-C", HERE])


def _load(fast=False):
    name = "liboracle_fast.so" if fast else "liboracle.so"
    if name not in _LIBS:
        path = os.path.join(HERE, name)
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        lib.orc_f16_zig.restype = ctypes.c_float
        lib.orc_f16_zig.argtypes = [ctypes.c_uint16]
        lib.orc_f16_rust.restype = ctypes.c_float
        lib.orc_f16_rust.argtypes = [ctypes.c_uint16]
        lib.orc_quantize_per_channel_int8.argtypes = [vp, sz, sz, vp, vp]
        lib.orc_quantize_weights_int8.argtypes = [vp, sz, sz, vp, vp]
        lib.orc_qgemm_int8.argtypes = [sz, sz, sz, vp, sz, vp, sz, vp, sz, vp, vp]
        lib.orc_naive_int8_gemm.argtypes = [sz, sz, sz, vp, sz, vp, sz, vp, sz, vp, vp]
        lib.orc_q4_0_gemv.argtypes = [sz, sz, vp, vp, vp]
        lib.orc_dequant.argtypes = [ctypes.c_int, vp, sz, vp]
        lib.orc_sgemm_nt.argtypes = [sz, sz, sz, vp, sz, vp, sz, vp, sz]
        lib.orc_block_matmul.argtypes = [ctypes.c_int, sz, sz, sz, vp, vp, vp, vp]
        f32 = ctypes.c_float
        lib.orc_exp.restype = f32
        lib.orc_exp.argtypes = [f32]
        lib.orc_rmsnorm.argtypes = [vp, vp, sz, sz, f32, vp]
        lib.orc_rope_tables.argtypes = [ctypes.c_double, sz, sz, vp, vp]
        lib.orc_rope_inplace.argtypes = [vp, vp, vp, sz, sz, sz, sz]
        lib.orc_softmax.argtypes = [vp, sz]
        lib.orc_sgemm_nn.argtypes = [sz, sz, sz, vp, sz, vp, sz, vp, sz]
        lib.orc_attention_decode.argtypes = [vp, vp, vp, sz, sz, sz, sz, sz, vp]
        lib.orc_fused_attention.argtypes = [sz, sz, sz, vp, vp, vp, vp]
        lib.orc_silu_mul.argtypes = [vp, vp, sz, vp]
        lib.orc_swiglu.argtypes = [vp, vp, sz, vp]
        lib.orc_argmax.restype = ctypes.c_uint32
        lib.orc_argmax.argtypes = [vp, sz]
        _LIBS[name] = lib
    return _LIBS[name]


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def f16_zig(bits):
    return _load().orc_f16_zig(int(bits))


def f16_rust(bits):
    return _load().orc_f16_rust(int(bits))


def quantize_per_channel_int8(x, channels, channel_size):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(channels * channel_size, dtype=np.int8)
    scales = np.empty(channels, dtype=np.float32)
    st = _load().orc_quantize_per_channel_int8(_p(x), channels, channel_size, _p(out),
                                               _p(scales))
    return st, out, scales


def quantize_weights_int8(w, n, k):
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty(k * n, dtype=np.int8)
    scales = np.empty(n, dtype=np.float32)
    _load().orc_quantize_weights_int8(_p(w), n, k, _p(out), _p(scales))
    return out, scales


def qgemm_int8(m, n, k, a, b, sa, sb, fast=False):
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    sa = np.ascontiguousarray(sa, dtype=np.float32)
    sb = np.ascontiguousarray(sb, dtype=np.float32)
    c = np.zeros(m * n, dtype=np.float32)
    st = _load(fast).orc_qgemm_int8(m, n, k, _p(a), k, _p(b), n, _p(c), n, _p(sa), _p(sb))
    return st, c


def naive_int8_gemm(m, n, k, a, b, sa, sb):
    c = np.zeros(m * n, dtype=np.float32)
    _load().orc_naive_int8_gemm(m, n, k, _p(np.ascontiguousarray(a, np.int8)), k,
                                _p(np.ascontiguousarray(b, np.int8)), n, _p(c), n,
                                _p(np.ascontiguousarray(sa, np.float32)),
                                _p(np.ascontiguousarray(sb, np.float32)))
    return c


def q4_0_gemv(n, k, a, b_q4, fast=False):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b_q4, dtype=np.uint8)
    c = np.zeros(n, dtype=np.float32)
    st = _load(fast).orc_q4_0_gemv(n, k, _p(a), _p(b), _p(c))
    return st, c


def dequant(fmt, blocks, numel):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(numel, dtype=np.float32)
    st = _load().orc_dequant(FMT[fmt] if isinstance(fmt, str) else int(fmt), _p(blocks), numel,
                             _p(out))
    return st, out


def sgemm_nt(m, n, k, a, b, fast=False):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    c = np.empty(m * n, dtype=np.float32)
    st = _load(fast).orc_sgemm_nt(m, n, k, _p(a), k, _p(b), k, _p(c), n)
    return st, c


def block_matmul(fmt, m, n, k, x, blocks):
    """The reference's LM route for a block format: dequant to f32, matmul_t."""
    st, w = dequant(fmt, blocks, n * k)
    if st:
        return st, None
    return sgemm_nt(m, n, k, x, w)


# ---- language-model epilogues (synapse_oracle_lm.c) ----------------------

def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def exp32(x):
    return _load().orc_exp(float(x))


def rmsnorm(x, w, h, eps, fast=True):
    x = _f32(x)
    out = np.empty_like(x)
    _load(fast).orc_rmsnorm(_p(x), _p(_f32(w)), x.size // h, h, eps, _p(out))
    return out


def rope_tables(base, max_pos, hd):
    c = np.empty(max_pos * (hd // 2), dtype=np.float32)
    s = np.empty_like(c)
    _load().orc_rope_tables(float(base), max_pos, hd, _p(c), _p(s))
    return c, s


def rope_inplace(qk, cos_t, sin_t, seq, heads, hd, pos_off, fast=True):
    assert qk.dtype == np.float32 and qk.flags.c_contiguous
    _load(fast).orc_rope_inplace(_p(qk), _p(cos_t), _p(sin_t), seq, heads, hd, pos_off)


def softmax(x):
    x = _f32(x).copy()
    _load().orc_softmax(_p(x), x.size)
    return x


def sgemm_nn(m, n, k, a, b, fast=False):
    a, b = _f32(a), _f32(b)
    c = np.empty(m * n, dtype=np.float32)
    st = _load(fast).orc_sgemm_nn(m, n, k, _p(a), k, _p(b), n, _p(c), n)
    return st, c


def attention_decode(q, kc, vc, length, n_heads, n_kv, hd, window=0, fast=True):
    q, kc, vc = _f32(q), _f32(kc), _f32(vc)
    out = np.empty(n_heads * hd, dtype=np.float32)
    _load(fast).orc_attention_decode(_p(q), _p(kc), _p(vc), length, n_heads, n_kv, hd,
                                     window, _p(out))
    return out


def fused_attention(seq_q, seq_k, hd, q, k, v, fast=True):
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(seq_q * hd, dtype=np.float32)
    st = _load(fast).orc_fused_attention(seq_q, seq_k, hd, _p(q), _p(k), _p(v), _p(out))
    return st, out


def silu_mul(g, u):
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    _load().orc_silu_mul(_p(g), _p(u), g.size, _p(out))
    return out


def swiglu(g, u):
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    _load().orc_swiglu(_p(g), _p(u), g.size, _p(out))
    return out


def argmax(x):
    x = _f32(x)
    return int(_load().orc_argmax(_p(x), x.size))
