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
