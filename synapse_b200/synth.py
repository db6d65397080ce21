"""Seeded synthetic inputs with the shapes and value distributions of the
quantized-matmul sweep (weights in every format, f32 activations).

Distributions: quant codes uniform over each format's code range; f16 block
scales |N(0, 0.01)| rounded to nearest f16; INT8 per-row scales |N(0, 0.01)|
as f32; activations N(0, 1). All draws use numpy PCG64.
"""
import numpy as np

from .api import QFormat, row_bytes

SWEEP_N = (1024, 3072, 4096, 11008, 14336)
SWEEP_K = (1024, 2048, 4096)
SWEEP_M = (1, 16, 128, 512)
FORMATS = (QFormat.INT8_KN, QFormat.Q4_0, QFormat.Q8_0, QFormat.Q4_K, QFormat.Q6_K)


def _f16_bits(rng, count, sigma=0.01):
    return np.abs(rng.normal(0.0, sigma, count)).astype(np.float16).view(np.uint16)


def gen_weight(fmt, n, k, rng):
    """Returns (data, scales): the reference's storage bytes of an [n, k]
    weight (INT8_KN: int8 [k, n] + f32 scales [n]; block formats: raw
    blocks as uint8, scales None)."""
    fmt = QFormat(fmt)
    if fmt == QFormat.INT8_KN:
        q = rng.integers(-127, 128, size=(k, n), dtype=np.int8)
        s = np.abs(rng.normal(0.0, 0.01, n)).astype(np.float32)
        return q, s
    nb = n * row_bytes(fmt, k)
    if fmt == QFormat.Q4_0:
        blk = np.empty((nb // 18, 18), dtype=np.uint8)
        blk[:, 0:2] = _f16_bits(rng, nb // 18).view(np.uint8).reshape(-1, 2)
        blk[:, 2:] = rng.integers(0, 256, size=(nb // 18, 16), dtype=np.uint8)
    elif fmt == QFormat.Q8_0:
        blk = np.empty((nb // 34, 34), dtype=np.uint8)
        blk[:, 0:2] = _f16_bits(rng, nb // 34).view(np.uint8).reshape(-1, 2)
        blk[:, 2:] = rng.integers(-127, 128, size=(nb // 34, 32), dtype=np.int8).view(np.uint8)
    elif fmt == QFormat.Q4_K:
        cnt = nb // 144
        blk = np.empty((cnt, 144), dtype=np.uint8)
        blk[:, 0:2] = _f16_bits(rng, cnt).view(np.uint8).reshape(-1, 2)
        blk[:, 2:4] = _f16_bits(rng, cnt).view(np.uint8).reshape(-1, 2)
        blk[:, 4:] = rng.integers(0, 256, size=(cnt, 140), dtype=np.uint8)
    elif fmt == QFormat.Q6_K:
        cnt = nb // 210
        blk = np.empty((cnt, 210), dtype=np.uint8)
        blk[:, 0:208] = rng.integers(0, 256, size=(cnt, 208), dtype=np.uint8)
        blk[:, 208:210] = _f16_bits(rng, cnt).view(np.uint8).reshape(-1, 2)
    return blk.reshape(-1), None


def gen_activations(m, k, rng):
    return rng.normal(0.0, 1.0, size=(m, k)).astype(np.float32)


def format_bytes(fmt, n, k):
    """Algorithmic weight bytes of one [n, k] matrix in its reference format."""
    fmt = QFormat(fmt)
    return n * row_bytes(fmt, k) + (4 * n if fmt == QFormat.INT8_KN else 0)
