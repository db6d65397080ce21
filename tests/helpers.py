"""Test helpers: the reference tests' deterministic generators and metrics."""
import numpy as np


def lcg_fill(count, seed, scale=1.0):
    """fillData / fillRandom of zig/tests/test_qmatmul.zig:16-24 and
    zig/tests/test_quantize.zig:17-25: s = s*1103515245 + 12345 (u32),
    value = i16(s >> 16 as i32) / 32768 * range."""
    out = np.empty(count, dtype=np.float32)
    s = seed & 0xFFFFFFFF
    for i in range(count):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        bits = s - (1 << 32) if s >= (1 << 31) else s
        sh = (bits >> 16) & 0xFFFF
        sh = sh - 0x10000 if sh >= 0x8000 else sh
        out[i] = np.float32(np.float32(sh) / np.float32(32768.0)) * np.float32(scale)
    return out


def xorshift_vec(count, seed):
    """pseudo_random_vec of int8_linear.rs:216-230: xorshift64, then
    (state as f32 / u64::MAX as f32) * 2 - 1."""
    out = np.empty(count, dtype=np.float32)
    st = seed & 0xFFFFFFFFFFFFFFFF
    umax = np.float32(18446744073709551615.0)
    for i in range(count):
        st ^= (st << 13) & 0xFFFFFFFFFFFFFFFF
        st ^= st >> 7
        st ^= (st << 17) & 0xFFFFFFFFFFFFFFFF
        out[i] = np.float32(np.float32(np.float32(st) / umax) * np.float32(2.0) - np.float32(1.0))
    return out


def quantize_per_column_int8(data, rows, cols):
    """quantizePerColumnInt8 (zig/src/ops/quantize.zig:52-86), used by the
    reference's qmatmul test to build B."""
    d = np.asarray(data, dtype=np.float32).reshape(rows, cols)
    sc = np.abs(d).max(axis=0).astype(np.float32)
    sc = np.where(sc == 0, np.float32(1.0), (sc / np.float32(127.0)).astype(np.float32))
    inv = (np.float32(127.0) / (sc * np.float32(127.0)).astype(np.float32)).astype(np.float32)
    scaled = (d * inv[None, :]).astype(np.float32)
    r = np.clip(np.sign(scaled) * np.floor(np.abs(scaled) + 0.5), -127, 127)
    return r.astype(np.int8).reshape(-1), sc.astype(np.float32)


def frobenius_rel(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.sum(ref * ref)
    return 0.0 if den == 0 else float(np.sqrt(np.sum((a - ref) ** 2) / den))


def max_rel_err(y, ref):
    """Normwise max relative error: max|y - ref| / max|ref| (the 1e-3 bar for
    f32-accumulated matmul outputs)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(y - ref)) / den) if den > 0 else float(np.max(np.abs(y)))
