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


# ---------------------------------------------------------------------------
# Weight-file writers (the layouts the reference's loaders read)
# ---------------------------------------------------------------------------
GGUF_TYPES = {"F32": 0, "F16": 1, "Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14}


def _gguf_str(s):
    b = s.encode()
    return len(b).to_bytes(8, "little") + b


def gguf_bytes(tensors, meta=(), version=3, alignment=32):
    """A GGUF file as make_gguf_raw (weight_loading/gguf.rs:768-789) builds
    one, generalised: tensors = [(name, ggml_type, dims ne0-first, raw
    bytes)], meta = [(key, value)] with int -> u32, float -> f32, str ->
    string, list of str -> array of strings. Tensor data is aligned to
    `alignment` inside the data section."""
    import struct
    out = bytearray()
    out += struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(meta))
    for k, v in meta:
        out += _gguf_str(k)
        if isinstance(v, bool):
            out += struct.pack("<IB", 7, int(v))
        elif isinstance(v, int):
            out += struct.pack("<II", 4, v)
        elif isinstance(v, float):
            out += struct.pack("<If", 6, v)
        elif isinstance(v, str):
            out += struct.pack("<I", 8) + _gguf_str(v)
        else:
            out += struct.pack("<IIQ", 9, 8, len(v)) + b"".join(_gguf_str(x) for x in v)
    offs, off = [], 0
    for name, typ, dims, raw in tensors:
        offs.append(off)
        off = (off + len(raw) + alignment - 1) // alignment * alignment
    for (name, typ, dims, raw), o in zip(tensors, offs):
        out += _gguf_str(name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", typ, o)
    out += b"\0" * ((-len(out)) % alignment)
    data = bytearray()
    for (name, typ, dims, raw), o in zip(tensors, offs):
        data += b"\0" * (o - len(data))
        data += raw
    return bytes(out + data)


def safetensors_bytes(tensors, metadata=None):
    """tensors = [(name, dtype, shape, raw bytes)] -> safetensors file bytes
    (make_safetensors, weight_loading/safetensors.rs:310-342)."""
    import json
    import struct
    header, data = {}, bytearray()
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape),
                        "data_offsets": [len(data), len(data) + len(raw)]}
        data += raw
    h = json.dumps(header).encode()
    return struct.pack("<Q", len(h)) + h + bytes(data)
