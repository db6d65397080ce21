"""Seeded synthetic inputs with the shapes and value distributions of the
quantized-matmul sweep (weights in every format, f32 activations).

Distributions: quant codes uniform over each format's code range; f16 block
scales |N(0, 0.01)| rounded to nearest f16; INT8 per-row scales |N(0, 0.01)|
as f32; activations N(0, 1). All draws use numpy PCG64.
"""
import numpy as np

from .formats import QFormat, row_bytes

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


# ---------------------------------------------------------------------------
# Random-init language models with the shapes of the benchmark configs
# ---------------------------------------------------------------------------

def lm_config(name):
    """Model configs in the reference's JSON schema (configs/*.json) with the
    shapes of the benchmark configs: qwen3-0.6b (head_dim 128, as the real
    checkpoint), llama-3.2-1b, mistral-7b (vocab 32000, RoPE base 1e6, sliding
    window 4096), and small test shapes."""
    def cfg(h, L, V, hq, hkv, hd, ff, eps, base, window=0):
        att = {"type": "SlidingWindow" if window else "GQA", "num_heads": hq,
               "num_kv_heads": hkv, "head_dim": hd}
        if window:
            att["window_size"] = window
        return {"name": name,
                "architecture": {"hidden_size": h, "num_layers": L, "vocab_size": V,
                                 "max_sequence_length": 32768, "tie_word_embeddings": True},
                "attention": att, "norm": {"type": "RMSNorm", "eps": eps},
                "ffn": {"type": "SwiGLU", "intermediate_size": ff},
                "position": {"type": "RoPE", "base": base, "max_position_embeddings": 32768},
                "quantization": {"type": "F32"}}
    table = {
        "qwen3-0.6b": cfg(1024, 28, 151936, 16, 8, 128, 3072, 1e-6, 1e6),
        "llama-3.2-1b": cfg(2048, 16, 128256, 32, 8, 64, 8192, 1e-5, 5e5),
        "mistral-7b": cfg(4096, 32, 32000, 32, 8, 128, 14336, 1e-5, 1e6, window=4096),
        # test shapes
        "tiny": cfg(128, 2, 512, 4, 2, 32, 256, 1e-6, 1e6),
        "tiny-hd64": cfg(256, 2, 640, 4, 1, 64, 512, 1e-5, 5e5),
        "tiny-window": cfg(256, 2, 640, 8, 2, 32, 512, 1e-5, 1e6, window=24),
        "tiny-k-tp": cfg(256, 2, 640, 8, 2, 64, 512, 1e-5, 5e5),
    }
    return table[name]


def quantize_rows_int8(w):
    """Per-output-row INT8 weight quantisation (MinMaxCalibration +
    QuantizedLinear::from_f32_with_scales, int8_linear.rs:21-70): scale =
    max|row|/127 (1 for a zero row), q = clamp(round(w * (1/scale)), -128,
    127) with round half away from zero; returns (q [K, N], scales [N])."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.abs(w).max(axis=1)
    scale = np.where(amax == 0, np.float32(1.0), amax / np.float32(127.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    x = (w * inv[:, None]).astype(np.float32).astype(np.float64)
    r = np.sign(x) * np.floor(np.abs(x) + 0.5)
    q = np.clip(r, -128, 127).astype(np.int8)
    q[amax == 0] = 0
    return np.ascontiguousarray(q.T), scale


def gen_lm_weights(cfg, fmt, seed=1234, dequant=None, qk_norm=None):
    """Random-init weights of a decoder-only LM in the runner's naming.

    INT8_KN: every linear is N(0, 0.02) f32 quantised per output row; the tied
    LM head is quantised from the N(0, 0.02) embedding. Block formats: random
    blocks as in the matmul sweep for every linear including the LM head,
    and the embedding is the dequantised LM head (`dequant(fmt, blocks, n*k)`
    must return the f32 values). Norm weights are 1.0. qk_norm (default: for
    Qwen-style configs with head_dim 128 or the test shapes) adds q/k norms.
    """
    fmt = QFormat[fmt] if isinstance(fmt, str) else QFormat(fmt)
    rng = np.random.default_rng(seed)
    a, at = cfg["architecture"], cfg["attention"]
    h, L, V = a["hidden_size"], a["num_layers"], a["vocab_size"]
    hd = at["head_dim"]
    qd, kvd = at["num_heads"] * hd, at["num_kv_heads"] * hd
    ff = cfg["ffn"]["intermediate_size"]
    if qk_norm is None:
        qk_norm = cfg.get("name", "").startswith(("qwen", "tiny"))
    shapes = {"self_attn.q_proj": (qd, h), "self_attn.k_proj": (kvd, h),
              "self_attn.v_proj": (kvd, h), "self_attn.o_proj": (h, qd),
              "mlp.gate_proj": (ff, h), "mlp.up_proj": (ff, h), "mlp.down_proj": (h, ff)}
    w = {}

    def linear(n, k):
        if fmt == QFormat.INT8_KN:
            f = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
            q, s = quantize_rows_int8(f)
            return ("INT8_KN", q, s)
        blocks, _ = gen_weight(fmt, n, k, rng)
        return (fmt.name, blocks)

    ones = np.ones(h, np.float32)
    for i in range(L):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = ones
        w[p + "post_attention_layernorm.weight"] = ones
        if qk_norm:
            w[p + "self_attn.q_norm.weight"] = np.ones(hd, np.float32)
            w[p + "self_attn.k_norm.weight"] = np.ones(hd, np.float32)
        for nm, (n, k) in shapes.items():
            w[p + nm + ".weight"] = linear(n, k)
    w["model.norm.weight"] = ones
    if fmt == QFormat.INT8_KN:
        emb = rng.standard_normal((V, h), dtype=np.float32) * np.float32(0.02)
        w["model.embed_tokens.weight"] = emb
        q, s = quantize_rows_int8(emb)
        w["lm_head.weight"] = ("INT8_KN", q, s)
    else:
        blocks, _ = gen_weight(fmt, V, h, rng)
        w["lm_head.weight"] = (fmt.name, blocks)
        if dequant is None:
            raise ValueError("block-format models need dequant() for the tied embedding")
        w["model.embed_tokens.weight"] = np.asarray(dequant(fmt, blocks, V * h),
                                                    dtype=np.float32).reshape(V, h)
    return w
