"""Models loaded from weight files give the logits of the same weights
staged tensor by tensor (bit-exact), on the GPU:
  * GGUF (syn_cuda_model_load_gguf): raw Q4_0 / Q8_0 / Q4_K / Q6_K blocks,
    llama.cpp names, the llama converter's Q/K row order, tied embedding
    dequantised on the device; the repack cache gives the same model;
  * safetensors (syn_cuda_model_load_safetensors): f16 / bf16 checkpoints
    quantised to INT8 on the device as the reference's --quantize load
    (converter.rs + int8.rs:78-152), against the oracle's quantisation of the
    converted f32 weights.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import GGUF_TYPES, gguf_bytes, safetensors_bytes

pytestmark = pytest.mark.gpu

sb = pytest.importorskip("synapse_b200")
from synapse_b200 import synth  # noqa: E402

HF_TO_GGUF = {"input_layernorm": "attn_norm", "post_attention_layernorm": "ffn_norm",
              "self_attn.q_proj": "attn_q", "self_attn.k_proj": "attn_k",
              "self_attn.v_proj": "attn_v", "self_attn.o_proj": "attn_output",
              "self_attn.q_norm": "attn_q_norm", "self_attn.k_norm": "attn_k_norm",
              "mlp.gate_proj": "ffn_gate", "mlp.up_proj": "ffn_up", "mlp.down_proj": "ffn_down"}


def _permute_rows(raw, n, k, fmt, heads):
    """The llama GGUF converter's Q/K row order: checkpoint row
    h*hd + a*hd/2 + i is stored at h*hd + 2i + a."""
    rb = sb.row_bytes(sb.QFormat[fmt], k)
    rows = np.frombuffer(raw, np.uint8).reshape(n, rb)
    hd = n // heads
    out = np.empty_like(rows)
    for h in range(heads):
        for i in range(hd // 2):
            for a in range(2):
                out[h * hd + 2 * i + a] = rows[h * hd + a * (hd // 2) + i]
    return out.tobytes()


def _gguf_model_file(cfg, w, fmt, path):
    a, at = cfg["architecture"], cfg["attention"]
    L, h = a["num_layers"], a["hidden_size"]
    hq, hkv, hd = at["num_heads"], at["num_kv_heads"], at["head_dim"]
    ff = cfg["ffn"]["intermediate_size"]
    shapes = {"q_proj": (hq * hd, h), "k_proj": (hkv * hd, h), "v_proj": (hkv * hd, h),
              "o_proj": (h, hq * hd), "gate_proj": (ff, h), "up_proj": (ff, h),
              "down_proj": (h, ff)}
    t = []
    for i in range(L):
        for hf, gg in HF_TO_GGUF.items():
            name = f"model.layers.{i}.{hf}.weight"
            if name not in w:
                continue
            v = w[name]
            if isinstance(v, tuple):
                n, k = shapes[hf.split(".")[-1]]
                raw = np.asarray(v[1]).tobytes()
                if hf in ("self_attn.q_proj", "self_attn.k_proj"):
                    raw = _permute_rows(raw, n, k, fmt, hq if hf.endswith("q_proj") else hkv)
                t.append((f"blk.{i}.{gg}.weight", GGUF_TYPES[fmt], [k, n], raw))
            else:  # norms as F16 (exact for these values)
                t.append((f"blk.{i}.{gg}.weight", 1, [v.size],
                          np.asarray(v, np.float32).astype(np.float16).tobytes()))
    t.append(("output_norm.weight", 0, [h], np.asarray(w["model.norm.weight"], np.float32).tobytes()))
    t.append(("token_embd.weight", GGUF_TYPES[fmt], [h, a["vocab_size"]],
              np.asarray(w["lm_head.weight"][1]).tobytes()))  # tied: no output.weight
    meta = [("general.architecture", "llama"), ("llama.block_count", L),
            ("llama.embedding_length", h), ("llama.feed_forward_length", ff),
            ("llama.attention.head_count", hq), ("llama.attention.head_count_kv", hkv),
            ("llama.attention.key_length", hd),
            ("llama.attention.layer_norm_rms_epsilon", float(cfg["norm"]["eps"])),
            ("llama.rope.freq_base", float(cfg["position"]["base"])),
            ("llama.context_length", 4096)]
    path.write_bytes(gguf_bytes(t, meta))


def _same_run(m1, m2, prompt, steps=6):
    m1.reset()
    m2.reset()
    t1, l1 = m1.forward_prefill(prompt)
    t2, l2 = m2.forward_prefill(prompt)
    assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
    for _ in range(steps):
        n1, l1 = m1.forward_one([t1])
        n2, l2 = m2.forward_one([t2])
        assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
        t1, t2 = int(n1[0]), int(n2[0])
        assert t1 == t2


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_gguf_model_equals_per_tensor_upload(ctx, fmt, tmp_path):
    cfg = synth.lm_config("tiny-hd64")
    w = synth.gen_lm_weights(cfg, fmt, seed=8, dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])
    path = tmp_path / "m.gguf"
    _gguf_model_file(cfg, w, fmt, path)
    ref = sb.Model(ctx, cfg, w, 64)
    got = sb.Model.from_gguf(ctx, path, 64)
    for sec in ("attention", "ffn"):
        for k in ("num_heads", "num_kv_heads", "head_dim", "intermediate_size"):
            if k in cfg[sec]:
                assert got.cfg[sec][k] == cfg[sec][k]
    _same_run(ref, got, [3, 9, 27, 81, 243, 100])
    got.close()
    # the repack cache: first load writes, second reads every weight
    cache = tmp_path / "cache"
    cache.mkdir()
    m1 = sb.Model.from_gguf(ctx, path, 64, cache_dir=cache)
    assert m1.cache_hits() == 0
    m2 = sb.Model.from_gguf(ctx, path, 64, cache_dir=cache)
    L = cfg["architecture"]["num_layers"]
    assert m2.cache_hits() == 4 * L + 1  # qkv, o, gate/up, down per layer + LM head
    _same_run(ref, m2, [5, 6, 7, 8])
    for m in (m1, m2, ref):
        m.close()


def _f16_weights(cfg, dtype, rng):
    """HF-named float checkpoint (f16 or bf16 bits for the linears and the
    embedding) and the reference's view of it: f32 by the loader's rule."""
    a, at = cfg["architecture"], cfg["attention"]
    h, L, V = a["hidden_size"], a["num_layers"], a["vocab_size"]
    hq, hkv, hd = at["num_heads"], at["num_kv_heads"], at["head_dim"]
    ff = cfg["ffn"]["intermediate_size"]
    shapes = {"self_attn.q_proj": (hq * hd, h), "self_attn.k_proj": (hkv * hd, h),
              "self_attn.v_proj": (hkv * hd, h), "self_attn.o_proj": (h, hq * hd),
              "mlp.gate_proj": (ff, h), "mlp.up_proj": (ff, h), "mlp.down_proj": (h, ff)}

    def bits(n, k):
        x = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        x.reshape(-1)[:7] = [1e-7, -3e-6, 6e-8, 0.0, -0.0, 2e-5, 5e-7]  # f16 subnormals
        if dtype == "F16":
            return x.astype(np.float16).view(np.uint16)
        return (x.view(np.uint32) >> 16).astype(np.uint16)

    def conv(b):
        if dtype == "F16":
            flat = b.reshape(-1)
            lut = np.array([O.f16_rust(i) for i in range(65536)], np.float32)
            return lut[flat].reshape(b.shape)
        return (b.astype(np.uint32) << 16).view(np.float32)

    file_t, ref_w = [], {}
    for i in range(L):
        p = f"model.layers.{i}."
        for nm in ("input_layernorm", "post_attention_layernorm"):
            v = np.ones(h, np.float32)
            file_t.append((p + nm + ".weight", "F32", [h], v.tobytes()))
            ref_w[p + nm + ".weight"] = v
        for nm, (n, k) in shapes.items():
            b = bits(n, k)
            file_t.append((p + nm + ".weight", dtype, [n, k], b.tobytes()))
            q, s = O.quantize_weights_int8(conv(b), n, k)
            ref_w[p + nm + ".weight"] = ("INT8_KN", q, s)
    file_t.append(("model.norm.weight", "F32", [h], np.ones(h, np.float32).tobytes()))
    ref_w["model.norm.weight"] = np.ones(h, np.float32)
    e = bits(V, h)
    file_t.append(("model.embed_tokens.weight", dtype, [V, h], e.tobytes()))
    ref_w["model.embed_tokens.weight"] = conv(e)
    q, s = O.quantize_weights_int8(conv(e), V, h)  # tied LM head (int8.rs:127-139)
    ref_w["lm_head.weight"] = ("INT8_KN", q, s)
    return file_t, ref_w


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_safetensors_int8_model_equals_oracle_quantisation(ctx, dtype, tmp_path):
    cfg = synth.lm_config("tiny")
    cfg = dict(cfg)
    rng = np.random.default_rng(12)
    file_t, ref_w = _f16_weights(cfg, dtype, rng)
    path = tmp_path / "m.safetensors"
    path.write_bytes(safetensors_bytes(file_t, metadata={"format": "pt"}))
    ref = sb.Model(ctx, cfg, ref_w, 48)
    got = sb.Model.from_safetensors(ctx, path, cfg, 48)
    _same_run(ref, got, [1, 17, 250, 3, 77])
    ref.close()
    got.close()


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_quantize_weights_int8_half_bit_exact(dtype):
    rng = np.random.default_rng(3)
    n, k = 96, 320
    x = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    x[0, :5] = [1e-7, -6e-8, 0, 3e-5, 1.0]
    x[1] = 0.0  # a zero row: scale 1, zero codes
    if dtype == "F16":
        b = x.astype(np.float16).view(np.uint16)
        f = np.array([O.f16_rust(int(v)) for v in b.reshape(-1)], np.float32).reshape(n, k)
    else:
        b = (x.view(np.uint32) >> 16).astype(np.uint16)
        f = (b.astype(np.uint32) << 16).view(np.float32)
    q, s = sb.quantize_weights_int8_half(torch.from_numpy(b.view(np.int16)).cuda(), dtype, n, k)
    qo, so = O.quantize_weights_int8(f, n, k)
    assert np.array_equal(q.cpu().numpy().view(np.int8), qo)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
