"""Weight-file parsers of the C ABI (syn_gguf_*, syn_safetensors_*,
syn_convert_to_f32), on the host -- no GPU. Known-answer cases are the
reference's own loader tests (weight_loading/gguf.rs:700-830 and
safetensors.rs:350-470), restated against files written by
tests/helpers.py."""
import struct

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import GGUF_TYPES, gguf_bytes, safetensors_bytes


@pytest.fixture(scope="module")
def sb():
    import synapse_b200
    return synapse_b200


def _write(tmp_path, name, data):
    p = tmp_path / name
    p.write_bytes(data)
    return p


def test_gguf_q4_0_block_kat(sb, tmp_path):
    # gguf.rs:790-821: delta 1.0 (0x3C00), bytes 0x10 -> even -8, odd -7
    block = struct.pack("<H", 0x3C00) + bytes([0x10] * 16)
    p = _write(tmp_path, "q4.gguf", gguf_bytes([("q4_tensor", GGUF_TYPES["Q4_0"], [32], block)]))
    g = sb.GGUFFile(p)
    [(name, typ, dims, raw)] = g.tensors()
    assert (name, typ, dims, raw) == ("q4_tensor", 2, [32], block)
    st, vals = O.dequant("Q4_0", np.frombuffer(raw, np.uint8), 32)
    assert list(vals[0::2]) == [-8.0] * 16 and list(vals[1::2]) == [-7.0] * 16
    g.close()


def test_gguf_metadata_and_f32_tensor(sb, tmp_path):
    # gguf.rs:724-766: one string metadata KV, then a 2-element F32 tensor
    data = struct.pack("<ff", 42.0, 43.0)
    meta = [("general.name", "test"), ("general.architecture", "llama"),
            ("llama.block_count", 2), ("tokenizer.ggml.tokens", ["a", "bc", ""]),
            ("llama.rope.freq_base", 500000.0), ("flag", True)]
    p = _write(tmp_path, "w.gguf", gguf_bytes([("w", 0, [2], data)], meta))
    g = sb.GGUFFile(p)
    [(name, typ, dims, raw)] = g.tensors()
    assert np.frombuffer(raw, np.float32).tolist() == [42.0, 43.0]
    assert g.meta_str("general.name") == "test"
    assert g.meta_num("llama.block_count") == 2
    assert g.meta_num("llama.rope.freq_base") == 500000.0
    assert g.meta_num("flag") == 1.0
    with pytest.raises(sb.SynapseError):
        g.meta_num("tokenizer.ggml.tokens")  # arrays are skipped, not kept
    g.close()


@pytest.mark.parametrize("version", [2, 3])
def test_gguf_versions_and_alignment(sb, tmp_path, version):
    a = np.arange(8, dtype=np.float32).tobytes()
    b = np.arange(3, dtype=np.float32).tobytes()
    f = gguf_bytes([("a", 0, [8], a), ("b", 0, [3], b)], [("general.alignment", 64)],
                   version=version, alignment=64)
    g = sb.GGUFFile(_write(tmp_path, "al.gguf", f))
    t = {n: r for n, _, _, r in g.tensors()}
    assert t["a"] == a and t["b"] == b
    g.close()


@pytest.mark.parametrize("corrupt", ["magic", "version", "truncated", "beyond"])
def test_gguf_rejects_bad_files(sb, tmp_path, corrupt):
    good = gguf_bytes([("w", 0, [4], np.zeros(4, np.float32).tobytes())], [("k", 1)])
    bad = bytearray(good)
    if corrupt == "magic":
        bad[0:4] = b"GGUX"
    elif corrupt == "version":
        bad[4:8] = struct.pack("<I", 4)
    elif corrupt == "truncated":
        bad = bad[:30]
    else:
        bad = bad[:-4]  # the tensor's bytes end past the file
    with pytest.raises(sb.SynapseError) as e:
        sb.GGUFFile(_write(tmp_path, "bad.gguf", bytes(bad)))
    assert e.value.status == 2


def test_gguf_unknown_type_has_no_size(sb, tmp_path):
    # gguf.rs:823-829 rejects GGML type 99 when dequantising; here the
    # parser reports 0 bytes and the model loader refuses it
    g = sb.GGUFFile(_write(tmp_path, "u.gguf", gguf_bytes([("bad", 99, [32], bytes(64))])))
    [(name, typ, dims, raw)] = g.tensors()
    assert typ == 99 and raw == b""
    g.close()


def test_gguf_runner_names(sb):
    f = sb.gguf_runner_name
    assert f("token_embd.weight") == "model.embed_tokens.weight"
    assert f("output_norm.weight") == "model.norm.weight"
    assert f("output.weight") == "lm_head.weight"
    assert f("blk.0.attn_norm.weight") == "model.layers.0.input_layernorm.weight"
    assert f("blk.31.ffn_down.weight") == "model.layers.31.mlp.down_proj.weight"
    assert f("blk.7.attn_output.weight") == "model.layers.7.self_attn.o_proj.weight"
    assert f("blk.3.attn_k_norm.weight") == "model.layers.3.self_attn.k_norm.weight"
    assert f("blk.3.ffn_norm.weight") == "model.layers.3.post_attention_layernorm.weight"
    for bad in ("blk..attn_q.weight", "blk.1a.attn_q.weight", "blk.1.rope_freqs", "rope_freqs.weight"):
        assert f(bad) is None


def test_gguf_config_from_metadata(sb, tmp_path):
    from synapse_b200 import synth
    meta = [("general.architecture", "llama"), ("llama.block_count", 16),
            ("llama.embedding_length", 2048), ("llama.feed_forward_length", 8192),
            ("llama.attention.head_count", 32), ("llama.attention.head_count_kv", 8),
            ("llama.attention.key_length", 64), ("llama.rope.freq_base", 500000.0),
            ("llama.attention.layer_norm_rms_epsilon", 1e-5), ("llama.context_length", 131072)]
    emb = [("token_embd.weight", GGUF_TYPES["Q4_0"], [2048, 256], bytes(256 * 64 * 18))]
    g = sb.GGUFFile(_write(tmp_path, "c.gguf", gguf_bytes(emb, meta)))
    cfg = g.config()
    want = synth.lm_config("llama-3.2-1b")
    for sec in ("attention", "ffn", "position"):
        for k, v in want[sec].items():
            if k in cfg[sec]:
                assert cfg[sec][k] == pytest.approx(v), (sec, k)
    a = cfg["architecture"]
    assert (a["hidden_size"], a["num_layers"], a["vocab_size"]) == (2048, 16, 256)
    assert a["tie_word_embeddings"] is True
    assert cfg["norm"]["eps"] == pytest.approx(1e-5)
    g.close()


# ------------------------------- safetensors -------------------------------

def test_safetensors_f32_f16_bf16(sb, tmp_path):
    # safetensors.rs:352-402
    fa = np.array([1.5, -2.25, 3.0], np.float32)
    f = safetensors_bytes([("weight_a", "F32", [3], fa.tobytes()),
                           ("w16", "F16", [3], np.array([0x3C00, 0x4000, 0x3800], np.uint16).tobytes()),
                           ("wb", "BF16", [3], np.array([0x3F80, 0x4000, 0xBF80], np.uint16).tobytes())],
                          metadata={"format": "pt"})
    st = sb.SafetensorsFile(_write(tmp_path, "a.safetensors", f))
    t = st.tensors()
    assert set(t) == {"weight_a", "w16", "wb"}  # __metadata__ skipped
    assert np.array_equal(t["weight_a"][2], fa)
    assert t["w16"][2].tolist() == [1.0, 2.0, 0.5]
    assert t["wb"][2].tolist() == [1.0, 2.0, -1.0]
    st.close()


def test_safetensors_errors(sb, tmp_path):
    # safetensors.rs:404-424: unsupported dtype, truncated file
    hdr = b'{"t":{"dtype":"INT4","shape":[2],"data_offsets":[0,1]}}'
    with pytest.raises(sb.SynapseError) as e:
        sb.SafetensorsFile(_write(tmp_path, "u.st", struct.pack("<Q", len(hdr)) + hdr + b"\0"))
    assert e.value.status == 12
    with pytest.raises(sb.SynapseError) as e:
        sb.SafetensorsFile(_write(tmp_path, "t.st", bytes(4)))
    assert e.value.status == 2
    f = safetensors_bytes([("w", "F32", [4], bytes(16))])
    with pytest.raises(sb.SynapseError) as e:
        sb.SafetensorsFile(_write(tmp_path, "b.st", f[:-4]))  # data past the end
    assert e.value.status == 2


def test_f16_conversion_matches_the_loader_for_every_pattern(sb):
    """syn_convert_to_f32 (F16) == converter.rs:12-40 (the oracle's
    f16_rust) for all 65536 bit patterns, including the halved subnormals."""
    import ctypes
    bits = np.arange(65536, dtype=np.uint16)
    got = np.empty(65536, np.float32)
    assert sb.lib.syn_convert_to_f32(1, bits.ctypes.data_as(ctypes.c_void_p), 65536,
                                     got.ctypes.data_as(ctypes.c_void_p)) == 0
    want = np.array([O.f16_rust(int(b)) for b in bits], np.float32)
    nan = np.isnan(want)  # NaN payloads do not survive the ctypes float return
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
