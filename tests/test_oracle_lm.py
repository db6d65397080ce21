"""CPU tests of the oracle's LM epilogues and model runner against the
reference's own tests (ops/norm.rs, ops/rope.rs, generation/sampler.rs,
models/lm/causal_lm.rs) and basic invariants. No GPU."""
import numpy as np
import pytest

from oracle import oracle as O
from oracle.lm import OracleLM
from synapse_b200 import synth


def test_rmsnorm_unit_rms_and_direction():
    # ops/norm.rs:103-126
    out = O.rmsnorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 4, 1e-8)
    assert abs(np.sqrt(np.mean(out.astype(np.float64) ** 2)) - 1.0) < 0.01
    out = O.rmsnorm(np.array([3, 4, 0, 0], np.float32), np.ones(4, np.float32), 4, 1e-8)
    assert abs(out[0] / out[1] - 0.75) < 1e-5


def test_rmsnorm_uses_vechsum_order():
    # lanes of stride 4, then the tail: differs from a plain left-to-right sum
    rng = np.random.default_rng(3)
    x = rng.standard_normal(1027).astype(np.float32)
    sq = (x * x).astype(np.float32)
    lanes = np.zeros(4, np.float32)
    for i in range(0, 1024, 4):
        lanes = (lanes + sq[i:i + 4]).astype(np.float32)
    s = np.float32(np.float32(np.float32(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])
    for i in range(1024, 1027):
        s = np.float32(s + sq[i])
    scale = np.float32(1.0) / np.float32(np.sqrt(np.float32(s / np.float32(1027) + np.float32(1e-6))))
    want = ((x * np.float32(1.0)).astype(np.float32) * scale).astype(np.float32)
    got = O.rmsnorm(x, np.ones(1027, np.float32), 1027, 1e-6)
    assert np.array_equal(got, want)


def test_rope_position_zero_identity_and_norm_preserved():
    # ops/rope.rs:72-123
    c, s = O.rope_tables(1e6, 16, 8)
    x = np.arange(1, 17, dtype=np.float32)
    y = x.copy()
    O.rope_inplace(y, c, s, 1, 2, 8, 0)
    assert np.allclose(y, x)
    y = x.copy()
    O.rope_inplace(y, c, s, 1, 2, 8, 10)
    assert np.abs(y - x).sum() > 1e-3
    assert abs(np.linalg.norm(y) - np.linalg.norm(x)) < 1e-4


def test_argmax_ties_and_nan():
    # generation/sampler.rs:217-224: last maximal index, NaN compares Equal
    assert O.argmax(np.array([1, 3, 3, 2], np.float32)) == 2
    assert O.argmax(np.array([5, np.nan, 3, 1], np.float32)) == 2
    assert O.argmax(np.array([5, 1, np.nan], np.float32)) == 2
    assert O.argmax(np.array([0.0, -0.0], np.float32)) == 1


def test_softmax_and_swiglu():
    p = O.softmax(np.array([1, 2, 3, -np.inf], np.float32))
    assert abs(p.sum() - 1) < 1e-6 and p[3] == 0
    g = np.linspace(-4, 4, 11).astype(np.float32)
    u = np.ones(11, np.float32)
    ref = g / (1 + np.exp(-g.astype(np.float64)))
    assert np.allclose(O.silu_mul(g, u), ref, rtol=1e-6)
    assert np.allclose(O.swiglu(g, u), ref, rtol=1e-6)


def test_fused_attention_matches_naive_softmax():
    rng = np.random.default_rng(5)
    for S in (1, 7, 33, 70):
        q, k, v = (rng.standard_normal((S, 16)).astype(np.float32) for _ in range(3))
        st, o = O.fused_attention(S, S, 16, q, k, v)
        s = (q.astype(np.float64) @ k.T.astype(np.float64)) / 4.0
        s[np.triu_indices(S, 1)] = -np.inf
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        assert st == 0 and np.allclose(o.reshape(S, 16), p @ v, atol=1e-5)


@pytest.mark.parametrize("fmt", ["INT8_KN", "Q4_0"])
def test_oracle_prefill_then_decode_matches_longer_prefill(fmt):
    # models/lm/causal_lm.rs:742-860: prefill + decode logits == forward logits
    cfg = synth.lm_config("tiny")
    w = synth.gen_lm_weights(cfg, fmt, seed=7, dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])
    ids = [5, 17, 300, 42, 9, 128]
    a = OracleLM(cfg, w, 32)
    a.forward_prefill(ids[:-1])
    la = a.forward_one(ids[-1])
    b = OracleLM(cfg, w, 32)
    lb = b.forward_prefill(ids)
    assert np.allclose(la, lb, rtol=1e-3, atol=1e-4)
    assert np.argmax(la) == np.argmax(lb)


def test_oracle_greedy_generation_is_deterministic():
    cfg = synth.lm_config("tiny")
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=11)
    t1, m1 = OracleLM(cfg, w, 64).generate_greedy([1, 2, 3, 4], 12)
    t2, _ = OracleLM(cfg, w, 64).generate_greedy([1, 2, 3, 4], 12)
    assert t1 == t2 and len(t1) == 12 and all(0 <= t < 512 for t in t1)
    assert all(m >= 0 for m in m1)


@pytest.mark.parametrize("fmt", ["Q4_0", "Q4_K"])
def test_threaded_oracle_bit_identical(fmt):
    """The oracle's column-sliced threaded matmul (used to make full-size
    parity runs affordable) gives the bits of the single-call one, for
    prefill (M > 16, tiled) and decode (M = 1) alike."""
    cfg = synth.lm_config("tiny-hd64")
    w = synth.gen_lm_weights(cfg, fmt, seed=5, dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])
    prompt = list(range(3, 23))
    a = OracleLM(cfg, w, 48)
    b = OracleLM(cfg, w, 48, threads=3)
    la, lb = a.forward_prefill(prompt), b.forward_prefill(prompt)
    assert np.array_equal(la, lb)
    for t in (5, 77, 300):
        assert np.array_equal(a.forward_one(t), b.forward_one(t))
