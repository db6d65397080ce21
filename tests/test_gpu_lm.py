"""GPU parity of the decoder-layer kernels and the model runner against the
CPU oracle (oracle/synapse_oracle_lm.c, oracle/lm.py) on seeded inputs.

Bit-exact: RMSNorm, SwiGLU, argmax, RoPE tables, KV-cache contents,
attention (decode and prefill), and the whole INT8 model (logits and greedy
tokens). Block-format models compute their matmuls on tensor cores with fp16
activations, so their logits are compared with a normwise tolerance and
their tokens wherever the oracle's top-2 margin exceeds the observed error.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle.lm import OracleLM

pytestmark = pytest.mark.gpu

sb = pytest.importorskip("synapse_b200")
from synapse_b200 import synth  # noqa: E402


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def exact(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a, b)


def close(a, b, flash):
    """Bit-exact for the reference-order kernels; within f32 reassociation
    (1e-5 of the row's magnitude) for the parallel-order ones."""
    if not flash:
        return exact(a, b)
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.allclose(a, b, rtol=1e-5, atol=1e-5 * np.abs(b).max())


@pytest.mark.parametrize("h", [4, 7, 128, 1024, 1027, 4096])
@pytest.mark.parametrize("rows", [1, 3])
def test_rmsnorm_bit_exact(h, rows):
    rng = np.random.default_rng(h + rows)
    x = rng.standard_normal((rows, h)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(h)).astype(np.float32)
    got = sb.rmsnorm(cuda(x), cuda(w), 1e-6).cpu().numpy()
    assert exact(got, O.rmsnorm(x, w, h, 1e-6).reshape(rows, h))
    d = rng.standard_normal((rows, h)).astype(np.float32)
    r = cuda(x)
    got = sb.add_rmsnorm(r, cuda(d), cuda(w), 1e-5).cpu().numpy()
    xs = (x + d).astype(np.float32)
    assert exact(r.cpu().numpy(), xs)
    assert exact(got, O.rmsnorm(xs, w, h, 1e-5).reshape(rows, h))


@pytest.mark.parametrize("n", [1, 6, 1030, 3072])
def test_swiglu_bit_exact(n):
    rng = np.random.default_rng(n)
    g = (4 * rng.standard_normal((2, n))).astype(np.float32)
    u = rng.standard_normal((2, n)).astype(np.float32)
    got0 = sb.swiglu(cuda(g), cuda(u), 0).cpu().numpy()
    got1 = sb.swiglu(cuda(g), cuda(u), 1).cpu().numpy()
    for r in range(2):
        assert exact(got0[r], O.silu_mul(g[r], u[r]))
        assert exact(got1[r], O.swiglu(g[r], u[r]))


def test_argmax_bit_exact():
    rng = np.random.default_rng(1)
    cases = [rng.standard_normal(151936).astype(np.float32),
             np.array([1, 3, 3, 2], np.float32),
             np.array([5, np.nan, 3, 1], np.float32),
             np.array([5, 1, np.nan], np.float32),
             np.array([0.0, -0.0, -1.0], np.float32),
             np.full(5000, 2.0, np.float32)]
    big = rng.standard_normal(128256).astype(np.float32)
    big[[7, 90000, 128000]] = 50.0
    cases.append(big)
    for c in cases:
        got = int(sb.argmax(cuda(c[None, :])).cpu()[0])
        assert got == O.argmax(c), (c[:8], got)


def test_rope_tables_match_oracle():
    for base, hd in ((1e6, 128), (5e5, 64), (10000.0, 32)):
        c, s = sb.rope_tables(base, 300, hd)
        oc, os_ = O.rope_tables(base, 300, hd)
        assert exact(c.reshape(-1), oc) and exact(s.reshape(-1), os_)


def _oracle_head_norm_rope(x, w, heads, hd, eps, cos, sin, pos):
    x = x.astype(np.float32).copy()
    if w is not None:
        x = O.rmsnorm(x, w, hd, eps)
    O.rope_inplace(x, cos, sin, 1, heads, hd, pos)
    return x


@pytest.mark.parametrize("hq,hkv,hd", [(4, 2, 32), (8, 2, 64), (16, 8, 128), (32, 8, 128)])
@pytest.mark.parametrize("lengths", [(1, 5), (63, 64), (65, 130), (257, 600)])
@pytest.mark.parametrize("window,norm", [(0, True), (24, False)])
@pytest.mark.parametrize("flash", [False, True])
def test_attention_decode_bit_exact(ctx, hq, hkv, hd, lengths, window, norm, flash):
    # contexts past 128 / 256 rows take the exact kernel's unstaged K rows and
    # its second V pass
    rng = np.random.default_rng(hq * 1000 + hd + lengths[0] + window)
    max_seq, B = max(160, max(lengths) + 8), 2
    qd, kvd = hq * hd, hkv * hd
    eps = 1e-6
    cache = sb.KVCache(ctx, max_seq, hkv, hd, 1, batch=B)
    cos, sin = sb.rope_tables(1e6, max_seq, hd)
    oc, os_ = O.rope_tables(1e6, max_seq, hd)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norm else None
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norm else None
    hist = []
    for b, L in enumerate(lengths):
        prev = L - 1
        kh = rng.standard_normal((max(prev, 1), kvd)).astype(np.float32)
        vh = rng.standard_normal((max(prev, 1), kvd)).astype(np.float32)
        if prev:
            cache.append(0, cuda(kh[:prev]), cuda(vh[:prev]), seq=b)
            cache.advance(prev, seq=b)
        hist.append((kh[:prev], vh[:prev]))
    qkv = rng.standard_normal((B, qd + 2 * kvd)).astype(np.float32)
    out = sb.attention_decode(cache, 0, cuda(qkv), hq, cuda(qn) if norm else None,
                              cuda(kn) if norm else None, eps, cuda(cos), cuda(sin),
                              window=window, batch=B, flash=flash).cpu().numpy()
    for b, L in enumerate(lengths):
        pos = L - 1
        q = _oracle_head_norm_rope(qkv[b, :qd], qn, hq, hd, eps, oc, os_, pos)
        k = _oracle_head_norm_rope(qkv[b, qd:qd + kvd], kn, hkv, hd, eps, oc, os_, pos)
        v = qkv[b, qd + kvd:]
        kc = np.concatenate([hist[b][0], k[None, :]])
        vc = np.concatenate([hist[b][1], v[None, :]])
        want = O.attention_decode(q, kc, vc, L, hq, hkv, hd, window)
        assert close(out[b], want, flash), (b, L, np.abs(out[b] - want).max())
        kv, vv = cache.view(0, b)
        assert exact(kv[pos].cpu().numpy(), k) and exact(vv[pos].cpu().numpy(), v)
        assert cache.length(b) == L - 1  # not advanced
    cache.close()


@pytest.mark.parametrize("flash", [False, True])
def test_attention_decode_long_context(ctx, flash):
    """4000 positions: the grouped flash kernel runs more than 32 splits per
    (row, KV head), the exact kernel many passes of staged V rows."""
    rng = np.random.default_rng(4000)
    hq, hkv, hd, L = 8, 2, 128, 4000
    max_seq, eps = L + 8, 1e-6
    qd, kvd = hq * hd, hkv * hd
    cache = sb.KVCache(ctx, max_seq, hkv, hd, 1, batch=1)
    cos, sin = sb.rope_tables(1e6, max_seq, hd)
    oc, os_ = O.rope_tables(1e6, max_seq, hd)
    kh = rng.standard_normal((L - 1, kvd)).astype(np.float32)
    vh = rng.standard_normal((L - 1, kvd)).astype(np.float32)
    cache.append(0, cuda(kh), cuda(vh), seq=0)
    cache.advance(L - 1, seq=0)
    qkv = rng.standard_normal((1, qd + 2 * kvd)).astype(np.float32)
    out = sb.attention_decode(cache, 0, cuda(qkv), hq, None, None, eps, cuda(cos), cuda(sin),
                              batch=1, flash=flash).cpu().numpy()
    q = _oracle_head_norm_rope(qkv[0, :qd], None, hq, hd, eps, oc, os_, L - 1)
    k = _oracle_head_norm_rope(qkv[0, qd:qd + kvd], None, hkv, hd, eps, oc, os_, L - 1)
    want = O.attention_decode(q, np.concatenate([kh, k[None]]),
                              np.concatenate([vh, qkv[0, qd + kvd:][None]]), L, hq, hkv, hd, 0)
    assert close(out[0], want, flash), np.abs(out[0] - want).max()
    cache.close()


@pytest.mark.parametrize("S", [1, 5, 16, 17, 33, 40, 70, 130])
@pytest.mark.parametrize("hq,hkv,hd,flash", [(4, 2, 32, False), (8, 2, 128, False),
                                             (4, 2, 64, True), (8, 2, 128, True)])
def test_attention_prefill_bit_exact(ctx, S, hq, hkv, hd, flash):
    rng = np.random.default_rng(S * 7 + hd)
    qd, kvd = hq * hd, hkv * hd
    eps = 1e-6
    cache = sb.KVCache(ctx, 160, hkv, hd, 2, batch=2)
    cos, sin = sb.rope_tables(1e6, 160, hd)
    oc, os_ = O.rope_tables(1e6, 160, hd)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    qkv = rng.standard_normal((S, qd + 2 * kvd)).astype(np.float32)
    out = sb.attention_prefill(cache, 1, cuda(qkv), hq, cuda(qn), cuda(kn), eps, cuda(cos),
                               cuda(sin), seq=1, flash=flash).cpu().numpy()
    q = O.rmsnorm(qkv[:, :qd], qn, hd, eps)
    k = O.rmsnorm(qkv[:, qd:qd + kvd], kn, hd, eps)
    O.rope_inplace(q, oc, os_, S, hq, hd, 0)
    O.rope_inplace(k, oc, os_, S, hkv, hd, 0)
    q3, k3 = q.reshape(S, hq, hd), k.reshape(S, hkv, hd)
    v3 = qkv[:, qd + kvd:].reshape(S, hkv, hd)
    g = hq // hkv
    for h in range(hq):
        st, o = O.fused_attention(S, S, hd, q3[:, h], k3[:, h // g], v3[:, h // g])
        assert close(out[:, h * hd:(h + 1) * hd], o.reshape(S, hd), flash), h
    kv, vv = cache.view(1, 1)
    assert exact(kv[:S].cpu().numpy(), k.reshape(S, kvd))
    assert exact(vv[:S].cpu().numpy(), qkv[:, qd + kvd:])
    cache.close()


@pytest.mark.parametrize("S", [200, 511, 700])
@pytest.mark.parametrize("hd", [64, 128])
def test_attention_prefill_tensor_core_long(ctx, S, hd):
    """The block-format prefill attention (tcgen05, split bf16 operands) on
    prompts of several 128-query tiles and 64-key tiles, against
    syn_fused_attention's restatement: normwise error <= 1e-4."""
    rng = np.random.default_rng(S + hd)
    hq, hkv = 4, 2
    qd, kvd = hq * hd, hkv * hd
    eps = 1e-6
    cache = sb.KVCache(ctx, 768, hkv, hd, 1, batch=1)
    cos, sin = sb.rope_tables(1e6, 768, hd)
    oc, os_ = O.rope_tables(1e6, 768, hd)
    qkv = (3 * rng.standard_normal((S, qd + 2 * kvd))).astype(np.float32)
    out = sb.attention_prefill(cache, 0, cuda(qkv), hq, None, None, eps, cuda(cos),
                               cuda(sin), seq=0, flash=True).cpu().numpy()
    q = qkv[:, :qd].copy()
    k = qkv[:, qd:qd + kvd].copy()
    O.rope_inplace(q, oc, os_, S, hq, hd, 0)
    O.rope_inplace(k, oc, os_, S, hkv, hd, 0)
    q3, k3 = q.reshape(S, hq, hd), k.reshape(S, hkv, hd)
    v3 = qkv[:, qd + kvd:].reshape(S, hkv, hd)
    for h in range(hq):
        st, o = O.fused_attention(S, S, hd, q3[:, h], k3[:, h // 2], v3[:, h // 2])
        o = o.reshape(S, hd)
        err = np.max(np.abs(out[:, h * hd:(h + 1) * hd] - o)) / np.max(np.abs(o))
        # products are f32-grade (split operands), the MMA's fp32 sums and the
        # 3x-scaled inputs' peaky softmax give a few 1e-6 normwise
        assert err <= 1e-4, (h, err)
    cache.close()


def test_kvcache_lengths_and_full(ctx):
    c = sb.KVCache(ctx, 4, 1, 8, 2, batch=2)
    z = torch.zeros(3, 8, device="cuda")
    c.append(0, z, z, seq=1)
    c.advance(3, seq=1)
    assert c.length(1) == 3 and c.length(0) == 0
    with pytest.raises(sb.SynapseError) as e:
        c.advance(2, seq=1)  # CacheFull -> INVALID_ARG (mapError)
    assert e.value.status == 2
    c.truncate(5, seq=1)
    assert c.length(1) == 3  # truncateTo only shortens
    c.truncate(1, seq=1)
    assert c.length(1) == 1
    c.reset(seq=1)
    assert c.length(1) == 0
    c.close()


def _gpu_model(ctx, cfg, w, max_seq, max_batch=1):
    return sb.Model(ctx, cfg, w, max_seq, max_batch)


@pytest.mark.parametrize("name", ["tiny", "tiny-hd64", "tiny-window"])
def test_int8_model_bit_exact_tokens_and_logits(ctx, name):
    cfg = synth.lm_config(name)
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=21)
    prompt = [3, 77, 140, 9, 255, 31, 64]
    steps = 40
    ref = OracleLM(cfg, w, 64)
    m = _gpu_model(ctx, cfg, w, 64)
    lref = ref.forward_prefill(prompt)
    tok, lg = m.forward_prefill(prompt)
    assert exact(lg, lref)
    assert tok == O.argmax(lref)
    for i in range(steps):
        lref = ref.forward_one(tok)
        nxt, lg = m.forward_one([tok])
        assert exact(lg[0], lref), (i, np.abs(lg[0] - lref).max())
        assert int(nxt[0]) == O.argmax(lref)
        tok = int(nxt[0])
    assert m.seq_len() == len(prompt) + steps
    m.close()


def test_int8_model_batch_matches_single_sequences(ctx):
    cfg = synth.lm_config("tiny")
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=5)
    prompts = [[1, 2, 3, 4, 5], [400, 300, 200]]
    m = _gpu_model(ctx, cfg, w, 64, max_batch=2)
    toks = [m.forward_prefill(p, seq=i, want_logits=False)[0] for i, p in enumerate(prompts)]
    refs = [OracleLM(cfg, w, 64) for _ in prompts]
    rt = [refs[i].forward_prefill(p) for i, p in enumerate(prompts)]
    assert toks == [O.argmax(x) for x in rt]
    for step in range(12):
        nxt, lg = m.forward_one(toks)
        for i in range(2):
            lr = refs[i].forward_one(toks[i])
            assert exact(lg[i], lr), (step, i)
        toks = [int(t) for t in nxt]
    m.close()


def test_int8_model_greedy_generation_and_reset(ctx):
    cfg = synth.lm_config("tiny")
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=9)
    m = _gpu_model(ctx, cfg, w, 64)
    t1 = m.generate_greedy([10, 20, 30], 24)
    ref, _ = OracleLM(cfg, w, 64).generate_greedy([10, 20, 30], 24)
    assert t1 == ref
    with pytest.raises(sb.SynapseError):
        m.forward_prefill([1, 2])  # the sequence is not empty
    m.reset()
    assert m.seq_len() == 0
    assert m.generate_greedy([10, 20, 30], 24) == ref
    m.truncate(5)
    assert m.seq_len() == 5
    # chained on-device generation gives the same tokens
    m.reset()
    first, _ = m.forward_prefill([10, 20, 30], want_logits=False)
    assert first == ref[0]
    assert m.generate(23)[0].tolist() == ref[1:]
    assert m.seq_len() == 3 + 23
    m.close()


def test_int8_model_generate_batch(ctx):
    cfg = synth.lm_config("tiny-window")
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=17)
    prompts = [[5, 6, 7, 8], [99, 98]]
    m = _gpu_model(ctx, cfg, w, 96, max_batch=2)
    for i, p in enumerate(prompts):
        m.forward_prefill(p, seq=i, want_logits=False)
    got = m.generate(40, batch=2)
    for i, p in enumerate(prompts):
        ref, _ = OracleLM(cfg, w, 96).generate_greedy(p, 41)
        assert got[i].tolist() == ref[1:], i
    m.close()


@pytest.mark.parametrize("fmt,name", [("Q4_0", "tiny"), ("Q8_0", "tiny"), ("Q4_K", "tiny-hd64"),
                                      ("Q6_K", "tiny-hd64")])
def test_block_model_logits_within_tolerance(ctx, fmt, name):
    cfg = synth.lm_config(name)
    w = synth.gen_lm_weights(cfg, fmt, seed=13,
                             dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])
    prompt = [7, 8, 9, 100, 200, 11, 12, 13, 14, 15]
    ref = OracleLM(cfg, w, 64)
    m = _gpu_model(ctx, cfg, w, 64)
    lref = ref.forward_prefill(prompt)
    tok, lg = m.forward_prefill(prompt)
    err = np.linalg.norm(lg - lref) / np.linalg.norm(lref)
    assert err < 5e-3, err
    for i in range(16):
        srt = np.sort(lref)
        if O.argmax(lref) != tok:
            # a disagreement is only allowed where the oracle's top-2 margin
            # is below the observed logit error; nothing is compared after it
            assert srt[-1] - srt[-2] <= np.abs(lg - lref).max(), (i, srt[-1] - srt[-2])
            break
        lref = ref.forward_one(tok)
        nxt, lgs = m.forward_one([tok])
        lg = lgs[0]
        err = np.linalg.norm(lg - lref) / np.linalg.norm(lref)
        assert err < 5e-3, (i, err)
        tok = int(nxt[0])
    m.close()


def test_qwen3_0p6b_int8_greedy_64_tokens_identical(ctx):
    """Config 1 at full size: 16-token prompt, 64 greedy tokens, token ids and
    final logits identical to the oracle (int8.rs:593-709)."""
    cfg = synth.lm_config("qwen3-0.6b")
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=1234)
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, cfg["architecture"]["vocab_size"], 16).tolist()
    m = _gpu_model(ctx, cfg, w, 128)
    got = m.generate_greedy(prompt, 64)
    m.close()
    ref, margins = OracleLM(cfg, w, 128).generate_greedy(prompt, 64)
    assert got == ref, (got, ref, margins)


@pytest.mark.parametrize("fmt", ["INT8_KN", "Q4_0", "Q6_K"])
@pytest.mark.parametrize("fast", [False, True])
def test_qmatmul_rmsnorm_fused_equals_separate(ctx, fmt, fast):
    """The fused RMSNorm + GEMV gives the bits of rmsnorm then matmul (and the
    residual sum); with fast=False the norm is the reference-order one."""
    rng = np.random.default_rng(7)
    n, k = 640, 1024
    f = sb.QFormat[fmt]
    data, scales = synth.gen_weight(f, n, k, rng)
    w = sb.QuantizedWeight(ctx, f, data, n, k, scales)
    r = cuda(rng.standard_normal((1, k)).astype(np.float32))
    d = cuda(rng.standard_normal((1, k)).astype(np.float32))
    nw = cuda((1 + 0.1 * rng.standard_normal(k)).astype(np.float32))
    ro = torch.empty_like(r)
    y = w.matmul_rmsnorm(r, nw, 1e-6, delta=d, residual_out=ro, parallel_sum=fast)
    if not fast:
        r2 = r.clone()
        x = sb.add_rmsnorm(r2, d, nw, 1e-6)
        assert exact(ro.cpu().numpy(), r2.cpu().numpy())
        assert exact(y.cpu().numpy(), w.matmul(x).cpu().numpy())
    else:
        xs = (r + d).cpu().numpy()
        x = xs / np.sqrt((xs.astype(np.float64) ** 2).mean() + 1e-6) * nw.cpu().numpy()
        yr = w.matmul(torch.from_numpy(x.astype(np.float32)).cuda()).cpu().numpy()
        assert np.allclose(y.cpu().numpy(), yr, rtol=1e-3, atol=1e-3 * np.abs(yr).max())
    w.close()
