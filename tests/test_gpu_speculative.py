"""Speculative decoding with KV rollback on the device
(syn_cuda_decode_span, syn_cuda_generate_speculative; reference:
generation/pipeline.rs:281-396 and syn_kvcache_truncate,
zig/src/ffi/exports.zig:1935-1940).

A span step over n new positions gives, row for row, the logits of n
one-token decode steps (bit-exact for INT8: the same matmul and attention
reductions), without advancing the cache. Speculative generation verifies
every draft token, so it emits the plain greedy sequence.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

sb = pytest.importorskip("synapse_b200")
from synapse_b200 import synth  # noqa: E402


def _model(ctx, fmt, name, max_seq=96):
    cfg = synth.lm_config(name)
    if fmt == "INT8_KN":
        w = synth.gen_lm_weights(cfg, fmt, seed=41)
    else:
        w = synth.gen_lm_weights(cfg, fmt, seed=41,
                                 dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])
    return sb.Model(ctx, cfg, w, max_seq)


@pytest.mark.parametrize("name", ["tiny", "tiny-window"])
def test_span_equals_sequential_decode_int8(ctx, name):
    m = _model(ctx, "INT8_KN", name)
    prompt = [4, 8, 15, 16, 23, 42]
    tok, _ = m.forward_prefill(prompt)
    seq_toks, seq_logits = [tok], []
    for _ in range(5):
        nxt, lg = m.forward_one([seq_toks[-1]])
        seq_logits.append(lg[0])
        seq_toks.append(int(nxt[0]))
    m.reset()
    m.forward_prefill(prompt, want_logits=False)
    n0 = m.seq_len()
    out, lg = m.decode_span(seq_toks[:5], want_logits=True)
    assert m.seq_len() == n0  # not advanced
    assert out.tolist() == seq_toks[1:6]
    for i in range(5):
        assert np.array_equal(lg[i].view(np.uint32), seq_logits[i].view(np.uint32)), i
    m.close()


@pytest.mark.parametrize("fmt,name", [("INT8_KN", "tiny"), ("INT8_KN", "tiny-window"),
                                      ("Q4_0", "tiny"), ("Q4_K", "tiny-hd64")])
@pytest.mark.parametrize("k", [1, 4, 7])
def test_speculative_emits_the_greedy_sequence(ctx, fmt, name, k):
    m = _model(ctx, fmt, name)
    prompt = [3, 77, 140, 9, 255, 31]
    want = m.generate_greedy(prompt, 40)
    m.reset()
    got, drafted, accepted = m.generate_speculative(prompt, 40, k=k, draft_layers=1)
    assert got == want
    assert drafted >= accepted >= 0 and drafted > 0
    # the cache holds the prompt and every emitted token but the last
    assert m.seq_len() == len(prompt) + 39
    # and decoding continues from there as usual
    nxt, _ = m.forward_one([got[-1]], want_logits=False)
    m.reset()
    ref = m.generate_greedy(prompt, 41)
    assert int(nxt[0]) == ref[-1]
    m.close()


def test_speculative_full_draft_accepts_everything(ctx):
    """A draft of all layers is the full model: every draft token is kept."""
    m = _model(ctx, "INT8_KN", "tiny")
    L = m.cfg["architecture"]["num_layers"]
    got, drafted, accepted = m.generate_speculative([5, 6, 7], 25, k=4, draft_layers=L)
    m.reset()
    assert got == m.generate_greedy([5, 6, 7], 25)
    assert accepted == drafted
    m.close()


def test_span_many_argmax_segments(ctx):
    """A vocabulary of several argmax segments (2048 logits each): the span
    step's per-row greedy tokens after one-token steps of other widths."""
    import copy
    cfg = copy.deepcopy(synth.lm_config("tiny"))
    cfg["architecture"]["vocab_size"] = 9000
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=43)
    m = sb.Model(ctx, cfg, w, 96)
    prompt = [4, 8, 15, 16, 23, 42, 8000, 8999]
    want = m.generate_greedy(prompt, 20)
    m.reset()
    got, _, _ = m.generate_speculative(prompt, 20, k=5, draft_layers=1)
    assert got == want
    m.close()
