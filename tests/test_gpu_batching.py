"""Continuous batching on a paged KV cache (syn_cuda_model_set_kv_paging,
syn_cuda_decode_step_slots). The reference decodes one sequence at a time
(generation/pipeline.rs:197-280, a contiguous cache per layer in
kv_cache/cache.rs:26-340); here sequences join (prefill into a free slot)
and leave (reset) between batched steps, and each one's greedy tokens must
equal its own single-sequence run -- bit-exact logits for INT8, whose
matmul rows and attention reductions do not depend on the batch.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

sb = pytest.importorskip("synapse_b200")
from synapse_b200 import synth  # noqa: E402


def _weights(fmt, name):
    cfg = synth.lm_config(name)
    if fmt == "INT8_KN":
        return cfg, synth.gen_lm_weights(cfg, fmt, seed=77)
    return cfg, synth.gen_lm_weights(cfg, fmt, seed=77,
                                     dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])


def _solo(ctx, cfg, w, prompt, steps):
    m = sb.Model(ctx, cfg, w, 128)
    tok, lg = m.forward_prefill(prompt)
    toks, logits = [tok], [lg]
    for _ in range(steps):
        nxt, l2 = m.forward_one([toks[-1]])
        toks.append(int(nxt[0]))
        logits.append(l2[0])
    m.close()
    return toks, logits


@pytest.mark.parametrize("fmt,name", [("INT8_KN", "tiny"), ("INT8_KN", "tiny-window"),
                                      ("Q4_0", "tiny")])
@pytest.mark.parametrize("page", [0, 16])
def test_sequences_join_and_leave(ctx, fmt, name, page):
    cfg, w = _weights(fmt, name)
    prompts = {"A": [3, 5, 7, 9, 11], "B": list(range(40, 73)), "C": [100, 4],
               "D": list(range(200, 219))}
    steps = 30
    solo = {k: _solo(ctx, cfg, w, p, steps) for k, p in prompts.items()}
    m = sb.Model(ctx, cfg, w, 128, max_batch=3, kv_page=page, kv_pages=24 if page else 0)
    live = {}   # slot -> (name, generated tokens, logits)
    free0 = m.kv_pages_free() if page else None

    def join(name, slot):
        tok, lg = m.forward_prefill(prompts[name], seq=slot)
        live[slot] = (name, [tok], [lg])

    join("A", 0)
    join("B", 2)
    for step in range(3 * steps):
        if step == 5:
            join("C", 1)
        if step == 12:   # A finished early: leaves, D takes its slot
            name, toks, _ = live.pop(0)
            m.reset(0)
            join("D", 0)
        slots = sorted(s for s, (n, t, _) in live.items() if len(t) <= steps)
        if not slots:
            break
        nxt, lg = m.decode_slots(slots, [live[s][1][-1] for s in slots], want_logits=True)
        for i, s in enumerate(slots):
            live[s][1].append(int(nxt[i]))
            live[s][2].append(lg[i])
        for s in list(live):  # retire finished sequences
            n, t, l = live[s]
            if len(t) > steps:
                want_t, want_l = solo[n]
                assert t == want_t, n
                if fmt == "INT8_KN":
                    for a, b in zip(l, want_l):
                        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), n
                else:
                    for a, b in zip(l, want_l):
                        assert np.max(np.abs(a - b)) <= 1e-4 * np.max(np.abs(b)), n
                live.pop(s)
                m.reset(s)
                if page:
                    assert m.kv_pages_free() >= 0
    assert not live
    if page:
        assert m.kv_pages_free() == free0  # every page came back
    m.close()


def test_paged_pool_exhaustion_is_reported(ctx):
    cfg, w = _weights("INT8_KN", "tiny")
    m = sb.Model(ctx, cfg, w, 128, max_batch=2, kv_page=16, kv_pages=3)
    m.forward_prefill(list(range(1, 40)), seq=0)  # 39 positions: 3 pages
    with pytest.raises(sb.SynapseError) as e:
        m.forward_prefill([1, 2, 3], seq=1)
    assert e.value.status == 3
    m.reset(0)
    assert m.kv_pages_free() == 3
    m.close()
