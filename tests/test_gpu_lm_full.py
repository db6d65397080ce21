"""Full-size greedy-decode parity of the block-format configs against the
CPU oracle of the reference's f32 route (oracle/lm.py restating
CausalLM::{forward_prefill, forward_one}, models/lm/causal_lm.rs:195-280,
with weights dequantised as weight_loading/gguf.rs:255-487 does):

  config 3  LLaMA-3.2-1B shape, Q4_K, 512-token prompt, batch 1; and batch 8
            (eight 64-token prompts, decoded together by the batched runner)
  config 4  Mistral-7B shape, Q4_0, TP1; a 32-token prompt instead of 2048
            (the CPU oracle needs 28 GB of f32 weights and about a second per
            token on a host core; the decode path is the same)
  config 5  Qwen3-0.6B shape, Q8_0, 32 sequences with prompt lengths uniform
            in [128, 2048] served together; the three shortest are checked

Each checked sequence emits 64 greedy tokens. The block formats' matmuls
meet a 1e-3 tolerance rather than bit equality, so token ids must match
at every step unless the oracle's top-2 logit margin at the first
divergence is below the observed logit error (max |gpu - oracle| of that
step); that case is reported with both numbers, and the sequences are not
compared beyond it. Random-init weights from the benchmark's generators.
"""
import os
import threading

import numpy as np
import pytest

from oracle import oracle as O
from oracle.lm import OracleLM

pytestmark = pytest.mark.gpu

sb = pytest.importorskip("synapse_b200")
from synapse_b200 import synth  # noqa: E402

STEPS = 64
THREADS = max(1, min(32, os.cpu_count() or 1))


def _weights(cfg, fmt):
    return synth.gen_lm_weights(cfg, fmt, seed=1234,
                                dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])


def _check_step(step, gpu_tok, gpu_logits, ref_logits, report):
    """True while the sequences agree; on the first divergence asserts that
    the oracle's top-2 margin is below the observed logit error."""
    ref_tok = O.argmax(ref_logits)
    err = float(np.max(np.abs(gpu_logits - ref_logits)))
    report["max_logit_err"] = max(report.get("max_logit_err", 0.0), err)
    rel = err / max(float(np.max(np.abs(ref_logits))), 1e-30)
    report["max_rel_err"] = max(report.get("max_rel_err", 0.0), rel)
    if gpu_tok == ref_tok:
        return True
    srt = np.sort(ref_logits)
    margin = float(srt[-1] - srt[-2])
    report["diverged_at"] = step
    report["margin"] = margin
    report["err"] = err
    assert margin <= err, f"step {step}: tokens {gpu_tok} vs {ref_tok}, margin {margin} > err {err}"
    return False


def _run_batch(model, refs, prompts, seqs, others=None):
    """Prefills prompts[i] into GPU sequence seqs[i] (and oracle refs[i]),
    then decodes all GPU sequences [0, max(seqs)] together; compares the
    sequences in `seqs`; `others` maps further GPU-only sequences, already
    prefilled, to their first token. Returns one report per checked
    sequence."""
    reports = [dict() for _ in seqs]
    ref_logits = [None] * len(seqs)

    def ref_prefill(i):
        ref_logits[i] = refs[i].forward_prefill(prompts[i])
    ts = [threading.Thread(target=ref_prefill, args=(i,)) for i in range(len(seqs))]
    for t in ts:
        t.start()
    toks = dict(others or {})
    gpu_logits = {}
    for i, s in enumerate(seqs):
        tok, lg = model.forward_prefill(prompts[i], seq=s)
        toks[s], gpu_logits[s] = tok, lg
    for t in ts:
        t.join()
    batch = max(list(seqs) + list(toks)) + 1
    alive = [True] * len(seqs)
    for step in range(STEPS):
        for i, s in enumerate(seqs):
            if alive[i]:
                alive[i] = _check_step(step, toks[s], gpu_logits[s], ref_logits[i], reports[i])
        if step == STEPS - 1 or not any(alive):
            break
        cur = [toks.get(s, 0) for s in range(batch)]
        nxt, lgs = model.forward_one(cur)

        def ref_one(i):
            if alive[i]:
                ref_logits[i] = refs[i].forward_one(toks[seqs[i]])
        ts = [threading.Thread(target=ref_one, args=(i,)) for i in range(len(seqs))]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        for s in range(batch):
            toks[s] = int(nxt[s])
            gpu_logits[s] = lgs[s]
    for i, r in enumerate(reports):
        r.setdefault("diverged_at", None)
        print(f"seq {seqs[i]}: identical tokens for "
              f"{STEPS if r['diverged_at'] is None else r['diverged_at']} of {STEPS} steps; "
              f"max logit error {r['max_logit_err']:.3e} "
              f"({r['max_rel_err']:.2e} of max |logit|)"
              + ("" if r["diverged_at"] is None else
                 f"; divergence at top-2 margin {r['margin']:.3e} <= error {r['err']:.3e}"))
    return reports


def test_config3_llama_q4_k_batch1_512_prompt(ctx):
    cfg = synth.lm_config("llama-3.2-1b")
    w = _weights(cfg, "Q4_K")
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, cfg["architecture"]["vocab_size"], 512).tolist()
    model = sb.Model(ctx, cfg, w, 512 + STEPS + 8)
    ref = OracleLM(cfg, w, 512 + STEPS + 8, threads=THREADS)
    del w
    _run_batch(model, [ref], [prompt], [0])
    model.close()


def test_config3_llama_q4_k_batch8(ctx):
    cfg = synth.lm_config("llama-3.2-1b")
    w = _weights(cfg, "Q4_K")
    rng = np.random.default_rng(4321)
    prompts = [rng.integers(0, cfg["architecture"]["vocab_size"], 64).tolist() for _ in range(8)]
    model = sb.Model(ctx, cfg, w, 64 + STEPS + 8, max_batch=8)
    base = OracleLM(cfg, w, 64 + STEPS + 8, threads=max(1, THREADS // 8))
    del w
    refs = [base] + [base.fork() for _ in range(7)]
    _run_batch(model, refs, prompts, list(range(8)))
    model.close()


def test_config4_mistral_q4_0_tp1(ctx):
    try:
        import psutil
        if psutil.virtual_memory().available < 48 * 2 ** 30:
            pytest.skip("the f32 oracle of the 7B shape needs about 40 GB of host memory")
    except ImportError:
        pass
    cfg = synth.lm_config("mistral-7b")
    w = _weights(cfg, "Q4_0")
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, cfg["architecture"]["vocab_size"], 32).tolist()
    model = sb.Model(ctx, cfg, w, 32 + STEPS + 8)
    ref = OracleLM(cfg, w, 32 + STEPS + 8, threads=THREADS)
    del w
    _run_batch(model, [ref], [prompt], [0])
    model.close()


def test_config5_qwen3_q8_0_serving_32(ctx):
    cfg = synth.lm_config("qwen3-0.6b")
    w = _weights(cfg, "Q8_0")
    V = cfg["architecture"]["vocab_size"]
    rng = np.random.default_rng(1234)
    lens = rng.integers(128, 2049, 32)
    prompts = [rng.integers(0, V, int(n)).tolist() for n in lens]
    checked = sorted(np.argsort(lens)[:3].tolist())
    model = sb.Model(ctx, cfg, w, 2048 + STEPS + 8, max_batch=32)
    base = OracleLM(cfg, w, int(lens[checked].max()) + STEPS + 8, threads=max(1, THREADS // 3))
    del w
    refs = [base] + [base.fork() for _ in range(len(checked) - 1)]
    # the unchecked sequences are prefilled on the GPU only
    others = {s: model.forward_prefill(prompts[s], seq=s, want_logits=False)[0]
              for s in range(32) if s not in checked}
    _run_batch(model, refs, [prompts[s] for s in checked], checked, others)
    model.close()
