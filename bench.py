"""Benchmark of the quantized-matmul decode path (M=1).

One step = one pass of the decode GEMV sweep: every weight format (INT8
W8A8, Q4_0, Q8_0, Q4_K, Q6_K) x N in {1024, 3072, 4096, 11008, 14336} x
K in {1024, 2048, 4096}, M = 1 -- 75 fused dequant GEMVs over ~0.96 GB of
weights resident in HBM (larger than the 126 MB L2, so every step streams
from DRAM). `value` = algorithmic bytes (weights in their reference format +
f32 activations + f32 outputs) / device time, summed over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl synapse|reference]

--impl reference times the CPU oracle restatement of the reference's route
(the reference itself is Zig/Rust and cannot be built here) on all host
threads, on the same workload; it prints the same JSON line.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s + qmatmul HBM GB/s (% of ~8 TB/s peak) at 1/2/4/8 B200"
WORKLOAD = "qmatmul decode sweep M=1: 5 formats x N{1024,3072,4096,11008,14336} x K{1024,2048,4096}"
FALLBACK_HBM = 6650.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM, "fallback"


CASE_FILTER = None  # "FMT:N:K" restricts the sweep to one GEMV (profiling runs)


def sweep_cases():
    from synapse_b200 import synth
    from synapse_b200.formats import QFormat
    cases = [(fmt, n, k) for fmt in synth.FORMATS for n in synth.SWEEP_N for k in synth.SWEEP_K]
    if CASE_FILTER:
        f, n, k = CASE_FILTER.split(":")
        cases = [(QFormat[f], int(n), int(k))]
    return cases


def case_bytes(fmt, n, k, m=1):
    from synapse_b200 import synth
    return synth.format_bytes(fmt, n, k) + 4 * m * k + 4 * m * n


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def traffic_from_profile(fmt_name):
    """DRAM bytes per algorithmic byte of the dominant kernel from the
    committed ncu summary (profiles/qgemv_traffic.json), if present."""
    p = os.path.join(ROOT, "profiles", "qgemv_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    e = d.get(fmt_name)
    if not e:
        return None
    return float(e["dram_bytes"]) / float(e["algo_bytes"])


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
DECODE_MODEL = "qwen3-0.6b"
DECODE_PROMPT, DECODE_STEPS = 16, 128


def decode_bytes_per_token(cfg, ctx_len):
    """HBM bytes one decode step must read: every linear weight in its
    reference INT8 format (+ f32 per-row scales), the LM head, one embedding
    row, and the f32 K/V of `ctx_len` cached positions in every layer."""
    a, at = cfg["architecture"], cfg["attention"]
    h, L, V = a["hidden_size"], a["num_layers"], a["vocab_size"]
    hd = at["head_dim"]
    qd, kvd = at["num_heads"] * hd, at["num_kv_heads"] * hd
    ff = cfg["ffn"]["intermediate_size"]
    per_layer = sum(n * k + 4 * n for n, k in ((qd + 2 * kvd, h), (h, qd), (2 * ff, h), (h, ff)))
    return L * per_layer + V * h + 4 * V + 4 * h + L * 2 * kvd * 4 * ctx_len


def run_decode(args, local_rank, dist, cpu_leg):
    """Config 1 (Qwen3-0.6B shape, INT8 per-row weights, random init): a
    16-token prompt, then 128 greedy decode steps at batch 1.
    device: syn_cuda_generate (each step one CUDA graph, chained on the
    device); e2e: syn_cuda_decode_step per token (host token in, host token
    out, synchronous)."""
    import torch
    import synapse_b200 as sb
    from synapse_b200 import synth
    cfg = synth.lm_config(DECODE_MODEL)
    w = synth.gen_lm_weights(cfg, "INT8_KN", seed=1234)
    ctx = sb.Context(local_rank)
    max_seq = DECODE_PROMPT + DECODE_STEPS + 8
    m = sb.Model(ctx, cfg, w, max_seq)
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, cfg["architecture"]["vocab_size"], DECODE_PROMPT).tolist()
    res = {}

    def sync_all():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for rep in range(max(1, args.warmup // 3) + 1):  # first passes warm up (graph capture)
        m.reset()
        sync_all()
        t0 = time.perf_counter()
        m.forward_prefill(prompt, want_logits=False)
        t1 = time.perf_counter()
        toks = m.generate(DECODE_STEPS - 1)
        t2 = time.perf_counter()
        res = {"prefill_s": t1 - t0, "decode_s": t2 - t1}
    dec_s = res["decode_s"]
    if dist is not None:
        tt = torch.tensor([dec_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dec_s = float(tt.item())
    world = dist.get_world_size() if dist is not None else 1
    n_dec = DECODE_STEPS - 1
    tok_s = world * n_dec / dec_s
    # e2e: one public-API call per token with host buffers
    m.reset()
    tok, _ = m.forward_prefill(prompt, want_logits=False)
    seq = [tok]
    for _ in range(3):
        nxt, _ = m.forward_one([seq[-1]], want_logits=False)
        seq.append(int(nxt[0]))
    m.reset()
    tok, _ = m.forward_prefill(prompt, want_logits=False)
    sync_all()
    t0 = time.perf_counter()
    seq = [tok]
    for _ in range(n_dec):
        nxt, _ = m.forward_one([seq[-1]], want_logits=False)
        seq.append(int(nxt[0]))
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        tt = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    same = seq[1:] == toks[0].tolist()
    avg_ctx = DECODE_PROMPT + (n_dec + 1) / 2.0
    bpt = decode_bytes_per_token(cfg, avg_ctx)
    peak, src = peaks()
    out = {
        "model": "Qwen3-0.6B shape (28 layers, d 1024, 16/8 heads x 128, ff 3072, vocab 151936), "
                 "random-init N(0,0.02), INT8 per-row W8A8",
        "prompt_tokens": DECODE_PROMPT, "decode_steps": n_dec, "batch": 1,
        "tok_s": round(tok_s, 1), "ms_per_token": round(dec_s / n_dec * 1e3, 4),
        "prefill_tok_s": round(world * DECODE_PROMPT / res["prefill_s"], 1),
        "e2e_tok_s": round(world * n_dec / e2e_s, 1),
        "e2e": {"api": "syn_cuda_decode_step per token", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "device_and_e2e_tokens_identical": bool(same),
        "hbm_bytes_per_token": int(bpt),
        "roofline": {"bound": "hbm", "achieved": round(bpt * n_dec / dec_s / 1e9, 1),
                     "peak": peak, "unit": "GB/s",
                     "frac": round(bpt * n_dec / dec_s / 1e9 / peak, 4), "peak_source": src},
        # per layer: QKV (norm fused), attention, O, gate/up (norm fused),
        # SwiGLU, down; then embedding+norm, LM head (norm fused), argmax
        "gpu_launches_per_token": 6 * cfg["architecture"]["num_layers"] + 3,
    }
    if cpu_leg:
        out["cpu_baseline"] = cpu_decode_sample(cfg, w, prompt)
    m.close()
    ctx.close()
    return out


TP_MODEL, TP_FMT, TP_PROMPT, TP_STEPS = "mistral-7b", "Q4_0", 2048, 512


def run_tp_decode(args, rank, world, local_rank, dist):
    """Config 4 (the Mistral-7B shape, Q4_0 weights, random init): a
    2048-token prefill, then 511 greedy decode steps at batch 1, with the
    model tensor-parallel over all ranks (Megatron split, NCCL all-reduce
    after O and down, logits all-gather). Weak in weights per GPU, strong in
    work: the same model on 1, 2, 4, 8 GPUs."""
    import torch
    import synapse_b200 as sb
    from synapse_b200 import synth
    cfg = synth.lm_config(TP_MODEL)
    a = cfg["architecture"]
    ctx = sb.Context(local_rank)
    if world > 1:
        obj = [sb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.tp_init(rank, world, obj[0])

    def gpu_dequant(f, b, n):
        w = sb.QuantizedWeight(ctx, f, b, a["vocab_size"], a["hidden_size"])
        out = w.dequant()
        w.close()
        return out
    w = synth.gen_lm_weights(cfg, TP_FMT, seed=1234, dequant=gpu_dequant)
    m = sb.Model(ctx, cfg, w, TP_PROMPT + TP_STEPS + 8)
    del w
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, a["vocab_size"], TP_PROMPT).tolist()

    def sync_all():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def maxr(v):
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    res = None
    for _ in range(2):  # the first pass captures the decode graph
        m.reset()
        sync_all()
        t0 = time.perf_counter()
        m.forward_prefill(prompt, want_logits=False)
        t1 = time.perf_counter()
        toks = m.generate(TP_STEPS - 1)
        t2 = time.perf_counter()
        res = (maxr(t1 - t0), maxr(t2 - t1), toks)
    pre_s, dec_s, toks = res
    n_dec = TP_STEPS - 1
    # e2e: one public-API call per token (host token in / out)
    m.reset()
    tok, _ = m.forward_prefill(prompt, want_logits=False)
    sync_all()
    t0 = time.perf_counter()
    seq = [tok]
    for _ in range(n_dec):
        nxt, _ = m.forward_one([seq[-1]], want_logits=False)
        seq.append(int(nxt[0]))
    e2e_s = maxr(time.perf_counter() - t0)
    h, L, ff = a["hidden_size"], a["num_layers"], cfg["ffn"]["intermediate_size"]
    at = cfg["attention"]
    qd, kvd = at["num_heads"] * at["head_dim"], at["num_kv_heads"] * at["head_dim"]
    wbytes = (L * ((qd + 2 * kvd) * h + h * qd + 2 * ff * h + h * ff) + a["vocab_size"] * h) \
        * 18 // 32
    ctx_avg = TP_PROMPT + (n_dec + 1) / 2.0
    kv = L * 2 * kvd * 4 * ctx_avg
    per_gpu = (wbytes + kv) / world
    peak, src = peaks()
    out = {
        "model": "Mistral-7B shape (32 layers, d 4096, 32/8 heads x 128, ff 14336, vocab 32000, "
                 "window 4096), random-init Q4_0 blocks",
        "tp": world, "prompt_tokens": TP_PROMPT, "decode_steps": n_dec, "batch": 1,
        "prefill_tok_s": round(TP_PROMPT / pre_s, 1),
        "tok_s": round(n_dec / dec_s, 1), "ms_per_token": round(dec_s / n_dec * 1e3, 4),
        "e2e_tok_s": round(n_dec / e2e_s, 1),
        "device_and_e2e_tokens_identical": bool(seq[1:] == toks[0].tolist()),
        "hbm_bytes_per_token_per_gpu": int(per_gpu),
        "roofline": {"bound": "hbm", "achieved": round(per_gpu * n_dec / dec_s / 1e9, 1),
                     "peak": peak, "unit": "GB/s",
                     "frac": round(per_gpu * n_dec / dec_s / 1e9 / peak, 4), "peak_source": src},
        "prefill_roofline": roof_tensor(lm_prefill_flops(cfg, TP_PROMPT) / pre_s / world),
    }
    m.close()
    ctx.close()
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_lm_sample(cfg, TP_FMT)
    return out


def lm_linear_shapes(cfg):
    """(n, k) of every linear of one decoder layer (reference naming order)."""
    a, at = cfg["architecture"], cfg["attention"]
    h, hd = a["hidden_size"], at["head_dim"]
    qd, kvd = at["num_heads"] * hd, at["num_kv_heads"] * hd
    ff = cfg["ffn"]["intermediate_size"]
    return [(qd, h), (kvd, h), (kvd, h), (h, qd), (ff, h), (ff, h), (h, ff)]


def lm_weight_bytes(cfg, fmt):
    """Bytes of every linear weight plus the LM head in the reference format."""
    from synapse_b200 import synth
    from synapse_b200.formats import QFormat
    f = QFormat[fmt]
    a = cfg["architecture"]
    per_layer = sum(synth.format_bytes(f, n, k) for n, k in lm_linear_shapes(cfg))
    return a["num_layers"] * per_layer + synth.format_bytes(f, a["vocab_size"], a["hidden_size"])


def lm_kv_bytes(cfg, positions):
    """f32 K and V of `positions` cached positions over all layers."""
    at = cfg["attention"]
    return cfg["architecture"]["num_layers"] * 2 * at["num_kv_heads"] * at["head_dim"] * 4 * \
        positions


def lm_prefill_flops(cfg, tokens):
    """2 x linear parameters per token, causal attention (QK^T and PV over
    the visible positions), and the LM head for the last token only."""
    a, at = cfg["architecture"], cfg["attention"]
    params = sum(n * k for n, k in lm_linear_shapes(cfg))
    L = a["num_layers"]
    att = L * at["num_heads"] * at["head_dim"] * 2 * 2 * tokens * (tokens + 1) / 2
    return 2.0 * L * params * tokens + att + 2.0 * a["vocab_size"] * a["hidden_size"]


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def cpu_lm_sample(cfg, fmt, prompt_len=8, decode_steps=3):
    """The oracle restatement of the reference's f32 LM route on 1 core, for
    shapes whose full run takes hours there: one decoder layer plus the
    embedding, final norm and LM head are run on a prompt_len-token prompt
    and decode_steps steps; the LM head is timed alone; the per-layer time is
    scaled to the model's layer count. Prefill is extrapolated linearly in
    tokens (the quadratic attention term is left out, which favours the
    CPU), decode at a prompt_len-token context."""
    import copy
    from oracle import oracle as O
    from oracle.lm import OracleLM
    from synapse_b200 import synth
    L = cfg["architecture"]["num_layers"]
    one = copy.deepcopy(cfg)
    one["architecture"]["num_layers"] = 1
    dq = (lambda f, b, n: O.dequant(f.name, b, n)[1]) if fmt != "INT8_KN" else None
    w = synth.gen_lm_weights(one, fmt, seed=1234, dequant=dq)
    lm = OracleLM(one, w, prompt_len + decode_steps + 4)
    V = cfg["architecture"]["vocab_size"]
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, V, prompt_len).tolist()
    lm.forward_prefill(prompt)  # first touch of the weights
    lm.reset()
    t0 = time.perf_counter()
    logits = lm.forward_prefill(prompt)
    t_pre = time.perf_counter() - t0
    tok = int(np.argmax(logits))
    t0 = time.perf_counter()
    for _ in range(decode_steps):
        tok = int(np.argmax(lm.forward_one(tok)))
    t_dec = (time.perf_counter() - t0) / decode_steps
    head = lm.lm_head
    x = np.ones(cfg["architecture"]["hidden_size"], np.float32)
    t0 = time.perf_counter()
    for _ in range(decode_steps):
        head.forward(x, 1)
    t_head = (time.perf_counter() - t0) / decode_steps
    dec_full = t_head + L * max(t_dec - t_head, 0.0)
    pre_full = t_head + L * max(t_pre - t_head, 0.0)
    del w, lm, head
    return {"decode_tok_s": round(1.0 / dec_full, 4),
            "prefill_tok_s": round(prompt_len / pre_full, 4),
            "cores": 1, "kind": "port",
            "sample": f"oracle f32 route, 1 of {L} layers + LM head, {prompt_len}-token prompt "
                      f"and {decode_steps} decode steps on 1 thread; extrapolated to {L} layers "
                      "(prefill linear in tokens, decode at a short context)"}


def cpu_decode_sample(cfg, w, prompt, budget_s=20.0):
    """The oracle restatement of QuantizedCausalLM (oracle/lm.py) on 1 core:
    the same prompt, then decode steps until ~budget_s."""
    from oracle.lm import OracleLM
    lm = OracleLM(cfg, w, DECODE_PROMPT + 64)
    t0 = time.perf_counter()
    logits = lm.forward_prefill(prompt)
    t1 = time.perf_counter()
    tok = int(np.argmax(logits))
    n = 0
    while time.perf_counter() - t1 < budget_s and n < 32:
        logits = lm.forward_one(tok)
        tok = int(np.argmax(logits))
        n += 1
    t2 = time.perf_counter()
    return {"value": round(n / (t2 - t1), 3), "unit": "tok/s", "cores": 1, "kind": "port",
            "prefill_tok_s": round(len(prompt) / (t1 - t0), 3),
            "sample": f"oracle QuantizedCausalLM restatement, {len(prompt)}-token prefill then "
                      f"{n} decode steps, 1 thread"}


def _timed_generate(m, steps, batch):
    """Device-chained greedy steps (syn_cuda_generate); the first call
    captures the step graph and is not timed."""
    import torch
    m.generate(2, batch=batch)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    m.generate(steps, batch=batch)
    torch.cuda.synchronize()
    return time.perf_counter() - t0


def roof_hbm(bytes_per_s, bytes_per_step):
    peak, src = peaks()
    return {"bound": "hbm", "achieved": round(bytes_per_s / 1e9, 1), "peak": peak,
            "unit": "GB/s", "frac": round(bytes_per_s / 1e9 / peak, 4), "peak_source": src,
            "bytes_per_step": int(bytes_per_step)}


def roof_tensor(flops_per_s):
    peak, src = tensor_peak()
    return {"bound": "tensor", "achieved": round(flops_per_s / 1e12, 1), "peak": peak,
            "unit": "TFLOP/s", "frac": round(flops_per_s / 1e12 / peak, 4),
            "peak_source": src + " bf16 dense (the block formats multiply fp16 operands)"}


def run_configs(local_rank, cpu_leg=False):
    """Configs 3 and 5 of the baseline (random-init weights, seeded random
    prompts), one GPU:
    - 3: the LLaMA-3.2-1B shape with Q4_K weights; a 512-token prompt, then
      256 greedy decode steps at batch 1 and at batch 8 (8 prompts);
    - 5: the Qwen3-0.6B shape with Q8_0 weights serving 32 sequences, prompt
      lengths uniform in [128, 2048], then 256 decode steps each."""
    import torch
    import synapse_b200 as sb
    from synapse_b200 import synth
    ctx = sb.Context(local_rank)
    out = {}
    for key, name, fmt in (("llama_3_2_1b_q4_k", "llama-3.2-1b", "Q4_K"),
                           ("qwen3_0p6b_q8_0_serving", "qwen3-0.6b", "Q8_0")):
        cfg = synth.lm_config(name)
        a = cfg["architecture"]

        def gpu_dequant(f, b, n, a=a):
            w = sb.QuantizedWeight(ctx, f, b, a["vocab_size"], a["hidden_size"])
            o = w.dequant()
            w.close()
            return o
        w = synth.gen_lm_weights(cfg, fmt, seed=1234, dequant=gpu_dequant)
        rng = np.random.default_rng(1234)
        steps = 256
        if key.startswith("llama"):
            P, B = 512, 8
            m = sb.Model(ctx, cfg, w, P + steps + 8, max_batch=B)
            del w
            prompts = [rng.integers(0, a["vocab_size"], P).tolist() for _ in range(B)]
            m.forward_prefill(prompts[0], seq=0, want_logits=False)  # warm-up
            m.reset()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            m.forward_prefill(prompts[0], seq=0, want_logits=False)
            torch.cuda.synchronize()
            pre = time.perf_counter() - t0
            t1 = _timed_generate(m, steps - 3, 1)
            m.reset()
            for i in range(B):
                m.forward_prefill(prompts[i], seq=i, want_logits=False)
            t8 = _timed_generate(m, steps - 3, B)
            n = steps - 3
            wb = lm_weight_bytes(cfg, fmt)
            kv = lm_kv_bytes(cfg, P + 2 + n / 2.0)
            b1, b8 = wb + kv, wb + B * kv
            out[key] = {"prompt_tokens": P, "prefill_tok_s": round(P / pre, 1),
                        "decode_tok_s_batch1": round(n / t1, 1),
                        "decode_tok_s_batch8": round(B * n / t8, 1),
                        "timed_steps": n,
                        "roofline": {
                            "decode_batch1": roof_hbm(b1 * n / t1, b1),
                            "decode_batch8": roof_hbm(b8 * n / t8, b8),
                            "prefill": roof_tensor(lm_prefill_flops(cfg, P) / pre)}}
            if cpu_leg:
                out[key]["cpu_baseline"] = cpu_lm_sample(cfg, fmt)
        else:
            B = 32
            m = sb.Model(ctx, cfg, w, 2048 + steps + 8, max_batch=B)
            del w
            lens = rng.integers(128, 2049, B)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for i in range(B):
                m.forward_prefill(rng.integers(0, a["vocab_size"], int(lens[i])).tolist(), seq=i,
                                  want_logits=False)
            torch.cuda.synchronize()
            pre = time.perf_counter() - t0
            td = _timed_generate(m, steps - 3, B)
            n = steps - 3
            # KV positions read per step: each sequence's prompt, the two
            # warm-up tokens and on average half of the timed steps
            bstep = lm_weight_bytes(cfg, fmt) + lm_kv_bytes(cfg, float(lens.sum()) +
                                                           B * (2 + n / 2.0))
            out[key] = {"sequences": B, "prompt_tokens_total": int(lens.sum()),
                        "prefill_tok_s": round(float(lens.sum()) / pre, 1),
                        "decode_tok_s": round(B * n / td, 1),
                        "ms_per_step": round(td / n * 1e3, 3),
                        "timed_steps": n,
                        "roofline": {"decode": roof_hbm(bstep * n / td, bstep)}}
        m.close()
    ctx.close()
    return out


def run_config2_batched(local_rank, reps=5):
    """Config 2 at M = 16, 128 and 512: every (format, N, K) of the decode
    sweep as a batched matmul through the public QuantizedWeight.matmul (the
    tcgen05 GEMMs; M = 16 may take the GEMV). Per (format, M): the 15 shapes
    back to back, `reps` timed passes with the L2 flushed between passes
    (CUDA events around the matmuls only). M = 16 is reported against HBM
    (weight bytes), M = 128 / 512 against the tensor pipe (INT8 kind::i8
    against twice the measured bf16 peak, the nominal dense int8 rate)."""
    import torch
    import synapse_b200 as sb
    from synapse_b200 import synth
    ctx = sb.Context(local_rank)
    rng = np.random.default_rng(4321)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    out = {}
    hbm_peak, _ = peaks()
    for fmt in synth.FORMATS:
        ws = []
        for n in synth.SWEEP_N:
            for k in synth.SWEEP_K:
                data, scales = synth.gen_weight(fmt, n, k, rng)
                ws.append((sb.QuantizedWeight(ctx, fmt, data, n, k, scales), n, k))
        wbytes = sum(synth.format_bytes(fmt, n, k) for _, n, k in ws)
        for m in (16, 128, 512):
            xs = {k: torch.from_numpy(synth.gen_activations(m, k, rng)).cuda()
                  for k in synth.SWEEP_K}
            ys = [torch.empty(m, n, device="cuda") for _, n, _ in ws]

            def run():
                for (w, n, k), y in zip(ws, ys):
                    w.matmul(xs[k], out=y)
            for _ in range(2):
                run()
            torch.cuda.synchronize()
            ms = 0.0
            for _ in range(reps):
                flush.fill_(1)
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record()
                run()
                e1.record()
                torch.cuda.synchronize()
                ms += e0.elapsed_time(e1)
            sec = ms / 1e3 / reps
            flops = sum(2.0 * m * n * k for _, n, k in ws)
            entry = {"us_per_pass": round(sec * 1e6, 1), "shapes": len(ws),
                     "tflops": round(flops / sec / 1e12, 1)}
            if m == 16:
                entry["roofline"] = roof_hbm(wbytes / sec, wbytes)
            else:
                r = roof_tensor(flops / sec)
                if fmt == sb.QFormat.INT8_KN:
                    r["peak"] = round(2 * r["peak"], 1)
                    r["frac"] = round(r["achieved"] / r["peak"], 4)
                    r["unit"] = "TOP/s"
                    r["peak_source"] = "2x the measured bf16 dense peak (nominal dense int8 rate)"
                entry["roofline"] = r
            out[f"{fmt.name}:M{m}"] = entry
            del xs, ys
        for w, _, _ in ws:
            w.close()
    del flush
    ctx.close()
    return {"workload": "config 2: 5 formats x N{1024,3072,4096,11008,14336} x K{1024,2048,4096} "
                        "at M 16/128/512, one pass = the 15 shapes of a format",
            "l2": "flushed (256 MB write) between timed passes", "per_format_m": out}


def run_gemm_case(args):
    """--gemm FMT:M:N:K: times one prefill matmul (tcgen05 GEMM) on cuda:0 and
    prints its TFLOP/s (profiling aid; not the benchmark line)."""
    import torch
    import synapse_b200 as sb
    from synapse_b200 import synth
    f, m, n, k = args.gemm.split(":")
    m, n, k = int(m), int(n), int(k)
    fmt = sb.QFormat[f]
    ctx = sb.Context(0)
    rng = np.random.default_rng(1234)
    data, scales = synth.gen_weight(fmt, n, k, rng)
    w = sb.QuantizedWeight(ctx, fmt, data, n, k, scales)
    x = torch.from_numpy(synth.gen_activations(m, k, rng)).cuda()
    y = torch.empty(m, n, device="cuda")
    for _ in range(args.warmup):
        w.matmul(x, out=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(args.steps):
        w.matmul(x, out=y)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"gemm": args.gemm, "us": round(us, 2),
                      "tflops": round(2 * m * n * k / us / 1e6, 1)}), flush=True)


def run_attn_case(args):
    """--attn MODE:B:L:HQ:HKV:HD: times one decode-attention launch on cuda:0
    (MODE exact = the reference-order kernel, flash = the block-format
    models' grouped kernel) for B rows whose caches hold L-1 positions, and
    prints the KV bytes it must read per second (profiling aid; not the
    benchmark line)."""
    import torch
    import synapse_b200 as sb
    mode, b, L, hq, hkv, hd = args.attn.split(":")
    b, L, hq, hkv, hd = int(b), int(L), int(hq), int(hkv), int(hd)
    ctx = sb.Context(0)
    rng = np.random.default_rng(7)
    cache = sb.KVCache(ctx, L + 8, hkv, hd, 1, batch=b)
    kvd, qd = hkv * hd, hq * hd
    for i in range(b):
        kh = torch.from_numpy(rng.standard_normal((L - 1, kvd)).astype(np.float32)).cuda()
        vh = torch.from_numpy(rng.standard_normal((L - 1, kvd)).astype(np.float32)).cuda()
        cache.append(0, kh, vh, seq=i)
        cache.advance(L - 1, seq=i)
    cos, sin = sb.rope_tables(1e6, L + 8, hd)
    cos, sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    qkv = torch.from_numpy(rng.standard_normal((b, qd + 2 * kvd)).astype(np.float32)).cuda()

    def run():
        return sb.attention_decode(cache, 0, qkv, hq, None, None, 1e-6, cos, sin, batch=b,
                                   flash=mode == "flash")
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    kv_bytes = b * L * 2 * kvd * 4
    print(json.dumps({"attn": args.attn, "us": round(us, 2),
                      "kv_GB/s": round(kv_bytes / us / 1e3, 1)}), flush=True)
    cache.close()
    ctx.close()


def run_decode_only(args, local_rank):
    """The config-1 decode leg alone (one process, no sweep, no CPU leg): the
    command the decode-step launch list is taken from."""
    import torch
    torch.cuda.set_device(local_rank)
    out = run_decode(args, local_rank, None, cpu_leg=False)
    print(json.dumps({"decode": out}), flush=True)


def run_tp_decode_only(args, local_rank):
    """The config-4 decode leg alone on one GPU (TP1): the command its
    launch list is taken from."""
    import torch
    torch.cuda.set_device(local_rank)
    out = run_tp_decode(args, 0, 1, local_rank, None)
    print(json.dumps({"tp_decode": out}), flush=True)


def run_synapse(args, rank, world, local_rank):
    import torch
    import synapse_b200 as sb
    from synapse_b200 import synth

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    ctx = sb.Context(local_rank)
    rng = np.random.default_rng(1234)
    cases = []
    for fmt, n, k in sweep_cases():
        data, scales = synth.gen_weight(fmt, n, k, rng)
        w = sb.QuantizedWeight(ctx, fmt, data, n, k, scales)
        x_host = synth.gen_activations(1, k, rng)
        x = torch.from_numpy(x_host).to(dev)
        y = torch.empty(1, n, dtype=torch.float32, device=dev)
        x_pin = torch.from_numpy(x_host).pin_memory()
        y_pin = torch.empty(1, n, dtype=torch.float32).pin_memory()
        cases.append(dict(fmt=fmt, n=n, k=k, w=w, x=x, y=y, x_pin=x_pin, y_pin=y_pin,
                          bytes=case_bytes(fmt, n, k)))
        del data
    step_bytes = sum(c["bytes"] for c in cases)
    stream = torch.cuda.current_stream(dev)
    from synapse_b200.graph import CapturedSequence
    fmt_names = sorted({sb.QFormat(c["fmt"]).name for c in cases},
                       key=lambda nm: int(sb.QFormat[nm]))
    by_fmt = {nm: [c for c in cases if sb.QFormat(c["fmt"]).name == nm] for nm in fmt_names}

    def gemvs(cs):
        def run():
            for c in cs:
                c["w"].matmul(c["x"], out=c["y"])
        return run

    # e2e buffers: per format, the step's activations live in one pinned host
    # buffer and its outputs come back into one, as a caller batching a
    # decode step would hold them; one H2D and one D2H copy per format.
    e2e = {}
    for nm in fmt_names:
        cs = by_fmt[nm]
        kx = sum(c["k"] for c in cs)
        ny = sum(c["n"] for c in cs)
        hx = torch.cat([c["x_pin"].reshape(-1) for c in cs]).pin_memory()
        hy = torch.empty(ny, dtype=torch.float32).pin_memory()
        dx = torch.empty(kx, dtype=torch.float32, device=dev)
        dy = torch.empty(ny, dtype=torch.float32, device=dev)
        views, ox, oy = [], 0, 0
        for c in cs:
            views.append((c, dx[ox:ox + c["k"]].view(1, -1), dy[oy:oy + c["n"]].view(1, -1)))
            ox += c["k"]
            oy += c["n"]
        e2e[nm] = (hx, hy, dx, dy, views)

    def gemvs_e2e(nm):
        hx, hy, dx, dy, views = e2e[nm]

        def run():
            dx.copy_(hx, non_blocking=True)
            for c, xv, yv in views:
                c["w"].matmul(xv, out=yv)
            hy.copy_(dy, non_blocking=True)
        return run

    # One CUDA graph per format (15 GEMVs each); a step replays the five.
    graphs = {nm: CapturedSequence(gemvs(by_fmt[nm]), dev) for nm in fmt_names}
    graphs_e2e = {nm: CapturedSequence(gemvs_e2e(nm), dev) for nm in fmt_names}

    def barrier():
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def timed(gs):
        """K timed steps of replays; returns (total ms, per-format ms)."""
        for _ in range(args.warmup):
            for nm in fmt_names:
                gs[nm].replay()
        barrier()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(fmt_names) + 1)]
              for _ in range(args.steps)]
        barrier()
        # Keep the device busy while the host enqueues every replay, so the
        # timed region measures device time, not host submission latency.
        torch.cuda._sleep(20_000_000)
        for s in range(args.steps):
            ev[s][0].record(stream)
            for i, nm in enumerate(fmt_names):
                gs[nm].replay()
                ev[s][i + 1].record(stream)
        barrier()
        total = ev[0][0].elapsed_time(ev[-1][-1])
        per = {nm: sum(ev[s][i].elapsed_time(ev[s][i + 1]) for s in range(args.steps))
               for i, nm in enumerate(fmt_names)}
        return total, per

    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    ms, fmt_ms = timed(graphs)
    clk = clocks.stop()
    if dist is not None:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_per_step = ms / args.steps
    value = world * step_bytes * args.steps / (ms / 1e3) / 1e9

    fmt_bytes = {nm: args.steps * sum(c["bytes"] for c in by_fmt[nm]) for nm in fmt_names}
    per_format = {nm: {"GB/s": round(fmt_bytes[nm] / (fmt_ms[nm] / 1e3) / 1e9, 1),
                       "ms_per_step": round(fmt_ms[nm] / args.steps, 4)} for nm in fmt_names}
    dom = max(fmt_ms, key=fmt_ms.get)
    launches_dom = len(by_fmt[dom])
    achieved = fmt_bytes[dom] / (fmt_ms[dom] / 1e3) / 1e9
    peak, peak_src = peaks()
    ratio = traffic_from_profile(dom)
    traffic = None
    if ratio is not None:
        traffic = ratio * (fmt_bytes[dom] / args.steps / launches_dom)

    # e2e: the public API with host buffers (pinned): every step copies each
    # GEMV's x host->device and reads its y back device->host.
    ems, _ = timed(graphs_e2e)
    if dist is not None:
        tt = torch.tensor([ems], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ems = float(tt.item())
    e2e_value = world * step_bytes * args.steps / (ems / 1e3) / 1e9
    h2d = sum(4 * c["k"] for c in cases)
    d2h = sum(4 * c["n"] for c in cases)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample()
    decode = None
    tp_decode = None
    if not args.no_decode:
        decode = run_decode(args, local_rank, dist,
                            cpu_leg=rank == 0 and world == 1 and not args.no_cpu_baseline)
        tp_decode = run_tp_decode(args, rank, world, local_rank, dist)
    configs = None
    config2 = None
    if not args.no_decode and world == 1 and not args.no_configs:
        configs = run_configs(local_rank, cpu_leg=not args.no_cpu_baseline)
        config2 = run_config2_batched(local_rank)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 W8A8 (INT8); int16-split activations x 4/6/8-bit codes (block formats)",
            "dtype_detail": "INT8: int8 x int8 -> int32 as the reference. Block formats: each f32 "
                            "activation block is rounded to a 16-bit integer (per-block scale, "
                            "split into two byte planes) and dotted with the packed codes as "
                            "exact int32 block sums, then f32 accumulation; normwise error "
                            "<= 1e-3 against the reference's f32 route",
            "data": "synthetic (seeded PCG64; codes uniform, f16 scales |N(0,0.01)|, x N(0,1))",
            "config": {"workload": WORKLOAD, "m": 1, "formats": 5, "shapes": 15,
                       "weight_bytes_per_step": int(sum(c["w"].format_bytes for c in cases)),
                       "l2": "inputs larger than L2 (0.96 GB of weights per step)",
                       "parallelism": f"replicas x{world}"},
            "hbm_frac": round(value / world / peak, 4),
            "per_format": per_format,
            "roofline": {"bound": "hbm", "kernel": f"k_qgemv<{dom}> ({launches_dom} launches/step)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "traffic": traffic},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": len(cases) * args.steps,
            "launch": "one CUDA graph per format (15 GEMVs), 5 replays per step",
            "clocks": clk,
            "cpu_baseline": cpu,
            "decode": decode,
            "tp_decode": tp_decode,
            "configs_3_5": configs,
            "config_2_batched": config2,
            # the multi-GPU work of this path: config-4 tensor-parallel decode
            # over all N ranks (TP1 at N=1); `value` stays the sharded sweep
            "tp_decode_tok_s": tp_decode["tok_s"] if tp_decode else None,
            "tp_decode_roofline_frac": tp_decode["roofline"]["frac"] if tp_decode else None,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU legs (the oracle restatement of the reference's route)
# ---------------------------------------------------------------------------
class RefRoute:
    """Per-case CPU work of the reference's own route for one M=1 GEMV:
    INT8: quantize_per_channel_int8 + qgemm_int8 (int8_linear.rs:87-117);
    Q4_0: syn_q4_0_gemv (qmatmul.zig:276-343); Q8_0/Q4_K/Q6_K: dequantised
    at load (gguf.rs), then f32 matmul_t (matmul.zig:223-300)."""

    def __init__(self, fmt, n, k, rng):
        from synapse_b200 import synth
        from synapse_b200.formats import QFormat
        from oracle import oracle
        self.o = oracle
        self.fmt, self.n, self.k = QFormat(fmt), n, k
        self.data, self.scales = synth.gen_weight(fmt, n, k, rng)
        self.x = synth.gen_activations(1, k, rng).reshape(-1)
        self.bytes = case_bytes(fmt, n, k)
        if self.fmt in (QFormat.Q8_0, QFormat.Q4_K, QFormat.Q6_K):
            st, self.wf = oracle.dequant(int(self.fmt), self.data, n * k)
        self.x = np.ascontiguousarray(self.x)
        self.y = np.zeros(n, np.float32)

    def run(self, r0, r1):
        """Rows [r0, r1) of the output (threads split rows), on raw pointers
        so that no copy lands inside the timed region."""
        import ctypes
        from synapse_b200.formats import QFormat
        lib = self.o._load(fast=True)
        n, k, rows = self.n, self.k, r1 - r0
        P = lambda a, off=0: ctypes.c_void_p(a.ctypes.data + off)  # noqa: E731
        y = self.y
        if self.fmt == QFormat.INT8_KN:
            xq = np.empty(k, np.int8)
            xs = np.empty(1, np.float32)
            lib.orc_quantize_per_channel_int8(P(self.x), 1, k, P(xq), P(xs))
            lib.orc_qgemm_int8(1, rows, k, P(xq), k, P(self.data, r0), n, P(y, 4 * r0), n,
                               P(xs), P(self.scales, 4 * r0))
        elif self.fmt == QFormat.Q4_0:
            rb = k // 32 * 18
            lib.orc_q4_0_gemv(rows, k, P(self.x), P(self.data, r0 * rb), P(y, 4 * r0))
        else:
            lib.orc_sgemm_nt(1, rows, k, P(self.x), k, P(self.wf, 4 * r0 * k), k, P(y, 4 * r0), n)


def run_ref_step(routes, threads):
    if threads <= 1:
        for r in routes:
            r.run(0, r.n)
        return
    for r in routes:
        chunk = (r.n + threads - 1) // threads
        ts = [threading.Thread(target=r.run, args=(i * chunk, min(r.n, (i + 1) * chunk)))
              for i in range(threads) if i * chunk < r.n]
        for t in ts:
            t.start()
        for t in ts:
            t.join()


def sample_routes(rng, per_format_shapes):
    from synapse_b200 import synth
    routes = []
    for fmt in synth.FORMATS:
        for (n, k) in per_format_shapes:
            routes.append(RefRoute(fmt, n, k, rng))
    return routes


SAMPLE_SHAPES = [(1024, 1024), (3072, 2048), (4096, 4096), (11008, 4096), (14336, 1024)]


def cpu_baseline_sample(budget_s=10.0):
    """1-core timing of the oracle restatement of the reference's route on
    the whole M=1 sweep (the GPU arm's step), repeated for about budget_s."""
    rng = np.random.default_rng(1234)
    routes = [RefRoute(fmt, n, k, rng) for fmt, n, k in sweep_cases()]
    run_ref_step(routes, 1)
    reps = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or reps < 1:
        run_ref_step(routes, 1)
        reps += 1
    t = time.perf_counter() - t0
    total_b = reps * sum(r.bytes for r in routes)
    return {"value": round(total_b / t / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{reps} pass(es) of the whole step ({len(routes)} GEMVs), oracle -O3 "
                      "build, 1 thread"}


def run_reference(args, rank, world):
    """The reference's CPU route for the same workload as the GPU arm: all 75
    GEMVs of the M=1 sweep per step, same shapes, formats and value
    distributions. The reference's implementation is single-threaded
    (synapse-core's wrappers are !Sync; the Zig kernels run on the calling
    thread), so it runs on one thread pinned to one core. Neither torch nor
    the CUDA library is loaded in this process: the inputs come from
    synapse_b200.synth (numpy only) and the arithmetic from the oracle's
    -O3 build."""
    if rank != 0:
        return
    try:
        cpu = sorted(os.sched_getaffinity(0))[0]
        os.sched_setaffinity(0, {cpu})
    except (AttributeError, OSError):
        cpu = None
    rng = np.random.default_rng(1234)
    routes = [RefRoute(fmt, n, k, rng) for fmt, n, k in sweep_cases()]
    for _ in range(args.warmup):
        run_ref_step(routes, 1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run_ref_step(routes, 1)
    t = time.perf_counter() - t0
    step_bytes = sum(r.bytes for r in routes)
    value = step_bytes * args.steps / t / 1e9
    sample = (f"the whole step: {len(routes)} GEMVs of the M=1 sweep (5 formats x 15 (N,K)), "
              f"oracle -O3 build, 1 thread pinned to cpu {cpu} of {os.cpu_count()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (block formats), int8 (W8A8)",
        "data": "synthetic (seeded PCG64; codes uniform, f16 scales |N(0,0.01)|, x N(0,1))",
        "config": {"workload": WORKLOAD, "m": 1, "formats": 5, "shapes": 15,
                   "same_config": True, "sample": sample},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": 1,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference is Zig + Rust with no toolchain here or on the GPU box: this is "
                "the C restatement of its route (quantize + qgemm_int8, q4_0_gemv, "
                "dequantise-at-load + f32 GEMV), single-threaded as the reference is",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="synapse", choices=["synapse", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the model decode leg")
    ap.add_argument("--case", default=None, help="FMT:N:K -- time one GEMV only (profiling)")
    ap.add_argument("--gemm", default=None, help="FMT:M:N:K -- time one GEMM only (profiling)")
    ap.add_argument("--attn", default=None,
                    help="exact|flash:B:L:HQ:HKV:HD -- time one decode attention (profiling)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the config-3/5 decode legs (LLaMA Q4_K batch 1/8, Qwen3 Q8_0 serving)")
    ap.add_argument("--decode-only", action="store_true",
                    help="run only the config-1 decode leg (profiling one decode step)")
    ap.add_argument("--tp-decode-only", action="store_true",
                    help="the config-4 (Mistral-7B shape) decode leg alone on one GPU")
    args = ap.parse_args()
    global CASE_FILTER
    CASE_FILTER = args.case
    if args.case:
        args.no_cpu_baseline = True
        args.no_decode = True
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.gemm:
        run_gemm_case(args)
    elif args.attn:
        run_attn_case(args)
    elif args.decode_only:
        run_decode_only(args, local_rank)
    elif args.tp_decode_only:
        run_tp_decode_only(args, local_rank)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_synapse(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
