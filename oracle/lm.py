"""CPU oracle of the reference's decoder-only LM forward (TEST INFRASTRUCTURE
ONLY: used by tests/ and bench.py's CPU-baseline legs as the checker; the
shipped CUDA path never imports it).

Restates, step for step:
  * QuantizedCausalLM::{forward_prefill, forward_one} and
    QuantizedDecoderLayer (quantization/lm/int8.rs:171-709) for INT8 weights
    (W8A8: activations quantized per call, a1, then qgemm_int8);
  * CausalLM::{forward_prefill, forward_one} and the f32 DecoderLayer
    (models/lm/causal_lm.rs:195-280, models/lm/decoder_layer.rs:590-730) for
    the block formats, whose weights the reference dequantizes to f32 at load
    (weight_loading/gguf.rs:126-147) and multiplies with matmul_t;
  * cached_attention_{decode,prefill} (ops/attention.rs:24-247) and the KV
    cache (kv_cache/cache.rs, zig/src/ops/kvcache.zig:13-170).
The arithmetic lives in liboracle (synapse_oracle*.c); this file is the
orchestration.

Weights use the Hugging Face tensor names that the reference's weight map
reads. Linear weights are given as
  ("INT8_KN", q_kn int8 [K*N], scales f32 [N])     (int8_linear.rs:7-18 layout)
  (fmt, blocks uint8)                               (raw GGUF block rows)
and norms / the embedding as f32 arrays.
"""
import numpy as np

from . import oracle as O


def layer_names(i):
    p = f"model.layers.{i}."
    return {
        "attn_norm": p + "input_layernorm.weight",
        "ffn_norm": p + "post_attention_layernorm.weight",
        "q_norm": p + "self_attn.q_norm.weight",
        "k_norm": p + "self_attn.k_norm.weight",
        "wq": p + "self_attn.q_proj.weight",
        "wk": p + "self_attn.k_proj.weight",
        "wv": p + "self_attn.v_proj.weight",
        "wo": p + "self_attn.o_proj.weight",
        "gate": p + "mlp.gate_proj.weight",
        "up": p + "mlp.up_proj.weight",
        "down": p + "mlp.down_proj.weight",
    }


class _Linear:
    def __init__(self, spec, n, k, threads=1):
        self.n, self.k = n, k
        self.threads = threads
        self.int8 = spec[0] == "INT8_KN"
        if self.int8:
            self.q = np.ascontiguousarray(spec[1], dtype=np.int8)
            self.s = np.ascontiguousarray(spec[2], dtype=np.float32)
        else:
            st, w = O.dequant(spec[0], spec[1], n * k)
            assert st == 0, st
            self.w = w

    def forward(self, x, m):
        """QuantizedLinear::forward (int8_linear.rs:87-130) or matmul_t."""
        if self.int8:
            st, xq, sx = O.quantize_per_channel_int8(x, m, self.k)
            assert st == 0
            return self.forward_pre_quantized(xq, sx, m)
        if self.threads > 1 and self.n >= 128:
            return self._forward_threaded(x, m)
        st, y = O.sgemm_nt(m, self.n, self.k, x, self.w, fast=True)
        assert st == 0
        return y

    def _forward_threaded(self, x, m):
        """The same sgemm split over output columns in slices of whole
        64-column blocks: every output keeps its micro-kernel and its
        summation order (the column blocks of matmul.zig:125-347 start at
        multiples of 8 and 64), so the result is bit-identical to one call.
        The C calls release the GIL."""
        import ctypes
        import threading
        lib = O._load(fast=True)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(m * self.n, np.float32)
        per = (self.n + self.threads - 1) // self.threads
        per = (per + 63) // 64 * 64
        vp = ctypes.c_void_p
        res = []

        def run(r0, r1):
            res.append(lib.orc_sgemm_nt(m, r1 - r0, self.k, vp(x.ctypes.data), self.k,
                                        vp(self.w.ctypes.data + 4 * r0 * self.k), self.k,
                                        vp(y.ctypes.data + 4 * r0), self.n))
        ts = [threading.Thread(target=run, args=(r0, min(self.n, r0 + per)))
              for r0 in range(0, self.n, per)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        assert all(r == 0 for r in res), res
        return y

    def forward_pre_quantized(self, xq, sx, m):
        st, y = O.qgemm_int8(m, self.n, self.k, xq, self.q, sx, self.s, fast=True)
        assert st == 0
        return y


class OracleLM:
    def __init__(self, cfg, weights, max_seq, threads=1):
        a, at = cfg["architecture"], cfg["attention"]
        self.h = a["hidden_size"]
        self.L = a["num_layers"]
        self.V = a["vocab_size"]
        self.Hq, self.Hkv, self.hd = at["num_heads"], at["num_kv_heads"], at["head_dim"]
        self.window = at.get("window_size", 0) if at.get("type") == "SlidingWindow" else 0
        self.ff = cfg["ffn"]["intermediate_size"]
        self.eps = np.float32(cfg["norm"]["eps"])
        self.max_seq = max_seq
        qd, kvd = self.Hq * self.hd, self.Hkv * self.hd
        self.cos, self.sin = O.rope_tables(cfg["position"]["base"], max_seq, self.hd)
        self.embed = np.ascontiguousarray(weights["model.embed_tokens.weight"], np.float32)
        self.final_norm = weights["model.norm.weight"]
        self.layers = []
        for i in range(self.L):
            nm = layer_names(i)
            ly = {
                "attn_norm": weights[nm["attn_norm"]],
                "ffn_norm": weights[nm["ffn_norm"]],
                "q_norm": weights.get(nm["q_norm"], np.zeros(0, np.float32)),
                "k_norm": weights.get(nm["k_norm"], np.zeros(0, np.float32)),
                "wq": _Linear(weights[nm["wq"]], qd, self.h, threads),
                "wk": _Linear(weights[nm["wk"]], kvd, self.h, threads),
                "wv": _Linear(weights[nm["wv"]], kvd, self.h, threads),
                "wo": _Linear(weights[nm["wo"]], self.h, qd, threads),
                "gate": _Linear(weights[nm["gate"]], self.ff, self.h, threads),
                "up": _Linear(weights[nm["up"]], self.ff, self.h, threads),
                "down": _Linear(weights[nm["down"]], self.h, self.ff, threads),
            }
            self.layers.append(ly)
        self.lm_head = _Linear(weights["lm_head.weight"], self.V, self.h, threads)
        self.int8 = self.lm_head.int8
        self.kc = np.zeros((self.L, max_seq, kvd), np.float32)
        self.vc = np.zeros((self.L, max_seq, kvd), np.float32)
        self.pos = 0

    def reset(self):
        self.pos = 0

    def fork(self):
        """Another sequence over the same (read-only) weights: its own empty
        KV cache, so a batch of sequences costs one copy of the f32 weights."""
        import copy
        other = copy.copy(self)
        other.kc = np.zeros_like(self.kc)
        other.vc = np.zeros_like(self.vc)
        other.pos = 0
        return other

    # -- pieces --------------------------------------------------------------
    def _embed(self, ids):
        x = np.zeros((len(ids), self.h), np.float32)
        for t, i in enumerate(ids):
            if i < self.V:
                x[t] = self.embed[i]
        return x.reshape(-1)

    def _headnorm(self, x, w, heads):
        """apply_headwise_rmsnorm (ops/norm.rs:78-92): empty weight = identity."""
        if w is None or len(w) == 0:
            return x.copy()
        return O.rmsnorm(x, w, self.hd, self.eps)

    def _qkv(self, ly, x, m):
        if self.int8:
            st, xq, sx = O.quantize_per_channel_int8(x, m, self.h)
            assert st == 0
            return (ly["wq"].forward_pre_quantized(xq, sx, m),
                    ly["wk"].forward_pre_quantized(xq, sx, m),
                    ly["wv"].forward_pre_quantized(xq, sx, m))
        return ly["wq"].forward(x, m), ly["wk"].forward(x, m), ly["wv"].forward(x, m)

    def _ffn(self, ly, x, m):
        if self.int8:
            st, xq, sx = O.quantize_per_channel_int8(x, m, self.h)
            g = ly["gate"].forward_pre_quantized(xq, sx, m)
            u = ly["up"].forward_pre_quantized(xq, sx, m)
            hid = O.silu_mul(g, u)
        else:
            g, u = ly["gate"].forward(x, m), ly["up"].forward(x, m)
            hid = O.swiglu(g, u)
        return ly["down"].forward(hid, m)

    def _layer_prefill(self, li, x, S):
        ly = self.layers[li]
        qd, kvd = self.Hq * self.hd, self.Hkv * self.hd
        normed = O.rmsnorm(x, ly["attn_norm"], self.h, self.eps)
        q, k, v = self._qkv(ly, normed, S)
        # cached_attention_prefill (ops/attention.rs:153-247)
        q = self._headnorm(q, ly["q_norm"], self.Hq)
        k = self._headnorm(k, ly["k_norm"], self.Hkv)
        O.rope_inplace(q, self.cos, self.sin, S, self.Hq, self.hd, 0)
        O.rope_inplace(k, self.cos, self.sin, S, self.Hkv, self.hd, 0)
        assert self.pos + S <= self.max_seq, "KV cache full"
        self.kc[li, self.pos:self.pos + S] = k.reshape(S, kvd)
        self.vc[li, self.pos:self.pos + S] = v.reshape(S, kvd)
        groups = self.Hq // self.Hkv
        q3 = q.reshape(S, self.Hq, self.hd)
        k3 = k.reshape(S, self.Hkv, self.hd)
        v3 = v.reshape(S, self.Hkv, self.hd)
        att = np.empty((S, self.Hq, self.hd), np.float32)
        for hh in range(self.Hq):
            kvh = hh // groups
            st, o = O.fused_attention(S, S, self.hd, q3[:, hh], k3[:, kvh], v3[:, kvh])
            assert st == 0
            att[:, hh] = o.reshape(S, self.hd)
        attn_out = ly["wo"].forward(att.reshape(-1), S)
        res = (x + attn_out).astype(np.float32)
        normed = O.rmsnorm(res, ly["ffn_norm"], self.h, self.eps)
        return (res + self._ffn(ly, normed, S)).astype(np.float32)

    def _layer_decode(self, li, x, pos):
        ly = self.layers[li]
        kvd = self.Hkv * self.hd
        normed = O.rmsnorm(x, ly["attn_norm"], self.h, self.eps)
        q, k, v = self._qkv(ly, normed, 1)
        # cached_attention_decode (ops/attention.rs:24-147)
        q = self._headnorm(q, ly["q_norm"], self.Hq)
        k = self._headnorm(k, ly["k_norm"], self.Hkv)
        O.rope_inplace(q, self.cos, self.sin, 1, self.Hq, self.hd, pos)
        O.rope_inplace(k, self.cos, self.sin, 1, self.Hkv, self.hd, pos)
        assert pos < self.max_seq, "KV cache full"
        self.kc[li, pos] = k.reshape(kvd)
        self.vc[li, pos] = v.reshape(kvd)
        att = O.attention_decode(q, self.kc[li], self.vc[li], pos + 1, self.Hq, self.Hkv,
                                 self.hd, self.window)
        attn_out = ly["wo"].forward(att, 1)
        res = (x + attn_out).astype(np.float32)
        normed = O.rmsnorm(res, ly["ffn_norm"], self.h, self.eps)
        return (res + self._ffn(ly, normed, 1)).astype(np.float32)

    # -- model API -------------------------------------------------------------
    def forward_prefill(self, ids):
        """Returns the logits of the last prompt token (int8.rs:593-634)."""
        S = len(ids)
        x = self._embed(ids)
        for li in range(self.L):
            x = self._layer_prefill(li, x, S)
        self.pos += S
        last = O.rmsnorm(x[(S - 1) * self.h:], self.final_norm, self.h, self.eps)
        return self.lm_head.forward(last, 1)

    def forward_one(self, token):
        """int8.rs:637-709 / causal_lm.rs forward_one."""
        pos = self.pos
        x = self._embed([token])
        for li in range(self.L):
            x = self._layer_decode(li, x, pos)
        self.pos += 1
        x = O.rmsnorm(x, self.final_norm, self.h, self.eps)
        return self.lm_head.forward(x, 1)

    def generate_greedy(self, prompt, steps):
        """generation/pipeline.rs:197-280 with GreedySampler: the first token
        comes from the prefill logits, each later one from forward_one of the
        previous token. Returns (tokens, top-2 margins)."""
        toks, margins = [], []
        logits = self.forward_prefill(prompt)
        for _ in range(steps):
            t = O.argmax(logits)
            toks.append(t)
            srt = np.sort(logits)
            margins.append(float(srt[-1] - srt[-2]))
            if len(toks) == steps:
                break
            logits = self.forward_one(t)
        return toks, margins
