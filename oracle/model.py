"""CPU restatement of the reference engine's model graphs — TEST INFRASTRUCTURE ONLY.

Mirrors, node for node, QwenModel / GemmaModel / SmolModel::forward
(cactus/models/model_qwen.cpp:51-172, model_gemma.cpp:57-176, model_smol.cpp:43-143),
Model::prefill / Model::decode (cactus/engine/engine_model.cpp:170-297) and
KVCache::update_from_graph (cactus/engine/engine_cache.cpp:101-337), with every
kernel computed by the refcpu restatement. Greedy decode is the graph-level
sample(logits, 0, 0, 0) = first-max argmax (kernel_nn.cpp:451-467).

Reads a model folder written in the reference layout (config.txt + .weights files) with
its own minimal parser (graph_io.cpp:497-566), independent of the product package.
"""
from __future__ import annotations

import math
import os
import struct

import numpy as np

from . import refcpu as R


def read_weights(path):
    buf = open(path, "rb").read()
    if buf[:4] != b"CACT":
        raise ValueError("Invalid tensor file: missing CACT magic number")
    _, _, alignment, ndim = struct.unpack_from("<IIII", buf, 4)
    dims = struct.unpack_from("<QQQQ", buf, 20)
    prec, = struct.unpack_from("<I", buf, 52)
    nbytes, sbytes = struct.unpack_from("<QQ", buf, 56)
    G, ng = struct.unpack_from("<II", buf, 72)
    alignment = alignment or 1
    al = lambda o: (o + alignment - 1) // alignment * alignment
    shape = tuple(int(d) for i, d in enumerate(dims) if i < ndim and d > 0)
    hdr = al(80)
    doff = al(hdr + sbytes) if sbytes else hdr
    scales = np.frombuffer(buf, np.float16, sbytes // 2, hdr).reshape(-1, ng) if sbytes else None
    raw = np.frombuffer(buf, np.uint8, nbytes, doff)
    if prec == 0:
        return {"prec": "INT8", "data": raw.view(np.int8).reshape(shape), "scales": scales, "G": G}
    if prec == 3:
        return {"prec": "INT4", "data": raw.reshape(shape[0], -1), "scales": scales, "G": G, "shape": shape}
    if prec == 1:
        return {"prec": "FP16", "data": raw.view(np.float16).reshape(shape)}
    raise ValueError(f"unsupported precision {prec}")


def read_config(folder):
    cfg = {"vocab_size": 151936, "num_layers": 28, "hidden_dim": 1024, "ffn_intermediate_dim": 3072,
           "attention_heads": 16, "attention_kv_heads": 8, "attention_head_dim": 128, "layer_norm_eps": 1e-6,
           "rope_theta": 1e6, "tie_word_embeddings": True, "model_type": "qwen"}
    for line in open(os.path.join(folder, "config.txt")):
        line = line.strip()
        if not line or line.startswith("#") or "=" not in line:
            continue
        k, v = (s.strip() for s in line.split("=", 1))
        if k in ("layer_norm_eps", "rope_theta"):
            cfg[k] = float(v)
        elif k == "tie_word_embeddings":
            cfg[k] = v in ("true", "1")
        elif k == "model_type":
            cfg[k] = v.lower()
        elif k in cfg:
            cfg[k] = int(v)
    return cfg


class RefKVCache:
    """KVCache (engine.h:325-382, engine_cache.cpp:25-337): INT8 per (token, head, 128-group)."""

    def __init__(self, layers, kv_heads, head_dim, window=512, sink=4):
        self.L, self.H, self.D = layers, kv_heads, head_dim
        self.window, self.sink = window, sink
        self.k = [None] * layers
        self.v = [None] * layers
        self.ks = [None] * layers
        self.vs = [None] * layers
        self.current = 0
        self.total = 0

    def reset(self):
        self.current = 0
        self.total = 0

    def update(self, k_nodes, v_nodes, seq_len):
        old = self.current
        new_total = old + seq_len
        self.total += seq_len
        sliding = self.window > 0 and new_total > self.window
        for l in range(self.L):
            kn = k_nodes[l].reshape(-1, self.H, self.D)
            vn = v_nodes[l].reshape(-1, self.H, self.D)
            kq, ksc = R.quantize_kv(kn)
            vq, vsc = R.quantize_kv(vn)
            if kn.shape[0] == new_total:  # first branch: node holds the whole sequence
                if not sliding:
                    self.k[l], self.v[l], self.ks[l], self.vs[l] = kq, vq, ksc, vsc
                else:
                    skip = new_total - self.window
                    rw = self.window - self.sink
                    sel = np.r_[0:self.sink, self.sink + skip:self.sink + skip + rw]
                    self.k[l], self.v[l] = kq[sel], vq[sel]
                    self.ks[l], self.vs[l] = ksc[sel], vsc[sel]
            else:  # incremental branch
                if not sliding:
                    cat = lambda a, b: b if a is None or old == 0 else np.concatenate([a[:old], b], 0)
                    self.k[l], self.v[l] = cat(self.k[l], kq), cat(self.v[l], vq)
                    self.ks[l], self.vs[l] = cat(self.ks[l], ksc), cat(self.vs[l], vsc)
                else:
                    W = self.window
                    def grow(a, fill):
                        if a.shape[0] < W:
                            pad = np.full((W - a.shape[0],) + a.shape[1:], fill, a.dtype)
                            a = np.concatenate([a, pad], 0)
                        return a.copy()
                    arrs = [grow(self.k[l], 0), grow(self.v[l], 0), grow(self.ks[l], 1), grow(self.vs[l], 1)]
                    tts = W - self.sink - seq_len
                    if tts > 0 and old > self.sink:
                        src = old - tts
                        if src > self.sink:
                            for a in arrs:
                                a[self.sink:self.sink + tts] = a[src:src + tts].copy()
                    app = W - seq_len
                    for a, n in zip(arrs, (kq, vq, ksc, vsc)):
                        a[app:app + seq_len] = n
                    self.k[l], self.v[l], self.ks[l], self.vs[l] = arrs
        self.current = self.window if sliding else new_total


class RefModel:
    def __init__(self, folder, context_size=512, window=None, sink=4, causal_fix=False):
        self.cfg = c = read_config(folder)
        self.type = c["model_type"]
        rd = lambda n: read_weights(os.path.join(folder, n))
        self.embed = rd("token_embeddings.weights")
        self.out_norm = rd("output_norm.weights")["data"]
        self.lm = self.embed if c["tie_word_embeddings"] else rd("output_weight.weights")
        self.layers = []
        for i in range(c["num_layers"]):
            p = f"layer_{i}_"
            lw = {k: rd(p + k + ".weights") for k in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate",
                                                      "ffn_up", "ffn_down")}
            for k in ("input_norm", "post_attn_norm"):
                lw[k] = rd(p + k + ".weights")["data"]
            if self.type in ("qwen", "gemma"):
                lw["attn_q_norm"] = rd(p + "attn_q_norm.weights")["data"]
                lw["attn_k_norm"] = rd(p + "attn_k_norm.weights")["data"]
            if self.type == "gemma":
                lw["pre_ffn_norm"] = rd(p + "pre_ffn_norm.weights")["data"]
                lw["post_ffn_norm"] = rd(p + "post_ffn_norm.weights")["data"]
            self.layers.append(lw)
        self.H, self.D = c["hidden_dim"], c["attention_head_dim"]
        self.Hq, self.Hkv = c["attention_heads"], c["attention_kv_heads"]
        self.eps = c["layer_norm_eps"]
        self.scale = 1.0 / math.sqrt(256.0) if self.type == "gemma" else 1.0 / math.sqrt(self.D)
        w = min(context_size, 512) if window is None else window
        if self.type == "gemma":
            w, sink = 0, 0  # GemmaModel::post_init (model_gemma.cpp:17-19)
        self.kv = RefKVCache(c["num_layers"], self.Hkv, self.D, w, sink)
        self.last_logits = None
        # causal-correct masking after the window slid (an option of the device engine, not
        # of the reference: there the mask uses the total position)
        self.causal_fix = causal_fix

    # ---- kernels on graph nodes
    def linear(self, x, w):
        if w["prec"] == "FP16":
            return R.matmul_f16(x, w["data"])
        q, s = R.quantize_activations(x)
        if w["prec"] == "INT8":
            return R.matmul_int8(q, s, w["data"], w["scales"], w["G"])
        return R.matmul_int4(q, s, w["data"], w["scales"], w["G"])

    def embedding(self, tokens):
        e = self.embed
        ids = np.asarray(tokens, np.uint32)
        if e["prec"] == "FP16":
            return R.embedding_f16(e["data"], ids)
        if e["prec"] == "INT8":
            return R.embedding_int8(e["data"], e["scales"], e["G"], ids)
        V, H = e["shape"]
        rows = np.stack([R.unpack_int4(e["data"][i], H) for i in ids]).astype(np.int8)
        return R.embedding_int8(rows, e["scales"][ids], e["G"], np.arange(len(ids), dtype=np.uint32))

    def is_global(self, l):
        return self.type == "gemma" and ((l + 1) % 6) == 0

    # ---- one graph execution (forward with use_cache=True)
    def forward(self, tokens):
        S = len(tokens)
        pos = self.kv.total
        hidden = self.embedding(tokens)
        if self.type == "gemma":
            hidden = R.scalar_multiply(hidden, math.sqrt(self.H))
        k_nodes, v_nodes = [], []
        for l, lw in enumerate(self.layers):
            xn = R.rms_norm(hidden, lw["input_norm"], self.eps)
            q = self.linear(xn, lw["attn_q"])
            k = self.linear(xn, lw["attn_k"])
            v = self.linear(xn, lw["attn_v"])
            if self.type in ("qwen", "gemma"):
                q = R.rms_norm(q.reshape(S * self.Hq, self.D), lw["attn_q_norm"], self.eps)
                k = R.rms_norm(k.reshape(S * self.Hkv, self.D), lw["attn_k_norm"], self.eps)
            q4 = q.reshape(1, S, self.Hq, self.D)
            k4 = k.reshape(1, S, self.Hkv, self.D)
            v4 = v.reshape(1, S, self.Hkv, self.D)
            theta = (1e6 if self.is_global(l) else 1e4) if self.type == "gemma" else self.cfg["rope_theta"]
            if self.cfg["rope_theta"] > 0:
                q4 = R.rope(q4, pos, theta)
                k4 = R.rope(k4, pos, theta)
            k_nodes.append(k4)
            v_nodes.append(v4)
            if self.kv.current > 0:
                n = self.kv.current
                attn = R.attention_hybrid(q4, self.kv.k[l][:n], self.kv.v[l][:n], self.kv.ks[l][:n],
                                          self.kv.vs[l][:n], k4, v4, self.scale, n if self.causal_fix else pos)
            else:
                win = 512 if (self.type == "gemma" and not self.is_global(l)) else 0
                attn = R.attention(q4, k4, v4, self.scale, pos, win, True)
            o = self.linear(attn.reshape(S, self.Hq * self.D), lw["attn_output"])
            if self.type == "gemma":
                h1 = R.add_clipped(hidden, R.rms_norm(o, lw["post_attn_norm"], self.eps))
                pm = R.rms_norm(h1, lw["pre_ffn_norm"], self.eps)
                g = R.multiply(R.gelu(self.linear(pm, lw["ffn_gate"])), self.linear(pm, lw["ffn_up"]))
                d = self.linear(g, lw["ffn_down"])
                hidden = R.add_clipped(h1, R.rms_norm(d, lw["post_ffn_norm"], self.eps))
            else:
                h1 = R.add(hidden, o)
                n2 = R.rms_norm(h1, lw["post_attn_norm"], self.eps)
                g = R.multiply(R.silu(self.linear(n2, lw["ffn_gate"])), self.linear(n2, lw["ffn_up"]))
                hidden = R.add(h1, self.linear(g, lw["ffn_down"]))
        final = R.rms_norm(hidden, self.out_norm, self.eps)
        return final, k_nodes, v_nodes

    def prefill(self, tokens, chunk=256):
        tokens = list(tokens)
        if not tokens:
            return
        def run(ch):
            _, kn, vn = self.forward(ch)
            self.kv.update(kn, vn, len(ch))
        if len(tokens) <= chunk:
            run(tokens)
            return
        full = (len(tokens) - 1) // chunk
        for c in range(full):
            run(tokens[c * chunk:(c + 1) * chunk])
        run(tokens[full * chunk:])

    def decode_argmax(self, tokens):
        final, kn, vn = self.forward(list(tokens))
        last = final[-1:].copy()
        self.last_logits = self.linear(last, self.lm)[0]
        self.kv.update(kn, vn, len(tokens))
        return R.argmax(self.last_logits)

    def generate_greedy(self, prompt, max_new):
        self.kv.reset()
        prompt = list(prompt)
        if len(prompt) > 1:
            self.prefill(prompt[:-1])
        out = []
        tok = prompt[-1]
        for _ in range(max_new):
            tok = self.decode_argmax([tok])
            out.append(tok)
        return out
