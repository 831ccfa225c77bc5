"""Restatement of cactus_sample_f16's non-greedy branch (kernel_nn.cpp:469-651) — TEST
INFRASTRUCTURE ONLY. fp16 arithmetic uses numpy float16 (single rounding of the exact
float32 product), exp is (float)exp((double)x) like the rest of the restatement, and the
uniform sample is passed in (the reference draws it from std::mt19937 seeded by a clock).
"""
import math

import numpy as np

NEG_INF = np.float16(-np.inf)


def _exp(x: np.float32) -> np.float32:
    return np.float32(math.exp(float(np.float32(x))))


def sample_f16(logits, temperature, top_p, top_k, uniform, history=()):
    logits = np.asarray(logits, np.float16)
    V = logits.size
    if temperature == 0.0 and top_p <= 0.0 and top_k == 0:
        return int(np.argmax(logits.astype(np.float32)))  # first max (strict '>')
    f = logits.copy()
    if temperature > 0:
        inv_t = np.float16(np.float32(1.0) / np.float32(temperature))
        f = (f * inv_t).astype(np.float16)
    if len(history):
        pinv = np.float16(np.float32(1.0) / np.float32(1.1))
        pen = np.float16(1.1)
        for tok in history:
            if tok < V:
                f[tok] = np.float16(f[tok] * (pinv if f[tok] > np.float16(0) else pen))
    if top_k > 0 and top_k < V:
        kth = np.sort(f.astype(np.float32))[::-1][top_k - 1]
        f[f.astype(np.float32) < kth] = NEG_INF
    if 0.0 < top_p < 1.0:
        alive = [i for i in range(V) if f[i] != NEG_INF]
        order = sorted(alive, key=lambda i: (-float(f[i]), i))
        if order:
            mx = f[order[0]]
            probs = [_exp(np.float32(f[i]) - np.float32(mx)) for i in order]
            s = np.float32(0)
            for p in probs:
                s = np.float32(s + p)
            cum = np.float32(0)
            cut = False
            for j, i in enumerate(order):
                cum = np.float32(cum + np.float32(probs[j] / s))
                if cum > np.float32(top_p) and j > 0:
                    cut = True
                if cut:
                    f[i] = NEG_INF
    mx = f.astype(np.float32).max()
    if mx == -np.inf:
        return 0
    probs = np.zeros(V, np.float32)
    s = np.float32(0)
    for i in range(V):
        if f[i] != NEG_INF:
            probs[i] = _exp(np.float32(f[i]) - np.float32(np.float16(mx)))
            s = np.float32(s + probs[i])
    if s == 0:
        return 0
    if np.float32(uniform) <= 0:  # the reference's scan returns index 0 for a zero sample
        return 0
    cum = np.float32(0)
    for i in range(V):
        if probs[i] == 0:
            continue
        cum = np.float32(cum + np.float32(probs[i] / s))
        if cum >= np.float32(uniform):
            return i
    for i in range(V - 1, -1, -1):
        if probs[i] / s > 0:
            return i
    return 0
