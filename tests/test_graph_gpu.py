"""The CactusGraph C++ API (include/cactus/graph.h) on the device.

tests/native/graph_api_test.cpp is compiled against libcactus_b200.so and run: it checks
the known answers of the reference's graph tests and builds a quantized attention block
(rms_norm -> INT8 matmuls -> rope -> GQA attention -> INT4 matmul -> residual -> activations
-> INT8 lm head -> index / softmax / greedy sample) from .weights files. Every node it dumps is
compared bit for bit with the same composition of oracle functions.
"""
import os
import subprocess

import numpy as np
import pytest

import cactus_b200 as cb
from cactus_b200 import weights as W
from oracle import refcpu as R

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
M, K, HQ, HKV, D, V, G = 3, 128, 2, 1, 64, 500, 32


def _build(tmp):
    cb.lib()
    exe = os.path.join(tmp, "graph_api_test")
    pkg = os.path.join(ROOT, "cactus_b200")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "native", "graph_api_test.cpp"), "-L", pkg, "-lcactus_b200",
                    f"-Wl,-rpath,{pkg}", "-o", exe], check=True)
    return exe


def _load(path):
    f = W.read_weights(path)
    return np.ascontiguousarray(f.data), np.ascontiguousarray(f.scales)


def test_graph_api(tmp_path):
    d = str(tmp_path)
    rng = np.random.default_rng(11)
    x = rng.standard_normal((M, K)).astype(np.float16)
    x.tofile(os.path.join(d, "x.bin"))
    W.save_tensor(os.path.join(d, "attn_norm.weights"), 1 + 0.1 * rng.standard_normal(K), "INT8")
    for name, shape, prec in (("wq", (HQ * D, K), "INT8"), ("wk", (HKV * D, K), "INT8"), ("wv", (HKV * D, K), "INT8"),
                              ("wo", (K, HQ * D), "INT4"), ("lm", (V, K), "INT8")):
        W.save_tensor(os.path.join(d, f"{name}.weights"), rng.standard_normal(shape) * 0.2, prec, group_size=G)
    W.save_tensor(os.path.join(d, "emb_f16.weights"),
                  np.array([[1, 5, 9], [2, 6, 10], [3, 7, 11], [4, 8, 12]], np.float32), "FP16")

    # inputs of the LFM2 / Whisper / encoder ops (native families())
    x_dw, w_dw = rng.standard_normal((1, 20, 16)).astype(np.float16), (rng.standard_normal((16, 1, 4)) * 0.5).astype(np.float16)
    x_k3, w_k3 = rng.standard_normal((1, 8, 12)).astype(np.float16), (rng.standard_normal((6, 8, 3)) * 0.3).astype(np.float16)
    x_ln = (rng.standard_normal((3, 40)) * 2).astype(np.float16)
    w_ln, b_ln = rng.standard_normal(40).astype(np.float16), (rng.standard_normal(40) * 0.1).astype(np.float16)
    for name, arr in (("x_dw", x_dw), ("w_dw", w_dw), ("x_k3", x_k3), ("w_k3", w_k3), ("x_ln", x_ln), ("w_ln", w_ln),
                      ("b_ln", b_ln)):
        arr.tofile(os.path.join(d, f"{name}.bin"))

    exe = _build(d)
    r = subprocess.run([exe, d], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout and "0 failures" in r.stdout

    nw = W.read_weights(os.path.join(d, "attn_norm.weights")).data
    wq, sq = _load(os.path.join(d, "wq.weights"))
    wk, sk = _load(os.path.join(d, "wk.weights"))
    wv, sv = _load(os.path.join(d, "wv.weights"))
    wo, so = _load(os.path.join(d, "wo.weights"))
    wl, sl = _load(os.path.join(d, "lm.weights"))
    xn = R.rms_norm(x, nw, 1e-6)
    q = R.rope(R.linear_fp16_act(xn, wq, sq, G).reshape(1, M, HQ, D), 0, 1e6)
    aq, asc = R.quantize_activations(xn)
    k = R.rope(R.matmul_int8(aq, asc, wk, sk, G).reshape(1, M, HKV, D), 0, 1e6)
    v = R.matmul_int8(aq, asc, wv, sv, G).reshape(1, M, HKV, D)
    att = R.attention(q, k, v, 0.125)
    h = R.add(R.linear_fp16_act(att.reshape(M, HQ * D), wo, so, G, int4=True), x)
    z = R.scalar_multiply(R.add_clipped(R.multiply(R.silu(h), R.gelu(h)), h), 0.5)
    logits = R.linear_fp16_act(z, wl, sl, G)

    def got(name, dtype, shape):
        return np.fromfile(os.path.join(d, f"out_{name}.bin"), dtype).reshape(shape)

    for name, ref in (("xn", xn), ("q", q), ("k", k), ("v", v), ("att", att), ("h", h), ("logits", logits),
                      ("last", logits[M - 1]), ("probs", R.softmax(logits))):
        g = got(name, np.float16, ref.shape)
        assert np.array_equal(g.view(np.uint16), ref.view(np.uint16)), name
    assert int(got("tok", np.uint32, (1,))[0]) == int(np.argmax(logits[M - 1].astype(np.float32)))
    for name, ref in (("dw", R.conv1d_causal_depthwise(x_dw, w_dw.reshape(16, 4), 2)), ("k3", R.conv1d_k3(x_k3, w_k3, 2)),
                      ("ln", R.layernorm(x_ln, w_ln, b_ln, 1e-5))):
        g = got(name, np.float16, ref.shape)
        assert np.array_equal(g.view(np.uint16), ref.view(np.uint16)), name
    prof = open(os.path.join(d, "profile.txt")).read()
    assert "MATMUL" in prof and "TOTAL" in prof
