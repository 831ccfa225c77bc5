"""Pins the CPU restatement (oracle/) against the reference's own tests and fixtures.

Each test restates one reference test's semantics (cited per test), so the oracle
is anchored to the reference before it is used to check the CUDA path.
"""
import ctypes
import json
import os

import numpy as np
import pytest

from cactus_b200 import weights as W

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _libc_rand_stream():
    libc = ctypes.CDLL("libc.so.6")
    libc.srand(1)  # glibc's default seed: the reference tests never call srand
    return libc


def test_matmul_int8_grouped_formula_pin(ref):
    """tests/test_kernel.cpp:214-303: M=2,K=128,N=4,G=64 vs the scalar formula, max abs err < 0.1."""
    libc = _libc_rand_stream()
    RAND_MAX = 2147483647
    M, K, N, G = 2, 128, 4, 64
    A = np.array([np.float16((np.float32(libc.rand()) / np.float32(RAND_MAX) - np.float32(0.5)) * np.float32(0.5))
                  for _ in range(M * K)], np.float16).reshape(M, K)
    B = np.array([(libc.rand() % 128) - 64 for _ in range(N * K)], np.int8).reshape(N, K)
    ng = K // G
    Bs = np.maximum(np.abs(B.reshape(N, ng, G).astype(np.float32)).max(axis=2) / np.float32(127), np.float32(1e-6))
    Bs = Bs.astype(np.float16)
    Aq, As = ref.quantize_activations(A)
    C = ref.matmul_int8(Aq, As, B, Bs, G).astype(np.float32)
    Cref = np.zeros((M, N), np.float32)
    for m in range(M):
        a_scale = max(np.float32(np.abs(A[m].astype(np.float32)).max()) / np.float32(127.0), np.float32(1e-10))
        aq = np.clip(np.round(A[m].astype(np.float32) / a_scale), -128, 127).astype(np.int32)
        for n in range(N):
            acc = np.float32(0)
            for g in range(ng):
                gs = int(np.dot(aq[g * G:(g + 1) * G], B[n, g * G:(g + 1) * G].astype(np.int32)))
                acc += np.float32(gs) * (a_scale * np.float32(Bs[n, g]))
            Cref[m, n] = acc
    assert np.abs(C - Cref).max() < 0.1


def test_matmul_int4_grouped_formula_pin(ref):
    """tests/test_kernel.cpp:305-405: packed INT4 (low nibble = even k) vs the scalar formula."""
    libc = _libc_rand_stream()
    RAND_MAX = 2147483647
    M, K, N, G = 2, 128, 4, 64
    A = np.array([np.float16((np.float32(libc.rand()) / np.float32(RAND_MAX) - np.float32(0.5)) * np.float32(0.5))
                  for _ in range(M * K)], np.float16).reshape(M, K)
    Bu = np.array([(libc.rand() % 16) - 8 for _ in range(N * K)], np.int8).reshape(N, K)
    Bp = ((Bu[:, 0::2] & 0x0F) | ((Bu[:, 1::2] & 0x0F) << 4)).astype(np.uint8)
    ng = K // G
    Bs = np.maximum(np.abs(Bu.reshape(N, ng, G).astype(np.float32)).max(axis=2) / np.float32(7), np.float32(1e-6))
    Bs = Bs.astype(np.float16)
    Aq, As = ref.quantize_activations(A)
    C = ref.matmul_int4(Aq, As, Bp, Bs, G).astype(np.float32)
    unpacked = ref.unpack_int4(Bp.reshape(-1), N * K).reshape(N, K)
    assert np.array_equal(unpacked, Bu)
    Cref = np.zeros((M, N), np.float32)
    for m in range(M):
        a_scale = max(np.float32(np.abs(A[m].astype(np.float32)).max()) / np.float32(127.0), np.float32(1e-10))
        aq = np.clip(np.round(A[m].astype(np.float32) / a_scale), -128, 127).astype(np.int32)
        for n in range(N):
            acc = np.float32(0)
            for g in range(ng):
                gs = int(np.dot(aq[g * G:(g + 1) * G], Bu[n, g * G:(g + 1) * G].astype(np.int32)))
                acc += np.float32(gs) * (a_scale * np.float32(Bs[n, g]))
            Cref[m, n] = acc
    assert np.abs(C - Cref).max() < 0.1


def test_softmax_known_answer(ref):
    """tests/test_graph.cpp:206-218 and tests/test_kernel.cpp:137-158."""
    x = np.array([[1, 2, 3], [4, 5, 6]], np.float16)
    y = ref.softmax(x).astype(np.float32)
    exp = np.array([0.09003, 0.24473, 0.66524], np.float32)
    assert np.abs(y - exp[None, :]).max() < 0.01
    x2 = np.array([[1, 2, 3], [2, 3, 4], [3, 4, 5], [4, 5, 6]], np.float16)
    assert np.abs(ref.softmax(x2).astype(np.float32).sum(1) - 1).max() < 1e-2
    # wide rows go through the 32-lane polynomial-exp path
    rng = np.random.default_rng(1)
    xw = rng.standard_normal((3, 1000)).astype(np.float16)
    assert np.abs(ref.softmax(xw).astype(np.float32).sum(1) - 1).max() < 2e-2


def test_rms_norm_formula(ref):
    """tests/test_graph.cpp:176-204 (eps 1e-5, tolerance 0.01)."""
    x = np.arange(1, 9, dtype=np.float16).reshape(1, 8)
    w = np.ones(8, np.float16)
    y = ref.rms_norm(x, w, 1e-5).astype(np.float32)
    ss = np.float32(np.sum(x.astype(np.float32) ** 2))
    inv = np.float32(1) / np.sqrt(ss / np.float32(8) + np.float32(1e-5))
    exp = (x.astype(np.float32) * inv).astype(np.float16).astype(np.float32)
    assert np.abs(y - exp).max() < 0.01


def test_matmul_f16_known_answer(ref):
    """tests/test_graph.cpp:75-90: [2,3] x [3,2] (not pretransposed) = {22,28,49,64}."""
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float16)
    b = np.array([[1, 2], [3, 4], [5, 6]], np.float16)
    c = ref.matmul_f16(a, np.ascontiguousarray(b.T))
    assert c.astype(np.float32).tolist() == [[22, 28], [49, 64]]


def test_rope_changes_input_and_is_rotation(ref):
    """tests/test_kernel.cpp:161-184 plus the rotation identity |y| ~ |x| per pair."""
    rng = np.random.default_rng(42)
    x = rng.uniform(-2, 2, (1, 2, 1, 4)).astype(np.float16)
    y = ref.rope(x, 0, 10000.0)
    assert np.array_equal(y[:, 0], x[:, 0])  # position 0 is the identity
    assert np.abs(y.astype(np.float32) - x.astype(np.float32)).max() > 1e-3
    xb = rng.standard_normal((1, 8, 2, 128)).astype(np.float16)
    yb = ref.rope(xb, 100, 1e6).astype(np.float32)
    xf = xb.astype(np.float32)
    nx = xf[..., :64] ** 2 + xf[..., 64:] ** 2
    ny = yb[..., :64] ** 2 + yb[..., 64:] ** 2
    assert np.abs(nx - ny).max() < 0.05 * max(1.0, nx.max())


def test_attention_nonzero_and_matches_fp64_softmax(ref):
    """tests/test_kernel.cpp:186-212 (non-zero output) and a float64 softmax formula check."""
    rng = np.random.default_rng(3)
    B, S, Hq, Hkv, D = 1, 40, 4, 2, 64
    q = rng.standard_normal((B, S, Hq, D)).astype(np.float16)
    k = rng.standard_normal((B, S, Hkv, D)).astype(np.float16)
    v = rng.standard_normal((B, S, Hkv, D)).astype(np.float16)
    scale = 1.0 / np.sqrt(D)
    o = ref.attention(q, k, v, scale).astype(np.float64)
    assert np.any(o != 0)
    qf, kf, vf = (t.astype(np.float64) for t in (q, k, v))
    for h in range(Hq):
        s = qf[0, :, h] @ kf[0, :, h // 2].T * scale
        s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        exp = p @ vf[0, :, h // 2]
        # the reference's quadratic 2^x approximation leaves a few-percent error per weight
        assert np.abs(o[0, :, h] - exp).max() < 0.1


def test_hybrid_attention_equals_fp16_attention_when_cache_is_exact(ref):
    """kernel_attention.cpp:257-482: with an exactly representable INT8 cache the hybrid path
    computes the same softmax (with expf) as the fp16 path over the concatenated keys."""
    rng = np.random.default_rng(5)
    L, Hkv, Hq, D = 37, 2, 4, 128
    kc = rng.integers(-127, 128, (L, Hkv, D)).astype(np.int8)
    vc = rng.integers(-127, 128, (L, Hkv, D)).astype(np.int8)
    ks = np.full((L, Hkv, 1), 1.0 / 64, np.float32)
    vs = np.full((L, Hkv, 1), 1.0 / 64, np.float32)
    kn = rng.standard_normal((1, 1, Hkv, D)).astype(np.float16)
    vn = rng.standard_normal((1, 1, Hkv, D)).astype(np.float16)
    q = rng.standard_normal((1, 1, Hq, D)).astype(np.float16)
    o = ref.attention_hybrid(q, kc, vc, ks, vs, kn, vn, 1 / np.sqrt(D), L).astype(np.float64)
    kall = np.concatenate([kc.astype(np.float64) / 64, kn[0].astype(np.float64)], 0)
    vall = np.concatenate([vc.astype(np.float64) / 64, vn[0].astype(np.float64)], 0)
    for h in range(Hq):
        s = kall[:, h // 2] @ q[0, 0, h].astype(np.float64) / np.sqrt(D)
        p = np.exp(s - s.max())
        p /= p.sum()
        assert np.abs(o[0, 0, h] - p @ vall[:, h // 2]).max() < 2e-3


def test_kv_quantize_roundtrip(ref):
    """kernel_quants.cpp:223-293: per (token, head, 128-group) absmax/127 with RNE."""
    rng = np.random.default_rng(7)
    x = rng.standard_normal((5, 8, 128)).astype(np.float16)
    q, s = ref.quantize_kv(x)
    deq = q.astype(np.float32) * s
    err = np.abs(deq - x.astype(np.float32)).max(axis=2)
    assert np.all(err <= s[..., 0] * 0.5 + 1e-6)
    assert np.all(np.abs(q).max(axis=2) == 127)


def test_fast_exp_and_tanh_shapes(ref):
    """kernel_utils.h:108-163: the reference's polynomial exp and Pade tanh (not libm)."""
    assert ref.lib().ref_fast_exp(0.0) == 1.0
    assert 0.9 < ref.lib().ref_fast_exp(1.0) / np.e < 1.0  # its polynomial undershoots e
    assert ref.lib().ref_fast_tanh(5.0) == 1.0 and ref.lib().ref_fast_tanh(-5.0) == -1.0
    t = ref.lib().ref_fast_tanh(0.5)
    assert abs(t - 0.5 * (27 + 0.25) / (27 + 9 * 0.25)) < 1e-6


def test_argmax_first_max_wins(ref):
    """kernel_nn.cpp:451-467: strict '>' keeps the first of equal maxima."""
    x = np.array([0, 3, 1, 3, 2], np.float16)
    assert ref.argmax(x) == 1


def test_embedding_int8_dequant(ref):
    """graph_ops_tensor.cpp:226-260: fp16(int8 * fp32(scale)) per group."""
    rng = np.random.default_rng(9)
    w = rng.standard_normal((50, 64), dtype=np.float32) * np.float32(0.02)
    q, s = W.quantize_int8(w, 32)
    ids = np.array([3, 0, 49, 3], np.uint32)
    out = ref.embedding_int8(q, s, 32, ids)
    exp = (q[ids].astype(np.float32).reshape(4, 2, 32) * s[ids].astype(np.float32)[:, :, None]).reshape(4, 64)
    assert np.array_equal(out, exp.astype(np.float16))


@pytest.mark.parametrize("fname", sorted(json.load(open(os.path.join(GOLDEN, "manifest.json")))))
def test_weight_packing_bit_exact(fname, ref, tmp_path):
    """Our converter and the oracle quantizer reproduce the reference quantizer's bytes."""
    meta = json.load(open(os.path.join(GOLDEN, "manifest.json")))[fname]
    w = np.load(os.path.join(GOLDEN, meta["input"]))
    gold = open(os.path.join(GOLDEN, fname), "rb").read()
    out = tmp_path / fname
    W.save_tensor(out, w, meta["precision"], meta["group_size"] or 128)
    assert out.read_bytes() == gold
    f = W.read_weights(os.path.join(GOLDEN, fname))
    if meta["precision"] == "INT8":
        q, s = ref.quantize_weights_int8(w, meta["group_size"])
        assert np.array_equal(q, f.data) and np.array_equal(s.view(np.uint16), f.scales.view(np.uint16))
    elif meta["precision"] == "INT4":
        p, s = ref.quantize_weights_int4(w, meta["group_size"])
        assert np.array_equal(p, f.data) and np.array_equal(s.view(np.uint16), f.scales.view(np.uint16))
    else:
        assert np.array_equal(f.data.view(np.uint16), w.astype(np.float16).view(np.uint16))


def test_weights_reader_rejects_corrupt_files(tmp_path):
    """graph_io.cpp:497-566 error behaviour: bad magic and truncated data raise."""
    good = open(os.path.join(GOLDEN, "randn_16x256.int8.g32.weights"), "rb").read()
    bad = tmp_path / "bad.weights"
    bad.write_bytes(b"XXXX" + good[4:])
    with pytest.raises(ValueError, match="magic"):
        W.read_weights(bad)
    bad.write_bytes(good[:-10])
    with pytest.raises(ValueError, match="corrupted"):
        W.read_weights(bad)
    bad.write_bytes(good[:40])
    with pytest.raises(ValueError, match="too small"):
        W.read_weights(bad)
