"""The restatement (oracle/refcpu.c, oracle/model.py, oracle/sample.py) against the reference's
OWN C++ compiled on this host (oracle/ref.py: cactus/kernel, graph, engine and models built
against oracle/neon_shim/arm_neon.h). Bit-exact on every kernel of the hot path and on the
greedy tokens and fp16 logits of all three model families.

The reference's NEON matmuls walk a quantisation group in 64-element steps (its tests require
group_size >= 64, tests/test_kernel.cpp:215,306), so matmul and engine comparisons use G = 64
and 128. Skipped where the reference library has not been built (no reference tree here).
"""
import numpy as np
import pytest

from cactus_b200 import convert
from cactus_b200 import weights as W
from oracle import model as OM
from oracle import ref as RF
from oracle import refcpu as R
from oracle import sample as OS

pytestmark = pytest.mark.skipif(not RF.available(), reason="oracle/_ref/libcactus_ref.so not built")


def h(rng, *shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


def same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype
    if a.dtype == np.float16:
        assert np.array_equal(a.view(np.uint16), b.view(np.uint16)), \
            f"{np.count_nonzero(a.view(np.uint16) != b.view(np.uint16))} of {a.size} differ"
    else:
        assert np.array_equal(a, b)


@pytest.mark.parametrize("M,K", [(1, 1024), (3, 1000), (16, 256), (128, 1024), (2, 7), (5, 4096)])
def test_activation_quantization(M, K):
    rng = np.random.default_rng(M * 31 + K)
    x = h(rng, M, K, scale=2.0)
    x[0, :3] = np.float16(0.5)  # ties for the rounding rule
    if M > 2:
        x[2] = 0  # an all-zero row (scale clamps at 1e-10)
    qa, sa = R.quantize_activations(x)
    qb, sb = RF.quantize_activations(x)
    same(qa, qb)
    same(sa, sb)


@pytest.mark.parametrize("M,K,N,G", [(1, 1024, 3072, 128), (4, 1024, 96, 128), (7, 512, 36, 64), (128, 1024, 64, 128),
                                     (1, 2048, 40, 64), (9, 3072, 20, 128), (16, 256, 17, 64)])
def test_matmul_int8_and_int4(M, K, N, G):
    rng = np.random.default_rng(M + K + N + G)
    w = rng.standard_normal((N, K)).astype(np.float32) * np.float32(0.02)
    x = h(rng, M, K)
    q, s = R.quantize_activations(x)
    b8, s8 = W.quantize_int8(w, G)
    same(R.matmul_int8(q, s, b8, s8, G), RF.matmul_int8(q, s, b8, s8, G))
    b4, s4 = W.quantize_int4(w, G)
    same(R.matmul_int4(q, s, b4, s4, G), RF.matmul_int4(q, s, b4, s4, G))


@pytest.mark.parametrize("M,K,N", [(1, 640, 300), (3, 640, 64), (5, 100, 19), (1, 27, 8), (8, 1024, 33)])
def test_matmul_f16(M, K, N):
    rng = np.random.default_rng(K + N)
    a, bt = h(rng, M, K), h(rng, N, K, scale=0.05)
    same(R.matmul_f16(a, bt), RF.matmul_f16(a, bt))


@pytest.mark.parametrize("rows,d", [(1, 1024), (48, 128), (5, 640), (3, 256), (2, 100)])
def test_rms_norm(rows, d):
    rng = np.random.default_rng(rows * d)
    x, w = h(rng, rows, d, scale=3.0), h(rng, d)
    same(R.rms_norm(x, w, 1e-6), RF.rms_norm(x, w, 1e-6))


@pytest.mark.parametrize("S,H,D,start,theta", [(1, 16, 128, 191, 1e6), (7, 8, 128, 0, 1e6), (3, 4, 256, 4095, 1e4),
                                               (5, 32, 64, 1000, 5e5)])
def test_rope(S, H, D, start, theta):
    rng = np.random.default_rng(S * H + start)
    x = h(rng, 1, S, H, D)
    same(R.rope(x, start, theta), RF.rope(x, start, theta))


@pytest.mark.parametrize("shape", [(1, 151936), (4, 1000), (3, 37)])
def test_softmax(shape):
    x = h(np.random.default_rng(shape[1]), *shape, scale=4.0)
    same(R.softmax(x), RF.softmax(x))


@pytest.mark.parametrize("n", [3072, 8195, 13])
def test_activations_and_elementwise(n):
    rng = np.random.default_rng(n)
    a, b = h(rng, n, scale=4.0), h(rng, n, scale=4.0)
    a[:4] = [60000, -60000, 5.0, -5.0]
    b[:4] = [9000, -9000, 0.0, 0.0]
    # The reference runs SiLU / GELU in worker chunks with a scalar libm tail per chunk, so the
    # positions on the libm formula follow the host's pool size: the restatement set to the
    # same pool size gives the same bits everywhere.
    R.set_chunk_pool(RF.pool_workers())
    try:
        same(R.silu(a), RF.silu(a))
        same(R.gelu(a), RF.gelu(a))
    finally:
        R.set_chunk_pool(0)
    same(R.add(a, b), RF.add(a, b))
    same(R.add_clipped(a, b), RF.add_clipped(a, b))
    same(R.multiply(a, b), RF.multiply(a, b))


@pytest.mark.parametrize("S,Skv,Hq,Hkv,D,pos,win,causal", [
    (12, 12, 16, 8, 128, 0, 0, True), (5, 40, 4, 1, 256, 35, 0, True), (70, 70, 4, 1, 256, 0, 16, True),
    (33, 33, 32, 8, 64, 0, 0, True), (9, 9, 2, 2, 64, 0, 0, False), (1, 37, 8, 4, 128, 36, 0, True)])
def test_attention_f16(S, Skv, Hq, Hkv, D, pos, win, causal):
    rng = np.random.default_rng(S * Skv + D)
    q, k, v = h(rng, 1, S, Hq, D), h(rng, 1, Skv, Hkv, D), h(rng, 1, Skv, Hkv, D)
    scale = 1.0 / np.sqrt(D)
    same(R.attention(q, k, v, scale, pos, win, causal), RF.attention(q, k, v, scale, pos, win, causal))


@pytest.mark.parametrize("S,L,Hq,Hkv,D", [(1, 191, 16, 8, 128), (3, 40, 4, 1, 256), (1, 1024, 32, 8, 64),
                                          (6, 100, 8, 8, 128), (1, 513, 16, 8, 128)])
def test_attention_hybrid_int8_cache(S, L, Hq, Hkv, D):
    rng = np.random.default_rng(S + L + D)
    kc, ks = R.quantize_kv(h(rng, L, Hkv, D))
    vc, vs = R.quantize_kv(h(rng, L, Hkv, D))
    q, kn, vn = h(rng, 1, S, Hq, D), h(rng, 1, S, Hkv, D), h(rng, 1, S, Hkv, D)
    scale = 1.0 / np.sqrt(D)
    a = R.attention_hybrid(q, kc, vc, ks, vs, kn, vn, scale, L)
    b = RF.attention_hybrid(q, kc, vc, ks, vs, kn, vn, scale, L)
    same(a, b)


@pytest.mark.parametrize("S,H,D", [(5, 8, 128), (1, 1, 256), (3, 8, 64)])
def test_quantize_kv_and_unpack(S, H, D):
    rng = np.random.default_rng(S * H * D)
    x = h(rng, S, H, D, scale=2.0)
    qa, sa = R.quantize_kv(x)
    qb, sb = RF.quantize_kv(x)
    same(qa, qb)
    same(sa.reshape(sb.shape), sb)
    packed = rng.integers(0, 256, 64).astype(np.uint8)
    same(R.unpack_int4(packed, 128), RF.unpack_int4(packed, 128))


def test_sampler_against_reference_sample_f16():
    """cactus_sample_f16 as compiled, its process-wide repetition history included: the
    restatement given the reference's mt19937 draw and the same history picks the same ids."""
    rng = np.random.default_rng(11)
    history = []
    for i, (temp, top_p, top_k) in enumerate([(0.7, 0.0, 20), (1.0, 0.9, 40), (0.6, 0.95, 0), (0.8, 0.0, 0),
                                              (1.2, 0.5, 64), (0.5, 0.0, 1), (0.9, 0.8, 5)]):
        V = 3000
        logits = h(rng, V, scale=3.0)
        if history:
            logits[history[-1]] = np.float16(9.0)  # make the penalty matter
        seed = 1000 + i
        got = RF.sample_f16(logits, temp, top_p, top_k, seed)
        exp = OS.sample_f16(logits, temp, top_p, top_k, RF.mt19937_uniform(seed), history[-128:])
        assert got == exp, (i, got, exp)
        history.append(got)


@pytest.mark.parametrize("family,G,prec", [
    ("qwen", 128, None), ("qwen", 64, None), ("smol", 128, {"attn": "INT4", "mlp": "INT4", "embed": "INT4"}),
    ("gemma", 128, {"attn": "INT8", "mlp": "INT4", "embed": "FP16"}), ("gemma", 64, None)])
def test_engine_greedy_tokens_and_logits(tmp_path, family, G, prec):
    """Model::prefill (two 256-token chunks) then greedy decode through the reference's own
    engine, against oracle/model.py: identical tokens and bit-identical fp16 logits."""
    kw = {"precision": prec} if prec else {}
    arch = convert.tiny(family, layers=2, group_size=G, **kw)
    folder = convert.make_model(str(tmp_path), arch, seed=3, norm_std=0.1)
    prompt = np.random.default_rng(5).integers(0, arch.vocab_size, 300).tolist()
    ref = RF.RefEngine(folder, arch.vocab_size)
    ours = OM.RefModel(folder)
    R.set_chunk_pool(RF.pool_workers())
    ref.reset()
    ours.kv.reset()
    ref.prefill(prompt[:-1])
    ours.prefill(prompt[:-1])
    ta = tb = prompt[-1]
    for step in range(10):
        ta = ref.decode_argmax([ta])
        tb = ours.decode_argmax([tb])
        same(ours.last_logits, ref.last_logits)
        assert ta == tb, step
    R.set_chunk_pool(0)
    ref.close()


def test_engine_sliding_window_matches(tmp_path):
    """The reference's sink + sliding-window KV cache (window 24, sink 4) through prefill and
    decode past the window."""
    arch = convert.tiny("qwen", layers=2, group_size=128)
    folder = convert.make_model(str(tmp_path), arch, seed=9, norm_std=0.1)
    prompt = np.random.default_rng(2).integers(0, arch.vocab_size, 40).tolist()
    ref = RF.RefEngine(folder, arch.vocab_size)
    ref.set_window(24, 4)
    ours = OM.RefModel(folder, window=24, sink=4)
    R.set_chunk_pool(RF.pool_workers())
    ref.reset()
    ours.kv.reset()
    ref.prefill(prompt[:-1], 16)
    ours.prefill(prompt[:-1], 16)
    ta = tb = prompt[-1]
    for step in range(8):
        ta = ref.decode_argmax([ta])
        tb = ours.decode_argmax([tb])
        same(ours.last_logits, ref.last_logits)
        assert ta == tb
    R.set_chunk_pool(0)
    ref.close()


@pytest.mark.parametrize("N,Lx,C,K,dil", [(1, 37, 64, 3, 1), (2, 20, 48, 4, 2), (1, 50, 32, 11, 1), (1, 64, 40, 17, 3)])
def test_conv1d_causal_depthwise(N, Lx, C, K, dil):
    rng = np.random.default_rng(N + Lx + C + K)
    x, w = h(rng, N, Lx, C), h(rng, C, K, scale=0.5)
    same(R.conv1d_causal_depthwise(x, w, dil), RF.conv1d_causal_depthwise(x, w, dil))


@pytest.mark.parametrize("N,Cin,Lx,Cout,stride", [(1, 80, 30, 24, 1), (2, 17, 9, 8, 2), (1, 5, 1, 3, 1)])
def test_conv1d_k3(N, Cin, Lx, Cout, stride):
    rng = np.random.default_rng(N + Cin + Lx + Cout)
    x, w = h(rng, N, Cin, Lx), h(rng, Cout, Cin, 3, scale=0.3)
    same(R.conv1d_k3(x, w, stride), RF.conv1d_k3(x, w, stride))


@pytest.mark.parametrize("rows,F", [(3, 768), (5, 384), (1, 1000), (2, 7)])
def test_layernorm(rows, F):
    """compute_layernorm_node through a one-node graph of the reference. The restatement fuses
    `variance += diff * diff` as the reference's compilers contract it (clang, -ffp-contract=on).
    The x86 g++ build used here leaves that loop-carried accumulation unfused whatever the
    contraction flags, so a variance can differ in its last bit and, rarely, an output by one
    fp16 unit in the last place: everything else must be identical."""
    rng = np.random.default_rng(rows + F)
    x, w, b = h(rng, rows, F, scale=2.0), h(rng, F), h(rng, F, scale=0.1)
    a, r = R.layernorm(x, w, b, 1e-5), RF.layernorm(x, w, b, 1e-5)
    ai, ri = a.view(np.int16).astype(np.int32), r.view(np.int16).astype(np.int32)
    assert np.abs(ai - ri).max() <= 1
    assert np.count_nonzero(ai != ri) <= max(1, a.size // 1000)
