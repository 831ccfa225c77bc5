"""Kernel-level parity: every C-ABI entry point against the CPU restatement (oracle/).

Integer / byte outputs and the fp16 outputs whose arithmetic is reproduced op-for-op
(quantized matmul, RMSNorm, RoPE, elementwise, softmax lanes, embedding, argmax, the
reference-order attention kernels) are required to be bit-exact; attention is also checked
against the north-star tolerance (normwise max relative error <= 1e-2).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import cactus_b200 as cb
from cactus_b200 import weights as W
from tests.gpu_util import dev, empty, host, ptr, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(scope="module")
def L():
    return cb.lib()


def f16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


def same_bits(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.dtype == np.float16:
        return np.array_equal(a.view(np.uint16), b.view(np.uint16))
    return np.array_equal(a, b)


# ----------------------------------------------------------------------------- quantization
@pytest.mark.parametrize("M,K", [(1, 1024), (4, 3072), (3, 1000), (2, 640)])
def test_quantize_activations_bit_exact(L, ref, M, K):
    rng = np.random.default_rng(M * 7 + K)
    x = f16(rng, (M, K))
    if M > 1:
        x[1] = 0  # all-zero row: scale floor 1e-10
    qd, sd = empty((M, K), np.int8), empty((M,), np.float32)
    cb.check(L.cactus_cuda_quantize_activations(ptr(dev(x)), ptr(qd), ptr(sd), M, K, None))
    q, s = ref.quantize_activations(x)
    assert same_bits(host(qd, np.int8), q)
    assert same_bits(host(sd, np.float32), s)


def _weights(rng, N, K, G, int4=False):
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    return W.quantize_int4(w, G) if int4 else W.quantize_int8(w, G)


@pytest.mark.parametrize("int4", [False, True])
@pytest.mark.parametrize("M,K,N,G", [(1, 1024, 3072, 32), (1, 1024, 3072, 128), (2, 2048, 1000, 64),
                                      (5, 640, 520, 32), (8, 1024, 4096, 128), (13, 3072, 1024, 32),
                                      (1, 8192, 264, 32),
                                      # wide outputs: the lane-per-row GEMV (ragged N)
                                      (1, 1024, 19000, 32), (3, 2048, 20480, 128), (4, 512, 18950, 32),
                                      (2, 1024, 6150, 128), (1, 768, 16390, 32),
                                      # 16 <= M: the mma.sync GEMM, or the tcgen05 GEMM for shapes of
                                      # one wave of its tiles or more (both forced below)
                                      (16, 1024, 3072, 32), (127, 2048, 1024, 32), (64, 3072, 1024, 128),
                                      (33, 640, 512, 32), (200, 1024, 4096, 64), (17, 576, 960, 32),
                                      (130, 1024, 96, 128), (64, 128, 32, 32), (128, 256, 64, 64),
                                      (300, 896, 4864, 32), (513, 1024, 160, 32), (96, 640, 512, 32),
                                      # at least one wave (148) of 128 x 128 tiles: the tcgen05 GEMM
                                      (128, 256, 18944, 32), (300, 640, 6400, 64), (1100, 1024, 2176, 128),
                                      (2048, 1024, 1536, 32)])
def test_matmul_prequantized_bit_exact(L, ref, int4, M, K, N, G):
    if int4 and G % 32:
        pytest.skip("INT4 groups are multiples of 32")
    rng = np.random.default_rng(K + N + M)
    B, Bs = _weights(rng, N, K, G, int4)
    x = f16(rng, (M, K))
    Aq, As = ref.quantize_activations(x)
    C = empty((M, N), np.float16)
    fn = L.cactus_cuda_matmul_int4 if int4 else L.cactus_cuda_matmul_int8
    cb.check(fn(ptr(dev(Aq)), ptr(dev(As)), ptr(dev(B)), ptr(dev(Bs)), ptr(C), M, K, N, G, None))
    exp = ref.matmul_int4(Aq, As, B, Bs, G) if int4 else ref.matmul_int8(Aq, As, B, Bs, G)
    assert same_bits(host(C, np.float16), exp)


@pytest.mark.parametrize("int4", [False, True])
@pytest.mark.parametrize("M", [1, 128])
def test_config1_graph_matmul_bit_exact(L, ref, int4, M):
    """Config 1: FP16 activations [M,1024] ~N(0,1) x weights [1024 -> 3072] ~N(0,0.02), G=32, seed 0."""
    rng = np.random.default_rng(0)
    w = rng.standard_normal((3072, 1024), dtype=np.float32) * np.float32(0.02)
    B, Bs = W.quantize_int4(w, 32) if int4 else W.quantize_int8(w, 32)
    x = rng.standard_normal((M, 1024)).astype(np.float16)
    C = empty((M, 3072), np.float16)
    fn = L.cactus_cuda_linear_int4 if int4 else L.cactus_cuda_linear_int8
    cb.check(fn(ptr(dev(x)), ptr(dev(B)), ptr(dev(Bs)), ptr(C), M, 1024, 3072, 32, None))
    exp = ref.linear_fp16_act(x, B, Bs, 32, int4=int4)
    got = host(C, np.float16)
    assert same_bits(got, exp)
    assert rel_err(got, exp) <= TOL


@pytest.mark.parametrize("int4", [False, True])
@pytest.mark.parametrize("M", [1, 5, 8, 12])
def test_linear_llama_down_projection_bit_exact(L, ref, int4, M):
    """Llama-3.2-1B down projection (K = 8192, N = 2048, G = 32) with fused activation
    quantisation: the rows one GEMV launch holds shrink with K, so M > 4 runs in chunks."""
    rng = np.random.default_rng(8192 + M)
    B, Bs = _weights(rng, 2048, 8192, 32, int4)
    x = f16(rng, (M, 8192))
    C = empty((M, 2048), np.float16)
    fn = L.cactus_cuda_linear_int4 if int4 else L.cactus_cuda_linear_int8
    cb.check(fn(ptr(dev(x)), ptr(dev(B)), ptr(dev(Bs)), ptr(C), M, 8192, 2048, 32, None))
    assert same_bits(host(C, np.float16), ref.linear_fp16_act(x, B, Bs, 32, int4=int4))


def test_matmul_rejects_bad_shapes(L):
    rng = np.random.default_rng(1)
    B, Bs = _weights(rng, 16, 96, 32)
    x = f16(rng, (1, 96))
    C = empty((1, 16), np.float16)
    rc = L.cactus_cuda_linear_int8(ptr(dev(x)), ptr(dev(B)), ptr(dev(Bs)), ptr(C), 1, 96, 16, 24, None)
    assert rc != 0 and b"multiple" in L.cactus_cuda_last_error()


@pytest.mark.parametrize("M,K,N", [(1, 640, 1000), (3, 64, 37), (2, 100, 9), (1, 640, 262144), (5, 648, 77),
                                   (8, 136, 33), (4, 640, 1001), (9, 64, 40), (2, 24, 300)])
def test_matmul_f16_bit_exact(L, ref, M, K, N):
    rng = np.random.default_rng(K)
    A = f16(rng, (M, K))
    Bt = f16(rng, (N, K), 0.05)
    C = empty((M, N), np.float16)
    cb.check(L.cactus_cuda_matmul_f16(ptr(dev(A)), ptr(dev(Bt)), ptr(C), M, K, N, None))
    assert same_bits(host(C, np.float16), ref.matmul_f16(A, Bt))


# ----------------------------------------------------------------------------- norms / rope
@pytest.mark.parametrize("rows,dims", [(5, 1024), (16, 128), (3, 640), (2, 100), (1, 7)])
def test_rms_norm_bit_exact(L, ref, rows, dims):
    rng = np.random.default_rng(dims)
    x = f16(rng, (rows, dims), 3.0)
    w = (1 + 0.1 * rng.standard_normal(dims)).astype(np.float16)
    y = empty((rows, dims), np.float16)
    cb.check(L.cactus_cuda_rms_norm_f16(ptr(dev(x)), ptr(dev(w)), ptr(y), rows, dims, 1e-6, None))
    assert same_bits(host(y, np.float16), ref.rms_norm(x, w, 1e-6))


# ----------------------------------------------------------------------------- other families' kernels
@pytest.mark.parametrize("N,Lx,C,K,dil", [(1, 37, 64, 3, 1), (2, 20, 48, 4, 2), (1, 50, 32, 11, 1), (1, 9, 16, 8, 1),
                                          (1, 64, 40, 17, 3), (3, 1, 5, 3, 1), (1, 300, 1024, 3, 1)])
def test_conv1d_causal_depthwise_bit_exact(L, ref, N, Lx, C, K, dil):
    """LFM2's causal depthwise conv (kernel_conv.cpp:15-110): 8-tap lane blocks, tails, dilation."""
    rng = np.random.default_rng(N * 1000 + Lx + C + K)
    x, w = f16(rng, (N, Lx, C)), f16(rng, (C, K), 0.5)
    y = empty((N, Lx, C), np.float16)
    cb.check(L.cactus_cuda_conv1d_causal_depthwise_f16(ptr(dev(x)), ptr(dev(w)), ptr(y), N, Lx, C, K, dil, None))
    assert same_bits(host(y, np.float16), ref.conv1d_causal_depthwise(x, w, dil))


@pytest.mark.parametrize("N,Cin,Lx,Cout,stride", [(1, 80, 30, 24, 1), (2, 17, 9, 8, 2), (1, 5, 1, 3, 1),
                                                  (1, 40, 33, 16, 2), (1, 80, 3000, 64, 1), (1, 384, 200, 96, 2)])
def test_conv1d_k3_bit_exact(L, ref, N, Cin, Lx, Cout, stride):
    """Whisper's front-end conv1d, kernel 3, padding 1 (kernel_conv.cpp:112-227), strides 1 and 2."""
    rng = np.random.default_rng(N + Cin + Lx + Cout)
    x, w = f16(rng, (N, Cin, Lx)), f16(rng, (Cout, Cin, 3), 0.3)
    out_len = (Lx - 1) // stride + 1
    y = empty((N, Cout, out_len), np.float16)
    cb.check(L.cactus_cuda_conv1d_f16_k3(ptr(dev(x)), ptr(dev(w)), ptr(y), N, Lx, Cin, Cout, stride, None))
    assert same_bits(host(y, np.float16), ref.conv1d_k3(x, w, stride))


@pytest.mark.parametrize("rows,F", [(3, 768), (5, 384), (1, 1000), (2, 7), (70, 1280), (1, 14528)])
def test_layernorm_bit_exact(L, ref, rows, F):
    """compute_layernorm_node (graph_ops_nn.cpp:373-457): in-order mean and variance sums."""
    rng = np.random.default_rng(rows + F)
    x, w, b = f16(rng, (rows, F), 2.0), f16(rng, (F,)), f16(rng, (F,), 0.1)
    y = empty((rows, F), np.float16)
    cb.check(L.cactus_cuda_layernorm_f16(ptr(dev(x)), ptr(dev(w)), ptr(dev(b)), ptr(y), rows, F, 1e-5, None))
    assert same_bits(host(y, np.float16), ref.layernorm(x, w, b, 1e-5))


def test_layernorm_rejects_oversized_rows(L):
    y = empty((1, 16), np.float16)
    assert L.cactus_cuda_layernorm_f16(ptr(y), ptr(y), ptr(y), ptr(y), 1, 14529, 1e-5, None) != 0
    assert b"feature count" in L.cactus_cuda_last_error()


@pytest.mark.parametrize("B,S,H,D,start,theta", [(1, 7, 3, 128, 100, 1e6), (2, 5, 2, 64, 0, 5e5),
                                                  (1, 3, 1, 12, 9, 1e4), (1, 1, 8, 256, 4095, 1e4)])
def test_rope_bit_exact(L, ref, B, S, H, D, start, theta):
    rng = np.random.default_rng(D + start)
    x = f16(rng, (B, S, H, D))
    y = empty((B, S, H, D), np.float16)
    cb.check(L.cactus_cuda_rope_f16(ptr(dev(x)), ptr(y), B, S, H, D, start, theta, None))
    assert same_bits(host(y, np.float16), ref.rope(x, start, theta))


# ----------------------------------------------------------------------------- attention
@pytest.mark.parametrize("B,S,Skv,Hq,Hkv,D,off,win", [
    (1, 40, 40, 4, 2, 64, 0, 0),       # causal prefill, GQA
    (1, 128, 128, 16, 8, 128, 0, 0),   # Qwen-shaped first chunk
    (2, 33, 33, 4, 1, 256, 0, 0),      # Gemma-shaped heads, batch 2
    (1, 70, 70, 4, 1, 256, 0, 16),     # sliding window (Gemma local)
    (1, 5, 21, 2, 2, 32, 16, 0),       # queries appended after a prefix
])
def test_attention_f16_parity(L, ref, B, S, Skv, Hq, Hkv, D, off, win):
    rng = np.random.default_rng(S * Hq + D)
    q, k, v = f16(rng, (B, S, Hq, D)), f16(rng, (B, Skv, Hkv, D)), f16(rng, (B, Skv, Hkv, D))
    scale = 1.0 / np.sqrt(D)
    o = empty((B, S, Hq, D), np.float16)
    cb.check(L.cactus_cuda_attention_f16(ptr(dev(q)), ptr(dev(k)), ptr(dev(v)), ptr(o), B, S, Skv, Hq, Hkv, D,
                                         scale, off, win, 1, None))
    exp = ref.attention(q, k, v, scale, off, win, True)
    got = host(o, np.float16)
    assert rel_err(got, exp) <= TOL
    # block partition, quadratic exp, lane orders and online-softmax sequence are reproduced
    assert same_bits(got, exp)


def test_matmul_tcgen05_every_supported_shape_bit_exact():
    """The tcgen05 GEMM forced onto every shape it supports (CACTUS_B200_GEMM=tc: K % 128 == 0,
    N % 128 == 0, G in 32 / 64 / 128, INT8 and INT4, any M), on the GEMM parity cases above,
    run in a child pytest process."""
    env = dict(os.environ, CACTUS_B200_GEMM="tc")
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.abspath(__file__), "-q", "-m", "gpu", "-p",
                        "no:cacheprovider", "-k", "matmul_prequantized or config1"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_matmul_mma_sync_path_bit_exact():
    """The mma.sync GEMM (the default for the shapes the tcgen05 GEMM does not take; forced for
    all with CACTUS_B200_GEMM=mma, read once per process) on the GEMM parity cases above, run
    in a child pytest process."""
    env = dict(os.environ, CACTUS_B200_GEMM="mma")
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.abspath(__file__), "-q", "-m", "gpu", "-p",
                        "no:cacheprovider", "-k", "matmul_prequantized or config1"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_gemv_row_streaming_path_bit_exact():
    """The row-streaming GEMV (opt-in: CACTUS_B200_GEMV=rows, read once per process) on every
    GEMV parity case above (M <= 15: pre-quantised, fused quantisation, config 1, Llama K=8192),
    run in a child pytest process."""
    env = dict(os.environ, CACTUS_B200_GEMV="rows")
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.abspath(__file__), "-q", "-m", "gpu", "-p",
                        "no:cacheprovider", "-k", "matmul_prequantized or config1 or llama_down"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_gemv_lane_path_bit_exact():
    """The lane-per-row GEMV (the default for wide outputs; forced for every shape it
    supports with CACTUS_B200_GEMV=lanes, read once per process) on every GEMV parity case above
    and on the engine's decode paths (fused RMSNorm prologues, GLU epilogues), in child pytest
    processes."""
    env = dict(os.environ, CACTUS_B200_GEMV="lanes")
    here = os.path.dirname(os.path.abspath(__file__))
    for path, sel in ((os.path.abspath(__file__), "matmul_prequantized or config1 or llama_down or linear"),
                      (os.path.join(here, "test_engine_gpu.py"), "not qwen3_0_6b")):
        r = subprocess.run([sys.executable, "-m", "pytest", path, "-q", "-m", "gpu", "-p", "no:cacheprovider",
                            "-k", sel], env=env, capture_output=True, text=True, timeout=900)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


# L_ >= 512: the key-split kernels (attention_split.cu); below: one CTA per query
@pytest.mark.parametrize("B,S,L_,Hq,Hkv,D", [(1, 1, 127, 16, 8, 128), (1, 1, 1024, 32, 8, 64),
                                             (1, 1, 4096, 4, 1, 256), (1, 4, 60, 16, 8, 128),
                                             (1, 1, 0, 16, 8, 128), (1, 1, 8191, 16, 8, 128),
                                             (2, 1, 700, 16, 8, 128), (1, 3, 600, 4, 1, 256),
                                             (3, 2, 511, 16, 8, 128), (1, 1, 2080, 8, 8, 128)])
def test_attention_hybrid_parity(L, ref, B, S, L_, Hq, Hkv, D):
    rng = np.random.default_rng(L_ + Hq + B)
    kc = np.zeros((B, max(L_, 1), Hkv, D), np.int8)
    vc = np.zeros_like(kc)
    for b in range(B):
        kq, ksb = ref.quantize_kv(f16(rng, (max(L_, 1), Hkv, D)))
        vq, vsb = ref.quantize_kv(f16(rng, (max(L_, 1), Hkv, D)))
        kc[b], vc[b] = kq, vq
        if b == 0:  # the reference indexes the scales without a batch offset
            ks, vs = ksb, vsb
    kn, vn = f16(rng, (B, S, Hkv, D)), f16(rng, (B, S, Hkv, D))
    q = f16(rng, (B, S, Hq, D))
    scale = 1.0 / np.sqrt(D)
    o = empty((B, S, Hq, D), np.float16)
    cb.check(L.cactus_cuda_attention_hybrid_int8_fp16(
        ptr(dev(q)), ptr(dev(kc)), ptr(dev(vc)), ptr(dev(ks)), ptr(dev(vs)), ptr(dev(kn)), ptr(dev(vn)), ptr(o),
        B, S, L_, S, Hq, Hkv, D, scale, L_, 1, 128, None))
    exp = ref.attention_hybrid(q, kc[:, :L_], vc[:, :L_], ks, vs, kn, vn, scale, L_)
    got = host(o, np.float16)
    assert rel_err(got, exp) <= TOL
    assert same_bits(got, exp)  # reference order at every length


@pytest.mark.parametrize("S,H,D,G", [(5, 8, 128, 128), (3, 1, 256, 128), (2, 2, 100, 128)])
def test_quantize_kv_bit_exact(L, ref, S, H, D, G):
    rng = np.random.default_rng(D)
    x = f16(rng, (S, H, D))
    ng = (D + G - 1) // G
    q, s = empty((S, H, D), np.int8), empty((S, H, ng), np.float32)
    cb.check(L.cactus_cuda_quantize_kv_fp16_to_int8(ptr(dev(x)), ptr(q), ptr(s), S, H, D, G, None))
    rq, rs = ref.quantize_kv(x, G)
    assert same_bits(host(q, np.int8), rq) and same_bits(host(s, np.float32), rs)


# ----------------------------------------------------------------------------- elementwise
@pytest.mark.parametrize("n", [3072, 8 * 1000 + 5])
def test_elementwise_bit_exact(L, ref, n):
    rng = np.random.default_rng(n)
    a, b = f16(rng, (n,), 3.0), f16(rng, (n,), 3.0)
    a[:4] = np.array([60000, -60000, 0, 1], np.float16)
    b[:4] = np.array([60000, -60000, 0, -1], np.float16)
    vec = (n // 8) * 8
    for name, fn, exp in [
        ("silu", lambda o: L.cactus_cuda_silu_f16(ptr(dev(a)), ptr(o), n, None), ref.silu(a)),
        ("gelu", lambda o: L.cactus_cuda_gelu_f16(ptr(dev(a)), ptr(o), n, None), ref.gelu(a)),
        ("add", lambda o: L.cactus_cuda_add_f16(ptr(dev(a)), ptr(dev(b)), ptr(o), n, None), ref.add(a, b)),
        ("addc", lambda o: L.cactus_cuda_add_f16_clipped(ptr(dev(a)), ptr(dev(b)), ptr(o), n, None),
         ref.add_clipped(a, b)),
        ("mul", lambda o: L.cactus_cuda_multiply_f16(ptr(dev(a)), ptr(dev(b)), ptr(o), n, None), ref.multiply(a, b)),
        ("smul", lambda o: L.cactus_cuda_scalar_multiply_f16(ptr(dev(a)), ptr(o), n, 25.298221, None),
         ref.scalar_multiply(a, 25.298221)),
    ]:
        o = empty((n,), np.float16)
        cb.check(fn(o), name)
        got = host(o, np.float16)
        # the scalar tails of silu/gelu call expf/tanhf, whose last bits may differ from libm
        assert same_bits(got[:vec], exp[:vec]), name
        assert np.allclose(got.astype(np.float32), exp.astype(np.float32), rtol=2e-3, atol=1e-3), name


@pytest.mark.parametrize("rows,V", [(4, 3), (2, 1000), (1, 151936), (3, 64)])
def test_softmax(L, ref, rows, V):
    rng = np.random.default_rng(V)
    x = f16(rng, (rows, V), 2.0)
    y = empty((rows, V), np.float16)
    cb.check(L.cactus_cuda_softmax_f16(ptr(dev(x)), ptr(y), rows, V, None))
    got, exp = host(y, np.float16), ref.softmax(x)
    vv = (V // 32) * 32
    assert same_bits(got[:, :vv], exp[:, :vv])
    assert np.allclose(got.astype(np.float32), exp.astype(np.float32), rtol=1e-2, atol=1e-4)


def test_embedding_and_argmax_exact(L, ref):
    rng = np.random.default_rng(11)
    w = rng.standard_normal((500, 256), dtype=np.float32) * np.float32(0.02)
    q, s = W.quantize_int8(w, 32)
    ids = np.array([7, 0, 499, 7, 250], np.uint32)
    o = empty((5, 256), np.float16)
    cb.check(L.cactus_cuda_embedding_int8(ptr(dev(q)), ptr(dev(s)), 32, 500, 256, ptr(dev(ids)), 5, ptr(o), None))
    assert same_bits(host(o, np.float16), ref.embedding_int8(q, s, 32, ids))
    t16 = w.astype(np.float16)
    cb.check(L.cactus_cuda_embedding_f16(ptr(dev(t16)), 500, 256, ptr(dev(ids)), 5, ptr(o), None))
    assert same_bits(host(o, np.float16), ref.embedding_f16(t16, ids))
    for V in (1, 5, 151936, 262144):
        x = f16(rng, (2, V))
        x[1, V // 3] = 50
        x[1, (2 * V) // 3] = 50  # tie: the first index wins
        out = empty((1,), np.uint32)
        cb.check(L.cactus_cuda_argmax_f16(ptr(dev(x)), 2, V, ptr(out), None))
        assert int(host(out, np.uint32)[0]) == ref.argmax(x[1])


def test_unpack_int4_exact(L, ref):
    rng = np.random.default_rng(2)
    p = rng.integers(0, 256, 333, dtype=np.uint8)
    o = empty((666,), np.int8)
    cb.check(L.cactus_cuda_unpack_int4_to_int8(ptr(dev(p)), ptr(o), 666, None))
    assert same_bits(host(o, np.int8), ref.unpack_int4(p, 666))


def test_no_device_error_after_suite(L):
    assert L.cactus_cuda_device_error(None) == 0
