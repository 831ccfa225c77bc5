"""Full-shape parity for BASELINE configs 3, 4 and 5 on the B200, against the restatement
(oracle/, itself pinned bit-exact to the reference's own C++ in tests/test_oracle_vs_reference.py).

  config 3: Gemma-3-270m shape (18 layers, hidden 640, 4/1 heads of 256, GeGLU 2048, vocab
            262144, FP16 tied lm head, INT8 attention / INT4 MLP, 5:1 local / global), a
            4096-token random prompt, 32 greedy steps;
  config 4: Llama-3.2-1B shape (16 layers, hidden 2048, 32/8 heads of 64, SwiGLU 8192,
            vocab 128256, INT4 G32), one sequence at context 1024 and a batch of 8;
  config 5: decode attention at the sweep's corners (32768 keys; 64 sequences x 4096 keys;
            the FP16 cache through cactus_cuda_attention_f16) and 512 causal queries after
            4096 cached keys.
Greedy tokens must be identical; logits and attention outputs bit-identical.
"""
import os

import numpy as np
import pytest

import cactus_b200 as cb
from cactus_b200 import convert
from cactus_b200.engine import Engine
from oracle import model as OM
from oracle import refcpu as R
from tests.gpu_util import dev, empty, host, ptr

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("CACTUS_SKIP_FULL") == "1", reason="full-size models disabled")]


def _bits(a):
    return np.ascontiguousarray(a, np.float16).view(np.uint16)


@pytest.fixture(autouse=True)
def _threads():
    R.set_threads(os.cpu_count() or 1)


def test_config3_gemma_4096_prompt_32_greedy_steps():
    arch = convert.gemma3_270m(32)
    folder = convert.make_model(convert.default_model_dir(arch), arch, seed=0)
    prompt = np.random.default_rng(3).integers(0, arch.vocab_size, 4096).tolist()
    eng = Engine(folder, context_size=4096 + 40)
    got = eng.generate_greedy(prompt, 32).tolist()
    logits = eng.last_logits()
    eng.close()
    ref = OM.RefModel(folder, context_size=4096 + 40)
    exp = ref.generate_greedy(prompt, 32)
    assert got == exp
    assert np.array_equal(_bits(logits), _bits(ref.last_logits))


def test_config4_llama_context_1024_and_batch_8():
    arch = convert.llama3_2_1b(32)
    folder = convert.make_model(convert.default_model_dir(arch), arch, seed=0)
    rng = np.random.default_rng(4)
    ref = OM.RefModel(folder, context_size=1100, window=0, sink=0)
    # one sequence at context 1024: four 256-token prefill chunks, then 32 greedy steps
    p1 = rng.integers(0, arch.vocab_size, 1024).astype(np.uint32)
    eng = Engine(folder, context_size=1100, max_batch=8)
    eng.set_cache_window(0, 0)
    got = eng.generate_greedy(p1, 32).tolist()
    logits = eng.last_logits()
    assert got == ref.generate_greedy(p1.tolist(), 32)
    assert np.array_equal(_bits(logits), _bits(ref.last_logits))
    # a batch of 8 independent sequences (each prefilled as its own Model::prefill), 16 steps
    pb = rng.integers(0, arch.vocab_size, (8, 160)).astype(np.uint32)
    batch = eng.generate_batch_greedy(pb, 16)
    eng.close()
    for b in range(8):
        assert batch[b].tolist() == ref.generate_greedy(pb[b].tolist(), 16), b


def _kv(rng, B, L, Hkv, D):
    kc = np.zeros((B, L, Hkv, D), np.int8)
    vc = np.zeros_like(kc)
    ks = vs = None
    for b in range(B):
        kq, ksb = R.quantize_kv((rng.standard_normal((L, Hkv, D))).astype(np.float16))
        vq, vsb = R.quantize_kv((rng.standard_normal((L, Hkv, D))).astype(np.float16))
        kc[b], vc[b] = kq, vq
        if b == 0:  # the reference indexes the scales without a batch offset
            ks, vs = ksb, vsb
    return kc, vc, ks, vs


@pytest.mark.parametrize("B,S,L", [(1, 1, 32768), (64, 1, 4096), (1, 512, 4096)])
def test_config5_int8_cache_corners(B, S, L):
    """cactus_attention_hybrid_int8_fp16 (16 q / 8 kv heads, D = 128) at the sweep's corners."""
    L_ = cb.lib()
    Hq, Hkv, D = 16, 8, 128
    rng = np.random.default_rng(B + S + L)
    kc, vc, ks, vs = _kv(rng, B, L, Hkv, D)
    kn = rng.standard_normal((B, S, Hkv, D)).astype(np.float16)
    vn = rng.standard_normal((B, S, Hkv, D)).astype(np.float16)
    q = rng.standard_normal((B, S, Hq, D)).astype(np.float16)
    scale = 1.0 / np.sqrt(D)
    o = empty((B, S, Hq, D), np.float16)
    cb.check(L_.cactus_cuda_attention_hybrid_int8_fp16(
        ptr(dev(q)), ptr(dev(kc)), ptr(dev(vc)), ptr(dev(ks)), ptr(dev(vs)), ptr(dev(kn)), ptr(dev(vn)), ptr(o),
        B, S, L, S, Hq, Hkv, D, scale, L, 1, 128, None))
    exp = R.attention_hybrid(q, kc, vc, ks, vs, kn, vn, scale, L)
    assert np.array_equal(_bits(host(o, np.float16)), _bits(exp))


@pytest.mark.parametrize("B,L", [(1, 32768), (8, 4096), (1, 512)])
def test_config5_fp16_cache_decode(B, L):
    """The FP16 KV cache of config 5: one query after L cached fp16 keys / values through
    cactus_attention_f16 (kernel_attention.cpp:10-255), position offset L."""
    L_ = cb.lib()
    Hq, Hkv, D = 16, 8, 128
    rng = np.random.default_rng(L + B)
    k = rng.standard_normal((B, L + 1, Hkv, D)).astype(np.float16)
    v = rng.standard_normal((B, L + 1, Hkv, D)).astype(np.float16)
    q = rng.standard_normal((B, 1, Hq, D)).astype(np.float16)
    scale = 1.0 / np.sqrt(D)
    o = empty((B, 1, Hq, D), np.float16)
    cb.check(L_.cactus_cuda_attention_f16(ptr(dev(q)), ptr(dev(k)), ptr(dev(v)), ptr(o), B, 1, L + 1, Hq, Hkv, D,
                                          scale, L, 0, 1, None))
    exp = R.attention(q, k, v, scale, L, 0, True)
    assert np.array_equal(_bits(host(o, np.float16)), _bits(exp))
