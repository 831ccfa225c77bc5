"""The B200 path against the reference's OWN C++ (oracle/_ref/libcactus_ref.so: cactus/kernel,
graph, engine and models compiled from the reference tree, run on this box's host cores).

Group size 128: the reference's NEON matmuls are defined for groups that are multiples of 64
(tests/test_kernel.cpp:215,306). Shapes are chosen so that no SiLU worker chunk of the
reference ends in a scalar tail on this host (kernel_nn.cpp:13-43 with parallel_for): there
the reference takes libm's exp and its bits follow the host's core count.
"""
import numpy as np
import pytest

import cactus_b200 as cb
from cactus_b200 import convert
from cactus_b200 import weights as W
from cactus_b200.engine import Engine
from oracle import ref as RF
from tests.gpu_util import dev, empty, host, ptr

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not RF.available(), reason="reference library not built")]


def _bits(a):
    return np.asarray(a, np.float16).view(np.uint16)


def _no_silu_tails(rows, ffn):
    return not RF.chunk_tails(rows * ffn).any()


@pytest.mark.parametrize("M,int4", [(1, False), (1, True), (128, False), (7, True)])
def test_linear_g128_equals_reference(M, int4):
    """Config-1 shape (K 1024, N 3072) at G = 128: quantised activations and the grouped
    matmul through the C ABI equal cactus_fp16_max_abs / cactus_fp16_to_int8 /
    cactus_matmul_int8|int4 of the reference."""
    L = cb.lib()
    rng = np.random.default_rng(M + int4)
    w = rng.standard_normal((3072, 1024)).astype(np.float32) * np.float32(0.02)
    x = rng.standard_normal((M, 1024)).astype(np.float16)
    b, s = (W.quantize_int4 if int4 else W.quantize_int8)(w, 128)
    out = empty((M, 3072), np.float16)
    fn = L.cactus_cuda_linear_int4 if int4 else L.cactus_cuda_linear_int8
    cb.check(fn(ptr(dev(x)), ptr(dev(b)), ptr(dev(s)), ptr(out), M, 1024, 3072, 128, None), "linear")
    q, qs = RF.quantize_activations(x)
    exp = (RF.matmul_int4 if int4 else RF.matmul_int8)(q, qs, b, s, 128)
    assert np.array_equal(_bits(host(out, np.float16)), _bits(exp))


@pytest.mark.parametrize("family,prec", [
    ("qwen", None), ("gemma", {"attn": "INT8", "mlp": "INT4", "embed": "FP16"}),
    ("smol", {"attn": "INT4", "mlp": "INT4", "embed": "INT4"})])
def test_tiny_engines_equal_reference(tmp_path, family, prec):
    """Greedy generation of each family through the device engine against the reference's
    Model (prefill + decode): the same 16 tokens and the same fp16 logits."""
    kw = {"precision": prec} if prec else {}
    if family == "gemma":
        kw.update(layers=6, heads=4, kv_heads=1, head_dim=64)
    arch = convert.tiny(family, group_size=128, **{"layers": 2, **kw})
    folder = convert.make_model(str(tmp_path), arch, seed=3, norm_std=0.1)
    P = next(p for p in range(41, 200) if _no_silu_tails(p - 1, arch.ffn_intermediate_dim))
    prompt = np.random.default_rng(7).integers(0, arch.vocab_size, P).tolist()
    ref = RF.RefEngine(folder, arch.vocab_size)
    exp = ref.generate_greedy(prompt, 16)
    eng = Engine(folder, context_size=512)
    got = eng.generate_greedy(prompt, 16).tolist()
    assert got == exp
    assert np.array_equal(_bits(eng.last_logits()), _bits(ref.last_logits))
    eng.close()
    ref.close()


def test_qwen3_0_6b_g128_greedy_equals_reference():
    """Config-2 shape (28 layers, hidden 1024, 16/8 heads, FFN 3072, vocab 151936) with INT8
    group-128 weights: 128 random prompt ids, then 32 greedy steps through the persistent
    decode step; every token and the last step's 151936 fp16 logits equal the reference's."""
    arch = convert.qwen3_0_6b(128)
    folder = convert.make_model(convert.default_model_dir(arch), arch, seed=0)
    assert _no_silu_tails(127, arch.ffn_intermediate_dim) and _no_silu_tails(1, arch.ffn_intermediate_dim)
    prompt = np.random.default_rng(0).integers(0, arch.vocab_size, 128).tolist()
    eng = Engine(folder, context_size=512)
    got = eng.generate_greedy(prompt, 32).tolist()
    assert eng.decode_path() == 2
    ref = RF.RefEngine(folder, arch.vocab_size)
    exp = ref.generate_greedy(prompt, 32)
    assert got == exp
    assert np.array_equal(_bits(eng.last_logits()), _bits(ref.last_logits))
    eng.close()
    ref.close()
