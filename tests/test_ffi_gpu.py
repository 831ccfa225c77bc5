"""The reference's C FFI (include/cactus_ffi.h) and the device sampler.

cactus_init / cactus_complete / cactus_tokenize / cactus_reset / cactus_destroy behave as
cactus/ffi/cactus_init.cpp and cactus_complete.cpp (JSON fields, defaults, prefix reuse,
error JSON); the non-greedy sampler matches the restatement of cactus_sample_f16.
"""
import ctypes as C
import json

import numpy as np
import pytest

import cactus_b200 as cb
from cactus_b200 import convert
from oracle import model as OM
from oracle import sample as OS
from tests.gpu_util import dev, empty, host, ptr

pytestmark = pytest.mark.gpu

CALLBACK = C.CFUNCTYPE(None, C.c_char_p, C.c_uint32, C.c_void_p)


@pytest.fixture(scope="module")
def folder(tmp_path_factory):
    return convert.make_model(str(tmp_path_factory.mktemp("ffi_qwen")), convert.tiny("qwen", layers=2), seed=5,
                              norm_std=0.1)


def _complete(L, h, content, options):
    buf = C.create_string_buffer(1 << 16)
    msgs = json.dumps([{"role": "user", "content": content}]).encode()
    got = []
    cbf = CALLBACK(lambda tok, tid, ud: got.append(int(tid)))
    n = L.cactus_complete(h, msgs, buf, len(buf), json.dumps(options).encode(), None, cbf, None)
    return n, json.loads(buf.value.decode()), got


def test_complete_streams_tokens_and_reuses_prefix(folder):
    L = cb.lib()
    h = L.cactus_init(folder.encode(), None)
    assert h, L.cactus_get_last_error()
    prompt = np.random.default_rng(2).integers(0, 1000, 12).tolist()
    # greedy at graph level needs top_k 0 after Model::decode's defaulting, so the FFI path
    # samples; with temperature 0 and top_k 1 the single survivor is the argmax of the
    # repetition-penalised logits
    opts = {"max_tokens": 6, "temperature": 0.0, "top_p": 0.0, "top_k": 1, "confidence_threshold": 0.0}
    n, r, streamed = _complete(L, h, " ".join(map(str, prompt)), opts)
    assert n > 0 and r["success"] is True and r["cloud_handoff"] is False
    toks = [int(t) for t in r["response"].split()]
    assert len(toks) == 6 and streamed == toks
    assert r["prefill_tokens"] == 12 and r["decode_tokens"] == 6
    # before any token enters the process-wide repetition history, top_k 1 is the argmax
    ref = OM.RefModel(folder, context_size=512)
    assert toks[0] == ref.generate_greedy(prompt, 1)[0]
    # tokenization round trip
    out = (C.c_uint32 * 32)()
    nt = C.c_size_t(0)
    assert L.cactus_tokenize(h, b"5 6, 7", out, 32, C.byref(nt)) == 0 and list(out[:nt.value]) == [5, 6, 7]
    assert L.cactus_tokenize(h, b"1 2 3", out, 2, C.byref(nt)) == -2
    # a follow-up conversation that extends the processed tokens only prefills the suffix
    n2, r2, _ = _complete(L, h, " ".join(map(str, prompt + toks + [7, 8])), opts)
    assert r2["success"] and r2["prefill_tokens"] == 2
    L.cactus_reset(h)
    n3, r3, _ = _complete(L, h, " ".join(map(str, prompt)), opts)
    assert r3["prefill_tokens"] == 12
    L.cactus_destroy(h)


def test_complete_errors_and_cloud_handoff(folder):
    L = cb.lib()
    buf = C.create_string_buffer(4096)
    assert L.cactus_complete(None, b"[]", buf, len(buf), None, None, None, None) == -1
    assert json.loads(buf.value)["success"] is False
    assert L.cactus_init(b"/nonexistent/model", None) is None
    assert b"Failed to initialize" in L.cactus_get_last_error()
    h = L.cactus_init(folder.encode(), None)
    assert L.cactus_complete(h, b"[]", buf, len(buf), None, None, None, None) == -1
    assert "No messages" in json.loads(buf.value)["error"]
    # the default confidence threshold 0.7 hands a near-uniform random-init model to the cloud
    n, r, _ = _complete(L, h, "1 2 3 4", {"max_tokens": 4})
    assert n > 0 and r["cloud_handoff"] is True and r["success"] is False
    small = C.create_string_buffer(16)
    msgs = json.dumps([{"role": "user", "content": "1 2 3"}]).encode()
    assert L.cactus_complete(h, msgs, small, len(small), b'{"confidence_threshold": 0}', None, None, None) == -1
    L.cactus_destroy(h)


@pytest.mark.parametrize("temp,top_p,top_k,u", [(0.0, 0.0, 20, 0.37), (0.7, 0.0, 20, 0.91), (1.0, 0.9, 40, 0.5),
                                                (0.6, 0.95, 20, 0.02), (0.0, 0.0, 1, 0.5), (1.3, 0.5, 64, 0.999)])
def test_sampler_matches_restatement(temp, top_p, top_k, u):
    L = cb.lib()
    rng = np.random.default_rng(int(u * 1000) + top_k)
    V = 5000
    logits = (rng.standard_normal(V) * 3).astype(np.float16)
    logits[17] = logits.max()  # a tie at the top
    hist = rng.integers(0, V, 10).astype(np.uint32)
    work = empty((V,), np.float16)
    out = empty((1,), np.uint32)
    cb.check(L.cactus_cuda_sample_f16(ptr(dev(logits)), 1, V, temp, top_p, top_k, u, ptr(dev(hist)), len(hist),
                                      ptr(work), ptr(out), None))
    assert int(host(out, np.uint32)[0]) == OS.sample_f16(logits, temp, top_p, top_k, u, hist.tolist())


@pytest.mark.parametrize("V,temp,top_p,top_k,u,ties", [
    (5000, 0.7, 0.0, 0, 0.5, 0),        # no top-k, no top-p: all 5000 logits survive
    (5000, 0.7, 0.0, 0, 0.999, 0),
    (5000, 1.0, 0.9, 0, 0.3, 0),        # top-p over all logits (no top-k)
    (5000, 0.0, 0.5, 0, 0.8, 0),        # top-p alone at temperature 0
    (5000, 0.8, 0.0, 2000, 0.6, 0),     # top-k beyond the shared-memory candidate list
    (5000, 0.9, 0.7, 1500, 0.4, 0),
    (5000, 0.7, 0.0, 20, 0.5, 2000),    # 2000 equal logits with top-k 20: ties keep all 2000
    (5000, 1.0, 0.6, 20, 0.7, 2000),    # the top-p cut falls inside a run of equal values
    (151936, 0.6, 0.9, 0, 0.42, 0),     # the Qwen vocabulary with top-p only
])
def test_sampler_many_candidates_match_restatement(V, temp, top_p, top_k, u, ties):
    """More survivors than the 1024-entry shared-memory list (kernel_nn.cpp:520-650 with
    any top_k): the top-p runs and the final in-order draw walk all V entries."""
    L = cb.lib()
    rng = np.random.default_rng(V + top_k + ties + int(u * 100))
    logits = (rng.standard_normal(V) * 3).astype(np.float16)
    if ties:
        logits[:] = np.minimum(logits, np.float16(5.0))
        logits[rng.permutation(V)[:ties]] = np.float16(6.0)
    hist = rng.integers(0, V, 10).astype(np.uint32)
    work = empty((V,), np.float16)
    exp = OS.sample_f16(logits, temp, top_p, top_k, u, hist.tolist())
    for entry in ("sample", "noalloc"):
        out = empty((1,), np.uint32)
        if entry == "sample":
            cb.check(L.cactus_cuda_sample_f16(ptr(dev(logits)), 1, V, temp, top_p, top_k, u, ptr(dev(hist)),
                                              len(hist), ptr(work), ptr(out), None))
        else:
            cb.check(L.cactus_cuda_sample_f16_noalloc(ptr(dev(logits)), 1, V, temp, top_p, top_k, u,
                                                      ptr(dev(hist)), len(hist), ptr(out), None))
        assert int(host(out, np.uint32)[0]) == exp, entry
    assert L.cactus_cuda_device_error(None) == 0


def test_entropy_kernel():
    L = cb.lib()
    rng = np.random.default_rng(4)
    logits = rng.standard_normal(3000).astype(np.float16)
    out = empty((1,), np.float32)
    cb.check(L.cactus_cuda_entropy_f16(ptr(dev(logits)), 1, 3000, ptr(out), None))
    x = logits.astype(np.float64)
    p = np.exp(x - x.max())
    p /= p.sum()
    ent = -(p[p > 1e-10] * np.log(p[p > 1e-10])).sum() / np.log(3000)
    assert abs(float(host(out, np.float32)[0]) - ent) < 1e-5
