"""CPU checks of the model-level oracle (oracle/model.py) and of the synthetic-model writer."""
import numpy as np
import pytest

from cactus_b200 import convert
from oracle import model as OM


def _fill(n, hk, d, value):
    return np.full((n, hk, d), value, np.float16)


def test_kv_cache_sliding_window_pin():
    """tests/test_kv_cache.cpp:21-131: window 16, sink 4; updates of 10, 6 and 10 tokens
    leave 16 cached tokens, the sink intact and total_seq_len 26."""
    L, H, D = 2, 8, 64
    kv = OM.RefKVCache(L, H, D, window=16, sink=4)
    kv.update([_fill(10, H, D, l + 1.0) for l in range(L)], [_fill(10, H, D, l + 2.0) for l in range(L)], 10)
    assert kv.current == 10
    kv.update([_fill(6, H, D, l + 10.0) for l in range(L)], [_fill(6, H, D, l + 20.0) for l in range(L)], 6)
    assert kv.current == 16
    kv.update([_fill(10, H, D, 100.0) for _ in range(L)], [_fill(10, H, D, 100.0) for _ in range(L)], 10)
    assert kv.current == 16 and kv.total == 26
    sink_q = np.round(1.0 / kv.ks[0][0, 0, 0])
    assert np.all(np.abs(kv.k[0][:4].astype(np.int32) - sink_q) <= 2)
    # newest tokens sit at the end of the window
    deq = kv.k[0][-10:].astype(np.float32) * kv.ks[0][-10:]
    assert np.allclose(deq, 100.0, rtol=1e-2)


def test_kv_cache_first_update_longer_than_window():
    """engine_cache.cpp:163-231: a first update longer than the window keeps the sink tokens
    and the most recent window - sink tokens."""
    kv = OM.RefKVCache(1, 1, 32, window=8, sink=2)
    toks = np.stack([np.full((1, 32), t + 1, np.float16) for t in range(20)])
    kv.update([toks], [toks], 20)
    deq = (kv.k[0].astype(np.float32) * kv.ks[0]).reshape(8, 32)[:, 0]
    assert np.allclose(deq, [1, 2, 15, 16, 17, 18, 19, 20], rtol=1e-2)


@pytest.fixture(scope="module")
def tiny_folder(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tiny_qwen"))
    return convert.make_model(d, convert.tiny("qwen", layers=2), seed=0, norm_std=0.1)


def test_oracle_greedy_is_deterministic_and_incremental(tiny_folder):
    m = OM.RefModel(tiny_folder)
    prompt = np.random.default_rng(1).integers(0, 1000, 12).tolist()
    a = m.generate_greedy(prompt, 6)
    b = m.generate_greedy(prompt, 6)
    assert a == b and all(0 <= t < 1000 for t in a)
    # prefill in chunks gives the same continuation as one chunk (chunked prefill path)
    m.kv.reset()
    m.prefill(prompt[:-1], chunk=4)
    c = [m.decode_argmax([prompt[-1]])]
    assert c[0] == a[0]


def test_synthetic_model_layout(tiny_folder):
    import os
    names = set(os.listdir(tiny_folder))
    for n in ("config.txt", "token_embeddings.weights", "output_norm.weights", "layer_0_attn_q.weights",
              "layer_1_ffn_down.weights", "layer_0_attn_q_norm.weights"):
        assert n in names
    cfg = OM.read_config(tiny_folder)
    assert cfg["num_layers"] == 2 and cfg["model_type"] == "qwen"
