"""Engine-level parity on the B200: greedy generations and KV-cache contents of the
device-resident engine against the CPU restatement of the reference engine (oracle/model.py).

Greedy parity = identical argmax tokens (graph-level sample(logits, 0, 0, 0)); the logits
themselves are compared with the north-star tolerance (normwise max relative error <= 1e-2).
"""
import os

import numpy as np
import pytest

from cactus_b200 import convert
from cactus_b200.engine import Engine
from oracle import model as OM

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


TINY = {
    "qwen": lambda: convert.tiny("qwen", layers=2),
    "gemma": lambda: convert.tiny("gemma", layers=6, heads=4, kv_heads=1, head_dim=64, hidden=256, ffn=512,
                                  precision={"attn": "INT8", "mlp": "INT4", "embed": "FP16"}),
    "smol": lambda: convert.tiny("smol", layers=2, precision={"attn": "INT4", "mlp": "INT4", "embed": "INT4"},
                                 theta=5e5),
    "qwen_g128": lambda: convert.tiny("qwen", layers=2, group_size=128),
}


@pytest.fixture(scope="module")
def folders(tmp_path_factory):
    out = {}
    for k, fn in TINY.items():
        out[k] = convert.make_model(str(tmp_path_factory.mktemp(k)), fn(), seed=3, norm_std=0.1)
    return out


@pytest.mark.parametrize("kind", list(TINY))
def test_greedy_generation_matches_oracle(folders, kind):
    folder = folders[kind]
    prompt = np.random.default_rng(7).integers(0, 1000, 21).tolist()
    eng = Engine(folder, context_size=512)
    got = eng.generate_greedy(prompt, 16).tolist()
    ref = OM.RefModel(folder, context_size=512)
    exp = ref.generate_greedy(prompt, 16)
    assert got == exp
    assert _rel(eng.last_logits(), ref.last_logits) <= TOL
    # the KV cache holds the same INT8 values and scales
    n, total = eng.kv_state()
    assert (n, total) == (ref.kv.current, ref.kv.total)
    # layer 0's keys/values depend only on bit-exact kernels: identical INT8 bytes and scales
    k, v, ks, vs = eng.read_kv(0)
    assert np.array_equal(k, ref.kv.k[0][:n]) and np.array_equal(v, ref.kv.v[0][:n])
    assert np.array_equal(ks, ref.kv.ks[0][:n]) and np.array_equal(vs, ref.kv.vs[0][:n])
    last = ref.cfg["num_layers"] - 1
    k, v, ks, vs = eng.read_kv(last)
    deq = lambda q, s: q.astype(np.float32).reshape(q.shape[0], q.shape[1], s.shape[-1], -1) * s[..., None]
    assert _rel(deq(k, ks), deq(ref.kv.k[last][:n], ref.kv.ks[last][:n])) <= TOL
    eng.close()


def test_prefill_chunks_and_long_prompt(folders):
    """Model::prefill splits prompts longer than the chunk (engine_model.cpp:198-218)."""
    folder = folders["qwen"]
    prompt = np.random.default_rng(8).integers(0, 1000, 300).tolist()
    eng = Engine(folder, context_size=1024)
    eng.set_cache_window(0, 0)
    got = eng.generate_greedy(prompt, 8).tolist()
    ref = OM.RefModel(folder, context_size=1024, window=0, sink=0)
    assert got == ref.generate_greedy(prompt, 8)
    eng.close()


def test_causal_fix_mode_after_the_window_slid(folders):
    """A 300-token prompt with window 128: the second prefill chunk runs after the cache slid,
    where the reference's mask uses the total position (its queries see the chunk's later
    keys). Default mode reproduces that; cactus_engine_set_causal_fix masks by the cache
    index. Both match the restatement in the same mode, and the two modes differ."""
    folder = folders["qwen"]
    prompt = np.random.default_rng(13).integers(0, 1000, 300).tolist()
    logits = {}
    for fix in (False, True):
        eng = Engine(folder, context_size=512)
        eng.set_cache_window(128, 4)
        eng.set_causal_fix(fix)
        got = eng.generate_greedy(prompt, 8).tolist()
        logits[fix] = eng.last_logits()
        eng.close()
        ref = OM.RefModel(folder, context_size=512, window=128, sink=4, causal_fix=fix)
        assert got == ref.generate_greedy(prompt, 8)
        assert _rel(logits[fix], ref.last_logits) <= TOL
    assert not np.array_equal(logits[False].view(np.uint16), logits[True].view(np.uint16))


def test_sliding_window_matches_oracle(folders):
    """Sink + sliding window cache (engine_cache.cpp:163-329) with window 16 and 4 sinks."""
    folder = folders["qwen"]
    prompt = np.random.default_rng(9).integers(0, 1000, 11).tolist()
    eng = Engine(folder, context_size=64)
    eng.set_cache_window(16, 4)
    got = eng.generate_greedy(prompt, 20).tolist()
    ref = OM.RefModel(folder, context_size=64, window=16, sink=4)
    exp = ref.generate_greedy(prompt, 20)
    assert got == exp
    assert eng.kv_state() == (ref.kv.current, ref.kv.total) == (16, 30)
    k, v, ks, vs = eng.read_kv(1)
    assert np.array_equal(k, ref.kv.k[1]) and np.array_equal(ks, ref.kv.ks[1])
    eng.close()


def test_batched_sequences_are_independent(folders):
    """Independent sequences decoded together equal their single-sequence runs (config 4 path)."""
    folder = folders["smol"]
    prompts = np.random.default_rng(10).integers(0, 1000, (4, 9)).astype(np.uint32)
    eng = Engine(folder, context_size=256, max_batch=4)
    batch = eng.generate_batch_greedy(prompts, 8)
    ref = OM.RefModel(folder, context_size=256)
    for b in range(4):
        single = eng.generate_greedy(prompts[b], 8)
        assert batch[b].tolist() == single.tolist()
        assert single.tolist() == ref.generate_greedy(prompts[b].tolist(), 8)
    eng.close()


def test_batched_llama_ffn_width_matches_oracle(tmp_path_factory):
    """Llama-3.2-1B's FFN width (8192, INT4 G32): the down projection's K = 8192 limits one GEMV
    launch to 4 activation rows, so a batch of 6 runs it in row chunks."""
    arch = convert.tiny("smol", layers=1, hidden=256, ffn=8192, heads=4, kv_heads=2, head_dim=64,
                        precision={"attn": "INT4", "mlp": "INT4", "embed": "INT4"}, theta=5e5)
    folder = convert.make_model(str(tmp_path_factory.mktemp("llama_ffn")), arch, seed=5, norm_std=0.1)
    prompts = np.random.default_rng(11).integers(0, 1000, (6, 7)).astype(np.uint32)
    eng = Engine(folder, context_size=128, max_batch=6)
    batch = eng.generate_batch_greedy(prompts, 6)
    eng.close()
    ref = OM.RefModel(folder, context_size=128)
    for b in range(6):
        assert batch[b].tolist() == ref.generate_greedy(prompts[b].tolist(), 6)


@pytest.mark.parametrize("kind,batch", [("gemma", 1), ("smol", 3)])
def test_graph_decode_over_long_cache_matches_oracle(folders, kind, batch):
    """Decode graphs over caches of 512+ keys run the exact key-split attention with the
    lengths read on the device; tokens must equal the oracle's for every sequence."""
    folder = folders[kind]
    P = 530
    prompts = np.random.default_rng(12).integers(0, 1000, (batch, P)).astype(np.uint32)
    ref = OM.RefModel(folder, context_size=600, window=0, sink=0)
    exp = [ref.generate_greedy(prompts[b].tolist(), 6) for b in range(batch)]
    eng = Engine(folder, context_size=600, max_batch=batch)
    eng.set_cache_window(0, 0)
    got = eng.generate_batch_greedy(prompts, 6) if batch > 1 else eng.generate_greedy(prompts[0], 6)[None]
    assert eng.decode_path() == 1  # the CUDA-graph decode
    for b in range(batch):
        assert got[b].tolist() == exp[b]
    if batch == 1:
        assert _rel(eng.last_logits(), ref.last_logits) <= TOL
    eng.close()


PERSISTENT_KINDS = {
    "qwen": lambda: convert.tiny("qwen", layers=2),
    "qwen_g128": lambda: convert.tiny("qwen", layers=2, group_size=128),
    "qwen_d128": lambda: convert.tiny("qwen", layers=3, heads=4, kv_heads=1, head_dim=128, hidden=384, ffn=768,
                                      vocab=2048),
    "llama_int8": lambda: convert.tiny("smol", layers=2, theta=5e5),
    "smol_576": lambda: convert.tiny("smol", layers=2, hidden=576, heads=9, kv_heads=3, head_dim=64, ffn=1536,
                                     theta=1e5),
}


@pytest.mark.parametrize("kind", list(PERSISTENT_KINDS))
def test_persistent_decode_matches_graph_path_and_oracle(tmp_path_factory, kind):
    """The single-launch persistent decode step and the per-op CUDA-graph path produce the
    same tokens, bit-identical logits and KV-cache bytes, and both match the oracle."""
    folder = convert.make_model(str(tmp_path_factory.mktemp("p_" + kind)), PERSISTENT_KINDS[kind](), seed=4,
                                norm_std=0.1)
    prompt = np.random.default_rng(9).integers(0, 1000, 40).tolist()
    res = {}
    for mode in (-1, 1):
        eng = Engine(folder, context_size=512)
        eng.decode_path(mode)
        toks = eng.generate_greedy(prompt, 24).tolist()
        res[mode] = (toks, eng.decode_path(), eng.last_logits(), eng.read_kv(1), eng.kv_state())
        eng.close()
    assert res[-1][1] == 2 and res[1][1] == 1
    assert res[-1][0] == res[1][0]
    assert np.array_equal(res[-1][2].view(np.uint16), res[1][2].view(np.uint16))
    for a, b in zip(res[-1][3], res[1][3]):
        assert np.array_equal(a, b)
    assert res[-1][4] == res[1][4]
    ref = OM.RefModel(folder, context_size=512)
    assert res[-1][0] == ref.generate_greedy(prompt, 24)


def test_bounded_waits_give_up_and_the_next_call_succeeds(tmp_path_factory):
    """Every wait of the persistent decode step is bounded. With the bound lowered to one poll
    (CACTUS_B200_SPIN_LIMIT, read when an engine is created) the first wait on a weight slot or
    on another block's tagged activations gives up: the step raises the abort word, every block
    leaves at its next wait (the producer after its copies in flight land), the call reports
    the failure and the device error word records it. Nothing faults; an engine created
    afterwards decodes normally in the same process."""
    import cactus_b200 as cb
    folder = convert.make_model(str(tmp_path_factory.mktemp("spin")), PERSISTENT_KINDS["qwen"](), seed=4,
                                norm_std=0.1)
    prompt = np.random.default_rng(9).integers(0, 1000, 40).tolist()
    L = cb.lib()
    assert L.cactus_cuda_device_error(None) == 0
    os.environ["CACTUS_B200_SPIN_LIMIT"] = "1"
    try:
        eng = Engine(folder, context_size=512)
        with pytest.raises(cb.CactusError, match="bounded wait"):
            eng.generate_greedy(prompt, 4)
        assert eng.decode_path() == 2
        eng.close()
    finally:
        del os.environ["CACTUS_B200_SPIN_LIMIT"]
    assert L.cactus_cuda_device_error(None) in (1, 2)  # a slot (TMA) or tagged-word (flag) timeout
    assert L.cactus_cuda_device_error(None) == 0       # reading it cleared it
    eng = Engine(folder, context_size=512)
    got = eng.generate_greedy(prompt, 8).tolist()
    assert eng.decode_path() == 2
    eng.close()
    assert got == OM.RefModel(folder, context_size=512).generate_greedy(prompt, 8)
    assert L.cactus_cuda_device_error(None) == 0


def test_engine_rejects_out_of_range_tokens(folders):
    eng = Engine(folders["qwen"], context_size=64)
    with pytest.raises(Exception, match="out of bounds"):
        eng.generate_greedy([5, 1000000], 2)
    eng.close()


@pytest.mark.skipif(os.environ.get("CACTUS_SKIP_FULL") == "1", reason="full-size model disabled")
def test_qwen3_0_6b_greedy_32_tokens_identical(tmp_path_factory):
    """Config 2: Qwen3-0.6B-shaped INT8 (group 32) random-init model, 128 random prompt ids,
    32 greedy steps identical to the CPU restatement."""
    arch = convert.qwen3_0_6b(32)
    folder = convert.make_model(convert.default_model_dir(arch), arch, seed=0)
    prompt = np.random.default_rng(0).integers(0, arch.vocab_size, 128).tolist()
    eng = Engine(folder, context_size=512)
    got = eng.generate_greedy(prompt, 32).tolist()
    assert eng.decode_path() == 2  # the persistent single-launch step
    ref = OM.RefModel(folder, context_size=512)
    exp = ref.generate_greedy(prompt, 32)
    assert got == exp
    assert _rel(eng.last_logits(), ref.last_logits) <= TOL
    eng.close()
