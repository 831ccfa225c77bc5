"""ctypes wrapper over oracle/_ref/libcactus_ref.so — TEST INFRASTRUCTURE ONLY.

That library is the reference's OWN C++ (cactus/kernel, cactus/graph, cactus/engine,
cactus/models of the reference tree), compiled on this x86-64 host by ``make -C oracle ref``
against oracle/neon_shim/arm_neon.h, a portable restatement of the NEON intrinsics it uses,
plus oracle/ref_api.cpp (C entry points). It is the checker that pins the restatement
(oracle/refcpu.c, oracle/model.py) and the GPU path to the reference's actual outputs.

Caveat stated by the reference's own tests ("group_size must be >= 64",
tests/test_kernel.cpp:215,306): its NEON matmuls walk each quantisation group in 64-element
steps, so they are defined for group sizes that are multiples of 64. Comparisons against
this library use G = 64 or 128; G = 32 is pinned through the restatement's group formula.

The library is built only where the reference tree is present (this container); the built
file travels to the GPU box with the repository. ``available()`` says whether it can be loaded.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_ref", "libcactus_ref.so")
REF_TREE = os.environ.get("CACTUS_REFERENCE_TREE", "/root/reference")
_lib = None


def build(force: bool = False) -> str | None:
    """Compile the reference into oracle/_ref/ when its source tree is present."""
    if not os.path.isdir(os.path.join(REF_TREE, "cactus", "kernel")):
        return _SO if os.path.exists(_SO) else None
    jobs = str(max(1, min(16, os.cpu_count() or 1)))
    subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={REF_TREE}", "-j", jobs] + (["-B"] if force else []),
                   check=True)
    return _SO


def available() -> bool:
    return os.path.exists(_SO)


P = C.c_void_p
Z = C.c_size_t
F = C.c_float
I = C.c_int
U32 = C.c_uint32


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError("oracle/_ref/libcactus_ref.so is not built (make -C oracle ref)")
        L = C.CDLL(_SO)
        sig = {
            "ref_last_error": (C.c_char_p, []),
            "ref_model_create": (P, [C.c_char_p, Z]),
            "ref_model_destroy": (None, [P]),
            "ref_model_prefill": (I, [P, P, Z, Z]),
            "ref_model_decode_greedy": (I, [P, P, Z, P, P, Z]),
            "ref_model_decode": (I, [P, P, Z, F, F, Z, P]),
            "ref_model_reset": (I, [P]),
            "ref_model_forward_hidden": (I, [P, P, Z, P, I]),
            "ref_model_cache": (Z, [P, Z, P, P, P, P]),
            "ref_model_set_window": (I, [P, Z, Z]),
            "ref_matmul_int8": (None, [P, P, P, P, P, Z, Z, Z, Z]),
            "ref_matmul_int4": (None, [P, P, P, P, P, Z, Z, Z, Z]),
            "ref_matmul_f16": (None, [P, P, P, Z, Z, Z]),
            "ref_fp16_to_int8": (None, [P, P, Z, F]),
            "ref_fp16_max_abs": (F, [P, Z]),
            "ref_rms_norm": (None, [P, P, P, Z, Z, F]),
            "ref_conv1d_causal_depthwise": (None, [P, P, P, Z, Z, Z, Z, Z]),
            "ref_conv1d_k3": (None, [P, P, P, Z, Z, Z, Z, Z]),
            "ref_layernorm": (I, [P, P, P, P, Z, Z, F]),
            "ref_rope": (None, [P, P, Z, Z, Z, Z, Z, F]),
            "ref_softmax": (None, [P, P, Z, Z, Z]),
            "ref_silu": (None, [P, P, Z]),
            "ref_gelu": (None, [P, P, Z]),
            "ref_add": (None, [P, P, P, Z]),
            "ref_add_clipped": (None, [P, P, P, Z]),
            "ref_multiply": (None, [P, P, P, Z]),
            "ref_attention_f16": (None, [P, P, P, P, Z, Z, Z, Z, Z, Z, F, Z, Z, I]),
            "ref_attention_hybrid": (None, [P, P, P, P, P, P, P, P, Z, Z, Z, Z, Z, Z, Z, F, Z, I]),
            "ref_quantize_kv": (None, [P, P, P, Z, Z, Z]),
            "ref_unpack_int4": (None, [P, P, Z]),
            "ref_sample_f16": (None, [P, P, Z, F, F, Z, Z]),
            "ref_mt19937_uniform": (F, [Z]),
            "ref_pool_workers": (Z, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(P)


def _h(a):
    return np.ascontiguousarray(a, dtype=np.float16)


def err():
    return lib().ref_last_error().decode()


# ---- kernels ----
def quantize_activations(x):
    """graph_ops_nn.cpp:35-66 built from the reference's own cactus_fp16_max_abs / cactus_fp16_to_int8."""
    x = _h(x)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float32)
    L = lib()
    for m in range(M):
        row = np.ascontiguousarray(x[m])
        mx = L.ref_fp16_max_abs(_p(row), K)
        sc = np.float32(mx) / np.float32(127.0)
        if sc < np.float32(1e-10):
            sc = np.float32(1e-10)
        s[m] = sc
        out = np.empty(K, np.int8)
        L.ref_fp16_to_int8(_p(row), _p(out), K, float(sc))
        q[m] = out
    return q, s


def matmul_int8(a, a_scales, b, b_scales, group):
    a = np.ascontiguousarray(a, np.int8)
    M, K = a.shape
    N = b.shape[0]
    c = np.empty((M, N), np.float16)
    lib().ref_matmul_int8(_p(a), _p(np.ascontiguousarray(a_scales, np.float32)), _p(np.ascontiguousarray(b, np.int8)),
                          _p(_h(b_scales)), _p(c), M, K, N, group)
    return c


def matmul_int4(a, a_scales, b_packed, b_scales, group):
    a = np.ascontiguousarray(a, np.int8)
    M, K = a.shape
    N = b_packed.shape[0]
    c = np.empty((M, N), np.float16)
    lib().ref_matmul_int4(_p(a), _p(np.ascontiguousarray(a_scales, np.float32)),
                          _p(np.ascontiguousarray(b_packed, np.uint8)), _p(_h(b_scales)), _p(c), M, K, N, group)
    return c


def matmul_f16(a, bt):
    a, bt = _h(a), _h(bt)
    M, K = a.shape
    N = bt.shape[0]
    c = np.empty((M, N), np.float16)
    lib().ref_matmul_f16(_p(a), _p(bt), _p(c), M, K, N)
    return c


def rms_norm(x, w, eps):
    x = _h(x)
    y = np.empty_like(x)
    lib().ref_rms_norm(_p(x), _p(_h(w)), _p(y), x.shape[0], x.shape[1], eps)
    return y


def conv1d_causal_depthwise(x, w, dilation=1):
    x, w = _h(x), _h(w)
    N, L, C = x.shape
    y = np.empty_like(x)
    lib().ref_conv1d_causal_depthwise(_p(x), _p(w), _p(y), N, L, C, w.shape[1], dilation)
    return y


def conv1d_k3(x, w, stride=1):
    x, w = _h(x), _h(w)
    N, Cin, L = x.shape
    y = np.empty((N, w.shape[0], (L - 1) // stride + 1), np.float16)
    lib().ref_conv1d_k3(_p(x), _p(w), _p(y), N, L, Cin, w.shape[0], stride)
    return y


def layernorm(x, w, b, eps):
    """The reference's LAYERNORM graph node, run through a one-node CactusGraph."""
    x = _h(x)
    y = np.empty_like(x)
    if lib().ref_layernorm(_p(x), _p(_h(w)), _p(_h(b)), _p(y), x.shape[0], x.shape[1], eps) != 0:
        raise RuntimeError(lib().ref_last_error().decode())
    return y


def rope(x, start, theta):
    x = _h(x)
    B, S, H, D = x.shape
    y = np.empty_like(x)
    lib().ref_rope(_p(x), _p(y), B, S, H, D, start, theta)
    return y


def softmax(x):
    x = _h(x)
    y = np.empty_like(x)
    lib().ref_softmax(_p(x), _p(y), 1, x.shape[0], x.shape[1])
    return y


def _unary(name, x):
    x = _h(x)
    y = np.empty_like(x)
    getattr(lib(), name)(_p(x), _p(y), x.size)
    return y


def silu(x):
    return _unary("ref_silu", x)


def gelu(x):
    return _unary("ref_gelu", x)


def _binary(name, a, b):
    a, b = _h(a), _h(b)
    y = np.empty_like(a)
    getattr(lib(), name)(_p(a), _p(b), _p(y), a.size)
    return y


def add(a, b):
    return _binary("ref_add", a, b)


def add_clipped(a, b):
    return _binary("ref_add_clipped", a, b)


def multiply(a, b):
    return _binary("ref_multiply", a, b)


def attention(q, k, v, scale, pos_offset=0, window=0, causal=True):
    q, k, v = _h(q), _h(k), _h(v)
    B, S, Hq, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    o = np.empty_like(q)
    lib().ref_attention_f16(_p(q), _p(k), _p(v), _p(o), B, S, Skv, Hq, Hkv, D, scale, pos_offset, window, int(causal))
    return o


def attention_hybrid(q, kc, vc, ks, vs, kn, vn, scale, pos_offset, causal=True):
    q, kn, vn = _h(q), _h(kn), _h(vn)  # q [1, S, Hq, D]; new keys / values [1, S, Hkv, D]
    B, S, Hq, D = q.shape
    Hkv = kn.shape[2]
    o = np.empty_like(q)
    kc, vc = np.ascontiguousarray(kc, np.int8), np.ascontiguousarray(vc, np.int8)
    ks, vs = np.ascontiguousarray(ks, np.float32), np.ascontiguousarray(vs, np.float32)
    lib().ref_attention_hybrid(_p(q), _p(kc), _p(vc), _p(ks), _p(vs), _p(kn), _p(vn), _p(o), B, S, kc.shape[0],
                               kn.shape[1], Hq, Hkv, D, scale, pos_offset, int(causal))
    return o


def quantize_kv(x):
    x = _h(x)
    S, H, D = x.shape
    q = np.empty((S, H, D), np.int8)
    s = np.empty((S, H, (D + 127) // 128), np.float32)
    lib().ref_quantize_kv(_p(x), _p(q), _p(s), S, H, D)
    return q, s


def unpack_int4(packed, count):
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.empty(count, np.int8)
    lib().ref_unpack_int4(_p(packed), _p(out), count)
    return out


def sample_f16(logits, temperature, top_p, top_k, seed):
    """cactus_sample_f16 as compiled (its process-wide repetition history included)."""
    x = _h(logits)
    out = np.zeros(1, np.uint32)
    lib().ref_sample_f16(_p(x), _p(out), x.size, temperature, top_p, top_k, seed)
    return int(out[0])


def chunk_tails(n, gate=2500, per_thread=1250):
    """Positions where cactus_silu_f16 / cactus_gelu_f16 (parallel_for with SCALAR_EXPENSIVE
    {2500, 1250}, kernel_utils.h:410-437) run their scalar libm tail on this host: the last
    (chunk length % 8) elements of every worker chunk."""
    workers = int(lib().ref_pool_workers())
    t = 1 if n < gate else min(workers, max(1, -(-n // per_thread)))
    per = n // t  # parallel_for (kernel_utils.h:516-548): equal chunks, the last one takes the rest
    mask = np.zeros(n, bool)
    for w in range(t):
        start, end = w * per, (n if w == t - 1 else (w + 1) * per)
        mask[start + ((end - start) // 8) * 8:end] = True
    return mask


def pool_workers():
    return int(lib().ref_pool_workers())


def mt19937_uniform(seed):
    """The uniform sample cactus_sample_f16 draws for a given non-zero seed."""
    return float(lib().ref_mt19937_uniform(seed))


# ---- engine ----
def write_vocab(folder, vocab_size):
    """Model::init loads a tokenizer; a plain one-token-per-line vocab.txt satisfies it (the
    random-token workloads never encode text)."""
    path = os.path.join(folder, "vocab.txt")
    if not os.path.exists(path):
        with open(path, "w") as f:
            f.write("".join(f"t{i}\n" for i in range(vocab_size)))


class RefEngine:
    """The reference's Model (create_model's Qwen / Gemma / Smol classes) on a model folder."""

    def __init__(self, folder, vocab_size, context_size=512):
        write_vocab(folder, vocab_size)
        self.V = vocab_size
        self.h = lib().ref_model_create(folder.encode(), context_size)
        if not self.h:
            raise RuntimeError("reference Model::init failed: " + err())
        self.last_logits = None

    def close(self):
        if self.h:
            lib().ref_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def reset(self):
        lib().ref_model_reset(self.h)

    def set_window(self, window, sink=4):
        lib().ref_model_set_window(self.h, window, sink)

    def prefill(self, tokens, chunk=256):
        t = np.ascontiguousarray(tokens, np.uint32)
        if t.size and lib().ref_model_prefill(self.h, _p(t), t.size, chunk):
            raise RuntimeError(err())

    def forward_hidden(self, tokens, hidden_dim, update_cache=True):
        """One graph execution of the model's forward over `tokens` (use_cache = true):
        the final normed hidden states [S, hidden]; with update_cache, the step's K/V
        enter the cache as in Model::prefill."""
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty((t.size, hidden_dim), np.float16)
        if lib().ref_model_forward_hidden(self.h, _p(t), t.size, _p(out), int(update_cache)):
            raise RuntimeError(err())
        return out

    def cache(self, layer, kv_heads, head_dim):
        """(keys int8, values int8, key scales, value scales) of one layer's INT8 cache."""
        n = lib().ref_model_cache(self.h, layer, None, None, None, None)
        g = (head_dim + 127) // 128
        k = np.empty((n, kv_heads, head_dim), np.int8)
        v = np.empty_like(k)
        ks = np.empty((n, kv_heads, g), np.float32)
        vs = np.empty_like(ks)
        lib().ref_model_cache(self.h, layer, _p(k), _p(v), _p(ks), _p(vs))
        return k, v, ks, vs

    def decode_argmax(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.zeros(1, np.uint32)
        logits = np.empty(self.V, np.float16)
        if lib().ref_model_decode_greedy(self.h, _p(t), t.size, _p(out), _p(logits), self.V):
            raise RuntimeError(err())
        self.last_logits = logits
        return int(out[0])

    def generate_greedy(self, prompt, max_new, chunk=256):
        self.reset()
        prompt = list(prompt)
        if len(prompt) > 1:
            self.prefill(prompt[:-1], chunk)
        out, tok = [], prompt[-1]
        for _ in range(max_new):
            tok = self.decode_argmax([tok])
            out.append(tok)
        return out
