"""ctypes wrapper over oracle/_build/librefcpu.so — TEST INFRASTRUCTURE ONLY.

The CPU restatement of the Cactus reference kernels (see refcpu.h for the
reference citations). Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline / reference arm import this module; the product package never does.

All fp16 tensors are numpy float16 arrays; int8 / uint8 / float32 / uint32 as named.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "librefcpu.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile the restatement with oracle/Makefile (gcc, OpenMP)."""
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(os.path.join(_HERE, "refcpu.c")):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_SO)
        _declare(_lib)
    return _lib


P = C.c_void_p
Z = C.c_size_t
F = C.c_float
I = C.c_int


def _declare(L):
    sig = {
        "ref_set_threads": (None, [I]),
        "ref_get_threads": (I, []),
        "ref_fp16_max_abs": (F, [P, Z]),
        "ref_fp16_to_int8": (None, [P, P, Z, F]),
        "ref_quantize_activations": (None, [P, P, P, Z, Z]),
        "ref_matmul_int8": (None, [P, P, P, P, P, Z, Z, Z, Z]),
        "ref_matmul_int4": (None, [P, P, P, P, P, Z, Z, Z, Z]),
        "ref_matmul_f16": (None, [P, P, P, Z, Z, Z]),
        "ref_rms_norm_f16": (None, [P, P, P, Z, Z, F]),
        "ref_conv1d_causal_depthwise_f16": (None, [P, P, P, Z, Z, Z, Z, Z]),
        "ref_conv1d_f16_k3": (None, [P, P, P, Z, Z, Z, Z, Z]),
        "ref_layernorm_f16": (None, [P, P, P, P, Z, Z, F]),
        "ref_rope_tables": (None, [P, P, Z, Z, F]),
        "ref_rope_f16": (None, [P, P, Z, Z, Z, Z, Z, F]),
        "ref_attention_f16": (None, [P, P, P, P, Z, Z, Z, Z, Z, Z, F, Z, Z, I]),
        "ref_attention_hybrid_int8_fp16": (None, [P, P, P, P, P, P, P, P, Z, Z, Z, Z, Z, Z, Z, F, Z, I, Z]),
        "ref_quantize_kv": (None, [P, P, P, Z, Z, Z, Z]),
        "ref_fast_exp": (F, [F]),
        "ref_fast_tanh": (F, [F]),
        "ref_silu_f16": (None, [P, P, Z]),
        "ref_set_chunk_pool": (None, [I]),
        "ref_gelu_f16": (None, [P, P, Z]),
        "ref_add_f16": (None, [P, P, P, Z]),
        "ref_add_f16_clipped": (None, [P, P, P, Z]),
        "ref_multiply_f16": (None, [P, P, P, Z]),
        "ref_scalar_multiply_f16": (None, [P, P, Z, F]),
        "ref_softmax_f16": (None, [P, P, Z, Z]),
        "ref_embedding_int8": (None, [P, P, Z, Z, P, Z, Z, P]),
        "ref_embedding_f16": (None, [P, P, Z, Z, P]),
        "ref_argmax_f16": (C.c_uint32, [P, Z]),
        "ref_unpack_int4": (None, [P, P, Z]),
        "ref_quantize_weights_int8": (None, [P, P, P, Z, Z, Z]),
        "ref_quantize_weights_int4": (None, [P, P, P, Z, Z, Z]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def set_threads(n: int):
    lib().ref_set_threads(int(n))


def threads() -> int:
    return int(lib().ref_get_threads())


def quantize_activations(x):
    x = _c(x, np.float16)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty((M,), np.float32)
    lib().ref_quantize_activations(_p(x), _p(q), _p(s), M, K)
    return q, s


def matmul_int8(Aq, As, B, Bs, group_size):
    Aq, As, B, Bs = _c(Aq, np.int8), _c(As, np.float32), _c(B, np.int8), _c(Bs, np.float16)
    M, K = Aq.shape
    N = B.shape[0]
    C_ = np.empty((M, N), np.float16)
    lib().ref_matmul_int8(_p(Aq), _p(As), _p(B), _p(Bs), _p(C_), M, K, N, group_size)
    return C_


def matmul_int4(Aq, As, Bp, Bs, group_size):
    Aq, As, Bp, Bs = _c(Aq, np.int8), _c(As, np.float32), _c(Bp, np.uint8), _c(Bs, np.float16)
    M, K = Aq.shape
    N = Bp.shape[0]
    C_ = np.empty((M, N), np.float16)
    lib().ref_matmul_int4(_p(Aq), _p(As), _p(Bp), _p(Bs), _p(C_), M, K, N, group_size)
    return C_


def matmul_f16(A, Bt):
    A, Bt = _c(A, np.float16), _c(Bt, np.float16)
    M, K = A.shape
    N = Bt.shape[0]
    C_ = np.empty((M, N), np.float16)
    lib().ref_matmul_f16(_p(A), _p(Bt), _p(C_), M, K, N)
    return C_


def linear_fp16_act(x, W, Ws, group_size, int4=False):
    """compute_matmul_node with FP16 activations (graph_ops_nn.cpp:150-209)."""
    q, s = quantize_activations(x)
    return matmul_int4(q, s, W, Ws, group_size) if int4 else matmul_int8(q, s, W, Ws, group_size)


def rms_norm(x, w, eps):
    x, w = _c(x, np.float16), _c(w, np.float16)
    rows, dims = x.shape
    y = np.empty_like(x)
    lib().ref_rms_norm_f16(_p(x), _p(w), _p(y), rows, dims, eps)
    return y


def conv1d_causal_depthwise(x, w, dilation=1):
    """cactus_conv1d_causal_depthwise_f16: x [N, L, C], w [C, K] -> [N, L, C] (kernel_conv.cpp:15-110)."""
    x, w = _c(x, np.float16), _c(w, np.float16)
    N, L, C = x.shape
    y = np.empty_like(x)
    lib().ref_conv1d_causal_depthwise_f16(_p(x), _p(w), _p(y), N, L, C, w.shape[1], dilation)
    return y


def conv1d_k3(x, w, stride=1):
    """cactus_conv1d_f16_k3: x [N, C_in, L], w [C_out, C_in, 3] -> [N, C_out, (L-1)//stride + 1]
    (kernel_conv.cpp:112-227)."""
    x, w = _c(x, np.float16), _c(w, np.float16)
    N, Cin, L = x.shape
    Cout = w.shape[0]
    y = np.empty((N, Cout, (L - 1) // stride + 1), np.float16)
    lib().ref_conv1d_f16_k3(_p(x), _p(w), _p(y), N, L, Cin, Cout, stride)
    return y


def layernorm(x, w, b, eps):
    """compute_layernorm_node with fp16 tensors (graph_ops_nn.cpp:373-457): x [rows, F]."""
    x, w, b = _c(x, np.float16), _c(w, np.float16), _c(b, np.float16)
    rows, F = x.shape
    y = np.empty_like(x)
    lib().ref_layernorm_f16(_p(x), _p(w), _p(b), _p(y), rows, F, eps)
    return y


def rope_tables(n_pos, head_dim, theta):
    c = np.empty((n_pos, head_dim // 2), np.float16)
    s = np.empty((n_pos, head_dim // 2), np.float16)
    lib().ref_rope_tables(_p(c), _p(s), n_pos, head_dim, theta)
    return c, s


def rope(x, start_pos, theta):
    x = _c(x, np.float16)
    B, S, H, D = x.shape
    y = np.empty_like(x)
    lib().ref_rope_f16(_p(x), _p(y), B, S, H, D, start_pos, theta)
    return y


def attention(q, k, v, scale, position_offset=0, window_size=0, is_causal=True):
    q, k, v = _c(q, np.float16), _c(k, np.float16), _c(v, np.float16)
    B, S, Hq, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    o = np.empty_like(q)
    lib().ref_attention_f16(_p(q), _p(k), _p(v), _p(o), B, S, Skv, Hq, Hkv, D, scale,
                            position_offset, window_size, 1 if is_causal else 0)
    return o


def attention_hybrid(q, k_cache, v_cache, k_scales, v_scales, k_new, v_new, scale,
                     position_offset, is_causal=True, quant_group_size=128):
    q = _c(q, np.float16)
    B, S, Hq, D = q.shape
    k_new, v_new = _c(k_new, np.float16), _c(v_new, np.float16)
    new_len, Hkv = k_new.shape[1], k_new.shape[2]
    k_cache, v_cache = _c(k_cache, np.int8), _c(v_cache, np.int8)
    cache_len = k_cache.shape[1] if k_cache.ndim == 4 else k_cache.shape[0]
    k_scales, v_scales = _c(k_scales, np.float32), _c(v_scales, np.float32)
    o = np.zeros_like(q)
    lib().ref_attention_hybrid_int8_fp16(_p(q), _p(k_cache), _p(v_cache), _p(k_scales), _p(v_scales),
                                         _p(k_new), _p(v_new), _p(o), B, S, cache_len, new_len, Hq, Hkv, D,
                                         scale, position_offset, 1 if is_causal else 0, quant_group_size)
    return o


def quantize_kv(x, group_size=128):
    """x: [seq, kv_heads, head_dim] fp16 -> (int8 same shape, fp32 scales [seq, kv_heads, groups])."""
    x = _c(x, np.float16)
    S, H, D = x.shape
    ng = (D + group_size - 1) // group_size
    q = np.empty((S, H, D), np.int8)
    s = np.empty((S, H, ng), np.float32)
    lib().ref_quantize_kv(_p(x), _p(q), _p(s), S, H, D, group_size)
    return q, s


def _unary(fn, x):
    x = _c(x, np.float16)
    y = np.empty_like(x)
    fn(_p(x), _p(y), x.size)
    return y


def set_chunk_pool(workers: int):
    """0: SiLU / GELU take the vector formula everywhere but the tensor's own tail (the GPU's
    rule); P > 0: the reference's worker chunks on a host with P pool workers."""
    lib().ref_set_chunk_pool(int(workers))


def silu(x):
    return _unary(lib().ref_silu_f16, x)


def gelu(x):
    return _unary(lib().ref_gelu_f16, x)


def _binary(fn, a, b):
    a, b = _c(a, np.float16), _c(b, np.float16)
    assert a.shape == b.shape
    y = np.empty_like(a)
    fn(_p(a), _p(b), _p(y), a.size)
    return y


def add(a, b):
    return _binary(lib().ref_add_f16, a, b)


def add_clipped(a, b):
    return _binary(lib().ref_add_f16_clipped, a, b)


def multiply(a, b):
    return _binary(lib().ref_multiply_f16, a, b)


def scalar_multiply(x, s):
    x = _c(x, np.float16)
    y = np.empty_like(x)
    lib().ref_scalar_multiply_f16(_p(x), _p(y), x.size, s)
    return y


def softmax(x):
    x = _c(x, np.float16)
    V = x.shape[-1]
    rows = x.size // V
    y = np.empty_like(x)
    lib().ref_softmax_f16(_p(x), _p(y), rows, V)
    return y


def embedding_int8(table, scales, group_size, ids):
    table, scales = _c(table, np.int8), _c(scales, np.float16)
    ids = _c(ids, np.uint32)
    V, H = table.shape
    out = np.empty((ids.size, H), np.float16)
    lib().ref_embedding_int8(_p(table), _p(scales), group_size, scales.shape[1], _p(ids), ids.size, H, _p(out))
    return out


def embedding_f16(table, ids):
    table = _c(table, np.float16)
    ids = _c(ids, np.uint32)
    out = np.empty((ids.size, table.shape[1]), np.float16)
    lib().ref_embedding_f16(_p(table), _p(ids), ids.size, table.shape[1], _p(out))
    return out


def argmax(logits):
    logits = _c(logits, np.float16).reshape(-1)
    return int(lib().ref_argmax_f16(_p(logits), logits.size))


def unpack_int4(packed, count):
    packed = _c(packed, np.uint8)
    out = np.empty((count,), np.int8)
    lib().ref_unpack_int4(_p(packed), _p(out), count)
    return out


def quantize_weights_int8(w, group_size):
    w = _c(w, np.float32)
    N, K = w.shape
    q = np.empty((N, K), np.int8)
    s = np.empty((N, K // group_size), np.float16)
    lib().ref_quantize_weights_int8(_p(w), _p(q), _p(s), N, K, group_size)
    return q, s


def quantize_weights_int4(w, group_size):
    w = _c(w, np.float32)
    N, K = w.shape
    p = np.empty((N, K // 2), np.uint8)
    s = np.empty((N, K // group_size), np.float16)
    lib().ref_quantize_weights_int4(_p(w), _p(p), _p(s), N, K, group_size)
    return p, s
