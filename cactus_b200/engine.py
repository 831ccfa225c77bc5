"""Python handle over the engine C ABI (include/cactus_b200_engine.h).

Thin ctypes plumbing for tests and the benchmark: arrays cross as HOST numpy buffers,
exactly as a C caller of the reference's engine would pass them.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import CactusError, lib


class Engine:
    def __init__(self, model_folder: str, context_size: int = 512, max_batch: int = 1, device: int = 0):
        L = lib()
        self._L = L
        self.h = L.cactus_engine_create(model_folder.encode(), context_size, max_batch, device)
        if not self.h:
            raise CactusError("cactus_engine_create failed: " + L.cactus_engine_last_error().decode())
        info = np.zeros(8, np.uint32)
        self._check(L.cactus_engine_info(self.h, info.ctypes.data_as(C.c_void_p)), "info")
        (self.vocab, self.num_layers, self.hidden, self.heads, self.kv_heads, self.head_dim, self.ffn,
         self.model_type) = (int(v) for v in info)

    def _check(self, rc, what):
        if rc != 0:
            raise CactusError(f"{what} failed ({rc}): {self._L.cactus_engine_last_error().decode()}")

    def close(self):
        if self.h:
            self._L.cactus_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        self._check(self._L.cactus_engine_reset(self.h), "reset")

    def set_cache_window(self, window: int, sink: int = 4):
        self._check(self._L.cactus_engine_set_cache_window(self.h, window, sink), "set_cache_window")

    def set_causal_fix(self, on: bool = True):
        """Causal-correct masking of prefill chunks after the window slid (off = reference)."""
        self._check(self._L.cactus_engine_set_causal_fix(self.h, 1 if on else 0), "set_causal_fix")

    def prefill(self, tokens, chunk_size: int = 256):
        t = np.ascontiguousarray(tokens, np.uint32)
        self._check(self._L.cactus_engine_prefill(self.h, t.ctypes.data_as(C.c_void_p), t.size, chunk_size), "prefill")

    def decode(self, tokens, temperature=0.0, top_p=0.0, top_k=0):
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.zeros(1, np.uint32)
        ent = np.zeros(1, np.float32)
        self._check(self._L.cactus_engine_decode(self.h, t.ctypes.data_as(C.c_void_p), t.size, temperature, top_p,
                                                 top_k, out.ctypes.data_as(C.c_void_p),
                                                 ent.ctypes.data_as(C.c_void_p)), "decode")
        return int(out[0])

    def generate_greedy(self, prompt, max_new: int):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max_new, np.uint32)
        self._check(self._L.cactus_engine_generate_greedy(self.h, p.ctypes.data_as(C.c_void_p), p.size, max_new,
                                                          out.ctypes.data_as(C.c_void_p)), "generate")
        return out

    def generate_batch_greedy(self, prompts, max_new: int):
        p = np.ascontiguousarray(prompts, np.uint32)
        B, P = p.shape
        out = np.zeros((B, max_new), np.uint32)
        self._check(self._L.cactus_engine_generate_batch_greedy(self.h, p.ctypes.data_as(C.c_void_p), B, P, max_new,
                                                                out.ctypes.data_as(C.c_void_p)), "generate_batch")
        return out

    def last_logits(self):
        out = np.zeros(self.vocab, np.float16)
        self._check(self._L.cactus_engine_last_logits(self.h, out.ctypes.data_as(C.c_void_p), self.vocab), "logits")
        return out

    def decode_path(self, mode: int = 0) -> int:
        """Decode path of the last generate (0 host loop, 1 CUDA graph, 2 persistent step);
        mode -1 re-enables the persistent step, 1 disables it for later calls."""
        return int(self._L.cactus_engine_decode_path(self.h, mode))

    def stats(self):
        out = np.zeros(8, np.float64)
        self._check(self._L.cactus_engine_stats(self.h, out.ctypes.data_as(C.c_void_p)), "stats")
        keys = ("prefill_ms", "decode_ms", "launches", "graph_replays", "graph_nodes", "weight_bytes",
                "kv_capacity", "kv_window")
        return dict(zip(keys, out.tolist()))

    def kv_state(self):
        out = np.zeros(2, np.uint64)
        self._check(self._L.cactus_engine_kv_state(self.h, out.ctypes.data_as(C.c_void_p)), "kv_state")
        return int(out[0]), int(out[1])

    def read_kv(self, layer: int):
        n, _ = self.kv_state()
        ng = (self.head_dim + 127) // 128
        k = np.zeros((n, self.kv_heads, self.head_dim), np.int8)
        v = np.zeros_like(k)
        ks = np.zeros((n, self.kv_heads, ng), np.float32)
        vs = np.zeros_like(ks)
        self._check(self._L.cactus_engine_read_kv(self.h, layer, k.ctypes.data_as(C.c_void_p),
                                                  v.ctypes.data_as(C.c_void_p), ks.ctypes.data_as(C.c_void_p),
                                                  vs.ctypes.data_as(C.c_void_p)), "read_kv")
        return k, v, ks, vs
