"""cactus_b200 — B200-native (sm_100a) backend for the Cactus quantized transformer hot path.

The compute lives in the in-tree shared library ``libcactus_b200.so`` (hand-written CUDA
kernels behind the C ABI of ``include/cactus_b200.h`` plus the C++ graph / engine / FFI
layers). This package only loads it; there is no Python or CPU fallback: ``lib()``
raises if the library is missing or was built without the CUDA kernels.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcactus_b200.so")
_lib = None


class CactusError(RuntimeError):
    pass


def lib():
    """Load libcactus_b200.so (built by ``cactus_b200.build``); raise if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CactusError(f"{LIB_PATH} is missing: run `python -m cactus_b200.build` (nvcc, sm_100a)")
        _lib = C.CDLL(LIB_PATH)
        from . import _abi
        _abi.declare(_lib)
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().cactus_cuda_last_error().decode(errors="replace")
        raise CactusError(f"{what} failed ({rc}): {msg}")
