"""ctypes signatures for the C ABI, read from the public headers in ``include/``.

Parsing the headers keeps the Python binding and the C declarations from drifting;
tests/test_abi.py checks that every declared symbol is exported by the library.
"""
from __future__ import annotations

import ctypes as C
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = ("cactus_b200.h", "cactus_b200_engine.h", "cactus_ffi.h")

_SCALAR = {
    "int": C.c_int,
    "unsigned": C.c_uint,
    "uint32_t": C.c_uint32,
    "uint64_t": C.c_uint64,
    "size_t": C.c_size_t,
    "float": C.c_float,
    "double": C.c_double,
    "bool": C.c_bool,
    "void": None,
    "cactus_model_t": C.c_void_p,
    "cactus_engine_t": C.c_void_p,
    "cactus_token_callback": C.c_void_p,
}


def _ctype(t: str):
    t = t.replace("const", "").strip()
    if t.endswith("*"):
        base = t[:-1].strip()
        return C.c_char_p if base == "char" else C.c_void_p
    return _SCALAR[t]


def parse(header_text: str, macro: str):
    text = re.sub(r"/\*.*?\*/", "", header_text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for ret, name, args in re.findall(macro + r"\s+([\w\s\*]+?)\s*\b(\w+)\s*\(([^)]*)\)\s*;", text):
        argl = [a.strip() for a in args.split(",") if a.strip() and a.strip() != "void"]
        types = [_ctype(re.sub(r"\b\w+$", "", a).strip() if not a.strip().endswith("*") else a) for a in argl]
        out[name] = (_ctype(ret), types)
    return out


def declared():
    sigs = {}
    for h in HEADERS:
        path = os.path.join(ROOT, "include", h)
        if not os.path.exists(path):
            continue
        text = open(path).read()
        for macro in ("CB_API", "CACTUS_FFI_EXPORT"):
            sigs.update(parse(text, macro))
    return sigs


def declare(lib) -> None:
    for name, (res, args) in declared().items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue  # tests/test_abi.py reports missing exports
        fn.restype = res
        fn.argtypes = args
