"""The C-ABI library loads on a CPU-only host and exports every symbol include/*.h declares."""
import os
import re

import cactus_b200 as cb
from cactus_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_declared_symbol():
    L = cb.lib()
    sigs = _abi.declared()
    assert len(sigs) >= 25
    missing = [n for n in sigs if not hasattr(L, n)]
    assert missing == [], missing


def test_headers_parse_completely():
    # every declaration line with an export macro is picked up by the binding parser
    for h in _abi.HEADERS:
        p = os.path.join(ROOT, "include", h)
        if not os.path.exists(p):
            continue
        text = re.sub(r"/\*.*?\*/", "", open(p).read(), flags=re.S)
        n_decl = len(re.findall(r"\b(CB_API|CACTUS_FFI_EXPORT)\s+[\w\s\*]+?\b\w+\s*\(", text))
        parsed = sum(len(_abi.parse(open(p).read(), m)) for m in ("CB_API", "CACTUS_FFI_EXPORT"))
        assert parsed == n_decl, h


def test_error_reporting_without_gpu():
    L = cb.lib()
    # argument validation happens before any CUDA call
    rc = L.cactus_cuda_linear_int8(None, None, None, None, 1, 96, 16, 24, None)
    assert rc == -1
    assert b"multiple" in L.cactus_cuda_last_error()
    assert L.cactus_cuda_version() >= 1
