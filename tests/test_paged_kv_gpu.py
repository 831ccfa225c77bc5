"""The engine on the paged KV cache (CACTUS_B200_KV_PAGE = tokens per page): every engine
parity test (sliding window with sinks, chunked prefill, long caches through the key-split
attention in decode graphs, batched sequences, the persistent decode step, the causal-fix
mode) and the full-shape Llama-3.2-1B batch (config 4) re-run in a child process whose
engines keep their caches in pages handed out through block tables. Pages are given out
from the end of the pool, so no sequence's pages are physically in order."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _child(page, files, select):
    env = dict(os.environ, CACTUS_B200_KV_PAGE=str(page))
    r = subprocess.run([sys.executable, "-m", "pytest", *[os.path.join(HERE, f) for f in files], "-q", "-m", "gpu",
                        "-p", "no:cacheprovider", "-k", select],
                       env=env, capture_output=True, text=True, timeout=1200, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("page", [16, 64])
def test_engine_parity_on_paged_cache(page):
    _child(page, ["test_engine_gpu.py"], "not qwen3_0_6b")


@pytest.mark.skipif(os.environ.get("CACTUS_SKIP_FULL") == "1", reason="full-size models disabled")
def test_config4_batch_on_paged_cache():
    _child(64, ["test_full_shapes_gpu.py"], "config4")
