"""cactus_cuda_sample_f16_noalloc (static scratch, no allocation) against the caller-scratch
entry cactus_cuda_sample_f16 through the C ABI: same token on two calls in a row."""
import numpy as np
import pytest

import cactus_b200 as cb
from tests.gpu_util import dev, empty, host, ptr

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("V,temp,top_p,top_k", [(5000, 0.7, 0.0, 20), (151936, 0.6, 0.95, 20), (262144, 1.0, 0.9, 40),
                                                (4096, 0.0, 0.0, 0)])
def test_noalloc_sampler_matches_scratch_entry(V, temp, top_p, top_k):
    L = cb.lib()
    rng = np.random.default_rng(V + top_k)
    work = empty((V,), np.float16)
    for call in range(2):  # two calls in a row, different logits and draws
        logits = (rng.standard_normal(V) * 3).astype(np.float16)
        hist = rng.integers(0, V, 12).astype(np.uint32)
        u = float(rng.uniform(0.01, 0.99))
        d_logits, d_hist = dev(logits), dev(hist)
        a, b = empty((1,), np.uint32), empty((1,), np.uint32)
        cb.check(L.cactus_cuda_sample_f16(ptr(d_logits), 1, V, temp, top_p, top_k, u, ptr(d_hist), len(hist),
                                          ptr(work), ptr(a), None))
        cb.check(L.cactus_cuda_sample_f16_noalloc(ptr(d_logits), 1, V, temp, top_p, top_k, u, ptr(d_hist),
                                                  len(hist), ptr(b), None))
        assert int(host(a, np.uint32)[0]) == int(host(b, np.uint32)[0]), (call, V)
    assert L.cactus_cuda_device_error(None) == 0


def test_noalloc_sampler_rejects_oversized_vocab():
    L = cb.lib()
    out = empty((1,), np.uint32)
    logits = empty((262145,), np.float16)
    rc = L.cactus_cuda_sample_f16_noalloc(ptr(logits), 1, 262145, 0.7, 0.0, 20, 0.5, None, 0, ptr(out), None)
    assert rc != 0 and b"exceeds the static scratch" in L.cactus_cuda_last_error()
