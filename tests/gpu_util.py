"""Device-memory plumbing for the GPU parity tests: numpy <-> torch CUDA tensors.

torch is used only to allocate device memory and copy bytes; every computation under
test runs through the C ABI of libcactus_b200.so.
"""
import numpy as np

_NP2T = {}


def torch():
    import torch as _t
    return _t


def dev(a: np.ndarray):
    """Copy a numpy array to a fresh CUDA tensor (bytes preserved)."""
    t = torch()
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return t.from_numpy(a.view(np.int16).copy()).cuda()
    if a.dtype == np.uint32:
        return t.from_numpy(a.view(np.int32).copy()).cuda()
    if a.dtype == np.uint16:
        return t.from_numpy(a.view(np.int16).copy()).cuda()
    return t.from_numpy(a.copy()).cuda()


def empty(shape, dtype):
    t = torch()
    tdt = {np.float16: t.int16, np.int8: t.int8, np.uint8: t.uint8, np.float32: t.float32,
           np.uint32: t.int32, np.int32: t.int32}[np.dtype(dtype).type]
    return t.zeros(shape, dtype=tdt, device="cuda")


def host(x, dtype):
    """Copy a CUDA tensor back as a numpy array of `dtype` (bytes preserved)."""
    torch().cuda.synchronize()
    a = x.cpu().numpy()
    return a.view(dtype)


_KEEP = []


def ptr(x):
    """Device address of a tensor. The tensor is kept alive until release() so that a
    temporary (e.g. ``ptr(dev(a))``) cannot be recycled by the caching allocator while a
    kernel that reads it is still queued."""
    _KEEP.append(x)
    return x.data_ptr()


def release():
    torch().cuda.synchronize()
    _KEEP.clear()


def rel_err(got, ref):
    """Normwise max relative error max|d| / max|ref| (the parity metric for fp outputs)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0))
