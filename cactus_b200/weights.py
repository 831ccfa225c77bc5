"""The Cactus ``.weights`` tensor file format and its group quantizer (converter side).

Format (reader: cactus/graph/graph_io.cpp:497-566, writer: python/src/tensor_io.py:163-321):
80-byte little-endian header — magic ``CACT``, u32 version=1, u32 flags (bit0 has
scales, bit2 transposed), u32 alignment=32, u32 ndim, 4 x u64 dims, u32 precision
(0 INT8, 1 FP16, 2 FP32, 3 INT4), u64 data_bytes, u64 scales_bytes, u32 group_size,
u32 num_groups — padded to the alignment, then fp16 scales ``[N, num_groups]``,
padding, then the data (int8 row-major ``[N, K]``; INT4 as ``[N, K/2]`` bytes with
the even k in the low nibble; FP16 row-major).

The quantizer follows tensor_io.py:82-282 on float32 input: per row and per group of
G along K, ``scale = float32(absmax / 127)`` (``/ 7`` for INT4) floored at 1e-10,
``q = clip(round_half_even(w / scale))``, scales stored as fp16. The writer and the
quantizer are bit-exact against fixtures produced by the reference's own
``save_tensor_with_header`` (tests/golden).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"CACT"
VERSION = 1
ALIGNMENT = 32
HEADER_SIZE = 80
FLAG_HAS_SCALES = 1 << 0
FLAG_TRANSPOSED = 1 << 2
PREC_INT8, PREC_FP16, PREC_FP32, PREC_INT4 = 0, 1, 2, 3
_PREC_NAMES = {PREC_INT8: "INT8", PREC_FP16: "FP16", PREC_FP32: "FP32", PREC_INT4: "INT4"}


def _align(off: int, a: int) -> int:
    r = off % a
    return off if r == 0 else off + (a - r)


@dataclass
class WeightsFile:
    shape: tuple
    precision: str  # "INT8" | "INT4" | "FP16" | "FP32"
    group_size: int
    num_groups: int
    data: np.ndarray  # int8 [N,K] | uint8 packed [N,K/2] | float16 | float32
    scales: np.ndarray | None  # float16 [N, num_groups]
    flags: int = 0


def quantize_int8(w: np.ndarray, group_size: int):
    """Symmetric per-group INT8 (tensor_io.py:82-106). Returns (int8 [N,K], fp16 scales [N,K/G])."""
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    if K % group_size:
        raise ValueError("K must be a multiple of the group size")
    g = w.reshape(N, K // group_size, group_size)
    scales = (np.max(np.abs(g), axis=2) / np.float32(127.0)).astype(np.float32)
    scales = np.maximum(scales, np.float32(1e-10))
    q = np.clip(np.round(g / scales[:, :, None]), -128, 127).astype(np.int8)
    return q.reshape(N, K), scales.astype(np.float16)


def quantize_int4(w: np.ndarray, group_size: int):
    """Symmetric per-group INT4 packed two per byte, low nibble = even k (tensor_io.py:199-230)."""
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    if K % group_size or K % 2:
        raise ValueError("K must be even and a multiple of the group size")
    g = w.reshape(N, K // group_size, group_size)
    scales = (np.max(np.abs(g), axis=2) / np.float32(7.0)).astype(np.float32)
    scales = np.maximum(scales, np.float32(1e-10))
    q = np.clip(np.round(g / scales[:, :, None]), -8, 7).astype(np.int8).reshape(N, K)
    packed = ((q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)).astype(np.uint8)
    return packed, scales.astype(np.float16)


def _header(shape, prec, data_bytes, scales_bytes, group_size, num_groups, flags) -> bytes:
    h = bytearray()
    h += MAGIC
    h += struct.pack("<IIII", VERSION, flags, ALIGNMENT, len(shape))
    for i in range(4):
        h += struct.pack("<Q", shape[i] if i < len(shape) else 0)
    h += struct.pack("<I", prec)
    h += struct.pack("<QQ", data_bytes, scales_bytes)
    h += struct.pack("<II", group_size, num_groups)
    assert len(h) == HEADER_SIZE
    h += b"\x00" * (_align(HEADER_SIZE, ALIGNMENT) - HEADER_SIZE)
    return bytes(h)


def write_quantized(path, data: np.ndarray, scales: np.ndarray | None, shape, precision: str,
                    group_size: int = 0, transposed: bool = False):
    """Write already-quantized data in the .weights layout."""
    path = Path(path)
    flags = FLAG_TRANSPOSED if transposed else 0
    with open(path, "wb") as f:
        if precision in ("INT8", "INT4"):
            flags |= FLAG_HAS_SCALES
            sb = scales.astype(np.float16).tobytes()
            prec = PREC_INT8 if precision == "INT8" else PREC_INT4
            f.write(_header(shape, prec, data.nbytes, len(sb), group_size, scales.shape[-1], flags))
            f.write(sb)
            end = _align(HEADER_SIZE, ALIGNMENT) + len(sb)
            f.write(b"\x00" * (_align(end, ALIGNMENT) - end))
            f.write(np.ascontiguousarray(data).tobytes())
        elif precision == "FP16":
            d = np.ascontiguousarray(data, dtype=np.float16)
            f.write(_header(shape, PREC_FP16, d.nbytes, 0, 0, 0, flags))
            f.write(d.tobytes())
        else:
            raise ValueError(f"unsupported precision {precision}")


def save_tensor(path, w: np.ndarray, precision: str, group_size: int = 128, gemma_norm: bool = False):
    """Quantize and write a float32 tensor (save_tensor_with_header, tensor_io.py:40-321).

    Names containing ``norm``/``bias``/``vision`` are forced to FP16 as in the reference
    (tensor_io.py:71-74); Gemma norms get +1 (tensor_io.py:62-64) when ``gemma_norm``.
    """
    path = Path(path)
    w = np.asarray(w, dtype=np.float32)
    if gemma_norm and "norm" in path.name:
        w = w + np.float32(1.0)
    if precision in ("INT8", "INT4") and any(x in path.name for x in ("norm", "bias", "vision")):
        precision = "FP16"
    shape = list(w.shape)
    if precision in ("INT8", "INT4") and w.ndim in (1, 2):
        w2 = w.reshape(1, -1) if w.ndim == 1 else w
        if precision == "INT8":
            q, s = quantize_int8(w2, group_size)
        else:
            q, s = quantize_int4(w2, group_size)
        write_quantized(path, q, s, shape, precision, group_size)
    else:
        write_quantized(path, w.astype(np.float16), None, shape, "FP16")


def read_weights(path) -> WeightsFile:
    """Parse a .weights file (graph_io.cpp:497-566)."""
    buf = Path(path).read_bytes()
    if len(buf) < HEADER_SIZE:
        raise ValueError("File too small: insufficient data for header")
    if buf[:4] != MAGIC:
        raise ValueError("Invalid tensor file: missing CACT magic number")
    version, flags, alignment, ndim = struct.unpack_from("<IIII", buf, 4)
    dims = struct.unpack_from("<QQQQ", buf, 20)
    prec, = struct.unpack_from("<I", buf, 52)
    data_bytes, scales_bytes = struct.unpack_from("<QQ", buf, 56)
    group_size, num_groups = struct.unpack_from("<II", buf, 72)
    alignment = alignment or 1
    shape = tuple(int(d) for i, d in enumerate(dims) if i < ndim and d > 0)
    hdr = _align(HEADER_SIZE, alignment)
    if scales_bytes:
        s_off = hdr
        d_off = _align(s_off + scales_bytes, alignment)
    else:
        s_off, d_off = 0, hdr
    if d_off + data_bytes > len(buf):
        raise ValueError("File corrupted: data extends beyond file size")
    scales = None
    if scales_bytes:
        scales = np.frombuffer(buf, np.float16, scales_bytes // 2, s_off).reshape(-1, num_groups)
    raw = np.frombuffer(buf, np.uint8, data_bytes, d_off)
    name = _PREC_NAMES.get(prec)
    if name is None:
        raise ValueError(f"unknown precision {prec}")
    if name == "INT8":
        data = raw.view(np.int8).reshape(shape)
    elif name == "INT4":
        data = raw.reshape(shape[0] if len(shape) == 2 else 1, -1)
    elif name == "FP16":
        data = raw.view(np.float16).reshape(shape)
    else:
        data = raw.view(np.float32).reshape(shape)
    return WeightsFile(shape, name, group_size, num_groups, data, scales, flags)
