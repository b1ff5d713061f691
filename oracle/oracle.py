"""ctypes wrapper of the CPU oracle (liboracle.so, built from zn_oracle.c).

TEST INFRASTRUCTURE ONLY: the cuzipnn_b200 package never imports this module.  The tests, the
smoke check and the benchmark's CPU baseline use it as the checker for the CUDA library.  Every
function restates part of the reference (ruihe774/cuZipNN); the C source cites the file:line of
each piece.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

# src/cuzipnn/_codec.py:47-64: dtype code -> (torch dtype name, element size).
DTYPE_CODES = {
    1: ("bool", 1),
    2: ("uint8", 1),
    3: ("int8", 1),
    4: ("int16", 2),
    5: ("int32", 4),
    6: ("int64", 8),
    7: ("float16", 2),
    8: ("bfloat16", 2),
    9: ("float32", 4),
    10: ("float64", 8),
    11: ("float8_e4m3fn", 1),
    12: ("float8_e5m2", 1),
    13: ("uint16", 2),
    14: ("uint32", 4),
    15: ("uint64", 8),
    16: ("complex64", 8),
}
CODE_OF = {name: code for code, (name, _) in DTYPE_CODES.items()}
# src/cuzipnn/_codec.py:66-67: only bfloat16 and float32 get the exponent bit reordering.
REORDER = {"bfloat16", "float32"}
BLOB_VERSION = 3

_i64p = ctypes.POINTER(ctypes.c_int64)
_u8p = ctypes.c_void_p


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_split.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _u8p, ctypes.c_int64]
        L.orc_merge.argtypes = [_u8p, _u8p, _u8p, ctypes.c_int64, ctypes.c_int, ctypes.c_int64, ctypes.c_int]
        L.orc_copy_chunks.argtypes = [_u8p, _u8p, _u8p, _u8p, _u8p, ctypes.c_int64, ctypes.c_int]
        L.orc_crc32.argtypes = [ctypes.c_uint32, _u8p, ctypes.c_int64]
        L.orc_crc32.restype = ctypes.c_uint32
        L.orc_crc32_segments.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _u8p]
        L.orc_sub_chunks.argtypes = [ctypes.c_int64, ctypes.c_int64]
        L.orc_sub_chunks.restype = ctypes.c_int
        L.orc_normalize.argtypes = [_u8p, ctypes.c_int64, _u8p]
        L.orc_ans_max_payload.argtypes = [ctypes.c_int64, ctypes.c_int]
        L.orc_ans_max_payload.restype = ctypes.c_int64
        L.orc_ans_encode.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int, _u8p, ctypes.c_int64]
        L.orc_ans_encode.restype = ctypes.c_int64
        L.orc_ans_decode.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _u8p]
        L.orc_ans_decode.restype = ctypes.c_int
        L.orc_blob_bound.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64]
        L.orc_blob_bound.restype = ctypes.c_int64
        L.orc_compress.argtypes = [
            _u8p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u8p,
            ctypes.c_int64, ctypes.c_int, ctypes.c_double, ctypes.c_int64, ctypes.c_int, _u8p,
            ctypes.c_int64, ctypes.c_int,
        ]
        L.orc_compress.restype = ctypes.c_int64
        L.orc_decompress.argtypes = [_u8p, ctypes.c_int64, _u8p, ctypes.c_int64, ctypes.c_int, ctypes.c_int]
        L.orc_decompress.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _u8(data) -> np.ndarray:
    """Contiguous uint8 view of bytes, a numpy array or a CPU torch tensor."""
    if isinstance(data, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(data), dtype=np.uint8)
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    t = data.detach().cpu().contiguous()  # a torch tensor
    return t.reshape(-1).view(_torch_uint8()).numpy()


def _torch_uint8():
    import torch

    return torch.uint8


def split(x_bytes, n: int, k: int, reorder: bool, stride: int) -> np.ndarray:
    """Planes of n k-byte elements: planar[b * stride + e] (src/cuzipnn/_kernels.py:34-54)."""
    x = _u8(x_bytes)
    planar = np.zeros(k * stride, dtype=np.uint8)
    lib().orc_split(_ptr(x), n, k, int(reorder), _ptr(planar), stride)
    return planar


def merge(src_tbl, base, n: int, k: int, chunk_bytes: int, reorder: bool) -> np.ndarray:
    """Inverse of split through an offset table (src/cuzipnn/_kernels.py:57-105)."""
    tbl = np.ascontiguousarray(src_tbl, dtype=np.int64)
    b = _u8(base)
    out = np.zeros(n * k, dtype=np.uint8)
    lib().orc_merge(_ptr(tbl), _ptr(b), _ptr(out), n, k, chunk_bytes, int(reorder))
    return out


def crc32(data, crc: int = 0) -> int:
    d = _u8(data)
    return int(lib().orc_crc32(crc, _ptr(d), d.size))


def crc32_segments(data, seg: int) -> np.ndarray:
    d = _u8(data)
    m = -(-d.size // seg)
    out = np.zeros(m, dtype=np.uint32)
    if m:
        lib().orc_crc32_segments(_ptr(d), d.size, seg, _ptr(out))
    return out


def sub_chunks(chunk_bytes: int, sub_chunk_bytes: int) -> int:
    return int(lib().orc_sub_chunks(chunk_bytes, sub_chunk_bytes))


def normalize(counts, m: int) -> np.ndarray:
    c = np.ascontiguousarray(counts, dtype=np.uint32)
    f = np.zeros(256, dtype=np.uint32)
    lib().orc_normalize(_ptr(c), m, _ptr(f))
    return f


def ans_encode(symbols, n_sub: int) -> bytes:
    s = _u8(symbols)
    cap = int(lib().orc_ans_max_payload(s.size, n_sub))
    out = np.zeros(cap, dtype=np.uint8)
    size = int(lib().orc_ans_encode(_ptr(s), s.size, n_sub, _ptr(out), cap))
    if size < 0:
        raise RuntimeError(f"oracle ANS encode failed ({size})")
    return out[:size].tobytes()


def ans_max_payload(m: int, n_sub: int) -> int:
    return int(lib().orc_ans_max_payload(m, n_sub))


def ans_decode(payload, m: int) -> np.ndarray:
    p = _u8(payload)
    out = np.zeros(m, dtype=np.uint8)
    rc = int(lib().orc_ans_decode(_ptr(p), p.size, m, _ptr(out)))
    if rc != 0:
        raise ValueError(f"oracle ANS decode failed ({rc})")
    return out


def compress(
    x_bytes,
    shape,
    dtype_name: str,
    *,
    chunk_bytes: int = 131072,
    sub_chunk_bytes: int = 8192,
    passthrough_threshold: float = 0.95,
    min_compress_bytes: int = 65536,
    version: int = BLOB_VERSION,
    threads: int = 0,
) -> bytes:
    """Blob bytes for a tensor given as raw row-major bytes (src/cuzipnn/_codec.py:231-413)."""
    code = CODE_OF[dtype_name]
    k = DTYPE_CODES[code][1]
    x = _u8(x_bytes)
    n = x.size // k
    shape = tuple(int(s) for s in shape)
    shp = np.array(shape if shape else [0], dtype=np.int64)
    cap = int(lib().orc_blob_bound(n, k, len(shape), chunk_bytes))
    out = np.zeros(cap, dtype=np.uint8)
    n_sub = sub_chunks(chunk_bytes, sub_chunk_bytes)
    size = int(
        lib().orc_compress(
            _ptr(x), n, k, code, int(dtype_name in REORDER), len(shape), _ptr(shp), chunk_bytes,
            n_sub, float(passthrough_threshold), min_compress_bytes, version, _ptr(out), cap, threads,
        )
    )
    if size < 0:
        raise RuntimeError(f"oracle compress failed ({size})")
    return out[:size].tobytes()


def parse_header(blob: bytes):
    """(dtype name, shape, flags, chunk_bytes, n_comp, numel, version) of a blob
    (src/cuzipnn/_codec.py:416-428)."""
    import struct

    magic, version, code, ndim, flags, chunk_bytes, n_comp, n = struct.unpack_from("<4sBBBBIIQ", blob)
    if magic != b"ZNNG" or code not in DTYPE_CODES:
        raise ValueError("not a cuzipnn blob")
    shape = struct.unpack_from(f"<{ndim}q", blob, 24)
    return DTYPE_CODES[code][0], shape, flags, chunk_bytes, n_comp, n, version


def decompress(blob, *, version: int = BLOB_VERSION, threads: int = 0) -> np.ndarray:
    """Raw row-major bytes of the tensor in a blob (src/cuzipnn/_codec.py:431-542)."""
    b = _u8(blob)
    name, shape, _, _, _, n, _ = parse_header(b.tobytes()[: 24 + 8 * 64])
    k = DTYPE_CODES[CODE_OF[name]][1]
    out = np.zeros(n * k, dtype=np.uint8)
    rc = int(lib().orc_decompress(_ptr(b), b.size, _ptr(out), out.size, version, threads))
    if rc != 0:
        raise ValueError(f"oracle decompress failed ({rc})")
    return out
