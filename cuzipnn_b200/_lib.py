"""ctypes binding of libcuzipnn_b200.so (the C ABI in include/cuzipnn_b200.h).

The library is the only implementation of the codec: if it is missing or fails to load, importing
this module raises.  There is no CPU or Triton fallback.
"""

from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libcuzipnn_b200.so")

ZN_OK = 0
ZN_ERR_INVALID = -1
ZN_ERR_CUDA = -2
ZN_ERR_SPACE = -3
ABI_VERSION = 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_sz = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "zn_version": (_i32, []),
    "zn_last_error": (ctypes.c_char_p, []),
    "zn_launch_count": (ctypes.c_uint64, []),
    "zn_timing_enable": (_i32, [ctypes.c_char_p, _i32]),
    "zn_timing_read": (_i32, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "zn_split": (_i32, [_p, _i64, _i32, _i32, _p, _i64, _p]),
    "zn_merge": (_i32, [_p, _p, _p, _i64, _i32, _i64, _i32, _p]),
    "zn_copy_chunks": (_i32, [_p, _p, _p, _i64, _i64, _i32, _p]),
    "zn_ans_max_compressed_chunk_bytes": (_i64, [_i64, _i32]),
    "zn_ans_compress_temp_bytes": (_sz, [_i64, _i64, _i32]),
    "zn_ans_compress": (_i32, [_p, _p, _i64, _i64, _p, _p, _p, _i32, _p, _sz, _p]),
    "zn_ans_decompress_temp_bytes": (_sz, [_i64]),
    "zn_ans_decompress": (_i32, [_p, _p, _p, _i64, _p, _p, _p, _sz, _p]),
    "zn_crc32_temp_bytes": (_sz, [_i64, _i64]),
    "zn_crc32": (_i32, [_p, _i64, _i64, _p, _p, _sz, _p]),
    "zn_crc32_noalloc": (_i32, [_p, _i64, _i64, _p, _p]),
    "zn_compress_bound": (_i64, [_i64, _i32, _i32, _i64]),
    "zn_compress_temp_bytes": (_sz, [_i64, _i32, _i64, _i32]),
    "zn_compress": (_i32, [_p, _i64, _i32, _i32, _p, _i32, _i64, _i32, ctypes.c_double, _p, _i64, _p, _p, _sz, _p]),
    "zn_decompress_temp_bytes": (_sz, [_i64, _i32, _i64]),
    "zn_compress_batch_temp_bytes": (_sz, [_i32, _p, _i32, _i64, _i32]),
    "zn_compress_batch": (_i32, [_i32, _p, _p, _i32, _i32, _p, _p, _i64, _i32, ctypes.c_double, _p, _p, _p, _p, _sz, _p]),
    "zn_decompress_batch_temp_bytes": (_sz, [_i32, _p, _i32, _p]),
    "zn_decompress_batch": (_i32, [_i32, _p, _p, _p, _i32, _i32, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "zn_decompress": (_i32, [_p, _i64, _i64, _i32, _i32, _i32, _i64, _i64, _p, _p, _p, _sz, _p]),
}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python cuzipnn_b200/_build.py` "
            "(or __graft_entry__.build()); the codec has no fallback"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.zn_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH} has ABI {lib.zn_version()}, expected {ABI_VERSION}")
    return lib


lib = _load()


def check(status: int, what: str) -> None:
    """Map a nonzero status of the C ABI to an exception (as _nvcomp._check does for nvCOMP)."""
    if status == ZN_OK:
        return
    msg = lib.zn_last_error().decode(errors="replace")
    if status == ZN_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed with status {status}: {msg}")


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(lib.zn_launch_count())


KERNELS = ("hist", "encode", "scan", "pack", "dscan", "decode", "decode_overflow", "crc")


class KernelTimer:
    """CUDA-event timing of the library's kernel launches (zn_timing_enable), e.g.
    `with KernelTimer() as kt: ...` then kt.times[name] = (total_ms, launches)."""

    def __init__(self, kernel: str = "*"):
        self.kernel = kernel
        self.times: dict[str, tuple[float, int]] = {}

    def __enter__(self):
        lib.zn_timing_read(None, None, None)  # drop stale records
        lib.zn_timing_enable(self.kernel.encode(), 1)
        return self

    def __exit__(self, *exc):
        lib.zn_timing_enable(None, 0)
        for name in KERNELS:
            ms = ctypes.c_double()
            n = ctypes.c_int64()
            check(lib.zn_timing_read(name.encode(), ctypes.byref(ms), ctypes.byref(n)), "zn_timing_read")
            if n.value:
                self.times[name] = (ms.value, n.value)
        lib.zn_timing_read(None, None, None)
        return False
