"""Batched entropy coder with the interface of the reference's nvCOMP bindings
(src/cuzipnn/_nvcomp.py:170-257), backed by the ZNR2 rANS kernels of libcuzipnn_b200.so.

Same names, argument meaning and errors (a failed call raises RuntimeError); the payloads are
ZNR2, not nvCOMP ANS.  The whole-tensor codec does not go through this module.
"""

import torch

from . import _lib

NVCOMP_SUCCESS = 0
MAX_CHUNK_BYTES = 1 << 24
DECOMPRESS_INPUT_ALIGNMENT = 8
MIN_SUB_CHUNKS = 4
MAX_SUB_CHUNKS = 64


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def max_compressed_chunk_bytes(chunk_bytes: int, sub_chunks: int) -> int:
    out = int(_lib.lib.zn_ans_max_compressed_chunk_bytes(chunk_bytes, sub_chunks))
    if out < 0:
        raise RuntimeError(f"max_compressed_chunk_bytes failed for ({chunk_bytes}, {sub_chunks})")
    return out


def compress(in_ptrs, in_bytes, chunk_bytes, total_bytes, out_ptrs, out_bytes, statuses, sub_chunks) -> None:
    """Asynchronously rANS-compress a batch of chunks on the current stream (_nvcomp.py:179-218).
    in_ptrs/out_ptrs are int64 device addresses, in_bytes/out_bytes int64, statuses int32."""
    n = in_ptrs.numel()
    tb = int(_lib.lib.zn_ans_compress_temp_bytes(n, chunk_bytes, sub_chunks))
    temp = torch.empty(max(tb, 1), dtype=torch.uint8, device=in_ptrs.device)
    _lib.check(
        _lib.lib.zn_ans_compress(in_ptrs.data_ptr(), in_bytes.data_ptr(), chunk_bytes, n, out_ptrs.data_ptr(),
                                 out_bytes.data_ptr(), statuses.data_ptr(), sub_chunks, temp.data_ptr(), tb,
                                 _stream(in_ptrs)),
        "zn_ans_compress",
    )


def decompress(in_ptrs, in_bytes, out_capacity, chunk_bytes, total_bytes, out_ptrs) -> torch.Tensor:
    """Asynchronously decompress a batch of rANS chunks on the current stream (_nvcomp.py:221-257).
    Returns the int32 per-chunk statuses (the reference allocates them but never reads them)."""
    n = in_ptrs.numel()
    statuses = torch.empty(n, dtype=torch.int32, device=in_ptrs.device)
    tb = int(_lib.lib.zn_ans_decompress_temp_bytes(n))
    temp = torch.empty(max(tb, 1), dtype=torch.uint8, device=in_ptrs.device)
    _lib.check(
        _lib.lib.zn_ans_decompress(in_ptrs.data_ptr(), in_bytes.data_ptr(), out_capacity.data_ptr(), n,
                                   out_ptrs.data_ptr(), statuses.data_ptr(), temp.data_ptr(), tb,
                                   _stream(in_ptrs)),
        "zn_ans_decompress",
    )
    return statuses
