"""Byte-plane kernels with the signatures of the reference's Triton module
(src/cuzipnn/_kernels.py:134-188), backed by libcuzipnn_b200.so.

The whole-tensor codec does not call these (its split and merge are fused into the coder); they
are the drop-in seam for code written against the reference's internals.
"""

import torch

from . import _lib


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def split(x: torch.Tensor, planar: torch.Tensor, stride: int, reorder: bool) -> None:
    """Byte b of (reordered) element e goes to planar[b * stride + e] (_kernels.py:134-148)."""
    _lib.check(
        _lib.lib.zn_split(x.data_ptr(), x.numel(), x.element_size(), int(reorder), planar.data_ptr(),
                          stride, _stream(x)),
        "zn_split",
    )


def merge(src_tbl: torch.Tensor, base: torch.Tensor, out: torch.Tensor, chunk_bytes: int, reorder: bool) -> None:
    """src_tbl holds int64 byte offsets from base.data_ptr(), each a multiple of 8
    (_kernels.py:151-176)."""
    _lib.check(
        _lib.lib.zn_merge(src_tbl.data_ptr(), base.data_ptr(), out.data_ptr(), out.numel(), out.element_size(),
                          chunk_bytes, int(reorder), _stream(out)),
        "zn_merge",
    )


def copy_chunks(src_tbl: torch.Tensor, dst_tbl: torch.Tensor, nbytes: torch.Tensor, max_bytes: int, pad: bool) -> None:
    """src_tbl/dst_tbl hold int64 device addresses; a chunk with nbytes 0 is skipped
    (_kernels.py:179-188)."""
    _lib.check(
        _lib.lib.zn_copy_chunks(src_tbl.data_ptr(), dst_tbl.data_ptr(), nbytes.data_ptr(), src_tbl.numel(),
                                max_bytes, int(pad), _stream(src_tbl)),
        "zn_copy_chunks",
    )
