"""ZipNN on the B200: bit reordering, byte grouping and rANS coding in hand-written sm_100a kernels.

This module keeps the public API, argument checks, device rules and blob container of the
reference (ruihe774/cuZipNN, src/cuzipnn/_codec.py) and replaces its GPU pipeline (Triton split,
nvCOMP ANS, a blocking host-side passthrough decision, table upload and two copy passes) with one
call into libcuzipnn_b200.so per direction.

The container (src/cuzipnn/_codec.py:3-20), little-endian, with every section starting on an
8-byte boundary:

    bytes 0-3    "ZNNG"             byte 4   version (3 here)     byte 5   dtype code
    byte 6       ndim               byte 7   flags: 1 = exponent bits reordered, 2 = stored raw
    bytes 8-11   chunk_bytes        bytes 12-15  n_comp           bytes 16-23  numel
    then         ndim int64 dimensions

A tensor below min_compress_bytes is "stored": chunk_bytes and n_comp are 0 and its bytes follow
the header as they are.  Any other tensor has K byte streams (K = element size) cut into
nch = ceil(numel / chunk_bytes) chunks, and after the header come: an int32 per (stream, chunk)
unit with the bytes it occupies, an int32 per rANS-coded unit with its index (ascending), padding
to 8, and the units themselves in (stream, chunk) order, each padded to 8 bytes.

Version 3 marks coded units as ZNR2 rANS payloads (include/cuzipnn_b200.h), not nvCOMP ANS
streams; version-2 blobs of the reference are therefore rejected, as the reference rejects
versions other than its own (src/cuzipnn/_codec.py:423-424).
"""

from __future__ import annotations

import contextlib
import ctypes
import functools
import math
import struct
import threading
import zlib
from collections.abc import Buffer

import numpy as np
import torch

from . import _lib

_MAGIC = b"ZNNG"
_VERSION = 3
_FIXED = struct.Struct("<4sBBBBIIQ")
_FLAG_REORDER = 1
_FLAG_STORED = 2
_MAX_NDIM = 64
MAX_CHUNK_BYTES = 1 << 24
MIN_SUB_CHUNKS = 4
MAX_SUB_CHUNKS = 64

DEFAULT_CHUNK_BYTES = 128 * 1024
DEFAULT_SUB_CHUNK_BYTES = 8 * 1024
DEFAULT_PASSTHROUGH_THRESHOLD = 0.95
DEFAULT_MIN_COMPRESS_BYTES = 64 * 1024
DEFAULT_CHECKSUM_CHUNK_BYTES = 16 * 1024

# src/cuzipnn/_codec.py:47-64
_DTYPES = {
    1: torch.bool,
    2: torch.uint8,
    3: torch.int8,
    4: torch.int16,
    5: torch.int32,
    6: torch.int64,
    7: torch.float16,
    8: torch.bfloat16,
    9: torch.float32,
    10: torch.float64,
    11: torch.float8_e4m3fn,
    12: torch.float8_e5m2,
    13: torch.uint16,
    14: torch.uint32,
    15: torch.uint64,
    16: torch.complex64,
}
_CODES = {dtype: code for code, dtype in _DTYPES.items()}
# As in ZipNN, only bfloat16 and float32 get the exponent bit reordering.
_REORDER = {torch.bfloat16, torch.float32}


def _align8(x: int) -> int:
    return (x + 7) & ~7


def _sub_chunks(chunk_bytes: int, sub_chunk_bytes: int) -> int:
    """Sub-chunk count: chunk_bytes / sub_chunk_bytes rounded up to a power of 2 in [4, 64]
    (src/cuzipnn/_codec.py:83-86)."""
    count = 1 << (-(-chunk_bytes // sub_chunk_bytes) - 1).bit_length()
    return min(max(count, MIN_SUB_CHUNKS), MAX_SUB_CHUNKS)


def _layout(ndim: int, total: int, n_comp: int) -> tuple[int, int, int]:
    """Where the unit-size table, the coded-index table and the unit data start in a blob with
    `total` units of which n_comp are coded (the container of _codec.py:89-93)."""
    head = _FIXED.size + 8 * ndim
    return head, head + 4 * total, _align8(head + 4 * (total + n_comp))


def _check_device(compute_device: torch.device | str | None) -> torch.device | None:
    """Parse compute_device and insist on a CUDA device (the rule of _codec.py:96-103).  No CUDA
    call is made, so a bad value is reported the same way on a machine without a GPU."""
    if compute_device is None:
        return None
    dev = compute_device if isinstance(compute_device, torch.device) else torch.device(compute_device)
    if dev.type == "cuda":
        return dev
    raise ValueError(f"compute_device must be a CUDA device, not {dev}")


def _gpu(x: torch.Tensor, compute_device: torch.device | None) -> torch.device:
    """The GPU a call works on, with an explicit index: the device the caller named, else the
    tensor's own GPU, else the current CUDA device (the rule of _codec.py:106-113)."""
    if compute_device is not None:
        dev = compute_device
    elif x.is_cuda:
        dev = x.device
    else:
        dev = torch.device("cuda")
    return dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())


def _stream(device: torch.device) -> int:
    """Raw handle of the device's current stream (as torch.cuda.current_stream(device).cuda_stream,
    without building a Stream object on every call)."""
    return torch._C._cuda_getCurrentRawStream(device.index)


def _on(device: torch.device):
    """torch.cuda.device(device), or nothing when it is the current device already."""
    if torch.cuda.current_device() == device.index:
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _remember(blob: torch.Tensor, dtype: torch.dtype, shape: tuple[int, ...], flags: int, chunk_bytes: int,
              n: int) -> torch.Tensor:
    """Keep the header fields of a GPU blob made here on the returned tensor object, with the
    blob's version counter, address and size: decompressing the unchanged blob then needs no host
    read of its header (a synchronization that would drain the stream).  Any in-place write to
    the blob or to a view of its storage bumps the shared version counter and voids the record."""
    blob._zn_header = (blob._version, blob.data_ptr(), blob.numel(), dtype, shape, flags, chunk_bytes, n)
    return blob


def _capacity_views(out: torch.Tensor, offs: list[int]) -> tuple[torch.Tensor, ...]:
    """One view of `out` per region [offs[j], offs[j + 1]) (the last to the end), by one split."""
    return out.split([b - a for a, b in zip(offs, offs[1:] + [out.numel()])])


def _trim_and_remember(out: torch.Tensor, views, sizes: list[int], offs: list[int], fields: list[tuple]) -> None:
    """Trim each capacity view of `out` to its blob's size (resize_ shrinks a view in place; the
    storage stays) and give it the record _remember makes, fields[j] = (dtype, shape, flags,
    chunk_bytes, n).  The views share the buffer's version counter (bumped by each resize_, so it
    is read after them), and each view's address and size follow from the offsets, so no view is
    asked for them."""
    for v, size in zip(views, sizes):
        v.resize_(size)
    ver, base = out._version, out.data_ptr()
    for v, o, size, f in zip(views, offs, sizes, fields):
        v._zn_header = (ver, base + o, size) + f


def _known_header(blob: torch.Tensor):
    """(dtype, shape, flags, chunk_bytes, n) of a GPU blob from _remember, if it still applies."""
    h = getattr(blob, "_zn_header", None)
    if h is None or not blob.is_cuda or h[0] != blob._version or h[1] != blob.data_ptr() or h[2] != blob.numel():
        return None
    return h[3:]


def _crc32(data: torch.Tensor, checksum_chunk_bytes: int) -> torch.Tensor:
    """Enqueue the CRC-32 of each checksum_chunk_bytes-byte chunk of `data`, a contiguous uint8
    CUDA tensor (_codec.py:116-131).  The last chunk may be shorter.  Returns uint32 on the GPU."""
    nbytes = data.numel()
    m = -(-nbytes // checksum_chunk_bytes)
    crc = torch.empty(m, dtype=torch.uint32, device=data.device)
    if m:
        tb = int(_lib.lib.zn_crc32_temp_bytes(nbytes, checksum_chunk_bytes))
        temp = torch.empty(max(tb, 1), dtype=torch.uint8, device=data.device)
        _lib.check(
            _lib.lib.zn_crc32(
                data.data_ptr(), nbytes, checksum_chunk_bytes, crc.data_ptr(), temp.data_ptr(), tb,
                _stream(data.device),
            ),
            "zn_crc32",
        )
    return crc


def _fill_stored(
    blob: torch.Tensor, offset: int, x: torch.Tensor, checksum_chunk_bytes: int | None
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Write the tensor's bytes behind the header of a host blob (blob[offset:]) and, when
    checksums are asked for, hash the finished blob segment by segment with zlib on the host: a
    blob this small costs less to hash there than to send to the GPU and back (the stored path of
    _codec.py:134-147)."""
    blob[offset:].view(x.dtype).view(x.shape).copy_(x)
    if checksum_chunk_bytes is None:
        return blob, None
    return blob, _host_crc32(blob, checksum_chunk_bytes)


def _host_crc32(blob: torch.Tensor, checksum_chunk_bytes: int) -> torch.Tensor:
    """zlib CRC-32 of each checksum_chunk_bytes-byte segment of a host uint8 tensor (the last one
    possibly shorter), as a uint32 tensor."""
    raw = memoryview(blob.numpy())
    starts = range(0, len(raw), checksum_chunk_bytes)
    return torch.tensor([zlib.crc32(raw[i : i + checksum_chunk_bytes]) for i in starts], dtype=torch.uint32)


def compress_tensor(
    tensor: torch.Tensor,
    *,
    chunk_bytes: int = DEFAULT_CHUNK_BYTES,
    sub_chunk_bytes: int = DEFAULT_SUB_CHUNK_BYTES,
    passthrough_threshold: float = DEFAULT_PASSTHROUGH_THRESHOLD,
    min_compress_bytes: int = DEFAULT_MIN_COMPRESS_BYTES,
    pin_memory: bool = False,
    compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = True,
) -> torch.Tensor:
    """Compress a tensor losslessly on the GPU; returns a 1-D uint8 tensor."""
    blob, _ = _compress(
        tensor,
        chunk_bytes=chunk_bytes,
        sub_chunk_bytes=sub_chunk_bytes,
        passthrough_threshold=passthrough_threshold,
        min_compress_bytes=min_compress_bytes,
        checksum_chunk_bytes=None,
        pin_memory=pin_memory,
        compute_device=compute_device,
        readback_to_cpu=readback_to_cpu,
    )
    return blob


def compress_tensor_with_crc32(
    tensor: torch.Tensor,
    *,
    chunk_bytes: int = DEFAULT_CHUNK_BYTES,
    sub_chunk_bytes: int = DEFAULT_SUB_CHUNK_BYTES,
    passthrough_threshold: float = DEFAULT_PASSTHROUGH_THRESHOLD,
    min_compress_bytes: int = DEFAULT_MIN_COMPRESS_BYTES,
    checksum_chunk_bytes: int = DEFAULT_CHECKSUM_CHUNK_BYTES,
    pin_memory: bool = False,
    compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """compress_tensor, plus the CRC-32 (as zlib.crc32) of each checksum_chunk_bytes-byte chunk
    of the blob, the last one possibly shorter, as a 1-D uint32 tensor on the blob's device.

    The blob is the same as compress_tensor's.  The checksums are computed on the GPU before the
    blob is copied back (on the CPU for tensors below min_compress_bytes, which are stored
    uncompressed); hash_tensor_with_crc32(blob) reproduces them, so a blob can be verified before
    it is passed to decompress_tensor.
    """
    blob, checksums = _compress(
        tensor,
        chunk_bytes=chunk_bytes,
        sub_chunk_bytes=sub_chunk_bytes,
        passthrough_threshold=passthrough_threshold,
        min_compress_bytes=min_compress_bytes,
        checksum_chunk_bytes=checksum_chunk_bytes,
        pin_memory=pin_memory,
        compute_device=compute_device,
        readback_to_cpu=readback_to_cpu,
    )
    assert checksums is not None
    return blob, checksums


def hash_tensor_with_crc32(
    tensor: torch.Tensor,
    *,
    checksum_chunk_bytes: int = DEFAULT_CHECKSUM_CHUNK_BYTES,
    compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = True,
) -> torch.Tensor:
    """CRC-32 (as zlib.crc32) of each checksum_chunk_bytes-byte chunk of the tensor's bytes in
    row-major order, the last one possibly shorter, computed on the GPU.  Returns a 1-D uint32
    tensor."""
    if checksum_chunk_bytes <= 0:
        raise ValueError("checksum_chunk_bytes must be positive")
    x = tensor.detach()
    device = _gpu(x, _check_device(compute_device))
    with torch.cuda.device(device):
        if x.is_cuda:
            x = x.to(device, non_blocking=True, memory_format=torch.contiguous_format).contiguous()
        else:
            x = _upload(x.contiguous(), device)
        crc = _crc32(x.view(-1).view(torch.uint8), checksum_chunk_bytes)
        return crc.cpu() if readback_to_cpu else crc


def _check_args(
    tensor: torch.Tensor,
    chunk_bytes: int,
    sub_chunk_bytes: int,
    passthrough_threshold: float,
    min_compress_bytes: int,
    checksum_chunk_bytes: int | None,
    pin_memory: bool,
    compute_device: torch.device | str | None,
    readback_to_cpu: bool,
) -> tuple[torch.device | None, int]:
    """Argument checks in the reference's order and wording (_codec.py:243-262)."""
    compute_device = _check_device(compute_device)
    if pin_memory and not readback_to_cpu:
        raise ValueError("pin_memory requires readback_to_cpu")
    if tensor.dtype not in _CODES:
        raise TypeError(f"unsupported dtype {tensor.dtype}")
    if chunk_bytes % 8 or not 0 < chunk_bytes <= MAX_CHUNK_BYTES:
        raise ValueError(f"chunk_bytes must be a multiple of 8 in (0, {MAX_CHUNK_BYTES}]")
    if passthrough_threshold <= 0 or passthrough_threshold > 1:
        raise ValueError("passthrough_threshold must be in (0, 1]")
    if sub_chunk_bytes <= 0:
        raise ValueError("sub_chunk_bytes must be positive")
    if min_compress_bytes < 0:
        raise ValueError("min_compress_bytes must be non-negative")
    if checksum_chunk_bytes is not None and checksum_chunk_bytes <= 0:
        raise ValueError("checksum_chunk_bytes must be positive")
    sub_chunks = _sub_chunks(chunk_bytes, sub_chunk_bytes)
    if tensor.dim() > _MAX_NDIM:
        raise ValueError(f"at most {_MAX_NDIM} dimensions are supported")
    return compute_device, sub_chunks


def _header(tensor: torch.Tensor, flags: int, chunk_bytes: int, n_comp: int) -> bytes:
    """The fixed header and shape (_codec.py:270-292)."""
    return _header_bytes(tensor.dtype, tuple(tensor.shape), flags, chunk_bytes, n_comp)


@functools.lru_cache(maxsize=4096)
def _header_bytes(dtype: torch.dtype, shape: tuple[int, ...], flags: int, chunk_bytes: int, n_comp: int) -> bytes:
    """Header bytes by their fields: a model's tensors share few shapes, so most are packed once."""
    fixed = _FIXED.pack(_MAGIC, _VERSION, _CODES[dtype], len(shape), flags, chunk_bytes, n_comp, math.prod(shape))
    return fixed + struct.pack(f"<{len(shape)}q", *shape)


def _compress(
    tensor: torch.Tensor,
    *,
    chunk_bytes: int,
    sub_chunk_bytes: int,
    passthrough_threshold: float,
    min_compress_bytes: int,
    checksum_chunk_bytes: int | None,
    pin_memory: bool,
    compute_device: torch.device | str | None,
    readback_to_cpu: bool,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    compute_device, sub_chunks = _check_args(
        tensor, chunk_bytes, sub_chunk_bytes, passthrough_threshold, min_compress_bytes,
        checksum_chunk_bytes, pin_memory, compute_device, readback_to_cpu,
    )

    x = tensor.detach()
    k, n, reorder = x.element_size(), x.numel(), x.dtype in _REORDER
    header_size = _FIXED.size + 8 * tensor.dim()

    # Stored path and empty tensors (_codec.py:294-306): no GPU work with readback_to_cpu.
    if n * k < min_compress_bytes or n == 0:
        stored = n * k < min_compress_bytes
        head = _header(tensor, _FLAG_STORED if stored else _FLAG_REORDER if reorder else 0,
                       0 if stored else chunk_bytes, 0)
        if readback_to_cpu:
            blob = _populated_empty(header_size + n * k, pin_memory=pin_memory)
            blob[:header_size].copy_(torch.frombuffer(bytearray(head), dtype=torch.uint8))
            return _fill_stored(blob, header_size, x, checksum_chunk_bytes)
        device = _gpu(x, compute_device)
        with _on(device):
            blob = torch.empty(header_size + n * k, dtype=torch.uint8, device=device)
            blob[:header_size].copy_(torch.frombuffer(bytearray(head), dtype=torch.uint8))
            blob[header_size:].view(x.dtype).view(x.shape).copy_(x)
            crc = None if checksum_chunk_bytes is None else _crc32(blob, checksum_chunk_bytes)
            flags = _FLAG_STORED if stored else _FLAG_REORDER if reorder else 0
            return _remember(blob, x.dtype, tuple(x.shape), flags, 0 if stored else chunk_bytes, n), crc

    device = _gpu(x, compute_device)
    with _on(device):
        if not x.is_cuda:
            x = _upload(x.contiguous(), device)
        elif not (x.get_device() == device.index and x.is_contiguous()):
            x = x.to(device, non_blocking=True, memory_format=torch.contiguous_format).contiguous()
        if x.data_ptr() % 16:  # only the address and the size of the contiguous input are used
            x = x.clone()
        shape = tuple(tensor.shape)
        head = _header_bytes(x.dtype, shape, _FLAG_REORDER if reorder else 0, chunk_bytes, 0)
        cap = int(_lib.lib.zn_compress_bound(n, k, len(shape), chunk_bytes))
        temp_bytes = int(_lib.lib.zn_compress_temp_bytes(n, k, chunk_bytes, sub_chunks))
        # The blob is packed into a buffer at least as large as the input (README "API").
        out = torch.empty(cap, dtype=torch.uint8, device=device)
        temp = torch.empty(max(temp_bytes, 1), dtype=torch.uint8, device=device)
        size_dev = torch.empty(1, dtype=torch.int64, device=device)
        _lib.check(
            _lib.lib.zn_compress(
                x.data_ptr(), n, k, int(reorder), head, len(head), chunk_bytes, sub_chunks,
                float(passthrough_threshold), out.data_ptr(), cap, size_dev.data_ptr(),
                temp.data_ptr(), temp_bytes, _stream(device),
            ),
            "zn_compress",
        )
        size = int(size_dev.item())
        comp = out[:size]
        crc = None
        if checksum_chunk_bytes is not None:
            crc = _crc32(comp, checksum_chunk_bytes)
        if not readback_to_cpu:
            return _remember(comp, tensor.dtype, shape, _FLAG_REORDER if reorder else 0, chunk_bytes, n), crc
        if pin_memory:
            blob = _populated_empty(size, pin_memory=True)
            # With a crc, crc.cpu() below syncs the stream, so blob is complete on return.
            blob.copy_(comp, non_blocking=crc is not None)
        else:
            blob = _host_empty(size)
            _download(comp, blob)
        return blob, None if crc is None else crc.cpu()


def _parse_header(prefix: Buffer, off: int = 0, length: int | None = None
                  ) -> tuple[torch.dtype, tuple[int, ...], int, int, int, int]:
    """(_codec.py:416-428) The header in prefix[off : off + length] (default: to the end)."""
    prefix = memoryview(prefix)
    if length is None:
        length = len(prefix) - off
    if length < _FIXED.size:
        raise ValueError("blob is too short")
    magic, version, code, ndim, flags, chunk_bytes, n_comp, n = _FIXED.unpack_from(prefix, off)
    if magic != _MAGIC or version != _VERSION or code not in _DTYPES:
        raise ValueError("not a cuzipnn blob")
    if length < _FIXED.size + 8 * ndim:
        raise ValueError("blob is too short")
    shape = struct.unpack_from(f"<{ndim}q", prefix, off + _FIXED.size)
    return _DTYPES[code], shape, flags, chunk_bytes, n_comp, n


# Status words of the calling thread's latest decompress call per device (0 = no decoding error).
# Per thread, so that threads decoding on one device do not overwrite each other's status.
_STATUS = threading.local()


def _set_status(device: torch.device, status: torch.Tensor) -> None:
    if not hasattr(_STATUS, "by_dev"):
        _STATUS.by_dev = {}
    _STATUS.by_dev[device.index] = status


def last_decode_status(device: torch.device | str | int | None = None) -> int:
    """Error bits the device kernels reported for this thread's latest decompress_tensor (or
    decompress_tensors) call on `device` (synchronizes with it).  0 means every unit decoded and
    validated; nonzero means the blob was malformed (the affected elements were zeroed).
    decompress_tensor checks this itself when it synchronizes anyway (readback_to_cpu=True)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    st = getattr(_STATUS, "by_dev", {}).get(dev.index if dev.type == "cuda" else int(dev))
    if st is None:
        return 0
    bits = 0
    for v in st.cpu().tolist():  # one word per blob of the latest call: OR them
        bits |= int(v)
    return bits


def _check_out(out: torch.Tensor, dtype: torch.dtype, shape: tuple[int, ...], cpu: bool) -> None:
    """A caller's output tensor must match the blob's tensor: same dtype (TypeError otherwise), same
    shape, contiguous, and on the CPU (readback_to_cpu) or a GPU (ValueError otherwise)."""
    if out.dtype != dtype:
        raise TypeError(f"out has dtype {out.dtype}, the blob holds {dtype}")
    if tuple(out.shape) != tuple(shape):
        raise ValueError(f"out has shape {tuple(out.shape)}, the blob holds {tuple(shape)}")
    if not out.is_contiguous():
        raise ValueError("out must be contiguous")
    if cpu and out.is_cuda:
        raise ValueError("out must be a CPU tensor with readback_to_cpu")
    if not cpu and not out.is_cuda:
        raise ValueError("out must be a CUDA tensor without readback_to_cpu")


def decompress_tensor(
    blob: torch.Tensor,
    *,
    compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decompress a blob produced by compress_tensor; the blob may be on the CPU or the GPU.

    With `out` (an addition to the reference's signature, whose call allocates its result each
    time), the tensor is decoded straight into the caller's storage and `out` is returned: a
    contiguous tensor of the blob's dtype and shape, on a GPU (it sets the compute device, which
    compute_device must then name too) or, with readback_to_cpu, on the CPU.  A loader can so fill
    pre-allocated weights without an extra copy or allocation.

    Passing a blob that is not from `compress_tensor` gives an unspecified result (never an
    out-of-bounds access); last_decode_status() reports it.
    """
    compute_device = _check_device(compute_device)
    if blob.dtype != torch.uint8 or blob.dim() != 1:
        raise ValueError("blob must be a 1-D uint8 tensor")

    known = _known_header(blob)
    blob = blob.detach()
    if known is not None:  # an unchanged GPU blob made here: its header is on the host already
        dtype, shape, flags, chunk_bytes, n = known
        n_comp = -1  # read from the blob by the device
    else:
        prefix_len = min(blob.numel(), _FIXED.size + 8 * _MAX_NDIM)
        prefix_tensor = blob[:prefix_len].to("cpu", memory_format=torch.contiguous_format).contiguous()
        prefix = (ctypes.c_byte * prefix_len).from_address(prefix_tensor.data_ptr())
        dtype, shape, flags, chunk_bytes, n_comp, n = _parse_header(prefix)
    reorder = bool(flags & _FLAG_REORDER)
    if out is not None:
        _check_out(out, dtype, shape, readback_to_cpu)
        if out.is_cuda:
            if compute_device is not None and _gpu(blob, compute_device) != out.device:
                raise ValueError("out is not on compute_device")
            compute_device = out.device

    if flags & _FLAG_STORED:
        # Stored uncompressed: copy the bytes after the header straight to the target device.
        header_size = _FIXED.size + 8 * len(shape)
        nbytes = math.prod(shape) * dtype.itemsize
        if blob.numel() < header_size + nbytes:
            raise ValueError("blob is truncated")
        if out is None:
            if readback_to_cpu:
                out = _populated_empty(nbytes).view(dtype).view(shape)
            else:
                out = torch.empty(shape, dtype=dtype, device=_gpu(blob, compute_device))
        out.view(-1).view(torch.uint8).copy_(blob[header_size : header_size + nbytes])
        return out

    if n == 0:
        if out is not None:
            return out
        return torch.empty(
            shape, dtype=dtype, device="cpu" if readback_to_cpu else _gpu(blob, compute_device)
        )
    if math.prod(shape) != n or chunk_bytes <= 0:
        raise ValueError("not a cuzipnn blob")
    device = _gpu(blob, compute_device)
    host_out = out if readback_to_cpu else None
    y = out if (out is not None and not readback_to_cpu) else torch.empty(shape, dtype=dtype, device=device)

    k = y.element_size()
    if n_comp >= 0:
        nch = -(-n // chunk_bytes)
        _, _, data_off = _layout(len(shape), k * nch, n_comp)
        if blob.numel() < data_off:
            raise ValueError("blob is truncated")

    with _on(device):
        x = blob
        if not x.is_cuda:
            x = _upload(x.contiguous(), device)
        elif not (x.device == device and x.is_contiguous()):
            x = x.to(device, non_blocking=True, memory_format=torch.contiguous_format).contiguous()
        if x.data_ptr() % 8:
            x = x.clone()
        # A pinned blob is uploaded asynchronously, but the caller may reuse it once we return.
        uploaded = torch.cuda.Event() if blob.is_pinned() else None
        if uploaded is not None:
            uploaded.record()
        temp_bytes = int(_lib.lib.zn_decompress_temp_bytes(n, k, chunk_bytes))
        temp = torch.empty(max(temp_bytes, 1), dtype=torch.uint8, device=device)
        status = torch.empty(1, dtype=torch.int32, device=device)  # set by the call
        _lib.check(
            _lib.lib.zn_decompress(
                x.data_ptr(), x.numel(), n, k, int(reorder), len(shape), chunk_bytes, n_comp,
                y.data_ptr(), status.data_ptr(), temp.data_ptr(), temp_bytes, _stream(device),
            ),
            "zn_decompress",
        )
        _set_status(device, status)

        if uploaded is not None:
            uploaded.synchronize()

        if readback_to_cpu:
            src = y
            y = host_out if host_out is not None else (
                _host_empty(src.numel() * src.element_size()).view(src.dtype).view_as(src))
            _download(src, y)
            if int(status.item()):
                raise ValueError(f"blob is corrupt (decoder status {int(status.item())})")

        return y


def _ptr_array(ctype, values):
    return (ctype * len(values))(*values)


_PIPELINE_BYTES = 1 << 29  # sub-batch of host-resident inputs (upload overlapped with the kernels)
_DEVICE_BATCH_BYTES = 1 << 32  # sub-batch of device-resident inputs (launched while the host prepares the next)
# The first sub-batch of a call is launched once _FIRST_BATCH bytes are read, so that the GPU
# starts soon; each later one is _BATCH_GROWTH times larger (up to the batch limit), so that the
# kernels of one batch run while the host prepares the next.  512 MB keep the kernels of the first
# batch busy (0.3-0.5 ms) for as long as the host needs to read and launch the next hundred or so
# tensors (a few microseconds each), and take the host only a few tensors of a model to gather.
_FIRST_BATCH = 1 << 29
_BATCH_GROWTH = 16


def _batch_limit(limit: int, launched: int) -> int:
    """Input bytes of the next sub-batch of a call after `launched` sub-batches."""
    return min(limit, _FIRST_BATCH * _BATCH_GROWTH ** min(launched, 16))


_TINY_BYTES = 65536  # stored tensors up to this size decode into views of one shared buffer per call
_COPY_BATCH_MAX = 1 << 29  # largest single copy of one zn_copy_chunks launch (65535 tiles of 8 KiB)


_SIDE_STREAMS: dict[tuple[int, int], torch.cuda.Stream] = {}


def _side_stream(device: torch.device, which: int) -> torch.cuda.Stream:
    """The upload (0) or download (1) stream of a device, created once: the caching allocator keeps
    a pool per stream, so reusing the streams lets later calls reuse the staging memory."""
    key = (device.index, which)
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = torch.cuda.Stream(device)
    return _SIDE_STREAMS[key]


def _copy_batch(device: torch.device, srcs: list[int], dsts: list[int], sizes: list[int]) -> None:
    """Many small device copies (8-byte aligned addresses) in one zn_copy_chunks launch; the address
    table goes to the GPU in one pinned copy."""
    n = len(srcs)
    if n == 0:
        return
    host = torch.from_numpy(np.array(srcs + dsts + sizes, dtype=np.int64)).pin_memory()
    tbl = host.to(device, non_blocking=True)
    base = tbl.data_ptr()
    _lib.check(
        _lib.lib.zn_copy_chunks(base, base + 8 * n, base + 16 * n, n, max(sizes), 0, _stream(device)),
        "zn_copy_chunks",
    )


def _stored_blobs_gpu(items: list[tuple[int, torch.Tensor, int, bytes, tuple]], device: torch.device
                      ) -> dict[int, torch.Tensor]:
    """Blobs of the stored path (header + raw bytes) for many tensors, built on the GPU by one
    header upload and one batched copy.  items: (index, tensor, its bytes, header, header fields
    for _remember).  Each blob is a view into one shared buffer (256-byte aligned)."""
    dev = device.index
    offs, pos = [], 0
    for _, _, nb, head, _ in items:
        offs.append(pos)
        pos += (len(head) + nb + 255) & ~255
    out = torch.empty(pos, dtype=torch.uint8, device=device)
    views = _capacity_views(out, offs)
    hdev = torch.frombuffer(bytearray(b"".join(h for _, _, _, h, _ in items)), dtype=torch.uint8).pin_memory()
    hdev = hdev.to(device, non_blocking=True)
    srcs, dsts, sizes = [], [], []
    hpos, hbase, obase = 0, hdev.data_ptr(), out.data_ptr()
    for (_, x, nb, head, _), o in zip(items, offs):
        hl = len(head)
        srcs.append(hbase + hpos)
        dsts.append(obase + o)
        sizes.append(hl)
        hpos += hl
        if nb:
            if not (x.is_cuda and x.get_device() == dev and x.is_contiguous() and x.data_ptr() % 8 == 0):
                x = x.detach().to(device, non_blocking=True, memory_format=torch.contiguous_format).contiguous()
                if x.data_ptr() % 8:
                    x = x.clone()
            srcs.append(x.data_ptr())
            dsts.append(obase + o + hl)
            sizes.append(nb)
    # `hdev` and the staged inputs were allocated on this stream, so the caching allocator reuses
    # their memory only after the copy has run.
    _copy_batch(device, srcs, dsts, sizes)
    _trim_and_remember(out, views, [len(h) + nb for _, _, nb, h, _ in items], offs, [f for *_, f in items])
    return {it[0]: v for it, v in zip(items, views)}


def compress_tensors(
    tensors: list[torch.Tensor],
    *,
    chunk_bytes: int = DEFAULT_CHUNK_BYTES,
    sub_chunk_bytes: int = DEFAULT_SUB_CHUNK_BYTES,
    passthrough_threshold: float = DEFAULT_PASSTHROUGH_THRESHOLD,
    min_compress_bytes: int = DEFAULT_MIN_COMPRESS_BYTES,
    pin_memory: bool = False,
    compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = True,
) -> list[torch.Tensor]:
    """compress_tensor over a list of tensors, with one kernel launch per stage for each batch of
    tensors of an element size (batches of about _DEVICE_BATCH_BYTES, launched while the host
    prepares the next).  Each blob equals compress_tensor's.

    With readback_to_cpu=False the blobs are views into one shared GPU buffer per batch.  Host
    inputs are uploaded in batches of about _PIPELINE_BYTES on a side stream, so that uploads,
    kernels and (with readback_to_cpu) downloads of different batches overlap; with pin_memory the
    read-back blobs of a batch are views into one pinned buffer.  Tensors are checked as the list
    is read, so an invalid tensor raises after the batches before it may have been launched (their
    results are dropped)."""
    blobs: list[torch.Tensor | None] = [None] * len(tensors)
    small: list[tuple[int, int, int]] = []  # (index, element size, numel) of the stored path and empty tensors, handled after the coded launches
    sub_chunks = _sub_chunks(chunk_bytes, sub_chunk_bytes) if sub_chunk_bytes > 0 else 0
    cd = _check_device(compute_device)

    def compress_small(device: torch.device | None) -> None:
        batch = []
        for i, k, n in small:
            t = tensors[i]
            if (device is not None and not readback_to_cpu and n * k <= _COPY_BATCH_MAX
                    and (t.get_device() == device.index if cd is None and t.is_cuda else _gpu(t, cd) == device)):
                stored = n * k < min_compress_bytes
                dtype, shape = t.dtype, tuple(t.shape)
                flags = _FLAG_STORED if stored else _FLAG_REORDER if dtype in _REORDER else 0
                cbf = 0 if stored else chunk_bytes
                batch.append((i, t, n * k, _header_bytes(dtype, shape, flags, cbf, 0), (dtype, shape, flags, cbf, n)))
            else:
                blobs[i] = compress_tensor(t, chunk_bytes=chunk_bytes, sub_chunk_bytes=sub_chunk_bytes,
                                           passthrough_threshold=passthrough_threshold,
                                           min_compress_bytes=min_compress_bytes, pin_memory=pin_memory,
                                           compute_device=compute_device, readback_to_cpu=readback_to_cpu)
        if batch:
            for i, b in _stored_blobs_gpu(batch, device).items():
                blobs[i] = b

    device: torch.device | None = None
    stream = copy_in = None
    pending: list[list] = []

    def launch(k: int, reorder: bool, idx: list[int]) -> None:
        """Stage a batch's inputs on the device (host tensors go up on the copy stream, so that the
        upload of one batch overlaps the kernels of the previous one) and launch its kernels."""
        nonlocal copy_in
        host = any(not tensors[i].is_cuda for i in idx)
        if host and copy_in is None:
            copy_in = _side_stream(device, 0)
        up = copy_in if host else stream
        with torch.cuda.stream(up) if host else contextlib.nullcontext():  # `stream` is current already
            xs = []
            dev = device.index
            for i in idx:
                x = tensors[i]
                if not x.is_cuda:
                    x = _upload(x.detach().contiguous(), device)
                    if x.data_ptr() % 16:
                        x = x.clone()
                elif not (x.get_device() == dev and x.is_contiguous() and x.data_ptr() % 16 == 0):
                    x = x.detach().to(device, non_blocking=True, memory_format=torch.contiguous_format).contiguous()
                    if x.data_ptr() % 16:
                        x = x.clone()
                xs.append(x)  # only its address and size are used
        if up is not stream:
            stream.wait_stream(up)
            for x in xs:
                x.record_stream(stream)
        out, offs, sizes, temp, fields = _launch_compress_batch(
            device, xs, [tensors[i] for i in idx], k, reorder, chunk_bytes, sub_chunks, passthrough_threshold)
        sizes_host = None
        if readback_to_cpu:  # each batch's sizes come back on their own, batches keep running
            sizes_host = torch.empty(len(idx), dtype=torch.int64, pin_memory=True)
            sizes_host.copy_(sizes, non_blocking=True)
        done = torch.cuda.Event()
        done.record(stream)
        # The staged inputs and the scratch are only used on `stream` from here on, so the
        # caching allocator may hand their memory to later batches in stream order.
        del xs, temp
        # Without readback, each blob will be a view into the batch buffer: made now, at its
        # capacity, while the kernels run, and trimmed to the blob's size after the sync.
        views = None if readback_to_cpu else _capacity_views(out, offs)
        pending.append([idx, out, offs, sizes, sizes_host, done, fields, views])

    # Coded tensors are launched in batches of one element size as the list is read (the first
    # batch smaller), so that the GPU starts while the host reads the rest.
    cur: dict[tuple[int, bool], tuple[list[int], int]] = {}
    with contextlib.ExitStack() as ctx:
        for i, t in enumerate(tensors):
            if i == 0:  # the scalar arguments once, then each tensor's dtype and rank
                cd, sub_chunks = _check_args(t, chunk_bytes, sub_chunk_bytes, passthrough_threshold,
                                             min_compress_bytes, None, pin_memory, compute_device, readback_to_cpu)
            elif t.dtype not in _CODES:
                raise TypeError(f"unsupported dtype {t.dtype}")
            elif t.dim() > _MAX_NDIM:
                raise ValueError(f"at most {_MAX_NDIM} dimensions are supported")
            k, n = t.element_size(), t.numel()
            if n * k < min_compress_bytes or n == 0:
                small.append((i, k, n))
                continue
            if device is None:
                device = _gpu(t.detach(), cd)
                ctx.enter_context(torch.cuda.device(device))
                stream = torch.cuda.current_stream(device)
            key = (k, t.dtype in _REORDER)
            idx, nbytes = cur.get(key, ([], 0))
            idx.append(i)
            nbytes += n * k
            if nbytes >= _batch_limit(_DEVICE_BATCH_BYTES if t.is_cuda else _PIPELINE_BYTES, len(pending)):
                launch(key[0], key[1], idx)
                idx, nbytes = [], 0
            cur[key] = (idx, nbytes)
        if device is None:
            if small and not readback_to_cpu:
                dev = _gpu(tensors[small[0][0]].detach(), cd)
                with torch.cuda.device(dev):
                    compress_small(dev)
            else:
                compress_small(None)
            return blobs  # type: ignore[return-value]
        for (k, reorder), (idx, _) in cur.items():
            if idx:
                launch(k, reorder, idx)
        # The small tensors' host work overlaps the coded kernels.
        compress_small(device)
        if not readback_to_cpu:
            all_sizes = torch.cat([p[3] for p in pending]).cpu().tolist()  # the one synchronization
            pos = 0
            for idx, out, offs, _, _, _, fields, views in pending:
                _trim_and_remember(out, views, all_sizes[pos : pos + len(idx)], offs, fields)
                for i, v in zip(idx, views):
                    blobs[i] = v
                pos += len(idx)
            return blobs  # type: ignore[return-value]
        copy_out = _side_stream(device, 1)
        for entry in pending:
            idx, out, offs, _, sizes_host, done, _, _ = entry
            done.synchronize()
            sizes_b = sizes_host.tolist()
            if pin_memory:  # one pinned buffer per batch (cheaper than one pinned allocation per blob)
                hoffs = [0]
                for size in sizes_b:
                    hoffs.append(hoffs[-1] + ((size + 15) & ~15))
                hbuf = torch.empty(hoffs[-1], dtype=torch.uint8, pin_memory=True)
            copy_out.wait_event(done)
            with torch.cuda.stream(copy_out):
                for j, (i, o, size) in enumerate(zip(idx, offs, sizes_b)):
                    if pin_memory:
                        blob = hbuf[hoffs[j] : hoffs[j] + size]
                        blob.copy_(out[o : o + size], non_blocking=True)
                    else:
                        blob = _host_empty(size)
                        _download(out[o : o + size], blob)
                    blobs[i] = blob
            out.record_stream(copy_out)  # its memory returns to the allocator after the downloads
            entry[1] = out = None
        # Blobs are complete on return, and the device buffers outlive every copy that reads them.
        copy_out.synchronize()
        stream.synchronize()
    return blobs  # type: ignore[return-value]


def _launch_compress_batch(device, xs, srcs, k, reorder, chunk_bytes, sub_chunks, threshold):
    """zn_compress_batch for device tensors `xs` (flat, 16-byte aligned; `srcs` the original
    tensors, for the headers) on the current stream: one blob buffer holding every blob at
    offs[j] (capacity zn_compress_bound each), a device int64 size per blob, the scratch, and the
    header fields of each blob (for _trim_and_remember)."""
    flags = _FLAG_REORDER if reorder else 0
    heads, caps, offs, ns, fields = [], [], [], [], []
    total_cap = 0
    for x, t in zip(xs, srcs):
        shape = tuple(t.shape)
        heads.append(_header_bytes(t.dtype, shape, flags, chunk_bytes, 0))
        n = x.numel()
        ns.append(n)
        fields.append((t.dtype, shape, flags, chunk_bytes, n))
        cap = int(_lib.lib.zn_compress_bound(n, k, len(shape), chunk_bytes))
        caps.append(cap)
        offs.append(total_cap)
        total_cap += (cap + 255) & ~255
    out = torch.empty(total_cap, dtype=torch.uint8, device=device)
    nj = len(xs)
    sizes = torch.empty(nj, dtype=torch.int64, device=device)
    n_arr = _ptr_array(ctypes.c_int64, ns)
    tb = int(_lib.lib.zn_compress_batch_temp_bytes(nj, n_arr, k, chunk_bytes, sub_chunks))
    temp = torch.empty(max(tb, 1), dtype=torch.uint8, device=device)
    # Every header in one host buffer; the library copies them into its job table during the call.
    hbuf = ctypes.create_string_buffer(b"".join(heads))
    hptrs, hpos = [], ctypes.addressof(hbuf)
    for h in heads:
        hptrs.append(hpos)
        hpos += len(h)
    _lib.check(
        _lib.lib.zn_compress_batch(
            nj, _ptr_array(ctypes.c_void_p, [x.data_ptr() for x in xs]), n_arr, k, int(reorder),
            _ptr_array(ctypes.c_void_p, hptrs),
            _ptr_array(ctypes.c_int, [len(h) for h in heads]), chunk_bytes, sub_chunks, float(threshold),
            _ptr_array(ctypes.c_void_p, [out.data_ptr() + o for o in offs]),
            _ptr_array(ctypes.c_int64, caps), sizes.data_ptr(), temp.data_ptr(), tb, _stream(device),
        ),
        "zn_compress_batch",
    )
    return out, offs, sizes, temp, fields


def decompress_tensors(
    blobs: list[torch.Tensor],
    *,
    compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = False,
    out: list[torch.Tensor | None] | None = None,
) -> list[torch.Tensor]:
    """decompress_tensor over a list of blobs, with one kernel launch per stage for each batch of
    blobs of an element size (batches of about _DEVICE_BATCH_BYTES, or _PIPELINE_BYTES for host
    blobs, launched while the host prepares the next).  Decoding errors are reported by
    last_decode_status().  Stored-path tensors of up to _TINY_BYTES decoded on the GPU are views
    into one buffer per call (one allocation instead of one per small tensor).

    `out`, if given, has one entry per blob: None (allocate, as above) or the caller's tensor to
    decode into, with decompress_tensor's rules for `out` (on the call's compute device without
    readback_to_cpu); the returned list then holds those tensors.  Blobs are checked as the list is
    read, so an invalid blob raises after the batches before it may have been launched (their
    results are dropped)."""
    compute_device = _check_device(compute_device)
    if out is not None and len(out) != len(blobs):
        raise ValueError("out must have one entry per blob")
    dest = list(out) if out is not None else [None] * len(blobs)
    outs: list[torch.Tensor | None] = [None] * len(blobs)
    # Header fields, read as the list is walked: unchanged GPU blobs made by this module carry
    # theirs (_remember); the other GPU blobs' headers come to the host in one copy per device when
    # the first of them is reached (prefixes[i] = (buffer, offset, length)); CPU blobs are read in
    # place.
    prefixes: list[tuple[memoryview, int, int] | None] = [None] * len(blobs)
    plen_max = _FIXED.size + 8 * _MAX_NDIM

    def fetch_prefixes(i: int) -> None:
        """The prefixes of blob i and of every later GPU blob on its device without a record."""
        dev = blobs[i].device
        idx = [j for j in range(i, len(blobs))
               if prefixes[j] is None and blobs[j].is_cuda and blobs[j].device == dev
               and blobs[j].dtype == torch.uint8 and blobs[j].dim() == 1
               and (j == i or _known_header(blobs[j]) is None)]
        plens = [min(blobs[j].numel(), plen_max) for j in idx]
        flat, offs = _gather_prefixes(dev, [blobs[j] for j in idx], plens)
        for j, o, p in zip(idx, offs, plens):
            prefixes[j] = (flat, o, p)

    def header(i: int, blob: torch.Tensor) -> tuple:
        """(dtype, shape, flags, chunk_bytes, n_comp, n) of blob i; n_comp = -1: the device reads it."""
        h = _known_header(blob)
        if h is not None:
            dtype, shape, flags, chunk_bytes, n = h
            return dtype, shape, flags, chunk_bytes, -1, n
        if prefixes[i] is None:
            if blob.is_cuda:
                fetch_prefixes(i)
            else:
                p = min(blob.numel(), plen_max)
                prefixes[i] = (memoryview(blob[:p].contiguous().numpy()), 0, p)
        return _parse_header(*prefixes[i])

    small: list[tuple[int, torch.dtype, tuple[int, ...], int]] = []  # stored / empty, after the launches

    def decompress_small() -> None:
        """Stored blobs on the GPU decode into GPU tensors by one batched copy; the rest (CPU blobs,
        CPU outputs, empty tensors) take decompress_tensor."""
        srcs, dsts, sizes = [], [], []
        tiny: dict[torch.dtype, list] = {}  # outputs placed in one buffer per dtype below
        bdev = None  # the one device (index) whose stored blobs are batched
        if compute_device is None:
            cdi = None
        else:
            cdi = compute_device.index if compute_device.index is not None else torch.cuda.current_device()
        for i, dtype, shape, flags in small:
            b = blobs[i]
            header_size = _FIXED.size + 8 * len(shape)
            nbytes = math.prod(shape) * dtype.itemsize
            bi = b.get_device() if b.is_cuda else None
            d = dest[i]
            src = b.data_ptr() + header_size
            if (flags & _FLAG_STORED and bi is not None and not readback_to_cpu and 0 < nbytes <= _COPY_BATCH_MAX
                    and src % 8 == 0 and cdi in (None, bi) and bdev in (None, bi)
                    and (d is None or (d.is_cuda and d.get_device() == bi and d.data_ptr() % 8 == 0))):
                bdev = bi
                if b.numel() < header_size + nbytes:
                    raise ValueError("blob is truncated")
                srcs.append(src)
                sizes.append(nbytes)
                if d is None and nbytes <= _TINY_BYTES:
                    tiny.setdefault(dtype, []).append((i, shape, nbytes // dtype.itemsize, len(dsts)))
                    dsts.append(0)
                else:
                    y = torch.empty(shape, dtype=dtype, device=b.device) if d is None else d
                    dsts.append(y.data_ptr())
                    outs[i] = y
            else:
                outs[i] = decompress_tensor(b, compute_device=compute_device, readback_to_cpu=readback_to_cpu,
                                            out=d)
        if srcs:
            dev = torch.device("cuda", bdev)
            for dtype, group in tiny.items():
                # Each output is a view of its region (256-byte aligned) of one buffer, shaped in
                # place by resize_ (the storage stays): one tensor made per output.
                step = 256 // dtype.itemsize
                offs, pos = [], 0
                for _, _, numel, _ in group:
                    offs.append(pos)
                    pos += -(-numel // step) * step
                buf = torch.empty(pos, dtype=dtype, device=dev)
                base, isz = buf.data_ptr(), dtype.itemsize
                for v, o, (i, shape, _, j) in zip(_capacity_views(buf, offs), offs, group):
                    v.resize_(shape)
                    outs[i] = v
                    dsts[j] = base + o * isz
            with torch.cuda.device(dev):
                _copy_batch(dev, srcs, dsts, sizes)

    # Coded blobs are launched in batches as they are parsed, so that the GPU starts on the first
    # batch while the host prepares the next.  Host-resident blobs go up on a copy stream in
    # smaller batches, so that the upload of one batch overlaps the decoding of the previous one.
    device: torch.device | None = None
    stream = copy_in = status = None
    uploaded: list[torch.cuda.Event] = []
    pos = 0
    launched = 0  # sub-batches launched so far
    cur: dict[tuple[int, bool], tuple[list, int]] = {}

    def launch(k: int, reorder: bool, items: list) -> None:
        nonlocal copy_in, pos, launched
        launched += 1
        host = any(not blobs[i].is_cuda for i, _ in items)
        if host and copy_in is None:
            copy_in = _side_stream(device, 0)
        up = copy_in if host else stream
        with torch.cuda.stream(up) if host else contextlib.nullcontext():  # `stream` is current already
            xs = []
            dev = device.index
            for i, _ in items:
                x = blobs[i]
                if not x.is_cuda:
                    x = _upload(x.contiguous(), device)
                    if x.data_ptr() % 8:
                        x = x.clone()
                elif not (x.get_device() == dev and x.is_contiguous() and x.data_ptr() % 8 == 0):
                    x = x.to(device, non_blocking=True, memory_format=torch.contiguous_format).contiguous()
                    if x.data_ptr() % 8:
                        x = x.clone()
                xs.append(x)
            if host and any(blobs[i].is_pinned() for i, _ in items):
                ev = torch.cuda.Event()
                ev.record(up)
                uploaded.append(ev)
        if up is not stream:
            stream.wait_stream(up)
            for x in xs:
                x.record_stream(stream)
        ys, meta = [], []
        for i, (dtype, shape, chunk_bytes, n_comp, n) in items:
            y = dest[i] if dest[i] is not None and not readback_to_cpu else None
            ys.append(torch.empty(shape, dtype=dtype, device=device) if y is None else y)
            meta.append((n, len(shape), chunk_bytes, n_comp))
        nj = len(items)
        n_arr = _ptr_array(ctypes.c_int64, [m[0] for m in meta])
        c_arr = _ptr_array(ctypes.c_int64, [m[2] for m in meta])
        tb = int(_lib.lib.zn_decompress_batch_temp_bytes(nj, n_arr, k, c_arr))
        temp = torch.empty(max(tb, 1), dtype=torch.uint8, device=device)
        _lib.check(
            _lib.lib.zn_decompress_batch(
                nj, _ptr_array(ctypes.c_void_p, [x.data_ptr() for x in xs]),
                _ptr_array(ctypes.c_int64, [x.numel() for x in xs]), n_arr, k, int(reorder),
                _ptr_array(ctypes.c_int, [m[1] for m in meta]), c_arr,
                _ptr_array(ctypes.c_int64, [m[3] for m in meta]),
                _ptr_array(ctypes.c_void_p, [y.data_ptr() for y in ys]), status.data_ptr() + 4 * pos,
                temp.data_ptr(), tb, stream.cuda_stream,
            ),
            "zn_decompress_batch",
        )
        pos += nj
        for (i, _), y in zip(items, ys):
            outs[i] = y

    for i, blob in enumerate(blobs):
        if blob.dtype != torch.uint8 or blob.dim() != 1:
            raise ValueError("blob must be a 1-D uint8 tensor")
        dtype, shape, flags, chunk_bytes, n_comp, n = header(i, blob)
        if dest[i] is not None:
            _check_out(dest[i], dtype, shape, readback_to_cpu)
            if dest[i].is_cuda and dest[i].device != _gpu(blob, compute_device):
                raise ValueError("out is not on the compute device")
        if flags & _FLAG_STORED or n == 0:
            small.append((i, dtype, shape, flags))
            continue
        if math.prod(shape) != n or chunk_bytes <= 0:
            raise ValueError("not a cuzipnn blob")
        k = dtype.itemsize
        if n_comp >= 0:
            nch = -(-n // chunk_bytes)
            _, _, data_off = _layout(len(shape), k * nch, n_comp)
            if blob.numel() < data_off:
                raise ValueError("blob is truncated")
        if device is None:
            device = _gpu(blob, compute_device)
            stream = torch.cuda.current_stream(device)
            # One status word per coded blob of this call, each set by the decoder (last_decode_status
            # ORs the words of the coded blobs).
            status = torch.empty(len(blobs), dtype=torch.int32, device=device)
        key = (k, bool(flags & _FLAG_REORDER))
        items, nbytes = cur.get(key, ([], 0))
        items.append((i, (dtype, shape, chunk_bytes, n_comp, n)))
        nbytes += blob.numel()
        limit = _PIPELINE_BYTES if not blob.is_cuda else _DEVICE_BATCH_BYTES
        if nbytes >= _batch_limit(limit, launched):
            with torch.cuda.device(device):
                launch(key[0], key[1], items)
            items, nbytes = [], 0
        cur[key] = (items, nbytes)
    if device is None:
        decompress_small()
        return outs  # type: ignore[return-value]
    with torch.cuda.device(device):
        for (k, reorder), (items, _) in cur.items():
            if items:
                launch(k, reorder, items)
        _set_status(device, status[:pos])
        decompress_small()
        for ev in uploaded:
            ev.synchronize()
        if readback_to_cpu:
            for i, y in enumerate(outs):
                if y is not None and y.is_cuda:
                    host = dest[i] if dest[i] is not None else (
                        _host_empty(y.numel() * y.element_size()).view(y.dtype).view_as(y))
                    _download(y, host)
                    outs[i] = host
    return outs  # type: ignore[return-value]


def _gather_prefixes(device: torch.device, bs: list[torch.Tensor], plen: list[int]) -> tuple[memoryview, list[int]]:
    """The first plen[j] bytes of each device blob, in one device-to-host copy: one host buffer and
    the offset of each prefix in it.  A batched device copy into one buffer when every blob is
    8-byte aligned, else a concatenation."""
    with torch.cuda.device(device):
        step = _FIXED.size + 8 * _MAX_NDIM
        ptrs = [b.data_ptr() for b in bs]
        if all(p % 8 == 0 for p in ptrs) and all(plen):
            buf = torch.empty(len(bs) * step, dtype=torch.uint8, device=device)
            base = buf.data_ptr()
            _copy_batch(device, ptrs, list(range(base, base + len(bs) * step, step)), plen)
            return memoryview(buf.cpu().numpy()), list(range(0, len(bs) * step, step))
        flat = memoryview(torch.cat([b[:p] for b, p in zip(bs, plen)]).cpu().numpy())
        offs, pos = [], 0
        for p in plen:
            offs.append(pos)
            pos += p
        return flat, offs


# Host copies between the GPU and pageable memory of at least _BOUNCE_MIN bytes run through two
# pinned bounce buffers of _BOUNCE_BYTES (per thread and device): the DMA of one piece overlaps the
# host copy of the previous one (PyTorch spreads a large host copy over its CPU threads, which also
# fault the destination's fresh pages in parallel).  A plain copy to or from pageable memory is
# staged by the driver one piece at a time on one thread.
_BOUNCE_BYTES = 1 << 25
_BOUNCE_MIN = 1 << 23
_BOUNCE = threading.local()


def _bounce(device: torch.device) -> tuple[list[torch.Tensor], list[torch.cuda.Event]]:
    cache = getattr(_BOUNCE, "by_dev", None)
    if cache is None:
        cache = _BOUNCE.by_dev = {}
    b = cache.get(device.index)
    if b is None:
        b = cache[device.index] = ([torch.empty(_BOUNCE_BYTES, dtype=torch.uint8, pin_memory=True) for _ in range(2)],
                                   [torch.cuda.Event(), torch.cuda.Event()])
    return b


def _host_empty(size: int) -> torch.Tensor:
    """A pageable host buffer for a download: fresh pages for a bounced copy (which faults them in
    on many threads), pre-faulted ones for a plain copy."""
    return torch.empty(size, dtype=torch.uint8) if size >= _BOUNCE_MIN else _populated_empty(size)


def _download(src: torch.Tensor, dst: torch.Tensor) -> None:
    """Copy contiguous GPU tensor `src` into contiguous host tensor `dst` (same byte size) on the
    current stream; returns once dst holds the data."""
    s8, d8 = src.reshape(-1).view(torch.uint8), dst.reshape(-1).view(torch.uint8)
    n = s8.numel()
    if n < _BOUNCE_MIN or dst.is_pinned():
        d8.copy_(s8)
        return
    bufs, evs = _bounce(src.device)
    stream = torch.cuda.current_stream(src.device)
    prev = None
    for i, off in enumerate(range(0, n, _BOUNCE_BYTES)):
        j, m = i % 2, min(_BOUNCE_BYTES, n - off)
        evs[j].synchronize()  # the buffer's previous use (an upload of this thread) is done
        bufs[j][:m].copy_(s8[off : off + m], non_blocking=True)
        evs[j].record(stream)
        if prev is not None:
            pj, poff, pm = prev
            evs[pj].synchronize()
            d8[poff : poff + pm].copy_(bufs[pj][:pm])
        prev = (j, off, m)
    pj, poff, pm = prev
    evs[pj].synchronize()
    d8[poff : poff + pm].copy_(bufs[pj][:pm])


def _upload(src: torch.Tensor, device: torch.device) -> torch.Tensor:
    """A copy on `device` of contiguous host tensor `src`, enqueued on the current stream; src may
    be reused once this returns."""
    n = src.numel() * src.element_size()
    if n < _BOUNCE_MIN or src.is_pinned():
        return src.to(device, non_blocking=True)
    dst = torch.empty(src.shape, dtype=src.dtype, device=device)
    s8, d8 = src.reshape(-1).view(torch.uint8), dst.reshape(-1).view(torch.uint8)
    bufs, evs = _bounce(device)
    stream = torch.cuda.current_stream(device)
    for i, off in enumerate(range(0, n, _BOUNCE_BYTES)):
        j, m = i % 2, min(_BOUNCE_BYTES, n - off)
        evs[j].synchronize()  # the DMA that last read this buffer is done
        bufs[j][:m].copy_(s8[off : off + m])
        d8[off : off + m].copy_(bufs[j][:m], non_blocking=True)
        evs[j].record(stream)
    return dst


def _populated_empty(size: int, *, pin_memory: bool = False) -> torch.Tensor:
    """A CPU buffer whose pages are already faulted in (_codec.py:545-550)."""
    t = torch.empty(size, dtype=torch.uint8, pin_memory=pin_memory)
    if not pin_memory:
        # There are other page sizes, but all >= 4KB.
        t[::4096].fill_(1)
    return t
