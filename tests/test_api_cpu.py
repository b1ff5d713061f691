"""Host-side behaviour that needs no GPU: the C ABI loads and exports what include/*.h declares,
argument checks raise what the reference raises (src/cuzipnn/_codec.py:243-262, :420-443), and
the stored path (no GPU work with readback_to_cpu) matches the oracle byte for byte."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

import cuzipnn_b200 as z
from cuzipnn_b200 import _codec, _lib
from oracle import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in os.listdir(os.path.join(REPO, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(REPO, "include", fn)).read()
            names += re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(zn_[a-z_0-9]+)\s*\(", text, re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 18
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name


def test_abi_host_queries():
    assert _lib.lib.zn_version() == _lib.ABI_VERSION
    assert _lib.lib.zn_ans_max_compressed_chunk_bytes(131072, 16) >= 2 * 131072
    assert _lib.lib.zn_ans_max_compressed_chunk_bytes(131072, 3) == -1
    assert _lib.lib.zn_compress_bound(0, 2, 1, 4096) == 32
    assert _lib.lib.zn_compress_temp_bytes(100_000, 2, 4096, 5) == 0  # not a power of two


def test_abi_rejects_bad_arguments_without_a_gpu():
    # Invalid arguments are refused before any CUDA call.
    rc = _lib.lib.zn_compress(None, 10, 3, 0, b"\0" * 24, 24, 4096, 16, 0.95, None, 0, None, None, 0, None)
    assert rc == _lib.ZN_ERR_INVALID and b"bad arguments" in _lib.lib.zn_last_error()
    assert _lib.lib.zn_split(None, 10, 2, 1, None, 5, None) == _lib.ZN_ERR_INVALID
    assert _lib.lib.zn_crc32(None, 10, 0, None, None, 0, None) == _lib.ZN_ERR_INVALID
    assert _lib.lib.zn_decompress(None, 0, 5, 3, 0, 1, 4096, 0, None, None, None, 0, None) == _lib.ZN_ERR_INVALID


def w(n, dtype=torch.bfloat16):
    return (torch.randn(n) * 0.02).to(dtype)


@pytest.mark.parametrize("thr", [0.0, -0.5, 1.01])
def test_bad_threshold(thr):
    with pytest.raises(ValueError, match="passthrough_threshold"):
        z.compress_tensor(w(100), passthrough_threshold=thr)


def test_bad_sub_chunk_bytes():
    with pytest.raises(ValueError, match="sub_chunk_bytes"):
        z.compress_tensor(w(100), sub_chunk_bytes=0)


@pytest.mark.parametrize("chunk", [0, 12, -8, (1 << 24) + 8])
def test_bad_chunk_bytes(chunk):
    with pytest.raises(ValueError, match="chunk_bytes"):
        z.compress_tensor(w(100), chunk_bytes=chunk)


def test_bad_min_compress_bytes():
    with pytest.raises(ValueError, match="min_compress_bytes"):
        z.compress_tensor(w(100), min_compress_bytes=-1)


@pytest.mark.parametrize("seg", [0, -1])
def test_bad_checksum_chunk_bytes(seg):
    with pytest.raises(ValueError, match="checksum_chunk_bytes"):
        z.compress_tensor_with_crc32(w(100), checksum_chunk_bytes=seg)
    with pytest.raises(ValueError, match="checksum_chunk_bytes"):
        z.hash_tensor_with_crc32(w(100), checksum_chunk_bytes=seg)


def test_pin_memory_requires_readback():
    with pytest.raises(ValueError, match="pin_memory"):
        z.compress_tensor(w(100), pin_memory=True, readback_to_cpu=False)


@pytest.mark.parametrize("device", ["cpu", torch.device("meta")])
def test_bad_compute_device(device):
    x = w(100)
    blob = z.compress_tensor(x)
    for f in (z.compress_tensor, z.compress_tensor_with_crc32, z.hash_tensor_with_crc32):
        with pytest.raises(ValueError, match="compute_device"):
            f(x, compute_device=device)
    with pytest.raises(ValueError, match="compute_device"):
        z.decompress_tensor(blob, compute_device=device)


def test_unsupported_dtype_and_rank():
    with pytest.raises(TypeError):
        z.compress_tensor(torch.zeros(4, dtype=torch.complex128))
    with pytest.raises(ValueError, match="dimensions"):
        z.compress_tensor(torch.zeros([1] * 65))


def test_bad_blob():
    with pytest.raises(ValueError):
        z.decompress_tensor(torch.zeros(64, dtype=torch.uint8))
    with pytest.raises(ValueError, match="1-D uint8"):
        z.decompress_tensor(torch.zeros(2, 32, dtype=torch.uint8))
    with pytest.raises(ValueError, match="too short"):
        z.decompress_tensor(torch.zeros(5, dtype=torch.uint8))


def test_reference_v2_blob_is_rejected(golden):
    with pytest.raises(ValueError, match="not a cuzipnn blob"):
        z.decompress_tensor(torch.from_numpy(golden["blob/bf16_4k/blob"].copy()))


def test_sub_chunk_known_answers():
    assert _codec._sub_chunks(128 << 10, 8 << 10) == 16
    assert _codec._sub_chunks(128 << 10, 7 << 10) == 32
    assert _codec._sub_chunks(16 << 10, 8 << 10) == 4
    assert _codec._sub_chunks(1 << 24, 1) == 64
    for c in (8, 1000, 4096, 1 << 17):
        for s in (1, 7, 1000, 8192, 1 << 30):
            assert _codec._sub_chunks(c, s) == O.sub_chunks(c, s)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int8, torch.complex64, torch.bool,
                                   torch.float8_e5m2, torch.uint64])
@pytest.mark.parametrize("shape", [(), (0,), (3, 0, 5), (7,), (17, 33, 5)])
def test_stored_path_on_host_matches_oracle(dtype, shape):
    """Stored blobs never touch the GPU with readback_to_cpu; they equal the oracle's and decode
    back on the host."""
    x = torch.randint(0, 100, shape).to(dtype) if dtype in (torch.uint64, torch.bool) else torch.randn(shape).to(dtype)
    nbytes = x.numel() * x.element_size()
    blob = z.compress_tensor(x, min_compress_bytes=nbytes + 1)
    raw = x.contiguous().reshape(-1).view(torch.uint8).numpy() if nbytes else np.zeros(0, np.uint8)
    ref = O.compress(raw, x.shape, str(x.dtype).split(".")[-1], min_compress_bytes=nbytes + 1)
    assert blob.numpy().tobytes() == ref
    y = z.decompress_tensor(blob, readback_to_cpu=True)
    assert y.dtype == x.dtype and y.shape == x.shape
    assert y.reshape(-1).view(torch.uint8).numpy().tobytes() == raw.tobytes()


def test_stored_crc_on_host():
    x = w(1000)
    blob, crc = z.compress_tensor_with_crc32(x, checksum_chunk_bytes=100)
    assert crc.tolist() == O.crc32_segments(blob.numpy(), 100).tolist()


def test_trimmed_views_carry_the_records_remember_makes():
    """The batched calls' blob views (capacity views of one buffer, trimmed in place) hold exactly
    their bytes and the same header records _remember computes from the views themselves; a later
    in-place write to any view of the buffer voids every record."""
    from cuzipnn_b200 import _codec as C

    out = torch.arange(5000, dtype=torch.int64).to(torch.uint8)
    offs, sizes = [0, 1024, 2048, 4096], [1000, 17, 2048, 904]
    fields = [(torch.bfloat16, (3, 4), 1, 131072, 12), (torch.float32, (5,), 0, 131072, 5),
              (torch.uint8, (2048,), 2, 0, 2048), (torch.float16, (), 0, 4096, 1)]
    views = C._capacity_views(out, offs)
    assert [v.numel() for v in views] == [1024, 1024, 2048, 904]
    C._trim_and_remember(out, views, sizes, offs, fields)
    for v, o, n, f in zip(views, offs, sizes, fields):
        assert v.numel() == n and v.is_contiguous()
        assert torch.equal(v, out[o : o + n])
        rec = v._zn_header
        C._remember(v, *f)
        assert rec == v._zn_header
        assert C._known_header(v) is None  # a CPU tensor: records only apply to GPU blobs
    views[1].add_(0)  # in place: the shared version counter moves for every view
    assert all(v._zn_header[0] != v._version for v in views)
