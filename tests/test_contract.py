"""The reference's API contract (its tests/test_roundtrip.py inventory) on the CUDA path.

Round trips must be bit-exact (compared through integer views, so NaN payloads count), blobs
deterministic, and every keyword argument must behave as in src/cuzipnn/_codec.py.
"""

import ctypes
import math
import zlib

import pytest
import torch

import cuzipnn_b200 as z
from cuzipnn_b200 import _codec, _kernels

pytestmark = pytest.mark.gpu

CHUNK = 4096  # small chunks: moderate tensors span many chunks
ALL_RAW = 1e-9  # every chunk budget truncates to 0 bytes
INT_OF = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}
FLOATS = [torch.bfloat16, torch.float16, torch.float32, torch.float64, torch.float8_e4m3fn, torch.float8_e5m2]
OTHERS = [torch.bool, torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64, torch.complex64,
          torch.uint16, torch.uint32, torch.uint64]


def bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(INT_OF[t.element_size()])


def weights(dtype, n, device="cuda"):
    return (torch.randn(n, device=device) * 0.02).to(dtype)


def roundtrip(x, **kw):
    kw.setdefault("min_compress_bytes", 0)
    blob = z.compress_tensor(x, **kw)
    assert blob.device.type == "cpu" and blob.dtype == torch.uint8 and blob.dim() == 1
    assert blob.is_pinned() == kw.get("pin_memory", False)
    y = z.decompress_tensor(blob)
    assert y.is_cuda and y.dtype == x.dtype and y.shape == x.shape
    assert torch.equal(bits(y), bits(x.cuda()))
    return blob


def is_stored(blob) -> bool:
    return bool(int(blob[7]) & _codec._FLAG_STORED)


@pytest.mark.parametrize("dtype", FLOATS)
@pytest.mark.parametrize("n", [1, 7, CHUNK - 1, CHUNK, CHUNK + 1, 10 * CHUNK + 13, 1_000_003])
def test_float_sizes(dtype, n):
    roundtrip(weights(dtype, n), chunk_bytes=CHUNK)


@pytest.mark.parametrize("dtype", OTHERS)
def test_other_dtypes(dtype):
    if dtype == torch.bool:
        x = torch.rand(100_003, device="cuda") < 0.3
    elif dtype == torch.complex64:
        x = torch.randn(100_003, dtype=dtype, device="cuda")
    elif dtype in (torch.uint16, torch.uint32, torch.uint64):
        x = torch.randint(0, 200, (100_003,), device="cuda").to(dtype)
    else:
        x = torch.randint(-100, 100, (100_003,), device="cuda").to(dtype)
    roundtrip(x, chunk_bytes=CHUNK)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_pinned_output(dtype):
    roundtrip(weights(dtype, 10 * CHUNK + 13), chunk_bytes=CHUNK, pin_memory=True)
    roundtrip(torch.empty(0, dtype=dtype), pin_memory=True)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_default_chunks_compress(dtype):
    blob = roundtrip(weights(dtype, 5_000_000))
    assert blob.numel() < 0.95 * 5_000_000 * torch.finfo(dtype).bits // 8


@pytest.mark.parametrize("shape", [(), (0,), (3, 0, 5), (1,), (17, 33, 5), (2, 3, 4, 5, 6)])
def test_shapes(shape):
    roundtrip(weights(torch.bfloat16, math.prod(shape)).reshape(shape), chunk_bytes=CHUNK)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_special_values(dtype):
    fi = torch.finfo(dtype)
    vals = [0.0, -0.0, math.inf, -math.inf, math.nan, fi.max, -fi.max, fi.tiny, fi.tiny / 4, -fi.tiny / 8]
    roundtrip(torch.tensor(vals, dtype=dtype).repeat(1000).cuda(), chunk_bytes=CHUNK)


@pytest.mark.parametrize("int_dtype,float_view", [(torch.int8, torch.float8_e5m2), (torch.int16, torch.bfloat16),
                                                  (torch.int32, torch.float32)])
def test_every_bit_pattern(int_dtype, float_view):
    info = torch.iinfo(int_dtype)
    b = torch.randint(info.min, info.max, (300_001,), dtype=int_dtype, device="cuda")
    blob = roundtrip(b.view(float_view), chunk_bytes=CHUNK)
    # Random bits are incompressible: everything is stored raw with little overhead.
    assert blob.numel() < b.numel() * b.element_size() * 1.01


def test_zeros_compress_well():
    blob = roundtrip(torch.zeros(1_000_000, dtype=torch.bfloat16, device="cuda"))
    assert blob.numel() < 0.1 * 2_000_000


def test_non_contiguous_input():
    x = weights(torch.bfloat16, 300 * 400).reshape(300, 400)
    roundtrip(x.t(), chunk_bytes=CHUNK)
    roundtrip(x[::3, 1::2], chunk_bytes=CHUNK)


def test_unaligned_fp8_view():
    roundtrip(weights(torch.float8_e4m3fn, 100_001)[3:], chunk_bytes=CHUNK)


def test_cpu_input_and_cpu_blob():
    x = weights(torch.bfloat16, 100_000, device="cpu")
    blob = z.compress_tensor(x, chunk_bytes=CHUNK)
    y = z.decompress_tensor(blob.cpu())
    assert y.is_cuda and torch.equal(bits(x), bits(y).cpu())


@pytest.mark.parametrize("n", [0, 100_000])
def test_decompress_to_cpu(n):
    x = weights(torch.bfloat16, n)
    blob = z.compress_tensor(x, chunk_bytes=CHUNK)
    for b in (blob, blob.cuda()):
        y = z.decompress_tensor(b, readback_to_cpu=True)
        assert y.device.type == "cpu" and y.shape == x.shape
        assert torch.equal(bits(y), bits(x).cpu())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int8, torch.complex64])
@pytest.mark.parametrize("min_compress_bytes", [0, _codec.DEFAULT_MIN_COMPRESS_BYTES])
def test_zero_dim_to_cpu(dtype, min_compress_bytes):
    x = torch.tensor(1.5, device="cuda").to(dtype)
    blob = z.compress_tensor(x, min_compress_bytes=min_compress_bytes)
    assert is_stored(blob) == (min_compress_bytes > 0)
    for b in (blob, blob.cuda()):
        y = z.decompress_tensor(b, readback_to_cpu=True)
        assert y.device.type == "cpu" and y.dtype == dtype and y.shape == ()
        assert torch.equal(bits(y), bits(x).cpu())


def test_unaligned_blob_view():
    x = weights(torch.float32, 100_000)
    blob = z.compress_tensor(x, chunk_bytes=CHUNK)
    padded = torch.empty(blob.numel() + 3, dtype=torch.uint8, device="cuda")
    padded[3:] = blob
    assert torch.equal(bits(z.decompress_tensor(padded[3:])), bits(x))


def test_deterministic():
    x = weights(torch.bfloat16, 1_000_003)
    assert torch.equal(z.compress_tensor(x, chunk_bytes=CHUNK), z.compress_tensor(x, chunk_bytes=CHUNK))


def test_stale_device_memory_does_not_leak():
    x = weights(torch.bfloat16, 4_000_003)
    blobs = []
    for fill in (0x00, 0xA5):
        torch.cuda.empty_cache()
        torch.full((256 << 20,), fill, dtype=torch.uint8, device="cuda")  # freed dirty into the cache
        blobs.append(z.compress_tensor(x, chunk_bytes=CHUNK))
    assert torch.equal(*blobs)


def test_bytes_past_view_do_not_leak():
    base = torch.randint(0, 256, (CHUNK + 16,), dtype=torch.uint8, device="cuda")
    x = base[: CHUNK + 3]
    blobs = []
    for fill in (0x00, 0xA5):
        base[CHUNK + 3 :] = fill
        blobs.append(roundtrip(x, chunk_bytes=CHUNK, passthrough_threshold=ALL_RAW))
    assert torch.equal(*blobs)


def test_non_default_stream():
    x = weights(torch.bfloat16, 1_000_003)
    ref = z.compress_tensor(x, chunk_bytes=CHUNK)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        s.wait_stream(torch.cuda.default_stream())
        blob = z.compress_tensor(x, chunk_bytes=CHUNK)
        y = z.decompress_tensor(blob)
    torch.cuda.synchronize()
    assert torch.equal(blob, ref) and torch.equal(bits(y), bits(x))


def test_tiny_threshold_stores_everything_raw():
    blob = roundtrip(weights(torch.bfloat16, 100_000), chunk_bytes=CHUNK, passthrough_threshold=ALL_RAW)
    assert blob.numel() >= 200_000


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("sub_chunk_bytes", [1, 1000, 8 * 1024, 32 * 1024, 1 << 30])
def test_sub_chunk_bytes(dtype, sub_chunk_bytes):
    # decompress_tensor needs no matching argument: the payload records its sub-chunk count.
    roundtrip(weights(dtype, 1_000_003), sub_chunk_bytes=sub_chunk_bytes)


def test_larger_sub_chunks_compress_better():
    x = weights(torch.bfloat16, 2_000_000)
    small, large = (z.compress_tensor(x, sub_chunk_bytes=s).numel() for s in (2 << 10, 32 << 10))
    assert large < small


def mixed_int8(n_chunks):
    parts = [torch.randint(0, 256, (CHUNK,), dtype=torch.uint8) if i % 2 == 0 else torch.zeros(CHUNK, dtype=torch.uint8)
             for i in range(n_chunks)]
    return torch.cat(parts + [torch.randint(0, 256, (13,), dtype=torch.uint8)]).cuda()


@pytest.mark.parametrize("layout", ["offset", "strided", "offset_in_misaligned_storage"])
def test_unaligned_cpu_blob_view(layout):
    x = mixed_int8(7)
    blob = z.compress_tensor(x, chunk_bytes=CHUNK, min_compress_bytes=0)
    if layout == "offset":
        view = torch.cat([torch.zeros(3, dtype=torch.uint8), blob])[3:]
    elif layout == "strided":
        view = torch.stack([blob, blob], 1)[:, 0]
    else:
        buf = bytearray(blob.numel() + 4)
        torch.frombuffer(buf, dtype=torch.uint8)[4:].copy_(blob)
        view = torch.frombuffer(memoryview(buf)[3:], dtype=torch.uint8)[1:]
    assert torch.equal(z.decompress_tensor(view), x)


def zipnn_planes(u: torch.Tensor, k: int, reorder: bool) -> torch.Tensor:
    """ZipNN's reorder and byte grouping, restated in torch (the reference's test helper
    restates ZipNN's data_manipulation_dtype{16,32}.c the same way)."""
    w = 8 * k
    v = u.to(torch.int64) & ((1 << w) - 1)
    if reorder:
        v = (((v >> (w - 9)) & 0xFF) << (w - 8)) | (((v >> (w - 1)) & 1) << (w - 9)) | (v & ((1 << (w - 9)) - 1))
    return torch.stack([((v >> (8 * b)) & 0xFF).to(torch.uint8) for b in range(k)])


@pytest.mark.parametrize("dtype,reorder", [(torch.bfloat16, True), (torch.float32, True), (torch.float16, False)])
def test_split_matches_zipnn(dtype, reorder):
    x = torch.randn(10_001, device="cuda").to(dtype)
    n, k = x.numel(), x.element_size()
    planar = torch.empty(k * n, dtype=torch.uint8, device="cuda")
    _kernels.split(x, planar, n, reorder)
    ref = zipnn_planes(x.cpu().view(INT_OF[k]), k, reorder)
    assert torch.equal(planar.view(k, n).cpu(), ref)
    if dtype == torch.bfloat16:  # ZipNN's 16-bit formula
        v = x.cpu().view(torch.int16).to(torch.int64) & 0xFFFF
        c = ((v << 1) & 0xFF00) | ((v >> 8) & 0x80) | (v & 0x7F)
        assert torch.equal(ref[1], (c >> 8).to(torch.uint8)) and torch.equal(ref[0], (c & 0xFF).to(torch.uint8))


@pytest.mark.parametrize("dtype,stride", [(torch.float32, 800_000_000), (torch.float32, 800_000_008),
                                          (torch.float64, 320_000_000), (torch.float64, 320_000_008)])
def test_split_large_stride(dtype, stride):
    # (K - 1) * stride >= 2**31: stream offsets must not wrap.
    x = torch.randn(4099, device="cuda").to(dtype)
    n, k = x.numel(), x.element_size()
    planar = torch.zeros(k * stride, dtype=torch.uint8, device="cuda")
    _kernels.split(x, planar, stride, False)
    ref = zipnn_planes(x.cpu().view(INT_OF[k]), k, False)
    for b in range(k):
        assert torch.equal(planar[b * stride : b * stride + n].cpu(), ref[b])
    del planar


def test_pinned_blob_reusable_after_return():
    x = weights(torch.bfloat16, 1_000_003)
    blob = z.compress_tensor(x, chunk_bytes=CHUNK, pin_memory=True)
    z.decompress_tensor(blob)
    torch.cuda._sleep(1 << 30)  # the upload is still queued when decompress_tensor returns
    y = z.decompress_tensor(blob)
    blob.zero_()
    assert torch.equal(bits(y), bits(x))


@pytest.mark.parametrize("dtype", FLOATS + OTHERS)
@pytest.mark.parametrize("shape", [(), (0,), (3, 0, 5), (1,), (7,), (17, 33, 5)])
def test_stored_roundtrip(dtype, shape):
    if dtype in (torch.uint16, torch.uint32, torch.uint64):
        x = torch.randint(0, 1000, shape, device="cuda").to(dtype)
    else:
        x = torch.randn(shape, device="cuda").to(dtype)
    nbytes = x.numel() * x.element_size()
    blob = roundtrip(x, min_compress_bytes=nbytes + 1)
    assert is_stored(blob) and blob.numel() == 24 + 8 * len(shape) + nbytes
    y = z.decompress_tensor(blob, readback_to_cpu=True)
    assert y.device.type == "cpu" and torch.equal(bits(y), bits(x.cpu()))


def test_stored_boundary():
    x = weights(torch.bfloat16, 1000)
    assert is_stored(z.compress_tensor(x, min_compress_bytes=2001))
    assert not is_stored(roundtrip(x, min_compress_bytes=2000))


def test_default_min_compress_bytes():
    small = weights(torch.bfloat16, _codec.DEFAULT_MIN_COMPRESS_BYTES // 2 - 1)
    large = weights(torch.bfloat16, _codec.DEFAULT_MIN_COMPRESS_BYTES // 2)
    assert is_stored(z.compress_tensor(small)) and not is_stored(z.compress_tensor(large))
    for x in (small, large):
        assert torch.equal(bits(z.decompress_tensor(z.compress_tensor(x))), bits(x))


def test_stored_non_contiguous_and_cpu_input():
    x = weights(torch.float32, 30 * 40).reshape(30, 40)
    for v in (x.t(), x[::3, 1::2], x.cpu().t()):
        blob = z.compress_tensor(v, pin_memory=True)
        assert is_stored(blob) and blob.is_pinned()
        assert torch.equal(bits(z.decompress_tensor(blob)), bits(v.cuda()))
        assert torch.equal(bits(z.decompress_tensor(blob.cuda())), bits(v.cuda()))


@pytest.mark.parametrize("device", ["cpu", "cuda"])
def test_stored_unaligned_blob_view(device):
    x = weights(torch.float64, 101)
    blob = z.compress_tensor(x)
    padded = torch.empty(blob.numel() + 3, dtype=torch.uint8, device=device)
    padded[3:] = blob
    assert torch.equal(bits(z.decompress_tensor(padded[3:])), bits(x))


def test_stored_truncated():
    blob = z.compress_tensor(weights(torch.bfloat16, 100))
    assert is_stored(blob)
    with pytest.raises(ValueError, match="truncated"):
        z.decompress_tensor(blob[:-1])


def crc_ref(t, chunk=_codec.DEFAULT_CHECKSUM_CHUNK_BYTES):
    t = t.detach().cpu().contiguous()
    b = ctypes.string_at(t.data_ptr(), t.numel() * t.element_size())
    return [zlib.crc32(b[i : i + chunk]) for i in range(0, len(b), chunk)]


@pytest.mark.parametrize(
    "make",
    [
        pytest.param(lambda: weights(torch.bfloat16, 1_000_003), id="bf16"),
        pytest.param(lambda: weights(torch.float32, 300_001).cpu(), id="fp32-cpu"),
        pytest.param(lambda: mixed_int8(7), id="int8-mixed"),
        pytest.param(lambda: weights(torch.float16, 1000).reshape(10, 100).t(), id="fp16-t"),
        pytest.param(lambda: torch.empty(3, 0, 5, device="cuda"), id="empty"),
    ],
)
@pytest.mark.parametrize("min_compress_bytes", [0, 1 << 30])
@pytest.mark.parametrize("checksum_chunk_bytes", [8, 1000, 16 * 1024, 1 << 30])
def test_crc32_matches_zlib(make, min_compress_bytes, checksum_chunk_bytes):
    x = make()
    kw = {"chunk_bytes": CHUNK, "min_compress_bytes": min_compress_bytes}
    blob, crc = z.compress_tensor_with_crc32(x, checksum_chunk_bytes=checksum_chunk_bytes, **kw)
    assert torch.equal(blob, z.compress_tensor(x, **kw))
    assert is_stored(blob) == (min_compress_bytes > 0)
    assert crc.dtype == torch.uint32 and crc.device.type == "cpu" and crc.dim() == 1
    assert crc.tolist() == crc_ref(blob, checksum_chunk_bytes)


def test_crc32_default_chunk():
    blob, crc = z.compress_tensor_with_crc32(weights(torch.bfloat16, 1_000_003))
    assert crc.numel() == math.ceil(blob.numel() / (16 * 1024)) > 1
    assert crc.tolist() == crc_ref(blob)


def test_hash_blob_matches_checksums():
    x = weights(torch.bfloat16, 1_000_003)
    blob, crc = z.compress_tensor_with_crc32(x, chunk_bytes=CHUNK, pin_memory=True)
    assert blob.is_pinned()
    padded = torch.empty(blob.numel() + 3, dtype=torch.uint8, device="cuda")
    padded[3:] = blob
    for view in (blob, blob.cuda(), padded[3:], torch.stack([blob, blob], 1)[:, 0]):
        assert torch.equal(z.hash_tensor_with_crc32(view), crc)
    assert torch.equal(bits(z.decompress_tensor(blob)), bits(x))


def test_hash_tensor():
    x = weights(torch.float32, 30 * 40).reshape(30, 40)
    for t in (x, x.t(), x.cpu().t(), x[::3, 1::2], torch.tensor(1.5), torch.empty(0)):
        crc = z.hash_tensor_with_crc32(t, checksum_chunk_bytes=1000)
        assert crc.dtype == torch.uint32 and crc.device.type == "cpu"
        assert crc.tolist() == crc_ref(t, 1000)


def test_crc32_localizes_corruption():
    blob, crc = z.compress_tensor_with_crc32(weights(torch.bfloat16, 1_000_003), chunk_bytes=CHUNK)
    for pos in (0, 16 * 1024 - 1, 16 * 1024, blob.numel() // 2, blob.numel() - 1):
        bad = blob.clone()
        bad[pos] ^= 1
        diff = (z.hash_tensor_with_crc32(bad).to(torch.int64) != crc.to(torch.int64)).nonzero()
        assert diff.view(-1).tolist() == [pos // (16 * 1024)]


def test_crc32_non_default_stream():
    x = weights(torch.bfloat16, 1_000_003)
    ref = z.compress_tensor_with_crc32(x, chunk_bytes=CHUNK)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        s.wait_stream(torch.cuda.default_stream())
        blob, crc = z.compress_tensor_with_crc32(x, chunk_bytes=CHUNK)
        assert torch.equal(z.hash_tensor_with_crc32(blob), crc)
    assert torch.equal(blob, ref[0]) and torch.equal(crc, ref[1])


@pytest.mark.parametrize("n", [0, 7, 100_000])
@pytest.mark.parametrize("cpu_input", [False, True])
def test_no_readback(n, cpu_input):
    x = weights(torch.bfloat16, n, device="cpu" if cpu_input else "cuda")
    kw = {"chunk_bytes": CHUNK}
    ref, ref_crc = z.compress_tensor_with_crc32(x, **kw)
    blob = z.compress_tensor(x, readback_to_cpu=False, **kw)
    gblob, crc = z.compress_tensor_with_crc32(x, readback_to_cpu=False, **kw)
    for t in (blob, gblob, crc):
        assert t.is_cuda and t.device.index == torch.cuda.current_device()
    assert torch.equal(blob.cpu(), ref) and torch.equal(gblob.cpu(), ref)
    assert torch.equal(crc.cpu(), ref_crc)
    h = z.hash_tensor_with_crc32(ref, readback_to_cpu=False)
    assert h.is_cuda and torch.equal(h.cpu(), ref_crc)
    y = z.decompress_tensor(ref)
    assert y.is_cuda and torch.equal(bits(y), bits(x.cuda()))
    for b in (ref, blob):
        y = z.decompress_tensor(b, readback_to_cpu=True, compute_device="cuda")
        assert not y.is_cuda and torch.equal(bits(y), bits(x.cpu()))


def test_compute_device():
    x = weights(torch.bfloat16, 100_000, device="cpu")
    dev = f"cuda:{torch.cuda.current_device()}"
    blob, crc = z.compress_tensor_with_crc32(x, compute_device=dev, readback_to_cpu=False)
    assert str(blob.device) == dev and str(crc.device) == dev
    assert str(z.hash_tensor_with_crc32(x, compute_device=dev, readback_to_cpu=False).device) == dev
    assert str(z.decompress_tensor(blob.cpu(), compute_device=dev).device) == dev
