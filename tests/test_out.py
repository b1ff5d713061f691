"""decompress_tensor(out=...) and decompress_tensors(out=[...]): decoding straight into the caller's
storage (the reference allocates its result on every call, src/cuzipnn/_codec.py:463, :472).

The argument checks and the stored path run on the CPU (a stored blob needs no GPU); the GPU tests
check that coded, stored and empty tensors decode bit-exactly into the caller's tensor, which the
call returns (same storage)."""

import pytest
import torch

import cuzipnn_b200 as z


def _bits(t):
    t = t.contiguous().view(-1)
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


def test_stored_blob_into_cpu_out():
    x = torch.arange(100, dtype=torch.float32).reshape(10, 10)
    blob = z.compress_tensor(x)  # 400 bytes < min_compress_bytes: the stored path, no GPU
    dst = torch.full((10, 10), -1.0)
    y = z.decompress_tensor(blob, readback_to_cpu=True, out=dst)
    assert y.data_ptr() == dst.data_ptr() and torch.equal(dst, x)


@pytest.mark.parametrize("bad,err", [
    (torch.empty(10, 10, dtype=torch.float64), TypeError),
    (torch.empty(100), ValueError),
    (torch.empty(10, 20)[:, :10], ValueError),
])
def test_out_mismatch_raises(bad, err):
    blob = z.compress_tensor(torch.zeros(10, 10))
    with pytest.raises(err):
        z.decompress_tensor(blob, readback_to_cpu=True, out=bad)
    with pytest.raises(err):
        z.decompress_tensors([blob], readback_to_cpu=True, out=[bad])


def test_out_list_length():
    blob = z.compress_tensor(torch.zeros(4))
    with pytest.raises(ValueError):
        z.decompress_tensors([blob, blob], readback_to_cpu=True, out=[None])


def test_cpu_out_without_readback_raises():
    blob = z.compress_tensor(torch.zeros(4))
    with pytest.raises(ValueError):
        z.decompress_tensor(blob, out=torch.empty(4))


def _cases(device):
    g = torch.Generator(device=device).manual_seed(3)
    coded = (torch.randn(1000, 777, generator=g, device=device) * 0.02).to(torch.bfloat16)
    coded32 = torch.randn(300_001, generator=g, device=device)
    stored = torch.randn(3, 5, generator=g, device=device).to(torch.float16)
    big_stored = torch.randn(70_000, generator=g, device=device)  # stored, above the tiny size
    empty = torch.empty(0, 4, dtype=torch.bfloat16, device=device)
    return [coded, coded32, stored, big_stored, empty]


@pytest.mark.gpu
def test_decompress_tensor_into_gpu_out():
    for x in _cases("cuda"):
        blob = z.compress_tensor(x, readback_to_cpu=False, min_compress_bytes=300_000)
        dst = torch.full_like(x, 7) if x.numel() else torch.empty_like(x)
        y = z.decompress_tensor(blob, out=dst)
        torch.cuda.synchronize()
        assert y.data_ptr() == dst.data_ptr() and y.shape == x.shape
        assert torch.equal(_bits(dst), _bits(x))
        assert z.last_decode_status() == 0
        # From a CPU blob into a GPU tensor, and into a CPU tensor with readback_to_cpu.
        cblob = blob.cpu()
        dst2 = torch.zeros_like(x)
        assert z.decompress_tensor(cblob, out=dst2).data_ptr() == dst2.data_ptr()
        assert torch.equal(_bits(dst2), _bits(x))
        host = torch.zeros(x.shape, dtype=x.dtype)
        assert z.decompress_tensor(blob, readback_to_cpu=True, out=host).data_ptr() == host.data_ptr()
        assert torch.equal(_bits(host), _bits(x.cpu()))
    # An empty tensor with min_compress_bytes=0 has a header-only, non-stored blob.
    e = torch.empty(0, 3, device="cuda")
    blob = z.compress_tensor(e, readback_to_cpu=False, min_compress_bytes=0)
    dst = torch.empty_like(e)
    assert z.decompress_tensor(blob, out=dst) is dst


@pytest.mark.gpu
def test_decompress_tensors_into_gpu_out():
    xs = _cases("cuda")
    blobs = z.compress_tensors(xs, readback_to_cpu=False, min_compress_bytes=300_000)
    dsts = [torch.zeros_like(x) for x in xs]
    dsts[1] = None  # mixed: this one is allocated by the call
    ys = z.decompress_tensors(blobs, out=dsts)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    for x, y, d in zip(xs, ys, dsts):
        assert torch.equal(_bits(y), _bits(x))
        if d is not None:
            assert y.data_ptr() == d.data_ptr()
    hosts = [torch.zeros(x.shape, dtype=x.dtype) for x in xs]
    ys = z.decompress_tensors(blobs, readback_to_cpu=True, out=hosts)
    for x, y, h in zip(xs, ys, hosts):
        assert y.data_ptr() == h.data_ptr() and torch.equal(_bits(h), _bits(x.cpu()))


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_out_on_another_device_raises():
    x = torch.randn(100_000, device="cuda:0")
    blob = z.compress_tensor(x, readback_to_cpu=False)
    with pytest.raises(ValueError):
        z.decompress_tensor(blob, out=torch.empty(100_000, device="cuda:1"), compute_device="cuda:0")
    with pytest.raises(ValueError):
        z.decompress_tensors([blob], out=[torch.empty(100_000, device="cuda:1")])
