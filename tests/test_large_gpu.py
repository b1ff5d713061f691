"""Sizes past 32-bit limits on the GPU: a bf16 tensor of more than 2^31 elements, and a blob of
more than 2^32 bytes (incompressible bytes, every unit stored raw).  Round trips must be bit for
bit; the blob of the large bf16 tensor must equal, unit for unit, the blobs of its pieces (so the
64-bit offsets are checked against small, independently coded blobs).  About 25 GB of device
memory at the peak."""

import pytest
import torch

import cuzipnn_b200 as z
from cuzipnn_b200 import _shard

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.reshape(-1).view(torch.int16)


def test_bf16_more_than_2_to_31_elements():
    n = (1 << 31) + 12345
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    step = 1 << 28
    for i in range(0, n, step):  # in slices, to bound the float32 temporary
        m = min(step, n - i)
        x[i : i + m] = (torch.randn(m, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    blob = z.compress_tensor(x, readback_to_cpu=False)
    ratio = blob.numel() / (2 * n)
    assert 0.659 < ratio < 0.665, ratio
    # The last chunks of the blob equal the blob of the same elements coded alone.
    C = 131072
    nch = -(-n // C)
    j0 = nch - 3
    part = _shard.split_chunk_range(blob, j0, nch)
    assert torch.equal(part, z.compress_tensor(x[j0 * C :], readback_to_cpu=False, min_compress_bytes=0))
    y = z.decompress_tensor(blob)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    assert torch.equal(_bits(y), _bits(x))


def test_blob_larger_than_2_to_32_bytes():
    n = (1 << 32) + (1 << 29) + 77  # uniform bytes: every unit is stored raw
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randint(0, 256, (n,), generator=g, device="cuda", dtype=torch.uint8)
    blob = z.compress_tensor(x, readback_to_cpu=False)
    assert blob.numel() > (1 << 32)
    y = z.decompress_tensor(blob)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    assert torch.equal(y, x)
