"""Batched API (compress_tensors / decompress_tensors): every blob equals the per-tensor one, and
round trips are exact, across element sizes, stored and empty tensors and mixed devices."""

import pytest
import torch

import cuzipnn_b200 as z

pytestmark = pytest.mark.gpu

INT_OF = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def bits(t):
    return t.contiguous().view(INT_OF[t.element_size()])


def mixed_tensors():
    g = torch.Generator(device="cuda").manual_seed(7)
    def w(*shape, dtype=torch.bfloat16, scale=0.02):
        return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dtype)
    return [
        w(1000, 777),
        w(3584),                                  # stored (below min_compress_bytes)
        w(300, 301, dtype=torch.float32),
        torch.empty(0, 5, device="cuda", dtype=torch.bfloat16),
        w(257, 1024, dtype=torch.float16),
        (torch.randn(400, 513, device="cuda", generator=g) * 16).clamp(-448, 448).to(torch.float8_e4m3fn),
        w(1, 131072 * 3 + 5),
        torch.randint(-100, 100, (70_001,), device="cuda", generator=g).to(torch.int32),
        w(64, 64).t(),                            # non-contiguous
        w(5, 131072 + 64).cpu(),                  # CPU input
    ]


@pytest.mark.parametrize("readback", [True, False])
def test_batch_blobs_equal_single(readback):
    ts = mixed_tensors()
    batch = z.compress_tensors(ts, readback_to_cpu=readback)
    for t, b in zip(ts, batch):
        single = z.compress_tensor(t, readback_to_cpu=readback)
        assert b.is_cuda == (not readback) or b.numel() == single.numel()
        assert torch.equal(b.cpu(), single.cpu())
    ys = z.decompress_tensors(batch)
    assert z.last_decode_status() == 0
    for t, y in zip(ts, ys):
        assert y.dtype == t.dtype and y.shape == t.shape and y.is_cuda
        assert torch.equal(bits(y).cpu(), bits(t).cpu())


def test_batch_small_chunks_and_options():
    ts = mixed_tensors()
    kw = dict(chunk_bytes=4096, sub_chunk_bytes=1000, passthrough_threshold=0.5, min_compress_bytes=0)
    batch = z.compress_tensors(ts, **kw)
    for t, b in zip(ts, batch):
        assert torch.equal(b, z.compress_tensor(t, **kw))
    ys = z.decompress_tensors([b.cuda() for b in batch], readback_to_cpu=True)
    for t, y in zip(ts, ys):
        assert y.device.type == "cpu" and torch.equal(bits(y), bits(t).cpu())


def test_batch_many_tensors():
    g = torch.Generator(device="cuda").manual_seed(3)
    ts = [(torch.randn(int(s), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
          for s in torch.randint(40_000, 600_000, (150,), generator=torch.Generator().manual_seed(1))]
    batch = z.compress_tensors(ts, readback_to_cpu=False)
    ys = z.decompress_tensors(batch)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    for t, y in zip(ts, ys):
        assert torch.equal(bits(y), bits(t))
    assert torch.equal(batch[17].cpu(), z.compress_tensor(ts[17]))


@pytest.mark.parametrize("pin", [True, False])
def test_host_inputs_pipelined_in_sub_batches(monkeypatch, pin):
    """Host tensors go up in several sub-batches (copy stream overlapped with the kernels); blobs
    still equal the per-tensor ones, and host blobs decode back in sub-batches too."""
    from cuzipnn_b200 import _codec

    monkeypatch.setattr(_codec, "_PIPELINE_BYTES", 1 << 20)
    ts = [t.cpu() for t in mixed_tensors()]
    if pin:
        ts = [t.pin_memory() if t.is_contiguous() else t for t in ts]
    batch = z.compress_tensors(ts, readback_to_cpu=True, pin_memory=pin)
    for t, b in zip(ts, batch):
        assert not b.is_cuda
        assert torch.equal(b, z.compress_tensor(t))
    outs = z.decompress_tensors(batch)
    assert z.last_decode_status() == 0
    for t, y in zip(ts, outs):
        assert y.is_cuda and y.dtype == t.dtype and y.shape == t.shape
        assert torch.equal(bits(y.cpu()), bits(t))


def test_status_covers_every_group(monkeypatch):
    """A corrupt blob in the first element-size group is reported even when later groups decode
    cleanly (one status word per coded blob of the call)."""
    from cuzipnn_b200 import _codec

    monkeypatch.setattr(_codec, "_PIPELINE_BYTES", 1 << 20)
    ts = mixed_tensors()
    blobs = [b.clone() for b in z.compress_tensors(ts, readback_to_cpu=True)]
    bad = blobs[0]
    bad[40:44] = torch.tensor([0xFF, 0xFF, 0xFF, 0x7F], dtype=torch.uint8)  # stored size past the end
    z.decompress_tensors(blobs)
    assert z.last_decode_status() != 0
    z.decompress_tensors([b for i, b in enumerate(blobs) if i != 0])
    assert z.last_decode_status() == 0


def test_device_inputs_in_sub_batches(monkeypatch):
    """Device tensors in several launch batches (the GPU starts on one while the host prepares the
    next): blobs equal the per-tensor ones and decode back exactly."""
    from cuzipnn_b200 import _codec

    monkeypatch.setattr(_codec, "_DEVICE_BATCH_BYTES", 1 << 20)
    ts = mixed_tensors()
    batch = z.compress_tensors(ts, readback_to_cpu=False)
    for t, b in zip(ts, batch):
        assert torch.equal(b.cpu(), z.compress_tensor(t))
    outs = z.decompress_tensors(batch)
    assert z.last_decode_status() == 0
    for t, y in zip(ts, outs):
        assert torch.equal(bits(y.cpu()), bits(t.cpu()))


def test_many_sub_batches_keep_stream_order(monkeypatch):
    """A call split into many sub-batches (the first one small, each later one larger) on a
    non-default stream: inputs written in place on that stream just before the call and results
    read on it just after (no synchronization in between) round-trip exactly."""
    from cuzipnn_b200 import _codec

    monkeypatch.setattr(_codec, "_FIRST_BATCH", 1 << 16)
    monkeypatch.setattr(_codec, "_DEVICE_BATCH_BYTES", 1 << 20)
    g = torch.Generator(device="cuda").manual_seed(8)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        xs = [torch.randn(n, generator=g, device="cuda").to(torch.bfloat16) for n in (300_000, 200_001, 500_000, 90_000)]
        refs = [x.clone() for x in xs]
        for x in xs:
            x.mul_(0.02)  # in place, on s, right before the call
        blobs = z.compress_tensors(xs, readback_to_cpu=False)
        outs = z.decompress_tensors(blobs)
        ok = [torch.equal(o.view(torch.int16), (r * 0.02).view(torch.int16)) for o, r in zip(outs, refs)]
        for x in xs:
            x.zero_()  # the inputs are free for reuse once the call returns
    torch.cuda.synchronize()
    assert all(ok)
    assert z.last_decode_status() == 0


def test_large_pageable_host_copies():
    """Host blobs and host tensors above the bounce threshold (copies through the pinned bounce
    buffers, in pieces that do not divide the size) round-trip exactly, per tensor and batched,
    with the pinned path unchanged."""
    g = torch.Generator().manual_seed(12)
    x = (torch.randn(70 * 1024 * 1024 // 4 + 3, generator=g) * 0.02)  # ~70 MiB fp32 on the host
    y = (torch.randn(9_000_001, generator=g) * 0.02).to(torch.bfloat16)
    blob = z.compress_tensor(x)  # host input, host blob
    assert not blob.is_cuda and not blob.is_pinned()
    assert torch.equal(blob, z.compress_tensor(x.cuda(), pin_memory=True))
    back = z.decompress_tensor(blob, compute_device="cuda")
    assert torch.equal(back.cpu(), x)
    assert torch.equal(z.decompress_tensor(blob, compute_device="cuda", readback_to_cpu=True), x)
    blobs = z.compress_tensors([x, y, x[:1000]])
    assert torch.equal(blobs[0], blob)
    outs = z.decompress_tensors(blobs, readback_to_cpu=True)
    assert torch.equal(outs[0], x) and torch.equal(outs[1].view(torch.int16), y.view(torch.int16))
    assert torch.equal(outs[2], x[:1000])
    h = z.hash_tensor_with_crc32(x, checksum_chunk_bytes=1 << 20)
    assert torch.equal(h, z.hash_tensor_with_crc32(x.cuda(), checksum_chunk_bytes=1 << 20))


def test_blob_records_and_headers_read_as_the_list_is_walked():
    """GPU blobs made by the batched call carry their header records (size, address and fields of
    the trimmed view); a list mixing recorded blobs with GPU blobs that have none (clones, written
    in place) and CPU blobs decodes exactly, whatever their order; an invalid blob after valid ones
    raises."""
    ts = mixed_tensors()
    ref = z.compress_tensors(ts)  # CPU blobs
    blobs = z.compress_tensors(ts, readback_to_cpu=False)
    for t, b, r in zip(ts, blobs, ref):
        assert b.is_cuda and b.is_contiguous() and b.numel() == r.numel()
        assert torch.equal(b.cpu(), r)
        h = b._zn_header
        assert (h[0], h[1], h[2]) == (b._version, b.data_ptr(), b.numel())
        assert h[3] == t.dtype and h[4] == tuple(t.shape)
    mix = []
    for j, (b, r) in enumerate(zip(blobs, ref)):
        if j % 3 == 1:
            mix.append(b.clone())  # no record: its header is gathered from the device
        elif j % 3 == 2:
            mix.append(r)          # a CPU blob
        else:
            mix.append(b)
    bumped = blobs[0]
    bumped[:1].copy_(bumped[:1])   # an in-place write voids its record (same bytes)
    mix.append(bumped)
    outs = z.decompress_tensors(mix)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    for t, y in zip(ts + [ts[0]], outs):
        assert y.shape == t.shape and y.dtype == t.dtype
        assert torch.equal(bits(y.cpu()), bits(t.cpu()))
    with pytest.raises(ValueError, match="1-D uint8"):
        z.decompress_tensors([blobs[0], blobs[2], blobs[4].view(torch.int8)])


def test_tiny_stored_outputs_of_many_dtypes_and_shapes():
    """Stored-path tensors of every element size and of 0-d, 1-d and 3-d shapes, mixed with coded
    ones, come back exact, contiguous and with their own shapes from one batched call (the tiny
    ones are views of one buffer per dtype, shaped in place)."""
    g = torch.Generator(device="cuda").manual_seed(21)
    ts = []
    for dtype in [torch.bool, torch.uint8, torch.int8, torch.float16, torch.bfloat16, torch.int32,
                  torch.float32, torch.int64, torch.float64, torch.complex64, torch.float8_e5m2]:
        for shape in [(), (1,), (7,), (3, 5, 2), (1000,), (4, 33, 3)]:
            x = torch.randn(shape, device="cuda", generator=g) if dtype != torch.complex64 else torch.randn(
                shape, device="cuda", generator=g, dtype=torch.complex64)
            ts.append(x.to(dtype) if dtype != torch.bool else x > 0)
    ts.insert(5, (torch.randn(300, 1000, device="cuda", generator=g) * 0.02).to(torch.bfloat16))  # coded
    blobs = z.compress_tensors(ts, readback_to_cpu=False)
    for t, b in zip(ts, blobs):
        assert torch.equal(b.cpu(), z.compress_tensor(t))
    outs = z.decompress_tensors(blobs)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    for t, y in zip(ts, outs):
        assert y.shape == t.shape and y.dtype == t.dtype and y.is_contiguous() and y.is_cuda
        assert torch.equal(y.view(-1).view(torch.uint8), t.reshape(-1).view(torch.uint8))
    # The outputs are independent: writing one leaves the others alone.
    outs[0].fill_(True)  # a 0-d bool tensor
    for t, y in zip(ts[1:], outs[1:]):
        assert torch.equal(y.view(-1).view(torch.uint8), t.reshape(-1).view(torch.uint8))
