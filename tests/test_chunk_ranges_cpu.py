"""Chunk-range sharding of one tensor (cuzipnn_b200._shard) without a GPU.

The oracle makes the whole tensor's blob and each rank's part (the blob of its chunk range as a
1-D tensor, coded with the whole tensor's parameters); the library's host-side assembly must join
the parts into the whole blob byte for byte, and its split must cut the whole blob back into the
parts.  A world-size-4 gloo run gathers the parts on one rank over point-to-point sends.  The GPU
side (compress_chunk_range on the device) is in tests/test_chunk_ranges_gpu.py."""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import cuzipnn_b200 as z
from oracle import oracle as O

C = 4096  # chunk_bytes (elements per chunk): several chunks at oracle-friendly sizes

_NAMES = {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.float16: "float16", torch.uint8: "uint8",
          torch.float64: "float64"}


def _tensor(dtype, n, seed):
    g = torch.Generator().manual_seed(seed)
    if dtype == torch.uint8:  # skewed bytes with a uniform stretch: coded and raw units
        x = (torch.randn(n, generator=g).abs() * 3).clamp(max=255).to(torch.uint8)
        x[n // 3 : n // 2] = torch.randint(0, 256, (n // 2 - n // 3,), generator=g, dtype=torch.uint8)
        return x
    return (torch.randn(n, generator=g) * 0.02).to(dtype)


def _blob(x, shape, **kw):
    raw = x.contiguous().view(-1).view(torch.uint8).numpy()
    return torch.from_numpy(np.frombuffer(O.compress(raw, shape, _NAMES[x.dtype], chunk_bytes=C, threads=1, **kw),
                                          dtype=np.uint8).copy())


def _parts(x, world):
    flat = x.reshape(-1)
    out = []
    for j0, j1 in z.plan_chunk_ranges(flat.numel(), C, world):
        part = flat[j0 * C : min(j1 * C, flat.numel())]
        out.append(_blob(part, (part.numel(),), min_compress_bytes=0))
    return out


def test_plan_chunk_ranges():
    assert z.plan_chunk_ranges(10 * C + 1, C, 4) == [(0, 3), (3, 6), (6, 9), (9, 11)]
    assert z.plan_chunk_ranges(2 * C, C, 3) == [(0, 1), (1, 2), (2, 2)]
    assert z.plan_chunk_ranges(0, C, 2) == [(0, 0), (0, 0)]
    for n in (1, C - 1, C, 5 * C + 7, 64 * C):
        for world in (1, 2, 3, 8):
            ranges = z.plan_chunk_ranges(n, C, world)
            assert ranges[0][0] == 0 and ranges[-1][1] == -(-n // C)
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [j1 - j0 for j0, j1 in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        z.plan_chunk_ranges(10, C, 0)


@pytest.mark.parametrize("dtype,n,shape", [
    (torch.bfloat16, 7 * C + 555, (7 * C + 555,)),
    (torch.float32, 6 * C, (6, C)),
    (torch.float16, 5 * C + 1, (5 * C + 1,)),
    (torch.uint8, 9 * C + 100, (9 * C + 100,)),
    (torch.float64, 3 * C + 17, (3 * C + 17, 1)),
])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_assemble_and_split_match_oracle(dtype, n, shape, world):
    x = _tensor(dtype, n, seed=n + world).reshape(shape)
    whole = _blob(x, shape, min_compress_bytes=0)  # the sizes here are below the default
    parts = _parts(x, world)
    assert torch.equal(z.assemble_chunk_ranges(parts, shape), whole)
    for (j0, j1), part in zip(z.plan_chunk_ranges(n, C, world), parts):
        assert torch.equal(z.split_chunk_range(whole, j0, j1), part), (j0, j1)
    # A rank without chunks may also hand in nothing.
    ranges = z.plan_chunk_ranges(n, C, world)
    sparse = [p if j1 > j0 else None for (j0, j1), p in zip(ranges, parts)]
    assert torch.equal(z.assemble_chunk_ranges(sparse, shape), whole)


def test_stored_and_empty_tensors_are_one_part():
    x = _tensor(torch.bfloat16, 100, seed=1)
    stored = _blob(x, (100,))  # below min_compress_bytes: stored path
    assert torch.equal(z.assemble_chunk_ranges([stored, None, None], (100,)), stored)
    with pytest.raises(ValueError):
        z.split_chunk_range(stored, 0, 1)
    empty = _blob(x[:0], (0, 5))
    assert torch.equal(z.assemble_chunk_ranges([empty, None], (0, 5)), empty)
    with pytest.raises(ValueError):
        z.assemble_chunk_ranges([None, None], (0, 5))


def test_mismatched_parts_are_rejected():
    x = _tensor(torch.bfloat16, 4 * C, seed=2)
    parts = _parts(x, 2)
    with pytest.raises(ValueError):
        z.assemble_chunk_ranges(parts[::-1] + [parts[0]], (4 * C,))  # too many elements
    with pytest.raises(ValueError):
        z.assemble_chunk_ranges(parts, (4 * C + 1,))
    y = _tensor(torch.float16, 4 * C, seed=2)
    with pytest.raises(ValueError):
        z.assemble_chunk_ranges([parts[0], _parts(y, 2)[1]], (4 * C,))  # dtypes differ
    short = _tensor(torch.bfloat16, 3 * C + 5, seed=3)
    with pytest.raises(ValueError):  # a part that is not the last holds a partial chunk
        z.assemble_chunk_ranges([_blob(short, (3 * C + 5,), min_compress_bytes=0), parts[1]], (5 * C + 5,))
    whole = _blob(x, (4 * C,), min_compress_bytes=0)
    with pytest.raises(ValueError):
        z.split_chunk_range(whole, 2, 5)
    with pytest.raises(ValueError):
        z.split_chunk_range(whole[:-8], 0, 4)  # truncated


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        x = _tensor(torch.bfloat16, 2 * C + 9, seed=4)  # 3 chunks over 4 ranks: rank 3 has none
        part = _parts(x, world)[rank] if rank < 3 else None
        got = z.gather_chunk_ranges(part, dst=1)
        if rank == 1:
            assert got[3] is None and len(got) == world
            np.save(os.path.join(outdir, "blob.npy"), z.assemble_chunk_ranges(got, (2 * C + 9,)).numpy())
        else:
            assert got is None
    finally:
        dist.destroy_process_group()


def test_gather_on_one_rank_gloo():
    port, outdir = _free_port(), tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 4, port, outdir)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    assert [p.exitcode for p in procs] == [0, 0, 0, 0]
    x = _tensor(torch.bfloat16, 2 * C + 9, seed=4)
    assert np.array_equal(np.load(os.path.join(outdir, "blob.npy")), _blob(x, (2 * C + 9,), min_compress_bytes=0).numpy())


def test_assembled_blob_checksums_equal_whole_tensor_crc():
    """assemble_chunk_ranges(..., checksum_chunk_bytes) gives compress_tensor_with_crc32's CRCs of
    the whole tensor (host blobs: the stored path, hashed with zlib)."""
    x = torch.randn(300, 7)
    parts = [z.compress_chunk_range(x, r, 3) for r in range(3)]
    blob, crc = z.assemble_chunk_ranges(parts, x.shape, checksum_chunk_bytes=100)
    ref_blob, ref_crc = z.compress_tensor_with_crc32(x, checksum_chunk_bytes=100)
    assert torch.equal(blob, ref_blob) and torch.equal(crc, ref_crc)
    with pytest.raises(ValueError):
        z.assemble_chunk_ranges(parts, x.shape, checksum_chunk_bytes=0)
