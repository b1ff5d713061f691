"""Chunk-range sharding of one large tensor on the GPU: each rank's part (compress_chunk_range)
joined by assemble_chunk_ranges equals the single-GPU blob byte for byte, and the ranks' chunk
ranges decompressed one by one give back the tensor.  Ranks run one after another on one GPU
here; the two-GPU test (skipped with fewer GPUs) runs one process per GPU and gathers the parts
over NCCL."""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import cuzipnn_b200 as z

pytestmark = pytest.mark.gpu


def _bits(t):
    t = t.contiguous().view(-1)
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


def _check(x, world, **kw):
    whole = z.compress_tensor(x, readback_to_cpu=False, **kw)
    parts = [z.compress_chunk_range(x, r, world, readback_to_cpu=False, **kw) for r in range(world)]
    blob = z.assemble_chunk_ranges(parts, x.shape)
    assert blob.device == x.device
    assert torch.equal(blob, whole)
    outs = [z.decompress_chunk_range(whole, r, world) for r in range(world)]
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    assert torch.equal(_bits(torch.cat(outs)), _bits(x))
    return parts


def test_7b_embedding_bf16_eight_ranges():
    """The 7B decoder's largest tensor (152064 x 3584 bf16, 1.09 GB, 4158 chunks) over 8 ranges."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(152064, 3584, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    _check(x, 8)


@pytest.mark.parametrize("dtype,shape,world", [
    (torch.float32, (4096, 4096), 3),
    (torch.float16, (1_000_003,), 5),
    (torch.uint8, (3, 1 << 20), 4),
    (torch.bfloat16, (300_000,), 16),  # more ranges than chunks: some ranks hold none
])
def test_ranges_of_other_dtypes(dtype, shape, world):
    g = torch.Generator(device="cuda").manual_seed(1)
    if dtype == torch.uint8:
        x = (torch.randn(shape, generator=g, device="cuda").abs() * 3).to(torch.uint8)
    else:
        x = (torch.randn(shape, generator=g, device="cuda") * 0.02).to(dtype)
    _check(x, world)


def test_small_chunks_and_stored_tensor():
    g = torch.Generator(device="cuda").manual_seed(2)
    x = (torch.randn(50_000, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    _check(x, 3, chunk_bytes=4096, sub_chunk_bytes=1024)
    small = x[:1000]  # below min_compress_bytes: rank 0 holds the whole (stored) blob
    parts = [z.compress_chunk_range(small, r, 3, readback_to_cpu=False) for r in range(3)]
    assert parts[1] is None and parts[2] is None
    assert torch.equal(z.assemble_chunk_ranges(parts, small.shape), z.compress_tensor(small, readback_to_cpu=False))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _big():
    g = torch.Generator().manual_seed(3)
    return (torch.randn(8192, 3584, generator=g) * 0.02).to(torch.bfloat16)


def _worker(rank, world, port, outdir):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        x = _big().cuda()
        part = z.compress_chunk_range(x, rank, world, readback_to_cpu=False)
        got = z.gather_chunk_ranges(part, dst=0)
        if rank == 0:
            np.save(os.path.join(outdir, "blob.npy"), z.assemble_chunk_ranges(got, x.shape).cpu().numpy())
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_ranges_gathered_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port, outdir = _free_port(), tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, outdir)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in procs] == [0, 0]
    ref = z.compress_tensor(_big().cuda(), readback_to_cpu=True)
    assert np.array_equal(np.load(os.path.join(outdir, "blob.npy")), ref.numpy())


def test_assembled_blob_checksums_on_gpu():
    """CRCs of an assembled coded blob equal compress_tensor_with_crc32's for the whole tensor."""
    g = torch.Generator(device="cuda").manual_seed(6)
    x = (torch.randn(1_000_003, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    parts = [z.compress_chunk_range(x, r, 4, readback_to_cpu=False) for r in range(4)]
    blob, crc = z.assemble_chunk_ranges(parts, x.shape, checksum_chunk_bytes=16384)
    ref_blob, ref_crc = z.compress_tensor_with_crc32(x, checksum_chunk_bytes=16384, readback_to_cpu=False)
    assert torch.equal(blob, ref_blob) and torch.equal(crc, ref_crc)
