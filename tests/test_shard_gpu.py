"""Whole-model sharding on two GPUs: each rank compresses its share of the tensors (plan_shards) on
its own GPU, and every blob equals the one a single GPU makes, byte for byte.  Skipped with fewer
than two GPUs."""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _model():
    g = torch.Generator().manual_seed(11)
    shapes = [(1024, 512), (300_001,), (4096,), (777, 129), (64,), (2048, 256)]
    dtypes = [torch.bfloat16, torch.float32, torch.bfloat16, torch.float16, torch.float32, torch.float8_e4m3fn]
    return [(torch.randn(s, generator=g) * (16 if d == torch.float8_e4m3fn else 0.02)).to(d) for s, d in zip(shapes, dtypes)]


def _worker(rank, world, outdir):
    import cuzipnn_b200 as z

    torch.cuda.set_device(rank)
    model = [t.cuda() for t in _model()]
    local = z.compress_shard(model, rank, world, min_compress_bytes=1024, readback_to_cpu=False)
    back = z.decompress_shard(local)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    for i, b in local.items():
        assert torch.equal(back[i].view(torch.uint8), model[i].view(torch.uint8)), i
        np.save(os.path.join(outdir, f"blob{i}.npy"), b.cpu().numpy())


def test_two_gpu_shards_equal_one_gpu_blobs():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import cuzipnn_b200 as z

    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, outdir)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert [p.exitcode for p in procs] == [0, 0]
    model = _model()
    ref = z.compress_tensors([t.cuda() for t in model], min_compress_bytes=1024)
    for i in range(len(model)):
        assert np.array_equal(np.load(os.path.join(outdir, f"blob{i}.npy")), ref[i].numpy()), i
