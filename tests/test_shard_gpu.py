"""Whole-model sharding: each rank compresses its share of the tensors on its own GPU, and every blob
equals the one a single GPU makes, byte for byte.

- plan_shards (whole tensors) over every visible GPU, one process per GPU (skipped with fewer than
  two GPUs);
- plan_model (large tensors by chunk range, the rest whole) with the ranks of 2, 3 and 8 GPUs run
  one after another on one GPU: whole blobs equal the single-GPU blobs, the parts of each split
  tensor assemble into its single-GPU blob, and each rank's decoded elements are its slice."""

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


def test_all_gpu_shards_equal_one_gpu_blobs():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two GPUs")
    import cuzipnn_b200 as z

    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, outdir)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert [p.exitcode for p in procs] == [0] * world
    model = _model()
    ref = z.compress_tensors([t.cuda() for t in model], min_compress_bytes=1024)
    for i in range(len(model)):
        assert np.array_equal(np.load(os.path.join(outdir, f"blob{i}.npy")), ref[i].numpy()), i


@pytest.mark.parametrize("world", [2, 3, 8])
def test_model_shards_by_rank_on_one_gpu(world):
    import cuzipnn_b200 as z

    g = torch.Generator(device="cuda").manual_seed(4)
    model = [(torch.randn(s, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
             for s in [(3000, 1000), (512, 256), (300_001,), (4096,), (200, 100)]]
    model.append(torch.randn(1_000_000, generator=g, device="cuda"))
    nb = [t.numel() * t.element_size() for t in model]
    whole_plan, split = z.plan_model(nb, world, split_bytes=2_000_000)
    assert split == [0, 5]
    ref = z.compress_tensors(model, readback_to_cpu=False)
    parts = {i: [] for i in split}
    for r in range(world):
        whole, mine = z.compress_model_shard(model, r, world, split_bytes=2_000_000, readback_to_cpu=False)
        assert sorted(whole) == whole_plan[r] and sorted(mine) == split
        for i, b in whole.items():
            assert torch.equal(b, ref[i]), (r, i)
        outs, pouts = z.decompress_model_shard(whole, mine)
        torch.cuda.synchronize()
        assert z.last_decode_status() == 0
        for i, y in outs.items():
            assert torch.equal(y.view(torch.int16 if y.element_size() == 2 else torch.int32),
                               model[i].view(torch.int16 if y.element_size() == 2 else torch.int32))
        for i, y in pouts.items():
            j0, j1 = z.plan_chunk_ranges(model[i].numel(), 131072, world)[r]
            flat = model[i].reshape(-1)[j0 * 131072 : j1 * 131072]
            assert torch.equal(y.view(torch.uint8), flat.view(torch.uint8)), (r, i)
            parts[i].append(mine[i])
    for i in split:
        assert torch.equal(z.assemble_chunk_ranges(parts[i], model[i].shape), ref[i]), i
