"""Whole-model sharding (cuzipnn_b200._shard) without a GPU: the LPT planner, a world-size-2 gloo
run whose blobs equal the single-process ones byte for byte, and a rank that fails before the
metadata gather (the surviving rank gets an error, it does not hang).

On the CPU the codec's stored path is used (every tensor below min_compress_bytes, blobs read back
to the host): it needs no GPU and exercises the same sharding, gather and assembly logic as the
GPU path (tests/test_shard_gpu.py runs that on two GPUs)."""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import cuzipnn_b200 as z

BIG = 1 << 40  # min_compress_bytes: every tensor takes the stored path


def _model():
    g = torch.Generator().manual_seed(7)
    shapes = [(300, 7), (64,), (5, 5, 5), (1000,), (17, 3), (2, 2), (0,), (129, 33), (8,)]
    dtypes = [torch.float32, torch.bfloat16, torch.float16, torch.int32, torch.float64, torch.uint8,
              torch.float32, torch.bfloat16, torch.int64]
    out = []
    for s, d in zip(shapes, dtypes):
        x = torch.randn(s, generator=g) * 100
        out.append(x.to(d))
    return out


def test_plan_shards_is_lpt_and_deterministic():
    sizes = [100, 5, 70, 70, 30, 1, 99, 0, 42]
    for world in (1, 2, 3, 4, 8, 12):
        a = z.plan_shards(sizes, world)
        assert a == z.plan_shards(sizes, world)
        flat = sorted(i for s in a for i in s)
        assert flat == list(range(len(sizes)))
        loads = [sum(sizes[i] for i in s) for s in a]
        assert max(loads) <= sum(sizes) / world + max(sizes)
    assert z.plan_shards(sizes, 2) == [[0, 1, 3, 4, 5, 7], [2, 6, 8]]  # worked by hand
    with pytest.raises(ValueError):
        z.plan_shards(sizes, 0)


def test_plan_model_splits_large_tensors_and_balances_the_rest():
    sizes = [1090, 1090] + [136] * 84 + [25] * 56 + [4] * 56 + [0, 3]
    for world in (1, 2, 3, 4, 8, 16):
        whole, split = z.plan_model(sizes, world)
        assert (whole, split) == z.plan_model(sizes, world)
        seen = sorted([i for w in whole for i in w] + split)
        assert seen == list(range(len(sizes)))
        assert all(sizes[i] > sum(sizes) // (2 * world) for i in split)
        if world == 1:
            assert split == []
        share = sum(sizes[i] for i in split) // world
        loads = [share + sum(sizes[i] for i in w) for w in whole]
        rest = [sizes[i] for i in range(len(sizes)) if i not in split]
        assert max(loads) <= sum(sizes) / world + max(rest), world
    assert z.plan_model(sizes, 8)[1] == [0, 1]
    assert z.plan_model(sizes, 2)[1] == []  # 1090 < half of a rank's share
    assert z.plan_model(sizes, 2, split_bytes=1000)[1] == [0, 1]
    with pytest.raises(ValueError):
        z.plan_model(sizes, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir, fail_rank):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        model = _model()
        local = z.compress_shard(model, rank, world, min_compress_bytes=BIG)
        if rank == fail_rank:
            raise SystemExit(3)  # this rank leaves before the metadata gather
        try:
            index = z.gather_index(local)
        except Exception as e:  # noqa: BLE001  (the surviving rank records what it saw)
            with open(os.path.join(outdir, f"error{rank}"), "w") as f:
                f.write(type(e).__name__ + ": " + str(e)[:200])
            return
        outs = z.decompress_shard(local, readback_to_cpu=True)
        for i, b in local.items():
            np.save(os.path.join(outdir, f"blob{i}.npy"), b.numpy())
            assert torch.equal(outs[i].view(torch.uint8) if outs[i].numel() else outs[i],
                               model[i].view(torch.uint8) if model[i].numel() else model[i])
        torch.save(index, os.path.join(outdir, f"index{rank}.pt"))
    finally:
        if rank != fail_rank:
            dist.destroy_process_group()


def _run(world, fail_rank=-1):
    port = _free_port()
    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, outdir, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    return outdir, [p.exitcode for p in procs]


def test_two_ranks_gloo_blobs_equal_single_process():
    outdir, codes = _run(2)
    assert codes == [0, 0]
    model = _model()
    ref = z.compress_tensors(model, min_compress_bytes=BIG)
    idx0 = torch.load(os.path.join(outdir, "index0.pt"))
    idx1 = torch.load(os.path.join(outdir, "index1.pt"))
    assert idx0 == idx1 and sorted(idx0) == list(range(len(model)))
    plan = z.plan_shards([t.numel() * t.element_size() for t in model], 2)
    for i, (r, size) in idx0.items():
        assert i in plan[r]
        blob = np.load(os.path.join(outdir, f"blob{i}.npy"))
        assert size == blob.size
        assert np.array_equal(blob, ref[i].numpy()), i


def test_rank_failure_is_reported_not_hung():
    outdir, codes = _run(2, fail_rank=1)
    assert codes[1] == 3
    err = open(os.path.join(outdir, "error0")).read()
    assert err  # rank 0's gather raised (peer gone or timeout) instead of blocking
