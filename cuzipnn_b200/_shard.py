"""Whole-model sharding over the GPUs of one box: one process per GPU, no collective on the data path.

The codec's units are independent, so a model shards by whole tensors: each rank compresses (or
decompresses) a disjoint subset of the tensors on its own GPU, and every blob is byte-identical to
the one a single GPU produces.  Only metadata crosses processes: which rank holds which blob, and
its size, through torch.distributed's object gather (gloo or NCCL).  A rank that fails or leaves
before that gather makes it raise on the other ranks (bounded by the process group's timeout)
instead of hanging them.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from ._codec import compress_tensors, decompress_tensors


def plan_shards(nbytes: Sequence[int], world: int) -> list[list[int]]:
    """Assign tensors (by byte size) to `world` ranks, longest first, each to the rank with the
    fewest bytes so far (ties: lowest rank).  Deterministic; returns each rank's tensor indices in
    ascending order.  The largest rank holds at most the mean plus the largest tensor."""
    if world <= 0:
        raise ValueError("world must be positive")
    loads = [0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(nbytes)), key=lambda i: (-int(nbytes[i]), i)):
        r = min(range(world), key=lambda q: (loads[q], q))
        shards[r].append(i)
        loads[r] += int(nbytes[i])
    for s in shards:
        s.sort()
    return shards


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def compress_shard(tensors: Sequence[torch.Tensor], rank: int, world: int, **kwargs) -> dict[int, torch.Tensor]:
    """Compress this rank's share of `tensors` (plan_shards) with compress_tensors on the current
    device; returns {tensor index: blob}.  Keyword arguments are compress_tensors'."""
    idx = plan_shards([_nbytes(t) for t in tensors], world)[rank]
    if not idx:
        return {}
    blobs = compress_tensors([tensors[i] for i in idx], **kwargs)
    return dict(zip(idx, blobs))


def decompress_shard(blobs: dict[int, torch.Tensor], **kwargs) -> dict[int, torch.Tensor]:
    """Decompress the blobs this rank holds ({tensor index: blob}) with decompress_tensors."""
    keys = sorted(blobs)
    if not keys:
        return {}
    outs = decompress_tensors([blobs[i] for i in keys], **kwargs)
    return dict(zip(keys, outs))


def gather_index(local: dict[int, torch.Tensor], group=None) -> dict[int, tuple[int, int]]:
    """Every rank learns where each blob lives: {tensor index: (rank, blob bytes)}.  Metadata only
    (an all_gather_object of this rank's index and sizes); the blobs stay where they are."""
    import torch.distributed as dist

    mine = [(i, int(b.numel())) for i, b in sorted(local.items())]
    parts: list[list[tuple[int, int]] | None] = [None] * dist.get_world_size(group)
    dist.all_gather_object(parts, mine, group=group)
    out: dict[int, tuple[int, int]] = {}
    for r, part in enumerate(parts):
        for i, size in part or []:
            if i in out:
                raise RuntimeError(f"tensor {i} is held by ranks {out[i][0]} and {r}")
            out[i] = (r, size)
    return out
