"""Sharding over the GPUs of one box, one process per GPU.

Whole models: the codec's units are independent, so a model shards by whole tensors: each rank
compresses (or decompresses) a disjoint subset of the tensors on its own GPU, and every blob is
byte-identical to the one a single GPU produces.  Only metadata crosses processes: which rank holds
which blob, and its size, through torch.distributed's object gather (gloo or NCCL).  A rank that
fails or leaves before that gather makes it raise on the other ranks (bounded by the process
group's timeout) instead of hanging them.

One large tensor: its chunks split into contiguous ranges, one per rank (compress_chunk_range);
the parts join into the whole tensor's blob on one rank (gather_chunk_ranges, then
assemble_chunk_ranges), byte for byte the blob a single GPU makes.  split_chunk_range and
decompress_chunk_range go the other way.
"""

from __future__ import annotations

import heapq
import math
import struct
from collections.abc import Sequence

import numpy as np
import torch

from . import _codec as C
from ._codec import compress_tensor, compress_tensors, decompress_tensor, decompress_tensors


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


# ---- one large tensor over several GPUs: contiguous chunk ranges -----------------------------
#
# A blob's units (stream b, chunk j) depend only on the chunk's elements and the codec
# parameters, so the chunks of one tensor split into contiguous ranges, one per rank.  Rank r
# compresses elements [j0 * C, min(j1 * C, n)) as a 1-D tensor with the whole tensor's
# parameters; its part is a complete blob whose units equal the whole tensor's units j0 .. j1 - 1
# byte for byte.  The whole blob is then the header, the concatenated stored_bytes slices, the
# comp_idx lists shifted to global unit indices, and for each stream b the parts' stream-b data
# segments in rank order (each unit is padded to 8 bytes, so segments join without gaps).


def plan_chunk_ranges(numel: int, chunk_bytes: int, world: int) -> list[tuple[int, int]]:
    """Split the ceil(numel / chunk_bytes) chunks of a tensor into `world` contiguous ranges
    [j0, j1), as even as possible (the first nch % world ranks get one chunk more)."""
    if world <= 0:
        raise ValueError("world must be positive")
    if chunk_bytes <= 0:
        raise ValueError("chunk_bytes must be positive")
    nch = -(-int(numel) // chunk_bytes)
    q, rem = divmod(nch, world)
    out, j = [], 0
    for r in range(world):
        k = q + (r < rem)
        out.append((j, j + k))
        j += k
    return out


def compress_chunk_range(
    tensor: torch.Tensor,
    rank: int,
    world: int,
    *,
    chunk_bytes: int = C.DEFAULT_CHUNK_BYTES,
    sub_chunk_bytes: int = C.DEFAULT_SUB_CHUNK_BYTES,
    passthrough_threshold: float = C.DEFAULT_PASSTHROUGH_THRESHOLD,
    min_compress_bytes: int = C.DEFAULT_MIN_COMPRESS_BYTES,
    pin_memory: bool = False,
    compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = True,
) -> torch.Tensor | None:
    """This rank's part of one tensor: its chunk range (plan_chunk_ranges) compressed on the
    current (or the given) device, as compress_tensor would (same keyword arguments).

    A tensor that takes the stored or the empty path has no chunks: rank 0 returns its whole blob
    and the other ranks None.  assemble_chunk_ranges joins the parts into the whole tensor's blob.
    Parts carry no checksums (a CRC segment of the whole blob spans parts): ask
    assemble_chunk_ranges for them (checksum_chunk_bytes), which hashes the assembled blob.
    """
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    C._check_args(tensor, chunk_bytes, sub_chunk_bytes, passthrough_threshold, min_compress_bytes, None,
                  pin_memory, compute_device, readback_to_cpu)
    kw = dict(chunk_bytes=chunk_bytes, sub_chunk_bytes=sub_chunk_bytes, passthrough_threshold=passthrough_threshold,
              pin_memory=pin_memory, compute_device=compute_device, readback_to_cpu=readback_to_cpu)
    n = tensor.numel()
    if n * tensor.element_size() < min_compress_bytes or n == 0:  # the stored or the empty path
        return compress_tensor(tensor, min_compress_bytes=min_compress_bytes, **kw) if rank == 0 else None
    j0, j1 = plan_chunk_ranges(n, chunk_bytes, world)[rank]
    part = tensor.detach().reshape(-1)[j0 * chunk_bytes : min(j1 * chunk_bytes, n)]
    # min_compress_bytes = 0: the part is coded like the whole tensor even when it is small.
    return compress_tensor(part, min_compress_bytes=0, **kw)


# ---- a whole model over several GPUs: large tensors by chunk range, the rest whole -------------


def plan_model(nbytes: Sequence[int], world: int, split_bytes: int | None = None) -> tuple[list[list[int]], list[int]]:
    """Plan a model's tensors (byte sizes `nbytes`) over `world` ranks for strong scaling.  Tensors
    of more than split_bytes bytes (default: half a rank's mean share, sum / (2 * world)) are split:
    every rank compresses its chunk range of each (plan_chunk_ranges), so they add about 1 / world
    of their bytes to every rank.  The other tensors go whole to ranks, longest first, each to the
    rank with the fewest bytes so far (ties: lowest rank).  Deterministic.

    Returns (whole, split): whole[r] = indices of the tensors rank r takes whole (ascending),
    split = indices of the split tensors (ascending)."""
    if world <= 0:
        raise ValueError("world must be positive")
    total = sum(int(b) for b in nbytes)
    if split_bytes is None:
        split_bytes = total // (2 * world)
    sizes = [int(b) for b in nbytes]
    split = [i for i, b in enumerate(sizes) if world > 1 and b > split_bytes]
    share = sum(sizes[i] for i in split) // world
    heap = [(share, r) for r in range(world)]  # (load, rank): the least-loaded, lowest rank first
    whole: list[list[int]] = [[] for _ in range(world)]
    cut = set(split)
    for i in sorted((i for i in range(len(sizes)) if i not in cut), key=lambda i: (-sizes[i], i)):
        load, r = heapq.heappop(heap)
        whole[r].append(i)
        heapq.heappush(heap, (load + sizes[i], r))
    for w in whole:
        w.sort()
    return whole, split


def _range_part(tensor: torch.Tensor, rank: int, world: int, chunk_bytes: int) -> torch.Tensor:
    """The flat elements of this rank's chunk range of a tensor (plan_chunk_ranges)."""
    n = tensor.numel()
    j0, j1 = plan_chunk_ranges(n, chunk_bytes, world)[rank]
    return tensor.detach().reshape(-1)[j0 * chunk_bytes : min(j1 * chunk_bytes, n)]


def compress_model_shard(
    tensors: Sequence[torch.Tensor], rank: int, world: int, *, split_bytes: int | None = None,
    plan: tuple[list[list[int]], list[int]] | None = None, **kwargs
) -> tuple[dict[int, torch.Tensor], dict[int, torch.Tensor]]:
    """This rank's share of a model (plan_model) compressed on the current device: returns (whole,
    parts), whole = {tensor index: blob} of the tensors it takes whole, parts = {tensor index: this
    rank's chunk-range part} of the split tensors (compress_chunk_range's blob; gather_chunk_ranges
    and assemble_chunk_ranges join the parts of all ranks into the tensor's blob).  One
    compress_tensors call covers the whole tensors and every part that is coded anyway; keyword
    arguments are compress_tensors'.  `plan`, if given, is plan_model's result for these tensors and
    this world (a loader plans a model once), else it is computed here."""
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    whole_idx, split = plan if plan is not None else plan_model([_nbytes(t) for t in tensors], world, split_bytes)
    chunk = kwargs.get("chunk_bytes", C.DEFAULT_CHUNK_BYTES)
    minb = kwargs.get("min_compress_bytes", C.DEFAULT_MIN_COMPRESS_BYTES)
    # The parts go first: they are large, so the call's first sub-batch fills (and its kernels
    # start) after a tensor or two.
    items, parts, part_keys = [], {}, []
    for i in split:
        t = tensors[i]
        if _nbytes(t) < minb or t.numel() == 0:  # the stored or the empty path: rank 0 holds it whole
            if rank == 0:
                parts[i] = compress_chunk_range(t, rank, world, **kwargs)
            continue
        part = _range_part(t, rank, world, chunk)
        if part.numel() * part.element_size() >= minb:
            items.append(part)
            part_keys.append(i)
        else:  # a short (or empty) range is coded with min_compress_bytes = 0, as compress_chunk_range does
            parts[i] = compress_chunk_range(t, rank, world, **kwargs)
    keys = list(whole_idx[rank])
    items += [tensors[i] for i in keys]
    blobs = compress_tensors(items, **kwargs) if items else []
    parts.update(zip(part_keys, blobs[: len(part_keys)]))
    whole = dict(zip(keys, blobs[len(part_keys) :]))
    return whole, parts


def decompress_model_shard(whole: dict[int, torch.Tensor], parts: dict[int, torch.Tensor], **kwargs
                           ) -> tuple[dict[int, torch.Tensor], dict[int, torch.Tensor]]:
    """Decompress what compress_model_shard returned, in one decompress_tensors call: (tensors by
    index, this rank's flat elements of each split tensor by index)."""
    wk, pk = sorted(whole), sorted(parts)
    outs = decompress_tensors([parts[i] for i in pk] + [whole[i] for i in wk], **kwargs) if wk or pk else []
    return dict(zip(wk, outs[len(pk) :])), {i: o.reshape(-1) for i, o in zip(pk, outs[: len(pk)])}


class _Tables:
    """Header and unit tables of a blob, read to the host (header, stored_bytes and comp_idx only)."""

    def __init__(self, blob: torch.Tensor):
        if blob.dtype != torch.uint8 or blob.dim() != 1:
            raise ValueError("blob must be a 1-D uint8 tensor")
        plen = min(blob.numel(), C._FIXED.size + 8 * C._MAX_NDIM)
        prefix = blob[:plen].cpu().numpy().tobytes()
        self.dtype, self.shape, self.flags, self.chunk_bytes, self.n_comp, self.n = C._parse_header(prefix)
        self.k = self.dtype.itemsize
        self.stored_path = bool(self.flags & C._FLAG_STORED)
        if self.stored_path:
            return
        if self.chunk_bytes <= 0 or math.prod(self.shape) != self.n:
            raise ValueError("not a cuzipnn blob")
        self.nch = -(-self.n // self.chunk_bytes)
        sizes_off, idx_off, self.data_off = C._layout(len(self.shape), self.k * self.nch, self.n_comp)
        if blob.numel() < self.data_off:
            raise ValueError("blob is truncated")
        tabs = blob[sizes_off : idx_off + 4 * self.n_comp].cpu().numpy()
        self.stored = tabs[: 4 * self.k * self.nch].view(np.int32).astype(np.int64)
        self.idx = tabs[4 * self.k * self.nch :].view(np.int32).astype(np.int64)
        if (self.stored < 0).any() or (self.idx < 0).any() or (self.idx >= self.k * self.nch).any():
            raise ValueError("not a cuzipnn blob")
        padded = (self.stored + 7) & ~7
        # Byte offset of every unit's data (unit u at unit_off[u], the data's end at unit_off[-1]).
        self.unit_off = self.data_off + np.concatenate(([0], np.cumsum(padded)))
        if blob.numel() < self.unit_off[-1]:
            raise ValueError("blob is truncated")

    def stream_segment(self, b: int) -> tuple[int, int]:
        """[start, end) of stream b's data in the blob."""
        return int(self.unit_off[b * self.nch]), int(self.unit_off[(b + 1) * self.nch])


def _join(prefix: bytes, pieces: list[tuple[torch.Tensor, int, int]], device: torch.device) -> torch.Tensor:
    """prefix followed by the byte ranges [s, e) of the given blobs, on `device`."""
    total = len(prefix) + sum(e - s for _, s, e in pieces)
    out = torch.empty(total, dtype=torch.uint8, device=device)
    out[: len(prefix)].copy_(torch.frombuffer(bytearray(prefix), dtype=torch.uint8))
    pos = len(prefix)
    for t, s, e in pieces:
        if e > s:
            out[pos : pos + e - s].copy_(t[s:e], non_blocking=t.is_cuda and out.is_cuda)
        pos += e - s
    return out


def _prefix(dtype, shape, flags, chunk_bytes, numel, stored: np.ndarray, idx: np.ndarray) -> bytes:
    head = C._FIXED.pack(C._MAGIC, C._VERSION, C._CODES[dtype], len(shape), flags, chunk_bytes, len(idx), numel)
    head += struct.pack(f"<{len(shape)}q", *shape)
    head += stored.astype("<i4").tobytes() + idx.astype("<i4").tobytes()
    return head + bytes(C._align8(len(head)) - len(head))


def assemble_chunk_ranges(
    parts: Sequence[torch.Tensor | None], shape: Sequence[int], *, device: torch.device | str | None = None,
    checksum_chunk_bytes: int | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """The blob of the whole tensor (shape `shape`) from the parts compress_chunk_range made, in
    rank order; byte for byte the blob compress_tensor makes of the whole tensor with the same
    arguments.  The blob is placed on `device` (default: the first part's device); parts on other
    devices are copied from there.  Raises ValueError if the parts do not fit together.

    With checksum_chunk_bytes, returns (blob, crc) instead, crc as compress_tensor_with_crc32
    gives it for the whole tensor (hash_tensor_with_crc32 of the assembled blob)."""
    blob = _assemble(parts, shape, device)
    if checksum_chunk_bytes is None:
        return blob
    if checksum_chunk_bytes <= 0:
        raise ValueError("checksum_chunk_bytes must be positive")
    if blob.is_cuda:
        return blob, C.hash_tensor_with_crc32(blob, checksum_chunk_bytes=checksum_chunk_bytes, readback_to_cpu=False)
    return blob, C._host_crc32(blob, checksum_chunk_bytes)


def _assemble(parts: Sequence[torch.Tensor | None], shape: Sequence[int], device) -> torch.Tensor:
    shape = tuple(int(s) for s in shape)
    live = [p for p in parts if p is not None]
    if not live:
        raise ValueError("no parts")
    device = live[0].device if device is None else torch.device(device)
    tabs = [_Tables(p) for p in live]
    n = math.prod(shape)
    if n == 0 or any(t.stored_path for t in tabs):
        # Stored or empty tensor: rank 0's part is the whole blob.
        if len(live) != 1 or tabs[0].shape != shape:
            raise ValueError("parts do not form one blob")
        return live[0].to(device)
    keep = [(p, t) for p, t in zip(live, tabs) if t.n > 0]  # ranks without chunks add nothing
    t0 = keep[0][1] if keep else tabs[0]
    for _, t in keep:
        if (t.dtype, t.flags, t.chunk_bytes, len(t.shape)) != (t0.dtype, t0.flags, t0.chunk_bytes, 1):
            raise ValueError("parts do not form one blob")
    # Every part but the last holds whole chunks.
    if any(t.n % t.chunk_bytes for _, t in keep[:-1]) or sum(t.n for _, t in keep) != n:
        raise ValueError("parts do not form one blob")
    k, cb = t0.k, t0.chunk_bytes
    nch = sum(t.nch for _, t in keep)
    stored, idx, pieces = [], [], []
    for b in range(k):
        j0 = 0
        for p, t in keep:
            stored.append(t.stored[b * t.nch : (b + 1) * t.nch])
            mine = t.idx[(t.idx >= b * t.nch) & (t.idx < (b + 1) * t.nch)]
            idx.append(mine - b * t.nch + b * nch + j0)
            pieces.append((p, *t.stream_segment(b)))
            j0 += t.nch
    prefix = _prefix(t0.dtype, shape, t0.flags, cb, n, np.concatenate(stored), np.concatenate(idx))
    return _join(prefix, pieces, device)


def split_chunk_range(blob: torch.Tensor, j0: int, j1: int) -> torch.Tensor:
    """The blob of chunks [j0, j1) of the tensor in `blob` (a 1-D tensor of elements
    [j0 * C, min(j1 * C, n))), on the blob's device: the part compress_chunk_range makes of that
    range.  Only the header and tables are read to the host; the data moves device to device."""
    t = _Tables(blob)
    if t.stored_path:
        raise ValueError("a stored blob has no chunks")
    if not 0 <= j0 <= j1 <= t.nch:
        raise ValueError("chunk range out of bounds")
    m = max(0, min(j1 * t.chunk_bytes, t.n) - j0 * t.chunk_bytes)
    if m == 0:
        return _join(_prefix(t.dtype, (0,), t.flags, t.chunk_bytes, 0, np.zeros(0, np.int64), np.zeros(0, np.int64)),
                     [], blob.device)
    stored, idx, pieces = [], [], []
    w = j1 - j0
    for b in range(t.k):
        lo, hi = b * t.nch + j0, b * t.nch + j1
        stored.append(t.stored[lo:hi])
        idx.append(t.idx[(t.idx >= lo) & (t.idx < hi)] - lo + b * w)
        pieces.append((blob, int(t.unit_off[lo]), int(t.unit_off[hi])))
    prefix = _prefix(t.dtype, (m,), t.flags, t.chunk_bytes, m, np.concatenate(stored), np.concatenate(idx))
    return _join(prefix, pieces, blob.device)


def decompress_chunk_range(
    blob: torch.Tensor, rank: int, world: int, *, compute_device: torch.device | str | None = None,
    readback_to_cpu: bool = False,
) -> torch.Tensor:
    """This rank's elements of the tensor in `blob`: the flat elements of its chunk range
    (plan_chunk_ranges), decompressed as decompress_tensor would.  A stored blob has no chunks:
    rank 0 gets the whole tensor (flattened) and the other ranks an empty one."""
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    t = _Tables(blob)
    if t.stored_path:
        if rank == 0:
            return decompress_tensor(blob, compute_device=compute_device, readback_to_cpu=readback_to_cpu).reshape(-1)
        dev = "cpu" if readback_to_cpu else C._gpu(blob, C._check_device(compute_device))
        return torch.empty(0, dtype=t.dtype, device=dev)
    j0, j1 = plan_chunk_ranges(t.n, t.chunk_bytes, world)[rank]
    part = split_chunk_range(blob, j0, j1)
    return decompress_tensor(part, compute_device=compute_device, readback_to_cpu=readback_to_cpu)


def gather_chunk_ranges(part: torch.Tensor | None, dst: int = 0, group=None) -> list[torch.Tensor | None] | None:
    """Bring every rank's part (compress_chunk_range) to rank `dst`, in rank order; other ranks
    get None.  Sizes go by an object all-gather, then each part by a point-to-point send (NCCL
    parts live on the rank's current GPU, gloo parts on the CPU).  This is the one data exchange
    of chunk-range sharding: the whole blob is assembled on one rank."""
    import torch.distributed as dist

    world, me = dist.get_world_size(group), dist.get_rank(group)
    dev = (torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl"
           else torch.device("cpu"))
    sizes: list[int | None] = [None] * world
    dist.all_gather_object(sizes, -1 if part is None else int(part.numel()), group=group)
    glob = (lambda r: r) if group is None else (lambda r: dist.get_global_rank(group, r))
    if me != dst:
        if part is not None and part.numel():
            dist.send(part.to(dev).contiguous(), dst=glob(dst), group=group)
        return None
    out: list[torch.Tensor | None] = []
    for r in range(world):
        size = sizes[r]
        if r == me:
            out.append(part)
        elif size is None or size < 0:
            out.append(None)
        else:
            buf = torch.empty(size, dtype=torch.uint8, device=dev)
            if size:
                dist.recv(buf, src=glob(r), group=group)
            out.append(buf)
    return out
