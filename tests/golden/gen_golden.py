"""Generate the golden fixtures in this folder from the reference's own code.

Run (in a container that has the reference checkout; nothing else reads it):

    python tests/golden/gen_golden.py /path/to/cuZipNN

It imports, from the reference checkout (ruihe774/cuZipNN):
  - src/cuzipnn/_kernels.py, run by Triton's CPU interpreter (TRITON_INTERPRET=1), for the
    byte-plane split / merge / chunk-copy vectors;
  - src/cuzipnn/_codec.py, run on the CPU, for whole blobs.  Its entropy coder (nvCOMP, absent)
    is replaced by a stand-in module that calls the oracle's ZNR2 rANS coder, so each blob is
    the reference's container, passthrough rule, tables, padding and CRC logic wrapped around
    the oracle's payloads.  The oracle's own compressor must reproduce these blobs byte for
    byte (with the version byte set to the reference's 2).

The outputs are small .npz files committed beside this script.  Inputs are seeded and stored in
the fixtures, so the tests never need the reference or this script.
"""

from __future__ import annotations

import contextlib
import ctypes
import importlib.util
import os
import sys
import types
import zlib

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402


def _load(name: str, path: str) -> types.ModuleType:
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _fake_nvcomp() -> types.ModuleType:
    """Stand-in for src/cuzipnn/_nvcomp.py with the same names, on host addresses."""
    m = types.ModuleType("refzn._nvcomp")
    m.NVCOMP_TYPE_CHAR = 0
    m.NVCOMP_SUCCESS = 0
    m.MAX_CHUNK_BYTES = 1 << 24
    m.DECOMPRESS_INPUT_ALIGNMENT = 8
    m.MIN_SUB_CHUNKS = 4
    m.MAX_SUB_CHUNKS = 64

    def max_compressed_chunk_bytes(chunk_bytes, sub_chunks):
        return O.ans_max_payload(chunk_bytes, sub_chunks)

    def compress(in_ptrs, in_bytes, chunk_bytes, total_bytes, out_ptrs, out_bytes, statuses, sub_chunks):
        for i in range(in_ptrs.numel()):
            data = ctypes.string_at(int(in_ptrs[i]), int(in_bytes[i]))
            payload = O.ans_encode(data, sub_chunks)
            ctypes.memmove(int(out_ptrs[i]), payload, len(payload))
            out_bytes[i] = len(payload)
            statuses[i] = 0

    def decompress(in_ptrs, in_bytes, out_capacity, chunk_bytes, total_bytes, out_ptrs):
        for i in range(in_ptrs.numel()):
            data = ctypes.string_at(int(in_ptrs[i]), int(in_bytes[i]))
            sym = O.ans_decode(data, int(out_capacity[i]))
            ctypes.memmove(int(out_ptrs[i]), sym.tobytes(), sym.size)

    def crc32(in_ptrs, in_bytes, max_bytes, out):
        for i in range(in_ptrs.numel()):
            out[i] = zlib.crc32(ctypes.string_at(int(in_ptrs[i]), int(in_bytes[i])))

    m.max_compressed_chunk_bytes = max_compressed_chunk_bytes
    m.compress = compress
    m.decompress = decompress
    m.crc32 = crc32
    return m


def load_reference(ref_root: str):
    src = os.path.join(ref_root, "src", "cuzipnn")
    pkg = types.ModuleType("refzn")
    pkg.__path__ = [src]
    sys.modules["refzn"] = pkg
    pkg._nvcomp = sys.modules["refzn._nvcomp"] = _fake_nvcomp()
    pkg._kernels = _load("refzn._kernels", os.path.join(src, "_kernels.py"))
    codec = _load("refzn._codec", os.path.join(src, "_codec.py"))
    # Run the orchestration on the CPU: the "GPU" is the host, and CUDA device scopes are no-ops.
    codec._gpu = lambda x, compute_device: torch.device("cpu")
    torch.cuda.device = lambda device: contextlib.nullcontext()
    return pkg._kernels, codec


_INT = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def raw_bytes_of(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    return t.reshape(-1).view(_INT[t.element_size()]).numpy().view(np.uint8).copy()


def make(kind: str, n: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    if kind in ("bfloat16", "float16", "float32", "float64"):
        return (torch.randn(n, generator=g) * 0.02).to(getattr(torch, kind))
    if kind == "float32_unit":
        return torch.randn(n, generator=g)
    if kind == "float8_e4m3fn":
        return (torch.randn(n, generator=g) * 16).clamp(-448, 448).to(torch.float8_e4m3fn)
    if kind == "float8_e5m2":
        return torch.randn(n, generator=g).to(torch.float8_e5m2)
    if kind == "bool":
        return torch.rand(n, generator=g) < 0.3
    if kind == "complex64":
        return torch.randn(n, dtype=torch.complex64, generator=g)
    if kind == "int8_mixed":
        parts = [
            torch.randint(0, 256, (4096,), dtype=torch.uint8, generator=g) if i % 2 == 0
            else torch.zeros(4096, dtype=torch.uint8)
            for i in range(n)
        ]
        return torch.cat(parts + [torch.randint(0, 256, (13,), dtype=torch.uint8, generator=g)])
    if kind == "zeros_bf16":
        return torch.zeros(n, dtype=torch.bfloat16)
    if kind == "bits_bf16":
        return torch.randint(-32768, 32767, (n,), dtype=torch.int16, generator=g).view(torch.bfloat16)
    if kind == "bits_f32":
        return torch.randint(-2**31, 2**31 - 1, (n,), dtype=torch.int32, generator=g).view(torch.float32)
    return torch.randint(-100, 100, (n,), generator=g).to(getattr(torch, kind))


# (name, kind, n, shape or None, compress kwargs)
BLOB_CASES = [
    ("bf16_4k", "bfloat16", 20000, None, dict(chunk_bytes=4096)),
    ("f32_4k", "float32", 10007, None, dict(chunk_bytes=4096)),
    ("f32_unit_default", "float32_unit", 133000, None, dict()),
    ("f16_4k_sub1000", "float16", 9000, None, dict(chunk_bytes=4096, sub_chunk_bytes=1000)),
    ("f64_4k", "float64", 3001, None, dict(chunk_bytes=4096)),
    ("fp8_4k", "float8_e4m3fn", 30000, None, dict(chunk_bytes=4096)),
    ("fp8e5m2_4k", "float8_e5m2", 7000, None, dict(chunk_bytes=4096)),
    ("int8_mixed", "int8_mixed", 7, None, dict(chunk_bytes=4096)),
    ("bool", "bool", 5003, None, dict(chunk_bytes=4096)),
    ("int16", "int16", 6000, None, dict(chunk_bytes=4096)),
    ("int32", "int32", 5000, None, dict(chunk_bytes=4096)),
    ("int64", "int64", 3000, None, dict(chunk_bytes=4096)),
    ("uint16", "uint16", 2500, None, dict(chunk_bytes=4096)),
    ("uint32", "uint32", 2500, None, dict(chunk_bytes=4096)),
    ("uint64", "uint64", 2500, None, dict(chunk_bytes=4096)),
    ("c64", "complex64", 2000, None, dict(chunk_bytes=4096)),
    ("zeros_default", "zeros_bf16", 300000, None, dict()),
    ("bits_bf16", "bits_bf16", 20001, None, dict(chunk_bytes=4096)),
    ("bits_f32", "bits_f32", 9001, None, dict(chunk_bytes=4096)),
    ("bf16_allraw", "bfloat16", 20000, None, dict(chunk_bytes=4096, passthrough_threshold=1e-9)),
    ("bf16_thr1", "bfloat16", 20000, None, dict(chunk_bytes=4096, passthrough_threshold=1.0)),
    ("bf16_thr05", "bfloat16", 20000, None, dict(chunk_bytes=4096, passthrough_threshold=0.5)),
    ("bf16_sub64", "bfloat16", 70000, None, dict(sub_chunk_bytes=1)),
    ("bf16_sub4", "bfloat16", 70000, None, dict(sub_chunk_bytes=1 << 30)),
    ("f32_one", "float32", 1, None, dict(chunk_bytes=4096)),
    ("bf16_shape", "bfloat16", 17 * 33 * 5, (17, 33, 5), dict(chunk_bytes=4096)),
    ("bf16_0dim", "bfloat16", 1, (), dict()),
    ("bf16_empty", "bfloat16", 0, (3, 0, 5), dict()),
    ("bf16_chunk8", "bfloat16", 1001, None, dict(chunk_bytes=8)),
    ("bf16_chunk_odd", "bfloat16", 5000, None, dict(chunk_bytes=1000)),
    ("stored_f32", "float32", 30 * 40, (30, 40), dict(min_compress_bytes=65536)),
    ("stored_boundary", "bfloat16", 1000, None, dict(min_compress_bytes=2001)),
    ("not_stored_boundary", "bfloat16", 1000, None, dict(min_compress_bytes=2000)),
]

CRC_CASES = [
    ("bf16_4k", 8), ("bf16_4k", 1000), ("bf16_4k", 16384), ("bf16_4k", 1 << 30),
    ("int8_mixed", 1000), ("stored_f32", 1000), ("stored_f32", 16384), ("bf16_empty", 16384),
]


def main(ref_root: str) -> None:
    kernels, codec = load_reference(ref_root)
    out: dict[str, np.ndarray] = {}

    # 1. Byte planes from the reference's Triton split (src/cuzipnn/_kernels.py:134-148).
    for kind, reorder in [
        ("bfloat16", True), ("float32", True), ("float16", False), ("float64", False),
        ("int16", False), ("int32", False), ("int64", False), ("float32_unit", True),
        ("bits_bf16", True), ("bits_f32", True),
    ]:
        x = make(kind, 4099, seed=11)
        n, k = x.numel(), x.element_size()
        stride = n + 37
        planar = torch.zeros(k * stride, dtype=torch.uint8)
        kernels.split(x, planar, stride, reorder)
        out[f"split/{kind}/x"] = raw_bytes_of(x)
        out[f"split/{kind}/meta"] = np.array([n, k, int(reorder), stride], dtype=np.int64)
        out[f"split/{kind}/planar"] = planar.numpy().copy()

    # 2. Merge through an offset table with streams in shuffled places (_kernels.py:151-176).
    for kind, reorder, chunk in [("bfloat16", True, 1000), ("float32", True, 1000),
                                 ("float16", False, 4096), ("int64", False, 512)]:
        x = make(kind, 5003, seed=12)
        n, k = x.numel(), x.element_size()
        nch = -(-n // chunk)
        stride = nch * chunk
        planar = torch.zeros(k * stride, dtype=torch.uint8)
        kernels.split(x, planar, stride, reorder)
        perm = torch.randperm(k * nch, generator=torch.Generator().manual_seed(3))
        base = torch.zeros(k * nch * chunk, dtype=torch.uint8)
        tbl = torch.empty(k * nch, dtype=torch.int64)
        for i in range(k * nch):
            b, j = divmod(i, nch)
            dst = int(perm[i]) * chunk
            base[dst : dst + chunk] = planar[b * stride + j * chunk : b * stride + (j + 1) * chunk]
            tbl[i] = dst
        y = torch.empty_like(x)
        kernels.merge(tbl, base, y.view(-1), chunk, reorder)
        out[f"merge/{kind}/base"] = base.numpy().copy()
        out[f"merge/{kind}/tbl"] = tbl.numpy().copy()
        out[f"merge/{kind}/meta"] = np.array([n, k, int(reorder), chunk], dtype=np.int64)
        out[f"merge/{kind}/out"] = raw_bytes_of(y)
        assert np.array_equal(out[f"merge/{kind}/out"], raw_bytes_of(x))

    # 3. Batched chunk copy, with and without padding (_kernels.py:179-188).
    g = torch.Generator().manual_seed(5)
    src = torch.randint(0, 256, (64 * 1024,), dtype=torch.uint8, generator=g)
    for pad in (False, True):
        dst = torch.full((80 * 1024,), 0xA5, dtype=torch.uint8)
        sizes = torch.tensor([0, 1, 7, 8, 9, 4096, 8191, 12345, 3], dtype=torch.int64)
        soff = torch.tensor([0, 8, 16, 64, 128, 1024, 8192, 24576, 60000], dtype=torch.int64)
        doff = torch.tensor([0, 16, 32, 80, 200, 2048, 16384, 40000, 70000], dtype=torch.int64)
        kernels.copy_chunks(src.data_ptr() + soff, dst.data_ptr() + doff, sizes, 12345, pad)
        key = "copy/pad" if pad else "copy/nopad"
        out[key + "/src"] = src.numpy().copy()
        out[key + "/sizes"] = sizes.numpy()
        out[key + "/soff"] = soff.numpy()
        out[key + "/doff"] = doff.numpy()
        out[key + "/dst"] = dst.numpy().copy()

    # 4. Sub-chunk counts (_codec.py:83-86) and passthrough budgets (_codec.py:74-80).
    sc = []
    for c in (8, 1000, 4096, 16 << 10, 128 << 10, 1 << 24):
        for s in (1, 7, 1000, 2 << 10, 7 << 10, 8 << 10, 32 << 10, 1 << 30):
            sc.append((c, s, codec._sub_chunks(c, s)))
    out["sub_chunks"] = np.array(sc, dtype=np.int64)
    rb = []
    for k, nch, n, c, thr in [(2, 3, 300000, 131072, 0.95), (4, 1, 7, 4096, 0.95),
                              (1, 5, 20000, 4096, 1e-9), (2, 2, 131073, 131072, 0.3333),
                              (8, 4, 16000, 4096, 1.0), (2, 1, 131072, 131072, 0.95)]:
        r = codec._raw_bytes(k, nch, n, c, thr, "cpu")
        rb.append(np.concatenate([[k, nch, n, c], r.numpy()]).astype(np.int64))
    out["raw_bytes/count"] = np.array([len(rb)], dtype=np.int64)
    for i, r in enumerate(rb):
        out[f"raw_bytes/{i}"] = r
    out["raw_bytes/thr"] = np.array([0.95, 0.95, 1e-9, 0.3333, 1.0, 0.95], dtype=np.float64)

    # 5. Whole blobs from the reference's _codec (v2) around the oracle's payloads.
    tensors = {}
    for name, kind, n, shape, kw in BLOB_CASES:
        x = make(kind, n, seed=sum(map(ord, name)))
        if shape is not None:
            x = x.reshape(shape)
        kw = dict(kw)
        kw.setdefault("min_compress_bytes", 0)
        blob = codec.compress_tensor(x, **kw)
        y = codec.decompress_tensor(blob.clone())
        assert y.dtype == x.dtype and tuple(y.shape) == tuple(x.shape)
        assert np.array_equal(raw_bytes_of(y), raw_bytes_of(x)), name
        tensors[name] = x
        out[f"blob/{name}/x"] = raw_bytes_of(x)
        out[f"blob/{name}/blob"] = blob.numpy().copy()
        out[f"blob/{name}/shape"] = np.array(list(x.shape), dtype=np.int64)
        out[f"blob/{name}/dtype"] = np.frombuffer(str(x.dtype).split(".")[-1].encode(), dtype=np.uint8)
        full = dict(chunk_bytes=131072, sub_chunk_bytes=8192, passthrough_threshold=0.95)
        full.update(kw)
        out[f"blob/{name}/kw"] = np.array(
            [full["chunk_bytes"], full["sub_chunk_bytes"], full["min_compress_bytes"]], dtype=np.int64
        )
        out[f"blob/{name}/thr"] = np.array([full["passthrough_threshold"]], dtype=np.float64)

    # 6. Checksums of whole blobs (compress_tensor_with_crc32, _codec.py:176-208, :116-147).
    for name, seg in CRC_CASES:
        kw = dict(next(c[4] for c in BLOB_CASES if c[0] == name))
        kw.setdefault("min_compress_bytes", 0)
        blob, crc = codec.compress_tensor_with_crc32(tensors[name], checksum_chunk_bytes=seg, **kw)
        assert np.array_equal(blob.numpy(), out[f"blob/{name}/blob"])
        out[f"crc/{name}/{seg}"] = crc.numpy().astype(np.uint32)

    path = os.path.join(HERE, "reference_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: gen_golden.py /path/to/cuZipNN (the reference checkout)")
    main(sys.argv[1])
