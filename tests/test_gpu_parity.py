"""CUDA path against the oracle and the reference-generated golden vectors (bit-exact).

Every test here runs the library through its C ABI (via the package's ctypes binding) on a GPU
and compares bytes: blobs against the reference container produced by the reference's own
_codec.py (tests/golden), ZNR2 payloads against the oracle's encoder, planes against the
reference's Triton split, CRCs against zlib.
"""

import zlib

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

_TORCH = {
    "bool": torch.bool, "uint8": torch.uint8, "int8": torch.int8, "int16": torch.int16,
    "int32": torch.int32, "int64": torch.int64, "float16": torch.float16,
    "bfloat16": torch.bfloat16, "float32": torch.float32, "float64": torch.float64,
    "float8_e4m3fn": torch.float8_e4m3fn, "float8_e5m2": torch.float8_e5m2,
    "uint16": torch.uint16, "uint32": torch.uint32, "uint64": torch.uint64,
    "complex64": torch.complex64,
}


def _tensor(raw: np.ndarray, dtype: str, shape) -> torch.Tensor:
    if raw.size == 0:
        return torch.empty(tuple(shape), dtype=_TORCH[dtype])
    t = torch.from_numpy(raw.copy()).view(_TORCH[dtype])
    return t.reshape(tuple(shape))


def _u8(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous().reshape(-1)
    return t.view(torch.uint8).numpy() if t.numel() else np.zeros(0, np.uint8)


def _blob_names(golden):
    return sorted({k.split("/")[1] for k in golden if k.startswith("blob/")})


@pytest.fixture(scope="module")
def z():
    import cuzipnn_b200

    return cuzipnn_b200


def test_blobs_equal_reference_container(golden, z):
    """compress_tensor on the GPU == the reference's _codec.py blob (version byte 3)."""
    for name in _blob_names(golden):
        raw = golden[f"blob/{name}/x"]
        dtype = golden[f"blob/{name}/dtype"].tobytes().decode()
        shape = golden[f"blob/{name}/shape"].tolist()
        chunk, sub, minc = golden[f"blob/{name}/kw"].tolist()
        thr = float(golden[f"blob/{name}/thr"][0])
        ref = golden[f"blob/{name}/blob"].copy()
        ref[4] = 3
        x = _tensor(raw, dtype, shape).cuda()
        blob = z.compress_tensor(x, chunk_bytes=chunk, sub_chunk_bytes=sub, passthrough_threshold=thr,
                                 min_compress_bytes=minc)
        assert np.array_equal(_u8(blob), ref), name
        y = z.decompress_tensor(blob)
        assert y.dtype == x.dtype and tuple(y.shape) == tuple(x.shape)
        assert np.array_equal(_u8(y), raw), name
        assert z.last_decode_status() == 0, name


@pytest.mark.parametrize(
    "dtype,n,chunk,sub",
    [
        ("bfloat16", 1_000_003, 131072, 8192),
        ("float32", 300_001, 131072, 8192),
        ("float16", 500_000, 4096, 1000),
        ("float8_e4m3fn", 700_001, 131072, 2048),
        ("bfloat16", 262144, 131072, 1 << 30),
        ("bfloat16", 200_000, 640, 8192),
        ("int32", 100_000, 4096, 8192),
        ("float64", 50_000, 4096, 8192),
        ("int16", 300_001, 131072, 8192),
    ],
)
def test_gpu_blob_equals_oracle(z, dtype, n, chunk, sub):
    g = torch.Generator().manual_seed(n)
    if dtype.startswith("float8"):
        x = (torch.randn(n, generator=g) * 16).clamp(-448, 448).to(_TORCH[dtype])
    elif dtype == "int32":
        x = torch.randint(-1000, 1000, (n,), generator=g, dtype=torch.int32)
    elif dtype == "int16":  # skewed low byte (coded), uniform high byte (raw): a coded first plane
        b = torch.empty(2 * n, dtype=torch.uint8)
        b[0::2] = (torch.randn(n, generator=g).abs() * 3).clamp(max=255).to(torch.uint8)
        b[1::2] = torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8)
        x = b.view(torch.int16)
    else:
        x = (torch.randn(n, generator=g) * 0.02).to(_TORCH[dtype])
    ref = O.compress(_u8(x), x.shape, dtype, chunk_bytes=chunk, sub_chunk_bytes=sub, min_compress_bytes=0,
                     threads=8)
    blob = z.compress_tensor(x.cuda(), chunk_bytes=chunk, sub_chunk_bytes=sub, min_compress_bytes=0)
    assert np.array_equal(_u8(blob), np.frombuffer(ref, dtype=np.uint8))
    assert np.array_equal(_u8(z.decompress_tensor(blob)), _u8(x))
    # And the GPU decodes the oracle's blob.
    y = z.decompress_tensor(torch.frombuffer(bytearray(ref), dtype=torch.uint8).cuda())
    assert np.array_equal(_u8(y), _u8(x))


@pytest.mark.parametrize("dtype", ["bfloat16", "float32", "float64"])
def test_overflow_pass_many_chunks(z, dtype):
    """Every chunk has several coded planes (16 distinct values: the low mantissa planes hold one
    symbol each), so every chunk goes to the overflow pass, whose CTAs (as many as fit on the GPU)
    decode several chunks each."""
    g = torch.Generator().manual_seed(5)
    n = 1 << 21
    x = (torch.randint(0, 16, (n,), generator=g).double() * 0.125).to(_TORCH[dtype])
    ref = O.compress(_u8(x), x.shape, dtype, chunk_bytes=2048, sub_chunk_bytes=2048, min_compress_bytes=0,
                     threads=8)
    blob = z.compress_tensor(x.cuda(), chunk_bytes=2048, sub_chunk_bytes=2048, min_compress_bytes=0)
    assert np.array_equal(_u8(blob), np.frombuffer(ref, dtype=np.uint8))
    y = z.decompress_tensor(blob)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    assert np.array_equal(_u8(y), _u8(x))


def test_split_matches_reference(golden):
    from cuzipnn_b200 import _kernels

    for kind in sorted({k.split("/")[1] for k in golden if k.startswith("split/")}):
        n, k, reorder, stride = golden[f"split/{kind}/meta"].tolist()
        x = torch.from_numpy(golden[f"split/{kind}/x"].copy()).cuda()
        x = x.view({1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[k])
        planar = torch.zeros(k * stride, dtype=torch.uint8, device="cuda")
        _kernels.split(x, planar, stride, bool(reorder))
        assert np.array_equal(planar.cpu().numpy(), golden[f"split/{kind}/planar"]), kind


def test_merge_matches_reference(golden):
    from cuzipnn_b200 import _kernels

    for kind in sorted({k.split("/")[1] for k in golden if k.startswith("merge/")}):
        n, k, reorder, chunk = golden[f"merge/{kind}/meta"].tolist()
        base = torch.from_numpy(golden[f"merge/{kind}/base"].copy()).cuda()
        tbl = torch.from_numpy(golden[f"merge/{kind}/tbl"].copy()).cuda()
        out = torch.empty(n * k, dtype=torch.uint8, device="cuda")
        out = out.view({1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[k])
        _kernels.merge(tbl, base, out, chunk, bool(reorder))
        assert np.array_equal(_u8(out), golden[f"merge/{kind}/out"]), kind


@pytest.mark.parametrize("pad", [False, True])
def test_copy_chunks_matches_reference(golden, pad):
    from cuzipnn_b200 import _kernels

    key = "copy/pad" if pad else "copy/nopad"
    src = torch.from_numpy(golden[key + "/src"].copy()).cuda()
    dst = torch.full((80 * 1024,), 0xA5, dtype=torch.uint8, device="cuda")
    soff = torch.from_numpy(golden[key + "/soff"].copy()).cuda()
    doff = torch.from_numpy(golden[key + "/doff"].copy()).cuda()
    sizes = torch.from_numpy(golden[key + "/sizes"].copy()).cuda()
    _kernels.copy_chunks(src.data_ptr() + soff, dst.data_ptr() + doff, sizes, 12345, pad)
    assert np.array_equal(dst.cpu().numpy(), golden[key + "/dst"])


def test_crc_matches_reference_and_zlib(golden, z):
    from cuzipnn_b200 import _codec

    for key in [k for k in golden if k.startswith("crc/")]:
        _, name, seg = key.split("/")
        blob = golden[f"blob/{name}/blob"].copy()
        blob[4] = 3
        d = torch.from_numpy(blob).cuda()
        crc = _codec._crc32(d, int(seg)).cpu().numpy()
        # The golden CRCs are of the version-2 blob; the version byte sits in the first segment.
        ref = golden[key].copy()
        ref[0] = zlib.crc32(blob[: int(seg)].tobytes())
        assert np.array_equal(crc, ref), key


@pytest.mark.parametrize("nbytes", [0, 1, 7, 8, 127, 128, 129, 4096, 100_003, 1 << 20, (1 << 20) + 13])
@pytest.mark.parametrize("seg", [1, 8, 100, 1000, 16384, 32768, 32769, 100_000, 1 << 30])
def test_crc_sizes(nbytes, seg):
    from cuzipnn_b200 import _codec

    data = np.random.default_rng(nbytes + seg).integers(0, 256, nbytes + 5, dtype=np.uint8)
    for off in (0, 3):
        d = torch.from_numpy(data[off : off + nbytes].copy())
        buf = torch.empty(nbytes + 16, dtype=torch.uint8, device="cuda")
        view = buf[off : off + nbytes]
        view.copy_(d)
        crc = _codec._crc32(view, seg).cpu().numpy()
        ref = [zlib.crc32(data[off + i : off + min(i + seg, nbytes)].tobytes()) for i in range(0, nbytes, seg)]
        assert crc.tolist() == ref, (nbytes, seg, off)


@pytest.mark.parametrize("sub_chunks", [4, 16, 64])
def test_ans_seam_matches_oracle(sub_chunks):
    from cuzipnn_b200 import _ans

    rng = np.random.default_rng(sub_chunks)
    chunk = 131072
    sizes = [chunk, 1, 8, 4099, 100_000, chunk]
    bufs = [np.clip(rng.normal(0, 6, s) + 120, 0, 255).astype(np.uint8) for s in sizes]
    bufs[-1] = rng.integers(0, 256, chunk, dtype=np.uint8)
    inp = [torch.from_numpy(b).cuda() for b in bufs]
    slot = _ans.max_compressed_chunk_bytes(chunk, sub_chunks)
    outs = [torch.zeros(slot, dtype=torch.uint8, device="cuda") for _ in inp]
    in_ptrs = torch.tensor([t.data_ptr() for t in inp], dtype=torch.int64, device="cuda")
    in_bytes = torch.tensor(sizes, dtype=torch.int64, device="cuda")
    out_ptrs = torch.tensor([t.data_ptr() for t in outs], dtype=torch.int64, device="cuda")
    out_bytes = torch.empty(len(inp), dtype=torch.int64, device="cuda")
    statuses = torch.empty(len(inp), dtype=torch.int32, device="cuda")
    _ans.compress(in_ptrs, in_bytes, chunk, sum(sizes), out_ptrs, out_bytes, statuses, sub_chunks)
    assert statuses.cpu().tolist() == [0] * len(inp)
    for b, o, nb in zip(bufs, outs, out_bytes.cpu().tolist()):
        assert o[:nb].cpu().numpy().tobytes() == O.ans_encode(b, sub_chunks)
    dec = [torch.zeros(s, dtype=torch.uint8, device="cuda") for s in sizes]
    st = _ans.decompress(out_ptrs, out_bytes, in_bytes, chunk, sum(sizes),
                         torch.tensor([t.data_ptr() for t in dec], dtype=torch.int64, device="cuda"))
    assert st.cpu().tolist() == [0] * len(inp)
    for b, d in zip(bufs, dec):
        assert np.array_equal(d.cpu().numpy(), b)


def test_corrupt_blob_sets_status_without_fault(z):
    """A damaged payload is reported through the status word; the GPU keeps working."""
    x = (torch.randn(300_000, device="cuda") * 0.02).to(torch.bfloat16)
    blob = z.compress_tensor(x, chunk_bytes=4096, min_compress_bytes=0)
    bad = blob.clone()
    n = bad.numel()
    bad[n // 2 : n // 2 + 64] ^= 0x5A  # inside some payload or raw unit
    y = z.decompress_tensor(bad)
    torch.cuda.synchronize()
    status = z.last_decode_status()
    # Either the damage hit raw bytes (decodes, differs) or a payload (status set).
    assert status != 0 or not torch.equal(y.view(torch.int16), x.view(torch.int16))
    # Truncated tables: stored sizes pointing past the end of the blob.
    bad2 = blob.clone()
    bad2[40:44] = torch.tensor([0xFF, 0xFF, 0xFF, 0x7F], dtype=torch.uint8)
    z.decompress_tensor(bad2)
    assert z.last_decode_status() != 0
    with pytest.raises(ValueError, match="corrupt"):
        z.decompress_tensor(bad2, readback_to_cpu=True)
    # The context is still usable.
    assert torch.equal(z.decompress_tensor(blob).view(torch.int16), x.view(torch.int16))


@pytest.mark.parametrize("dtype", ["bfloat16", "float32", "float16"])
def test_raw_planes_in_place_guess_right_and_wrong(z, dtype):
    """The encoder writes skipped (raw) planes straight to the blob place they have when every
    chunk codes one plane; the guess fails when some chunks code none (random bits) or more.
    Either way the blob equals the oracle's."""
    g = torch.Generator().manual_seed(3)
    C = 16384
    normal = (torch.randn(6 * C, generator=g) * 0.02).to(_TORCH[dtype])
    noise = torch.randint(0, 256, (6 * C * normal.element_size(),), generator=g, dtype=torch.uint8).view(_TORCH[dtype])
    zeros = torch.zeros(3 * C, dtype=_TORCH[dtype])
    cases = {"all normal": normal, "noise chunks": torch.cat([normal[: 3 * C], noise[: 2 * C], normal[3 * C :]]),
             "zero chunks": torch.cat([zeros, normal[:C + 5]])}
    for name, x in cases.items():
        ref = O.compress(_u8(x), x.shape, dtype, chunk_bytes=C, min_compress_bytes=0, threads=8)
        blob = z.compress_tensor(x.cuda(), chunk_bytes=C, min_compress_bytes=0)
        assert np.array_equal(_u8(blob), np.frombuffer(ref, dtype=np.uint8)), name
        assert np.array_equal(_u8(z.decompress_tensor(blob)), _u8(x)), name


def test_remembered_header_voided_by_in_place_writes(z):
    """GPU blobs made here carry their header fields, so decompressing them reads nothing back to
    the host; an in-place write to the blob (or a view of it) voids that record, so a damaged
    header is still caught, and damaged tables are reported through the status word."""
    x = (torch.randn(300_000, device="cuda") * 0.02).to(torch.bfloat16)
    for make in (lambda: z.compress_tensor(x, readback_to_cpu=False, chunk_bytes=65536),
                 lambda: z.compress_tensors([x, x[:1000]], readback_to_cpu=False, chunk_bytes=65536)[0]):
        blob = make()
        assert torch.equal(z.decompress_tensor(blob).view(torch.int16), x.view(torch.int16))
        assert torch.equal(z.decompress_tensors([blob])[0].view(torch.int16), x.view(torch.int16))
        blob[0] = 0  # the magic, through the tensor: the record no longer applies
        with pytest.raises(ValueError, match="not a cuzipnn blob"):
            z.decompress_tensor(blob)
        with pytest.raises(ValueError, match="not a cuzipnn blob"):
            z.decompress_tensors([blob])
        blob2 = make()
        blob2[12:16].view(torch.int32).fill_(1 << 30)  # n_comp far beyond the blob, via a view
        with pytest.raises(ValueError, match="truncated"):
            z.decompress_tensor(blob2)


def test_device_read_n_comp_with_truncated_blob(z):
    """zn_decompress with n_comp = -1 reads it from the blob on the device; tables that do not fit
    the blob are reported (kErrTable) and the output is zero-filled, with no fault."""
    from cuzipnn_b200 import _lib

    x = (torch.randn(200_000, device="cuda") * 0.02).to(torch.bfloat16)
    blob = z.compress_tensor(x, readback_to_cpu=False)
    n, k = x.numel(), 2
    s = torch.cuda.current_stream().cuda_stream
    tb = _lib.lib.zn_decompress_temp_bytes(n, k, 131072)
    temp = torch.empty(tb, dtype=torch.uint8, device="cuda")
    status = torch.full((1,), 123, dtype=torch.int32, device="cuda")
    for nbytes, want in ((blob.numel(), 0), (40, 4), (8, 4)):  # 4: the table error bit
        out = torch.full_like(x, 1.0)
        rc = _lib.lib.zn_decompress(blob.data_ptr(), nbytes, n, k, 1, 1, 131072, -1, out.data_ptr(),
                                    status.data_ptr(), temp.data_ptr(), tb, s)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) & 4 == want, nbytes
        if want == 0:
            assert int(status.item()) == 0
            assert torch.equal(out.view(torch.int16), x.view(torch.int16))
        else:
            assert int((out.view(torch.int16) != 0).sum()) == 0


@pytest.mark.parametrize("k,reorder", [(1, False), (2, True), (2, False), (4, True), (8, False)])
@pytest.mark.parametrize("xoff,poff,pad", [(0, 0, 0), (8, 0, 0), (0, 8, 8), (0, 3, 5), (-1, 0, 0)])
def test_split_merge_alignment_paths(k, reorder, xoff, poff, pad):
    """zn_split / zn_merge through the C ABI for every vector path: elements 16- or 8-byte aligned,
    or element-aligned only (xoff = -1: offset by one element, the scalar kernels); plane starts
    16-, 8- or 1-byte aligned (planar offset and stride); merge chunks not a multiple of 16 (groups
    that straddle chunks) and sources off 8-byte alignment.  Equal to the oracle byte for byte."""
    from cuzipnn_b200 import _lib

    n = 100_003
    xoff = k if xoff < 0 else xoff
    stride = n + pad
    g = torch.Generator().manual_seed(k * 31 + xoff + poff)
    raw = torch.randint(0, 256, (n * k,), generator=g, dtype=torch.uint8)
    s = torch.cuda.current_stream().cuda_stream
    xbuf = torch.zeros(n * k + 64, dtype=torch.uint8, device="cuda")
    xbuf[xoff : xoff + n * k].copy_(raw)
    pbuf = torch.zeros(k * stride + 64, dtype=torch.uint8, device="cuda")
    assert _lib.lib.zn_split(xbuf.data_ptr() + xoff, n, k, int(reorder), pbuf.data_ptr() + poff, stride, s) == 0
    ref = O.split(raw.numpy(), n, k, reorder, stride)
    assert np.array_equal(pbuf[poff : poff + k * stride].cpu().numpy(), ref)
    # Merge back from planes laid out with chunks of C elements (C a multiple of 8, not of 16 when
    # 1000), read through a base that is 8-byte aligned or not.
    for C, boff in ((1024, 0), (1000, 0), (1024, 3)):
        nch = -(-n // C)
        planes = O.split(raw.numpy(), n, k, reorder, nch * C)  # k planes of stride nch * C
        base = torch.zeros(planes.size + 64, dtype=torch.uint8, device="cuda")
        base[boff : boff + planes.size].copy_(torch.from_numpy(planes))
        tbl = torch.tensor([b * nch * C + j * C for b in range(k) for j in range(nch)], dtype=torch.int64, device="cuda")
        obuf = torch.zeros(n * k + 64, dtype=torch.uint8, device="cuda")
        rc = _lib.lib.zn_merge(tbl.data_ptr(), base.data_ptr() + boff, obuf.data_ptr() + xoff, n, k, C, int(reorder), s)
        assert rc == 0
        assert np.array_equal(obuf[xoff : xoff + n * k].cpu().numpy(), raw.numpy()), (C, boff)
