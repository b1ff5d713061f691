"""The CPU oracle against vectors produced by the reference's own code (tests/golden).

Pins every oracle piece that has a reference counterpart: the byte planes of the Triton split
(src/cuzipnn/_kernels.py:34-54), the merge (:57-105), the chunk copy (:108-131), the sub-chunk
count (src/cuzipnn/_codec.py:83-86), the passthrough budgets (:74-80), whole blobs of the
reference container around ZNR2 payloads (:231-413) and their CRC-32s (:116-147).
"""

import zlib

import numpy as np
import pytest

from oracle import oracle as O

BLOB_NAMES = None


def _names(golden, prefix):
    return sorted({k.split("/")[1] for k in golden if k.startswith(prefix + "/")})


def test_crc_check_value():
    assert O.crc32(b"123456789") == 0xCBF43926 == zlib.crc32(b"123456789")
    data = np.random.default_rng(0).integers(0, 256, 100_003, dtype=np.uint8)
    assert O.crc32(data) == zlib.crc32(data.tobytes())
    assert O.crc32(data[:0]) == 0


def test_split_matches_reference(golden):
    for kind in _names(golden, "split"):
        n, k, reorder, stride = golden[f"split/{kind}/meta"].tolist()
        planar = O.split(golden[f"split/{kind}/x"], n, k, bool(reorder), stride)
        ref = golden[f"split/{kind}/planar"]
        for b in range(k):
            # The reference leaves bytes past n in each stream unwritten (zeros in the fixture).
            assert np.array_equal(planar[b * stride : b * stride + n], ref[b * stride : b * stride + n]), kind


def test_merge_matches_reference(golden):
    for kind in _names(golden, "merge"):
        n, k, reorder, chunk = golden[f"merge/{kind}/meta"].tolist()
        out = O.merge(golden[f"merge/{kind}/tbl"], golden[f"merge/{kind}/base"], n, k, chunk, bool(reorder))
        assert np.array_equal(out, golden[f"merge/{kind}/out"]), kind


@pytest.mark.parametrize("pad", [False, True])
def test_copy_chunks_matches_reference(golden, pad):
    key = "copy/pad" if pad else "copy/nopad"
    dst = np.full(80 * 1024, 0xA5, dtype=np.uint8)
    src = golden[key + "/src"]
    lib = O.lib()
    soff, doff, sizes = (np.ascontiguousarray(golden[key + s]) for s in ("/soff", "/doff", "/sizes"))
    lib.orc_copy_chunks(src.ctypes.data, soff.ctypes.data, dst.ctypes.data, doff.ctypes.data,
                        sizes.ctypes.data, sizes.size, int(pad))
    assert np.array_equal(dst, golden[key + "/dst"])


def test_sub_chunks_matches_reference(golden):
    for c, s, count in golden["sub_chunks"].tolist():
        assert O.sub_chunks(c, s) == count, (c, s)
    # The reference's own known answers (tests/test_roundtrip.py:251-261).
    assert O.sub_chunks(128 << 10, 8 << 10) == 16
    assert O.sub_chunks(128 << 10, 7 << 10) == 32
    assert O.sub_chunks(16 << 10, 8 << 10) == 4
    assert O.sub_chunks(1 << 24, 1) == 64


def test_passthrough_budget_truncates(golden):
    # _codec.py:74-80 builds int64 budgets with torch.full(raw * threshold): truncation.
    thrs = golden["raw_bytes/thr"].tolist()
    for i in range(int(golden["raw_bytes/count"][0])):
        k, nch, n, c, *ref = golden[f"raw_bytes/{i}"].tolist()
        last = n - (nch - 1) * c
        ours = [int(float(c if j < nch - 1 else last) * thrs[i]) for _ in range(k) for j in range(nch)]
        assert ours == ref
    assert int(131072 * 0.95) == 124518


def test_blobs_match_reference_container(golden):
    names = _names(golden, "blob")
    assert len(names) >= 30
    for name in names:
        x = golden[f"blob/{name}/x"]
        shape = tuple(golden[f"blob/{name}/shape"].tolist())
        dtype = golden[f"blob/{name}/dtype"].tobytes().decode()
        chunk, sub, minc = golden[f"blob/{name}/kw"].tolist()
        thr = float(golden[f"blob/{name}/thr"][0])
        ref = golden[f"blob/{name}/blob"]
        ours = O.compress(x, shape, dtype, chunk_bytes=chunk, sub_chunk_bytes=sub,
                          passthrough_threshold=thr, min_compress_bytes=minc, version=2)
        assert ours == ref.tobytes(), name
        # And back: the oracle decodes the reference-packed blob to the original bytes.
        assert np.array_equal(O.decompress(ref, version=2), x), name


def test_blob_crcs_match_reference(golden):
    for key in [k for k in golden if k.startswith("crc/")]:
        _, name, seg = key.split("/")
        blob = golden[f"blob/{name}/blob"]
        assert np.array_equal(O.crc32_segments(blob, int(seg)), golden[key]), key


def test_stored_blob_size_formula(golden):
    # tests/test_roundtrip.py:383 in the reference: a stored blob is 24 + 8 * ndim + nbytes.
    for name in ("stored_f32", "stored_boundary"):
        blob = golden[f"blob/{name}/blob"]
        shape = golden[f"blob/{name}/shape"]
        assert blob.size == 24 + 8 * shape.size + golden[f"blob/{name}/x"].size
        assert blob[7] & 2
    assert not golden["blob/not_stored_boundary/blob"][7] & 2
