"""zn_crc32_noalloc: the CRC-32 entry point that allocates no device memory.

It exists for callers that cannot allocate on the GPU: code running in a process whose device
memory is already held by another allocator (a serving engine that reserved it for weights and KV
cache), and C hosts that only hold the pointers they were handed.  Its scratch is a fixed 2 MiB
array in device memory that all calls share and that keeps the previous call's contents.

The GPU test calls it through the C ABI twice in a row, on different sizes and segment lengths,
and requires the same CRCs (bit for bit) as zn_crc32 with a caller-allocated temp buffer, and as
zlib.  It must pass alone in a fresh process (the first call then also loads the device code) and
after the other tests: the file name makes pytest collect it last, and one test re-runs it in a
fresh Python process.
"""

import os
import subprocess
import sys
import zlib

import numpy as np
import pytest
import torch

from cuzipnn_b200 import _lib

SCRATCH_SLOTS = 1 << 19  # the fixed scratch: one slot per 32 KiB block of a long segment


def _crc_with_temp(buf: torch.Tensor, seg: int, stream: int) -> torch.Tensor:
    n = buf.numel()
    out = torch.empty(-(-n // seg), dtype=torch.int32, device=buf.device)
    tb = _lib.lib.zn_crc32_temp_bytes(n, seg)
    temp = torch.empty(max(tb, 1), dtype=torch.uint8, device=buf.device)
    _lib.check(_lib.lib.zn_crc32(buf.data_ptr(), n, seg, out.data_ptr(), temp.data_ptr(), tb, stream), "zn_crc32")
    return out


@pytest.mark.gpu
def test_noalloc_crc_equals_zn_crc32_on_consecutive_calls():
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(2024)
    # (bytes, segment, offset): a long-segment call, then a smaller one that reuses fewer scratch
    # slots than the first left behind, then segments short enough to skip the scratch.
    cases = [((9 << 20) + 77, (1 << 20) + 3, 3), ((3 << 20) + 5, 100_000, 0), (1_000_001, 20_000, 1)]
    for nbytes, seg, off in cases:
        assert -(-nbytes // seg) * -(-min(seg, nbytes) // 32768) <= SCRATCH_SLOTS
        host = rng.integers(0, 256, nbytes, dtype=np.uint8)
        store = torch.empty(nbytes + 16, dtype=torch.uint8, device="cuda")
        buf = store[off : off + nbytes]
        buf.copy_(torch.from_numpy(host))
        ref = _crc_with_temp(buf, seg, stream)
        out = torch.zeros_like(ref)
        torch.cuda.synchronize()
        allocs = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        rc = _lib.lib.zn_crc32_noalloc(buf.data_ptr(), nbytes, seg, out.data_ptr(), stream)
        _lib.check(rc, "zn_crc32_noalloc")
        torch.cuda.synchronize()
        assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == allocs
        assert torch.equal(out, ref), (nbytes, seg)
        zl = [zlib.crc32(host[i : i + seg].tobytes()) for i in range(0, nbytes, seg)]
        assert (out.cpu().numpy().view(np.uint32).tolist()) == zl, (nbytes, seg)


def test_noalloc_crc_rejects_sizes_beyond_its_scratch():
    # Checked on the host before any CUDA call, so this needs no GPU: 2^18 + 1 segments of 64 KiB
    # need 2^19 + 2 slots.  Null pointers show that nothing is read or launched.
    before = _lib.launch_count()
    nbytes = (1 << 34) + (1 << 16)
    rc = _lib.lib.zn_crc32_noalloc(None, nbytes, 1 << 16, None, None)
    assert rc == _lib.ZN_ERR_INVALID
    msg = _lib.lib.zn_last_error().decode()
    assert "scratch" in msg and str(SCRATCH_SLOTS) in msg and "zn_crc32" in msg
    assert _lib.launch_count() == before
    # Bad arguments are refused the same way.
    assert _lib.lib.zn_crc32_noalloc(None, -1, 4096, None, None) == _lib.ZN_ERR_INVALID
    assert _lib.lib.zn_crc32_noalloc(None, 10, 0, None, None) == _lib.ZN_ERR_INVALID
    assert _lib.lib.zn_crc32_noalloc(None, 0, 4096, None, None) == _lib.ZN_OK


@pytest.mark.gpu
def test_noalloc_crc_in_a_fresh_process():
    """The consecutive-calls test again, alone in a new Python process."""
    node = os.path.abspath(__file__) + "::test_noalloc_crc_equals_zn_crc32_on_consecutive_calls"
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider", node],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "1 passed" in r.stdout


@pytest.mark.gpu
def test_noalloc_crc_at_exactly_the_scratch_size():
    """2^18 segments of 32 KiB + 1 bytes need exactly 2^19 scratch slots (two blocks each): accepted,
    and equal to zn_crc32."""
    seg = 32768 + 1
    nseg = SCRATCH_SLOTS // 2
    nbytes = seg * nseg
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(9)
    buf = torch.randint(0, 256, (nbytes,), generator=g, device="cuda", dtype=torch.uint8)
    ref = _crc_with_temp(buf, seg, stream)
    out = torch.zeros_like(ref)
    _lib.check(_lib.lib.zn_crc32_noalloc(buf.data_ptr(), nbytes, seg, out.data_ptr(), stream), "zn_crc32_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    host = buf[-2 * seg:].cpu().numpy()
    assert out[-2:].cpu().numpy().view(np.uint32).tolist() == [zlib.crc32(host[:seg].tobytes()),
                                                              zlib.crc32(host[seg:].tobytes())]
    del buf
    # One byte more adds a segment of one byte, which needs two more slots: refused.
    assert _lib.lib.zn_crc32_noalloc(None, nbytes + 1, seg, None, None) == _lib.ZN_ERR_INVALID


def test_noalloc_crc_boundary_on_the_host():
    """The size check at the limit, with null pointers (nothing may be launched): one slot over the
    limit is refused with the scratch message, and a call at exactly the limit passes that check."""
    before = _lib.launch_count()
    # 2^19 + 1 slots: 2^19 + 1 segments of 32 KiB + 1 bytes would be 2 slots each, so use one
    # segment of (2^19 + 1) * 32 KiB bytes: one slot per 32 KiB block.
    over = (SCRATCH_SLOTS + 1) * 32768
    assert _lib.lib.zn_crc32_noalloc(None, over, over, None, None) == _lib.ZN_ERR_INVALID
    assert "scratch" in _lib.lib.zn_last_error().decode()
    assert _lib.launch_count() == before
    if torch.cuda.is_available():
        return  # at the limit the call would go on to launch on the null pointers
    at = SCRATCH_SLOTS * 32768
    rc = _lib.lib.zn_crc32_noalloc(None, at, at, None, None)
    assert rc != _lib.ZN_OK  # no GPU here: the symbol lookup fails, after the size check
    assert "need" not in _lib.lib.zn_last_error().decode()
    assert _lib.launch_count() == before
