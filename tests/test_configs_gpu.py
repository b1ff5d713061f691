"""The benchmark configurations at full size on the GPU, through size-independent properties: every
tensor round-trips bit for bit, the compression ratio sits just above the order-0 entropy bound of
the synthetic weights (the same bound the reference's nvCOMP coder is held to), CRCs of the blobs
verify, and sampled tensors equal the oracle's blobs byte for byte.

The 7B bf16 decoder (the benchmark workload) is checked the same way: every tensor through the
batched calls and through compress_tensor one at a time, and the oracle's blobs for a q_proj, a
down_proj, a stored norm and a 16-chunk range of the embedding."""

import math
import os
import sys

import numpy as np
import pytest
import torch

import cuzipnn_b200 as z
from oracle import oracle as O

sys.path.insert(0, os.path.dirname(__file__))
import model_configs as M  # noqa: E402

pytestmark = pytest.mark.gpu

_NAMES = {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.float16: "float16",
          torch.float8_e4m3fn: "float8_e4m3fn"}


def _bits(t):
    t = t.contiguous().view(-1)
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


def _nbytes(ts):
    return sum(t.numel() * t.element_size() for t in ts)


def _round_trip(model):
    blobs = z.compress_tensors(model, readback_to_cpu=False)
    outs = z.decompress_tensors(blobs)
    torch.cuda.synchronize()
    assert z.last_decode_status() == 0
    for i, (x, y) in enumerate(zip(model, outs)):
        assert y.dtype == x.dtype and y.shape == x.shape, i
        assert torch.equal(_bits(y), _bits(x)), i
    return blobs


def _oracle_check(model, blobs, idx):
    for i in idx:
        x = model[i].cpu()
        raw = x.contiguous().view(-1).view(torch.uint8).numpy()
        ref = O.compress(raw, x.shape, _NAMES[x.dtype], threads=os.cpu_count() or 1)
        assert np.array_equal(blobs[i].cpu().numpy(), np.frombuffer(ref, dtype=np.uint8)), i


def test_config1_fp32_4096x4096_cpu_blob_to_gpu():
    """torch.manual_seed(0); randn(4096, 4096) on the CPU, defaults: CPU blob, decompress to the
    GPU, torch.equal.  Order-0 bound of N(0, 1) fp32: 83.0 %."""
    torch.manual_seed(0)
    x = torch.randn(4096, 4096)
    blob = z.compress_tensor(x)
    assert not blob.is_cuda
    y = z.decompress_tensor(blob, compute_device="cuda")
    assert y.is_cuda and torch.equal(y.cpu(), x)
    ratio = blob.numel() / (x.numel() * 4)
    assert 0.829 < ratio < 0.835, ratio
    raw = x.view(-1).view(torch.uint8).numpy()
    assert blob.numpy().tobytes() == O.compress(raw, x.shape, "float32", threads=os.cpu_count() or 1)


def test_config3_t5_3b_fp32():
    model = M.build(M.t5_3b_fp32(), "cuda")
    assert len(model) == 558 and abs(_nbytes(model) - 11.40e9) < 0.01e9
    blobs = _round_trip(model)
    ratio = sum(b.numel() for b in blobs) / _nbytes(model)
    assert 0.829 < ratio < 0.835, ratio  # order-0 bound 83.0 %
    _oracle_check(model, blobs, [1, 2, 5, len(model) - 2])


def test_config4_qwen_4b_fp8_bf16():
    spec = M.qwen_4b_fp8()
    model = M.build(spec, "cuda")
    assert len(model) == 651 and abs(_nbytes(model) - 5.19e9) < 0.01e9
    blobs = _round_trip(model)
    fp8 = [i for i, t in enumerate(model) if t.dtype == torch.float8_e4m3fn]
    r8 = sum(blobs[i].numel() for i in fp8) / _nbytes([model[i] for i in fp8])
    assert 0.809 < r8 < 0.82, r8  # order-0 bound of the fp8 weights 80.9 %
    ratio = sum(b.numel() for b in blobs) / _nbytes(model)
    assert 0.75 < ratio < 0.79, ratio
    _oracle_check(model, blobs, [fp8[0], fp8[0] + 1, 3])


def test_config5_whisper_fp16_with_crc():
    """compress_tensor_with_crc32 (16 KiB segments) on every tensor, hash_tensor_with_crc32
    verification of every blob, then the batched round trip."""
    model = M.build(M.whisper_1b5_fp16(), "cuda")
    assert abs(_nbytes(model) - 3.087e9) < 0.01e9
    total = 0
    for i, x in enumerate(model):
        blob, crc = z.compress_tensor_with_crc32(x, checksum_chunk_bytes=16384, readback_to_cpu=False)
        assert torch.equal(z.hash_tensor_with_crc32(blob, checksum_chunk_bytes=16384, readback_to_cpu=False), crc), i
        total += blob.numel()
    ratio = total / _nbytes(model)
    assert 0.841 < ratio < 0.85, ratio  # order-0 bound of N(0, 0.02) fp16: 84.1 %
    _round_trip(model)


@pytest.mark.parametrize("dtype", [torch.bool, torch.int8, torch.int16, torch.int32, torch.int64, torch.uint8,
                                   torch.uint16, torch.uint32, torch.uint64, torch.float64, torch.float8_e5m2,
                                   torch.complex64])
def test_dtype_sweep_64mib_uniform(dtype):
    """64 MiB of uniform random bits per dtype: incompressible planes take the passthrough path,
    bool compresses to about an eighth."""
    g = torch.Generator(device="cuda").manual_seed(5)
    nbytes = 64 << 20
    if dtype == torch.bool:
        x = torch.randint(0, 2, (nbytes,), generator=g, device="cuda").bool()
    else:
        x = torch.randint(0, 256, (nbytes,), generator=g, device="cuda", dtype=torch.uint8).view(dtype)
    blob = z.compress_tensor(x, readback_to_cpu=False)
    y = z.decompress_tensor(blob)
    assert z.last_decode_status() == 0
    assert torch.equal(y.view(torch.uint8), x.view(torch.uint8))
    ratio = blob.numel() / nbytes
    if dtype == torch.bool:
        assert 0.12 < ratio < 0.135, ratio
    else:
        assert 0.99 < ratio < 1.001, ratio


def test_config2_7b_bf16_headline():
    """The 7B GQA decoder in bf16 (339 tensors, 15.23 GB), the workload bench.py measures."""
    import bench

    shapes = bench.model_shapes()
    model = bench.build_model("cuda")
    assert len(model) == 339 and abs(_nbytes(model) - 15.23e9) < 0.01e9
    blobs = _round_trip(model)
    ratio = sum(b.numel() for b in blobs) / _nbytes(model)
    assert 0.661 < ratio < 0.663, ratio  # order-0 bound of N(0, 0.02) bf16: 65.91 %
    # compress_tensor one tensor at a time gives the same blobs as the batched call.
    for i, x in enumerate(model):
        assert torch.equal(z.compress_tensor(x, readback_to_cpu=False), blobs[i]), i
    names = [n for n, _, _ in shapes]
    q = names.index("model.layers.3.self_attn.q_proj.weight")
    down = names.index("model.layers.27.mlp.down_proj.weight")
    norm = names.index("model.layers.5.input_layernorm.weight")
    assert blobs[norm].numel() == 24 + 8 + 3584 * 2  # the stored path
    _oracle_check(model, blobs, [q, down, norm])
    # Chunks 2000 .. 2015 of the embedding (152064 x 3584): the oracle's blob of those elements.
    emb = names.index("model.embed_tokens.weight")
    j0, j1, C = 2000, 2016, 131072
    part = z.split_chunk_range(blobs[emb], j0, j1)
    raw = model[emb].view(-1)[j0 * C : j1 * C].cpu().view(torch.uint8).numpy()
    ref = O.compress(raw, (raw.size // 2,), "bfloat16", min_compress_bytes=0, threads=os.cpu_count() or 1)
    assert np.array_equal(part.cpu().numpy(), np.frombuffer(ref, dtype=np.uint8))
