"""Several host threads on one GPU, each on its own stream: results stay exact, and each thread's
last_decode_status() reports its own calls only (the status words are kept per thread)."""

import threading

import pytest
import torch

import cuzipnn_b200 as z

pytestmark = pytest.mark.gpu


def test_threads_keep_their_own_results_and_status():
    g = torch.Generator(device="cuda").manual_seed(31)
    xs = [(torch.randn(300_000 + 7 * i, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for i in range(4)]
    blobs = [z.compress_tensor(x, chunk_bytes=4096, min_compress_bytes=0, readback_to_cpu=False) for x in xs]
    bad = blobs[0].clone()
    bad[40:44] = torch.tensor([0xFF, 0xFF, 0xFF, 0x7F], dtype=torch.uint8, device="cuda")  # a unit past the end
    torch.cuda.synchronize()
    start = threading.Barrier(3)
    out: dict[str, object] = {}

    def good(name, rounds=30):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                start.wait()
                ok = True
                for _ in range(rounds):
                    ys = [z.decompress_tensor(b) for b in blobs]
                    bs = z.compress_tensors(xs, chunk_bytes=4096, min_compress_bytes=0, readback_to_cpu=False)
                    ys2 = z.decompress_tensors(bs)
                    st = z.last_decode_status()
                    ok &= st == 0 and all(torch.equal(y.view(torch.int16), x.view(torch.int16))
                                          for y, x in zip(ys + ys2, xs + xs))
                out[name] = ok
        except Exception as e:  # reported by the main thread
            out[name] = e

    def corrupt(rounds=30):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                start.wait()
                sts = []
                for _ in range(rounds):
                    z.decompress_tensor(bad)
                    sts.append(z.last_decode_status())
                out["bad"] = all(v != 0 for v in sts)
        except Exception as e:
            out["bad"] = e

    threads = [threading.Thread(target=good, args=("a",)), threading.Thread(target=good, args=("b",)),
               threading.Thread(target=corrupt)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(300)
    torch.cuda.synchronize()
    assert out == {"a": True, "b": True, "bad": True}, out
    assert z.last_decode_status() == 0  # this thread decoded nothing
