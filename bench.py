#!/usr/bin/env python
"""Benchmark of the codec path on the 7B bf16 GQA decoder configuration.

Workload (per GPU): the weights of a 7B GQA decoder in bfloat16 -- 28 layers, hidden 3584, SwiGLU
MLP 18944, 28 query / 4 KV heads of dim 128 with q/k/v biases, RMSNorm vectors of ones, untied
embedding and LM head over a 152064 vocabulary: 339 tensors, 15.23 GB.  Matrices and biases are
N(0, 0.02) seeded per tensor (seed = tensor index), generated on the GPU; there is no checkpoint.

A step compresses every tensor (compress_tensors, blobs kept on the GPU) and decompresses every
blob (decompress_tensors): value = original bytes of all GPUs / step time, in GB/s (1e9).  The
inputs (15 GB) are far larger than the 126 MB L2, so no flush is needed between steps.  With
torchrun each rank processes its own copy of the model (weak scaling); times are the max over
ranks.  The line also reports, measured after the timed steps: `strong` (one copy of the model
over the ranks, plan_model), one tensor at a time on the device, the reference README's own
methodology (GPU tensor -> CPU blob -> GPU, one tensor at a time, best of two passes, wall clock),
`e2e` from pinned host tensors, `micro` (the byte-plane seams and CRC-32 on 1 GiB), the CPU
baseline and the SM clocks seen during the timed region.

--impl reference times the reference's CPU arm: the repository's C restatement of the codec path
(oracle/, the checker), on all host cores, on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

GB = 1e9
HIDDEN, INTER, LAYERS, VOCAB, HEADS, KV_HEADS, HEAD_DIM = 3584, 18944, 28, 152064, 28, 4, 128
WORKLOAD = (
    "7B GQA decoder bf16 weights: 28 layers, hidden 3584, SwiGLU 18944, 28 q / 4 kv heads x 128 with "
    "q/k/v biases, RMSNorm ones, untied embedding + LM head, vocab 152064; 339 tensors, 15.23 GB; "
    "compress_tensors + decompress_tensors (defaults: chunk_bytes 131072, sub_chunk_bytes 8192, "
    "passthrough 0.95, min_compress_bytes 65536)"
)


def model_shapes(layers: int | None = None) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) of the 7B bf16 decoder, in checkpoint order.  With `layers`, only that
    many decoder layers and no embedding / LM head (smaller cases for profiler captures)."""
    kv = KV_HEADS * HEAD_DIM
    full = layers is None
    out = [("model.embed_tokens.weight", (VOCAB, HIDDEN), "normal")] if full else []
    for i in range(LAYERS if full else layers):
        p = f"model.layers.{i}."
        out += [
            (p + "self_attn.q_proj.weight", (HIDDEN, HIDDEN), "normal"),
            (p + "self_attn.q_proj.bias", (HIDDEN,), "normal"),
            (p + "self_attn.k_proj.weight", (kv, HIDDEN), "normal"),
            (p + "self_attn.k_proj.bias", (kv,), "normal"),
            (p + "self_attn.v_proj.weight", (kv, HIDDEN), "normal"),
            (p + "self_attn.v_proj.bias", (kv,), "normal"),
            (p + "self_attn.o_proj.weight", (HIDDEN, HIDDEN), "normal"),
            (p + "mlp.gate_proj.weight", (INTER, HIDDEN), "normal"),
            (p + "mlp.up_proj.weight", (INTER, HIDDEN), "normal"),
            (p + "mlp.down_proj.weight", (HIDDEN, INTER), "normal"),
            (p + "input_layernorm.weight", (HIDDEN,), "ones"),
            (p + "post_attention_layernorm.weight", (HIDDEN,), "ones"),
        ]
    if full:
        out += [("model.norm.weight", (HIDDEN,), "ones"), ("lm_head.weight", (VOCAB, HIDDEN), "normal")]
    return out


def make_tensor(idx: int, shape, init: str, device) -> torch.Tensor:
    if init == "ones":
        return torch.ones(shape, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(idx)
    return (torch.randn(shape, generator=g, device=device) * 0.02).to(torch.bfloat16)


def build_model(device, layers: int | None = None) -> list[torch.Tensor]:
    return [make_tensor(i, s, init, device) for i, (_, s, init) in enumerate(model_shapes(layers))]


def nbytes(ts) -> int:
    return sum(t.numel() * t.element_size() for t in ts)


# ---- measurement helpers ----------------------------------------------------------------------


class ClockSampler:
    """nvidia-smi samples of SM clock, power and throttle reasons.  The sampler starts before the
    warm-up (nvidia-smi takes a while to start, longer with eight of them at once), and only the
    samples stamped inside the timed region (window()) are summarised."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def window(self, t0: float, t1: float) -> None:
        """The timed region, as time.time() values."""
        self.t0, self.t1 = t0, t1

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        import datetime

        rows = []
        try:
            for line in open(self.path):
                f = [v.strip() for v in line.split(",")]
                if len(f) < 10 or not f[2].replace(".", "").isdigit():
                    continue
                try:
                    ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                if self.t0 is None or self.t0 <= ts <= self.t1:
                    rows.append(f[1:])
            os.unlink(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = sorted(float(r[1]) for r in rows)
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": float(rows[0][2]), "reasons": sorted(reasons),
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def measured_hbm_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(path))["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def profile_traffic(kernel: str) -> float | None:
    """DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic byte of a kernel,
    from the `traffic_per_algo_byte:` line of its committed ncu summary profiles/<kernel>_*.md."""
    import glob
    import re

    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", f"{kernel}_*.md"))):
        m = re.search(r"^traffic_per_algo_byte:\s*([0-9.]+)", open(path).read(), re.M)
        if m:
            return float(m.group(1))
    return None


def cpu_round_trip(tensors, threads: int) -> tuple[float, float, int, int]:
    """The oracle's compress + decompress of host tensors: (compress s, decompress s, in, out bytes)."""
    import numpy as np

    from oracle import oracle as O

    raws = [t.cpu().contiguous().view(torch.int16).numpy().view(np.uint8) for t in tensors]
    t0 = time.perf_counter()
    blobs = [O.compress(r, t.shape, "bfloat16", threads=threads) for r, t in zip(raws, tensors)]
    t1 = time.perf_counter()
    for b, r in zip(blobs, raws):
        y = O.decompress(b, threads=threads)
        assert y.size == r.size
    t2 = time.perf_counter()
    return t1 - t0, t2 - t1, sum(r.size for r in raws), sum(len(b) for b in blobs)


def cpu_sample(device="cpu") -> list[torch.Tensor]:
    """Layer 0 of the model (q/k/v/o, gate/up/down, biases, norms): 466 MB, every tensor kind."""
    shapes = model_shapes()
    return [make_tensor(i, s, init, device) for i, (n, s, init) in enumerate(shapes) if ".layers.0." in n]


# ---- micro-benchmarks of the seam and CRC kernels ----------------------------------------------


def micro_benchmarks(device, reps: int = 10) -> dict:
    """Device time (CUDA events, mean of `reps` after 3 warm-up calls) of the byte-plane seam
    kernels on 1 GiB of bf16 N(0, 0.02) (zn_split with the exponent reorder into planes of stride
    nch * 131072, zn_merge back, checked bit for bit) and of zn_crc32 on 1 GiB of random bytes in
    16 KiB segments.  Rates are algorithmic bytes (split / merge: read + write; CRC: read) per
    second, inputs larger than L2."""
    from cuzipnn_b200 import _codec as C
    from cuzipnn_b200 import _kernels as K

    def timed(fn):
        for _ in range(3):
            fn()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps / 1e3

    n, chunk = 1 << 29, 131072
    g = torch.Generator(device=device).manual_seed(11)
    x = (torch.randn(n, generator=g, device=device) * 0.02).to(torch.bfloat16)
    nch = -(-n // chunk)
    stride = nch * chunk
    planar = torch.empty(2 * stride, dtype=torch.uint8, device=device)
    tbl = torch.tensor([b * stride + j * chunk for b in range(2) for j in range(nch)], dtype=torch.int64, device=device)
    y = torch.empty_like(x)
    t_split = timed(lambda: K.split(x, planar, stride, True))
    t_merge = timed(lambda: K.merge(tbl, planar, y, chunk, True))
    assert torch.equal(y.view(torch.int16), x.view(torch.int16))
    del planar, tbl, y
    data = torch.randint(0, 256, (1 << 30,), generator=g, device=device, dtype=torch.uint8)
    t_crc = timed(lambda: C._crc32(data, 16384))
    del data, x
    peak, _ = measured_hbm_peak()
    out = {}
    for name, nbytes, t in (("split", 4 * n, t_split), ("merge", 4 * n, t_merge), ("crc", 1 << 30, t_crc)):
        gbs = nbytes / t / GB
        out[name] = {"gbs": round(gbs, 1), "ms": round(t * 1e3, 4), "frac_of_measured_hbm": round(gbs / peak, 4),
                     "frac_of_8tbs_nominal": round(gbs / 8000, 4)}
    out["workload"] = ("split / merge: 2^29 bf16 (1 GiB), reorder, chunk 131072, read + write bytes; "
                       "crc: 1 GiB random bytes, 16 KiB segments, bytes read")
    return out


# ---- the reference arm --------------------------------------------------------------------------


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample = cpu_sample()
    times = []
    for step in range(args.warmup + args.steps):
        tc, td, nin, nout = cpu_round_trip(sample, threads)
        if step >= args.warmup:
            times.append(tc + td)
    t = sum(times) / len(times)
    value = nin / t / GB
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": "layer 0 (466 MB) per step", "ratio": round(nout / nin, 5)},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "compress + decompress of layer 0 (466 MB) with the C oracle (OpenMP)",
                         "note": "the C oracle: the scalar correctness checker of the tests, run on all host threads; not a tuned CPU codec, so ratios against it say nothing about the kernels"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "compress / decompress GB/s (original bytes) per B200 and 8-GPU box; ratio"


# ---- our arm ----------------------------------------------------------------------------------


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-one-at-a-time", action="store_true")
    ap.add_argument("--micro-only", action="store_true",
                    help="run only the seam and CRC micro-benchmarks and print their JSON")
    ap.add_argument("--no-micro", action="store_true")
    ap.add_argument("--no-strong", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="profile a smaller model: this many decoder layers, no embedding / LM head")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        run_reference(args)
        return

    import cuzipnn_b200 as z
    from cuzipnn_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    if local_world > 1:  # each rank's host copies (pageable blobs) get its share of the host cores
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // local_world))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.micro_only:
        m = micro_benchmarks(device)
        if rank == 0:
            print(json.dumps({"micro": m}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return

    model = build_model(device, args.layers)
    model_bytes = nbytes(model)
    torch.cuda.synchronize()

    def step():
        blobs = z.compress_tensors(model, readback_to_cpu=False)
        mid = torch.cuda.Event(enable_timing=True)
        mid.record()
        outs = z.decompress_tensors(blobs)
        return blobs, outs, mid

    # Correctness once, outside the timed region.
    blobs, outs, _ = step()
    for i in sorted({0, 1, 8, len(model) - 1}):
        assert torch.equal(outs[i].view(torch.int16), model[i].view(torch.int16)), i
    assert z.last_decode_status(device) == 0
    blob_bytes = sum(b.numel() for b in blobs)
    ratio = blob_bytes / model_bytes
    del blobs, outs

    clocks = ClockSampler(local).__enter__()  # running through the warm-up, summarised over the timed region
    for _ in range(args.warmup):
        step()
    barrier()
    launches0 = _lib.launch_count()
    ev = []
    with _lib.KernelTimer() as kt:
        barrier()
        w0 = time.time()
        for _ in range(args.steps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            blobs, outs, mid = step()
            b.record()
            ev.append((a, mid, b))
            del blobs, outs
        barrier()
        clocks.window(w0, time.time())
    clocks.__exit__(None, None, None)
    gpu_launches = _lib.launch_count() - launches0
    t_step = sum(a.elapsed_time(b) for a, _, b in ev) / len(ev) / 1e3
    t_comp = sum(a.elapsed_time(m) for a, m, _ in ev) / len(ev) / 1e3
    t_dec = sum(m.elapsed_time(b) for _, m, b in ev) / len(ev) / 1e3
    t_step, t_comp, t_dec = (max_over_ranks(v) for v in (t_step, t_comp, t_dec))
    value = world * model_bytes / t_step / GB

    # Roofline of the dominant kernel (largest summed device time in the timed region).
    times = kt.times
    dominant = max(times, key=lambda k: times[k][0])
    dom_ms, dom_n = times[dominant]
    step_s = dom_ms / args.steps / 1e3  # the kernel's device time per step (all its launches)
    coded = [t for t in model if t.numel() * t.element_size() >= 65536]
    coded_bytes = nbytes(coded)
    coded_blob = blob_bytes - (model_bytes - coded_bytes)  # stored blobs add header bytes only
    # Algorithmic bytes per step: the kernel's launches of one step cover all non-stored tensors
    # (one launch per batch of about 4 GB).
    algo = {"decode": coded_blob + coded_bytes, "encode": coded_bytes + coded_blob,
            "hist": coded_bytes, "pack": coded_bytes + coded_blob}.get(dominant, coded_bytes)
    peak, peak_src = measured_hbm_peak()
    achieved = algo / step_s / GB
    tr = profile_traffic(dominant + "_kernel")
    traffic = round(tr * algo) if tr else None
    roofline = {"bound": "hbm", "kernel": dominant + "_kernel", "achieved": round(achieved, 1),
                "peak": peak, "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "frac_of_8tbs_nominal": round(achieved / 8000.0, 4),
                "traffic": traffic, "algo_bytes_per_step": algo, "traffic_basis": "per step (all launches)",
                "kernel_ms_per_step": round(step_s * 1e3, 4), "launches_per_step": round(dom_n / args.steps, 2),
                "kernel_share": {k: round(v[0] / sum(x[0] for x in times.values()), 4) for k, v in times.items()}}

    # Strong scaling: one copy of the model over the ranks (plan_model: tensors above half a rank's
    # mean share split by chunk range, the rest whole, longest first): device time of
    # compress_model_shard + decompress_model_shard, max over ranks, 3 warm-up + 5 timed passes.
    # Measured before the sections with host copies, whose copy threads can keep the host busy
    # afterwards while several ranks run.
    strong = None
    if not args.no_strong:
        plan = z.plan_model([t.numel() * t.element_size() for t in model], world)  # once per model
        tc_, td_ = [], []
        for s_i in range(8):
            barrier()
            a = torch.cuda.Event(enable_timing=True)
            m = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            whole, parts = z.compress_model_shard(model, rank, world, plan=plan, readback_to_cpu=False)
            m.record()
            outs, pouts = z.decompress_model_shard(whole, parts)
            b.record()
            torch.cuda.synchronize()
            if s_i >= 3:
                tc_.append(a.elapsed_time(m) / 1e3)
                td_.append(m.elapsed_time(b) / 1e3)
            del whole, parts, outs, pouts
        sc, sd = max_over_ranks(sum(tc_) / len(tc_)), max_over_ranks(sum(td_) / len(td_))
        st = max_over_ranks(sum(c + d for c, d in zip(tc_, td_)) / len(tc_))
        strong = {"value": round(model_bytes / st / GB, 3), "unit": "GB/s", "ms_per_step": round(st * 1e3, 3),
                  "compress_gbs": round(model_bytes / sc / GB, 3), "decompress_gbs": round(model_bytes / sd / GB, 3),
                  "scaling": "strong", "split_tensors": len(plan[1]),
                  "workload": "one copy of the model over the ranks (plan_model: tensors above half a rank's "
                              "share split by chunk range, the rest whole, longest first)"}

    # One tensor at a time (the reference's own methodology), device time.
    ev1 = []
    for _ in range(0 if args.no_one_at_a_time else 1):
        a = torch.cuda.Event(enable_timing=True)
        m = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        bl = [z.compress_tensor(t, readback_to_cpu=False) for t in model]
        m.record()
        for x in bl:
            z.decompress_tensor(x)
        b.record()
        torch.cuda.synchronize()
        ev1.append((a.elapsed_time(m) / 1e3, m.elapsed_time(b) / 1e3))
        del bl
    one_c = max_over_ranks(min(v[0] for v in ev1)) if ev1 else None
    one_d = max_over_ranks(min(v[1] for v in ev1)) if ev1 else None

    # The reference README's methodology (README.md:29-39 of ruihe774/cuZipNN): GPU tensor -> CPU
    # blob (compress_tensor with its defaults) -> GPU tensor (decompress_tensor), one tensor at a
    # time, best of two passes, wall clock with the host copies included.
    readme = None
    if not args.no_one_at_a_time:
        best = [float("inf"), float("inf")]
        for _ in range(2):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            cb = [z.compress_tensor(t) for t in model]
            t1 = time.perf_counter()
            for b in cb:
                z.decompress_tensor(b, compute_device=device)
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            best = [min(best[0], t1 - t0), min(best[1], t2 - t1)]
            del cb
        rc_, rd_ = max_over_ranks(best[0]), max_over_ranks(best[1])
        readme = {"compress_gbs": round(world * model_bytes / rc_ / GB, 3),
                  "decompress_gbs": round(world * model_bytes / rd_ / GB, 3),
                  "path": "GPU tensor -> compress_tensor() defaults (CPU blob) -> decompress_tensor(blob, compute_device) "
                          "one tensor at a time, best of 2 passes, wall clock"}

    # End to end through the public API from pinned host memory: H2D of the inputs, CPU blobs,
    # H2D of the blobs, and a D2H read of a result word each step.
    host = [t.cpu().pin_memory() for t in model] if not args.no_e2e else []
    torch.cuda.synchronize()
    barrier()
    e2e_times = []
    h2d = d2h = 0
    e2e_warm = 2  # the first passes fill the pinned-memory pools (a first pass takes seconds)
    for s_i in range(0 if args.no_e2e else args.e2e_steps + e2e_warm):
        t0 = time.perf_counter()
        cblobs = z.compress_tensors(host, readback_to_cpu=True, pin_memory=True)
        outs = z.decompress_tensors(cblobs)
        check = outs[-1].view(-1)[:4].view(torch.uint8).cpu()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        if s_i >= e2e_warm:
            e2e_times.append(t1 - t0)
        sz = sum(b.numel() for b in cblobs)
        h2d, d2h = model_bytes + sz, sz + check.numel()
        del cblobs, outs
    del host
    e2e = None
    if e2e_times:
        t_e2e = max_over_ranks(sum(e2e_times) / len(e2e_times))
        e2e = {"value": round(world * model_bytes / t_e2e / GB, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(t_e2e * 1e3, 1),
               "path": "pinned host tensors -> compress_tensors(readback_to_cpu, pin_memory) -> decompress_tensors"}

    micro = None if args.no_micro else micro_benchmarks(device)

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tc, td, nin, _ = cpu_round_trip(cpu_sample(), threads)
        cpu_baseline = {"value": round(nin / (tc + td) / GB, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                        "sample": "compress + decompress of layer 0 (466 MB) with the C oracle (OpenMP)",
                        "note": "the C oracle: the scalar correctness checker of the tests, run on all host threads; not a tuned CPU codec, so ratios against it say nothing about the kernels"}

    barrier()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(t_step * 1e3, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u8",
            "data": "synthetic",
            "config": {"workload": WORKLOAD if args.layers is None else
                       f"first {args.layers} decoder layer(s) only ({len(model)} tensors, {model_bytes / GB:.3f} GB) of: "
                       + WORKLOAD,
                       "value": "original bytes / (compress + decompress time)",
                       "l2": f"inputs {model_bytes / GB:.3g} GB per GPU >> 126 MB L2 (no flush)",
                       "parallelism": f"{world} x replica"},
            "compress_gbs": round(world * model_bytes / t_comp / GB, 3),
            "decompress_gbs": round(world * model_bytes / t_dec / GB, 3),
            "ratio": round(ratio, 5),
            "one_tensor_at_a_time": None if one_c is None else {
                "compress_gbs": round(world * model_bytes / one_c / GB, 3),
                "decompress_gbs": round(world * model_bytes / one_d / GB, 3),
                "path": "device tensors, compress_tensor(readback_to_cpu=False) then decompress_tensor, device time"},
            "readme_methodology": readme,
            "roofline": roofline,
            "cpu_baseline": cpu_baseline,
            "clocks": clocks.summary(),
            "e2e": e2e,
            "strong": strong,
            "micro": micro,
            "gpu_launches": gpu_launches,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
