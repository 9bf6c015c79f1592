"""Benchmark of the fused token-selection pass (one JSON line on rank 0).

Workload (the one the headline metric is quoted on):
B=256 rows per GPU, V=163,840 fp32 logits N(0,1)*2 + 9 at 64 ids per row, a
packed allowed-token bitmask (~2% of bits: 4 blocks of 512 + ~1,200
singletons), temp 1.0, top_k 50, top_p 0.95, Philox Gumbel-max draw.

A step is one pm_sample_rows call over one batch.  `value` is whole-job rows/s
with inputs resident in HBM; `e2e` is the same metric through the public API
with pinned host buffers copied in and tokens copied out inside the timed
region.  Six device-resident input batches rotate, so that no step finds the
sectors it gathers in L2 (about 42 MB a batch; the L2 holds 126 MB), and a
cold number with L2 flushed before every step is reported beside it.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled rows/s at B=256,V=152k; logits HBM GB/s vs peak; p50 µs/step"
B_PER_GPU = 256
VOCAB = 163840
BYTES_PER_ROW = VOCAB * 4 + (VOCAB // 32) * 4  # logits + bitmask = 675,840 B
LAUNCHES_PER_STEP = 1  # k_sample_masked (masked rows, no penalties, no logit bias, top_k bounded)
N_BATCHES = 6  # device-resident input batches in rotation (see bench_config)
WORKLOAD = ("C3: 256 rows per GPU, V=163,840 fp32 logits + packed allowed-token bitmask (~2% set), "
            "temp 1.0, top_k 50, top_p 0.95, Philox Gumbel-max draw")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--c5-rows", type=int, default=1024,
                    help="rows of the C5 workload (smaller only for profiling captures)")
    ap.add_argument("--workload", default="c3",
                    choices=["c3", "c3u", "c5", "c5e", "c1", "c2", "c2b", "c4a", "c4b", "ngram", "think", "logprobs",
                             "lmhead"],
                    help="c3 (default): the headline metric's config; c5: C5 rows (one GPU: the unsharded pass; "
                         "torchrun: vocabulary-sharded over the ranks); c5e: eight vocabulary shards emulated on "
                         "one GPU; the rest: the other configs and the path's neighbours (n-gram drafts, "
                         "ThinkBudget, log-softmax rows)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_launch(kernel: str, workload: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum of
    one ncu capture) from the tab-separated table profiles/dram_traffic.tsv
    (kernel, workload, bytes per launch, source summary); None if absent."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.tsv")
    try:
        for line in open(path):
            f = line.rstrip("\n").split("\t")
            if len(f) >= 3 and f[0] == kernel and f[1] == workload:
                return float(f[2])
    except (OSError, ValueError):
        pass
    return None


def bench_config(world: int) -> dict:
    """The config dict both arms print for the C3 workload."""
    return {"workload": WORKLOAD, "rows_per_gpu": B_PER_GPU, "vocab": VOCAB, "n_gpus": world,
            "l2": f"{N_BATCHES} input batches in rotation (device-resident arm): their gathered sectors "
                  f"(~42 MB a batch) exceed the 126 MB L2; cold_us_per_step flushes L2 before every step",
            "noise": "Philox4x32-10"}


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        except OSError:
            pass
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def gather_bytes(mask) -> int:
    """Bytes the masked pass must read for these rows: the mask words plus
    every 32-byte sector of fp32 logits (8 tokens) holding an allowed token
    (a sector is touched iff its byte of the mask is non-zero)."""
    import numpy as np
    m = np.ascontiguousarray(mask).view(np.uint8)
    return int(mask.size * 4 + 32 * np.count_nonzero(m))


def make_inputs(seed: int):
    from paged_moe_b200 import workloads as W
    d = W.c3(seed=seed, B=B_PER_GPU, V=VOCAB)
    return d


def cpu_baseline(d, seconds: float):
    """The oracle (C restatement of the reference path) on all host cores over
    a bounded sample of the same workload: whole steps of 256 rows, repeated
    until `seconds` of wall time has passed (at least one)."""
    import numpy as np

    import oracle as O
    s = d["sampler"]
    osamp = O.Sampler(temp=s.temp, top_p=s.top_p, top_k=s.top_k)
    cores = os.cpu_count() or 1
    O.lib()
    rows = 0
    t0 = time.perf_counter()
    steps = 0
    while True:
        O.sample(d["logits"], osamp, mask=d["mask"], seed=1, offset=steps, nthreads=cores)
        rows += d["logits"].shape[0]
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": rows / el, "unit": "rows/s", "cores": cores, "kind": "port",
            "sample": f"{steps} full C3 steps x {d['logits'].shape[0]} rows, {el:.1f} s wall"}


def run_reference(args):
    """The reference arm: the oracle port (the reference's own sampler is
    mlx-lm over MLX, darwin-only) on all host cores, on the same C3 workload,
    metric and config as the device arm.  Loads no library of this package:
    the inputs come from paged_moe_b200.workloads, which is host-only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle as O
    d = make_inputs(seed=0)
    s = d["sampler"]
    osamp = O.Sampler(temp=s.temp, top_p=s.top_p, top_k=s.top_k)
    cores = os.cpu_count() or 1
    # each step is the full 256-row batch (about 0.1 s on 8 cores)
    n = B_PER_GPU
    x, m = d["logits"][:n], d["mask"][:n]
    for i in range(args.warmup):
        O.sample(x, osamp, mask=m, seed=1, offset=i, nthreads=cores)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        O.sample(x, osamp, mask=m, seed=1, offset=1000 + i, nthreads=cores)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    val = n * args.steps / tot
    line = {
        "metric": METRIC, "value": val, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * tot / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(args.gpus),
        "impl": "reference",
        "p50_us_per_step": 1e6 * statistics.median(times),
        "cpu_baseline": {"value": val, "unit": "rows/s", "cores": cores, "kind": "port",
                         "sample": f"{n} C3 rows per step, {args.steps} steps, oracle port on {cores} host threads "
                                   "(the reference's MLX path is darwin-only)"},
        "e2e": {"value": val, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def l2_flush_buffer(dev):
    """A device buffer twice the size of L2: writing it evicts every line."""
    import torch
    return torch.empty(64 << 20, dtype=torch.float32, device=dev)  # 256 MB


def run_ours(args):
    import numpy as np
    import torch

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", torch.cuda.current_device())
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        pg = dist
    import paged_moe_b200 as pm

    ds = [make_inputs(seed=1000 * rank + k) for k in range(N_BATCHES)]
    s = ds[0]["sampler"]
    xs = [torch.from_numpy(d["logits"]).to(dev) for d in ds]
    ms = [torch.from_numpy(d["mask"].view(np.int32)).to(dev) for d in ds]
    stream = torch.cuda.current_stream(dev)

    def step(i):
        k = i % N_BATCHES
        return pm.sample_rows(xs[k], s, mask=ms[k], seed=12345, offset=i, row_base=rank * B_PER_GPU)

    for i in range(max(args.warmup, N_BATCHES)):
        step(i)
    torch.cuda.synchronize(dev)
    # eager steps, one event each: the latency a caller that issues one call
    # per decode step sees (host issue time included)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    ev[0].record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
        ev[i + 1].record(stream)
    torch.cuda.synchronize(dev)
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    # cold steps: L2 flushed before each, events around the step alone
    flush = l2_flush_buffer(dev)
    cold = []
    for i in range(min(args.steps, 20)):
        flush.fill_(float(i))
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        step(2000 + i)
        c1.record(stream)
        torch.cuda.synchronize(dev)
        cold.append(c0.elapsed_time(c1))
    del flush
    # the timed region: the K steps captured once into a CUDA graph and
    # replayed, so the device runs them back to back; every replay recomputes
    # every step from its inputs (N_BATCHES batches in rotation)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(args.steps):
            step(args.warmup + i)
    g.replay()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    with Clocks(dev.index if world == 1 else local) as clk:
        t0.record(stream)
        g.replay()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    clocks = clk.summary()
    total_ms = t0.elapsed_time(t1)
    del g
    if pg:
        t = torch.tensor([total_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total_ms = float(t.item())
        pg.barrier()
    ms_step = total_ms / args.steps
    rows_total = B_PER_GPU * world
    value = rows_total / (ms_step / 1000.0)

    # end to end through the public API, inputs in pinned host memory and the
    # tokens read back every step.  The masked pass reads the host rows in
    # place: only the mask and the allowed logits cross the host link.  The
    # same with the whole rows copied to the device first is reported beside.
    hx = [torch.from_numpy(d["logits"]).pin_memory() for d in ds[:2]]
    hm = [torch.from_numpy(d["mask"].view(np.int32)).pin_memory() for d in ds[:2]]
    htok = torch.empty(B_PER_GPU, dtype=torch.int32).pin_memory()
    del xs, ms
    dx = torch.empty(hx[0].shape, dtype=hx[0].dtype, device=dev)
    dm = torch.empty(hm[0].shape, dtype=hm[0].dtype, device=dev)
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step(i):
        out = pm.sample_rows(hx[i & 1], s, mask=hm[i & 1], seed=777, offset=i, row_base=rank * B_PER_GPU)
        htok.copy_(out["tokens"], non_blocking=True)

    def e2e_copy_step(i):
        dx.copy_(hx[i & 1], non_blocking=True)
        dm.copy_(hm[i & 1], non_blocking=True)
        out = pm.sample_rows(dx, s, mask=dm, seed=777, offset=i, row_base=rank * B_PER_GPU)
        htok.copy_(out["tokens"], non_blocking=True)

    def e2e_time(fn):
        for i in range(2):
            fn(i)
        torch.cuda.synchronize(dev)
        if pg:
            pg.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(e2e_steps):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms_ = e0.elapsed_time(e1)
        if pg:
            t = torch.tensor([ms_], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms_ = float(t.item())
        return rows_total / (ms_ / e2e_steps / 1000.0)

    e2e_val = e2e_time(e2e_step)
    e2e_copy_val = e2e_time(e2e_copy_step)
    h2d = statistics.mean(gather_bytes(d["mask"]) for d in ds[:2])
    h2d_copy = hx[0].numel() * 4 + hm[0].numel() * 4
    d2h = htok.numel() * 4

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(ds[0], args.cpu_seconds)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = peaks()
    dense_bytes = BYTES_PER_ROW * B_PER_GPU
    sparse_bytes = statistics.mean(gather_bytes(d["mask"]) for d in ds)
    launch_s = ms_step / 1000.0  # one launch per step, back to back
    achieved = dense_bytes / launch_s / 1e9
    trf = traffic_per_launch("k_sample_masked", "C3")
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(world),
        "timing": "CUDA graph of the K steps, replayed once (events around the replay)",
        "eager_p50_us_per_step": 1000 * statistics.median(per),
        "eager_mean_us_per_step": 1000 * statistics.mean(per),
        "cold_us_per_step": 1000 * statistics.median(cold),
        "logits_gb_per_s": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": trf,
                     "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs",
                     "algorithmic_bytes_per_launch": dense_bytes,
                     "bytes_rule": "675,840 B per row (fp32 logits + packed mask) x 256 rows; the masked pass "
                                   "reads only the mask and the 32-byte sectors holding an allowed token "
                                   "(disallowed logits are -inf under the mask processor and change nothing)",
                     "sparse_bytes_per_launch": sparse_bytes,
                     "sparse_gb_per_s": sparse_bytes / launch_s / 1e9,
                     "dram_gb_per_s": None if trf is None else trf / launch_s / 1e9,
                     "dram_frac": None if trf is None else trf / launch_s / 1e9 / peak},
        "e2e": {"value": e2e_val, "unit": "rows/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "pinned host logits + mask read in place by the masked pass (mask words and the "
                        "32-byte sectors holding an allowed token cross the host link); tokens copied back",
                "full_copy": {"value": e2e_copy_val, "unit": "rows/s", "h2d_bytes_per_step": h2d_copy,
                              "d2h_bytes_per_step": d2h,
                              "path": "whole logits rows and mask copied host-to-device, then the pass"}},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "clocks": clocks,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def run_c5(args):
    """C5: B=1,024 rows, V=262,144 fp32 split into one contiguous slice per rank
    (a tensor-parallel LM head's output); temp 0.8, top_k 64, top_p 0.9.  A
    step is summarize -> NCCL all-gather of the summaries -> merge, on every
    rank; the job's value is 1,024 rows per step (strong scaling)."""
    import torch

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", torch.cuda.current_device())
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from paged_moe_b200 import shard as S
    from paged_moe_b200.params import SamplerSettings
    B, V = args.c5_rows, 262144
    spec = S.ShardSpec.of(rank, world, V)
    w = spec.hi - spec.lo
    s = SamplerSettings(temp=0.8, top_k=64, top_p=0.9)
    gen = torch.Generator(device=dev)
    xs = []
    for k in range(2):
        gen.manual_seed(1000 + k)
        x = torch.randn(B, V, device=dev, generator=gen) * 2.5
        idx = torch.randint(0, V, (B, 32), device=dev, generator=gen)
        x.scatter_add_(1, idx, torch.full((B, 32), 10.0, device=dev))
        xs.append(x[:, spec.lo:spec.hi].contiguous())
        del x
    stream = torch.cuda.current_stream(dev)

    import paged_moe_b200 as pm
    emulated = args.workload == "c5e"

    def step(i):
        if world > 1:
            return S.sample_vocab_sharded(xs[i & 1], s, vocab_total=V, seed=3, offset=i)
        if emulated:
            return S.emulate(xs[i & 1], 8, s, seed=3, offset=i)
        return pm.sample_rows(xs[i & 1], s, seed=3, offset=i)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with Clocks(dev.index) as clk:
        ev[0].record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
            ev[i + 1].record(stream)
        torch.cuda.synchronize(dev)
    clocks = clk.summary()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = peaks()
    ms_step = total_ms / args.steps
    bytes_gpu = B * w * 4
    achieved = bytes_gpu / (statistics.mean(per) / 1000.0) / 1e9
    line = {
        "metric": "sampled rows/s, vocabulary-sharded C5", "value": B / (ms_step / 1000.0), "unit": "rows/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": (f"C5: {B:,} rows, V=262,144 fp32 in {world} slices of {w} ids, temp 0.8, top_k 64, "
                                "top_p 0.9; summarize + all-gather + merge per step") if world > 1 else
                               (f"C5: {B:,} rows, V=262,144 fp32, temp 0.8, top_k 64, top_p 0.9; " +
                                ("eight vocabulary shards emulated on one GPU (summaries + merge)" if emulated else
                                 "one unsharded pass (streaming + per-row merge)")),
                   "l2": "two alternating input batches larger than L2 per rank" if B * w * 4 > 126e6 else
                         "two alternating input batches"},
        "p50_us_per_step": 1000 * statistics.median(per),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs",
                     "algorithmic_bytes_per_launch": bytes_gpu},
        # one GPU: streaming pass, row merge, exact pass for undecided top-p cuts
        "gpu_launches": (3 if world > 1 else (17 if emulated else 3)) * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_config(args):
    """The other BASELINE configs on one GPU (reported beside the headline):
    c1 (B=1 latency), c2 / c2b (bf16, 4,096-id Zipf histories, greedy / min_p),
    c4a / c4b (verify of 32 requests x 5 rows, residual / match)."""
    import numpy as np
    import torch

    import paged_moe_b200 as pm
    from paged_moe_b200 import workloads as W
    from paged_moe_b200.params import SamplerSettings
    dev = torch.device("cuda", 0)
    wl = args.workload
    # batches in rotation: enough that one pass over them exceeds the 126 MB
    # L2 twice (C1's 0.6 MB row is latency-bound and stays L2-resident)
    nb = {"c1": 2, "c2": 16, "c2b": 16, "c3u": 3, "c4a": 4, "c4b": 4, "ngram": 2, "think": 2, "logprobs": 6}[wl]
    if wl == "c3u":
        # C3's rows and filters without the mask: the dense filtered pass
        gen = torch.Generator(device=dev)
        xs = []
        for k in range(nb):
            gen.manual_seed(300 + k)
            x = torch.randn(256, 163840, device=dev, generator=gen) * 2.0
            idx = torch.randint(0, 163840, (256, 64), device=dev, generator=gen)
            x.scatter_add_(1, idx, torch.full((256, 64), 9.0, device=dev))
            xs.append(x)
        s = SamplerSettings(temp=1.0, top_k=50, top_p=0.95)
        rows, nbytes = 256, 256 * 163840 * 4

        def step(i):
            return pm.sample_rows(xs[i % nb], s, seed=5, offset=i)
        desc = "C3 rows without the mask: B=256, V=163,840 fp32, temp 1.0, top_k 50, top_p 0.95 (dense filtered pass)"
    elif wl == "c1":
        ds = [W.c1(seed=k) for k in range(nb)]
        xs = [torch.from_numpy(d["logits"]).to(dev) for d in ds]
        hs = [torch.from_numpy(d["hist"]).to(dev) for d in ds]
        s, p = ds[0]["sampler"], ds[0]["proc"]
        rows, nbytes = 1, 151936 * 4 + 256 * 4

        def step(i):
            return pm.sample_rows(xs[i % nb], s, p, history=hs[i % nb], seed=5, offset=i)
        desc = "C1: B=1, V=151,936 fp32, temp 0.7, top_k 20, top_p 0.8, repetition 1.05 over 256 ids"
    elif wl in ("c2", "c2b"):
        ds = [W.c2(seed=k, second=(wl == "c2b")) for k in range(nb)]
        xs = [torch.from_numpy(d["logits_bf16"].view(np.int16)).to(dev).view(torch.bfloat16) for d in ds]
        hs = [torch.from_numpy(d["hist"]).to(dev) for d in ds]
        s, p = ds[0]["sampler"], ds[0]["proc"]
        rows, nbytes = 64, 64 * (151936 * 2 + 4096 * 4)

        def step(i):
            return pm.sample_rows(xs[i % nb], s, p, history=hs[i % nb], seed=5, offset=i)
        desc = ("C2: B=64, V=151,936 bf16, 4,096-id Zipf histories, presence 0.5 + frequency 0.3, "
                + ("min_p 0.05 at temp 1" if wl == "c2b" else "argmax"))
    elif wl == "ngram":
        from paged_moe_b200 import ngram
        hs = [torch.from_numpy(W.ngram_histories(seed=k)).to(dev) for k in range(nb)]
        rows, nbytes = 32, 32 * 4096 * 4

        def step(i):
            return ngram.draft_ngram_batch(hs[i % nb], 4)
        desc = "n-gram drafts: 32 requests x 4,096-token histories (repeated spans), k=4, n 8..3"
    elif wl == "think":
        from paged_moe_b200.think_budget import ThinkBudget
        tb = ThinkBudget(W.SyntheticTokenizer(), chars=6000, close="", device=dev, slack=48)
        gens = [torch.from_numpy(np.random.default_rng(k).integers(0, 151935, (256, 2048)).astype(np.int32)).to(dev)
                for k in range(nb)]
        lg = torch.from_numpy(W.c1(seed=5, B=256)["logits"]).to(dev)
        st = SamplerSettings(temp=0.7, top_k=20, top_p=0.8)
        rows, nbytes = 256, 256 * 2048 * 4

        def step(i):
            return pm.sample_rows(lg, st, forced=tb.forced(gens[i % nb]), seed=5, offset=i)
        desc = ("ThinkBudget: 256 rows x 2,048 generated ids, vocabulary 151,936, budget 6,000 characters; "
                "the forced tokens then go through the sampling pass (temp 0.7, top_k 20, top_p 0.8)")
    elif wl == "logprobs":
        ds = [W.c1(seed=k, B=64) for k in range(nb)]
        xs = [torch.from_numpy(d["logits"]).to(dev) for d in ds]
        hs = [torch.from_numpy(d["hist"]).to(dev) for d in ds]
        p = ds[0]["proc"]
        rows, nbytes = 64, 64 * 151936 * 8
        outs = [torch.empty(64, 151936, dtype=torch.float32, device=dev) for _ in range(2)]

        def step(i):
            return pm.logprobs(xs[i % nb], p, history=hs[i % nb], out=outs[i & 1])
        desc = "log-softmax rows: B=64, V=151,936 fp32, repetition penalty 1.05 over 256 ids (read V, write V)"
    else:
        ds = [W.c4(seed=k) for k in range(nb)]
        tg = [torch.from_numpy(d["target"]).to(dev) for d in ds]
        dl = [torch.from_numpy(d["draft_logits"]).to(dev) for d in ds]
        dr = [torch.from_numpy(d["drafts"]).to(dev) for d in ds]
        yy = [torch.from_numpy(d["y"]).to(dev) for d in ds]
        ua = [torch.from_numpy(d["u_accept"]).to(dev) for d in ds]
        ur = [torch.from_numpy(d["u_residual"]).to(dev) for d in ds]
        resid = wl == "c4a"
        s = SamplerSettings(temp=1.0) if resid else SamplerSettings(temp=0.0)
        rows = 32 * 5
        nbytes = 32 * (5 + (4 if resid else 0)) * 151552 * 4

        def step(i):
            k = i % nb
            if resid:
                return pm.verify(tg[k], dr[k], yy[k], s, mode="residual", draft_logits=dl[k], u_accept=ua[k],
                                 u_residual=ur[k], seed=5, offset=i)
            return pm.verify(tg[k], dr[k], yy[k], s, mode="match", seed=5, offset=i)
        desc = ("C4: verify of 32 requests x (k=4 drafts + 1) rows, V=151,552 fp32, "
                + ("residual rejection sampling at temp 1 (p and q rows read)" if resid else
                   "greedy exact-match acceptance"))
    stream = torch.cuda.current_stream(dev)
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with Clocks(0) as clk:
        ev[0].record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
            ev[i + 1].record(stream)
        torch.cuda.synchronize(dev)
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    # the same steps replayed from a CUDA graph (no host work between them)
    ng = max(8, nb)  # every batch once per replay
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(ng):
            step(1000 + i)
    g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(4):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    graph_us = e0.elapsed_time(e1) * 1000 / (4 * ng)
    del g
    peak, peak_kind = peaks()
    ms = statistics.mean(per)
    line = {
        "metric": f"sampled rows/s ({wl.upper()}); p50 us/step", "value": rows / (ms / 1000.0), "unit": "rows/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": desc, "l2": f"{nb} input batches in rotation"},
        "eager_p50_us_per_step": 1000 * statistics.median(per),
        "graph_us_per_step": graph_us,
        "roofline": {"bound": "hbm", "achieved": nbytes / (graph_us * 1e-6) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": nbytes / (graph_us * 1e-6) / 1e9 / peak, "traffic": None,
                     "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs", "algorithmic_bytes_per_launch": nbytes,
                     "timing": "graph replay"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_lmhead(args):
    """The LM head fused with the sampler (the logits producer of the
    reference's decode step, pagedmoe/verify_decode.py:821): 256 rows of
    hidden size 2,048 into a vocabulary of 151,936 (a Qwen3-30B-A3B-class
    head; random-init bf16 weights), top_k 50, top_p 0.95 at temp 1, Philox
    draw.  Timed: the fused call, the unfused pair (the same GEMM writing
    fp32 logits, then the sampling pass) and cuBLAS's bf16 GEMM alone, each
    as a CUDA-graph replay.  Roofline: tensor-bound, 2 B H V flops a step
    against the measured sustained cuBLAS bf16 rate."""
    import torch

    import paged_moe_b200 as pm
    from paged_moe_b200 import engine
    from paged_moe_b200.params import SamplerSettings
    dev = torch.device("cuda", 0)
    B, H, V = 256, 2048, 151936
    gen = torch.Generator(device=dev).manual_seed(7)
    w = (torch.randn(V, H, device=dev, generator=gen) * 0.05).to(torch.bfloat16)
    hs = [torch.randn(B, H, device=dev, generator=gen).to(torch.bfloat16) for _ in range(2)]
    s = SamplerSettings(temp=1.0, top_k=50, top_p=0.95)
    buf = torch.empty(B, V, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def fused(i):
        return engine.lmhead_sample(hs[i & 1], w, s, seed=5, offset=i)

    def unfused(i):
        engine.lmhead_logits(hs[i & 1], w, out=buf)
        return pm.sample_rows(buf, s, seed=5, offset=i)

    def gemm(i):
        return engine.lmhead_logits(hs[i & 1], w, out=buf)

    def cublas(i):
        return hs[i & 1] @ w.T

    def graph_time(fn, n=8, reps=4):
        for i in range(max(args.warmup, 3)):
            fn(i)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                fn(100 + i)
        g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        del g
        return e0.elapsed_time(e1) * 1000 / (n * reps)

    # eager steps of the fused call (the headline of this line)
    for i in range(max(args.warmup, 3)):
        fused(i)
    torch.cuda.synchronize(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with Clocks(0) as clk:
        ev[0].record(stream)
        for i in range(args.steps):
            fused(args.warmup + i)
            ev[i + 1].record(stream)
        torch.cuda.synchronize(dev)
        t_fused = graph_time(fused)
        t_unfused = graph_time(unfused)
        t_gemm = graph_time(gemm)
        t_cublas = graph_time(cublas)
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    ms = statistics.mean(per)
    flops = 2.0 * B * H * V
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk, kind = float(json.load(f)["bf16_tflops_sustained"]), "measured"
    except Exception:
        tpk, kind = 1400.0, "fallback"
    ach = flops / (t_fused * 1e-6) / 1e12
    line = {
        "metric": "sampled rows/s (LM head fused with the sampler)", "value": B / (ms / 1000.0), "unit": "rows/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 operands, f32 accumulate", "data": "synthetic",
        "config": {"workload": f"LM head {B} x {H} -> {V} (random-init bf16 weights) + top_k 50, top_p 0.95, "
                               "temp 1, Philox draw", "l2": "weights 622 MB (> L2), two hidden batches"},
        "eager_p50_us_per_step": 1000 * statistics.median(per),
        "graph_us_per_step": t_fused,
        "unfused_graph_us_per_step": t_unfused,
        "gemm_only_graph_us": t_gemm,
        "cublas_bf16_gemm_graph_us": t_cublas,
        "roofline": {"bound": "tensor", "achieved": ach, "peak": tpk, "unit": "TFLOP/s", "frac": ach / tpk,
                     "traffic": traffic_per_launch("k_lmhead", "lmhead"),
                     "peak_source": f"{kind} MEASURED_PEAKS.json bf16_tflops_sustained",
                     "algorithmic_flops_per_launch": flops, "timing": "graph replay"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "lmhead":
        run_lmhead(args)
    elif args.workload in ("c5", "c5e"):
        run_c5(args)
    elif args.workload != "c3":
        run_config(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
