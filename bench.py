#!/usr/bin/env python
"""Benchmark of the B200 token sampler (drama3-mlx's sampling.c hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one pass of the sampler over one batch: config 5 of the baseline,
65536 rows x 4097 f32 logits per GPU with per-row temperature / top_p / top_k
and per-row seeds, plus the gather of the sampled ids to rank 0 when N > 1
(rows are sharded; weak scaling: every GPU samples its own 65536 rows). Rank 0
prints one JSON line. For N > 1 launch with torchrun (one process per GPU).

--impl reference times the reference's algorithm on the host cores instead:
the reference itself (src/sampling.c on mlx-c) cannot be built here, so the
timed CPU implementation is the C restatement in oracle/ (OpenMP over rows).
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
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT / "drama3-mlx_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

METRIC = "sampled rows/s at B×4097 logits & % of HBM roofline; p50 per-row latency µs"
V = 4097
ROWS = 65536
# algorithmic bytes per row: logits (4 B x V) + temperature, top_p, top_k (4 B
# each) + seed (8 B) read, id (4 B) written
BYTES_PER_ROW = 4 * V + 4 + 4 + 4 + 8 + 4
WORKLOAD = ("config5 scale-out: f32 logits [65536, 4097] per GPU ~N(0,3); per-row temperature "
            "U[0.5,1.2], top_p U[0.5,1.0], top_k U{1..64}, per-row seeds; ids gathered to rank 0")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=ROWS, help="rows per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-latency", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip configs 2-4 in the default line (rank 0, one GPU)")
    ap.add_argument("--workload", choices=["c5", "c3", "c4"], default="c5",
                    help="c5: the headline line; c3 (lm_head + sample) and c4 (tower frames) "
                         "print their own lines for the design notes")
    ap.add_argument("--batch", type=int, default=1024, help="c3: hidden-state rows B")
    ap.add_argument("--frames", type=int, default=200, help="c4: frames per stream")
    return ap.parse_args()


def env_ranks():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    """DRAM bytes per launch of the fast kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return float(d["dram_bytes_per_launch_full"])
    except Exception:
        return None


class Clocks:
    """SM clocks and clock-event (throttle) reasons sampled through NVML every
    quarter millisecond or so while the timed region runs (read-only queries)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, uuid: str | None, index: int = 0, interval_s: float = 0.001):
        self.uuid, self.index, self.interval_s = uuid, index, interval_s
        self.samples = []
        self.max_mhz = None
        self.err = None
        self._stop = None
        self._thread = None

    def _handle(self, nv):
        if self.uuid:
            u = self.uuid if self.uuid.startswith("GPU-") else "GPU-" + self.uuid
            try:
                return nv.nvmlDeviceGetHandleByUUID(u)
            except Exception:
                pass
        return nv.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception as e:  # no NVML: report it instead of clocks
            self.err = f"nvml unavailable: {e}"
            return self
        self._stop = threading.Event()

        def poll():
            while not self._stop.is_set():
                try:
                    self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                         int(get_reasons(h))))
                except Exception:
                    pass
                self._stop.wait(self.interval_s)

        # the main thread enqueues launches while holding the interpreter: switch
        # threads often so the poller runs during the timed region
        self._switch = sys.getswitchinterval()
        sys.setswitchinterval(1e-4)
        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            sys.setswitchinterval(self._switch)

    def summary(self):
        if self.err:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err]}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
        sm = [c for c, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples),
                "source": f"NVML, ~{self.interval_s * 1e3:g} ms polling during the timed region"}


def merge_clocks(per_rank: list[dict]) -> dict:
    """One clocks record for the job: the lowest per-rank median SM clock, the
    union of the throttle reasons seen on any rank, and each rank's record."""
    mhz = [c["sm_mhz"] for c in per_rank if c.get("sm_mhz") is not None]
    reasons = sorted({r for c in per_rank for r in c.get("reasons", [])})
    return {"sm_mhz": min(mhz) if mhz else None,
            "sm_max_mhz": next((c["sm_max_mhz"] for c in per_rank if c.get("sm_max_mhz")), None),
            "reasons": reasons, "per_rank": per_rank,
            "source": "NVML on every rank during the timed region; sm_mhz = lowest rank median"}


def cpu_baseline(x_host, T, p, k, seeds, target_s: float = 8.0):
    """The oracle (a port of the reference's sampling.c) on a bounded sample of
    the same rows, all host threads."""
    import numpy as np

    import oracle
    cores = os.cpu_count() or 1
    oracle.lib()
    n = len(x_host)
    oracle.sample_rows(x_host[:256], T[:256], p[:256], k[:256], seeds[:256], nthreads=cores)
    passes, t0 = 0, time.perf_counter()
    while True:  # whole passes over the sample until about target_s of CPU work
        oracle.sample_rows(x_host, T, p, k, seeds, nthreads=cores)
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    return {"value": n * passes / dt, "unit": "rows/s", "cores": cores, "kind": "port",
            "sample": f"the first {n} rows of the config-5 batch, {passes} passes, {dt:.1f} s "
                      "(oracle/d3s_oracle.c, OpenMP over rows)"}


def host_workload(rows: int, seed: int):
    """Config-5 rows on the host (numpy) for the CPU arm."""
    import numpy as np
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, V), dtype=np.float32)
    x *= np.float32(3.0)
    T = rng.uniform(0.5, 1.2, rows).astype(np.float32)
    p = rng.uniform(0.5, 1.0, rows).astype(np.float32)
    k = rng.integers(1, 65, rows).astype(np.int32)
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(seed * 1_000_003)
    return x, T, p, k, seeds


def run_reference(args):
    """The reference arm: the reference's algorithm for this path timed on the
    host cores. src/sampling.c needs mlx-c, which cannot be built here, so the
    timed implementation is its C restatement (oracle/d3s_oracle.c, OpenMP over
    rows, every host thread); each step samples a bounded slice of the same
    65536-row config-5 batch the GPU arm samples."""
    rank, world, _ = env_ranks()
    if rank != 0:
        return
    import numpy as np

    import oracle
    cores = os.cpu_count() or 1
    oracle.lib()
    x, T, p, k, seeds = host_workload(args.rows, 7)
    t0 = time.perf_counter()
    oracle.sample_rows(x[:512], T[:512], p[:512], k[:512], seeds[:512], nthreads=cores)
    rate = 512 / (time.perf_counter() - t0)
    per_step = int(min(len(x), max(256, rate * 1.5)))  # about 1.5 s of CPU work per step
    offs = [(i * per_step) % max(1, len(x) - per_step + 1) for i in range(args.warmup + args.steps)]
    for o in offs[:args.warmup]:
        oracle.sample_rows(x[o:o + per_step], T[o:o + per_step], p[o:o + per_step],
                           k[o:o + per_step], seeds[o:o + per_step], nthreads=cores)
    t0 = time.perf_counter()
    for o in offs[args.warmup:]:
        oracle.sample_rows(x[o:o + per_step], T[o:o + per_step], p[o:o + per_step],
                           k[o:o + per_step], seeds[o:o + per_step], nthreads=cores)
    dt = time.perf_counter() - t0
    value = per_step * args.steps / dt
    sample = (f"{per_step} rows per step, consecutive slices of the same {args.rows}-row config-5 "
              f"batch, oracle port, {cores} threads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "rows_per_gpu": args.rows, "rows_per_step": per_step,
                       "V": V},
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "src/sampling.c needs mlx-c (absent): the timed CPU implementation is its C restatement"}
    print(json.dumps(line), flush=True)


def cpu_one_thread_row_us(x_host, T, p, k, seeds, n: int = 2000):
    """Config 1's CPU reference: the oracle on one host thread, one row per
    call (p50 of single-row calls) and per row over a run of n rows."""
    import oracle
    oracle.lib()
    per_call = []
    for i in range(min(n, len(x_host), 400)):
        t0 = time.perf_counter()
        oracle.sample_rows(x_host[i:i + 1], T, p, k, seeds + i, nthreads=1)
        per_call.append((time.perf_counter() - t0) * 1e6)
    t0 = time.perf_counter()
    oracle.sample_rows(x_host[:n], T, p, k, seeds, nthreads=1)
    mean = (time.perf_counter() - t0) * 1e6 / min(n, len(x_host))
    per_call.sort()
    return {"c1_cpu_1thread_p50_us": per_call[len(per_call) // 2],
            "c1_cpu_1thread_mean_us_per_row": mean,
            "c1_cpu_note": "oracle/d3s_oracle.c (the C restatement of src/sampling.c), 1 thread; "
                           "p50 of single-row calls through ctypes, mean over a 2000-row run"}


def c1_latency(ctx, torch):
    """Config 1: one [1, 4097] f32 row per call on the global key. The device
    time of one call without host submission (a CUDA graph of 100 calls,
    replayed), events around single Python calls (host submission included),
    the host-buffer d3_sample call (host in, host out), and the CPU oracle on
    one thread."""
    import numpy as np

    import d3s
    import synth
    x = synth.c1_rows(1, seed=42)
    ids = torch.empty(1, dtype=torch.int32, device="cuda")
    d3s.seed(42)
    st = torch.cuda.current_stream()
    for _ in range(20):
        ctx.sample_top_k_top_p(x, 0.7, 30, 0.7, None, ids)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(500)]
    for a, b in evs:
        a.record(st)
        ctx.sample_top_k_top_p(x, 0.7, 30, 0.7, None, ids)
        b.record(st)
    torch.cuda.synchronize()
    dev = sorted(a.elapsed_time(b) * 1e3 for a, b in evs)
    # 100 calls captured once (keys frozen at capture) and replayed: the GPU
    # time of a call with no host work in between
    gs = torch.cuda.Stream()
    gs.wait_stream(st)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(gs):
        with torch.cuda.graph(graph, stream=gs):
            for _ in range(100):
                ctx.sample_top_k_top_p(x, 0.7, 30, 0.7, None, ids, stream=gs)
    torch.cuda.synchronize()
    graph_ms = _events_ms(torch, graph.replay, 20)
    del graph
    h = synth.to_host_logits(synth.c1_rows(1, seed=43))
    walls = []
    for i in range(1020):
        t0 = time.perf_counter()
        d3s.sample(h, 0.7, 30, 0.7, i)
        walls.append((time.perf_counter() - t0) * 1e6)
    walls = sorted(walls[20:])
    out = {"c1_device_graph_us_per_call": graph_ms * 1e3 / 100,
           "c1_device_p50_us": dev[len(dev) // 2], "c1_device_p99_us": dev[int(len(dev) * 0.99)],
           "c1_host_d3_sample_p50_us": walls[len(walls) // 2],
           "c1_host_d3_sample_p99_us": walls[int(len(walls) * 0.99)],
           "note": "device_graph: 100 calls in one CUDA graph; device_p50: events around one Python "
                   "call (host submission included); host_d3_sample: d3_sample, host logits in, "
                   "host id out, wall clock"}
    xs = synth.to_host_logits(synth.c1_rows(2000, seed=44))
    out.update(cpu_one_thread_row_us(xs, np.float32(0.7), np.float32(0.7), np.int32(30),
                                     np.uint64(42)))
    # the same host-in, host-out call from C on both sides, without numpy work
    # per call: the library's d3_sample and the oracle's, on preallocated arrays
    import ctypes

    import oracle
    Lg, Lc = d3s.lib(), oracle.lib()
    row = np.ascontiguousarray(xs[:1])
    res = np.zeros(1, np.int32)
    rp = row.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    op = res.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))

    def p50(fn, n=1020):
        ts = []
        for i in range(n):
            t0 = time.perf_counter()
            fn(i)
            ts.append((time.perf_counter() - t0) * 1e6)
        ts = sorted(ts[20:])
        return ts[len(ts) // 2], ts[int(len(ts) * 0.99)]

    g50, g99 = p50(lambda i: Lg.d3_sample(rp, 1, row.shape[1], 0.7, 30, 0.7, i, op))
    c50, c99 = p50(lambda i: Lc.d3o_d3_sample(rp, 1, row.shape[1], 0.7, 30, 0.7, i, op))
    out.update({"c1_host_d3_sample_c_call_p50_us": g50, "c1_host_d3_sample_c_call_p99_us": g99,
                "c1_cpu_1thread_c_call_p50_us": c50, "c1_cpu_1thread_c_call_p99_us": c99,
                "c1_c_call_note": "ctypes calls of the C functions on preallocated arrays: the "
                                  "library's d3_sample (host logits in, id out) and the oracle's "
                                  "d3o_d3_sample on one host thread"})
    return out


def measure_c2(ctx, torch, iters: int = 1000):
    """Config 2: bf16 [256, 4097] batches, per-row seeds, T 0.7 / top_p 0.7 /
    top_k 30, `iters` iterations over 64 distinct batches (134 MB, above L2)."""
    import synth
    N = 256
    xs = [synth.c2_logits(N, seed=500 + i) for i in range(64)]
    seeds = torch.arange(N, dtype=torch.int64, device="cuda") + 77
    ids = torch.empty(N, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream()

    def one(i):
        ctx.sample_rows(xs[i % 64], ids, temperature=0.7, top_p=0.7, top_k=30, seeds=seeds)

    for i in range(10):
        one(i)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(iters)]
    a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(st)
    for i, (a, b) in enumerate(evs):
        a.record(st)
        one(i)
        b.record(st)
    b0.record(st)
    torch.cuda.synchronize()
    per = sorted(a.elapsed_time(b) * 1e3 for a, b in evs)
    total_ms = a0.elapsed_time(b0)
    # one call on each of the 64 batches captured once and replayed: the GPU
    # time of a batch with no host submission in between
    gs = torch.cuda.Stream()
    gs.wait_stream(st)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(gs):
        with torch.cuda.graph(graph, stream=gs):
            for i in range(64):
                ctx.sample_rows(xs[i], ids, temperature=0.7, top_p=0.7, top_k=30, seeds=seeds,
                                stream=gs)
    torch.cuda.synchronize()
    reps = max(1, iters // 64)
    graph_us = _events_ms(torch, graph.replay, reps) * 1e3 / 64
    del graph
    peak, kind = load_peaks()
    bytes_batch = N * (2 * V + 8 + 4)
    p50 = per[len(per) // 2]
    ctx.check()
    return {"rows_per_s": N * iters / (total_ms / 1e3), "batch_p50_us": p50,
            "batch_p99_us": per[int(len(per) * 0.99)],
            "graph_us_per_batch": graph_us, "rows_per_s_graph": N / (graph_us * 1e-6),
            "roofline": {"bound": "hbm", "achieved": bytes_batch / (p50 * 1e-6) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": bytes_batch / (p50 * 1e-6) / 1e9 / peak,
                         "peak_source": kind, "bytes_per_batch": bytes_batch},
            "iterations": iters, "kernel": "one CTA per row, select in the same launch + wide (empty)",
            "note": "a batch is 2.1 MB: latency-bound (launch + one row per CTA), far under HBM; "
                    "rows_per_s and batch_p50 include the host's submission of each call, "
                    "graph_us_per_batch is 64 calls replayed from one CUDA graph"}


def measure_c3(ctx, torch, B: int, steps: int, warmup: int):
    """Config 3 at batch B: the lm_head projection alone (weight re-read from
    HBM: an L2-clearing read between launches) and the fused projection +
    sample call."""
    import d3s
    import synth
    D = 2048
    ctx.reserve(max(B, 1024))
    h, W = synth.c3_inputs(B, seed=7)
    logits = torch.empty(B, V, dtype=torch.bfloat16, device="cuda")
    ids = torch.empty(B, dtype=torch.int32, device="cuda")
    seeds = torch.arange(B, dtype=torch.int64, device="cuda")
    # the weight (16.8 MB) fits in L2: a 256 MB read between launches leaves
    # clean lines (a written buffer's write-back would compete with the reads)
    flush_buf = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    flush_out = torch.empty((), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()

    def timed(fn):
        evs = []
        for i in range(warmup + steps):
            torch.sum(flush_buf, dim=0, out=flush_out)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            fn()
            b.record(st)
            if i >= warmup:
                evs.append((a, b))
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in evs)

    proj_ms = timed(lambda: ctx.lmhead(h, W, out=logits))
    # the practical ceiling for this transfer size: torch's own reduction reading
    # the same weight bytes from HBM, timed the same way (a kernel this short is
    # dominated by launch, first-touch latency and ramp, not by bandwidth)
    read_ms = timed(lambda: torch.sum(W, dtype=torch.float32))
    fused_ms = timed(lambda: ctx.lmhead_sample(h, W, logits, ids, temperature=0.7, top_p=0.7,
                                               top_k=30, noise=d3s.NOISE_SEEDS, seeds=seeds))
    ctx.check()
    peak_gbs, gkind = load_peaks()
    peak_tf, tkind = load_tflops()
    bytes_ = V * D * 2 + B * D * 2 + B * V * 2
    flops = 2.0 * B * V * D
    gbs = bytes_ / (proj_ms / 1e3) / 1e9
    tfs = flops / (proj_ms / 1e3) / 1e12
    tensor = B > 64
    del flush_buf
    return {
        "B": B, "projection_us": proj_ms * 1e3, "fused_us": fused_ms * 1e3,
        "fused_rows_per_s": B / (fused_ms / 1e3),
        "projection_kernel": ("lmhead_gemv_kernel" if B <= 8 else
                              "lmhead_gemm2_kernel (tcgen05 cta_group::2)" if B >= 512 else
                              "lmhead_gemm_kernel (tcgen05, split-K)"),
        "roofline": ({"bound": "tensor", "achieved": tfs, "peak": peak_tf, "unit": "TFLOP/s",
                      "frac": tfs / peak_tf, "peak_source": tkind + " bf16 burst"} if tensor else
                     {"bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s",
                      "frac": gbs / peak_gbs, "peak_source": gkind}),
        "hbm_gbs": gbs, "tflops": tfs, "bytes": bytes_, "flops": flops,
        "calibration": {"torch_read_of_W_us": read_ms * 1e3,
                        "torch_read_GBs": V * D * 2 / (read_ms / 1e3) / 1e9,
                        "projection_vs_torch_read": read_ms / proj_ms,
                        "note": "torch.sum over W's 16.8 MB after the same L2-clearing read: "
                                "what a plain read of these bytes costs at this size"},
    }


def measure_c4(ctx, torch, frames: int):
    """Config 4: 512 streams x 9 codebook heads per frame (bf16 [512, 1024]
    rows, Zipf-biased), T 1.0, top_p 0.9, top_k 30, per-stream keys advanced in
    tower_decode_step order; each frame also draws main + retry on a
    [512, 4097] backbone row. Heads alone, the whole frame, and the frame
    replayed from one CUDA graph."""
    import synth
    S, H, Vh = 512, 9, 1024
    ctx.reserve(2 * S)
    bias = synth.zipf_bias(Vh, 11)
    heads = [synth.c4_logits(S, seed=100 + j, V=Vh, bias=bias) for j in range(H)]
    xb = synth.c1_rows(S, seed=5).to(torch.bfloat16)
    states = torch.randint(0, 2**31 - 1, (S, 2), dtype=torch.int32, device="cuda")
    hist = torch.zeros(S, 16, dtype=torch.int32, device="cuda")
    hl = torch.zeros(S, dtype=torch.int32, device="cuda")
    sub = torch.empty(S, 2 + H, 2, dtype=torch.int32, device="cuda")
    ids = torch.empty(S, dtype=torch.int32, device="cuda")

    def frame_on(stream=None):
        ctx.keys_next(states, 2 + H, sub=sub, stream=stream)
        ctx.frame_main(xb, sub, hist, hl, temperature=1.0, top_p=0.9, top_k=30,
                       semantic_start=1000, code_vocab=4096, eos_id=7, stream=stream)
        for j in range(H):
            ctx.sample_rows_keys(heads[j], ids, sub[:, 2 + j], temperature=1.0, top_p=0.9,
                                 top_k=30, stream=stream)

    def heads_only():
        for j in range(H):
            ctx.sample_rows_keys(heads[j], ids, sub[:, 2 + j], temperature=1.0, top_p=0.9, top_k=30)

    frames = max(1, frames)
    frame_ms = _events_ms(torch, frame_on, frames)
    heads_ms = _events_ms(torch, heads_only, frames)
    ctx.check()
    gs = torch.cuda.Stream()
    gs.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(gs):
        with torch.cuda.graph(graph, stream=gs):
            frame_on(gs)
    torch.cuda.synchronize()
    graph_ms = _events_ms(torch, graph.replay, frames)
    del graph
    ctx.check()
    peak, kind = load_peaks()
    head_bytes = H * S * (2 * Vh + 4)
    return {
        "head_rows_per_s": S * H / (heads_ms / 1e3), "ms_per_frame_heads": heads_ms,
        "ms_per_frame_all": frame_ms, "frame_rows_per_s": S * (H + 2) / (frame_ms / 1e3),
        "ms_per_frame_graph": graph_ms, "frame_rows_per_s_graph": S * (H + 2) / (graph_ms / 1e3),
        "frames": frames,
        "roofline": {"bound": "hbm", "achieved": head_bytes / (heads_ms / 1e3) / 1e9, "peak": peak,
                     "unit": "GB/s", "frac": head_bytes / (heads_ms / 1e3) / 1e9 / peak,
                     "peak_source": kind, "bytes_per_frame_heads": head_bytes},
        "note": "a head launch is 512 rows of 2 KB: launch-bound; the frame's rows stay in L2",
    }


def run_ours(args):
    import torch
    import torch.distributed as dist

    import d3s
    import shard
    import synth
    rank, world, local = env_ranks()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device(f"cuda:{local}"))
    rows = args.rows
    ctx = d3s.Context(local)
    ctx.reserve(rows)
    x, T, p, k, seeds = synth.c5_batch(rows, seed=1000 + rank)
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream()
    # N > 1: each rank's sampler writes its ids straight into rank 0's result
    # over NVLink (d3s_gather). A rank > 0 signals each step on a side stream
    # (after an event of its sampler's stream), overlapping its next step; rank
    # 0 completes the gather of step s on its own stream right after sampling
    # step s + 1, when every rank's signal for s has landed, so its wait ends at
    # once and never spins beside a sampler. Four slots let a rank run up to
    # three steps ahead of rank 0's gather.
    gather = d3s.Gather(local, world, rank, world * rows, shard.handle_exchange(), slots=4) \
        if world > 1 else None
    gather_out = torch.empty(world * rows, dtype=torch.int32, device="cuda") \
        if gather is not None and rank == 0 else None
    side = torch.cuda.Stream() if gather is not None and rank != 0 else None
    next_step = [0]     # the step the next sampler call writes
    pending = []        # rank 0: sampled steps whose gather is not yet complete

    def target():
        """Where this step's ids go: the local tensor, or (N > 1) this rank's
        rows of rank 0's result (waits until rank 0 released step - slots)."""
        return gather.begin(next_step[0], stream=st) if gather is not None else ids

    def sample(out):
        ctx.sample_rows(x, out, temperature=T, top_p=p, top_k=k, seeds=seeds)

    def finish(s_, host_out=None):
        """Rank 0: wait for every rank's ids of step s_ (on the sampler's
        stream), copy them to host_out if given, release the slot."""
        gather.end(s_, stream=st)
        if host_out is not None:
            gather.copy_result(s_, gather_out, stream=st)
            host_out.copy_(gather_out, non_blocking=True)
        gather.release(s_, stream=st)

    def collect(host_out=None, last=False):
        """After a sampler call (N > 1). Ranks > 0: signal on the side stream.
        Rank 0: complete the gather of the previous step (or, with last, of
        every step still pending)."""
        if gather is None:
            return
        s_ = next_step[0]
        next_step[0] += 1
        if rank != 0:
            ev = torch.cuda.Event()
            ev.record(st)
            side.wait_event(ev)
            gather.end(s_, stream=side)
            return
        pending.append(s_)
        while len(pending) > (0 if last else 1):
            finish(pending.pop(0), host_out)

    def drain(host_out=None):
        """End of a loop: rank 0 completes every pending step's gather; ranks
        > 0 order their stream after their last signal."""
        if gather is None:
            return
        if rank == 0:
            while pending:
                finish(pending.pop(0), host_out)
        else:
            st.wait_stream(side)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    lines = [0]

    def line_up():
        """N > 1: every GPU's stream waits at a start line until all ranks'
        streams reach it, so the timed work starts on all GPUs together (the
        processes leave the barrier at different host times, and rank 0, which
        waits for every rank's last step, would otherwise time that skew)."""
        if gather is not None:
            lines[0] += 1
            gather.line_up(lines[0], stream=st)

    def over_ranks(vals: list[float]) -> list[list[float]]:
        if world == 1:
            return [vals]
        t = torch.tensor(vals, device="cuda", dtype=torch.float64)
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [o.tolist() for o in out]

    barrier()
    for _ in range(args.warmup):
        sample(target())
        collect()
    drain()
    barrier()
    uuid = str(getattr(torch.cuda.get_device_properties(local), "uuid", "") or "")
    phys = int((os.environ.get("CUDA_VISIBLE_DEVICES", "") or str(local)).split(",")[local]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES", "").replace(",", "").isdigit() else local
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(args.steps)]
    with Clocks(uuid, phys, 0.00025 if rank == 0 else 0.001) as clk:
        line_up()
        start.record(st)
        for i in range(args.steps):
            out = target()
            kev[i][0].record(st)
            sample(out)
            kev[i][1].record(st)
            collect()
            kev[i][2].record(st)
        drain()  # the job ends when rank 0 holds the last step's ids
        end.record(st)
        barrier()
    elapsed_local = start.elapsed_time(end)
    kernel_ms = statistics.mean(a.elapsed_time(b) for a, b, _ in kev)
    collect_ms = statistics.mean(b.elapsed_time(c) for _, b, c in kev)
    per_rank = over_ranks([elapsed_local, kernel_ms, collect_ms])
    elapsed_ms = max(r[0] for r in per_rank)
    kernel_ms_max = max(r[1] for r in per_rank)
    if gather is not None:
        gather.check()
    ctx.check()
    clocks = clk.summary()
    if world > 1:
        all_clocks = [None] * world
        dist.all_gather_object(all_clocks, clocks)
        clocks = merge_clocks(all_clocks)

    # end to end through the C ABI with host buffers: pinned host -> device copy of
    # the step's inputs, the sampler, the ids to rank 0 (N > 1), device -> host
    # copy of the ids, every step
    e2e = None
    if not args.no_e2e:
        hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        hx.copy_(x)
        hT, hp, hk, hs = (t.cpu().pin_memory() for t in (T, p, k, seeds))
        hids = torch.empty(world * rows if rank == 0 else rows, dtype=torch.int32, pin_memory=True)
        dx, dT, dp, dk, ds = (torch.empty_like(t) for t in (x, T, p, k, seeds))
        did = torch.empty_like(ids)

        def e2e_step():
            dx.copy_(hx, non_blocking=True)
            dT.copy_(hT, non_blocking=True)
            dp.copy_(hp, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            ds.copy_(hs, non_blocking=True)
            if gather is None:
                ctx.sample_rows(dx, did, temperature=dT, top_p=dp, top_k=dk, seeds=ds)
                hids.copy_(did, non_blocking=True)
                return
            out = target()
            ctx.sample_rows(dx, out, temperature=dT, top_p=dp, top_k=dk, seeds=ds)
            collect(host_out=hids if rank == 0 else None)

        e2e_steps = max(3, min(args.steps, 10))
        for _ in range(2):
            e2e_step()
        drain(hids if rank == 0 else None)
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        line_up()
        a.record(st)
        for _ in range(e2e_steps):
            e2e_step()
        drain(hids if rank == 0 else None)
        b.record(st)
        barrier()
        e2e_ms = max(r[0] for r in over_ranks([a.elapsed_time(b)]))
        if gather is not None:
            gather.check()
        h2d = hx.numel() * hx.element_size() + sum(t.numel() * t.element_size() for t in (hT, hp, hk, hs))
        e2e = {"value": world * rows * e2e_steps / (e2e_ms / 1e3), "unit": "rows/s",
               "h2d_bytes_per_step": int(h2d) * world, "d2h_bytes_per_step": int(world * rows * 4),
               "steps": e2e_steps,
               "path": ("pinned host -> cudaMemcpyAsync -> d3s_sample -> ids to host" if world == 1 else
                        "per rank: pinned host -> cudaMemcpyAsync -> d3s_sample writing into rank 0's "
                        "result over NVLink (d3s_gather); rank 0: the N ids to host")}
        del hx

    cpu = None
    latency = None
    configs = None
    calibration = None
    if rank == 0 and world == 1:
        # what a plain read of the same logits costs: torch's own reductions over
        # the 1.07 GB, timed the same way (CUDA events, warm)
        read_ms = min(_events_ms(torch, lambda: torch.sum(x, dtype=torch.float32), 10),
                      _events_ms(torch, lambda: torch.amax(x, dim=1), 10))
        calibration = {"torch_read_of_logits_ms": read_ms,
                       "torch_read_GBs": x.numel() * x.element_size() / (read_ms * 1e-3) / 1e9,
                       "sampler_call_vs_read": read_ms / kernel_ms,
                       "note": "the faster of torch.sum and torch.amax(dim=1) over the logits: a "
                               "plain read of the bytes the sampler's stream reads"}
        if not args.no_latency:
            latency = c1_latency(ctx, torch)
        if not args.no_configs:
            configs = {"c2": measure_c2(ctx, torch),
                       "c3": {f"B{B}": measure_c3(ctx, torch, B, 20, 5) for B in (1, 64, 1024)},
                       "c4": measure_c4(ctx, torch, 200)}
        if not args.no_cpu_baseline:
            n = min(rows, 16384)
            cpu = cpu_baseline(synth.to_host_logits(x[:n]), T[:n].cpu().numpy(), p[:n].cpu().numpy(),
                               k[:n].cpu().numpy(), seeds[:n].cpu().numpy().astype("uint64"))

    if rank == 0:
        peak, peak_kind = load_peaks()
        bytes_per_launch = rows * BYTES_PER_ROW
        achieved = bytes_per_launch / (kernel_ms / 1e3) / 1e9
        traffic = load_traffic()
        line = {
            "metric": METRIC, "value": world * rows * args.steps / (elapsed_ms / 1e3), "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "rows_per_gpu": rows, "V": V, "global_batch": world * rows,
                       "parallelism": (f"rows sharded over {world} GPUs, ids written into rank 0's "
                                       "result over NVLink" if world > 1 else "one GPU"),
                       "l2": "inputs 1.07 GB per GPU > 126 MB L2 (no flush needed)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "one sampler call: sample_stats1_kernel<33,f32> + "
                                   "sample_select_kernel + sample_wide_kernel (the hand-off list)",
                         "kernel_ms": kernel_ms, "kernel_ms_max_over_ranks": kernel_ms_max,
                         "bytes_per_launch": bytes_per_launch},
            "per_rank_ms": [{"rank": r, "step_loop": v[0], "sample_mean": v[1],
                             "gather_step_mean": v[2]} for r, v in enumerate(per_rank)],
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": (3 + (2 if world > 1 else 0)) * args.steps,
            "cpu_baseline": cpu,
            "latency": latency,
            "calibration": calibration,
            "configs": configs,
        }
        print(json.dumps(line), flush=True)
    if gather is not None:
        barrier()
        gather.close()
    ctx.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def _events_ms(torch, fn, steps: int, warmup: int = 3) -> float:
    """Mean device time of fn() over `steps` calls (CUDA events, current stream)."""
    st = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(steps):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def load_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        for key in ("bf16_tflops", "bf16_tflops_burst"):
            if key in d:
                return float(d[key]), "measured"
    return 1590.0, "fallback"


def run_c3(args):
    """Config 3 on its own line: the lm_head projection and the fused
    projection + sample call at --batch B."""
    import torch

    import d3s
    torch.cuda.set_device(0)
    ctx = d3s.Context(0)
    r = measure_c3(ctx, torch, args.batch, args.steps, args.warmup)
    line = {"metric": "lm_head + sample rows/s (config 3)", "value": r["fused_rows_per_s"],
            "unit": "rows/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["fused_us"] / 1e3, "higher_is_better": True,
            "dtype": "bf16 x bf16 -> f32 accumulate -> bf16 logits", "data": "synthetic",
            "config": {"workload": f"config3: h bf16 [{args.batch}, 2048] ~N(0,1), W bf16 [{V}, 2048] "
                                   "~N(0,0.02), T 0.7, top_p 0.7, top_k 30, per-row seeds",
                       "l2": "256 MB buffer read between launches"}, **r}
    print(json.dumps(line), flush=True)
    ctx.close()


def run_c4(args):
    """Config 4 on its own line."""
    import torch

    import d3s
    torch.cuda.set_device(0)
    ctx = d3s.Context(0)
    r = measure_c4(ctx, torch, args.frames)
    line = {"metric": "tower head rows/s (config 4)", "value": r["head_rows_per_s"], "unit": "rows/s",
            "n_gpus": 1, "higher_is_better": True, "dtype": "bf16 logits, f32 math",
            "data": "synthetic",
            "config": {"workload": "config4: 512 streams x 9 heads, V=1024 bf16 ~N(0,2.5)+Zipf(1.1); "
                                   "frame main+retry on [512, 4097] bf16; T 1.0, top_p 0.9, top_k 30"},
            **r}
    print(json.dumps(line), flush=True)
    ctx.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "c3":
        run_c3(args)
    elif args.workload == "c4":
        run_c4(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
