"""Benchmark of the trnfft_b200 hot path (one JSON line on rank 0).

Default workload: batched 1-D complex FFT + IFFT
round trip, N = 1024, batch = 8192 per GPU, float32 planar re/im, entries
N(0,1) from a seed.  One step = trnfft.fft then trnfft.ifft of the batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU runs are launched one process per GPU by torch.distributed.run;
the batch is sharded (weak scaling: every rank transforms its own 8192 rows,
no collective on the data path) and the step time is the maximum over ranks.

Metric: GFLOP/s under the 5 N log2 N convention (two transforms per step),
whole-job aggregate.  ``value`` is timed with device-resident inputs and
CUDA events; ``e2e`` repeats the step through the public API with the inputs
copied from pinned host memory and the result copied back inside the timed
region.  L2 is flushed (256 MiB read sweep) before every timed step.

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/trnfft_oracle.py, the reference's own radix-2 path) on the host
cores, on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

N = 1024
BATCH = 8192
METRIC = "batched C2C FFT GFLOP/s (5N*log2N), FFT+IFFT round trip"
UNIT = "GFLOP/s"
FALLBACK_HBM_GBS = 6650.0
FLUSH_BYTES = 256 << 20


def flops_per_step(n=N, batch=BATCH):
    return 2 * 5.0 * n * math.log2(n) * batch


def algorithmic_bytes_per_launch(n=N, batch=BATCH):
    # read re+im, write re+im: 16 bytes per complex point
    return 16.0 * n * batch


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs"), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(kernel_key):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        v = d.get(kernel_key)
        if isinstance(v, dict):
            return v.get("dram_bytes_per_launch")
    return None


class ClockSampler:
    """Samples SM clocks and throttle reasons (NVML) while the timed region runs."""

    REASONS = {  # nvmlClocksEventReason bits
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.0005):
        self.index = index
        self.period = period_s
        self.sm = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self.ok = False

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            return self
        self._sample()
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()
        return self

    def _sample(self):
        nv = self.nv
        self.sm.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        try:
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        for name, b in self.REASONS.items():
            if bits & b:
                self.reasons.add(name)

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join(timeout=2)
            self._sample()

    def summary(self):
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    return world, rank, local


def allreduce_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rel_err(a, b):
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b))


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------------------
# CPU baseline: the oracle restatement of the reference's radix-2 algorithm
# ---------------------------------------------------------------------------


def cpu_reference_sample(rows: int, threads: int, seed: int = 0):
    """Times fft+ifft of `rows` rows of N=1024 with the oracle on `threads` threads."""
    from oracle import trnfft_oracle as O

    rng = np.random.default_rng(seed)
    xr = rng.standard_normal((rows, N)).astype(np.float32)
    xi = rng.standard_normal((rows, N)).astype(np.float32)

    def step(a, b):
        yr, yi = O.fft(a, b)
        return O.ifft(yr, yi)

    t0 = time.perf_counter()
    O.threaded_rows(step, (xr, xi), threads)
    return time.perf_counter() - t0


def cpu_baseline(budget_s: float = 10.0):
    threads = os.cpu_count() or 1
    rows = 512
    cpu_reference_sample(64, threads)  # warm-up
    done, elapsed = 0, 0.0
    while elapsed < budget_s:
        elapsed += cpu_reference_sample(rows, threads, seed=done)
        done += rows
    value = flops_per_step(N, done) / elapsed / 1e9
    return {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"oracle/trnfft_oracle.py radix-2 fft+ifft, N={N}, {done} rows "
                      f"(of {BATCH} per step) in {elapsed:.1f} s on {threads} threads"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    rows = 256
    for _ in range(args.warmup):
        cpu_reference_sample(rows, threads)
    times = [cpu_reference_sample(rows, threads, seed=k) for k in range(args.steps)]
    ms = 1000.0 * sum(times) / len(times) * (BATCH / rows)  # per full step of BATCH rows
    value = flops_per_step(N, rows) / (sum(times) / len(times)) / 1e9
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"batched C2C FFT+IFFT round trip, N={N}, batch={BATCH} per GPU "
                               "(BASELINE configs[0]); each step times a bounded sample of "
                               f"{rows} rows and reports the rate", "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{rows} rows of N={N} fft+ifft per step, oracle/trnfft_oracle.py"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------


def run_ours(args, world, rank, local):
    import trnfft_b200 as trnfft
    from trnfft_b200 import ComplexTensor

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    xr = torch.randn(BATCH, N, device=dev, generator=g)
    xi = torch.randn(BATCH, N, device=dev, generator=g)
    flush = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    flush_out = torch.empty(1, dtype=torch.float32, device=dev)

    def flush_l2():
        # read-only sweep of a buffer twice the L2 size: evicts every line
        # (dirty lines are written back here, not inside the timed kernel)
        torch.sum(flush, dim=0, keepdim=True, out=flush_out)
    x = ComplexTensor(xr, xi)

    def step():
        y = trnfft.fft(x)
        return trnfft.ifft(y)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    # The step (and each launch alone) is captured once as a CUDA graph, so the
    # device timing below contains no host dispatch gaps.  Before every timed
    # replay the L2 is flushed; the flush is enqueued first so the GPU is busy
    # while the events and the replay are queued behind it.
    st = torch.cuda.current_stream(dev)
    g_step, g_fft, g_ifft = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        y_step = step()
    with torch.cuda.graph(g_fft):
        y_fft = trnfft.fft(x)
    with torch.cuda.graph(g_ifft):
        y_ifft = trnfft.ifft(x)
    for g in (g_step, g_fft, g_ifft):
        g.replay()
    torch.cuda.synchronize()

    def timed(graph):
        flush_l2()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        graph.replay()
        e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1)

    launch_ms = []
    for _ in range(max(3, args.steps // 2)):
        launch_ms.append(timed(g_fft))
        launch_ms.append(timed(g_ifft))

    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        step_ms = [timed(g_step) for _ in range(args.steps)]
        torch.cuda.synchronize()
    barrier(world)
    ms_local = sum(step_ms) / len(step_ms)
    ms = allreduce_max(ms_local, world)
    value = world * flops_per_step() / (ms / 1e3) / 1e9
    ok = rel_err(y_step.real, xr) < 1e-5 and rel_err(y_fft.real, torch.fft.fft(torch.complex(xr, xi)).real) < 1e-5

    # end to end: pinned host inputs -> device -> fft -> ifft -> pinned host result
    hr = torch.empty(BATCH, N, dtype=torch.float32, pin_memory=True)
    hi = torch.empty(BATCH, N, dtype=torch.float32, pin_memory=True)
    hr.copy_(xr.cpu())
    hi.copy_(xi.cpu())
    outr = torch.empty_like(hr, pin_memory=True)
    outi = torch.empty_like(hi, pin_memory=True)
    dr = torch.empty_like(xr)
    di = torch.empty_like(xi)

    def e2e_step():
        dr.copy_(hr, non_blocking=True)
        di.copy_(hi, non_blocking=True)
        y = trnfft.ifft(trnfft.fft(ComplexTensor(dr, di)))
        outr.copy_(y.real, non_blocking=True)
        outi.copy_(y.imag, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        e2e_step()
        e1.record(st)
        e1.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    barrier(world)
    e2e_max = allreduce_max(sum(e2e_ms) / len(e2e_ms), world)
    e2e_value = world * flops_per_step() / (e2e_max / 1e3) / 1e9

    err = rel_err(y_step.real, xr)

    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    avg_launch = sum(launch_ms) / len(launch_ms)
    achieved = algorithmic_bytes_per_launch() / (avg_launch / 1e3) / 1e9
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"batched C2C FFT+IFFT round trip, N={N}, batch={BATCH} per GPU "
                               "(BASELINE configs[0])",
                   "global_batch": BATCH * world, "seq_len": N, "parallelism": f"batch-sharded x{world}",
                   "l2": "flushed before every timed step (256 MiB read sweep)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": profiled_traffic("k_c2c_n1024_b8192"),
                     "kernel": "k_c2c<10,5> (Stockham radix 32-32)",
                     "algorithmic_bytes_per_launch": algorithmic_bytes_per_launch(),
                     "avg_launch_ms": round(avg_launch, 5)},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "ms_per_step": round(e2e_max, 4),
                "h2d_bytes_per_step": 2 * BATCH * N * 4, "d2h_bytes_per_step": 2 * BATCH * N * 4},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
        "roundtrip_rel_l2": err, "parity_ok": bool(ok),
        "timing": "CUDA events around CUDA-graph replays of the step; L2 flushed before each",
    }
    if world == 1:
        out["cpu_baseline"] = cpu_baseline(args.cpu_budget)
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    args = ap.parse_args()
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
