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
import datetime
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


def measured_tensor_peak():
    """Dense TF32 tensor peak: half the measured dense bf16 cuBLAS rate (TF32 issues at half
    the bf16 rate on B200, 1.1 vs 2.25 PFLOP/s nominal)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return round(d["bf16_tflops"] / 2.0, 1), "measured bf16 / 2"
    return round(1590.0 / 2.0, 1), "fallback bf16 / 2"


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
            # a short collective timeout: a rank that stops answering ends the run in minutes
            dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                    timeout=datetime.timedelta(seconds=240))
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
# Workloads.  Each names its config, builds device inputs, a step (one pass of
# the hot path over one batch), its kernel launches, the work per step for
# the metric, the algorithmic HBM bytes of the dominant launch, and a bounded
# CPU sample of the same work on the oracle (the reference's algorithm).
# ---------------------------------------------------------------------------


def c2c_flops(n, batch):
    return 5.0 * n * math.log2(n) * batch


class Workload:
    metric = METRIC
    unit = UNIT
    dominant = None

    def release(self):
        """Drop the device inputs (the default run frees them before its extras)."""
        for k in ("xr", "xi", "xs", "x", "inputs", "step", "launches", "e2e_fn"):
            if hasattr(self, k):
                setattr(self, k, None)

    def cpu_sample(self, threads):
        raise NotImplementedError


class C2CRoundTrip(Workload):
    """fft then ifft of a (batch, n) planar complex batch (BASELINE configs[0] / [3])."""

    def __init__(self, n, batch, tag):
        self.n, self.batch, self.tag = n, batch, tag
        self.name = f"batched C2C FFT+IFFT round trip, N={n}, batch={batch} per GPU ({tag})"
        self.work = 2 * c2c_flops(n, batch)
        self.dom_bytes = 16.0 * n * batch
        smooth = n
        for f in (2, 3, 5, 7):
            while smooth % f == 0:
                smooth //= f
        alg = ("Stockham" if n & (n - 1) == 0 else
               ("direct mixed-radix" if smooth == 1 and n <= 8192 else "fused Bluestein"))
        self.dominant = f"{alg} C2C kernel, N={n}"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft
        from trnfft_b200 import ComplexTensor

        self.xr = torch.randn(self.batch, self.n, device=dev, generator=g)
        self.xi = torch.randn(self.batch, self.n, device=dev, generator=g)
        x = ComplexTensor(self.xr, self.xi)
        self.step = lambda: trnfft.ifft(trnfft.fft(x))
        self.launches = {"fft": lambda: trnfft.fft(x), "ifft": lambda: trnfft.ifft(x)}
        self.launches_per_step = 2
        self.inputs = [self.xr, self.xi]

        def from_inputs(ts):
            y = trnfft.ifft(trnfft.fft(ComplexTensor(ts[0], ts[1])))
            return [y.real, y.imag]

        self.e2e_fn = from_inputs

    def check(self, out):
        return rel_err(out.real, self.xr)

    def ref_full_units(self):
        return self.batch

    def ref_sample(self, T, units):
        g = torch.Generator().manual_seed(0)
        x = T.ComplexTensor(torch.randn(units, self.n, generator=g), torch.randn(units, self.n, generator=g))
        return (lambda: T.ifft(T.fft(x))), 2 * c2c_flops(self.n, units), f"{units} of {self.batch} rows"

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        rng = np.random.default_rng(0)
        xr = rng.standard_normal((rows, self.n)).astype(np.float32)
        xi = rng.standard_normal((rows, self.n)).astype(np.float32)
        prec = "fast"

        def f(a, b):
            yr, yi = O.fft(a, b, precision=prec)
            return O.ifft(yr, yi, precision=prec)

        t0 = time.perf_counter()
        O.threaded_rows(f, (xr, xi), threads)
        return time.perf_counter() - t0, 2 * c2c_flops(self.n, rows)


class SmallN(Workload):
    """BASELINE configs[1](a): batch 262144 forward FFTs for each of N = 64, 128, 256."""

    def __init__(self):
        self.batch = 262144
        self.ns = (64, 128, 256)
        self.name = "small-N batched C2C FFT, N=64,128,256, batch=262144 each (configs[1]a)"
        self.work = sum(c2c_flops(n, self.batch) for n in self.ns)
        self.dom_bytes = 16.0 * 256 * self.batch
        self.dominant = "Stockham C2C kernel, N=256"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft
        from trnfft_b200 import ComplexTensor

        self.xs = [ComplexTensor(torch.randn(self.batch, n, device=dev, generator=g),
                                 torch.randn(self.batch, n, device=dev, generator=g)) for n in self.ns]
        self.step = lambda: [trnfft.fft(x) for x in self.xs][-1]
        self.launches = {"fft256": lambda: trnfft.fft(self.xs[-1])}
        self.launches_per_step = 3
        self.inputs = [t for x in self.xs for t in (x.real, x.imag)]

        def from_inputs(ts):
            outs = []
            for k in range(3):
                y = trnfft.fft(ComplexTensor(ts[2 * k], ts[2 * k + 1]))
                outs += [y.real, y.imag]
            return outs

        self.e2e_fn = from_inputs

    def check(self, out):
        x = self.xs[-1]
        ref = torch.fft.fft(torch.complex(x.real, x.imag))
        return rel_err(torch.complex(out.real, out.imag), ref)

    def ref_full_units(self):
        return self.batch

    def ref_sample(self, T, units):
        g = torch.Generator().manual_seed(0)
        xs = [T.ComplexTensor(torch.randn(units, n, generator=g), torch.randn(units, n, generator=g))
              for n in self.ns]
        return ((lambda: [T.fft(x) for x in xs]), sum(c2c_flops(n, units) for n in self.ns),
                f"{units} of {self.batch} rows for each N")

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        rng = np.random.default_rng(0)
        t = 0.0
        work = 0.0
        for n in self.ns:
            xr = rng.standard_normal((rows, n)).astype(np.float32)
            xi = rng.standard_normal((rows, n)).astype(np.float32)
            t0 = time.perf_counter()
            O.threaded_rows(lambda a, b: O.fft(a, b), (xr, xi), threads)
            t += time.perf_counter() - t0
            work += c2c_flops(n, rows)
        return t, work


class Stft(Workload):
    """256 waveforms x 160000 samples, n_fft 512, hop 256, Hann, reflect."""

    metric = "STFT frames/s (256 x 160000 samples, n_fft 512, hop 256, onesided)"
    unit = "frames/s"

    def __init__(self):
        self.B, self.L, self.nfft, self.hop = 256, 160000, 512, 256
        self.frames = 1 + (self.L + 2 * (self.nfft // 2) - self.nfft) // self.hop
        self.name = "STFT 256 x 160000 samples, n_fft=512, hop=256, periodic Hann, reflect (configs[2])"
        self.work = float(self.B * self.frames)
        self.dom_bytes = 4.0 * self.B * self.L + 8.0 * self.B * self.frames * (self.nfft // 2 + 1)
        self.dominant = "fused STFT kernel (n_fft=512)"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft

        t = torch.arange(self.L, device=dev, dtype=torch.float32) / 16000.0
        x = torch.randn(self.B, self.L, device=dev, generator=g)
        f = 50.0 + 6950.0 * torch.rand(self.B, 8, 1, device=dev, generator=g)
        ph = 2 * math.pi * torch.rand(self.B, 8, 1, device=dev, generator=g)
        x = x + torch.sin(2 * math.pi * f * t + ph).sum(1)
        self.x = x.contiguous()
        self.win = torch.hann_window(self.nfft, device=dev)
        self.step = lambda: trnfft.stft(self.x, self.nfft, self.hop, window=self.win)
        self.launches = {"stft": self.step}
        self.launches_per_step = 1
        self.inputs = [self.x]
        self.e2e_fn = lambda ts: (lambda S: [S.real, S.imag])(
            trnfft.stft(ts[0], self.nfft, self.hop, window=self.win))

    def check(self, out):
        ref = torch.stft(self.x[:8], self.nfft, self.hop, window=self.win, center=True, pad_mode="reflect",
                         return_complex=True)
        return rel_err(torch.complex(out.real[:8], out.imag[:8]), ref)

    def ref_full_units(self):
        return self.B

    def ref_sample(self, T, units):
        g = torch.Generator().manual_seed(0)
        x = torch.randn(units, self.L, generator=g)
        win = torch.hann_window(self.nfft)
        return ((lambda: T.stft(x, self.nfft, self.hop, window=win)), float(units * self.frames),
                f"{units} of {self.B} waveforms")

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        rng = np.random.default_rng(0)
        w = rng.standard_normal((max(1, rows // 64), self.L)).astype(np.float32)
        t0 = time.perf_counter()
        O.threaded_rows(lambda a: O.stft(a, self.nfft, self.hop), (w,), threads)
        return time.perf_counter() - t0, float(w.shape[0] * self.frames)


class Large(Workload):
    metric = "single large C2C FFT GFLOP/s (5N*log2N)"
    e2e_rows = False

    """BASELINE configs[4]: one N = 2^30 complex forward FFT.

    One GPU: four column-tile passes.  N GPUs (torch.distributed.run): the four-step FFT of
    trnfft_b200.distributed with column-block input (rank p holds x[n1*N2 + n2] for n2 in its
    block); the last column pass stores its output straight into the owning ranks' row buffers
    over NVLink (CUDA IPC mappings), then each rank runs its row transforms; output
    X[k1 + N1*k2] for k1 in the rank's block.  Total work is fixed as N grows ("strong" scaling)."""

    def __init__(self, logn=30):
        self.logn = logn
        self.n = 1 << logn
        self.name = f"single 1-D C2C forward FFT, N=2^{logn} (8 GiB planar at 2^30) (configs[4])"
        self.work = c2c_flops(self.n, 1)
        self.dom_bytes = 4 * 16.0 * self.n  # four column-tile passes, each reads and writes all data
        self.dominant = "four column-tile passes (256 x 256 x 128 x 128), one fft"
        self.scaling = "strong"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft
        from trnfft_b200 import ComplexTensor

        world = int(os.environ.get("WORLD_SIZE", "1"))
        self.world = world
        if world == 1:
            from trnfft_b200 import distributed as D

            # the same four-step split as the multi-GPU run (2^16-point columns x 2^14-point
            # rows, transposed output order): three HBM passes on one GPU
            N1, N2 = D._split_n(self.n)
            self.xr = torch.randn(N1, N2, device=dev, generator=g)
            self.xi = torch.randn(N1, N2, device=dev, generator=g)
            x = ComplexTensor(self.xr, self.xi)
            self.step = lambda: D.fft_four_step_local(x, self.n)
            self.launches = {"fft": self.step}
            self.launches_per_step = 3
            self.dom_bytes = 3 * 16.0 * self.n
            self.min_bytes = 2 * 16.0 * self.n
            self.dominant = "four-step on one GPU: two column passes (twiddle fused) + one 16384-point row pass"
            self.name = (f"single 1-D C2C forward FFT, N=2^{self.logn}, four-step 2^16 x 2^14 on one GPU, "
                         "transposed output order (configs[4])")
            self.e2e_fn = lambda ts: (lambda y: [y.real, y.imag])(
                D.fft_four_step_local(ComplexTensor(ts[0], ts[1]), self.n))
            self.natural = lambda: trnfft.fft(ComplexTensor(self.xr.reshape(1, -1), self.xi.reshape(1, -1)))
        else:
            from trnfft_b200 import distributed as D

            N1, N2 = D._split_n(self.n)
            self.xr = torch.randn(N1, N2 // world, device=dev, generator=g)
            self.xi = torch.randn(N1, N2 // world, device=dev, generator=g)
            x = ComplexTensor(self.xr, self.xi)
            self.step = lambda: D.fft_distributed(x, self.n, natural_order=False, columns_in=True)
            self.launches = {}
            self.no_graph = True
            self.launches_per_step = 3  # two column passes (the second scatters to the peers) + one row pass
            self.e2e_fn = lambda ts: (lambda y: [y.real, y.imag])(
                D.fft_distributed(ComplexTensor(ts[0], ts[1]), self.n, natural_order=False, columns_in=True))
            self.name = (f"single 1-D C2C forward FFT, N=2^{self.logn} across {world} GPUs, four-step with the "
                         "exchange fused into the column kernel (NVLink peer stores) (configs[4])")
            self.dominant = "distributed four-step (column passes with peer-store exchange, row passes)"
            self.dom_bytes = 3 * 16.0 * self.n / world  # three passes, each reads and writes the local block
        self.inputs = [self.xr, self.xi]

    def ref_sample(self, T, units):
        from trnfft.nki.multicore import _stage_parallel_fft

        n = 1 << 20
        g = torch.Generator().manual_seed(0)
        x = T.ComplexTensor(torch.randn(n, generator=g), torch.randn(n, generator=g))
        return ((lambda: _stage_parallel_fft(x, 1, False)), c2c_flops(n, 1),
                "one N=2^20 transform through the reference's four-step _stage_parallel_fft")

    ref_fixed_units = True

    def check(self, out):
        # Parseval over all ranks: sum |X|^2 = N sum |x|^2
        ex = (self.xr.double() ** 2).sum() + (self.xi.double() ** 2).sum()
        eX = (out.real.double() ** 2).sum() + (out.imag.double() ** 2).sum()
        if self.world > 1:
            import torch.distributed as dist

            t = torch.stack([ex, eX])
            dist.all_reduce(t)
            ex, eX = t[0], t[1]
        return abs(float(eX / (ex * self.n)) - 1.0)

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        n = 1 << 20
        rng = np.random.default_rng(0)
        xr = rng.standard_normal(n).astype(np.float32)
        xi = rng.standard_normal(n).astype(np.float32)
        t0 = time.perf_counter()
        O.stage_parallel_fft(xr, xi, False)
        return time.perf_counter() - t0, c2c_flops(n, 1)


class Fft2(Workload):
    metric = "fft2 GFLOP/s (5N*log2N per row and column transform)"
    e2e_rows = False

    """BASELINE configs[4] second part: fft2 of a 16384 x 16384 complex field (1 GPU)."""

    def __init__(self, side=16384):
        self.s = side
        self.name = f"fft2 of a {side}x{side} complex fp32 field (configs[4], 1 GPU)"
        self.work = 2 * c2c_flops(side, side)
        # the passes that run: two strided column passes (16384 points > one 1024-point column
        # tile) and one row pass (k_c2c_big); the minimum is two passes (read + write once per axis)
        self.dom_bytes = 3 * 16.0 * side * side
        self.min_bytes = 2 * 16.0 * side * side
        self.dominant = "fft2: two strided column passes + one 16384-point row pass"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft
        from trnfft_b200 import ComplexTensor

        self.xr = torch.randn(self.s, self.s, device=dev, generator=g)
        self.xi = torch.randn(self.s, self.s, device=dev, generator=g)
        x = ComplexTensor(self.xr, self.xi)
        self.step = lambda: trnfft.fft2(x)
        self.launches = {"fft2": self.step}
        self.launches_per_step = 4
        self.inputs = [self.xr, self.xi]
        self.e2e_fn = lambda ts: (lambda y: [y.real, y.imag])(trnfft.fft2(ComplexTensor(ts[0], ts[1])))

    def check(self, out):
        ref = torch.fft.fft2(torch.complex(self.xr, self.xi))
        return rel_err(torch.complex(out.real, out.imag), ref)

    def ref_sample(self, T, units):
        s_ = 1024
        g = torch.Generator().manual_seed(0)
        x = T.ComplexTensor(torch.randn(s_, s_, generator=g), torch.randn(s_, s_, generator=g))
        return (lambda: T.fft2(x)), 2 * c2c_flops(s_, s_), "one 1024x1024 fft2"

    ref_fixed_units = True

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        s = 1024
        rng = np.random.default_rng(0)
        xr = rng.standard_normal((s, s)).astype(np.float32)
        xi = rng.standard_normal((s, s)).astype(np.float32)
        t0 = time.perf_counter()
        O.fft2(xr, xi)
        return time.perf_counter() - t0, 2 * c2c_flops(s, s)


class LinearWL(Workload):
    """BASELINE configs[1](b): ComplexLinear 4096 -> 4096 on a 16384 x 4096 complex input."""

    metric = "ComplexLinear GFLOP/s (8*M*N*K complex flops)"

    def __init__(self, M=16384, N=4096, K=4096):
        self.M, self.N, self.K = M, N, K
        self.name = f"ComplexLinear {K}->{N} on a {M}x{K} complex fp32 input, 3xTF32 tcgen05 (configs[1]b)"
        self.work = 8.0 * M * N * K
        self.dom_bytes = None
        self.dominant = "k_gemm_tf32 (three launches of three TF32 segments each: the three-product complex form)"
        self.bound = "tensor"
        # tensor-core work actually issued: 3 real products x 3 TF32 segments x 2MNK
        self.tensor_flops = 9 * 2.0 * M * N * K

    def setup(self, dev, g):
        import trnfft_b200 as trnfft
        from trnfft_b200 import ComplexTensor
        from trnfft_b200.nn import ComplexLinear

        torch.manual_seed(77)
        self.layer = ComplexLinear(self.K, self.N, bias=True).to(dev)
        self.xr = torch.randn(self.M, self.K, device=dev, generator=g)
        self.xi = torch.randn(self.M, self.K, device=dev, generator=g)
        x = ComplexTensor(self.xr, self.xi)
        torch.set_grad_enabled(False)
        self.step = lambda: self.layer(x)
        self.launches = {"linear": self.step}
        self.launches_per_step = 6  # 3 split kernels (x: real, imaginary, sum; the weight split is cached) + 3 GEMMs
        self.inputs = [self.xr, self.xi]
        self.e2e_fn = lambda ts: (lambda y: [y.real, y.imag])(self.layer(ComplexTensor(ts[0], ts[1])))

    def ref_full_units(self):
        return self.M

    def ref_sample(self, T, units):
        import trnfft.nn as TN

        torch.manual_seed(77)
        layer = TN.ComplexLinear(self.K, self.N, bias=True)
        g = torch.Generator().manual_seed(0)
        x = T.ComplexTensor(torch.randn(units, self.K, generator=g), torch.randn(units, self.K, generator=g))

        def f():
            with torch.no_grad():
                return layer(x)

        return f, 8.0 * units * self.N * self.K, f"{units} of {self.M} rows"

    def check(self, out):
        w_r, w_i = self.layer.W_re.weight, self.layer.W_im.weight
        xr, xi = self.xr[:256].double(), self.xi[:256].double()
        ref_r = xr @ w_r.double().t() - xi @ w_i.double().t()
        ref_i = xr @ w_i.double().t() + xi @ w_r.double().t()
        return rel_err(torch.complex(out.real[:256].double(), out.imag[:256].double()), torch.complex(ref_r, ref_i))

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        rng = np.random.default_rng(0)
        r = max(16, rows // 4)
        xr = rng.standard_normal((r, self.K)).astype(np.float32)
        xi = rng.standard_normal((r, self.K)).astype(np.float32)
        wr = rng.uniform(-1, 1, (self.N, self.K)).astype(np.float32) / 64
        wi = rng.uniform(-1, 1, (self.N, self.K)).astype(np.float32) / 64
        t0 = time.perf_counter()
        O.complex_linear(xr, xi, wr, wi)
        return time.perf_counter() - t0, 8.0 * r * self.N * self.K


class SmallNGemm(SmallN):
    """configs[1](a) on the DFT-as-GEMM tensor-core path."""

    def __init__(self):
        super().__init__()
        self.name = "small-N batched C2C FFT as DFT-GEMM (tcgen05 3xTF32), N=64,128,256, batch=262144 (configs[1]a)"
        self.dominant = "k_gemm_tf32 DFT-GEMM, N=256"
        self.bound = "tensor"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft

        trnfft.set_small_n_algorithm("gemm")
        super().setup(dev, g)
        self.tensor_flops = sum(9 * 2.0 * self.batch * n * n for n in (256,))  # three-product form, 3xTF32


class RealRoundTrip(Workload):
    """BASELINE configs[3] real part: rfft then irfft of 4096 real rows of n = 4093."""

    metric = "batched real FFT GFLOP/s (2.5N*log2N per real transform), rfft+irfft round trip"

    def __init__(self, n=4093, batch=4096):
        self.n, self.batch = n, batch
        self.name = f"rfft + irfft round trip, real fp32 rows of N={n}, batch={batch} (configs[3])"
        self.work = 2 * 2.5 * n * math.log2(n) * batch
        self.dom_bytes = 4.0 * n * batch + 8.0 * (n // 2 + 1) * batch  # one direction: real in, bins out
        self.dominant = f"real-input Bluestein kernel (two rows per transform), N={n}"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft

        self.x = torch.randn(self.batch, self.n, device=dev, generator=g)
        self.step = lambda: trnfft.irfft(trnfft.rfft(self.x), n=self.n)
        self.launches = {"rfft": lambda: trnfft.rfft(self.x)}
        self.launches_per_step = 2
        self.inputs = [self.x]
        self.e2e_fn = lambda ts: [trnfft.irfft(trnfft.rfft(ts[0]), n=self.n)]

    def check(self, out):
        return rel_err(out, self.x)

    def ref_full_units(self):
        return self.batch

    def ref_sample(self, T, units):
        g = torch.Generator().manual_seed(0)
        x = torch.randn(units, self.n, generator=g)
        return (lambda: T.irfft(T.rfft(x), n=self.n)), 2 * 2.5 * self.n * math.log2(self.n) * units, \
            f"{units} of {self.batch} rows"

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        rng = np.random.default_rng(0)
        x = rng.standard_normal((max(1, rows // 32), self.n)).astype(np.float32)
        t0 = time.perf_counter()
        yr, yi = O.rfft(x)
        O.irfft(yr, yi, n=self.n)
        return time.perf_counter() - t0, 2 * 2.5 * self.n * math.log2(self.n) * x.shape[0]


class Istft(Workload):
    """Inverse of BASELINE configs[2]: istft of the 256 x 257 x 626 spectrogram back to 256 x 160000
    samples (n_fft 512, hop 256, periodic Hann, centred), one fused kernel."""

    metric = "iSTFT frames/s (256 x 626 frames, n_fft 512, hop 256, onesided)"
    unit = "frames/s"

    def __init__(self):
        self.B, self.L, self.nfft, self.hop = 256, 160000, 512, 256
        self.frames = 1 + (self.L + 2 * (self.nfft // 2) - self.nfft) // self.hop
        self.name = "iSTFT 256 x 626 frames -> 160000 samples, n_fft=512, hop=256, periodic Hann (configs[2] inverse)"
        self.work = float(self.B * self.frames)
        bins = self.nfft // 2 + 1
        self.dom_bytes = 8.0 * self.B * bins * self.frames + 4.0 * self.B * self.L
        self.dominant = "fused iSTFT kernel (n_fft=512)"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft

        self.win = torch.hann_window(self.nfft, device=dev)
        x = torch.randn(self.B, self.L, device=dev, generator=g)
        self.x = x
        S = trnfft.stft(x, self.nfft, self.hop, window=self.win)
        self.sr, self.si = S.real.contiguous(), S.imag.contiguous()
        from trnfft_b200 import ComplexTensor

        self.step = lambda: trnfft.istft(ComplexTensor(self.sr, self.si), self.nfft, self.hop, window=self.win,
                                         length=self.L)
        self.launches = {"istft": self.step}
        self.launches_per_step = 1
        self.inputs = [self.sr, self.si]
        self.e2e_fn = lambda ts: [trnfft.istft(ComplexTensor(ts[0], ts[1]), self.nfft, self.hop, window=self.win,
                                               length=self.L)]

    def check(self, out):
        return rel_err(out, self.x)

    def ref_full_units(self):
        return self.B

    def ref_sample(self, T, units):
        g = torch.Generator().manual_seed(0)
        x = torch.randn(units, self.L, generator=g)
        win = torch.hann_window(self.nfft)
        S = T.stft(x, self.nfft, self.hop, window=win)
        return ((lambda: T.istft(S, self.nfft, self.hop, window=win, length=self.L)), float(units * self.frames),
                f"{units} of {self.B} spectrograms")

    def cpu_sample(self, threads, rows):
        from oracle import trnfft_oracle as O

        rng = np.random.default_rng(0)
        w = rng.standard_normal((max(1, rows // 64), self.L)).astype(np.float32)
        sr, si = O.stft(w, self.nfft, self.hop)
        t0 = time.perf_counter()
        O.istft(sr, si, self.nfft, self.hop, length=self.L)
        return time.perf_counter() - t0, float(w.shape[0] * self.frames)


class MaskApply(Workload):
    """complex_mask_apply on the configs[2] spectrogram shape (256 x 257 x 626), one fused kernel
    (the mask step between STFT and iSTFT)."""

    metric = "complex mask apply, complex elements/s (256 x 257 x 626)"
    unit = "elements/s"

    def __init__(self):
        self.shape = (256, 257, 626)
        self.count = 256 * 257 * 626
        self.name = "complex_mask_apply, mask and spectrogram 256 x 257 x 626 planar fp32 (configs[2] shape)"
        self.work = float(self.count)
        self.dom_bytes = 24.0 * self.count
        self.dominant = "fused complex multiply kernel (float4)"

    def setup(self, dev, g):
        from trnfft_b200 import ComplexTensor
        from trnfft_b200.nki.dispatch import complex_mask_apply

        self.m = ComplexTensor(torch.randn(*self.shape, device=dev, generator=g),
                               torch.randn(*self.shape, device=dev, generator=g))
        self.s = ComplexTensor(torch.randn(*self.shape, device=dev, generator=g),
                               torch.randn(*self.shape, device=dev, generator=g))
        self.step = lambda: complex_mask_apply(self.m, self.s)
        self.launches = {"mask": self.step}
        self.launches_per_step = 1
        self.inputs = [self.m.real, self.m.imag, self.s.real, self.s.imag]
        self.e2e_fn = lambda ts: (lambda y: [y.real, y.imag])(
            complex_mask_apply(ComplexTensor(ts[0], ts[1]), ComplexTensor(ts[2], ts[3])))

    def check(self, out):
        want = torch.complex(self.m.real, self.m.imag) * torch.complex(self.s.real, self.s.imag)
        return rel_err(torch.complex(out.real, out.imag), want)

    def ref_full_units(self):
        return self.shape[0]

    def ref_sample(self, T, units):
        from trnfft.nki.dispatch import complex_mask_apply as ref_mask

        g = torch.Generator().manual_seed(0)
        sh = (units,) + self.shape[1:]
        m = T.ComplexTensor(torch.randn(*sh, generator=g), torch.randn(*sh, generator=g))
        sp = T.ComplexTensor(torch.randn(*sh, generator=g), torch.randn(*sh, generator=g))
        return (lambda: ref_mask(m, sp)), float(units * self.shape[1] * self.shape[2]), f"{units} of {self.shape[0]} rows"

    def cpu_sample(self, threads, rows):
        rng = np.random.default_rng(0)
        r = max(1, rows // 16)
        sh = (r,) + self.shape[1:]
        a, b, c, d = (rng.standard_normal(sh).astype(np.float32) for _ in range(4))
        t0 = time.perf_counter()
        _ = (a * c - b * d, a * d + b * c)
        return time.perf_counter() - t0, float(np.prod(sh))


class C2CDouble(C2CRoundTrip):
    """precision="double": the fp64 kernels on a float32 batch (widened and rounded back on the
    device), fft + ifft round trip."""

    dtype = "f64"

    def __init__(self, n, batch, tag):
        super().__init__(n, batch, tag)
        self.name = f"batched C2C FFT+IFFT round trip in precision='double' (fp64 kernels), N={n}, batch={batch} ({tag})"
        self.dominant = f"fp64 C2C kernels, N={n}"

    def setup(self, dev, g):
        import trnfft_b200 as trnfft

        trnfft.set_precision("double")
        super().setup(dev, g)

    def ref_sample(self, T, units):
        T.set_precision("double")
        return super().ref_sample(T, units)


WORKLOADS = {
    "linear": LinearWL,
    "smalln_gemm": SmallNGemm,
    "c2c1024": lambda: C2CRoundTrip(N, BATCH, "BASELINE configs[0]"),
    "smalln": SmallN,
    "stft": Stft,
    "bluestein4093": lambda: C2CRoundTrip(4093, 4096, "BASELINE configs[3]"),
    "bluestein1000": lambda: C2CRoundTrip(1000, 4096, "BASELINE configs[3]"),
    "bluestein6000": lambda: C2CRoundTrip(6000, 4096, "BASELINE configs[3]"),
    "large": Large,
    "fft2": Fft2,
    "rows8192": lambda: C2CRoundTrip(8192, 8192, "one-pass rows of 8192 points (k_c2c_big)"),
    "rows16384": lambda: C2CRoundTrip(16384, 4096, "one-pass rows of 16384 points (k_c2c_big), the fft2 / four-step row pass"),
    "rfft4093": RealRoundTrip,
    "istft": Istft,
    "mask": MaskApply,
    "double4093": lambda: C2CDouble(4093, 4096, "BASELINE configs[3], precision double"),
    "double1024": lambda: C2CDouble(1024, 8192, "BASELINE configs[0], precision double"),
}


def make_workload(args):
    """Build the workload; --size shrinks the size-parametrised ones for profiling runs
    (large: log2 N, fft2: side, linear: M rows)."""
    if args.size:
        if args.workload == "large":
            return Large(args.size)
        if args.workload == "fft2":
            return Fft2(args.size)
        if args.workload == "linear":
            return LinearWL(M=args.size)
    return WORKLOADS[args.workload]()


def cpu_rate(wl, threads, budget_s, rows=256):
    wl.cpu_sample(threads, max(8, rows // 8))  # warm-up
    t_total, w_total, reps = 0.0, 0.0, 0
    while t_total < budget_s:
        t, w = wl.cpu_sample(threads, rows)
        t_total += t
        w_total += w
        reps += 1
        if t > budget_s:
            break
    return w_total / t_total, t_total, reps


def scale_value(v, unit):
    return v / 1e9 if unit == UNIT else v


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def import_reference():
    """The unmodified reference package installed in baseline/_ref, on its own CPU
    ('pytorch') backend, or None when it is not installed."""
    if not os.path.isdir(os.path.join(REF_DIR, "trnfft")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import trnfft as T

    T.set_backend("pytorch")
    T.set_precision("fast")
    return T


def calibrate_units(wl, T, target_s):
    """Largest sample (rows / waveforms, growing 4x up to the full workload) whose reference
    step stays within target_s.  The reference's per-call cost is mostly a fixed Python loop
    over butterfly stages, so larger samples are much cheaper per row."""
    if getattr(wl, "ref_fixed_units", False):
        return 1
    full = wl.ref_full_units()
    units, best = 4, None
    while True:
        fn, _, _ = wl.ref_sample(T, units)
        t0 = time.perf_counter()
        fn()
        dt = time.perf_counter() - t0
        if dt > target_s and best is not None:
            return best
        best = units
        if dt > target_s or units >= full:
            return best
        units = min(full, units * 4)


def time_reference(wl, T, steps, warmup, target_s=5.0):
    """Time `steps` reference steps (each one bounded sample of the workload) with
    perf_counter; returns (rate per second, mean s per step, sample description)."""
    units = calibrate_units(wl, T, target_s)
    fn, work, desc = wl.ref_sample(T, units)
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    mean = sum(ts) / len(ts)
    return work / mean, mean, desc


def cpu_baseline(wl, budget_s):
    """Reported CPU baseline: the reference itself (baseline/_ref) when installed, plus the
    NumPy port of its algorithm (oracle/trnfft_oracle.py) as a second entry."""
    threads = os.cpu_count() or 1
    out = {}
    T = import_reference()
    if T is not None:
        torch.set_num_threads(threads)
        steps = 3
        rate, mean, desc = time_reference(wl, T, steps, 1, target_s=min(2.0, budget_s / (steps + 3)))
        out = {"value": round(scale_value(rate, wl.unit), 4), "unit": wl.unit, "cores": threads,
               "kind": "reference",
               "sample": f"trnfft (baseline/_ref, backend 'pytorch', {threads} torch threads): {desc} per step, "
                         f"{steps} steps of {mean:.2f} s"}
    rate, t, reps = cpu_rate(wl, threads, budget_s / 2 if T is not None else budget_s)
    port = {"value": round(scale_value(rate, wl.unit), 4), "unit": wl.unit, "cores": threads, "kind": "port",
            "sample": f"oracle/trnfft_oracle.py ({wl.name}), {reps} bounded sample(s) in {t:.1f} s "
                      f"on {threads} host threads"}
    if not out:
        return port, None
    return out, port


def run_reference(args, world, rank):
    if rank != 0:
        return
    wl = make_workload(args)
    threads = os.cpu_count() or 1
    T = import_reference()
    if T is not None:
        torch.set_num_threads(threads)
        rate, mean, desc = time_reference(wl, T, args.steps, args.warmup)
        kind = "reference"
        sample = (f"trnfft {getattr(T, '__version__', '')} from baseline/_ref, backend 'pytorch', "
                  f"{threads} torch threads; each step = {desc}")
    else:
        # the reference is not installed: its algorithm restated in NumPy (oracle port)
        units = 256
        for _ in range(args.warmup):
            wl.cpu_sample(threads, 64)
        ts, works = [], []
        for _ in range(args.steps):
            t, w = wl.cpu_sample(threads, units)
            ts.append(t)
            works.append(w)
        rate, mean = sum(works) / sum(ts), sum(ts) / len(ts)
        kind = "port"
        sample = f"oracle/trnfft_oracle.py (the reference's algorithm in NumPy), {units} rows per step"
    value = round(scale_value(rate, wl.unit), 4)
    out = {
        "impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 * mean, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name + f"; reference CPU path, each step = {sample}",
                   "parallelism": f"{threads} host threads"},
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timing": "time.perf_counter around each step; ms_per_step is the measured mean step time",
    }
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------


def run_ours(args, world, rank, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    wl = make_workload(args)
    wl.setup(dev, g)
    flush = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    flush_out = torch.empty(1, dtype=torch.float32, device=dev)

    def flush_l2():
        # read-only sweep of a buffer twice the L2 size: evicts every line
        # (dirty lines are written back here, not inside the timed kernel)
        torch.sum(flush, dim=0, keepdim=True, out=flush_out)

    for _ in range(max(args.warmup, 3)):
        wl.step()
    torch.cuda.synchronize()

    # The step (and each launch alone) is captured once as a CUDA graph, so the
    # device timing below contains no host dispatch gaps.  Before every timed
    # replay the L2 is flushed; the flush is enqueued first so the GPU is busy
    # while the events and the replay are queued behind it.
    st = torch.cuda.current_stream(dev)

    class _Direct:  # steps with collectives run eagerly (no graph capture of NCCL)
        def __init__(self, fn):
            self.fn = fn
            self.out = None

        def replay(self):
            self.out = self.fn()

    if getattr(wl, "no_graph", False):
        g_step = _Direct(wl.step)
        g_launch = {k: _Direct(fn) for k, fn in wl.launches.items()} or {"step": _Direct(wl.step)}
        g_step.replay()
        y_step = g_step.out
    else:
        g_step = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step):
            y_step = wl.step()
        g_launch = {}
        for k, fn in wl.launches.items():
            gg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gg):
                fn()
            g_launch[k] = gg
    g_step.replay()
    for gg in g_launch.values():
        gg.replay()
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
        for gg in g_launch.values():
            launch_ms.append(timed(gg))

    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        step_ms = [timed(g_step) for _ in range(args.steps)]
        torch.cuda.synchronize()
    barrier(world)
    ms = allreduce_max(sum(step_ms) / len(step_ms), world)
    strong = getattr(wl, "scaling", "weak") == "strong"
    value = (1 if strong else world) * wl.work / (ms / 1e3)
    err = wl.check(y_step)
    del y_step

    # end to end through the public API: pinned host inputs -> device -> step -> pinned host results
    del g_step, g_launch
    host_in = [t.cpu().pin_memory() for t in wl.inputs]
    dev_in = [torch.empty_like(t) for t in wl.inputs]
    outs = wl.e2e_fn(dev_in)
    host_out = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
    h2d_bytes = sum(t.numel() * t.element_size() for t in host_in)
    d2h_bytes = sum(t.numel() * t.element_size() for t in host_out)

    if getattr(wl, "e2e_rows", True):
        # batched transforms: row chunks stream through the GPU with the upload of one chunk,
        # the transforms of the previous one and the download of the one before overlapped
        # (trnfft_b200.streaming.map_rows; PCIe copies both ways at once)
        from trnfft_b200.streaming import map_rows

        def e2e_step():
            map_rows(wl.e2e_fn, host_in, host_outputs=host_out)
    else:
        def e2e_step():
            for d, h in zip(dev_in, host_in):
                d.copy_(h, non_blocking=True)
            for h, o in zip(host_out, wl.e2e_fn(dev_in)):
                h.copy_(o, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = []
    for _ in range(max(3, min(args.steps, 10))):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        e2e_step()
        e1.record(st)
        e1.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    barrier(world)
    e2e_max = allreduce_max(sum(e2e_ms) / len(e2e_ms), world)
    e2e_value = (1 if strong else world) * wl.work / (e2e_max / 1e3)

    extras = {}
    if args.extras and args.workload == "c2c1024" and not args.size:
        del dev_in, host_in, host_out, outs
        wl.release()
        torch.cuda.empty_cache()
        if world > 1:
            extras["multi_gpu_check_rel_l2"] = multi_gpu_check(world, rank, dev)
        extras["large_four_step"] = large_extra(world, rank, dev)
        extras["fft2_16384_sharded"] = fft2_extra(world, rank, dev)

    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    avg_launch = sum(launch_ms) / len(launch_ms)
    # the profiled DRAM traffic describes the default single-GPU configuration only
    traffic = profiled_traffic(args.workload) if (world == 1 and not args.size) else None
    if getattr(wl, "bound", "hbm") == "tensor":
        tf = getattr(wl, "tensor_flops", None) or 3.0 * wl.work  # 3xTF32: three TF32 products per flop
        achieved_t = tf / (avg_launch / 1e3) / 1e12
        tpeak, tkind = measured_tensor_peak()
        roof = {"bound": "tensor", "achieved": round(achieved_t, 2), "peak": tpeak, "unit": "TFLOP/s",
                "frac": round(achieved_t / tpeak, 4), "peak_source": tkind, "traffic": traffic,
                "kernel": wl.dominant, "tensor_flops_per_launch": tf, "avg_launch_ms": round(avg_launch, 5)}
    achieved = (wl.dom_bytes or 1.0) / (avg_launch / 1e3) / 1e9
    out = {
        "metric": wl.metric, "value": round(scale_value(value, wl.unit), 3), "unit": wl.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": getattr(wl, "scaling", "weak"), "vs_baseline": None,
        "dtype": getattr(wl, "dtype", "f32"),
        "data": "synthetic",
        "config": {"workload": wl.name,
                   "parallelism": ("1 GPU" if world == 1 else
                                   (f"four-step over {world} GPUs" if strong else f"batch-sharded x{world}")),
                   "l2": "flushed before every timed step (256 MiB read sweep)"},
        "roofline": roof if getattr(wl, "bound", "hbm") == "tensor" else
                    {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": traffic, "kernel": wl.dominant,
                     "algorithmic_bytes_per_launch": wl.dom_bytes, "avg_launch_ms": round(avg_launch, 5),
                     **({"min_bytes_per_launch": wl.min_bytes,
                         "frac_of_min_bytes": round(wl.min_bytes / (avg_launch / 1e3) / 1e9 / peak, 4)}
                        if getattr(wl, "min_bytes", None) else {})},
        "e2e": {"value": round(scale_value(e2e_value, wl.unit), 3), "unit": wl.unit,
                "ms_per_step": round(e2e_max, 4),
                "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk.summary(),
        "check_rel_l2": err, "parity_ok": bool(err < 1e-5),
        "timing": "CUDA events around CUDA-graph replays of the step; L2 flushed before each",
    }
    out.update(extras)
    if world == 1 and args.cpu_budget > 0:
        cb, port = cpu_baseline(wl, args.cpu_budget)
        out["cpu_baseline"] = cb
        if port is not None:
            out["cpu_baseline_port"] = port
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# Extras printed beside the headline: parity of the multi-GPU exchanges against
# the single-GPU transforms, and the four-step 2^30 at this GPU count against
# the same algorithm on one GPU.
# ---------------------------------------------------------------------------


def _sum_sq(t):
    return float((t.double() ** 2).sum())


def multi_gpu_check(world, rank, dev):
    """rel-L2 of fft_distributed (2^24; column-block input with transposed output, contiguous
    input with natural output, and the NCCL exchange) and fft2_distributed (4096^2, both output
    layouts) against trnfft.fft / trnfft.fft2 of the whole input on one GPU."""
    import trnfft_b200 as trnfft
    from trnfft_b200 import ComplexTensor
    from trnfft_b200 import distributed as D

    out = {}
    g = torch.Generator(device=dev).manual_seed(4242)  # same input on every rank
    n = 1 << 24
    xr = torch.randn(n, device=dev, generator=g)
    xi = torch.randn(n, device=dev, generator=g)
    X = trnfft.fft(ComplexTensor(xr.reshape(1, n), xi.reshape(1, n)))
    Xr, Xi = X.real.reshape(-1), X.imag.reshape(-1)
    N1, N2 = D._split_n(n)
    r1 = N1 // world
    c2 = N2 // world
    # transposed output: Z[k1 local][k2] = X[k1 + N1 k2], k1 in this rank's block
    want_t = (Xr.reshape(N2, N1)[:, rank * r1:(rank + 1) * r1].t(), Xi.reshape(N2, N1)[:, rank * r1:(rank + 1) * r1].t())
    want_n = (Xr[rank * n // world:(rank + 1) * n // world], Xi[rank * n // world:(rank + 1) * n // world])
    cases = {
        "fft_distributed_2^24_columns_in_transposed": (
            lambda: D.fft_distributed(ComplexTensor(*D.column_block(xr, xi, n, world, rank)), n,
                                      natural_order=False, columns_in=True), want_t),
        "fft_distributed_2^24_natural": (
            lambda: D.fft_distributed(ComplexTensor(xr[rank * n // world:(rank + 1) * n // world],
                                                    xi[rank * n // world:(rank + 1) * n // world]), n), want_n),
        "fft_distributed_2^24_nccl_exchange": (
            lambda: D.fft_distributed(ComplexTensor(xr[rank * n // world:(rank + 1) * n // world],
                                                    xi[rank * n // world:(rank + 1) * n // world]), n,
                                      exchange="nccl"), want_n),
    }
    s_ = 4096
    fr = torch.randn(s_, s_, device=dev, generator=g)
    fi = torch.randn(s_, s_, device=dev, generator=g)
    F = trnfft.fft2(ComplexTensor(fr, fi))
    h = s_ // world
    rows = slice(rank * h, (rank + 1) * h)
    cols = slice(rank * (s_ // world), (rank + 1) * (s_ // world))
    cases["fft2_distributed_4096_natural"] = (
        lambda: D.fft2_distributed(ComplexTensor(fr[rows], fi[rows])), (F.real[rows], F.imag[rows]))
    cases["fft2_distributed_4096_column_blocks"] = (
        lambda: D.fft2_distributed(ComplexTensor(fr[rows], fi[rows]), natural_order=False),
        (F.real[:, cols], F.imag[:, cols]))
    for name, (fn, (wr, wi)) in cases.items():
        y = fn()
        torch.cuda.synchronize()
        num = _sum_sq(y.real.reshape(wr.shape) - wr) + _sum_sq(y.imag.reshape(wi.shape) - wi)
        den = _sum_sq(wr) + _sum_sq(wi)
        t = torch.tensor([num, den], dtype=torch.float64, device=dev)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(t)
        out[name] = float((t[0] / t[1]).sqrt())
    D.clear_exchanges()
    return out


def large_extra(world, rank, dev, steps=10, warmup=3, logn=30):
    """The four-step N=2^logn transform on `world` GPUs (max over ranks of the CUDA-event
    time) and, on rank 0, the same algorithm on one GPU."""
    from trnfft_b200 import ComplexTensor
    from trnfft_b200 import distributed as D

    n = 1 << logn
    N1, N2 = D._split_n(n)
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    st = torch.cuda.current_stream(dev)

    def time_fn(fn, collective):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if collective:
            barrier(world)
        ts = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sum(ts) / len(ts)

    res = {"n": f"2^{logn}", "split": f"{N1} x {N2}", "steps": steps}
    if world > 1:
        xr = torch.randn(N1, N2 // world, device=dev, generator=g)
        xi = torch.randn(N1, N2 // world, device=dev, generator=g)
        x = ComplexTensor(xr, xi)
        ms = time_fn(lambda: D.fft_distributed(x, n, natural_order=False, columns_in=True), True)
        res["ms"] = round(allreduce_max(ms, world), 4)
        del x, xr, xi
        D.clear_exchanges()
        torch.cuda.empty_cache()
    barrier(world)
    if rank == 0:
        xr = torch.randn(N1, N2, device=dev, generator=g)
        xi = torch.randn(N1, N2, device=dev, generator=g)
        x = ComplexTensor(xr, xi)
        ms1 = time_fn(lambda: D.fft_four_step_local(x, n), False)  # rank 0 alone: no collective
        res["ms_1gpu"] = round(ms1, 4)
        if world == 1:
            res["ms"] = res["ms_1gpu"]
        res["speedup_vs_1gpu"] = round(ms1 / res["ms"], 3)
        res["gflops"] = round(c2c_flops(n, 1) / (res["ms"] / 1e3) / 1e9, 1)
        del x, xr, xi
        torch.cuda.empty_cache()
    barrier(world)
    return res


def fft2_extra(world, rank, dev, side=16384, steps=10, warmup=3):
    """fft2 of a side x side field sharded by rows over `world` GPUs (fft2_distributed, natural
    row layout; max over ranks of the CUDA-event time) and, on rank 0, trnfft.fft2 of the whole
    field on one GPU."""
    import trnfft_b200 as trnfft
    from trnfft_b200 import ComplexTensor
    from trnfft_b200 import distributed as D

    st = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(7 + rank)

    def time_fn(fn, collective):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if collective:
            barrier(world)
        ts = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sum(ts) / len(ts)

    res = {"side": side, "steps": steps}
    if world > 1:
        hr = side // world
        x = ComplexTensor(torch.randn(hr, side, device=dev, generator=g), torch.randn(hr, side, device=dev, generator=g))
        res["ms"] = round(allreduce_max(time_fn(lambda: D.fft2_distributed(x), True), world), 4)
        res["ms_unchunked"] = round(allreduce_max(time_fn(lambda: D.fft2_distributed(x, chunks=1), True), world), 4)
        del x
        D.clear_exchanges()
        torch.cuda.empty_cache()
    barrier(world)
    if rank == 0:
        x = ComplexTensor(torch.randn(side, side, device=dev, generator=g),
                          torch.randn(side, side, device=dev, generator=g))
        res["ms_1gpu"] = round(time_fn(lambda: trnfft.fft2(x), False), 4)
        if world == 1:
            res["ms"] = res["ms_1gpu"]
        res["speedup_vs_1gpu"] = round(res["ms_1gpu"] / res["ms"], 3)
        res["gflops"] = round(2 * c2c_flops(side, side) / (res["ms"] / 1e3) / 1e9, 1)
        del x
        torch.cuda.empty_cache()
    barrier(world)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2c1024")
    ap.add_argument("--size", type=int, default=0, help="smaller case for profiling (large/fft2/linear)")
    ap.add_argument("--no-extras", dest="extras", action="store_false",
                    help="skip the multi-GPU parity check and the four-step 2^30 line of the default run")
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
