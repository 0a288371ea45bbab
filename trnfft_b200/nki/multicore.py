"""Multi-device dispatch (same API as trnfft/nki/multicore.py).

Two partition strategies, as in the reference:

1. Batch split (``_batch_split_fft``, trnfft/nki/multicore.py:222-260): the
   batch is cut into contiguous shards; shard i runs on visible CUDA device
   i mod device_count (all on one device when only one is visible).  No
   communication.  For one process per GPU, see ``trnfft_b200.distributed``.
2. Single-transform four-step (``_stage_parallel_fft``, multicore.py:151-219):
   N = n1*n2 with n1 the largest divisor <= sqrt(N), column transforms,
   twiddle exp(sign*2*pi*i*l*k1/N), row transforms, column-major flatten.  The
   twiddle runs on the device (the reference computes it on the host).

Off by default; ``TRNFFT_MULTICORE=1`` or ``set_multicore(True)`` enables it.
"""

from __future__ import annotations

import math
import os

import torch

from ..complex import ComplexTensor

HAS_TORCH_NEURONX = False
HAS_COLLECTIVES = torch.distributed.is_available()

_use_multicore = os.environ.get("TRNFFT_MULTICORE", "0") == "1"
_num_cores: int = 0


def set_multicore(enabled: bool, num_cores: int = 0) -> None:
    """Enable or disable multi-device dispatch; ``num_cores=0`` means all visible devices."""
    global _use_multicore, _num_cores
    _use_multicore = enabled
    _num_cores = num_cores


def get_multicore() -> bool:
    return _use_multicore


def multi_core_fft(x: ComplexTensor, inverse: bool = False) -> ComplexTensor:
    """Batch-split (batch > 1) or four-step (single transform) FFT when enabled."""
    from ..fft_core import fft_core

    if not _use_multicore:
        return fft_core(x, inverse=inverse)
    batch_size = x.real.shape[0] if x.real.dim() > 1 else 1
    if batch_size > 1:
        return _batch_split_fft(x, inverse, _resolve_num_cores(batch_size))
    n = x.shape[-1]
    try:
        n1, n2 = _factorize(n)
    except ValueError as exc:
        raise NotImplementedError(
            f"N={n} is prime — single-transform multi-core requires composite N. "
            "Use set_multicore(False) and trnfft.fft() for prime N, or ensure "
            "N is composite (e.g. a power of 2)."
        ) from exc
    return _stage_parallel_fft(x, _resolve_num_cores(min(n1, n2)), inverse)


def _visible_devices() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _resolve_num_cores(batch_size: int) -> int:
    """Requested shard count, else the visible CUDA device count, capped by the batch.

    With no CUDA device visible (host-only logic) it falls back to min(2, batch)
    like the reference's CPU default (multicore.py:118-131).
    """
    if _num_cores > 0:
        return min(_num_cores, batch_size)
    nd = _visible_devices()
    if nd > 0:
        return min(nd, batch_size)
    return min(2, batch_size)


def _factorize(n: int) -> tuple[int, int]:
    """(n1, n2) with n1*n2 == n and n1 the largest divisor <= sqrt(n) (multicore.py:134-148)."""
    n1 = math.isqrt(n)
    while n1 > 1 and n % n1 != 0:
        n1 -= 1
    if n1 <= 1:
        raise ValueError(f"n={n} has no non-trivial divisors (prime); row-column FFT not applicable")
    return n1, n // n1


def _stage_parallel_fft(x: ComplexTensor, num_cores: int, inverse: bool) -> ComplexTensor:
    """Four-step single transform in natural order (multicore.py:151-219)."""
    from .._device import place

    n = x.shape[-1]
    n1, n2 = _factorize(n)
    sign = 1.0 if inverse else -1.0
    (xr, xi), restore = place(x.real.reshape(n), x.imag.reshape(n))
    if n & (n - 1) == 0 and n > 1024 and n1 <= (1 << 20) and xr.dtype == torch.float32:
        # powers of two: the column transforms read the [n1][n2] view in place and multiply by
        # the twiddle W_N^{l k1} in their last pass (trnfft_exec_c2c_axis_tw), so neither the
        # transposed copy nor N-sized twiddle tables are built
        from .. import _lib

        yr = torch.empty(n1, n2, dtype=torch.float32, device=xr.device)
        yi = torch.empty_like(yr)
        plan = _lib.device_plan(n1, xr.device)
        twp = _lib.device_plan(n, xr.device)
        _lib.call("trnfft_exec_c2c_axis_tw", plan.handle, twp.handle, _lib.ptr(xr), _lib.ptr(xi), _lib.ptr(yr),
                  _lib.ptr(yi), 1, n2, 0, 0, int(bool(inverse)), 0, _lib.stream_ptr(xr.device))
        row = _batch_split_fft(ComplexTensor(yr, yi), inverse=inverse, num_cores=num_cores)
        return ComplexTensor(restore(row.real.T.contiguous().reshape(n)), restore(row.imag.T.contiguous().reshape(n)))
    col = _batch_split_fft(
        ComplexTensor(xr.reshape(n1, n2).T.contiguous(), xi.reshape(n1, n2).T.contiguous()),
        inverse=inverse, num_cores=num_cores,
    )
    yr, yi = col.real.T, col.imag.T  # (n1, n2): Y[k1, l]
    # twiddle exp(sign*2*pi*i*l*k1/N) with the exponent l*k1 reduced mod N in integers
    k1 = torch.arange(n1, device=xr.device, dtype=torch.int64).unsqueeze(1)
    l = torch.arange(n2, device=xr.device, dtype=torch.int64).unsqueeze(0)
    e = (l * k1) % n
    ang = (sign * 2.0 * math.pi / n) * e.to(torch.float64)
    tr = torch.cos(ang).to(torch.float32)
    ti = torch.sin(ang).to(torch.float32)
    zr = yr * tr - yi * ti
    zi = yr * ti + yi * tr
    row = _batch_split_fft(ComplexTensor(zr.contiguous(), zi.contiguous()), inverse=inverse, num_cores=num_cores)
    out_r = row.real.T.contiguous().reshape(n)
    out_i = row.imag.T.contiguous().reshape(n)
    return ComplexTensor(restore(out_r), restore(out_i))


def _batch_split_fft(x: ComplexTensor, inverse: bool, num_cores: int) -> ComplexTensor:
    """Cut the batch into ``num_cores`` shards and transform each (multicore.py:222-260)."""
    from ..fft_core import fft_core

    real, imag = x.real, x.imag
    batch = real.shape[0]
    actual = min(num_cores, batch)
    if actual <= 1:
        return fft_core(x, inverse=inverse)
    nd = _visible_devices()
    home = real.device
    results = []
    for i, (r, m) in enumerate(zip(real.chunk(actual, dim=0), imag.chunk(actual, dim=0), strict=True)):
        if nd > 1:
            dev = torch.device("cuda", i % nd)
            r, m = r.to(dev, non_blocking=True), m.to(dev, non_blocking=True)
        results.append(fft_core(ComplexTensor(r, m), inverse=inverse))
    out_r = torch.cat([o.real.to(home) for o in results], dim=0)
    out_i = torch.cat([o.imag.to(home) for o in results], dim=0)
    return ComplexTensor(out_r, out_i)
