"""1-D transform along the last dimension (same entry point as trnfft/fft_core.py:22-50).

``fft_core`` picks the plan (power of two -> Stockham or multi-pass kernels,
any other n -> fused Bluestein kernel) and runs it through the C ABI.  The
reference's device ladder (fft_core.py:1063-1150: DFT-as-GEMM for n <= 256,
mixed-radix / radix-8 / radix-4 Stockham, radix-2 butterflies) collapses into
those plans; every stage of a transform stays on chip.
"""

from __future__ import annotations

import torch

from . import _ops
from ._device import place
from .complex import ComplexTensor
from .plan import FFTPlan, create_plan
from .precision import _resolve


def fft_core(
    x: ComplexTensor,
    inverse: bool = False,
    plan: FFTPlan | None = None,
    precision: str | None = None,
) -> ComplexTensor:
    """Compute the 1-D FFT of ``x`` along its last dimension.

    ``plan`` is created (and cached) when None.  ``precision`` overrides the
    global mode for this call (validated like the reference's).
    """
    _resolve(precision)
    n = x.shape[-1]
    if n == 1:
        return x.clone()
    if plan is None:
        plan = create_plan(n, inverse=inverse)
    if plan.n != n:
        raise ValueError(f"plan is for n={plan.n}, input has n={n}")
    (xr, xi), restore = place(x.real, x.imag, allow_f64=True)
    if n == 0 or xr.numel() == 0:
        return ComplexTensor(restore(xr.clone()), restore(xi.clone()))
    yr, yi = _ops.c2c(xr, xi, bool(inverse), precision=_resolve(precision))
    return ComplexTensor(restore(yr), restore(yi))


def rfft_core(x: torch.Tensor) -> ComplexTensor:
    """Real-input transform along the last dimension, n//2+1 bins."""
    (xd,), restore = place(x, allow_f64=True)
    yr, yi = _ops.r2c(xd)
    return ComplexTensor(restore(yr), restore(yi))


def irfft_core(x: ComplexTensor, n: int) -> torch.Tensor:
    """Real result of the inverse transform of the Hermitian extension of ``x``."""
    (xr, xi), restore = place(x.real, x.imag, allow_f64=True)
    return restore(_ops.c2r(xr, xi, n))
