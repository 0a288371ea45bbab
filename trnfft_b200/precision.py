"""Precision-mode selection (same API as trnfft/precision.py:70-94).

``"fast"`` (default) and ``"double"`` are the modes that matter on B200:

* ``"fast"``: float32 kernels.  Power-of-two sizes run the Stockham kernels
  (about 2e-7 relative L2 error against an fp64 FFT).  Bluestein sizes use a
  chirp whose angle pi*(k^2 mod 2n)/n is reduced exactly in integers before
  it is rounded, so the float32 pipeline reaches about 4e-7 instead of the
  reference's 1e-4 (its float32 angle pi*k*k/n, trnfft/fft_core.py:1316-1320,
  loses ~1e-3 rad at k ~ 4000).
* ``"double"``: every transform runs the fp64 kernels (trnfft_exec_c2c_f64:
  twiddles, chirp, filter spectrum and butterflies in float64; float32 data is
  widened on the device and the result rounded back).  The reference promotes
  Bluestein to float64 (fft_core.py:1306-1309) and runs power-of-two sizes up
  to 1024 as an fp64 DFT (fft_core.py:1108-1110); here every size gets fp64,
  which is at least as accurate.  float64 tensors always take the fp64
  kernels and come back float64, as with the reference's torch backend.

The remaining modes (``"kahan"``, ``"bf16"``, ``"bf16_refined"``, ``"ozaki"``,
``"ozaki_hq"``) are Trainium PSUM-precision experiments of the reference
(fft_core.py:169-545).  They are accepted so that code which sets them keeps
working, and they run the float32 kernels.
"""

from __future__ import annotations

_VALID = ("fast", "kahan", "double", "bf16", "bf16_refined", "ozaki", "ozaki_hq")

_precision: str = "fast"


def set_precision(mode: str) -> None:
    """Set the global precision mode."""
    global _precision
    if mode not in _VALID:
        raise ValueError(f"precision mode must be one of {_VALID}; got {mode!r}")
    _precision = mode


def get_precision() -> str:
    """Return the current global precision mode."""
    return _precision


def _resolve(precision) -> str:
    """Resolve an optional per-call precision override against the global."""
    if precision is None:
        return _precision
    if precision not in _VALID:
        raise ValueError(f"precision must be one of {_VALID} or None; got {precision!r}")
    return precision
