"""trnfft_b200 — B200-native (sm_100a) implementation of trnfft's FFT hot path.

Drop-in for ``import trnfft``: the same public names, signatures and
semantics (trnfft/__init__.py:13-68), with every transform running on
hand-written CUDA kernels through the C ABI in include/trnfft_b200.h::

    import trnfft_b200 as trnfft
    X = trnfft.fft(x)
"""

__version__ = "0.1.0"

from .api import (
    fft,
    fft2,
    fftn,
    hfft,
    ifft,
    ifftn,
    ihfft,
    irfft,
    irfft2,
    irfftn,
    istft,
    rfft,
    rfft2,
    rfftn,
    stft,
)
from .complex import ComplexTensor, complex_matmul
from .nki import HAS_NKI, get_backend, set_backend
from .plan import FFTPlan, clear_plan_cache, create_plan, get_small_n_algorithm, set_small_n_algorithm
from .precision import get_precision, set_precision


def set_ozaki_product_precision_verified(verified: bool) -> None:
    """Accepted for API compatibility (trnfft/fft_core.py:200-218); Ozaki modes run fp32 kernels."""
    return None


__all__ = [
    "fft", "ifft", "rfft", "hfft", "ihfft", "irfft", "fft2", "fftn", "ifftn", "rfft2", "irfft2",
    "rfftn", "irfftn", "stft", "istft",
    "ComplexTensor", "complex_matmul",
    "create_plan", "clear_plan_cache", "FFTPlan", "set_small_n_algorithm", "get_small_n_algorithm",
    "HAS_NKI", "set_backend", "get_backend",
    "set_precision", "set_ozaki_product_precision_verified", "get_precision",
]
