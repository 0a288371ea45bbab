"""Backend switch and multi-device dispatch (same names as trnfft/nki/__init__.py).

On B200 there is one backend: the CUDA kernels of libtrnfft_b200.so.  The
module keeps the reference's package path so ``from trnfft.nki import
set_backend, multi_core_fft`` style imports keep working.
"""

from .dispatch import (
    HAS_NKI,
    complex_gemm,
    complex_linear,
    complex_mask_apply,
    get_backend,
    set_backend,
)
from .multicore import get_multicore, multi_core_fft, set_multicore

butterfly_stage_kernel = None

__all__ = [
    "HAS_NKI",
    "set_backend",
    "get_backend",
    "complex_gemm",
    "complex_mask_apply",
    "complex_linear",
    "butterfly_stage_kernel",
    "set_multicore",
    "get_multicore",
    "multi_core_fft",
]
