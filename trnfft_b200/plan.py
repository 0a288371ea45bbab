"""FFT plans: algorithm selection plus cached device tables.

``FFTPlan``/``create_plan``/``clear_plan_cache`` keep the reference's
signatures and semantics (trnfft/plan.py:14-50): plans are frozen, cached by
(n, inverse), power-of-two sizes are COOLEY_TUKEY and every other size is
BLUESTEIN with padded_n = 2^bitlen(2n-2).

On B200 a plan also owns device state: the C-ABI plan for length n on each
device (Bluestein chirp and filter spectrum live there).  Those handles are
cached per (n, device) by ``trnfft_b200._lib.device_plan`` and released by
``clear_plan_cache``.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum, auto


class FFTAlgorithm(Enum):
    COOLEY_TUKEY = auto()
    BLUESTEIN = auto()


@dataclass(frozen=True)
class FFTPlan:
    n: int
    algorithm: FFTAlgorithm
    inverse: bool
    padded_n: int | None = None  # For Bluestein

    @property
    def is_power_of_2(self) -> bool:
        return self.algorithm == FFTAlgorithm.COOLEY_TUKEY


_plan_cache: dict[tuple, FFTPlan] = {}


def create_plan(n: int, inverse: bool = False) -> FFTPlan:
    key = (n, inverse)
    if key in _plan_cache:
        return _plan_cache[key]
    if n & (n - 1) == 0:
        plan = FFTPlan(n=n, algorithm=FFTAlgorithm.COOLEY_TUKEY, inverse=inverse)
    else:
        m = 1 << (2 * n - 2).bit_length()
        plan = FFTPlan(n=n, algorithm=FFTAlgorithm.BLUESTEIN, inverse=inverse, padded_n=m)
    _plan_cache[key] = plan
    return plan


def clear_plan_cache():
    _plan_cache.clear()
    from . import _lib

    _lib.clear_device_plans()


# Power-of-two transforms with n <= 256 can run either on the Stockham kernel
# (memory bound, one HBM pass) or as a DFT-as-GEMM on the tcgen05 tensor
# cores (X = x F with the n x n DFT matrix F, 3xTF32 for float32 accuracy),
# the B200 counterpart of the reference's NKI DFT-GEMM path for n <= 256
# (trnfft/fft_core.py:138, 221-251).  "stockham" is the default because it
# measured faster on B200 (the GEMM does O(n) more arithmetic per point).
_SMALL_N_MODES = ("stockham", "gemm")
_small_n_algorithm = "stockham"
DFT_GEMM_MAX_N = 256


def set_small_n_algorithm(mode: str) -> None:
    """Select the kernel for power-of-two n <= 256: "stockham" or "gemm"."""
    global _small_n_algorithm
    if mode not in _SMALL_N_MODES:
        raise ValueError(f"small-n algorithm must be one of {_SMALL_N_MODES}; got {mode!r}")
    _small_n_algorithm = mode


def get_small_n_algorithm() -> str:
    return _small_n_algorithm
